/*
 * fastmd_b200.h -- C ABI of libfastmd_b200.so, the B200 (sm_100a) kernels of
 * FastMD's per-step molecular-dynamics hot path.
 *
 * Conventions shared by every entry point:
 *   - all array arguments are DEVICE pointers (CUDA global memory of the
 *     current device) unless the name ends in `_host`;
 *   - sizes are int64_t element counts, strides are in elements;
 *   - `stream` is a cudaStream_t passed as void* (0 = legacy default stream);
 *     every kernel is launched on it and nothing synchronises, so every call
 *     is CUDA-graph capturable;
 *   - no entry point allocates device memory: outputs and workspaces are the
 *     caller's (workspace sizes are returned by the *_workspace_bytes calls);
 *   - the return value is an fmd_status; a launch error is reported as
 *     FMD_ERR_CUDA and the CUDA error string is kept for fmd_last_error();
 *   - data-dependent faults that a host check cannot see (an index out of
 *     range, a capacity overflow) never touch memory out of bounds: the kernel
 *     skips the access and raises a bit in the caller's int32 `flags` word
 *     (FMD_FLAG_*), read back by the caller after the step or window.
 *
 * The reference interface each entry point replaces is cited as
 * path:line inside the FastMD source tree (ICT-fushibo/fastMD).
 */
#ifndef FASTMD_B200_H
#define FASTMD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define FMD_API __attribute__((visibility("default")))
#else
#define FMD_API
#endif

typedef int32_t fmd_status;

#define FMD_OK 0
#define FMD_ERR_INVALID_ARGUMENT 1
#define FMD_ERR_CUDA 2
#define FMD_ERR_UNSUPPORTED 3
#define FMD_ERR_WORKSPACE 4

/* bits of the device-side `flags` word */
#define FMD_FLAG_INDEX_RANGE 1      /* an index argument was outside [0, n) */
#define FMD_FLAG_EDGE_OVERFLOW 2    /* more edges than the edge capacity */
#define FMD_FLAG_CANDIDATE_OVERFLOW 4 /* more candidates than the slot count */
#define FMD_FLAG_SKIN 8             /* an atom moved more than half the skin */
#define FMD_FLAG_NONFINITE 16       /* a non-finite position or momentum */
#define FMD_FLAG_CELL_RANGE 32      /* a fractional coordinate outside the cell grid */

/* ---------------------------------------------------------------- library */

/* ABI version of this header (major*10000 + minor*100 + patch). */
FMD_API int32_t fmd_version(void);
/* Static text of a status code. */
FMD_API const char* fmd_status_string(fmd_status status);
/* The CUDA error text of the last FMD_ERR_CUDA on this host thread. */
FMD_API const char* fmd_last_error(void);

/* ---------------------------------------------------- gather-cat (B1) */

/* One block of a gather-cat row: `width` columns taken from row
 * index[r] of `src` (or row r itself when `index` is NULL). `ld` is the
 * row stride of `src` in elements; `n_src` its row count (bounds check). */
typedef struct fmd_cat_part {
    const float* src;
    const int64_t* index;
    int64_t ld;
    int64_t n_src;
    int32_t width;
    int32_t _pad;
} fmd_cat_part;

/* out[r, :] = [part0(r) | part1(r) | ...] for r < rows; up to 4 parts of any
 * widths (mixed widths allowed, e.g. sender 128 | receiver 128 | basis 8).
 * Replaces the per-row Triton gather-cat of
 * fastmd/models/matris/op/triton_gather_cat.py:30 (cat3) and :203 (cat4),
 * and its mixed-width torch.cat fallback (triton_gather_cat.py:192). */
FMD_API fmd_status fmd_gather_cat(const fmd_cat_part* parts, int32_t n_parts, int64_t rows,
                          float* out, int64_t ldo, int32_t* flags, void* stream);

/* cat3 with the reference's argument list: out[r] = [A[r] | X[ia[r]] | X[ib[r]]],
 * out is [rows, 3D] contiguous (triton_gather_cat.py:181 aligned_gather_cat3). */
FMD_API fmd_status fmd_aligned_gather_cat3(const float* aligned, int64_t lda, const float* gathered,
                                   int64_t ldg, int64_t n_gathered, const int64_t* index_a,
                                   const int64_t* index_b, int64_t rows, int32_t dim,
                                   float* out, int32_t* flags, void* stream);

/* Backward of a gather block without atomics: for every source row n,
 *   grad[n, :] (=|+=) sum over the CSR run of n of gout[perm[j], col0 : col0+width]
 * in run order (deterministic). `off` is int64 [n_src + 1], `perm` int64 [rows]
 * (NULL: identity, i.e. the rows are sorted by this index). `accumulate` = 0
 * overwrites grad, 1 adds to it. Replaces the atomic scatter of
 * triton_gather_cat.py:59 (_aligned_gather_cat3_bwd) and :236 (cat4). */
FMD_API fmd_status fmd_gather_rows_bwd(const float* gout, int64_t ldgo, int32_t col0, int32_t width,
                               const int64_t* perm, const int64_t* off, int64_t n_src,
                               float* grad, int64_t ldg, int32_t accumulate, void* stream);

/* Strided row copy dst[r, :w] = src[r, :w] (the aligned block's gradient). */
FMD_API fmd_status fmd_copy_rows(const float* src, int64_t lds, float* dst, int64_t ldd, int64_t rows,
                         int32_t width, void* stream);

/* ------------------------------------------- CSR segment metadata (C1) */

/* off[s] = first row with segment[row] >= s, for s in [0, num_segment]
 * (segment sorted ascending, int64). The identity CSR of
 * fastmd/engine/dispatch.py:325-331 (sorted receivers). */
FMD_API fmd_status fmd_csr_offsets_sorted(const int64_t* segment, int64_t rows, int64_t num_segment,
                                  int64_t* off, void* stream);

/* Workspace for fmd_csr_build. */
FMD_API fmd_status fmd_csr_build_workspace_bytes(int64_t rows, int64_t num_segment, size_t* bytes);
/* Stable CSR of an unsorted segment array: perm lists the rows grouped by
 * segment, ascending row order inside a segment; off [num_segment + 1].
 * Segments outside [0, num_segment) raise FMD_FLAG_INDEX_RANGE and are
 * placed in no run. Replaces segment_attention_csr_metadata
 * (fastmd/models/matris/op/triton_segment_attention.py:824, argsort + searchsorted). */
FMD_API fmd_status fmd_csr_build(const int64_t* segment, int64_t rows, int64_t num_segment,
                         int64_t* perm, int64_t* off, void* workspace, size_t workspace_bytes,
                         int32_t* flags, void* stream);

/* ------------------------------------------------ segment sum (C1) */

/* out[s, :] = sum over j in [off[s], off[s+1]) of w[r_j, :] * v[r_j, :]
 * (v alone when w is NULL), r_j = perm[j] or j when perm is NULL; the sum
 * runs in run order with one FP32 accumulator per column (deterministic).
 * skip_segment >= 0: that segment's output row is 0.
 * Replaces fastmd/models/matris/op/triton_csr_segment_sum.py:71
 * (_csr_segsum_fwd) and csr_segment_sum :433. */
FMD_API fmd_status fmd_csr_segment_sum(const float* value, int64_t ldv, const float* weight, int64_t ldw,
                               const int64_t* perm, const int64_t* off, int64_t num_segment,
                               int32_t dim, int64_t skip_segment, float* out, int64_t ldo,
                               void* stream);

/* VJP: gvalue[r] = gout[seg[r]] * w[r] (gout[seg[r]] when w is NULL),
 * gweight[r] = gout[seg[r]] * v[r]; either output may be NULL. Rows whose
 * segment is skip_segment get exact zeros. Replaces
 * triton_csr_segment_sum.py:184 (_csr_segsum_bwd_rows). */
FMD_API fmd_status fmd_csr_segment_sum_bwd(const float* gout, const float* value, int64_t ldv,
                                   const float* weight, int64_t ldw, const int64_t* segment,
                                   int64_t rows, int64_t num_segment, int32_t dim,
                                   int64_t skip_segment, float* gvalue, float* gweight,
                                   int32_t* flags, void* stream);

/* -------------------------------------- Nose-Hoover chain integrator (F1/F3) */

/* Flat fp64 state of R replicas of n atoms each and chain length M:
 *   q [R*n*3] | p [R*n*3] | F [R*n*3] | eta [R*M] | p_eta [R*M] | E [R]
 * (the single-system layout of fastmd/execution/gpu_nhc.py:217 NHCState for R = 1).
 * `consts` is the fp64 table of gpu_nhc.py:113 nhc_constants:
 *   dt, dt/2, kT, 3N kT, 3 x (delta, delta/2, -delta/4, -delta), pad to 16, Q[M].
 * `masses` fp64 [n*R] (amu). One CTA integrates one replica. */

/* ASE step() first half: NHC(dt/2); p += dt/2 F(q_n); q += dt p / m.
 * f32_kick = 1 forms dt/2*F in float32 (NumPy NEP-50 for float32 forces).
 * Replaces gpu_nhc.py:360 _nhc_pre_force_kernel and replica_batch.py:75. */
FMD_API fmd_status fmd_nhc_pre_force(double* state, const double* masses, const double* consts,
                             int64_t n_atoms, int32_t n_replicas, int32_t tchain, int32_t tloop,
                             int32_t f32_kick, float* positions32, void* stream);

/* ASE step() second half: p += dt/2 F(q_{n+1}); NHC(dt/2); cache F (and E).
 * forces are float32 (forces_f64 NULL) or float64 (forces_f32 NULL),
 * [R*n*3]; energy (fp64 [R]) may be NULL. Replaces gpu_nhc.py:394
 * _nhc_post_force_kernel and replica_batch.py:89. */
FMD_API fmd_status fmd_nhc_post_force(double* state, const double* masses, const double* consts,
                              int64_t n_atoms, int32_t n_replicas, int32_t tchain, int32_t tloop,
                              int32_t f32_kick, const float* forces_f32, const double* forces_f64,
                              const double* energy, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FASTMD_B200_H */
