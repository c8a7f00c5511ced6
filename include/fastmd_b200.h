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
#define FMD_FLAG_WAIT_TIMEOUT 64    /* a bounded in-kernel wait gave up (about 1 s); outputs invalid */
#define FMD_FLAG_TRIPLET_OVERFLOW 128 /* more line-graph triplets than the triplet capacity */
#define FMD_FLAG_INVALID_PAIRS 256  /* a real edge without its reverse, or an odd edge count */

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

/* fmd_gather_rows_bwd for long runs (tens to hundreds of rows gathered by
 * each source row, e.g. the triplets of an atom): a CTA of 8 warps per
 * source row and 128 columns, warp w summing rows w, w + 8, ... of the run,
 * the partials added in warp order (deterministic; a different but fixed
 * summation order from fmd_gather_rows_bwd). 16-byte aligned rows and
 * widths, col0 and strides multiples of 4, else FMD_ERR_UNSUPPORTED. */
FMD_API fmd_status fmd_gather_rows_bwd_long(const float* gout, int64_t ldgo, int32_t col0, int32_t width,
                                            const int64_t* perm, const int64_t* off, int64_t n_src, float* grad,
                                            int64_t ldg, int32_t accumulate, void* stream);

/* Strided row copy dst[r, :w] = src[r, :w] (the aligned block's gradient). */
FMD_API fmd_status fmd_copy_rows(const float* src, int64_t lds, float* dst, int64_t ldd, int64_t rows,
                         int32_t width, void* stream);
/* bytes zero bytes at dst, stream-ordered (a memset, no kernel): the zero
 * planes and gradient buffers a model evaluation starts from (the torch
 * zeros / zero_ calls around the reference's model code). */
FMD_API fmd_status fmd_zero(void* dst, int64_t bytes, void* stream);

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

/* ------------------------------------------------- neighbour lists (A1-A3) */

/* R systems of n atoms share one cell (`cell_host`: 9 floats, row-major
 * lattice vectors, HOST memory); row r*n + a is atom a of system r and no
 * pair crosses systems (the disjoint-union graph of
 * fastmd/execution/replica_batch.py:126). Positions are float32 [R*n, 3]. */

/* Workspace of fmd_candidates_build for this cell, cutoff and size. */
FMD_API fmd_status fmd_cell_list_workspace_bytes(const float* cell_host, float cutoff, int64_t n_atoms,
                                                 int32_t n_systems, size_t* bytes);

/* Skin candidate list (full, both directions) within `candidate_cutoff` of
 * the wrapped positions, by a cell list: cand_nbr [R*n, bmax] (global rows,
 * unused slots = R*n), cand_shift [R*n, bmax, 3] integer images,
 * cand_count [R*n] (the true count; > bmax raises
 * FMD_FLAG_CANDIDATE_OVERFLOW). Each row is in canonical (neighbour, image)
 * order. When ref_positions/ref_wraps/wrap_delta are given, the refresh
 * snapshot is taken too (positions, their wraps; wrap delta zeroed).
 * Replaces FixedCapacityGraphBuilder.refresh_candidates
 * (fastmd/graph/fixed_capacity_builder.py:1675, :1519) over nvalchemiops'
 * batch_build_cell_list / batch_query_cell_list (neighbor_list_backend.py:134-154). */
FMD_API fmd_status fmd_candidates_build(const float* positions, const float* cell_host, int64_t n_atoms,
                                        int32_t n_systems, float candidate_cutoff, int32_t bmax,
                                        int32_t* cand_nbr, int32_t* cand_shift, int32_t* cand_count,
                                        float* ref_positions, int32_t* ref_wraps, int32_t* wrap_delta,
                                        void* workspace, size_t workspace_bytes, int32_t* flags, void* stream);

/* Workspace of fmd_refilter_edges. */
FMD_API fmd_status fmd_refilter_workspace_bytes(int64_t n_atoms, int32_t n_systems, size_t* bytes);

/* Per-step exact edges from the candidates (capture-safe, 2 kernels, one CTA
 * per system): wraps the positions (wrapped [R*n,3], wrap_delta since the
 * refresh), tests the skin (max_displacement [R]; 2*max > skin + 1e-6 raises
 * FMD_FLAG_SKIN), keeps the candidates with float32
 * dist2 = dx*dx+dy*dy+dz*dz < cutoff^2 in the reference's operation order,
 * and writes edge_index [e_capacity, 2] int32 (centre, neighbour),
 * edge_image [e_capacity, 3] float32 in canonical order (no sort), rows past
 * the real edges padded with far self-loops (pad_image_host, 3 ints, HOST),
 * minimum_image = 1: a lattice jump of the caller's coordinates since the
 * refresh is no motion (the skin test takes the minimum-image displacement),
 * n_edges [1] int64 (> e_capacity raises FMD_FLAG_EDGE_OVERFLOW), the
 * receiver CSR recv_off [R*n + 1] and the sender CSR send_off [R*n + 1] /
 * send_perm [e_capacity] (edge ids, each run ascending). Replaces
 * FixedCapacityGraphBuilder.build(rebuild_candidates=False)
 * (fixed_capacity_builder.py:2181: _count_neighbors_kernel :98,
 * _materialize_neighbors_kernel :189, _pad_self_loops_kernel :324,
 * _sort_edges :1968). A system's atoms are staged in shared memory (32 bytes
 * per atom + 4, at most 200 KB): at most 6,399 atoms per system; larger
 * systems return FMD_ERR_UNSUPPORTED and launch nothing. */
FMD_API fmd_status fmd_refilter_edges(const float* positions, const float* cell_host, int64_t n_atoms,
                                      int32_t n_systems, const float* ref_positions, const int32_t* ref_wraps,
                                      const int32_t* cand_nbr, const int32_t* cand_shift,
                                      const int32_t* cand_count, int32_t bmax, float cutoff, float skin,
                                      int64_t e_capacity, const int32_t* pad_image_host,
                                      int32_t minimum_image, float* wrapped,
                                      int32_t* wrap_delta, int32_t* edge_index, float* edge_image,
                                      int64_t* recv_off, int64_t* send_off, int32_t* send_perm, int64_t* n_edges,
                                      float* max_displacement, void* workspace, size_t workspace_bytes,
                                      int32_t* flags, void* stream);

/* fmd_refilter_edges for callers that cannot allocate device memory (no
 * counterpart in the reference): a C or Fortran MD host that links this
 * library without a CUDA allocator or memory pool of its own, or a caller
 * inside another framework whose memory manager owns the device. The same
 * arguments and results as fmd_refilter_edges, without the workspace: the
 * scratch is a static 1 MiB device array held by every GPU that loads the
 * library until exit, enough for n_atoms * n_systems <= 126,976 atoms (up to
 * 4,096 systems); larger calls return FMD_ERR_WORKSPACE and launch nothing.
 * The per-system limit of fmd_refilter_edges holds too (at most 6,399 atoms
 * per system, else FMD_ERR_UNSUPPORTED).
 * The first call on a device looks the array's device address up (once per
 * device, with that device current): make that first call before any stream
 * capture. All calls share the array, so calls that overlap on the GPU (two
 * streams, two host threads) race; serialise them. Nothing in it needs to
 * start at zero (every field is written before it is read). Allocates nothing. */
FMD_API fmd_status fmd_refilter_edges_noalloc(const float* positions, const float* cell_host, int64_t n_atoms,
                                              int32_t n_systems, const float* ref_positions,
                                              const int32_t* ref_wraps, const int32_t* cand_nbr,
                                              const int32_t* cand_shift, const int32_t* cand_count, int32_t bmax,
                                              float cutoff, float skin, int64_t e_capacity,
                                              const int32_t* pad_image_host, int32_t minimum_image, float* wrapped,
                                              int32_t* wrap_delta, int32_t* edge_index, float* edge_image,
                                              int64_t* recv_off, int64_t* send_off, int32_t* send_perm,
                                              int64_t* n_edges, float* max_displacement, int32_t* flags,
                                              void* stream);

/* Workspace of fmd_neighbor_list. */
FMD_API fmd_status fmd_neighbor_list_workspace_bytes(const float* cell_host, float cutoff, int64_t n_atoms,
                                                     int32_t bmax, size_t* bytes);

/* Ragged full neighbour list of one system (eager path): candidates at
 * cutoff + 1e-6 by the cell list, kept when |(q - p) + image @ cell| < cutoff
 * (float32), rows in canonical (centre, neighbour, image) order: center,
 * neighbor int64 [e_capacity], images int32 [e_capacity, 3], dist float32,
 * offsets int64 [n + 1] (edges per centre; offsets[n] = edge count, rows past
 * e_capacity are not written). wrapped (optional) receives the wrapped
 * positions. More than bmax candidates of an atom raises
 * FMD_FLAG_CANDIDATE_OVERFLOW (grow bmax and rerun); bmax of 2048 or more
 * returns FMD_ERR_UNSUPPORTED. One sweep of the cell list counts the kept
 * pairs and stores each centre's candidate keys (4 bytes each below 2^20
 * atoms, else 8; bmax + 1 per centre in the workspace); a second pass sorts
 * each centre's keys and writes its row. Replaces neighbor_list_nvidia
 * (fastmd/graph/gpu_graph_builder.py:108). */
FMD_API fmd_status fmd_neighbor_list(const float* positions, const float* cell_host, int64_t n_atoms,
                                     float cutoff, int32_t bmax, int64_t e_capacity, float* wrapped,
                                     int64_t* center, int64_t* neighbor, int32_t* images, float* dist,
                                     int64_t* offsets, void* workspace, size_t workspace_bytes,
                                     int32_t* flags, void* stream);

/* The edge-vector override of exact-rc self-loop padding: for every row r <
 * e_capacity, edge_vec_override[r] = pad_vector_host (3 floats) on the padded
 * rows (r >= min(*n_edges, e_capacity)), 0 on the real rows. The padded rows
 * themselves are fmd_refilter_edges' loops with pad_image (0, 0, 0).
 * Replaces the HAS_OVERRIDE part of _pad_self_loops_kernel
 * (fastmd/graph/fixed_capacity_builder.py:324). */
FMD_API fmd_status fmd_pad_vector_override(const int64_t* n_edges, int64_t e_capacity, const float* pad_vector_host,
                                           float* edge_vec_override, void* stream);

/* Float64 model positions of a float64 build: out[i] = p[i] - ((w0 c64[0] +
 * w1 c64[1]) + w2 c64[2]) (rows of the float64 cell, each operation rounded),
 * w = floor(float32(p[i]) @ inv(cell)) the whole lattice vectors of the
 * re-filter's float32 wrap (cell_host float32 row-major, its inverse the
 * float64 inverse rounded once), so the float64 positions and the float32
 * edges describe the same images. positions, out [n_atoms, 3] float64.
 * Replaces the float64 part of _float64_prologue_kernel
 * (fastmd/graph/fixed_capacity_builder.py:464) and the float64 addmm of the
 * build (:2266). */
FMD_API fmd_status fmd_model_positions_f64(const double* positions, int64_t n_atoms, const float* cell_host,
                                           const double* cell64_host, double* out, void* stream);

/* ------------------------------------------- dense layers (D2), IEEE FP32 */

/* y[m, n] (=|+=) act(a'[m, :] . op(w) + bias) on the CUDA cores, IEEE FP32,
 * one sequential FMA chain over k per output (deterministic).
 * op(w) = w^T for w [n, k] (trans_w = 1, the nn.Linear layout), w for w [k, n];
 * a' = a, or a * silu'(a_pre) when a_pre is given (the SiLU backward of the
 * previous layer fused into the operand load); act 0 = identity, 1 = SiLU
 * (y_pre, when given, receives the pre-activation). The TF32-off parity
 * path of the wide projections of fastmd/engine/kernels/triton_wide_gemm.py:482
 * (linear) and :534 (matmul), where the reference runs cuBLAS FP32. */
FMD_API fmd_status fmd_gemm_f32(const float* a, int64_t lda, const float* a_pre, int64_t lda_pre,
                                const float* w, int64_t ldw, int32_t trans_w, const float* bias, float* y,
                                int64_t ldy, float* y_pre, int64_t ldy_pre, int64_t m, int32_t n, int32_t k,
                                int32_t act, int32_t accumulate, void* stream);

/* ------------------------------- MatRIS bond pairs and line graph (A5) */

/* Reverse-edge pairing of directed edges (center, neighbor [E] int64, images
 * [E, 3] int32 within +-10): pair(e) = the edge whose forward key
 * (c N + n) 21^3 + code(image) equals e's reverse key (n N + c) 21^3 +
 * code(-image), located by lower bound among the sorted forward keys
 * (clamped to the last edge; presorted = 1 when the edges are in key order);
 * directed2undirected[e] = rank of min(e, pair(e)) among the distinct minima,
 * undirected2directed[u] = smallest edge of u (entries past *n_undirected set
 * to E), *n_undirected (device int64). Replaces _build_d2u
 * (fastmd/graph/gpu_graph_builder.py:217). */
FMD_API fmd_status fmd_reverse_pairs_workspace_bytes(int64_t n_edges, size_t* bytes);
FMD_API fmd_status fmd_reverse_pairs(const int64_t* center, const int64_t* neighbor, const int32_t* images,
                                     int64_t n_edges, int64_t n_atoms, int32_t presorted, void* workspace,
                                     size_t workspace_bytes, int32_t* directed2undirected,
                                     int32_t* undirected2directed, int64_t* n_undirected, int32_t* flags,
                                     void* stream);

/* Ordered bond pairs around each atom: the short edges (dist < cutoff),
 * stably grouped by centre (already grouped when presorted = 1), give an atom
 * with k of them the k (k - 1) rows [atom, u(first), first, u(second), second]
 * (int32 [t_capacity, 5]) in the order first = l / (k - 1), second =
 * l % (k - 1) skipping first. *n_triplets (device int64) receives the count;
 * rows past t_capacity are not written and raise FMD_FLAG_TRIPLET_OVERFLOW.
 * Replaces _build_line_graph (fastmd/graph/gpu_graph_builder.py:511). */
FMD_API fmd_status fmd_line_graph_workspace_bytes(int64_t n_edges, int64_t n_atoms, size_t* bytes);
FMD_API fmd_status fmd_line_graph(const int64_t* center, const float* dist, const int32_t* directed2undirected,
                                  int64_t n_edges, int64_t n_atoms, float cutoff, int32_t presorted,
                                  int64_t t_capacity, void* workspace, size_t workspace_bytes, int32_t* triplets,
                                  int64_t* n_triplets, int32_t* flags, void* stream);

/* The fixed-capacity MatRIS bond graph of a fixed-capacity build, capture-safe
 * (no count leaves the device). Input: edge_index [2 u_capacity, 2] int32 and
 * edge_image [2 u_capacity, 3] (integer images as float) whose first
 * min(*n_edges, 2 u_capacity) rows are the real edges in canonical (centre,
 * neighbour, image) order (what fmd_refilter_edges writes), the wrapped
 * positions [n_atoms, 3] they were computed from and the row-major host cell.
 * Output, bit-identical to the reference builder:
 *   the padded rows rewritten by the padding rule (FMD_PAD_SINK_ATOMS: both
 *   rows of padded pair p on sink n_atoms + p n_dummy / n_pad_u, image
 *   (3, 3, 3); FMD_PAD_FAR_SELF_LOOPS: the loops +pad_image / -pad_image of
 *   atom p mod n_atoms);
 *   directed2undirected [2 u_capacity], undirected2directed [u_capacity];
 *   line_graph [t_capacity, 5] int32 rows [atom, u1, e1, u2, e2] over the
 *   short edges (dist2 < line_cutoff^2 in the re-filter's FP32 order), then
 *   padded triplets on padded pairs;
 *   *n_triplets the triplet count (of the stored rows);
 *   flags: FMD_FLAG_INVALID_PAIRS, FMD_FLAG_EDGE_OVERFLOW when the edges leave
 *   no padded pair (>= 2 u_capacity), FMD_FLAG_TRIPLET_OVERFLOW.
 * On an overflow (those, or a flags word already holding FMD_FLAG_SKIN,
 * _CANDIDATE_OVERFLOW or _NONFINITE) every row, pair and triplet is the
 * all-padding topology instead. Replaces _materialize_pairs,
 * _materialize_line_graph / _line_graph_kernel, _pad_edges_kernel,
 * _pad_loop_pairs_kernel and the overflow topology
 * (fastmd/graph/fixed_capacity_builder.py:2001, :2101, :681, :292, :397,
 * :1474, :2163). */
#define FMD_PAD_SINK_ATOMS 0
#define FMD_PAD_FAR_SELF_LOOPS 1
FMD_API fmd_status fmd_bond_graph_workspace_bytes(int64_t n_atoms, int64_t e_capacity, size_t* bytes);
FMD_API fmd_status fmd_bond_graph(const float* positions, const float* cell, int64_t n_atoms, int32_t* edge_index,
                                  float* edge_image, const int64_t* n_edges, int64_t u_capacity, int64_t t_capacity,
                                  float line_cutoff, int32_t padding, int64_t n_dummy, const int32_t* pad_image,
                                  void* workspace, size_t workspace_bytes, int32_t* directed2undirected,
                                  int32_t* undirected2directed, int32_t* line_graph, int64_t* n_triplets,
                                  int32_t* flags, void* stream);

/* -------------------------- decomposed indexed-concat SiLU epilogue (B2) */

/* preact[r] = p0[r] + gathered[0].src[index_0[r]] + ... + bias (the FP32
 * additions in that order), core_act = silu(preact[:, :h]), gate_act =
 * silu(preact[:, h:]) with silu(x) = x / (1 + e^-x) evaluated as
 * x * (1 / (1 + e^-x)). p0 [rows, 2h] (row stride ldp0); up to 3 gathered
 * projections [n_src, 2h] (fmd_cat_part: src, index [rows] int64, ld, n_src;
 * width unused); bias [2h] or null; preact [rows, 2h], core_act and
 * gate_act [rows, h] contiguous. Index values outside [0, n_src) add
 * nothing and raise FMD_FLAG_INDEX_RANGE. Replaces
 * _cat3_gather_add_silu_fwd / _cat4_gather_add_silu_fwd
 * (fastmd/engine/kernels/decomposed_indexed_cat_silu_linear.py:97, :156). */
FMD_API fmd_status fmd_gather_add_silu(const float* p0, int64_t ldp0, const fmd_cat_part* gathered,
                                       int32_t n_gathered, const float* bias, int64_t rows, int32_t h,
                                       float* preact, float* core_act, float* gate_act, int32_t* flags,
                                       void* stream);

/* grad_pre[r] = [g_core s (1 + x (1 - s)) | g_gate s (1 + x (1 - s))] with x
 * the halves of preact and s = sigmoid(x): the per-row part of
 * _cat3_gather_add_silu_bwd / _cat4_gather_add_silu_bwd (:234, :383); the
 * gathered parts' gradients are its CSR row sums (fmd_gather_rows_bwd). */
FMD_API fmd_status fmd_silu_pair_bwd(const float* grad_core, const float* grad_gate, const float* preact,
                                     int64_t rows, int32_t h, float* grad_pre, int64_t ldgp, void* stream);

/* Self-test of the bounded mbarrier wait that every pipeline wait of the
 * tensor-core kernels uses (no counterpart in the reference, whose Triton
 * kernels have no bounded waits): one thread waits on a fresh barrier;
 * arrive = 1 arrives first (no flag), arrive = 0 lets nothing arrive, the
 * wait gives up after about a second and raises FMD_FLAG_WAIT_TIMEOUT in
 * `flags` (device int32). Nothing is in flight when it gives up, so the
 * context stays usable. */
FMD_API fmd_status fmd_wait_probe(int32_t arrive, int32_t* flags, void* stream);

/* The roofline denominator of fmd_gemm_tf32x3: one CTA per SM issuing `iters`
 * back-to-back tcgen05 kind::tf32 MMAs (M = 128, N = 128, K = 8, 262,144
 * flops each) with no data movement; time the launch with events on `stream`.
 * No counterpart in the reference (a measurement entry). */
FMD_API fmd_status fmd_tf32_mma_rate(int32_t iters, int32_t* flags, void* stream);

/* ------------------------------------------ MatRIS gated-LN epilogue */

/* out = silu(LN(core_x + core_lb)) * sigmoid(LN(gate_x + gate_lb))
 * (+ residual * res_weight) per row of width dim (<= 256), LN(x) =
 * (x - mean) rstd w + b with rstd = 1 / sqrt(var + eps); the per-row mean /
 * rstd of both halves are written for the backward. core_lb / gate_lb (both
 * or neither) are the preceding linears' biases; residual / res_weight (both
 * or neither). All [rows, dim] arrays contiguous. Replaces _gated_ln_fwd /
 * _gated_ln_fwd_2d (fastmd/models/matris/op/triton_gated_ln.py:57, :205). */
FMD_API fmd_status fmd_gated_ln(const float* core_x, const float* gate_x, const float* core_lb, const float* gate_lb,
                                const float* core_w, const float* core_b, const float* gate_w, const float* gate_b,
                                const float* residual, const float* res_weight, int64_t rows, int32_t dim,
                                float eps_core, float eps_gate, float* out, float* core_mean, float* core_rstd,
                                float* gate_mean, float* gate_rstd, void* stream);

/* Backward of fmd_gated_ln from its saved mean / rstd: grad_core_x,
 * grad_gate_x [rows, dim] and, when grad_residual is given,
 * grad_residual = grad_out * res_weight. Replaces _gated_ln_bwd /
 * _gated_ln_bwd_2d (triton_gated_ln.py:127, :280). */
FMD_API fmd_status fmd_gated_ln_bwd(const float* core_x, const float* gate_x, const float* core_lb,
                                    const float* gate_lb, const float* core_w, const float* core_b,
                                    const float* gate_w, const float* gate_b, const float* res_weight,
                                    const float* grad_out, const float* core_mean, const float* core_rstd,
                                    const float* gate_mean, const float* gate_rstd, int64_t rows, int32_t dim,
                                    float* grad_core_x, float* grad_gate_x, float* grad_residual, void* stream);

/* out[c] = sum over rows of x[r, c] (row stride ld), in a fixed order (128-row
 * partials, then their sum): the gradients of the folded linear biases
 * (triton_gated_ln.py:369 _linear_bias_grads). */
FMD_API fmd_status fmd_column_sum_workspace_bytes(int64_t rows, int32_t cols, size_t* bytes);
FMD_API fmd_status fmd_column_sum(const float* x, int64_t rows, int32_t cols, int64_t ld, void* workspace,
                                  size_t workspace_bytes, float* out, void* stream);

/* ------------------------------- MatRIS directed-pair aggregation */

#define FMD_PAIR_AVERAGE 0
#define FMD_PAIR_AVERAGE_BWD 1
#define FMD_PAIR_EXPAND 2
#define FMD_PAIR_EXPAND_BWD 3

/* The directed-edge <-> undirected-pair maps of the MatRIS atom graph over
 * pair_index [n_pairs, 2] int64 (a bijection onto the 2U directed rows):
 *   FMD_PAIR_AVERAGE      out[u] = (in[p0] + in[p1]) * 0.5   in [2U, dim], out [U, dim]
 *   FMD_PAIR_AVERAGE_BWD  out[p0] = out[p1] = in[u] * 0.5    in [U, dim],  out [2U, dim]
 *   FMD_PAIR_EXPAND       out[p0] = out[p1] = in[u]          in [U, dim],  out [2U, dim]
 *   FMD_PAIR_EXPAND_BWD   out[u] = in[p0] + in[p1]           in [2U, dim], out [U, dim]
 * `in` has row stride ldi (>= dim), `out` is contiguous. Index values outside
 * [0, 2U) raise FMD_FLAG_INDEX_RANGE (a gathered row reads as zero, a
 * scattered row is skipped). Replaces _directed_pair_average_fwd / _bwd and
 * _undirected_pair_expand_fwd / _bwd
 * (fastmd/models/matris/op/triton_directed_pair_aggregate.py:61, :83, :105, :127). */
FMD_API fmd_status fmd_pair_aggregate(int32_t op, const float* in, int64_t ldi, const int64_t* pair_index,
                                      int64_t n_pairs, int32_t dim, float* out, int32_t* flags, void* stream);

/* ----------------------------------- MatRIS residual add (frozen weight) */

#define FMD_RESIDUAL_ADD 0
#define FMD_RESIDUAL_ADD_BWD 1

/* FMD_RESIDUAL_ADD      out[r, c] = delta[r, c] + residual[r, c] * weight[c]
 * FMD_RESIDUAL_ADD_BWD  out[r, c] = residual[r, c] * weight[c]   (residual = the
 *                       output gradient; delta unused and may be NULL)
 * over rows x dim, each matrix with its own row stride (>= dim); the product is
 * rounded before the addition. Replaces _residual_add_fwd / _residual_add_bwd
 * (fastmd/models/matris/op/triton_residual_add.py:40, :64). */
FMD_API fmd_status fmd_residual_add(int32_t op, const float* delta, int64_t ldd, const float* residual, int64_t ldr,
                                    const float* weight, int64_t rows, int32_t dim, float* out, int64_t ldo,
                                    void* stream);

/* ------------------------------------------- segment attention (C2) */

/* out[s, :] = sum over the rows i of segment s of softmax(logits[i, :] over
 * the segment, per column) * value[i, :], over a CSR (off [S+1] int64; perm
 * [off[S]] int64 row ids, or null for the identity CSR row = j). The online
 * recurrence of the reference in FP32, per segment in CSR order. out, lse,
 * seg_max, seg_denom are [S, dim] contiguous; lse (m + log denom, -inf for an
 * empty or skipped segment), seg_max and seg_denom (the paired backward's
 * statistics) are optional. skip_segment (or -1) runs no rows: out 0.
 * Row ids outside [0, rows) raise FMD_FLAG_INDEX_RANGE and are skipped.
 * Replaces _csr_segment_attention_fwd and, called once per side,
 * _paired_csr_segment_attention_fwd
 * (fastmd/models/matris/op/triton_segment_attention.py:62, :210). */
FMD_API fmd_status fmd_segment_attention(const float* logits, int64_t ldl, const float* value, int64_t ldv,
                                         const int64_t* perm, const int64_t* off, int64_t rows, int64_t num_segment,
                                         int32_t dim, int64_t skip_segment, float* out, float* lse, float* seg_max,
                                         float* seg_denom, int32_t* flags, void* stream);

/* Backward of fmd_segment_attention: per segment the statistics again, then
 * per row alpha = e^(l - m) / denom, grad_value = alpha g, grad_logits =
 * alpha g (v - out) (+ alpha glse when glse is given). Rows of no visited
 * segment (the skipped one, rows outside a partial CSR) are not written.
 * Replaces _csr_segment_attention_bwd (triton_segment_attention.py:128). */
FMD_API fmd_status fmd_segment_attention_bwd(const float* logits, int64_t ldl, const float* value, int64_t ldv,
                                             const float* out, const float* gout, const float* glse,
                                             const int64_t* perm, const int64_t* off, int64_t rows,
                                             int64_t num_segment, int32_t dim, int64_t skip_segment,
                                             float* grad_logits, int64_t ldgl, float* grad_value, int64_t ldgv,
                                             int32_t* flags, void* stream);

/* Row backward of the paired attention (two segmentations of the same rows
 * sharing value): statistics [S, dim] of both sides from
 * fmd_segment_attention, per-row segment ids segment_a / segment_b. A row's
 * side in skip_segment contributes exactly 0. grad_value [rows, dim]
 * contiguous. Replaces _paired_segment_attention_bwd_rows
 * (triton_segment_attention.py:319). */
FMD_API fmd_status fmd_paired_segment_attention_bwd_rows(
    const float* logits_a, int64_t ldla, const float* logits_b, int64_t ldlb, const float* value, int64_t ldv,
    const float* gout_a, const float* gout_b, const float* out_a, const float* out_b, const float* max_a,
    const float* denom_a, const float* max_b, const float* denom_b, const int64_t* segment_a,
    const int64_t* segment_b, const float* glse_a, const float* glse_b, int64_t rows, int64_t num_segment,
    int32_t dim, int64_t skip_segment, float* grad_logits_a, int64_t ldga, float* grad_logits_b, int64_t ldgb,
    float* grad_value, int32_t* flags, void* stream);

/* ------------------------------------ dense layers (D2), tcgen05 3xTF32 */

/* hi = rna_tf32(w), lo = w - hi for w [rows, cols] (row stride ldw), written
 * [rows, cols], or [cols, rows] with transpose = 1 (the K-major operand of
 * dX = dY . w), with row stride ldo (a multiple of 4 for fmd_gemm_tf32x3).
 * Once per weight version: the weight split of
 * fastmd/engine/kernels/triton_wide_gemm.py:132 (_split_kernel). */
FMD_API fmd_status fmd_tf32_split(const float* w, int64_t rows, int64_t cols, int64_t ldw, int32_t transpose,
                                  float* hi, float* lo, int64_t ldo, void* stream);

#define FMD_ACT_NONE 0
#define FMD_ACT_SILU 1        /* y = silu(sum + bias + c) */
#define FMD_ACT_SILU_GRAD 2   /* y = (sum + bias) * silu'(c): c is a pre-activation, not added */
#define FMD_ACT_MASK 15
#define FMD_ACT_INPUT_SILU 16 /* or-ed in: the x operand enters as silu(x) */

/* y[m, n] (=|+=) act(x[m, :k] . w^T + bias + c) on the tcgen05 tensor cores
 * at FP32 accuracy (3xTF32: x_lo w_hi + x_hi w_lo + x_hi w_hi, a fresh TMEM
 * accumulator per 64-wide K chunk, the chunks summed in FP32), for w [n, k]
 * given as its fmd_tf32_split pair (w_hi, w_lo, row stride ldw). bias [n]
 * and the residual c [m, ldc] are optional; act is one of FMD_ACT_NONE,
 * FMD_ACT_SILU, FMD_ACT_SILU_GRAD (c required), optionally or-ed with
 * FMD_ACT_INPUT_SILU (the layers of an MLP chained on pre-activations, and
 * their backward). y may alias c (each element is read before it is written).
 * x, w_hi, w_lo 16-byte aligned with ldx, ldw multiples of 4 (TMA), else
 * FMD_ERR_UNSUPPORTED (as on a non-sm_100 device). A bounded in-kernel wait
 * that expires raises FMD_FLAG_WAIT_TIMEOUT in flags (may be null).
 * Replaces _wide_gemm_persistent / _wide_gemm_tiles behind linear and matmul
 * (fastmd/engine/kernels/triton_wide_gemm.py:105, :120, :482, :534). */
FMD_API fmd_status fmd_gemm_tf32x3(const float* x, int64_t ldx, const float* w_hi, const float* w_lo, int64_t ldw,
                                   const float* bias, const float* c, int64_t ldc, float* y, int64_t ldy, int64_t m,
                                   int32_t n, int32_t k, int32_t act, int32_t accumulate, int32_t* flags,
                                   void* stream);

/* One problem of fmd_gemm_tf32x3_grouped: the arguments of fmd_gemm_tf32x3. */
typedef struct fmd_gemm_problem {
    const float* x;
    int64_t ldx;
    const float* w_hi;
    const float* w_lo;
    int64_t ldw;
    const float* bias;
    const float* c;
    int64_t ldc;
    float* y;
    int64_t ldy;
    int64_t m;
    int32_t n, k, act, accumulate;
} fmd_gemm_problem;

/* Up to 4 independent fmd_gemm_tf32x3 problems in one launch (their tiles
 * concatenated over one persistent grid; each problem's results are those of
 * its own fmd_gemm_tf32x3 call, bit for bit). For a layer's per-l linears of
 * the NequIP/SevenNet planes (three small GEMMs whose launches would each cost
 * the fixed pipeline latency). Problems with m = 0 are skipped. */
FMD_API fmd_status fmd_gemm_tf32x3_grouped(const fmd_gemm_problem* problems, int32_t n_problems, int32_t* flags,
                                           void* stream);

/* ------------------------- MACE-architecture message passing (D1, D3, E2) */

/* The message-passing backbone of the MACE-architecture potential behind
 * fastmd/models/mace.py:356 (MACEAdapter.node_energy, upstream mace-torch
 * 0.3.16 ScaleShiftMACE): channels C (multiple of 32), hidden irreps
 * C x 0e + C x 1o, spherical harmonics l <= 1, correlation 3. Scalars are
 * [N, C], vectors [N, 3, C]; edges follow fmd_refilter_edges (edge_index,
 * edge_image, receiver CSR recv_off, sender CSR send_off/send_perm). */

/* Per edge e = (centre i <- neighbour j): r = pos[j] - pos[i] + image @ cell,
 * d = |r|; ysh [E, 4] = (sqrt(3) r/d, d) (16-byte aligned), phi [E, n_basis]
 * = sqrt(2/r_max) sin(n pi d / r_max) / d * f_cut(d / r_max) with the
 * polynomial cutoff of exponent poly_p (exactly 0 at d >= r_max). `cell` is
 * a DEVICE [3, 3] float32. The radial basis of the reference
 * (fastmd/models/matris/basis_function.py:139 BesselExpansion) in MACE's form. */
FMD_API fmd_status fmd_mace_edge_geometry(const float* positions, const float* cell, const int32_t* edge_index,
                                          const float* edge_image, int64_t n_edges, float r_max, int32_t n_basis,
                                          int32_t poly_p, float* ysh, float* phi, void* stream);

/* Backward of the edge geometry to the positions (the force chain, dE/dr):
 * grad_positions[a] (=|+=) scale * (sum over edges sent by a of g_r(e) - sum
 * over edges received by a of g_r(e)), through both CSRs (no atomics);
 * scale = -1 gives the forces. */
FMD_API fmd_status fmd_mace_edge_geometry_bwd(const float* ysh, const float* grad_y, const float* grad_phi,
                                              float r_max, int32_t n_basis, int32_t poly_p,
                                              const int32_t* edge_index, const int64_t* recv_off,
                                              const int64_t* send_off, const int32_t* send_perm, int64_t n_atoms,
                                              float* grad_positions, float scale, int32_t accumulate,
                                              void* stream);

/* The strain / cell derivative of the edge geometry for the stress (E1, E2):
 * with g_e = d(loss)/d(r_e) from the same gradients as
 * fmd_mace_edge_geometry_bwd, image_grad [3, 3] = scale * sum_e image_e^T g_e
 * (d(loss)/d(cell)) and virial [3, 3] = scale * sum_e r_e^T g_e (either may be
 * null; device float32, accumulated into when accumulate = 1). Edges from
 * *n_real_edges on (device int64, or all when null) are padding and skipped.
 * workspace: FMD_EDGE_VIRIAL_WORKSPACE_DOUBLES doubles of device scratch.
 * Deterministic (fixed grid, fixed reduction order). The cell leaf of the
 * reference's strain derivative (fastmd/engine/energy_derivative.py:110-132). */
#define FMD_EDGE_VIRIAL_WORKSPACE_DOUBLES 5328
FMD_API fmd_status fmd_mace_edge_virial(const float* ysh, const float* grad_y, const float* grad_phi, float r_max,
                                        int32_t n_basis, int32_t poly_p, const float* edge_image, int64_t n_edges,
                                        const int64_t* n_real_edges, double* workspace, float scale,
                                        float* image_grad, float* virial, int32_t accumulate, void* stream);

/* Fused gather -> channel-wise tensor-product message -> receiver segment sum:
 * A0[i] = inv_avg * sum_e (R0 s_t[j] + R3 (v_t[j].Y)/sqrt3),
 * A1[i] = inv_avg * sum_e (R1 s_t[j] Y + R2 v_t[j]) over the receiver run of i
 * (n_paths 2: layer without vector input, R [E, 2C]; 4: R [E, 4C]). */
FMD_API fmd_status fmd_mace_message(const float* R, int32_t n_paths, const float* s_t, const float* v_t,
                                    const float* ysh, const int32_t* edge_index, const int64_t* recv_off,
                                    int64_t n_atoms, int32_t channels, float inv_avg, float* A0, float* A1,
                                    void* stream);

/* Backward of fmd_mace_message: dR [E, P*C], dY [E, 3] (=|+= by accumulate_dy;
 * per receiver run) and ds_t [N, C], dv_t [N, 3, C] (per sender run), deterministic. */
FMD_API fmd_status fmd_mace_message_bwd(const float* dA0, const float* dA1, const float* R, int32_t n_paths,
                                        const float* s_t, const float* v_t, const float* ysh,
                                        const int32_t* edge_index, const int64_t* recv_off,
                                        const int64_t* send_off, const int32_t* send_perm, int64_t n_atoms,
                                        int32_t channels, float inv_avg, float* dR, float* dY,
                                        int32_t accumulate_dy, float* ds_t, float* dv_t, void* stream);

/* Symmetric contraction, correlation 3, l <= 1, element weights W0 [Z, 5, C]
 * (and W1 [Z, 4, C] for the vector output, NULL on the last layer). */
FMD_API fmd_status fmd_mace_product(const float* A0, const float* A1, const int32_t* elem, const float* W0,
                                    const float* W1, int64_t n_atoms, int32_t channels, float* B0, float* B1,
                                    void* stream);
FMD_API fmd_status fmd_mace_product_bwd(const float* dB0, const float* dB1, const float* A0, const float* A1,
                                        const int32_t* elem, const float* W0, const float* W1, int64_t n_atoms,
                                        int32_t channels, float* dA0, float* dA1, void* stream);

/* Element-dependent linear map (MACE's skip connection): y[r] (=|+=) x[r] @ W[z]
 * with z = elem[r / rows_per_atom], W [Z, c_in, c_out] (transpose: x @ W[z]^T). */
FMD_API fmd_status fmd_element_linear(const float* x, int64_t rows, int32_t rows_per_atom, const int32_t* elem,
                                      const float* W, int32_t c_in, int32_t c_out, int32_t transpose, float* y,
                                      int32_t accumulate, void* stream);

/* Node energies E_i = e0[elem_i] + scale * sum_t e_terms[t, i] + shift (fp64) and
 * the fp64 total of each of n_systems systems of n_atoms atoms (block tree). */
FMD_API fmd_status fmd_mace_node_energy(const float* e_terms, int32_t n_terms, int64_t ld_terms,
                                        const int32_t* elem, const double* e0, double scale, double shift,
                                        int64_t n_atoms, int32_t n_systems, double* node_energy, double* total,
                                        void* stream);
/* d_term[i] = scale * d_total[system of i] (the energy terms' gradient). */
FMD_API fmd_status fmd_mace_node_energy_bwd(const double* d_total, double scale, int64_t n_atoms,
                                            int32_t n_systems, float* d_term, void* stream);

/* The whole MACE-architecture energy and force evaluation of one step in ~10
 * fused kernels (the whole-step path; same mathematics as the fmd_mace_*
 * building blocks above). Weights are device pointers prepared once: the
 * radial MLP (per layer, hidden width 64) as [in][out] ("t") and [out][in]
 * copies, the channel mixings lin/out/up as [out][in] and [in][out] ("t"),
 * the symmetric-contraction weights prod0 [Z][5][C] / prod1 [Z][4][C], the
 * element skip matrices skip [Z][in][out] and skipt [Z][out][in], the
 * up-mixed element embedding s_t0 [Z][C], the readouts r0 [C], ra [RH][C],
 * rb [RH] and e0 [Z] (fp64). Pointers of absent pieces (layer 0's up and
 * skip, the last layer's vector output) are NULL.
 * Tensor-core radial MLPs: with radial_tc_min_edges > 0, the TF32 splits
 * (fmd_tf32_split) of W2, W3, W4 as [out][in] (radial_tc_hi/lo[0..2]) and as
 * [in][out] (radial_tc_t_hi/lo[0..2]) given, and the state's radial_pre
 * buffers given, a step of at least radial_tc_min_edges edge rows runs the
 * radial MLPs and their backward as chained fmd_gemm_tf32x3 GEMMs on the
 * pre-activations p1..p3 (3xTF32, FP32 accuracy) instead of the SIMT edge
 * kernels (IEEE FP32). The reference's own wide-GEMM rule takes the 3xTF32
 * path from 65,536 rows in a capture (fastmd/config.py:153,
 * fastmd/engine/kernels/triton_wide_gemm.py:339 _decide); the fused step's
 * whole-step crossover on a B200 lies near 8,192 edge rows (4 replicas of
 * 135 atoms), the host's default for radial_tc_min_edges. */
#define FMD_MACE_MAX_LAYERS 4
typedef struct fmd_mace_fused_weights {
    const float* radial_w1t[FMD_MACE_MAX_LAYERS];
    const float* radial_w2t[FMD_MACE_MAX_LAYERS];
    const float* radial_w3t[FMD_MACE_MAX_LAYERS];
    const float* radial_w4t[FMD_MACE_MAX_LAYERS];
    const float* radial_w1[FMD_MACE_MAX_LAYERS];
    const float* radial_w2[FMD_MACE_MAX_LAYERS];
    const float* radial_w3[FMD_MACE_MAX_LAYERS];
    const float* radial_w4[FMD_MACE_MAX_LAYERS];
    const float* lin0[FMD_MACE_MAX_LAYERS];
    const float* lin1[FMD_MACE_MAX_LAYERS];
    const float* lin0t[FMD_MACE_MAX_LAYERS];
    const float* lin1t[FMD_MACE_MAX_LAYERS];
    const float* out0[FMD_MACE_MAX_LAYERS];
    const float* out1[FMD_MACE_MAX_LAYERS];
    const float* out0t[FMD_MACE_MAX_LAYERS];
    const float* out1t[FMD_MACE_MAX_LAYERS];
    const float* up0[FMD_MACE_MAX_LAYERS];
    const float* up1[FMD_MACE_MAX_LAYERS];
    const float* up0t[FMD_MACE_MAX_LAYERS];
    const float* up1t[FMD_MACE_MAX_LAYERS];
    const float* prod0[FMD_MACE_MAX_LAYERS];
    const float* prod1[FMD_MACE_MAX_LAYERS];
    const float* skip0[FMD_MACE_MAX_LAYERS];
    const float* skip1[FMD_MACE_MAX_LAYERS];
    const float* skip0t[FMD_MACE_MAX_LAYERS];
    const float* skip1t[FMD_MACE_MAX_LAYERS];
    const float* s_t0;
    const float* r0;
    const float* ra;
    const float* rb;
    const double* e0;
    double scale;
    double shift;
    int32_t n_layers;
    int32_t n_basis;
    int32_t poly_p;
    int32_t readout_hidden;
    int32_t radial_hidden;
    float r_max;
    float inv_avg;
    int32_t _pad;
    const float* radial_tc_hi[3][FMD_MACE_MAX_LAYERS];
    const float* radial_tc_lo[3][FMD_MACE_MAX_LAYERS];
    const float* radial_tc_t_hi[3][FMD_MACE_MAX_LAYERS];
    const float* radial_tc_t_lo[3][FMD_MACE_MAX_LAYERS];
    int64_t radial_tc_min_edges;
    /* the node kernels' channel mixings on the tensor cores (with the radial path,
     * 2-layer models): TF32 hi / lo splits (fmd_tf32_split) of lin0, lin1, out0,
     * out1, up0, up1 as [out][in] (index 0..5) and as [in][out] (6..11); NULL:
     * the mixings stay in the node kernels on the CUDA cores */
    const float* node_tc_hi[12][FMD_MACE_MAX_LAYERS];
    const float* node_tc_lo[12][FMD_MACE_MAX_LAYERS];
    /* and the per-element skip mixings: splits of skip0t ([Z][out][in], the forward) and of skip0 (the
     * backward), index 0 / 1 */
    const float* skip_tc_hi[2][FMD_MACE_MAX_LAYERS];
    const float* skip_tc_lo[2][FMD_MACE_MAX_LAYERS];
} fmd_mace_fused_weights;

/* Persistent activations of the fused step (caller-owned device buffers,
 * sized for N atoms and E edge rows): per layer R/dR [E][P*C] (P = 2 for
 * layer 0, else 4), s_t [N][C], v_t/A1/A1l/v_out/dA1/dv_skip [N][3][C],
 * A0/A0l/s_out/dA0/ds_skip [N][C]; ysh [E][4] (16-byte aligned), dY and g_r
 * [E][3], e_term0 [N], node_energy [N] (fp64), elem [N] (element rows) and
 * groups [n_groups][4] (atom ids of the same element, -1 padding);
 * radial_pre[k][L] [E][64] the radial pre-activations p1..p3 of the
 * tensor-core path (NULL when it is not used) and flags (may be NULL) for
 * FMD_FLAG_WAIT_TIMEOUT of its GEMMs. */
typedef struct fmd_mace_fused_state {
    float* R[FMD_MACE_MAX_LAYERS];
    float* dR[FMD_MACE_MAX_LAYERS];
    float* s_t[FMD_MACE_MAX_LAYERS];
    float* v_t[FMD_MACE_MAX_LAYERS];
    float* A0[FMD_MACE_MAX_LAYERS];
    float* A1[FMD_MACE_MAX_LAYERS];
    float* A0l[FMD_MACE_MAX_LAYERS];
    float* A1l[FMD_MACE_MAX_LAYERS];
    float* s_out[FMD_MACE_MAX_LAYERS];
    float* v_out[FMD_MACE_MAX_LAYERS];
    float* dA0[FMD_MACE_MAX_LAYERS];
    float* dA1[FMD_MACE_MAX_LAYERS];
    float* ds_skip[FMD_MACE_MAX_LAYERS];
    float* dv_skip[FMD_MACE_MAX_LAYERS];
    float* ysh;
    float* dY;
    float* g_r;
    float* e_term0;
    double* node_energy;
    const int32_t* elem;
    const int32_t* groups;
    int64_t n_groups;
    float* radial_pre[3][FMD_MACE_MAX_LAYERS];
    int32_t* flags;
    /* the skip mixings of the tensor-core node path (per element, one GEMM problem per element present):
     * elem_order [N] the atoms sorted by element, elem_rank [N] its inverse (device), and n_elem_runs
     * host triples elem_runs_host [n][3] = (element row, first, count) over elem_order; NULL / 0: the skip
     * mixings stay on the CUDA cores */
    const int32_t* elem_order;
    const int32_t* elem_rank;
    int64_t n_elem_runs;
    const int64_t* elem_runs_host;
} fmd_mace_fused_state;

/* Energies and forces of one step: geometry, radial MLPs, messages, node
 * updates, the explicit backward and the force assembly
 * F_a = sum_{received e} dE/dr_e - sum_{sent e} dE/dr_e over both CSRs.
 * forces [N][3] float32, energy [n_systems] fp64 (deterministic sums).
 * edge_index / edge_image / send_perm may be NULL when n_edges is 0.
 * n_real_edges (device int64, may be NULL): the count of real rows; the
 * padding rows after it are skipped by the edge kernels. stages: -1 for the
 * whole step, else a bit mask of the kernels to launch (bit 0 edge forward,
 * 1 messages, 2 node forward, 3 last node update, 4 per-edge message
 * backward, 5 sender/node backward, 6 edge backward, 7 forces) -- a stage
 * launched alone reads what earlier stages left in `state` (for timing).
 * channels 32, 64 or 128. Replaces the energy-tap evaluation of the
 * whole-step runner (whole_step_cuda_graph.py:256 _evaluate with
 * fastmd/engine/energy_derivative.py:110 over mace.py:356). */
FMD_API fmd_status fmd_mace_fused_step(const fmd_mace_fused_weights* weights, const fmd_mace_fused_state* state,
                                       const float* positions, const float* cell, const int32_t* edge_index,
                                       const float* edge_image, int64_t n_edges, const int64_t* n_real_edges,
                                       const int64_t* recv_off,
                                       const int64_t* send_off, const int32_t* send_perm, int64_t atoms_per_system,
                                       int32_t n_systems, int32_t channels, float* forces, double* energy,
                                       int32_t stages, void* stream);

/* ------------------- NequIP-architecture (SevenNet-0-style) backbone (config 3) */

/* Per edge e (centre i receives from neighbour j with its image): the edge
 * vector r = pos[j] - pos[i] + image @ cell (rows at or past *n_real take
 * override_vec[e] instead when it is given: exact-rc padding), the real
 * spherical harmonics Y [E, 9] = [1 | sqrt3 u | sqrt15 xy, sqrt15 yz,
 * sqrt5/2 (3z^2 - 1), sqrt15 xz, sqrt15/2 (x^2 - y^2)] of u = r / |r|, the
 * radial functions B [E, n_basis] = sqrt(2/rc) sin(n pi d / rc) / d times the
 * polynomial envelope of order poly_p, and geo [E, 4] = (u, d) for the
 * backward. The NequIP/SevenNet edge embedding (fastmd/models/sevennet.py,
 * upstream sevenn 0.13.0). */
FMD_API fmd_status fmd_nequip_edge_basis(const float* positions, const float* cell_host, const int32_t* edge_index,
                                         const float* edge_image, const float* override_vec, const int64_t* n_real,
                                         int64_t n_edges, float r_max, int32_t n_basis, int32_t poly_p, float* Y,
                                         float* B, float* geo, void* stream);
/* grad_vec [E, 3] = dE/dr of every edge from dY [E, 9] and dB [E, n_basis]
 * (override rows: 0). */
FMD_API fmd_status fmd_nequip_edge_basis_bwd(const float* geo, const float* dY, const float* dB,
                                             const float* override_vec, const int64_t* n_real, int64_t n_edges,
                                             float r_max, int32_t n_basis, int32_t poly_p, float* grad_vec,
                                             void* stream);
/* The radial-weighted tensor-product convolution of node features x (480 N
 * floats, planar: [N, 128] l0 | [N, 3, 64] l1 | [N, 5, 32] l2; 16-byte
 * aligned) over the 15 coupling paths (l1, l2 -> l3 <= 2, path order l1, l2,
 * l3): messages (3136 N floats, planar: [N, 224] | [N, 3, 384] | [N, 5, 352],
 * a plane's channels the paths with that l3 in path order) = inv_avg * sum
 * over the receiver's edges (recv_off, rows sorted by centre) of W[e, path, u]
 * CG[path] . (x[j, l1, :, u] (x) Y[e, l2]); W [E, 960] (16-byte aligned), cg
 * the 615 dense coupling constants. Deterministic (one warp per receiver, its
 * edges in order). */
FMD_API fmd_status fmd_nequip_conv(const float* x, const float* Y, const float* W, const float* cg,
                                   const int32_t* edge_index, const int64_t* recv_off, int64_t n_atoms, float inv_avg,
                                   float* messages, void* stream);
/* Its backward from grad_messages (the messages' planar layout): grad_W
 * [E, 960] and grad_Y [E, 9] per receiver (grad_Y added to its contents
 * when accumulate_grad_y: the layers of a model share the harmonics), grad_x
 * (x's planar layout) per sender (send_off / send_perm; grad_x null: not
 * formed, for an input that needs no gradient). */
FMD_API fmd_status fmd_nequip_conv_bwd(const float* x, const float* Y, const float* W, const float* cg,
                                       const int32_t* edge_index, const int64_t* recv_off, const int64_t* send_off,
                                       const int32_t* send_perm, int64_t n_atoms, float inv_avg,
                                       const float* grad_messages, float* grad_x, float* grad_W, float* grad_Y,
                                       int32_t accumulate_grad_y, void* stream);
/* Forces of an edge-gradient model: forces[a] = sum over the edges a
 * receives (centre a, recv_off runs) of grad_vec[e] - sum over the edges a
 * sends (neighbour a, send_off runs of send_perm) of grad_vec[e], with
 * grad_vec [E, 3] = dE/d(edge vector r_j - r_i + image). A warp per atom, its
 * lanes over the two runs and a fixed xor tree: deterministic. Replaces the
 * position gradient autograd forms from the edge vectors (the reference's
 * -dE/dpos through torch.autograd.grad, fastmd/models/sevennet.py). */
FMD_API fmd_status fmd_edge_forces(const float* grad_vec, const int32_t* edge_index, const int64_t* recv_off,
                                   const int64_t* send_off, const int32_t* send_perm, int64_t n_atoms,
                                   float* forces, void* stream);

/* The self-connection of the three feature planes (x0 [N, 128], x1
 * [N, 3, 64], x2 [N, 5, 32]): out_l[n, m, c] = sum_u x_l[n, m, u]
 * w_l[elem[n], u, c], w_l [elements, U, U] (SevenNet's element-dependent
 * self-connection linear); transposed = 1 takes w_l[elem[n], c, u] instead
 * (the input gradient). elem: the atoms' element rows (atomic number - 1),
 * checked by the caller. */
FMD_API fmd_status fmd_nequip_self_connection(const float* x0, const float* x1, const float* x2, const int64_t* elem,
                                              const float* w0, const float* w1, const float* w2, int64_t n_atoms,
                                              int32_t transposed, float* out0, float* out1, float* out2,
                                              void* stream);
/* The gated nonlinearity closing an interaction block, plus its
 * self-connection sc (SevenNet's gate after the second linear): x0 =
 * silu(o0[:, :128]) + sc0; x1[n, m, c] = o1[n, m, c] sigmoid(o0[n, 128 + c]) +
 * sc1[n, m, c]; x2[n, m, c] = o2[n, m, c] sigmoid(o0[n, 192 + c]) +
 * sc2[n, m, c]. o0 [N, 224], o1 / sc1 / x1 [N, 3, 64], o2 / sc2 / x2
 * [N, 5, 32], sc0 / x0 [N, 128], all contiguous. */
FMD_API fmd_status fmd_nequip_gate(const float* o0, const float* o1, const float* o2, const float* sc0,
                                   const float* sc1, const float* sc2, int64_t n_atoms, float* x0, float* x1,
                                   float* x2, void* stream);
/* Its backward: grad_o0 / grad_o1 / grad_o2 from grad_x0 / grad_x1 / grad_x2
 * (the self-connection's gradient is grad_x itself). */
FMD_API fmd_status fmd_nequip_gate_bwd(const float* o0, const float* o1, const float* o2, const float* grad_x0,
                                       const float* grad_x1, const float* grad_x2, int64_t n_atoms, float* grad_o0,
                                       float* grad_o1, float* grad_o2, void* stream);

/* ------------------------------ MatRIS geometry, bases, forces (D1, E1) */

/* Per directed edge e = (centre c, neighbour n) [E, 2] int32 with image
 * [E, 3] float32 (lattice units): v = x[c] - (x[n] + image @ L) (image @ L
 * summed over the lattice rows in order), length[e] = |v|, unit [E, 3] =
 * v / |v|. `cell` is a DEVICE [3, 3] float32. An index outside [0, n_atoms)
 * raises FMD_FLAG_INDEX_RANGE (the row reads atom 0). The edge geometry of
 * fastmd/models/matris/processgraph.py:218-233 (process_graphs). */
FMD_API fmd_status fmd_matris_geometry(const float* positions, const float* cell, const int32_t* edge_index,
                                       const float* edge_image, int64_t n_edges, int64_t n_atoms, float* length,
                                       float* unit, int32_t* flags, void* stream);

/* Both Bessel bases of every bond u (length d = length[u2d[u]], or
 * length[u] when u2d is NULL), written rbf_atom [U, ldr] (freq_atom,
 * cutoff_atom) and rbf_line [U, ldr] (freq_line, cutoff_line), each
 * env(d / rc) sqrt(2 / rc) sin(f d / rc) / d with the polynomial envelope of
 * `exponent` in columns [0, n_basis) and zeros up to ldr (a padded K for the
 * projections that follow). Replaces the two BesselExpansion calls of
 * EdgeBasisEmbedding.forward_lengths (fastmd/models/matris/feature_embed.py:
 * 212-247; basis_function.py:31, :139). The frequencies are DEVICE float32
 * [n_basis]. */
FMD_API fmd_status fmd_matris_bessel(const float* length, const int32_t* u2d, int64_t n_bonds, int64_t n_edges,
                                     const float* freq_atom, const float* freq_line, int32_t n_basis,
                                     float cutoff_atom, float cutoff_line, float exponent, float* rbf_atom,
                                     float* rbf_line, int64_t ldr, void* stream);

/* grad_length [U] = sum over both bases of grad_atom / grad_line [U, ldg] .
 * d rbf / d length (frequencies frozen). The backward of fmd_matris_bessel. */
FMD_API fmd_status fmd_matris_bessel_bwd(const float* length, const int32_t* u2d, int64_t n_bonds,
                                         int64_t n_edges, const float* freq_atom, const float* freq_line,
                                         int32_t n_basis, float cutoff_atom, float cutoff_line, float exponent,
                                         const float* grad_atom, const float* grad_line, int64_t ldg,
                                         float* grad_length, void* stream);

/* Fourier basis of every triplet t = (atom, u1, e1, u2, e2) [T, 5] int32:
 * theta = acos((unit[e1] . unit[e2]) (1 - 1e-6)), basis [T, ldb] =
 * [2^-1/2, sin(f_k theta)..., cos(f_k theta)...] / sqrt(pi), zeros in the
 * columns past 1 + 2 n_freq. Replaces ThreebodyEmbedding.forward_vectors + FourierExpansion
 * (fastmd/models/matris/feature_embed.py:432-446, basis_function.py:102)
 * and the basis part of _threebody_fourier_fwd
 * (fastmd/models/matris/op/triton_threebody_fourier.py:48). */
FMD_API fmd_status fmd_matris_threebody(const float* unit, const int32_t* line_graph, int64_t n_triplets,
                                        int64_t n_edges, const float* freq, int32_t n_freq, float* basis,
                                        int64_t ldb, int32_t* flags, void* stream);

/* The backward of fmd_matris_threebody into the unit vectors, with no
 * atomics: grad_cos [T] (scratch, written) = dE / d(unit[e1] . unit[e2]) per
 * triplet, then for every bond u (pair_index [U, 2] int64: its two directed
 * rows) grad_unit of both rows = the sum, in CSR order, of grad_cos[t]
 * unit[e2] over the triplets whose first bond is u (perm1/off1, the CSR of
 * column 1) and of grad_cos[t] unit[e1] over those whose second bond is u
 * (perm2/off2, column 3). Every row named in pair_index is written.
 * Replaces _threebody_fourier_bwd
 * (fastmd/models/matris/op/triton_threebody_fourier.py:100). */
FMD_API fmd_status fmd_matris_threebody_bwd(const float* unit, const int32_t* line_graph, int64_t n_triplets,
                                            int64_t n_edges, const float* freq, int32_t n_freq,
                                            const float* grad_basis, int64_t ldg, const int64_t* pair_index,
                                            int64_t n_bonds, const int64_t* perm1, const int64_t* off1,
                                            const int64_t* perm2, const int64_t* off2, float* grad_cos,
                                            float* grad_unit, void* stream);

/* The line graph's refinement envelope: env [T, width] = base[u2[t]] *
 * base[u1[t]] per triplet t = (atom, u1, e1, u2, e2) [T, 5] int32 (the
 * source bond's row of the learnable envelope base [U, width] times the
 * target bond's), rows 16-byte aligned, width % 4 == 0 (else
 * FMD_ERR_UNSUPPORTED). Replaces _line_envelope_fwd
 * (fastmd/models/matris/op/triton_line_envelope.py:50) and the torch
 * gather-product of Refinement.refinement_rows (interaction_block.py:650-668). */
FMD_API fmd_status fmd_matris_line_envelope(const float* base, int64_t ldb, const int32_t* line_graph,
                                            int64_t n_triplets, int64_t n_bonds, int32_t width, float* env,
                                            int64_t lde, int32_t* flags, void* stream);

/* Its backward, with no atomics: grad_base[u] = sum over the triplets whose
 * target bond is u (perm1/off1: the CSR of column 1) of grad[t] * base[u2[t]],
 * then over those whose source bond is u (perm2/off2, column 3) of grad[t] *
 * base[u1[t]] (eight warps per bond, each taking every eighth triplet of
 * a side, their partials added in warp order: deterministic); every row of
 * grad_base [U, width] is written.
 * Replaces _line_envelope_bwd (triton_line_envelope.py:87). */
FMD_API fmd_status fmd_matris_line_envelope_bwd(const float* base, int64_t ldb, const int32_t* line_graph,
                                                int64_t n_bonds, int32_t width, const float* grad, int64_t ldg,
                                                const int64_t* perm1, const int64_t* off1, const int64_t* perm2,
                                                const int64_t* off2, float* grad_base, int64_t ldo,
                                                void* stream);

/* Forces and stress of the MatRIS energy from the gradients of its two
 * geometric leaves: grad_length [U] (bond lengths, on the bond's stored
 * direction u2d[u]; may be NULL) and grad_unit [E, 3] (may be NULL). Per edge
 * g_e = dE/dv_e = g_d unit + (g_u - (g_u . unit) unit) / length; forces [N, 3]
 * = sum over the atom's neighbour edges of g_e - sum over its centre edges
 * (recv_perm NULL: edges sorted by centre with offsets recv_off [N + 1];
 * send_perm/send_off the CSR of the neighbour column), summed per atom in
 * CSR order (no atomics). With virial_rows [N, 9] FP64 scratch, the per-atom
 * virial v_e (x) g_e over the centre edges; with stress [9] and/or virial
 * [9] (FP64), W = their sum over the atoms in a fixed order, stress =
 * stress_unit (W + W^T) / (2 |det cell|) (`cell` a DEVICE [3, 3] float32;
 * stress_unit = 160.21766208 for GPa).
 * Replaces ForceStressHead.forward's autograd forces and strain stress
 * (fastmd/models/matris/readout.py:200-230, processgraph.py:185-211). */
FMD_API fmd_status fmd_matris_forces(const float* length, const float* unit, const float* grad_length,
                                     const float* grad_unit, const int32_t* d2u, const int32_t* u2d,
                                     const int32_t* edge_index, int64_t n_edges, int64_t n_bonds, int64_t n_atoms,
                                     const int64_t* recv_perm, const int64_t* recv_off, const int64_t* send_perm,
                                     const int64_t* send_off, const float* cell, double stress_unit,
                                     float* forces, double* virial_rows, float* stress, double* virial,
                                     void* stream);

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

/* fmd_nhc_post_force for step n followed by fmd_nhc_pre_force for step n+1
 * in ONE launch (the state, bitwise, of the two calls in a row): the two
 * halves that meet between two force calls inside a whole-step window. The
 * reference runs them as two kernels (gpu_nhc.py:394 then :360). */
FMD_API fmd_status fmd_nhc_post_pre_force(double* state, const double* masses, const double* consts,
                                          int64_t n_atoms, int32_t n_replicas, int32_t tchain, int32_t tloop,
                                          int32_t f32_kick, const float* forces_f32, const double* forces_f64,
                                          const double* energy, float* positions32, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FASTMD_B200_H */
