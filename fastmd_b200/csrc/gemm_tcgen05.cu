// Wide-row FP32 GEMM on the Blackwell tensor cores: tcgen05.mma kind::tf32
// with TMA-fed shared-memory operands and TMEM accumulators, at FP32 accuracy
// (3xTF32). The frozen-weight projections of
// fastmd/engine/kernels/triton_wide_gemm.py (linear :482, matmul :534).
//
//   y[m, n] (=|+=) act( sum_chunks(in(x)[m, :k] . w^T) + bias + c )   w [n, k]
//
// act: SiLU or none; or the SiLU-derivative gate of a backward,
// y = (sum + bias) * silu'(c) with c the pre-activation (then not added).
// in(x): x, or silu(x) applied to the operand as it is split (the next layer
// of an MLP reading the previous layer's pre-activation).
//
// 3xTF32: v = v_hi + v_lo with v_hi = rna_tf32(v), v_lo = v - v_hi, and
// x . w ~ x_lo w_hi + x_hi w_lo + x_hi w_hi (the x_lo w_lo term is below FP32
// rounding; the small cross terms go first). The weight is split once per
// weight version (fmd_tf32_split); x is split in shared memory as it arrives.
// The tensor-core accumulator does not round its additions to nearest, so
// every 64-wide K chunk accumulates in its own TMEM buffer and the chunk sums
// are added in FP32 registers (round to nearest): the error stays flat in K
// (triton_wide_gemm.py:6-13 and _tile :83). A row's result depends on its own
// inputs only, not on m, its tile or the grid.
//
// One persistent CTA per SM (512 threads) walks 128 x 128 output tiles, N
// fastest (the column tiles of a row block run together and share x in L2).
// A stage is 64 of K, one chunk:
//   warp 0      TMA producer: x, w_hi, w_lo as two boxes [128 rows x 32 k]
//               each per stage into a 2-stage shared-memory ring (3 stages
//               for narrow tiles), 128-byte swizzle, zero fill past m, n, k
//   warp 1      TMEM owner and MMA issuer (one thread): per stage 8 K-steps
//               of 8, three products each, into the stage's own chunk
//               accumulator, M = 128, N = 128 (or the tile's width); A
//               (x_hi / x_lo) from TMEM, B (w) from shared memory; one commit
//               releases the stage's shared memory and A buffer, one its
//               accumulator
//   warps 4-7   splitter: row r of the x boxes (one thread per row, reading
//               the swizzled tile) -> x_hi, x_lo -> TMEM lane r (tcgen05.st),
//               double-buffered A operand
//   warps 8-15  epilogue: TMEM -> registers, chunk sums, bias, residual,
//               SiLU, stores; warp w reads TMEM lanes 32 (w % 4) .. +31 (its
//               32 rows) and columns 64 ((w - 8) / 4) .. +63 (narrow tiles:
//               32 ((w - 8) / 4) .. +31)
// TMEM (512 columns): 2 chunk accumulators of 128 columns, then 2 A buffers
// of 128 columns (x_hi k 0..63, x_lo k 0..63); for n <= 64 (narrow) 3
// accumulators of 64 columns, and the w boxes hold n rows (rounded up to 16)
// instead of 128. The single issuing thread pays a fixed cost per tcgen05
// instruction whatever the MMA's N (measured: about 64 cycles per MMA, twice
// that per commit, a few hundred per stage of waits), so the stage is as long
// as the shared memory allows. Keeping A out of shared memory halves the
// tensor core's shared-memory reads (B only).
// Every mbarrier wait is bounded (about a second): on expiry the CTA raises
// FMD_FLAG_WAIT_TIMEOUT, waits (bounded) for its copies and MMAs in flight,
// frees its TMEM and returns. No cluster launch and no multicast.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <string.h>

#include <mutex>

#include "common.cuh"

namespace fmd {
namespace {

// A stage is 64 of K: two TMA boxes of 32 (the 128-byte swizzle width) per operand. The single issuing
// thread pays a fixed cost per tcgen05 instruction (about 64 cycles per MMA and twice that per commit,
// whatever the MMA's N) plus a few hundred cycles per stage of waits and bookkeeping, so a stage of 24
// MMAs and 2 commits (its shared memory and A buffer released by one commit, the chunk accumulator by
// the other) keeps the tensor pipe fed where stages of 12 MMAs and 2.5 commits could not.
constexpr int kBM = 128, kBN = 128, kBK = 32, kStageK = 2 * kBK, kChunkK = kStageK;
static_assert(kBK == 32, "the stage MMA issue is written for 4 K-steps of 8 per box");
constexpr int kStages = 2, kNarrowStages = 3, kMaxStages = 3;
constexpr int kAccBufs = 2, kNarrowAccBufs = 3, kMaxAccBufs = 3, kABufs = 2;
static_assert(kABufs == 2, "the splitter alternates two A buffers");
constexpr int kThreads = 512;
constexpr int kSplitThreads = 128, kEpiThreads = 256;
constexpr uint32_t kTileBytes = kBM * kBK * 4;             // 16 KB: one box of x (or of a 128-row w)
constexpr uint32_t kStageBytes = 2 * 3 * kTileBytes;        // x, w_hi, w_lo: two boxes each (96 KB)
// narrow tiles (n <= 64): w boxes of at most 64 rows, so 3 stages fit where 2 did
constexpr uint32_t kNarrowWBytes = 64 * kBK * 4;                             // 8 KB
constexpr uint32_t kNarrowStageBytes = 2 * (kTileBytes + 2 * kNarrowWBytes);  // 64 KB
static_assert(kNarrowStages * kNarrowStageBytes <= kStages * kStageBytes, "narrow ring within the wide ring");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAccCols = kBN;         // one chunk accumulator: 128 lanes x 128 fp32
constexpr uint32_t kACols = 2 * kStageK;   // one A buffer: x_hi then x_lo, 64 columns each
constexpr uint32_t kNarrowAccCols = 64;    // n <= 64: one chunk accumulator of 64 columns
static_assert(kAccBufs * kAccCols + kABufs * kACols <= kTmemCols, "TMEM budget");
static_assert(kNarrowAccBufs * kNarrowAccCols + kABufs * kACols <= kTmemCols, "TMEM budget (narrow)");
constexpr unsigned long long kWaitNs = 1000000000ull;

struct Ctrl {
    uint64_t full[kMaxStages];       // TMA bytes landed (1 arrival + tx)
    uint64_t empty[kMaxStages];      // MMAs of the stage done (tcgen05.commit): its shared memory and its A buffer
    uint64_t a_full[kABufs];         // x_hi/x_lo of a stage in TMEM (kSplitThreads arrivals)
    uint64_t acc_full[kMaxAccBufs];  // chunk accumulator complete (tcgen05.commit)
    uint64_t acc_empty[kMaxAccBufs]; // chunk accumulator read out (kEpiThreads arrivals)
    uint64_t drain;                  // MMAs in flight on abort
    uint32_t tmem_base;
    int32_t abort;
};

// Output staging: one 32 x 32 fp32 box (4 KB, 128-byte swizzle) per epilogue warp, stored by TMA.
constexpr uint32_t kEpiBoxBytes = 32 * 32 * 4;
constexpr uint32_t kEpiBytes = (kEpiThreads / 32) * kEpiBoxBytes;
constexpr size_t kSmemBytes =
    size_t(kStages) * kStageBytes + kEpiBytes + sizeof(Ctrl) + 1024;  // + 1024-B alignment slack
static_assert(kSmemBytes <= 232448, "shared memory per block");

struct WideArgs {
    const float* bias;  // [n] or null
    const float* c;     // [m, ldc] residual or null
    int64_t ldc;
    float* y;
    int64_t ldy;
    int32_t* flags;
    int64_t m;
    int32_t n, k;
    int32_t act, accumulate;  // act: 0 none, 1 SiLU, 2 times silu'(c)
    int32_t in_silu;          // SiLU on the x operand before the split
    int32_t vec_c, vec_y;     // 16-byte row access valid
    int32_t tma_y;         // y stored through tmap_y (else direct stores)
    uint32_t w_box_bytes;  // bytes of one w_hi / w_lo box (128 B per row of the box)
};

// Up to kMaxGroup independent problems in one launch (fmd_gemm_tf32x3_grouped): their tiles concatenated
// in problem order; every role finds a tile's problem from the running tile counts.
constexpr int kMaxGroup = 4;
struct Group {
    WideArgs p[kMaxGroup];
    int32_t n_problems;
    int32_t tile_end[kMaxGroup];  // tiles of problems 0 .. p
};
struct GroupMaps {
    CUtensorMap x[kMaxGroup], wh[kMaxGroup], wl[kMaxGroup], y[kMaxGroup];
};

// the problem of tile t and the tile's index inside it (one problem: index 0 at compile time, so every
// argument is read at a static parameter offset)
template <bool GROUPED>
__device__ __forceinline__ int problem_of(const Group& G, int t, int& local) {
    if constexpr (!GROUPED) {
        local = t;
        return 0;
    }
    int p = 0;
    while (p + 1 < G.n_problems && t >= G.tile_end[p]) ++p;
    local = t - (p > 0 ? G.tile_end[p - 1] : 0);
    return p;
}

// ------------------------------------------------------------- PTX wrappers

__device__ __forceinline__ uint32_t su32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(su32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     su32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits for the phase of `parity` to complete. Gives up after kWaitNs, or
// as soon as another role of the CTA has given up (abort != 0, unless
// `ignore_abort`); returns false then and sets the CTA's abort word.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int32_t* abort,
                                          bool ignore_abort = false) {
    const uint32_t a = su32(bar);
    if (mbar_try_wait(a, parity)) return true;
    const unsigned long long t0 = global_ns();
    while (true) {
        if (mbar_try_wait(a, parity)) return true;
        if (!ignore_abort && *abort) return false;
        if (global_ns() - t0 > kWaitNs) {
            *abort = 1;
            return false;
        }
    }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(su32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(su32(bar))
        : "memory");
}

// Tile store shared -> global (bulk group); the box outside the tensor is not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(su32(src))
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_read_all() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
                 : "memory");
}

// D (=|+)= A . B^T with A [128 x 8] tf32 in TMEM (lane m, columns k) and B
// from a shared-memory descriptor.
__device__ __forceinline__ void tc_mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// The four K-steps of one product of a 32-wide K stage with every operand precomputed, so the issuing
// thread spends one instruction per MMA (back to back the tensor pipe takes an M = N = 128 MMA about
// every 64 cycles; per-MMA address or predicate arithmetic in a single issuing thread is slower than
// that). A from TMEM (columns a .. a + 31), B from the shared-memory descriptor b; ACC0: whether the
// first MMA adds to D (0 at the start of a chunk).
template <int ACC0>
__device__ __forceinline__ void tc_mma_k32_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc) {
    asm volatile(
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %3, %9, %10;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%2], %4, %9, 1;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%5], %6, %9, 1;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%7], %8, %9, 1;\n\t" ::"r"(d),
        "r"(a), "r"(a + 8), "l"(b), "l"(b + 2), "r"(a + 16), "l"(b + 4), "r"(a + 24), "l"(b + 6), "r"(idesc),
        "n"(ACC0)
        : "memory");
}

// 32 consecutive TMEM columns of this thread's lane (shape 32x32b, x32); with
// `wait`, then the wait for this thread's TMEM stores to land.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32], bool wait) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
    if (wait) asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 16 consecutive TMEM columns of this thread's lane (shape 32x32b, x16) from
// v[0..15]; with `wait`, then the wait for this thread's TMEM stores.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v, bool wait) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15]))
        : "memory");
    if (wait) asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 16 consecutive TMEM columns of this thread's lane (shape 32x32b, x16),
// with the wait in the same statement so no use can move above it.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float rna_tf32(float v) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
    return __uint_as_float(r);
}

// Shared-memory matrix descriptor of a K-major operand tile in the 128-byte
// swizzle: rows of 128 B (32 fp32), 8-row groups 1024 B apart (SBO), the
// leading offset unused (1), descriptor version 1, base offset 0 (tiles are
// 1024-B aligned), layout type 2 = SWIZZLE_128B. A K-step of 8 tf32 inside
// the swizzle atom advances the start address by 32 B (+2 in the field).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return uint64_t((saddr & 0x3FFFFu) >> 4) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
           (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// Instruction descriptor of kind::tf32: FP32 accumulator, A and B TF32,
// both K-major, no negation, N >> 3 at bit 17, M >> 4 at bit 24.
__device__ __forceinline__ uint32_t tf32_idesc(int m, int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

// SiLU as the reference's fused Triton epilogues evaluate it, x * sigmoid(x) with the hardware exp2
// and an approximate divide (a few ulp; 0 for large negative x, x for large positive x).
__device__ __forceinline__ float silu(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// d silu / dx = s (1 + x (1 - s)), s = sigmoid(x), with the same hardware exp2 and divide.
__device__ __forceinline__ float silu_grad(float x) {
    const float s = __fdividef(1.0f, 1.0f + __expf(-x));
    return s * (1.0f + x * (1.0f - s));
}

// ------------------------------------------------------------------ kernel

__device__ __forceinline__ void advance(int& slot, uint32_t& phase, int slots) {
    if (++slot == slots) {
        slot = 0;
        phase ^= 1u;
    }
}

// o[j] = act(acc[j] + bias[col] + c[row, col]) (+ y[row, col] when accumulating) for the 32 columns
// col0 .. col0 + 31 of this thread's row, or (act 2) o[j] = (acc[j] + bias[col]) * silu'(c[row, col]);
// nothing is read outside [0, m) x [0, n). Written as a few whole-row passes, each a straight run of
// predicated loads and arithmetic behind one uniform test: per-element tests inside one unrolled loop
// cost the epilogue warps an instruction fetch at every skipped block.
__device__ __forceinline__ void finish_values(const WideArgs& g, int64_t row, int col0, const float* acc,
                                              float (&o)[32]) {
    const bool row_ok = row < g.m;
    const bool full = col0 + 32 <= g.n;
#pragma unroll
    for (int j = 0; j < 32; ++j) o[j] = acc[j];
    if (g.bias != nullptr) {
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] += (col0 + j < g.n) ? __ldg(g.bias + col0 + j) : 0.0f;
    }
    if (g.c != nullptr && row_ok) {
        const float* cr = g.c + row * g.ldc + col0;
        float cv[32];
        if (full && g.vec_c) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                const float4 c4 = ldg4(cr + j);
                cv[j] = c4.x;
                cv[j + 1] = c4.y;
                cv[j + 2] = c4.z;
                cv[j + 3] = c4.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) cv[j] = (col0 + j < g.n) ? __ldg(cr + j) : 0.0f;
        }
        if (g.act == 2) {
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] *= silu_grad(cv[j]);
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] += cv[j];
        }
    }
    if (g.act == 1) {
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = silu(o[j]);
    }
    if (g.accumulate && row_ok) {  // y (=|+=): the previous y, read before this thread's store
        const float* yr = g.y + row * g.ldy + col0;
        if (full && g.vec_y) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                const float4 yv = *reinterpret_cast<const float4*>(yr + j);
                o[j] += yv.x;
                o[j + 1] += yv.y;
                o[j + 2] += yv.z;
                o[j + 3] += yv.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] += (col0 + j < g.n) ? yr[j] : 0.0f;
        }
    }
}

// The epilogue warps: warp (q, half) reads TMEM lanes 32 q .. +31 (its 32 rows) and the 32 PIECES
// columns from 32 PIECES half of each chunk accumulator (PIECES = 2: 128-column tiles; 1: narrow tiles of
// at most 64 columns), sums the chunks in FP32 (from zeros, as the reference starts from a zero
// accumulator), finishes the values and stores them (32 x 32 TMA boxes staged in shared memory, or
// direct row stores).
template <int PIECES, int ACC_BUFS, bool GROUPED>
__device__ __forceinline__ void epilogue_role(const Group& G, const GroupMaps& maps, Ctrl& ctl,
                                              volatile int32_t* abort, uint32_t tmem, unsigned char* epi_smem,
                                              int warp, int lane, int tiles, uint32_t acc_cols) {
    constexpr int W = 32 * PIECES;
    const int q = warp & 3, half = (warp - 8) >> 2;
    int cb = 0;
    uint32_t cph = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        int local;
        const int pi = problem_of<GROUPED>(G, t, local);
        const WideArgs& g = G.p[pi];
        const int n_tiles = (g.n + kBN - 1) / kBN;
        const int chunks = (g.k + kStageK - 1) / kStageK;
        const int64_t row = int64_t(local / n_tiles) * kBM + q * 32 + lane;
        const int col0 = (local % n_tiles) * kBN + half * W;
        float acc[W];
#pragma unroll
        for (int j = 0; j < W; ++j) acc[j] = 0.0f;
        bool ok = true;
        for (int ch = 0; ch < chunks; ++ch) {
            const bool got = mbar_wait(&ctl.acc_full[cb], cph, abort);
            if (!__all_sync(0xffffffffu, got)) {  // warp-uniform: tcgen05.ld is .sync.aligned
                *abort = 1;
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t ta = tmem + (uint32_t(q * 32) << 16) + uint32_t(cb) * acc_cols + uint32_t(half * W);
#pragma unroll
            for (int part = 0; part < 2 * PIECES; ++part) {
                float v[16];
                tmem_ld16(ta + uint32_t(part * 16), v);
#pragma unroll
                for (int j = 0; j < 16; ++j) acc[part * 16 + j] += v[j];
            }
            tc_fence_before();
            mbar_arrive(&ctl.acc_empty[cb]);
            advance(cb, cph, ACC_BUFS);
        }
        if (!ok) break;
        if (g.tma_y) {
            // stage each 32 x 32 piece in this warp's box (row = lane, 128-byte swizzle) and let
            // TMA store it: whole lines to L2 instead of 16-byte pieces of 32 rows
            float* box = reinterpret_cast<float*>(epi_smem + (warp - 8) * kEpiBoxBytes);
            const int row0 = int(row - lane);
#pragma unroll
            for (int piece = 0; piece < PIECES; ++piece) {
                float o[32];
                finish_values(g, row, col0 + piece * 32, acc + piece * 32, o);
                if (lane == 0) bulk_wait_read_all();  // the previous store has read the box
                __syncwarp();
                float4* b4 = reinterpret_cast<float4*>(box + lane * 32);
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    b4[c ^ (lane & 7)] = make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0 && row0 < g.m && col0 + piece * 32 < g.n)  // boxes with no element in y skipped
                    tma_store_2d(&maps.y[pi], box, col0 + piece * 32, row0);
            }
        } else if (row < g.m) {
            float* yr = g.y + row * g.ldy;
#pragma unroll
            for (int piece = 0; piece < PIECES; ++piece) {
                float o[32];
                finish_values(g, row, col0 + piece * 32, acc + piece * 32, o);
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    const int col = col0 + piece * 32 + j;
                    if (col + 4 <= g.n && g.vec_y) {
                        *reinterpret_cast<float4*>(yr + col) = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
                    } else {
#pragma unroll
                        for (int u = 0; u < 4; ++u)
                            if (col + u < g.n) yr[col + u] = o[j + u];
                    }
                }
            }
        }
    }
    if (lane == 0) bulk_wait_all();  // stores complete before the CTA exits
}

template <bool NARROW, bool GROUPED>
__global__ void __launch_bounds__(kThreads, 1)
    wide_gemm_tf32x3_kernel(const __grid_constant__ GroupMaps maps, const __grid_constant__ Group G) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* ring = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                           ~uintptr_t(1023));
    constexpr int stages = NARROW ? kNarrowStages : kStages;
    constexpr uint32_t stage_bytes = NARROW ? kNarrowStageBytes : kStageBytes;
    // a stage: [x box 0][x box 1][w_hi box 0][w_hi box 1][w_lo box 0][w_lo box 1]
    constexpr uint32_t w_box = NARROW ? kNarrowWBytes : kTileBytes;
    constexpr uint32_t wh_off = 2 * kTileBytes, wl_off = 2 * kTileBytes + 2 * w_box;
    unsigned char* epi_smem = ring + kStages * kStageBytes;
    Ctrl& ctl = *reinterpret_cast<Ctrl*>(epi_smem + kEpiBytes);
    volatile int32_t* abort = &ctl.abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles = G.tile_end[G.n_problems - 1];  // a chunk accumulator per 64-wide K stage
    constexpr int acc_bufs = NARROW ? kNarrowAccBufs : kAccBufs;
    constexpr uint32_t acc_cols = NARROW ? kNarrowAccCols : kAccCols;
    constexpr uint32_t a_base = acc_bufs * acc_cols;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&ctl.full[s], 1);
            mbar_init(&ctl.empty[s], 1);
        }
        for (int b = 0; b < kABufs; ++b) mbar_init(&ctl.a_full[b], kSplitThreads);
        for (int b = 0; b < acc_bufs; ++b) {
            mbar_init(&ctl.acc_full[b], 1);
            mbar_init(&ctl.acc_empty[b], kEpiThreads);
        }
        mbar_init(&ctl.drain, 1);
        ctl.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&ctl.tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl.tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------------------------------------------- producer
            uint32_t armed = 0, armed_ph = 0;  // bit s: stage s has been loaded / in the phase of bit s
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                int local;
                const int pi = problem_of<GROUPED>(G, t, local);
                const WideArgs& g = G.p[pi];
                const int n_tiles = (g.n + kBN - 1) / kBN;
                const int k_stages = (g.k + kStageK - 1) / kStageK;
                const int m0 = (local / n_tiles) * kBM, n0 = (local % n_tiles) * kBN;
                for (int ks = 0; ks < k_stages; ++ks) {
                    if (!mbar_wait(&ctl.empty[s], ph ^ 1u, abort)) {
                        ok = false;
                        break;
                    }
                    unsigned char* st = ring + s * stage_bytes;
                    const int k0 = ks * kStageK;
                    const bool two = k0 + kBK < g.k;  // the second box holds part of K
                    mbar_expect_tx(&ctl.full[s], (two ? 2u : 1u) * (kTileBytes + 2 * g.w_box_bytes));
                    tma_load_2d(st, &maps.x[pi], &ctl.full[s], k0, m0);
                    tma_load_2d(st + wh_off, &maps.wh[pi], &ctl.full[s], k0, n0);
                    tma_load_2d(st + wl_off, &maps.wl[pi], &ctl.full[s], k0, n0);
                    if (two) {
                        tma_load_2d(st + kTileBytes, &maps.x[pi], &ctl.full[s], k0 + kBK, m0);
                        tma_load_2d(st + wh_off + w_box, &maps.wh[pi], &ctl.full[s], k0 + kBK, n0);
                        tma_load_2d(st + wl_off + w_box, &maps.wl[pi], &ctl.full[s], k0 + kBK, n0);
                    }
                    armed |= 1u << s;
                    armed_ph = (armed_ph & ~(1u << s)) | (ph << s);
                    advance(s, ph, stages);
                }
            }
            if (!ok) {  // let the copies in flight land before the CTA exits
                for (int i = 0; i < stages; ++i)
                    if ((armed >> i) & 1u) mbar_wait(&ctl.full[i], (armed_ph >> i) & 1u, abort, true);
            } else {  // tail: the last stages' release arrivals land before the CTA exits
                for (int i = 0; i < stages && mbar_wait(&ctl.empty[s], ph ^ 1u, abort); ++i) advance(s, ph, stages);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------------------------- MMA issuer
            const uint32_t ring_addr = su32(ring);
            int s = 0, sa = 0, cb = 0;
            uint32_t ph = 0, aph = 0, cph = 0;
            bool ok = true, issued = false;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                int local;
                const WideArgs& g = G.p[problem_of<GROUPED>(G, t, local)];
                const int n_tiles = (g.n + kBN - 1) / kBN;
                const int k_stages = (g.k + kStageK - 1) / kStageK;
                const int n0 = (local % n_tiles) * kBN;
                const int nw = min(kBN, g.n - n0);
                const uint32_t idesc = tf32_idesc(kBM, (nw + 15) & ~15);
                for (int ks = 0; ks < k_stages; ++ks) {
                    // a stage is one chunk: its own accumulator, summed by the epilogue in FP32
                    if (!mbar_wait(&ctl.acc_empty[cb], cph ^ 1u, abort) || !mbar_wait(&ctl.full[s], ph, abort) ||
                        !mbar_wait(&ctl.a_full[sa], aph, abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem + uint32_t(cb) * acc_cols;
                    const uint32_t base = ring_addr + uint32_t(s) * stage_bytes;
                    const uint64_t wh = sw128_desc(base + wh_off), wl = sw128_desc(base + wl_off);
                    const uint32_t xh = tmem + a_base + uint32_t(sa) * kACols, xl = xh + kStageK;
                    // per box: the small cross terms first (x_lo w_hi, x_hi w_lo), then x_hi w_hi
                    tc_mma_k32_ts<0>(d, xl, wh, idesc);
                    tc_mma_k32_ts<1>(d, xh, wl, idesc);
                    tc_mma_k32_ts<1>(d, xh, wh, idesc);
                    if (ks * kStageK + kBK < g.k) {  // the second box (a descriptor step of w_box bytes)
                        constexpr uint64_t kBoxStep = w_box >> 4;
                        tc_mma_k32_ts<1>(d, xl + kBK, wh + kBoxStep, idesc);
                        tc_mma_k32_ts<1>(d, xh + kBK, wl + kBoxStep, idesc);
                        tc_mma_k32_ts<1>(d, xh + kBK, wh + kBoxStep, idesc);
                    }
                    issued = true;
                    tc_commit(&ctl.empty[s]);  // the stage's shared memory and its A buffer are free once done
                    tc_commit(&ctl.acc_full[cb]);
                    advance(s, ph, stages);
                    advance(sa, aph, kABufs);
                    advance(cb, cph, acc_bufs);
                }
            }
            if (!ok && issued) {  // the MMAs in flight finish before TMEM is freed
                tc_commit(&ctl.drain);
                mbar_wait(&ctl.drain, 0, abort, true);
            }
        }
    } else if (warp >= 4 && warp < 8) {
        // ------------------------------------------------------- x splitter
        // thread = row r of the tile = TMEM lane r; a box row's 32 floats sit in
        // 8 16-byte chunks, chunk c at position c ^ (r % 8) (128-byte swizzle).
        // The A buffer of stage j (j % 2) is free once stage j - 2's MMAs are done: the completion of
        // that stage's `empty` phase (use (j - 2) / stages of its ring slot). With two ring slots the
        // slot is this stage's own, whose reload already waited for it.
        const int q = warp & 3, r = q * 32 + lane;
        const uint32_t lane_addr = uint32_t(q * 32) << 16;
        int s = 0, sa = 0, j = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
            int local;
            const WideArgs& g = G.p[problem_of<GROUPED>(G, t, local)];
            const int k_stages = (g.k + kStageK - 1) / kStageK;
            for (int ks = 0; ks < k_stages; ++ks, ++j) {
                bool got = mbar_wait(&ctl.full[s], ph, abort);
                if (got && stages != kABufs && j >= kABufs) {
                    const int jp = j - kABufs;
                    got = mbar_wait(&ctl.empty[jp % stages], uint32_t(jp / stages) & 1u, abort);
                }
                if (!__all_sync(0xffffffffu, got)) {  // warp-uniform: tcgen05.st is .sync.aligned
                    *abort = 1;
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t ta = tmem + lane_addr + a_base + uint32_t(sa) * kACols;
                const int boxes = ks * kStageK + kBK < g.k ? 2 : 1;
                for (int b = 0; b < boxes; ++b) {
                    float h[32], v[32];
                    const float4* row = reinterpret_cast<const float4*>(ring + s * stage_bytes + b * kTileBytes + r * 128);
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const float4 f = row[c ^ (r & 7)];
                        v[4 * c] = f.x;
                        v[4 * c + 1] = f.y;
                        v[4 * c + 2] = f.z;
                        v[4 * c + 3] = f.w;
                    }
                    if (g.in_silu) {
#pragma unroll
                        for (int jj = 0; jj < 32; ++jj) v[jj] = silu(v[jj]);
                    }
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) {
                        h[jj] = rna_tf32(v[jj]);
                        v[jj] -= h[jj];
                    }
                    tmem_st32(ta + uint32_t(b * kBK), h, false);
                    tmem_st32(ta + uint32_t(kStageK + b * kBK), v, false);
                }
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                tc_fence_before();
                mbar_arrive(&ctl.a_full[sa]);
                advance(s, ph, stages);
                sa ^= 1;
            }
        }
    } else if (warp >= 8) {
        // --------------------------------------------------------- epilogue
        epilogue_role<NARROW ? 1 : 2, acc_bufs, GROUPED>(G, maps, ctl, abort, tmem, epi_smem, warp, lane, tiles, acc_cols);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                     : "memory");
    }
    if (threadIdx.x == 0 && ctl.abort) raise_flag(G.p[0].flags, FMD_FLAG_WAIT_TIMEOUT);
}

// hi = rna_tf32(w), lo = w - hi, row-major [rows, cols] or, with transpose,
// [cols, rows] (the K-major operand of dX = dY . w), output row stride ldo.
__global__ void tf32_split_kernel(const float* __restrict__ w, int64_t rows, int64_t cols, int64_t ldw,
                                  int transpose, float* __restrict__ hi, float* __restrict__ lo, int64_t ldo) {
    const int64_t total = rows * cols;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total;
         i += int64_t(gridDim.x) * blockDim.x) {
        int64_t r, c, o;
        if (transpose) {  // output row c, column r
            c = i / rows;
            r = i - c * rows;
            o = c * ldo + r;
        } else {
            r = i / cols;
            c = i - r * cols;
            o = r * ldo + c;
        }
        const float v = w[r * ldw + c];
        const float h = rna_tf32(v);
        hi[o] = h;
        lo[o] = v - h;
    }
}

// The tensor pipe's own kind::tf32 rate: one CTA per SM, one thread issuing
// `iters` back-to-back M = 128, N = 128, K = 8 MMAs (A from TMEM, B from
// shared memory, zero operands) with no data movement; the roofline
// denominator of the wide GEMM (2 * 128 * 128 * 8 flops per MMA).
__global__ void __launch_bounds__(128, 1) tf32_mma_rate_kernel(int iters, int32_t* flags) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* b = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                        ~uintptr_t(1023));
    __shared__ uint64_t bar;
    __shared__ uint32_t slot;
    __shared__ int32_t abort_word;
    for (int i = threadIdx.x; i < int(kTileBytes / 4); i += blockDim.x) reinterpret_cast<float*>(b)[i] = 0.f;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_word = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x < 32) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(su32(&slot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = slot;
    {  // A operand columns [128, 136) of every lane: zeros
        float z[16] = {};
        tmem_st16(tmem + (uint32_t((threadIdx.x >> 5) * 32) << 16) + 128u, z, true);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0) {
        const uint64_t bd = sw128_desc(su32(b));
        const uint32_t id = tf32_idesc(128, 128);
        for (int i = 0; i < iters; ++i) tc_mma_tf32_ts(tmem, tmem + 128u, bd, id, i > 0);
        tc_commit(&bar);
        if (!mbar_wait(&bar, 0, &abort_word)) raise_flag(flags, FMD_FLAG_WAIT_TIMEOUT);
    }
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x < 32) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem) : "memory");
    }
}

// Self-test of the bounded wait every pipeline barrier of this file uses (mbar_wait): one thread waits on
// a fresh barrier of count 1; with arrive = 1 it arrives first (the wait completes), with arrive = 0
// nothing ever arrives and the wait gives up after about a second, raising FMD_FLAG_WAIT_TIMEOUT. No copy,
// no MMA and no TMEM is involved, so the expired wait leaves nothing in flight.
__global__ void wait_probe_kernel(int arrive, int32_t* flags) {
    __shared__ uint64_t bar;
    __shared__ int32_t abort_word;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_word = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (arrive) mbar_arrive(&bar);
        if (!mbar_wait(&bar, 0, &abort_word)) raise_flag(flags, FMD_FLAG_WAIT_TIMEOUT);
    }
}

// ------------------------------------------------------------------- host

using EncodeTiled = PFN_cuTensorMapEncodeTiled_v12000;
using CtxGetCurrent = PFN_cuCtxGetCurrent_v4000;

struct DriverCalls {
    EncodeTiled encode = nullptr;
    CtxGetCurrent ctx_get_current = nullptr;
};

// Driver entry points through the runtime (no link against libcuda).
const DriverCalls& driver_calls() {
    static DriverCalls calls;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            calls.encode = reinterpret_cast<EncodeTiled>(p);
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            calls.ctx_get_current = reinterpret_cast<CtxGetCurrent>(p);
    });
    return calls;
}

// [rows, cols] fp32 with row stride ld (elements), box [128 rows x 32 cols],
// 128-byte swizzle, zero fill outside.
CUresult encode_operand(EncodeTiled enc, CUtensorMap* map, const float* base, int64_t rows, int64_t cols,
                        int64_t ld, uint32_t box_rows = kBM) {
    const cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
    const cuuint64_t strides[1] = {cuuint64_t(ld) * sizeof(float)};
    const cuuint32_t box[2] = {cuuint32_t(kBK), box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

struct DeviceInfo {
    bool ready = false;
    bool sm100 = false;
    int sms = 0;
};

// Per-device facts and the one-time shared-memory opt-in (a function
// attribute, set outside any stream capture on the first call).
fmd_status device_info(DeviceInfo* out) {
    static std::mutex mu;
    static DeviceInfo info[64];
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return record_cuda_error(err);
    if (dev < 0 || dev >= 64) return FMD_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(mu);
    DeviceInfo& d = info[dev];
    if (!d.ready) {
        int major = 0, sms = 0;
        if ((err = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
            (err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
            return record_cuda_error(err);
        d.sm100 = major == 10;
        d.sms = sms;
        if (d.sm100) {
            const void* kernels[4] = {(const void*)wide_gemm_tf32x3_kernel<false, false>,
                                      (const void*)wide_gemm_tf32x3_kernel<true, false>,
                                      (const void*)wide_gemm_tf32x3_kernel<false, true>,
                                      (const void*)wide_gemm_tf32x3_kernel<true, true>};
            for (int i = 0; i < 4 && err == cudaSuccess; ++i)
                err = cudaFuncSetAttribute(kernels[i], cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes));
            if (err != cudaSuccess) return record_cuda_error(err);
        }
        d.ready = true;
    }
    *out = d;
    return FMD_OK;
}

// Checks one problem and fills its kernel arguments and tensor maps (narrow: the w boxes hold n rows,
// rounded up to 16, instead of 128).
fmd_status check_problem(const fmd_gemm_problem& q) {
    const int32_t act = q.act;
    if (q.m == 0 && q.n >= 1 && q.k >= 1) return FMD_OK;  // skipped: nothing is read or written
    if (q.m < 0 || q.n < 1 || q.k < 1 || q.m > (int64_t(1) << 31) - kBM || q.x == nullptr || q.w_hi == nullptr ||
        q.w_lo == nullptr || q.y == nullptr || q.ldx < q.k || q.ldw < q.k || q.ldy < q.n ||
        (q.c != nullptr && q.ldc < q.n) || (act & ~(FMD_ACT_MASK | FMD_ACT_INPUT_SILU)) ||
        (act & FMD_ACT_MASK) > FMD_ACT_SILU_GRAD || ((act & FMD_ACT_MASK) == FMD_ACT_SILU_GRAD && q.c == nullptr))
        return FMD_ERR_INVALID_ARGUMENT;
    // TMA: 16-byte aligned bases and row strides
    if (!aligned16(q.x) || !aligned16(q.w_hi) || !aligned16(q.w_lo) || (q.ldx & 3) || (q.ldw & 3))
        return FMD_ERR_UNSUPPORTED;
    if (((q.m + kBM - 1) / kBM) * ((q.n + kBN - 1) / kBN) > INT32_MAX) return FMD_ERR_UNSUPPORTED;
    return FMD_OK;
}

fmd_status prepare_problem(const fmd_gemm_problem& q, bool narrow, EncodeTiled enc, WideArgs& g, CUtensorMap& tx,
                           CUtensorMap& twh, CUtensorMap& twl, CUtensorMap& ty, int64_t& tiles) {
    const int32_t act = q.act;
    tiles = ((q.m + kBM - 1) / kBM) * ((q.n + kBN - 1) / kBN);
    const uint32_t w_rows = narrow ? uint32_t((q.n + 15) & ~15) : uint32_t(kBN);
    CUresult r = encode_operand(enc, &tx, q.x, q.m, q.k, q.ldx);
    if (r == CUDA_SUCCESS) r = encode_operand(enc, &twh, q.w_hi, q.n, q.k, q.ldw, w_rows);
    if (r == CUDA_SUCCESS) r = encode_operand(enc, &twl, q.w_lo, q.n, q.k, q.ldw, w_rows);
    if (r != CUDA_SUCCESS) return record_error_text(FMD_ERR_CUDA, "cuTensorMapEncodeTiled failed, CUresult", r);
    // y through TMA stores (32 x 32 boxes) when its base and row stride allow it
    memset(&ty, 0, sizeof(ty));
    const bool tma_y = aligned16(q.y) && (q.ldy & 3) == 0 &&
                       encode_operand(enc, &ty, q.y, q.m, q.n, q.ldy, 32) == CUDA_SUCCESS;
    g.bias = q.bias;
    g.c = q.c;
    g.ldc = q.ldc;
    g.y = q.y;
    g.ldy = q.ldy;
    g.m = q.m;
    g.n = q.n;
    g.k = q.k;
    g.act = act & FMD_ACT_MASK;
    g.in_silu = (act & FMD_ACT_INPUT_SILU) != 0;
    g.accumulate = q.accumulate != 0;
    g.vec_c = q.c != nullptr && aligned16(q.c) && (q.ldc & 3) == 0;
    g.vec_y = aligned16(q.y) && (q.ldy & 3) == 0;
    g.tma_y = tma_y;
    g.w_box_bytes = w_rows * uint32_t(kBK * sizeof(float));
    return FMD_OK;
}

// The launch of up to kMaxGroup problems: narrow (64-column accumulators) when every n <= 64.
fmd_status launch_group(const fmd_gemm_problem* problems, int32_t n_problems, int32_t* flags, void* stream) {
    if (problems == nullptr || n_problems < 1 || n_problems > kMaxGroup) return FMD_ERR_INVALID_ARGUMENT;
    bool any = false;
    for (int i = 0; i < n_problems; ++i) {
        const fmd_status bad = check_problem(problems[i]);
        if (bad != FMD_OK) return bad;
        any = any || problems[i].m > 0;
    }
    DeviceInfo dev;
    fmd_status st = device_info(&dev);
    if (st != FMD_OK) return st;
    if (!dev.sm100) return FMD_ERR_UNSUPPORTED;
    if (!any) return FMD_OK;
    const DriverCalls& drv = driver_calls();
    if (drv.encode == nullptr || drv.ctx_get_current == nullptr)
        return record_error_text(FMD_ERR_CUDA, "driver entry point cuTensorMapEncodeTiled unavailable", 0);
    // The tensor-map encoder is a driver call: a host thread on which the runtime has not yet made the
    // primary context current (a fresh autograd worker, say) gets it bound first.
    CUcontext current = nullptr;
    if (drv.ctx_get_current(&current) != CUDA_SUCCESS || current == nullptr) {
        int dev_index = 0;
        cudaError_t err = cudaGetDevice(&dev_index);
        if (err == cudaSuccess) err = cudaSetDevice(dev_index);
        if (err != cudaSuccess) return record_cuda_error(err);
    }
    bool narrow = true;
    for (int i = 0; i < n_problems; ++i) narrow = narrow && problems[i].n <= int32_t(kNarrowAccCols);
    GroupMaps maps;
    Group G;
    memset(&maps, 0, sizeof(maps));
    memset(&G, 0, sizeof(G));
    int64_t total = 0;
    for (int i = 0; i < n_problems; ++i) {
        if (problems[i].m == 0) continue;  // nothing to compute
        int64_t tiles = 0;
        WideArgs g;
        memset(&g, 0, sizeof(g));
        st = prepare_problem(problems[i], narrow, drv.encode, g, maps.x[G.n_problems], maps.wh[G.n_problems],
                             maps.wl[G.n_problems], maps.y[G.n_problems], tiles);
        if (st != FMD_OK) return st;
        g.flags = flags;
        total += tiles;
        if (total > INT32_MAX) return FMD_ERR_UNSUPPORTED;
        G.p[G.n_problems] = g;
        G.tile_end[G.n_problems] = int32_t(total);
        ++G.n_problems;
    }
    if (G.n_problems == 0) return FMD_OK;
    const int grid = int(total < dev.sms ? total : dev.sms);
    const cudaStream_t s = as_stream(stream);
    if (G.n_problems == 1) {
        if (narrow) wide_gemm_tf32x3_kernel<true, false><<<grid, kThreads, kSmemBytes, s>>>(maps, G);
        else wide_gemm_tf32x3_kernel<false, false><<<grid, kThreads, kSmemBytes, s>>>(maps, G);
    } else {
        if (narrow) wide_gemm_tf32x3_kernel<true, true><<<grid, kThreads, kSmemBytes, s>>>(maps, G);
        else wide_gemm_tf32x3_kernel<false, true><<<grid, kThreads, kSmemBytes, s>>>(maps, G);
    }
    return check_launch();
}

}  // namespace
}  // namespace fmd

using namespace fmd;

extern "C" {

fmd_status fmd_tf32_split(const float* w, int64_t rows, int64_t cols, int64_t ldw, int32_t transpose, float* hi,
                          float* lo, int64_t ldo, void* stream) {
    if (rows < 0 || cols < 0 || (rows > 0 && cols > 0 && (w == nullptr || hi == nullptr || lo == nullptr)) ||
        ldw < cols || ldo < (transpose ? rows : cols))
        return FMD_ERR_INVALID_ARGUMENT;
    if (rows == 0 || cols == 0) return FMD_OK;
    tf32_split_kernel<<<grid_for(rows * cols, 256), 256, 0, as_stream(stream)>>>(w, rows, cols, ldw,
                                                                                 transpose != 0, hi, lo, ldo);
    return check_launch();
}

fmd_status fmd_wait_probe(int32_t arrive, int32_t* flags, void* stream) {
    if (flags == nullptr) return FMD_ERR_INVALID_ARGUMENT;
    wait_probe_kernel<<<1, 32, 0, as_stream(stream)>>>(arrive != 0, flags);
    return check_launch();
}

fmd_status fmd_tf32_mma_rate(int32_t iters, int32_t* flags, void* stream) {
    if (iters < 1) return FMD_ERR_INVALID_ARGUMENT;
    DeviceInfo dev;
    fmd_status st = device_info(&dev);
    if (st != FMD_OK) return st;
    if (!dev.sm100) return FMD_ERR_UNSUPPORTED;
    const int smem = int(kTileBytes) + 1024;
    tf32_mma_rate_kernel<<<dev.sms, 128, smem, as_stream(stream)>>>(iters, flags);
    return check_launch();
}

fmd_status fmd_gemm_tf32x3(const float* x, int64_t ldx, const float* w_hi, const float* w_lo, int64_t ldw,
                           const float* bias, const float* c, int64_t ldc, float* y, int64_t ldy, int64_t m,
                           int32_t n, int32_t k, int32_t act, int32_t accumulate, int32_t* flags, void* stream) {
    const fmd_gemm_problem q{x, ldx, w_hi, w_lo, ldw, bias, c, ldc, y, ldy, m, n, k, act, accumulate};
    return launch_group(&q, 1, flags, stream);
}

fmd_status fmd_gemm_tf32x3_grouped(const fmd_gemm_problem* problems, int32_t n_problems, int32_t* flags,
                                   void* stream) {
    return launch_group(problems, n_problems, flags, stream);
}

}  // extern "C"
