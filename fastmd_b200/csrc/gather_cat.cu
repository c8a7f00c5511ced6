// Gather-cat of node features onto edge rows (forward) and its CSR
// reduction (backward), plus the status/library entry points.
//
// Forward: every CTA owns a contiguous run of output rows; it stages the
// rows' gather indices in shared memory, then its threads walk the run's
// output as one flat sequence of 16-byte vectors, so each warp stores 512
// contiguous bytes and loads 16 contiguous bytes per lane from the source
// row the vector falls in. The output is written once (HBM-bound: the
// algorithmic bytes are the output plus the compulsory source rows).
//
// Backward: no atomics. The gradient of a source row is the sum of the
// gradient rows that gathered it, read through a CSR of the gather index
// (perm/off, or the identity for a sorted index); one warp reduces one
// source row in CSR order, so the result is deterministic.

#include <stdio.h>

#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"

namespace fmd {

static thread_local char g_last_error[256] = "";

fmd_status record_cuda_error(cudaError_t err) {
    snprintf(g_last_error, sizeof(g_last_error), "%s: %s", cudaGetErrorName(err),
             cudaGetErrorString(err));
    return FMD_ERR_CUDA;
}

fmd_status record_error_text(fmd_status status, const char* text, long long code) {
    snprintf(g_last_error, sizeof(g_last_error), "%s (%lld)", text, code);
    return status;
}

fmd_status grant_dynamic_smem(const void* kernel, size_t bytes, bool max_carveout) {
    if (bytes <= 48 * 1024) return FMD_OK;
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return record_cuda_error(err);
    static std::mutex mu;
    static std::map<std::pair<int, const void*>, size_t> granted;
    std::lock_guard<std::mutex> lock(mu);
    size_t& done = granted[std::make_pair(device, kernel)];
    if (bytes <= done) return FMD_OK;
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
    if (err == cudaSuccess && max_carveout)
        err = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (err != cudaSuccess) return record_cuda_error(err);
    done = bytes;
    return FMD_OK;
}

constexpr int kMaxParts = 4;
constexpr int kCatThreads = 256;
constexpr int kCatRowsPerCta = 32;

struct CatParams {
    const float* src[kMaxParts];
    const int64_t* index[kMaxParts];
    int64_t ld[kMaxParts];
    int64_t n_src[kMaxParts];
    int32_t start[kMaxParts + 1];  // column start of each part in vector units
    int32_t n_parts;
    int32_t row_vecs;              // vectors per output row
    int64_t rows;
    int64_t ldo;                   // in elements
    float* out;
    int32_t* flags;
};

// VEC = 4: float4 vectors (all widths, strides and pointers 16-byte aligned),
// VEC = 1: scalar fallback.
template <int VEC>
__global__ void __launch_bounds__(kCatThreads) gather_cat_kernel(CatParams p) {
    __shared__ int64_t s_index[kMaxParts][kCatRowsPerCta];
    const int64_t n_chunks = (p.rows + kCatRowsPerCta - 1) / kCatRowsPerCta;
    for (int64_t chunk = blockIdx.x; chunk < n_chunks; chunk += gridDim.x) {
        const int64_t row0 = chunk * kCatRowsPerCta;
        const int rows_here = int(p.rows - row0 < kCatRowsPerCta ? p.rows - row0 : kCatRowsPerCta);
        __syncthreads();
        for (int t = threadIdx.x; t < p.n_parts * kCatRowsPerCta; t += blockDim.x) {
            int part = t / kCatRowsPerCta, r = t % kCatRowsPerCta;
            int64_t idx = -1;
            if (r < rows_here) {
                if (p.index[part] != nullptr) {
                    idx = p.index[part][row0 + r];
                    if (idx < 0 || idx >= p.n_src[part]) {
                        raise_flag(p.flags, FMD_FLAG_INDEX_RANGE);
                        idx = -1;
                    }
                } else {
                    idx = row0 + r;
                }
            }
            s_index[part][r] = idx;
        }
        __syncthreads();
        // the flat vector walk t = r * row_vecs + v, stepped without a division per vector
        const int step_r = kCatThreads / p.row_vecs, step_v = kCatThreads - step_r * p.row_vecs;
        int r = threadIdx.x / p.row_vecs, v = threadIdx.x - r * p.row_vecs;
        for (; r < rows_here; r += step_r, v += step_v) {
            if (v >= p.row_vecs) {
                v -= p.row_vecs;
                ++r;
                if (r >= rows_here) break;
            }
            int part = 0;
#pragma unroll
            for (int k = 1; k < kMaxParts; ++k) part += (k < p.n_parts && v >= p.start[k]) ? 1 : 0;
            const int col = (v - p.start[part]) * VEC;
            const int64_t src_row = s_index[part][r];
            float* dst = p.out + (row0 + r) * p.ldo + int64_t(v) * VEC;
            // the output is written once and not read back here: evict-first stores keep the
            // gathered node tables in L2
            if constexpr (VEC == 4) {
                float4 val = f4_zero();
                if (src_row >= 0) val = ldg4(p.src[part] + src_row * p.ld[part] + col);
                __stcs(reinterpret_cast<float4*>(dst), val);
            } else {
                float val = 0.f;
                if (src_row >= 0) val = __ldg(p.src[part] + src_row * p.ld[part] + col);
                __stcs(dst, val);
            }
        }
    }
}

// One warp per (source row, 128-column chunk). Lanes own float4 columns; when a
// chunk is narrower than 32 vectors, the warp splits into row slots of LPR
// lanes that walk interleaved rows of the run, then the slots are folded
// with fixed-order shuffles.
template <int VEC>
__global__ void gather_rows_bwd_kernel(const float* __restrict__ gout, int64_t ldgo, int col0,
                                       int width, const int64_t* __restrict__ perm,
                                       const int64_t* __restrict__ off, int64_t n_src,
                                       float* __restrict__ grad, int64_t ldg, int accumulate,
                                       int lanes_per_row) {
    const int lane = threadIdx.x & 31;
    const int warps_per_cta = blockDim.x >> 5;
    const int width_v = (width + VEC - 1) / VEC;
    const int chunk_v = 32;  // vectors per chunk
    const int n_col_chunks = (width_v + chunk_v - 1) / chunk_v;
    const int64_t n_tasks = n_src * n_col_chunks;
    const int slots = 32 / lanes_per_row;
    const int slot = lane / lanes_per_row;
    const int sub = lane - slot * lanes_per_row;
    for (int64_t task = int64_t(blockIdx.x) * warps_per_cta + (threadIdx.x >> 5); task < n_tasks;
         task += int64_t(gridDim.x) * warps_per_cta) {
        const int64_t n = task / n_col_chunks;
        const int cchunk = int(task - n * n_col_chunks);
        const int v = cchunk * chunk_v + sub;
        const bool col_ok = sub < min(chunk_v, width_v - cchunk * chunk_v) && v < width_v;
        const int64_t start = off[n], end = off[n + 1];
        if constexpr (VEC == 4) {
            float4 acc = f4_zero();
            int64_t j = start + slot;
            // eight rows' loads in flight, added in row order (the same sums as one row at a time)
            for (; j + 7 * slots < end; j += 8 * slots) {
                int64_t r[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) r[q] = perm ? perm[j + q * slots] : j + q * slots;
                if (col_ok) {
                    float4 x[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) x[q] = ldg4(gout + r[q] * ldgo + col0 + v * 4);
#pragma unroll
                    for (int q = 0; q < 8; ++q) acc = f4_add(acc, x[q]);
                }
            }
            for (; j < end; j += slots) {
                const int64_t r = perm ? perm[j] : j;
                if (col_ok) acc = f4_add(acc, ldg4(gout + r * ldgo + col0 + v * 4));
            }
            for (int m = lanes_per_row; m < 32; m <<= 1) {
                float4 o = f4_shfl_xor(acc, m);
                // fold slot pairs in a fixed order: lower slot first
                acc = (slot & (m / lanes_per_row)) ? f4_add(o, acc) : f4_add(acc, o);
            }
            if (slot == 0 && col_ok) {
                float* dst = grad + n * ldg + v * 4;
                if (accumulate) acc = f4_add(*reinterpret_cast<float4*>(dst), acc);
                st4(dst, acc);
            }
        } else {
            float acc = 0.f;
            for (int64_t j = start + slot; j < end; j += slots) {
                const int64_t r = perm ? perm[j] : j;
                if (col_ok) acc += __ldg(gout + r * ldgo + col0 + v);
            }
            for (int m = lanes_per_row; m < 32; m <<= 1) {
                float o = __shfl_xor_sync(0xffffffffu, acc, m);
                acc = (slot & (m / lanes_per_row)) ? (o + acc) : (acc + o);
            }
            if (slot == 0 && col_ok) {
                float* dst = grad + n * ldg + v;
                *dst = accumulate ? (*dst + acc) : acc;
            }
        }
    }
}

template <int VEC>
__global__ void copy_rows_kernel(const float* __restrict__ src, int64_t lds, float* __restrict__ dst,
                                 int64_t ldd, int64_t rows, int width_v) {
    const int64_t total = rows * width_v;
    for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < total;
         t += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = t / width_v;
        const int v = int(t - r * width_v);
        if constexpr (VEC == 4) {
            st4(dst + r * ldd + v * 4, ldg4(src + r * lds + v * 4));
        } else {
            dst[r * ldd + v] = __ldg(src + r * lds + v);
        }
    }
}

// lanes per row slot: the smallest power of two holding the chunk's vectors
// Long runs (tens to hundreds of rows per source row): a CTA of kLongWarps warps per (source row,
// 128-column chunk); warp w sums rows w, w + kLongWarps, ... of the run (four rows' loads in flight), then
// warp 0 adds the warps' partials in warp order. Deterministic; float4 columns only.
constexpr int kLongWarps = 8;

__global__ void __launch_bounds__(32 * kLongWarps) gather_rows_bwd_long_kernel(
    const float* __restrict__ gout, int64_t ldgo, int col0, int width, const int64_t* __restrict__ perm,
    const int64_t* __restrict__ off, int64_t n_src, float* __restrict__ grad, int64_t ldg, int accumulate) {
    __shared__ float4 part[kLongWarps][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int width_v = width / 4;
    const int n_col_chunks = (width_v + 31) / 32;
    const int64_t n_tasks = n_src * n_col_chunks;
    for (int64_t task = blockIdx.x; task < n_tasks; task += gridDim.x) {
        const int64_t n = task / n_col_chunks;
        const int v = int(task - n * n_col_chunks) * 32 + lane;
        const bool col_ok = v < width_v;
        const int64_t start = off[n], end = off[n + 1];
        float4 acc = f4_zero();
        int64_t j = start + warp;
        for (; j + 3 * kLongWarps < end; j += 4 * kLongWarps) {
            int64_t r[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) r[q] = perm ? perm[j + q * kLongWarps] : j + q * kLongWarps;
            if (col_ok) {
                float4 x[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) x[q] = ldg4(gout + r[q] * ldgo + col0 + v * 4);
#pragma unroll
                for (int q = 0; q < 4; ++q) acc = f4_add(acc, x[q]);
            }
        }
        for (; j < end; j += kLongWarps) {
            const int64_t r = perm ? perm[j] : j;
            if (col_ok) acc = f4_add(acc, ldg4(gout + r * ldgo + col0 + v * 4));
        }
        part[warp][lane] = acc;
        __syncthreads();
        if (warp == 0 && col_ok) {
            float4 total = part[0][lane];
#pragma unroll
            for (int w = 1; w < kLongWarps; ++w) total = f4_add(total, part[w][lane]);
            float* dst = grad + n * ldg + v * 4;
            if (accumulate) total = f4_add(*reinterpret_cast<float4*>(dst), total);
            st4(dst, total);
        }
        __syncthreads();
    }
}

inline int lanes_for(int width_v) {
    int l = 1;
    while (l < width_v && l < 32) l <<= 1;
    return l;
}

}  // namespace fmd

using namespace fmd;

extern "C" {

int32_t fmd_version(void) { return 100; }

const char* fmd_status_string(fmd_status status) {
    switch (status) {
        case FMD_OK: return "ok";
        case FMD_ERR_INVALID_ARGUMENT: return "invalid argument";
        case FMD_ERR_CUDA: return "CUDA error";
        case FMD_ERR_UNSUPPORTED: return "unsupported";
        case FMD_ERR_WORKSPACE: return "workspace too small";
        default: return "unknown status";
    }
}

const char* fmd_last_error(void) { return g_last_error; }

fmd_status fmd_gather_cat(const fmd_cat_part* parts, int32_t n_parts, int64_t rows, float* out,
                          int64_t ldo, int32_t* flags, void* stream) {
    if (parts == nullptr || n_parts < 1 || n_parts > kMaxParts || rows < 0 || out == nullptr)
        return FMD_ERR_INVALID_ARGUMENT;
    CatParams p{};
    bool vec = aligned16(out) && (ldo % 4 == 0);
    int64_t width = 0;
    for (int k = 0; k < n_parts; ++k) {
        const fmd_cat_part& q = parts[k];
        if (q.src == nullptr || q.width < 0 || q.ld < q.width) return FMD_ERR_INVALID_ARGUMENT;
        p.src[k] = q.src;
        p.index[k] = q.index;
        p.ld[k] = q.ld;
        p.n_src[k] = q.index ? q.n_src : rows;
        vec = vec && aligned16(q.src) && (q.ld % 4 == 0) && (q.width % 4 == 0);
        width += q.width;
    }
    if (ldo < width) return FMD_ERR_INVALID_ARGUMENT;
    if (rows == 0 || width == 0) return FMD_OK;
    const int unit = vec ? 4 : 1;
    int32_t start = 0;
    for (int k = 0; k < n_parts; ++k) {
        p.start[k] = start;
        start += parts[k].width / unit;
    }
    for (int k = n_parts; k <= kMaxParts; ++k) p.start[k] = start;
    p.n_parts = n_parts;
    p.row_vecs = start;
    p.rows = rows;
    p.ldo = ldo;
    p.out = out;
    p.flags = flags;
    const int64_t chunks = (rows + kCatRowsPerCta - 1) / kCatRowsPerCta;
    const int grid = int(chunks < int64_t(kNumSMs) * 8 ? chunks : int64_t(kNumSMs) * 8);
    if (vec)
        gather_cat_kernel<4><<<grid, kCatThreads, 0, as_stream(stream)>>>(p);
    else
        gather_cat_kernel<1><<<grid, kCatThreads, 0, as_stream(stream)>>>(p);
    return check_launch();
}

fmd_status fmd_aligned_gather_cat3(const float* aligned, int64_t lda, const float* gathered,
                                   int64_t ldg, int64_t n_gathered, const int64_t* index_a,
                                   const int64_t* index_b, int64_t rows, int32_t dim, float* out,
                                   int32_t* flags, void* stream) {
    if (index_a == nullptr || index_b == nullptr) return FMD_ERR_INVALID_ARGUMENT;
    fmd_cat_part parts[3] = {
        {aligned, nullptr, lda, rows, dim, 0},
        {gathered, index_a, ldg, n_gathered, dim, 0},
        {gathered, index_b, ldg, n_gathered, dim, 0},
    };
    return fmd_gather_cat(parts, 3, rows, out, int64_t(3) * dim, flags, stream);
}

fmd_status fmd_gather_rows_bwd(const float* gout, int64_t ldgo, int32_t col0, int32_t width,
                               const int64_t* perm, const int64_t* off, int64_t n_src, float* grad,
                               int64_t ldg, int32_t accumulate, void* stream) {
    if (gout == nullptr || off == nullptr || grad == nullptr || width < 0 || n_src < 0 || col0 < 0 ||
        ldg < width || ldgo < col0 + width)
        return FMD_ERR_INVALID_ARGUMENT;
    if (n_src == 0 || width == 0) return FMD_OK;
    const bool vec = aligned16(gout) && aligned16(grad) && ldgo % 4 == 0 && ldg % 4 == 0 &&
                     col0 % 4 == 0 && width % 4 == 0;
    const int unit = vec ? 4 : 1;
    const int width_v = width / unit;
    const int lanes = lanes_for(width_v);
    const int n_col_chunks = (width_v + 31) / 32;
    const int threads = 256;
    const int grid = grid_for(n_src * n_col_chunks * 32, threads, 8);
    if (vec)
        gather_rows_bwd_kernel<4><<<grid, threads, 0, as_stream(stream)>>>(
            gout, ldgo, col0, width, perm, off, n_src, grad, ldg, accumulate, lanes);
    else
        gather_rows_bwd_kernel<1><<<grid, threads, 0, as_stream(stream)>>>(
            gout, ldgo, col0, width, perm, off, n_src, grad, ldg, accumulate, lanes);
    return check_launch();
}

fmd_status fmd_gather_rows_bwd_long(const float* gout, int64_t ldgo, int32_t col0, int32_t width,
                                   const int64_t* perm, const int64_t* off, int64_t n_src, float* grad, int64_t ldg,
                                   int32_t accumulate, void* stream) {
    if (gout == nullptr || off == nullptr || grad == nullptr || width < 0 || col0 < 0 || n_src < 0 ||
        ldgo < col0 + width || ldg < width)
        return FMD_ERR_INVALID_ARGUMENT;
    if (n_src == 0 || width == 0) return FMD_OK;
    if (!aligned16(gout) || !aligned16(grad) || ldgo % 4 || ldg % 4 || col0 % 4 || width % 4)
        return FMD_ERR_UNSUPPORTED;
    const int64_t tasks = n_src * ((width / 4 + 31) / 32);
    const int grid = int(tasks < int64_t(kNumSMs) * 8 ? tasks : int64_t(kNumSMs) * 8);
    gather_rows_bwd_long_kernel<<<grid, 32 * kLongWarps, 0, as_stream(stream)>>>(gout, ldgo, col0, width, perm, off,
                                                                                 n_src, grad, ldg, accumulate);
    return check_launch();
}

fmd_status fmd_zero(void* dst, int64_t bytes, void* stream) {
    if (bytes < 0 || (bytes > 0 && dst == nullptr)) return FMD_ERR_INVALID_ARGUMENT;
    if (bytes == 0) return FMD_OK;
    const cudaError_t err = cudaMemsetAsync(dst, 0, size_t(bytes), as_stream(stream));
    return err == cudaSuccess ? FMD_OK : record_cuda_error(err);
}

fmd_status fmd_copy_rows(const float* src, int64_t lds, float* dst, int64_t ldd, int64_t rows,
                         int32_t width, void* stream) {
    if (src == nullptr || dst == nullptr || rows < 0 || width < 0 || lds < width || ldd < width)
        return FMD_ERR_INVALID_ARGUMENT;
    if (rows == 0 || width == 0) return FMD_OK;
    const bool vec = aligned16(src) && aligned16(dst) && lds % 4 == 0 && ldd % 4 == 0 && width % 4 == 0;
    const int threads = 256;
    if (vec) {
        copy_rows_kernel<4><<<grid_for(rows * (width / 4), threads), threads, 0, as_stream(stream)>>>(
            src, lds, dst, ldd, rows, width / 4);
    } else {
        copy_rows_kernel<1><<<grid_for(rows * width, threads), threads, 0, as_stream(stream)>>>(
            src, lds, dst, ldd, rows, width);
    }
    return check_launch();
}

}  // extern "C"
