// Deterministic segment sums over a CSR of the rows (no atomics) and the CSR
// metadata they read.
//
// Forward: one warp reduces one (segment, 128-column chunk): lanes own
// float4 columns and walk the run in order; a chunk narrower than 32 vectors
// splits the warp into row slots that walk interleaved rows and are folded
// by fixed-order shuffles. Every output element is therefore a function of
// the CSR and the width only (bitwise reproducible), and each value row is
// read once with 16-byte coalesced loads (HBM-bound).
//
// Backward: row-parallel gather of gout[segment[r]] (coalesced over rows).
//
// Metadata: the identity CSR of sorted segments is a binary search per
// segment; the stable CSR of unsorted segments is a stable radix sort of
// (segment, row) pairs (CUB, header templates compiled here) followed by the
// same search over the sorted keys.

#include <cub/device/device_radix_sort.cuh>

#include "common.cuh"

namespace fmd {

template <int VEC>
__global__ void csr_segsum_kernel(const float* __restrict__ value, int64_t ldv,
                                  const float* __restrict__ weight, int64_t ldw,
                                  const int64_t* __restrict__ perm, const int64_t* __restrict__ off,
                                  int64_t num_segment, int dim, int64_t skip_segment,
                                  float* __restrict__ out, int64_t ldo, int lanes_per_row) {
    const int lane = threadIdx.x & 31;
    const int warps_per_cta = blockDim.x >> 5;
    const int width_v = (dim + VEC - 1) / VEC;
    const int n_col_chunks = (width_v + 31) / 32;
    const int64_t n_tasks = num_segment * n_col_chunks;
    const int slots = 32 / lanes_per_row;
    const int slot = lane / lanes_per_row;
    const int sub = lane - slot * lanes_per_row;
    for (int64_t task = int64_t(blockIdx.x) * warps_per_cta + (threadIdx.x >> 5); task < n_tasks;
         task += int64_t(gridDim.x) * warps_per_cta) {
        const int64_t s = task / n_col_chunks;
        const int cchunk = int(task - s * n_col_chunks);
        const int v = cchunk * 32 + sub;
        const bool col_ok = v < width_v && sub < 32;
        int64_t start = off[s], end = off[s + 1];
        if (s == skip_segment) end = start;
        if constexpr (VEC == 4) {
            float4 acc = f4_zero();
            for (int64_t j = start + slot; j < end; j += slots) {
                const int64_t r = perm ? perm[j] : j;
                if (col_ok) {
                    float4 x = ldg4(value + r * ldv + v * 4);
                    if (weight) x = f4_mul(ldg4(weight + r * ldw + v * 4), x);
                    acc = f4_add(acc, x);
                }
            }
            for (int m = lanes_per_row; m < 32; m <<= 1) acc = f4_add(acc, f4_shfl_xor(acc, m));
            if (slot == 0 && col_ok) st4(out + s * ldo + v * 4, acc);
        } else {
            float acc = 0.f;
            for (int64_t j = start + slot; j < end; j += slots) {
                const int64_t r = perm ? perm[j] : j;
                if (col_ok) {
                    float x = __ldg(value + r * ldv + v);
                    if (weight) x = __ldg(weight + r * ldw + v) * x;
                    acc += x;
                }
            }
            for (int m = lanes_per_row; m < 32; m <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
            if (slot == 0 && col_ok) out[s * ldo + v] = acc;
        }
    }
}

template <int VEC>
__global__ void csr_segsum_bwd_kernel(const float* __restrict__ gout, const float* __restrict__ value,
                                      int64_t ldv, const float* __restrict__ weight, int64_t ldw,
                                      const int64_t* __restrict__ segment, int64_t rows,
                                      int64_t num_segment, int width_v, int64_t skip_segment,
                                      float* __restrict__ gvalue, float* __restrict__ gweight,
                                      int32_t* flags) {
    const int64_t total = rows * width_v;
    const int64_t ldg = int64_t(width_v) * VEC;  // gout/gvalue/gweight are contiguous [*, dim]
    for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < total;
         t += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = t / width_v;
        const int v = int(t - r * width_v);
        const int64_t s = segment[r];
        const bool live = s >= 0 && s < num_segment && s != skip_segment;
        if ((s < 0 || s >= num_segment) && v == 0) raise_flag(flags, FMD_FLAG_INDEX_RANGE);
        if constexpr (VEC == 4) {
            const float4 g = live ? ldg4(gout + s * ldg + v * 4) : f4_zero();
            if (gvalue) st4(gvalue + r * ldg + v * 4, weight ? f4_mul(g, ldg4(weight + r * ldw + v * 4)) : g);
            if (gweight) st4(gweight + r * ldg + v * 4, live ? f4_mul(g, ldg4(value + r * ldv + v * 4)) : f4_zero());
        } else {
            const float g = live ? __ldg(gout + s * ldg + v) : 0.f;
            if (gvalue) gvalue[r * ldg + v] = weight ? g * __ldg(weight + r * ldw + v) : g;
            if (gweight) gweight[r * ldg + v] = live ? g * __ldg(value + r * ldv + v) : 0.f;
        }
    }
}

// off[s] = lower_bound(keys, s) for s in [0, num_segment]
template <typename K>
__global__ void lower_bound_kernel(const K* __restrict__ keys, int64_t rows, int64_t num_segment,
                                   int64_t* __restrict__ off) {
    for (int64_t s = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; s <= num_segment;
         s += int64_t(gridDim.x) * blockDim.x) {
        int64_t lo = 0, hi = rows;
        while (lo < hi) {
            const int64_t mid = (lo + hi) >> 1;
            if (int64_t(keys[mid]) < s) lo = mid + 1; else hi = mid;
        }
        off[s] = lo;
    }
}

__global__ void csr_keys_kernel(const int64_t* __restrict__ segment, int64_t rows, int64_t num_segment,
                                uint32_t* __restrict__ keys, int64_t* __restrict__ vals, int32_t* flags) {
    for (int64_t r = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; r < rows;
         r += int64_t(gridDim.x) * blockDim.x) {
        int64_t s = segment[r];
        if (s < 0 || s >= num_segment) {
            raise_flag(flags, FMD_FLAG_INDEX_RANGE);
            s = num_segment;  // sorted past every run
        }
        keys[r] = uint32_t(s);
        vals[r] = r;
    }
}

inline int lanes_for(int width_v) {
    int l = 1;
    while (l < width_v && l < 32) l <<= 1;
    return l;
}

inline size_t align_up(size_t x) { return (x + 255) & ~size_t(255); }

inline int key_bits(int64_t num_segment) {
    int bits = 1;
    while (bits < 32 && (int64_t(1) << bits) <= num_segment) ++bits;
    return bits;
}

inline fmd_status cub_temp_bytes(int64_t rows, size_t* bytes) {
    size_t temp = 0;
    cudaError_t err = cub::DeviceRadixSort::SortPairs(nullptr, temp, (const uint32_t*)nullptr,
                                                      (uint32_t*)nullptr, (const int64_t*)nullptr,
                                                      (int64_t*)nullptr, int64_t(rows), 0, 32);
    if (err != cudaSuccess) return record_cuda_error(err);
    *bytes = temp;
    return FMD_OK;
}

}  // namespace fmd

using namespace fmd;

extern "C" {

fmd_status fmd_csr_offsets_sorted(const int64_t* segment, int64_t rows, int64_t num_segment,
                                  int64_t* off, void* stream) {
    if ((rows > 0 && segment == nullptr) || off == nullptr || rows < 0 || num_segment < 0)
        return FMD_ERR_INVALID_ARGUMENT;
    const int threads = 256;
    lower_bound_kernel<int64_t><<<grid_for(num_segment + 1, threads), threads, 0, as_stream(stream)>>>(
        segment, rows, num_segment, off);
    return check_launch();
}

fmd_status fmd_csr_build_workspace_bytes(int64_t rows, int64_t num_segment, size_t* bytes) {
    if (bytes == nullptr || rows < 0 || num_segment < 0 || num_segment >= (int64_t(1) << 32) - 1)
        return FMD_ERR_INVALID_ARGUMENT;
    size_t temp = 0;
    fmd_status st = cub_temp_bytes(rows, &temp);
    if (st != FMD_OK) return st;
    *bytes = 2 * align_up(sizeof(uint32_t) * size_t(rows)) + align_up(sizeof(int64_t) * size_t(rows)) +
             align_up(temp);
    return FMD_OK;
}

fmd_status fmd_csr_build(const int64_t* segment, int64_t rows, int64_t num_segment, int64_t* perm,
                         int64_t* off, void* workspace, size_t workspace_bytes, int32_t* flags,
                         void* stream) {
    if ((rows > 0 && (segment == nullptr || perm == nullptr)) || off == nullptr || rows < 0 ||
        num_segment < 0 || num_segment >= (int64_t(1) << 32) - 1)
        return FMD_ERR_INVALID_ARGUMENT;
    size_t need = 0;
    fmd_status st = fmd_csr_build_workspace_bytes(rows, num_segment, &need);
    if (st != FMD_OK) return st;
    if (workspace == nullptr || workspace_bytes < need) return FMD_ERR_WORKSPACE;
    cudaStream_t s = as_stream(stream);
    const int threads = 256;
    if (rows == 0) {
        cudaError_t err = cudaMemsetAsync(off, 0, sizeof(int64_t) * size_t(num_segment + 1), s);
        return err == cudaSuccess ? FMD_OK : record_cuda_error(err);
    }
    char* ws = static_cast<char*>(workspace);
    uint32_t* keys_in = reinterpret_cast<uint32_t*>(ws);
    ws += align_up(sizeof(uint32_t) * size_t(rows));
    uint32_t* keys_out = reinterpret_cast<uint32_t*>(ws);
    ws += align_up(sizeof(uint32_t) * size_t(rows));
    int64_t* vals_in = reinterpret_cast<int64_t*>(ws);
    ws += align_up(sizeof(int64_t) * size_t(rows));
    size_t temp = 0;
    st = cub_temp_bytes(rows, &temp);
    if (st != FMD_OK) return st;
    csr_keys_kernel<<<grid_for(rows, threads), threads, 0, s>>>(segment, rows, num_segment, keys_in,
                                                              vals_in, flags);
    if ((st = check_launch()) != FMD_OK) return st;
    cudaError_t err = cub::DeviceRadixSort::SortPairs(ws, temp, keys_in, keys_out, vals_in, perm,
                                                      int64_t(rows), 0, key_bits(num_segment), s);
    if (err != cudaSuccess) return record_cuda_error(err);
    lower_bound_kernel<uint32_t><<<grid_for(num_segment + 1, threads), threads, 0, s>>>(
        keys_out, rows, num_segment, off);
    return check_launch();
}

fmd_status fmd_csr_segment_sum(const float* value, int64_t ldv, const float* weight, int64_t ldw,
                               const int64_t* perm, const int64_t* off, int64_t num_segment,
                               int32_t dim, int64_t skip_segment, float* out, int64_t ldo,
                               void* stream) {
    if (value == nullptr || off == nullptr || out == nullptr || dim < 0 || num_segment < 0 ||
        ldv < dim || ldo < dim || (weight != nullptr && ldw < dim))
        return FMD_ERR_INVALID_ARGUMENT;
    if (num_segment == 0 || dim == 0) return FMD_OK;
    const bool vec = aligned16(value) && aligned16(out) && ldv % 4 == 0 && ldo % 4 == 0 &&
                     dim % 4 == 0 && (weight == nullptr || (aligned16(weight) && ldw % 4 == 0));
    const int unit = vec ? 4 : 1;
    const int width_v = dim / unit;
    const int lanes = lanes_for(width_v);
    const int n_col_chunks = (width_v + 31) / 32;
    const int threads = 256;
    const int grid = grid_for(num_segment * n_col_chunks * 32, threads, 8);
    if (vec)
        csr_segsum_kernel<4><<<grid, threads, 0, as_stream(stream)>>>(
            value, ldv, weight, ldw, perm, off, num_segment, dim, skip_segment, out, ldo, lanes);
    else
        csr_segsum_kernel<1><<<grid, threads, 0, as_stream(stream)>>>(
            value, ldv, weight, ldw, perm, off, num_segment, dim, skip_segment, out, ldo, lanes);
    return check_launch();
}

fmd_status fmd_csr_segment_sum_bwd(const float* gout, const float* value, int64_t ldv,
                                   const float* weight, int64_t ldw, const int64_t* segment,
                                   int64_t rows, int64_t num_segment, int32_t dim,
                                   int64_t skip_segment, float* gvalue, float* gweight,
                                   int32_t* flags, void* stream) {
    if (gout == nullptr || segment == nullptr || rows < 0 || dim < 0 ||
        (gweight != nullptr && (value == nullptr || ldv < dim)) ||
        (weight != nullptr && ldw < dim))
        return FMD_ERR_INVALID_ARGUMENT;
    if (rows == 0 || dim == 0 || (gvalue == nullptr && gweight == nullptr)) return FMD_OK;
    bool vec = aligned16(gout) && dim % 4 == 0;
    if (gvalue) vec = vec && aligned16(gvalue);
    if (gweight) vec = vec && aligned16(gweight) && aligned16(value) && ldv % 4 == 0;
    if (weight) vec = vec && aligned16(weight) && ldw % 4 == 0;
    const int threads = 256;
    if (vec) {
        csr_segsum_bwd_kernel<4><<<grid_for(rows * (dim / 4), threads), threads, 0, as_stream(stream)>>>(
            gout, value, ldv, weight, ldw, segment, rows, num_segment, dim / 4, skip_segment, gvalue,
            gweight, flags);
    } else {
        csr_segsum_bwd_kernel<1><<<grid_for(rows * dim, threads), threads, 0, as_stream(stream)>>>(
            gout, value, ldv, weight, ldw, segment, rows, num_segment, dim, skip_segment, gvalue,
            gweight, flags);
    }
    return check_launch();
}

}  // extern "C"
