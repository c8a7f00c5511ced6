// Directed-edge <-> undirected-pair aggregation of the MatRIS atom graph.
// Each undirected edge u is stored as two directed rows pair[u] = (p0, p1);
// pair is a bijection between the U pairs and the 2U directed rows.
//
//   op 0  average      out[u]  = (in[p0] + in[p1]) * 0.5          in [2U, dim], out [U, dim]
//   op 1  average bwd  out[p0] = out[p1] = in[u] * 0.5            in [U, dim],  out [2U, dim]
//   op 2  expand       out[p0] = out[p1] = in[u]                  in [U, dim],  out [2U, dim]
//   op 3  expand bwd   out[u]  = in[p0] + in[p1]                  in [2U, dim], out [U, dim]
//
// (fastmd/models/matris/op/triton_directed_pair_aggregate.py:61, :83, :105,
// :127). Every output element is one FP32 addition and/or an exact halving,
// so the results equal the reference's bit for bit. The input keeps its row
// stride (a column view of a wider buffer is read in place); outputs are
// contiguous. Pure gathers and scatters, HBM-bound: one thread per (pair,
// 4-column group) with 16-byte loads and stores where the widths and the
// pointers allow it, else one thread per (pair, column); a warp covers 128
// consecutive columns of one pair, so rows move in full 512-byte segments.
// Index values outside [0, 2U) raise FMD_FLAG_INDEX_RANGE: a gathered row
// out of range reads as zero, a scattered row out of range is not written.

#include "common.cuh"

namespace fmd {
namespace {

constexpr int kThreads = 256;

template <int VEC>
struct Vec;
template <>
struct Vec<4> {
    using T = float4;
    __device__ static T load(const float* p) { return ldg4(p); }
    __device__ static void store(float* p, T v) { st4(p, v); }
    __device__ static T zero() { return f4_zero(); }
    __device__ static T add(T a, T b) { return f4_add(a, b); }
    __device__ static T half(T a) { return make_float4(a.x * 0.5f, a.y * 0.5f, a.z * 0.5f, a.w * 0.5f); }
};
template <>
struct Vec<1> {
    using T = float;
    __device__ static T load(const float* p) { return __ldg(p); }
    __device__ static void store(float* p, T v) { *p = v; }
    __device__ static T zero() { return 0.0f; }
    __device__ static T add(T a, T b) { return a + b; }
    __device__ static T half(T a) { return a * 0.5f; }
};

template <int OP, int VEC>
__global__ void __launch_bounds__(kThreads)
    pair_aggregate_kernel(const float* __restrict__ in, int64_t ldi, const int64_t* __restrict__ pair,
                          int64_t n_pairs, int dim, float* __restrict__ out, int32_t* flags) {
    using V = Vec<VEC>;
    const int groups = dim / VEC;
    const int64_t total = n_pairs * groups;
    const int64_t n_dir = 2 * n_pairs;
    for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < total; t += int64_t(gridDim.x) * blockDim.x) {
        const int64_t u = t / groups;
        const int c = int(t - u * groups) * VEC;
        const int64_t i0 = __ldg(pair + 2 * u), i1 = __ldg(pair + 2 * u + 1);
        const bool ok0 = i0 >= 0 && i0 < n_dir, ok1 = i1 >= 0 && i1 < n_dir;
        if (!(ok0 && ok1) && c == 0) raise_flag(flags, FMD_FLAG_INDEX_RANGE);
        if (OP == 0 || OP == 3) {  // gather two directed rows into pair row u
            const typename V::T v0 = ok0 ? V::load(in + i0 * ldi + c) : V::zero();
            const typename V::T v1 = ok1 ? V::load(in + i1 * ldi + c) : V::zero();
            const typename V::T s = V::add(v0, v1);
            V::store(out + u * dim + c, OP == 0 ? V::half(s) : s);
        } else {  // scatter pair row u into both directed rows
            typename V::T v = V::load(in + u * ldi + c);
            if (OP == 1) v = V::half(v);
            if (ok0) V::store(out + i0 * dim + c, v);
            if (ok1) V::store(out + i1 * dim + c, v);
        }
    }
}

template <int OP>
void launch(bool vec4, const float* in, int64_t ldi, const int64_t* pair, int64_t n_pairs, int dim, float* out,
            int32_t* flags, cudaStream_t s) {
    if (vec4) {
        const int64_t work = n_pairs * (dim / 4);
        pair_aggregate_kernel<OP, 4><<<grid_for(work, kThreads), kThreads, 0, s>>>(in, ldi, pair, n_pairs, dim, out,
                                                                                   flags);
    } else {
        pair_aggregate_kernel<OP, 1><<<grid_for(n_pairs * dim, kThreads), kThreads, 0, s>>>(in, ldi, pair, n_pairs,
                                                                                           dim, out, flags);
    }
}

}  // namespace
}  // namespace fmd

using namespace fmd;

extern "C" {

fmd_status fmd_pair_aggregate(int32_t op, const float* in, int64_t ldi, const int64_t* pair_index, int64_t n_pairs,
                              int32_t dim, float* out, int32_t* flags, void* stream) {
    if (op < 0 || op > 3 || n_pairs < 0 || dim < 1 || ldi < dim) return FMD_ERR_INVALID_ARGUMENT;
    if (n_pairs == 0) return FMD_OK;
    if (in == nullptr || pair_index == nullptr || out == nullptr) return FMD_ERR_INVALID_ARGUMENT;
    const bool vec4 = dim % 4 == 0 && ldi % 4 == 0 && aligned16(in) && aligned16(out);
    const cudaStream_t s = as_stream(stream);
    switch (op) {
        case 0: launch<0>(vec4, in, ldi, pair_index, n_pairs, dim, out, flags, s); break;
        case 1: launch<1>(vec4, in, ldi, pair_index, n_pairs, dim, out, flags, s); break;
        case 2: launch<2>(vec4, in, ldi, pair_index, n_pairs, dim, out, flags, s); break;
        default: launch<3>(vec4, in, ldi, pair_index, n_pairs, dim, out, flags, s); break;
    }
    return check_launch();
}

}  // extern "C"
