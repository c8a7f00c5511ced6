// Shared helpers of the libfastmd_b200 kernels: status plumbing, launch
// geometry for the 148-SM B200, warp reductions and vector-load predicates.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "fastmd_b200.h"

namespace fmd {

// B200: 148 SMs (2 dies x 74). Grid-stride kernels launch a multiple of it.
constexpr int kNumSMs = 148;

// Records the CUDA error text for fmd_last_error() (thread local).
fmd_status record_cuda_error(cudaError_t err);

// Records `text (code)` for fmd_last_error() and returns `status`.
fmd_status record_error_text(fmd_status status, const char* text, long long code);

// Raises `kernel`'s dynamic shared-memory limit to `bytes` on the CURRENT device
// when a launch there needs more than 48 KB and more than was granted on that
// device before (max_carveout: also asks for the largest shared-memory carveout).
// The attribute applies to the current device only, so the sizes granted are
// kept per (device, kernel) under a lock; a size already granted on the device
// makes no attribute call (so a launch inside a stream capture that follows an
// eager launch of the same size makes none).
fmd_status grant_dynamic_smem(const void* kernel, size_t bytes, bool max_carveout = false);

inline fmd_status check_launch() {
    cudaError_t err = cudaGetLastError();
    return err == cudaSuccess ? FMD_OK : record_cuda_error(err);
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Grid size for a grid-stride loop over `work` items with `threads` per CTA:
// enough CTAs to cover the work, capped at `per_sm` resident CTAs on every SM.
inline int grid_for(int64_t work, int threads, int per_sm = 8) {
    int64_t blocks = (work + threads - 1) / threads;
    int64_t cap = int64_t(kNumSMs) * per_sm;
    if (blocks > cap) blocks = cap;
    return blocks < 1 ? 1 : int(blocks);
}

__device__ __forceinline__ void raise_flag(int32_t* flags, int32_t bit) {
    if (flags != nullptr) atomicOr(flags, bit);
}

__device__ __forceinline__ float4 ldg4(const float* p) {
    return __ldg(reinterpret_cast<const float4*>(p));
}

__device__ __forceinline__ void st4(float* p, float4 v) {
    *reinterpret_cast<float4*>(p) = v;
}

__device__ __forceinline__ float4 f4_zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }

__device__ __forceinline__ float4 f4_add(float4 a, float4 b) {
    return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

__device__ __forceinline__ float4 f4_mul(float4 a, float4 b) {
    return make_float4(a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w);
}

__device__ __forceinline__ float4 f4_shfl_xor(float4 v, int mask) {
    v.x = __shfl_xor_sync(0xffffffffu, v.x, mask);
    v.y = __shfl_xor_sync(0xffffffffu, v.y, mask);
    v.z = __shfl_xor_sync(0xffffffffu, v.z, mask);
    v.w = __shfl_xor_sync(0xffffffffu, v.w, mask);
    return v;
}

}  // namespace fmd
