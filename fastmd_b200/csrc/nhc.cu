// Nose-Hoover-chain NVT integrator (ASE 3.29 NoseHooverChainNVT step split
// around the force call), fp64, one CTA per replica.
//
// The momenta of a replica stay in registers (EPT per thread) for the whole
// half step; the thermostat scalars (eta, p_eta, Q) are thread-redundant
// registers; the only cross-thread work is the block reduction of
// sum(p^2/m), done 1 + 3*tloop times per half step with a fixed tree
// (deterministic). A replica of more than 4,096 degrees of freedom runs on a
// thread-block cluster of CL CTAs of 512 threads (one CTA of 1,024 would hold
// 16 and more elements per thread in local memory): element
// (k CL + rank) THREADS + thread,
// the CTA totals combined through distributed shared memory in rank order,
// so every CTA of the cluster computes the same thermostat. This file is compiled with --fmad=false so every
// elementwise operation rounds exactly as the NumPy expressions of ASE do;
// exp is CUDA's double exp. The chain length is a template parameter so the
// chain arrays are registers, not local memory.

#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace fmd {

constexpr int kConstQ = 16;  // index of Q[0] in the constants table

template <int THREADS>
__device__ double block_sum(double v, double* smem) {
    constexpr int kWarps = THREADS / 32;
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();  // previous readers of smem are done
    if (lane == 0) smem[warp] = v;
    __syncthreads();
    double t = 0.0;
    if (lane < kWarps) t = smem[lane];
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) t += __shfl_xor_sync(0xffffffffu, t, m);
    return t;
}

template <int M>
struct Chain {
    double pe[M];
    double eta[M];
    double Q[M];
};

// ASE _integrate_p_eta_j for chain element J, ke2 = sum(p^2/m) of the current p
template <int M>
__device__ __forceinline__ void p_eta_j(Chain<M>& c, int J, double ke2, double kT, double ndof_kT,
                                        double delta2, double neg_delta4) {
    double pj = c.pe[J];
    double s = 1.0;
    if (J < M - 1) {
        s = exp((neg_delta4 * c.pe[J + 1]) / c.Q[J + 1]);
        pj = pj * s;
    }
    double g;
    if (J == 0) g = ke2 - ndof_kT;
    else g = (c.pe[J - 1] * c.pe[J - 1]) / c.Q[J - 1] - kT;
    pj = pj + delta2 * g;
    if (J < M - 1) pj = pj * s;
    c.pe[J] = pj;
}

// sum(p^2/m) over the replica: the CTA's block tree, then (CL > 1) the CTA totals of the cluster in rank
// order; smem[32], smem[33] alternate as the published CTA total (a CTA is never two sums ahead of
// another: each sum ends with a cluster barrier)
template <int EPT, int THREADS, int CL>
__device__ __forceinline__ double ke2_sum(const double (&p)[EPT], const double (&m)[EPT],
                                          const bool (&live)[EPT], double* smem, int& slot) {
    double acc = 0.0;
#pragma unroll
    for (int k = 0; k < EPT; ++k)
        if (live[k]) acc += (p[k] * p[k]) / m[k];
    double t = block_sum<THREADS>(acc, smem);
    if constexpr (CL > 1) {
        cg::cluster_group cluster = cg::this_cluster();
        double* pub = smem + 32 + slot;
        if (threadIdx.x == 0) *pub = t;
        cluster.sync();
        t = 0.0;
#pragma unroll
        for (int r = 0; r < CL; ++r) t += *cluster.map_shared_rank(pub, r);
        slot ^= 1;
    }
    return t;
}

// ASE integrate_nhc(p, dt/2) with the Suzuki-Yoshida 4th order sub-steps
template <int M, int EPT, int THREADS, int CL>
__device__ void nhc_half(double (&p)[EPT], const double (&m)[EPT], const bool (&live)[EPT],
                         Chain<M>& c, const double* __restrict__ consts, int tloop, double* smem, int& slot) {
    const double kT = consts[2];
    const double ndof_kT = consts[3];
    double ke2 = ke2_sum<EPT, THREADS, CL>(p, m, live, smem, slot);
    for (int t = 0; t < tloop; ++t) {
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const double delta = consts[4 + 4 * k];
            const double delta2 = consts[5 + 4 * k];
            const double neg_delta4 = consts[6 + 4 * k];
            const double neg_delta = consts[7 + 4 * k];
#pragma unroll
            for (int jj = 0; jj < M; ++jj) p_eta_j<M>(c, M - 1 - jj, ke2, kT, ndof_kT, delta2, neg_delta4);
#pragma unroll
            for (int j = 0; j < M; ++j) c.eta[j] = c.eta[j] + (delta * c.pe[j]) / c.Q[j];
            const double scale = exp((neg_delta * c.pe[0]) / c.Q[0]);
#pragma unroll
            for (int e = 0; e < EPT; ++e) p[e] = p[e] * scale;
            ke2 = ke2_sum<EPT, THREADS, CL>(p, m, live, smem, slot);
#pragma unroll
            for (int j = 0; j < M; ++j) p_eta_j<M>(c, j, ke2, kT, ndof_kT, delta2, neg_delta4);
        }
    }
}

struct NhcArgs {
    double* state;
    const double* masses;
    const double* consts;
    int64_t n_atoms;
    int32_t n_replicas;
    int32_t tloop;
    int32_t f32_kick;
    float* positions32;       // pre: float32 copy of q (may be null)
    const float* forces_f32;  // post
    const double* forces_f64; // post
    const double* energy;     // post (may be null)
};

template <int M>
__device__ __forceinline__ void load_chain(Chain<M>& c, const NhcArgs& a, int64_t n3R, int r) {
    const double* eta = a.state + 3 * n3R + int64_t(r) * M;
    const double* pe = a.state + 3 * n3R + int64_t(a.n_replicas) * M + int64_t(r) * M;
#pragma unroll
    for (int j = 0; j < M; ++j) {
        c.eta[j] = eta[j];
        c.pe[j] = pe[j];
        c.Q[j] = a.consts[kConstQ + j];
    }
}

template <int M>
__device__ __forceinline__ void store_chain(const Chain<M>& c, const NhcArgs& a, int64_t n3R, int r, bool writer) {
    if (!writer) return;
    double* eta = a.state + 3 * n3R + int64_t(r) * M;
    double* pe = a.state + 3 * n3R + int64_t(a.n_replicas) * M + int64_t(r) * M;
#pragma unroll
    for (int j = 0; j < M; ++j) {
        eta[j] = c.eta[j];
        pe[j] = c.pe[j];
    }
}

__device__ __forceinline__ double kick_of(double dt2, double f, int f32_kick) {
    if (f32_kick) return double(__fmul_rn(float(dt2), float(f)));
    return dt2 * f;
}

template <int M, int EPT, int THREADS, int CL>
__global__ void __launch_bounds__(THREADS) nhc_pre_force_kernel(NhcArgs a) {
    __shared__ double smem[34];
    const int r = blockIdx.x / CL, rank = blockIdx.x % CL;
    const bool writer = rank == 0 && threadIdx.x == 0;
    int slot = 0;
    const int64_t n3 = 3 * a.n_atoms;
    const int64_t n3R = n3 * a.n_replicas;
    double* q_ptr = a.state + int64_t(r) * n3;
    double* p_ptr = a.state + n3R + int64_t(r) * n3;
    const double* f_ptr = a.state + 2 * n3R + int64_t(r) * n3;
    const double* m_ptr = a.masses + int64_t(r) * a.n_atoms;
    double p[EPT], m[EPT];
    bool live[EPT];
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
        const int64_t i = threadIdx.x + (int64_t(k) * CL + rank) * THREADS;
        live[k] = i < n3;
        p[k] = live[k] ? p_ptr[i] : 0.0;
        m[k] = live[k] ? m_ptr[i / 3] : 1.0;
    }
    Chain<M> c;
    load_chain<M>(c, a, n3R, r);
    // (1) p = integrate_nhc(p, dt/2)
    nhc_half<M, EPT, THREADS, CL>(p, m, live, c, a.consts, a.tloop, smem, slot);
    const double dt = a.consts[0];
    const double dt2 = a.consts[1];
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
        if (!live[k]) continue;
        const int64_t i = threadIdx.x + (int64_t(k) * CL + rank) * THREADS;
        // (2) p += dt/2 F(q_n), the cached forces
        const double pk = p[k] + kick_of(dt2, f_ptr[i], a.f32_kick);
        // (3) q += dt p / m
        const double q = q_ptr[i] + (dt * pk) / m[k];
        q_ptr[i] = q;
        p_ptr[i] = pk;
        if (a.positions32) a.positions32[int64_t(r) * n3 + i] = float(q);
    }
    store_chain<M>(c, a, n3R, r, writer);
    if constexpr (CL > 1) cg::this_cluster().sync();  // no CTA leaves while another reads its total
}

template <int M, int EPT, int THREADS, int CL>
__global__ void __launch_bounds__(THREADS) nhc_post_force_kernel(NhcArgs a) {
    __shared__ double smem[34];
    const int r = blockIdx.x / CL, rank = blockIdx.x % CL;
    const bool writer = rank == 0 && threadIdx.x == 0;
    int slot = 0;
    const int64_t n3 = 3 * a.n_atoms;
    const int64_t n3R = n3 * a.n_replicas;
    double* p_ptr = a.state + n3R + int64_t(r) * n3;
    double* f_ptr = a.state + 2 * n3R + int64_t(r) * n3;
    const double* m_ptr = a.masses + int64_t(r) * a.n_atoms;
    const double dt2 = a.consts[1];
    double p[EPT], m[EPT];
    bool live[EPT];
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
        const int64_t i = threadIdx.x + (int64_t(k) * CL + rank) * THREADS;
        live[k] = i < n3;
        m[k] = live[k] ? m_ptr[i / 3] : 1.0;
        p[k] = 0.0;
        if (live[k]) {
            const int64_t g = int64_t(r) * n3 + i;
            const double f = a.forces_f32 ? double(a.forces_f32[g]) : a.forces_f64[g];
            // (4) p += dt/2 F(q_{n+1})
            p[k] = p_ptr[i] + kick_of(dt2, f, a.f32_kick);
            f_ptr[i] = f;  // cache F(q_{n+1}) for the next pre-force half
        }
    }
    Chain<M> c;
    load_chain<M>(c, a, n3R, r);
    // (5) p = integrate_nhc(p, dt/2)
    nhc_half<M, EPT, THREADS, CL>(p, m, live, c, a.consts, a.tloop, smem, slot);
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
        const int64_t i = threadIdx.x + (int64_t(k) * CL + rank) * THREADS;
        if (live[k]) p_ptr[i] = p[k];
    }
    store_chain<M>(c, a, n3R, r, writer);
    if constexpr (CL > 1) cg::this_cluster().sync();  // no CTA leaves while another reads its total
    if (a.energy && writer) a.state[3 * n3R + 2 * int64_t(a.n_replicas) * M + r] = a.energy[r];
}

// Step n's second half and step n+1's first half in one launch: p += dt/2 F(q_{n+1}); NHC(dt/2); F, E
// cached; NHC(dt/2); p += dt/2 F(q_{n+1}); q += dt p / m. The momenta, forces and chain stay in registers
// between the halves; every operation is the one of the two separate kernels in the same order, so the
// state is bitwise that of nhc_post_force_kernel followed by nhc_pre_force_kernel.
template <int M, int EPT, int THREADS, int CL>
__global__ void __launch_bounds__(THREADS) nhc_post_pre_kernel(NhcArgs a) {
    __shared__ double smem[34];
    const int r = blockIdx.x / CL, rank = blockIdx.x % CL;
    const bool writer = rank == 0 && threadIdx.x == 0;
    int slot = 0;
    const int64_t n3 = 3 * a.n_atoms;
    const int64_t n3R = n3 * a.n_replicas;
    double* q_ptr = a.state + int64_t(r) * n3;
    double* p_ptr = a.state + n3R + int64_t(r) * n3;
    double* f_ptr = a.state + 2 * n3R + int64_t(r) * n3;
    const double* m_ptr = a.masses + int64_t(r) * a.n_atoms;
    const double dt = a.consts[0];
    const double dt2 = a.consts[1];
    double p[EPT], m[EPT], f[EPT];
    bool live[EPT];
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
        const int64_t i = threadIdx.x + (int64_t(k) * CL + rank) * THREADS;
        live[k] = i < n3;
        m[k] = live[k] ? m_ptr[i / 3] : 1.0;
        p[k] = 0.0;
        f[k] = 0.0;
        if (live[k]) {
            const int64_t g = int64_t(r) * n3 + i;
            f[k] = a.forces_f32 ? double(a.forces_f32[g]) : a.forces_f64[g];
            p[k] = p_ptr[i] + kick_of(dt2, f[k], a.f32_kick);  // (4) of step n
            f_ptr[i] = f[k];
        }
    }
    Chain<M> c;
    load_chain<M>(c, a, n3R, r);
    nhc_half<M, EPT, THREADS, CL>(p, m, live, c, a.consts, a.tloop, smem, slot);  // (5) of step n
    if (a.energy && writer) a.state[3 * n3R + 2 * int64_t(a.n_replicas) * M + r] = a.energy[r];
    nhc_half<M, EPT, THREADS, CL>(p, m, live, c, a.consts, a.tloop, smem, slot);  // (1) of step n+1
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
        if (!live[k]) continue;
        const int64_t i = threadIdx.x + (int64_t(k) * CL + rank) * THREADS;
        const double pk = p[k] + kick_of(dt2, f[k], a.f32_kick);  // (2)
        const double q = q_ptr[i] + (dt * pk) / m[k];              // (3)
        q_ptr[i] = q;
        p_ptr[i] = pk;
        if (a.positions32) a.positions32[int64_t(r) * n3 + i] = float(q);
    }
    store_chain<M>(c, a, n3R, r, writer);
    if constexpr (CL > 1) cg::this_cluster().sync();  // no CTA leaves while another reads its total
}

// KIND 0: pre-force half, 1: post-force half, 2: post-force half then the next pre-force half; CL CTAs
// (a thread-block cluster) per replica
template <int KIND, int M, int EPT, int THREADS, int CL = 1>
inline fmd_status launch_nhc(const NhcArgs& a, cudaStream_t s) {
    auto kernel = KIND == 0 ? nhc_pre_force_kernel<M, EPT, THREADS, CL>
                            : (KIND == 1 ? nhc_post_force_kernel<M, EPT, THREADS, CL> : nhc_post_pre_kernel<M, EPT, THREADS, CL>);
    if constexpr (CL == 1) {
        kernel<<<a.n_replicas, THREADS, 0, s>>>(a);
        return check_launch();
    } else {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(unsigned(a.n_replicas) * CL, 1, 1);
        cfg.blockDim = dim3(THREADS, 1, 1);
        cfg.dynamicSmemBytes = 0;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = CL;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, a);
        return err == cudaSuccess ? check_launch() : record_cuda_error(err);
    }
}

// threads and elements per thread from 3n: the fewest threads (multiple of
// 32, <= 1024) with at most EPT elements each
template <int KIND, int M>
inline fmd_status dispatch_ept(const NhcArgs& a, cudaStream_t s) {
    const int64_t n3 = 3 * a.n_atoms;
    if (n3 <= 128) return launch_nhc<KIND, M, 1, 128>(a, s);
    if (n3 <= 512) return launch_nhc<KIND, M, 1, 512>(a, s);
    if (n3 <= 1024) return launch_nhc<KIND, M, 1, 1024>(a, s);
    if (n3 <= 2048) return launch_nhc<KIND, M, 2, 1024>(a, s);
    if (n3 <= 4096) return launch_nhc<KIND, M, 4, 1024>(a, s);
    // larger replicas: a cluster of 4 or 8 CTAs of 512 threads (registers for the elements and the chain)
    if (n3 <= 8192) return launch_nhc<KIND, M, 4, 512, 4>(a, s);
    if (n3 <= 16384) return launch_nhc<KIND, M, 4, 512, 8>(a, s);
    if (n3 <= 32768) return launch_nhc<KIND, M, 8, 512, 8>(a, s);
    return FMD_ERR_UNSUPPORTED;
}

template <int KIND>
inline fmd_status dispatch_chain(const NhcArgs& a, int tchain, cudaStream_t s) {
    switch (tchain) {
        case 1: return dispatch_ept<KIND, 1>(a, s);
        case 2: return dispatch_ept<KIND, 2>(a, s);
        case 3: return dispatch_ept<KIND, 3>(a, s);
        case 4: return dispatch_ept<KIND, 4>(a, s);
        case 5: return dispatch_ept<KIND, 5>(a, s);
        case 6: return dispatch_ept<KIND, 6>(a, s);
        case 7: return dispatch_ept<KIND, 7>(a, s);
        case 8: return dispatch_ept<KIND, 8>(a, s);
        default: return FMD_ERR_UNSUPPORTED;
    }
}

}  // namespace fmd

using namespace fmd;

extern "C" {

fmd_status fmd_nhc_pre_force(double* state, const double* masses, const double* consts,
                             int64_t n_atoms, int32_t n_replicas, int32_t tchain, int32_t tloop,
                             int32_t f32_kick, float* positions32, void* stream) {
    if (state == nullptr || masses == nullptr || consts == nullptr || n_atoms < 1 || n_replicas < 1 ||
        tloop < 1 || tchain < 1)
        return FMD_ERR_INVALID_ARGUMENT;
    NhcArgs a{state, masses, consts, n_atoms, n_replicas, tloop, f32_kick, positions32,
              nullptr, nullptr, nullptr};
    return dispatch_chain<0>(a, tchain, as_stream(stream));
}

fmd_status fmd_nhc_post_force(double* state, const double* masses, const double* consts,
                              int64_t n_atoms, int32_t n_replicas, int32_t tchain, int32_t tloop,
                              int32_t f32_kick, const float* forces_f32, const double* forces_f64,
                              const double* energy, void* stream) {
    if (state == nullptr || masses == nullptr || consts == nullptr || n_atoms < 1 || n_replicas < 1 ||
        tloop < 1 || tchain < 1 || ((forces_f32 == nullptr) == (forces_f64 == nullptr)))
        return FMD_ERR_INVALID_ARGUMENT;
    NhcArgs a{state, masses, consts, n_atoms, n_replicas, tloop, f32_kick, nullptr,
              forces_f32, forces_f64, energy};
    return dispatch_chain<1>(a, tchain, as_stream(stream));
}

fmd_status fmd_nhc_post_pre_force(double* state, const double* masses, const double* consts, int64_t n_atoms,
                                  int32_t n_replicas, int32_t tchain, int32_t tloop, int32_t f32_kick,
                                  const float* forces_f32, const double* forces_f64, const double* energy,
                                  float* positions32, void* stream) {
    if (state == nullptr || masses == nullptr || consts == nullptr || n_atoms < 1 || n_replicas < 1 ||
        tloop < 1 || tchain < 1 || ((forces_f32 == nullptr) == (forces_f64 == nullptr)))
        return FMD_ERR_INVALID_ARGUMENT;
    NhcArgs a{state, masses, consts, n_atoms, n_replicas, tloop, f32_kick, positions32,
              forces_f32, forces_f64, energy};
    return dispatch_chain<2>(a, tchain, as_stream(stream));
}

}  // extern "C"
