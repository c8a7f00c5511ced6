// NequIP-architecture (SevenNet-0-style) kernels: the edge basis (spherical
// harmonics l <= 2 and Bessel radial functions) with its backward, and the
// radial-weighted tensor-product convolution with its two backward kernels.
//
// Layouts (planar by l, m-major inside a plane, so that every per-l linear
// reads a plane as one [N (2l + 1), channels] matrix). Node features x: the
// planes [N, 128] (l0) | [N, 3, 64] (l1) | [N, 5, 32] (l2), 480 N floats.
// Messages m: [N, 224] | [N, 3, 384] | [N, 5, 352], 3136 N floats; inside a
// plane the channels are the outputs of the coupling paths (l1, l2 -> l3)
// with that l3, in path order (l1, then l2). Per-edge weights W [E, 960]:
// one weight per (path, channel of l1). Edge harmonics Y [E, 9] =
// [1 | sqrt3 u | sqrt15 xy, sqrt15 yz, sqrt5/2 (3z^2 - 1), sqrt15 xz,
// sqrt15/2 (x^2 - y^2)] of the unit edge vector u; CG [615] the 15 dense
// coupling tensors [2 l3 + 1][2 l1 + 1][2 l2 + 1] in path order.
//
// Convolution (one block of 4 warps per receiver i, its edges in CSR order;
// each warp owns a fixed set of paths, a lane per channel u; the receiver's
// 3136 accumulators in shared memory, each owned by one lane: deterministic):
//   m[i, path, u, m3] = inv_avg * sum_e W[e, path, u] sum_m1 A_e[path][m3][m1] x[j(e), l1, u, m1]
// with the edge's coupling matrices A_e[path][m3][m1] = sum_m2 CG[m3, m1, m2]
// Y[e, l2, m2] formed once per edge (179 floats) and shared by all channels:
// 8,512 FMA per edge and layer instead of 29,760.
// Backward per receiver (dW, dY of its edges) and per sender (dx of the atom
// through its sender CSR), the same sums transposed. Each path is a template
// instance: the coupling loops unroll with compile-time indices.

#include <utility>

#include "common.cuh"

namespace fmd {
namespace {

constexpr int kXW = 480;
constexpr int kMW = 3136;
constexpr int kWW = 960;
constexpr int kCGN = 615;

__host__ __device__ constexpr int dim_of(int l) { return 2 * l + 1; }
__host__ __device__ constexpr int mult_of(int l) { return l == 0 ? 128 : (l == 1 ? 64 : 32); }
__host__ __device__ constexpr int x_off(int l) { return l == 0 ? 0 : (l == 1 ? 128 : 320); }
__host__ __device__ constexpr int m_off_of(int l) { return l == 0 ? 0 : (l == 1 ? 224 : 1376); }
__host__ __device__ constexpr int m_mult(int l) { return l == 0 ? 224 : (l == 1 ? 384 : 352); }
__host__ __device__ constexpr int y_off(int l) { return l == 0 ? 0 : (l == 1 ? 1 : 4); }

// the 15 paths with their offsets (weights, message columns, coupling tensor)
struct PathInfo {
    int l1, l2, l3, w_off, m_off, cg_off;
};
constexpr PathInfo kPaths[15] = {
    {0, 0, 0, 0, 0, 0},        {0, 1, 1, 128, 224, 1},    {0, 2, 2, 256, 1376, 10},  {1, 0, 1, 384, 608, 35},
    {1, 1, 0, 448, 128, 44},   {1, 1, 1, 512, 800, 53},   {1, 1, 2, 576, 2016, 80},  {1, 2, 1, 640, 992, 125},
    {1, 2, 2, 704, 2336, 170}, {2, 0, 2, 768, 2656, 245}, {2, 1, 1, 800, 1184, 270}, {2, 1, 2, 832, 2816, 315},
    {2, 2, 0, 864, 192, 390},  {2, 2, 1, 896, 1280, 415}, {2, 2, 2, 928, 2976, 490}};

// a path's channel offset inside its l3 plane, and the staged-row index of its message (u, m3)
__host__ __device__ constexpr int c_off(const PathInfo& pi) {
    return (pi.m_off - m_off_of(pi.l3)) / dim_of(pi.l3);
}
__host__ __device__ constexpr int m_idx(const PathInfo& pi, int u, int m3) {
    return m_off_of(pi.l3) + m3 * m_mult(pi.l3) + c_off(pi) + u;
}
__host__ __device__ constexpr int x_idx(int l, int u, int m) { return x_off(l) + m * mult_of(l) + u; }
// every path's channels tile its l3 plane without gaps or overlaps, in path order
__host__ __device__ constexpr bool planes_tile() {
    int next[3] = {0, 0, 0};
    for (int p = 0; p < 15; ++p) {
        const PathInfo& pi = kPaths[p];
        if ((pi.m_off - m_off_of(pi.l3)) % dim_of(pi.l3) != 0 || c_off(pi) != next[pi.l3]) return false;
        next[pi.l3] += mult_of(pi.l1);
    }
    return next[0] == m_mult(0) && next[1] == m_mult(1) && next[2] == m_mult(2);
}
static_assert(planes_tile(), "message planes");

// the planar address of column t (0..479 / 0..3135) of atom row r
__device__ __forceinline__ int64_t x_planar(int64_t n, int64_t r, int t) {
    const int l = t < 128 ? 0 : (t < 320 ? 1 : 2);
    return n * x_off(l) + r * (dim_of(l) * mult_of(l)) + (t - x_off(l));
}
__device__ __forceinline__ int64_t m_planar(int64_t n, int64_t r, int t) {
    const int l = t < 224 ? 0 : (t < 1376 ? 1 : 2);
    return n * m_off_of(l) + r * (dim_of(l) * m_mult(l)) + (t - m_off_of(l));
}

struct Cell3 {
    float c[9];
};

// ------------------------------------------------------------------ edge basis

struct BasisArgs {
    const float* pos;
    Cell3 cell;
    const int32_t* edge_index;
    const float* edge_image;
    const float* override_vec;  // padded rows' edge vector (exact-rc loops), or null
    const int64_t* n_real;      // rows past it take the override vector (null: every row is real)
    int64_t n_edges;
    float r_max;
    int n_basis, poly_p;
    float* Y;                   // [E, 9]
    float* B;                   // [E, n_basis]
    float* geo;                 // [E, 4] unit vector and length
};

__device__ __forceinline__ float envelope(float x, int p, float& dx) {
    if (!(x < 1.f)) {
        dx = 0.f;
        return 0.f;
    }
    const float pf = float(p);
    const float xp = powf(x, pf - 1.f) * x;  // x^p
    const float a = (pf + 1.f) * (pf + 2.f) / 2.f, b = pf * (pf + 2.f), c = pf * (pf + 1.f) / 2.f;
    const float env = 1.f - a * xp + b * xp * x - c * xp * x * x;
    dx = (-a * pf * xp + b * (pf + 1.f) * xp * x - c * (pf + 2.f) * xp * x * x) / x;
    return env;
}

__global__ void nq_basis_kernel(BasisArgs a) {
    const int64_t n_real = a.n_real ? *a.n_real : a.n_edges;
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < a.n_edges; e += int64_t(gridDim.x) * blockDim.x) {
        float rx, ry, rz;
        if (e < n_real || a.override_vec == nullptr) {
            const int64_t i = a.edge_index[2 * e], j = a.edge_index[2 * e + 1];
            const float ix = a.edge_image[3 * e], iy = a.edge_image[3 * e + 1], iz = a.edge_image[3 * e + 2];
            const float* c = a.cell.c;
            rx = (a.pos[3 * j] - a.pos[3 * i]) + ((ix * c[0] + iy * c[3]) + iz * c[6]);
            ry = (a.pos[3 * j + 1] - a.pos[3 * i + 1]) + ((ix * c[1] + iy * c[4]) + iz * c[7]);
            rz = (a.pos[3 * j + 2] - a.pos[3 * i + 2]) + ((ix * c[2] + iy * c[5]) + iz * c[8]);
        } else {
            rx = a.override_vec[3 * e];
            ry = a.override_vec[3 * e + 1];
            rz = a.override_vec[3 * e + 2];
        }
        const float d = sqrtf((rx * rx + ry * ry) + rz * rz);
        const float inv = d > 0.f ? 1.f / d : 0.f;
        const float x = rx * inv, y = ry * inv, z = rz * inv;
        const float s3 = 1.7320508075688772f, s5 = 2.23606797749979f, s15 = 3.872983346207417f;
        float* Ye = a.Y + 9 * e;
        Ye[0] = 1.f;
        Ye[1] = s3 * x;
        Ye[2] = s3 * y;
        Ye[3] = s3 * z;
        Ye[4] = s15 * x * y;
        Ye[5] = s15 * y * z;
        Ye[6] = s5 * 0.5f * (3.f * z * z - 1.f);
        Ye[7] = s15 * x * z;
        Ye[8] = s15 * 0.5f * (x * x - y * y);
        float denv;
        const float env = envelope(d / a.r_max, a.poly_p, denv);
        const float pref = sqrtf(2.f / a.r_max);
        for (int n = 0; n < a.n_basis; ++n) {
            const float k = float(n + 1) * 3.14159265358979323846f / a.r_max;
            a.B[int64_t(a.n_basis) * e + n] = d > 0.f ? pref * sinf(k * d) * inv * env : 0.f;
        }
        a.geo[4 * e] = x;
        a.geo[4 * e + 1] = y;
        a.geo[4 * e + 2] = z;
        a.geo[4 * e + 3] = d;
    }
}

// g[e] = dE/d(edge vector) from dY and dB (padded override rows: 0)
__global__ void nq_basis_bwd_kernel(BasisArgs a, const float* __restrict__ dY, const float* __restrict__ dB,
                                    float* __restrict__ g) {
    const int64_t n_real = a.n_real ? *a.n_real : a.n_edges;
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < a.n_edges; e += int64_t(gridDim.x) * blockDim.x) {
        const float x = a.geo[4 * e], y = a.geo[4 * e + 1], z = a.geo[4 * e + 2], d = a.geo[4 * e + 3];
        float gx = 0.f, gy = 0.f, gz = 0.f;
        if ((e < n_real || a.override_vec == nullptr) && d > 0.f) {
            const float s3 = 1.7320508075688772f, s5 = 2.23606797749979f, s15 = 3.872983346207417f;
            const float* q = dY + 9 * e;
            // dE/du from the harmonics
            float ux = s3 * q[1] + s15 * (y * q[4] + z * q[7] + x * q[8]);
            float uy = s3 * q[2] + s15 * (x * q[4] + z * q[5] - y * q[8]);
            float uz = s3 * q[3] + s15 * (y * q[5] + x * q[7]) + 3.f * s5 * z * q[6];
            const float inv = 1.f / d;
            const float gu = (ux * x + uy * y) + uz * z;
            gx = (ux - gu * x) * inv;
            gy = (uy - gu * y) * inv;
            gz = (uz - gu * z) * inv;
            // dE/dd from the radial functions
            float denv;
            const float env = envelope(d / a.r_max, a.poly_p, denv);
            const float pref = sqrtf(2.f / a.r_max);
            float gd = 0.f;
            for (int n = 0; n < a.n_basis; ++n) {
                const float k = float(n + 1) * 3.14159265358979323846f / a.r_max;
                float sn, cs;
                sincosf(k * d, &sn, &cs);
                const float b = pref * sn * inv;
                const float db = pref * (k * cs * d - sn) * inv * inv;
                gd += dB[int64_t(a.n_basis) * e + n] * (db * env + b * denv / a.r_max);
            }
            gx += gd * x;
            gy += gd * y;
            gz += gd * z;
        }
        g[3 * e] = gx;
        g[3 * e + 1] = gy;
        g[3 * e + 2] = gz;
    }
}

// ------------------------------------------------------------------ convolution

struct ConvArgs {
    const float* x;          // 480 N floats, planar
    const float* Y;          // [E, 9]
    const float* W;          // [E, 960]
    const float* cg;         // [615]
    const int32_t* edge_index;
    const int64_t* recv_off;  // [N + 1] receiver CSR (rows sorted by centre)
    const int64_t* send_off;  // [N + 1] sender CSR
    const int32_t* send_perm;
    int64_t n_atoms;
    float inv_avg;
};

// A[path][m3][m1] = sum_m2 CG[path][m3, m1, m2] Y[e, l2, m2]: the edge's coupling matrices, shared by
// every channel u of a path (179 floats per edge); the lanes split their entries
__host__ __device__ constexpr int a_size(int P) { return dim_of(kPaths[P].l3) * dim_of(kPaths[P].l1); }
__host__ __device__ constexpr int a_off(int P) {
    int s = 0;
    for (int q = 0; q < P; ++q) s += a_size(q);
    return s;
}
constexpr int kAW = a_off(15);  // 179
template <int P>
__device__ __forceinline__ void path_coupling(const float* cg, const float* y, float* aw, int lane) {
    constexpr PathInfo pi = kPaths[P];
    constexpr int n1 = dim_of(pi.l1), n2 = dim_of(pi.l2);
    for (int t = lane; t < a_size(P); t += 32) {
        const int m3 = t / n1, m1 = t - m3 * n1;
        float s = 0.f;
#pragma unroll
        for (int m2 = 0; m2 < n2; ++m2) s = fmaf(cg[pi.cg_off + (m3 * n1 + m1) * n2 + m2], y[y_off(pi.l2) + m2], s);
        aw[a_off(P) + t] = s;
    }
}

template <int... P>
__device__ __forceinline__ void edge_couplings(const float* cg, const float* y, float* aw, int lane,
                                               std::integer_sequence<int, P...>) {
    (path_coupling<P>(cg, y, aw, lane), ...);
}

// the coupling matrices of edge e in the warp's aw (ends with a warp barrier)
__device__ __forceinline__ void load_couplings(const ConvArgs& a, const float* cg, int64_t e, float* aw, int lane) {
    float y[9];
#pragma unroll
    for (int q = 0; q < 9; ++q) y[q] = a.Y[9 * e + q];
    __syncwarp();  // the previous edge's readers are done
    edge_couplings(cg, y, aw, lane, std::make_integer_sequence<int, 15>{});
    __syncwarp();
}

// one path's contribution of edge e (lane channels u) into the receiver's accumulators:
// acc[m3, u] += W[e, path, u] sum_m1 A[m3][m1] x[j, l1, m1, u]
template <int P>
__device__ __forceinline__ void path_fwd(const float* ws, const float* xs, const float* aw, float* acc, int lane) {
    constexpr PathInfo pi = kPaths[P];
    constexpr int n1 = dim_of(pi.l1), n3 = dim_of(pi.l3), U = mult_of(pi.l1);
#pragma unroll 1
    for (int u = lane; u < U; u += 32) {
        const float w = ws[pi.w_off + u];
        float xv[n1];
#pragma unroll
        for (int m1 = 0; m1 < n1; ++m1) xv[m1] = xs[x_idx(pi.l1, u, m1)];
#pragma unroll
        for (int m3 = 0; m3 < n3; ++m3) {
            float s = 0.f;
#pragma unroll
            for (int m1 = 0; m1 < n1; ++m1) s = fmaf(aw[a_off(P) + m3 * n1 + m1], xv[m1], s);
            acc[m_idx(pi, u, m3)] = fmaf(w, s, acc[m_idx(pi, u, m3)]);
        }
    }
}

template <int... P>
__device__ __forceinline__ void all_paths_fwd(const float* ws, const float* xs, const float* aw, float* acc, int lane,
                                              std::integer_sequence<int, P...>) {
    (path_fwd<P>(ws, xs, aw, acc, lane), ...);
}

// A receiver's edges are shared by the 4 warps of its block: each warp owns a fixed set of paths
// (disjoint message columns, disjoint dW columns), balanced by FMA count per edge (U n3 n1 summed:
// 2048, 2080, 2176, 2208 of 8512). The block stages the edge's weight and sender rows once; a warp
// forms only its own paths' coupling matrices.
constexpr int kRecvThreads = 128;
using Warp0Paths = std::integer_sequence<int, 6, 8, 0>;
using Warp1Paths = std::integer_sequence<int, 9, 11, 10>;
using Warp2Paths = std::integer_sequence<int, 14, 2, 3, 12>;
using Warp3Paths = std::integer_sequence<int, 5, 7, 1, 13, 4>;

template <int... P>
__device__ __forceinline__ void couplings_of(const float* cg, const float* y, float* aw, int lane,
                                             std::integer_sequence<int, P...>) {
    (path_coupling<P>(cg, y, aw, lane), ...);
}

__device__ __forceinline__ void warp_couplings(int warp, const float* cg, const float* y, float* aw, int lane) {
    switch (warp) {
        case 0: couplings_of(cg, y, aw, lane, Warp0Paths{}); break;
        case 1: couplings_of(cg, y, aw, lane, Warp1Paths{}); break;
        case 2: couplings_of(cg, y, aw, lane, Warp2Paths{}); break;
        default: couplings_of(cg, y, aw, lane, Warp3Paths{}); break;
    }
}

// the edge's weight row (240 float4) and its sender's feature row (120 float4, from the three planes)
// over the block's 128 threads: loaded into registers (issued one edge ahead, so that the loads fly
// while the previous edge computes), then stored to shared memory
__device__ __forceinline__ void load_rows_block(const ConvArgs& a, int64_t e, int64_t j, float4* v, int tid) {
    constexpr int NW = kWW / 4, NX = kXW / 4;
    const float4* wsrc = reinterpret_cast<const float4*>(a.W + e * kWW);
#pragma unroll
    for (int r = 0; r < 3; ++r) {
        const int q = tid + kRecvThreads * r;
        if (q < NW)
            v[r] = wsrc[q];
        else if (q < NW + NX)
            v[r] = *reinterpret_cast<const float4*>(a.x + x_planar(a.n_atoms, j, 4 * (q - NW)));
    }
}

__device__ __forceinline__ void store_rows_block(const float4* v, float* ws, float* xs, int tid) {
    constexpr int NW = kWW / 4, NX = kXW / 4;
#pragma unroll
    for (int r = 0; r < 3; ++r) {
        const int q = tid + kRecvThreads * r;
        if (q < NW)
            reinterpret_cast<float4*>(ws)[q] = v[r];
        else if (q < NW + NX)
            reinterpret_cast<float4*>(xs)[q - NW] = v[r];
    }
}

__device__ __forceinline__ void load_y(const ConvArgs& a, int64_t e, float* y) {
#pragma unroll
    for (int q = 0; q < 9; ++q) y[q] = a.Y[9 * e + q];
}

// block shared memory: [cg 616 | acc 3136 | A 179 + 1 | W row 960 | x row 480]
constexpr int kFwdBlock = 616 + kMW + kAW + 1 + kWW + kXW;
static_assert((616 + kMW + kAW + 1) % 4 == 0 && (616 + kMW + kAW + 1 + kWW) % 4 == 0, "16-byte staged rows");

__global__ void __launch_bounds__(kRecvThreads) nq_conv_kernel(ConvArgs a, float* __restrict__ m) {
    extern __shared__ __align__(16) float nq_smem[];
    float* cg = nq_smem;
    float* acc = cg + 616;
    float* aw = acc + kMW;
    float* ws = aw + kAW + 1;
    float* xs = ws + kWW;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int t = tid; t < kCGN; t += kRecvThreads) cg[t] = a.cg[t];
    for (int64_t i = blockIdx.x; i < a.n_atoms; i += gridDim.x) {
        __syncthreads();  // the previous receiver's messages are written out
        for (int t = tid; t < kMW; t += kRecvThreads) acc[t] = 0.f;
        const int64_t e0 = a.recv_off[i], e1 = a.recv_off[i + 1];
        float4 v[3];
        if (e0 < e1) load_rows_block(a, e0, a.edge_index[2 * e0 + 1], v, tid);
        for (int64_t e = e0; e < e1; ++e) {
            float y[9];
            load_y(a, e, y);
            __syncthreads();  // the previous edge's rows are consumed
            store_rows_block(v, ws, xs, tid);
            if (e + 1 < e1) load_rows_block(a, e + 1, a.edge_index[2 * (e + 1) + 1], v, tid);
            warp_couplings(warp, cg, y, aw, lane);
            __syncthreads();
            switch (warp) {
                case 0: all_paths_fwd(ws, xs, aw, acc, lane, Warp0Paths{}); break;
                case 1: all_paths_fwd(ws, xs, aw, acc, lane, Warp1Paths{}); break;
                case 2: all_paths_fwd(ws, xs, aw, acc, lane, Warp2Paths{}); break;
                default: all_paths_fwd(ws, xs, aw, acc, lane, Warp3Paths{}); break;
            }
        }
        __syncthreads();
        for (int t = tid; t < kMW; t += kRecvThreads) m[m_planar(a.n_atoms, i, t)] = acc[t] * a.inv_avg;
    }
}
// dW[e, path, u] = sum_m3 g[u, m3] sum_m1 A[m3][m1] x[u, m1]; the lane's share of dY[e]: the path's
// T[m3][m1] = sum_u W g[u, m3] x[u, m1] over the lane's channels, times CG (lanes added by the caller)
template <int P>
__device__ __forceinline__ void path_bwd_edge(const float* ws, const float* xs, const float* cg, const float* aw,
                                              const float* dm, int64_t e, float* dW, float* dy, int lane) {
    constexpr PathInfo pi = kPaths[P];
    constexpr int n1 = dim_of(pi.l1), n2 = dim_of(pi.l2), n3 = dim_of(pi.l3), U = mult_of(pi.l1);
    float t[n3 * n1];
#pragma unroll
    for (int q = 0; q < n3 * n1; ++q) t[q] = 0.f;
#pragma unroll 1
    for (int u = lane; u < U; u += 32) {
        const float w = ws[pi.w_off + u];
        float xv[n1];
#pragma unroll
        for (int m1 = 0; m1 < n1; ++m1) xv[m1] = xs[x_idx(pi.l1, u, m1)];
        float gw = 0.f;
#pragma unroll
        for (int m3 = 0; m3 < n3; ++m3) {
            const float g = dm[m_idx(pi, u, m3)];
            float s = 0.f;
#pragma unroll
            for (int m1 = 0; m1 < n1; ++m1) {
                s = fmaf(aw[a_off(P) + m3 * n1 + m1], xv[m1], s);
                t[m3 * n1 + m1] = fmaf(w * g, xv[m1], t[m3 * n1 + m1]);
            }
            gw = fmaf(g, s, gw);
        }
        dW[e * kWW + pi.w_off + u] = gw;
    }
    // the lane's share of dY[e, l2]: its partial T folded with the coupling constants (the lanes' sums
    // are added by the caller's xor tree)
#pragma unroll
    for (int m2 = 0; m2 < n2; ++m2) {
        float acc = 0.f;
#pragma unroll
        for (int q = 0; q < n3 * n1; ++q) acc = fmaf(cg[pi.cg_off + q * n2 + m2], t[q], acc);
        dy[y_off(pi.l2) + m2] += acc;
    }
}

template <int... P>
__device__ __forceinline__ void all_paths_bwd_edge(const float* ws, const float* xs, const float* cg, const float* aw,
                                                   const float* dm, int64_t e, float* dW, float* dy,
                                                   int lane, std::integer_sequence<int, P...>) {
    (path_bwd_edge<P>(ws, xs, cg, aw, dm, e, dW, dy, lane), ...);
}

// per receiver: dW and dY of its edges; each warp its own paths (dW columns disjoint), dY from the
// warps' lane-folded partials summed in warp order
constexpr int kBwdBlock = 616 + kMW + kAW + 1 + kWW + kXW + 36;

__global__ void __launch_bounds__(kRecvThreads) nq_conv_bwd_edge_kernel(ConvArgs a, const float* __restrict__ dmsg,
                                                                        float* __restrict__ dW,
                                                                        float* __restrict__ dY, int accumulate_dy) {
    extern __shared__ __align__(16) float nq_smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float* cg = nq_smem;
    float* dm = cg + 616;
    float* aw = dm + kMW;
    float* ws = aw + kAW + 1;
    float* xs = ws + kWW;
    float* dyw = xs + kXW;  // [4][9]
    for (int t = tid; t < kCGN; t += kRecvThreads) cg[t] = a.cg[t];
    for (int64_t i = blockIdx.x; i < a.n_atoms; i += gridDim.x) {
        __syncthreads();  // the previous receiver is done
        for (int t = tid; t < kMW; t += kRecvThreads) dm[t] = dmsg[m_planar(a.n_atoms, i, t)] * a.inv_avg;
        for (int64_t e = a.recv_off[i]; e < a.recv_off[i + 1]; ++e) {
            float y[9];
            load_y(a, e, y);
            float4 v[3];  // no prefetch here: its registers cost a resident block per SM
            load_rows_block(a, e, a.edge_index[2 * e + 1], v, tid);
            __syncthreads();  // the previous edge's rows and dY partials are consumed
            store_rows_block(v, ws, xs, tid);
            warp_couplings(warp, cg, y, aw, lane);
            __syncthreads();
            float dy[9];
#pragma unroll
            for (int q = 0; q < 9; ++q) dy[q] = 0.f;
            switch (warp) {
                case 0: all_paths_bwd_edge(ws, xs, cg, aw, dm, e, dW, dy, lane, Warp0Paths{}); break;
                case 1: all_paths_bwd_edge(ws, xs, cg, aw, dm, e, dW, dy, lane, Warp1Paths{}); break;
                case 2: all_paths_bwd_edge(ws, xs, cg, aw, dm, e, dW, dy, lane, Warp2Paths{}); break;
                default: all_paths_bwd_edge(ws, xs, cg, aw, dm, e, dW, dy, lane, Warp3Paths{}); break;
            }
#pragma unroll
            for (int q = 0; q < 9; ++q)
                for (int d = 16; d > 0; d >>= 1) dy[q] += __shfl_xor_sync(0xffffffffu, dy[q], d);
            if (lane == 0)
#pragma unroll
                for (int q = 0; q < 9; ++q) dyw[warp * 9 + q] = dy[q];
            __syncthreads();
            if (tid < 9) {
                const float v = ((dyw[tid] + dyw[9 + tid]) + dyw[18 + tid]) + dyw[27 + tid];
                dY[9 * e + tid] = accumulate_dy ? dY[9 * e + tid] + v : v;
            }
        }
    }
}

// dx[j, l1, m1, u] += W[e, path, u] sum_m3 A[m3][m1] dm[i, l3, m3, path channel u] for the channels
// u in [U0, U0 + 32) and the components m1 in [M0, M1)
template <int P, int U0, int M0, int M1>
__device__ __forceinline__ void path_bwd_x(const ConvArgs& a, const float* aw, const float* const* dmi, int64_t e,
                                           float* dx, int lane) {
    constexpr PathInfo pi = kPaths[P];
    constexpr int n1 = dim_of(pi.l1), n3 = dim_of(pi.l3);
    static_assert(U0 + 32 <= mult_of(pi.l1) && 0 <= M0 && M0 < M1 && M1 <= n1, "work item");
    const int u = U0 + lane;
    const float w = a.W[e * kWW + pi.w_off + u];
    float g[n3];
#pragma unroll
    for (int m3 = 0; m3 < n3; ++m3) g[m3] = dmi[pi.l3][m3 * m_mult(pi.l3) + c_off(pi) + u];
#pragma unroll
    for (int m1 = M0; m1 < M1; ++m1) {
        float s = 0.f;
#pragma unroll
        for (int m3 = 0; m3 < n3; ++m3) s = fmaf(aw[a_off(P) + m3 * n1 + m1], g[m3], s);
        dx[x_idx(pi.l1, u, m1)] = fmaf(w, s, dx[x_idx(pi.l1, u, m1)]);
    }
}

template <int U0, int M0, int M1, int... P>
__device__ __forceinline__ void items_bwd_x(const ConvArgs& a, const float* aw, const float* const* dmi, int64_t e,
                                            float* dx, int lane) {
    (path_bwd_x<P, U0, M0, M1>(a, aw, dmi, e, dx, lane), ...);
}

// per sender j: dx[j] over its sender run, a block of 4 warps; each warp owns the dx entries of fixed
// (l1, 32-channel chunk, m1 range) items, so that every dx entry is summed by one lane in path and
// edge order (FMA per edge: 2112, 2208, 2208, 1984 of 8512). Every warp forms the edge's full coupling
// matrices in its own copy (no block barrier per edge); the receivers' message gradients are read from
// global memory, coalesced over the lanes' channels.
constexpr int kBxBlock = 616 + kXW + 4 * (kAW + 1);

__global__ void __launch_bounds__(kRecvThreads) nq_conv_bwd_x_kernel(ConvArgs a, const float* __restrict__ dmsg,
                                                                     float* __restrict__ dx_out) {
    extern __shared__ __align__(16) float nq_smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float* cg = nq_smem;
    float* dx = cg + 616;
    float* aw = dx + kXW + warp * (kAW + 1);
    for (int t = tid; t < kCGN; t += kRecvThreads) cg[t] = a.cg[t];
    for (int64_t j = blockIdx.x; j < a.n_atoms; j += gridDim.x) {
        __syncthreads();  // the previous sender is written out (and cg is loaded)
        for (int t = tid; t < kXW; t += kRecvThreads) dx[t] = 0.f;
        __syncthreads();
        for (int64_t s = a.send_off[j]; s < a.send_off[j + 1]; ++s) {
            const int64_t e = a.send_perm[s];
            const int64_t i = a.edge_index[2 * e];
            load_couplings(a, cg, e, aw, lane);
            // the receiver's message-gradient rows of the three planes
            const float* dmi[3] = {dmsg + m_planar(a.n_atoms, i, 0), dmsg + m_planar(a.n_atoms, i, m_off_of(1)),
                                   dmsg + m_planar(a.n_atoms, i, m_off_of(2))};
            switch (warp) {
                case 0:
                    items_bwd_x<0, 0, 3, 9, 10, 11, 12, 13, 14>(a, aw, dmi, e, dx, lane);
                    break;
                case 1:
                    items_bwd_x<0, 0, 3, 3, 4, 5, 6, 7, 8>(a, aw, dmi, e, dx, lane);
                    items_bwd_x<0, 0, 1, 0, 1, 2>(a, aw, dmi, e, dx, lane);
                    break;
                case 2:
                    items_bwd_x<32, 0, 3, 3, 4, 5, 6, 7, 8>(a, aw, dmi, e, dx, lane);
                    items_bwd_x<32, 0, 1, 0, 1, 2>(a, aw, dmi, e, dx, lane);
                    break;
                default:
                    items_bwd_x<0, 3, 5, 9, 10, 11, 12, 13, 14>(a, aw, dmi, e, dx, lane);
                    items_bwd_x<64, 0, 1, 0, 1, 2>(a, aw, dmi, e, dx, lane);
                    items_bwd_x<96, 0, 1, 0, 1, 2>(a, aw, dmi, e, dx, lane);
                    break;
            }
        }
        __syncthreads();
        for (int t = tid; t < kXW; t += kRecvThreads) dx_out[x_planar(a.n_atoms, j, t)] = dx[t] * a.inv_avg;
    }
}

// ------------------------------------------------------------------ gate
//
// The gated nonlinearity closing an interaction block, plus its self-connection:
//   x0[n, c] = silu(o0[n, c]) + sc0[n, c]                          (c < 128)
//   x1[n, m, c] = o1[n, m, c] sigmoid(o0[n, 128 + c]) + sc1[n, m, c]  (c < 64)
//   x2[n, m, c] = o2[n, m, c] sigmoid(o0[n, 192 + c]) + sc2[n, m, c]  (c < 32)
// (o0 [N, 224], o1 [N, 3, 64], o2 [N, 5, 32]). One thread per output element over the three planes;
// the backward, one thread per element of d o0 / d o1 / d o2, sums a gate's 3 or 5 products in order.

__device__ __forceinline__ float sigmoid_f(float v) { return 1.f / (1.f + expf(-v)); }

__global__ void __launch_bounds__(256) nq_gate_kernel(const float* __restrict__ o0, const float* __restrict__ o1,
                                                       const float* __restrict__ o2, const float* __restrict__ sc0,
                                                       const float* __restrict__ sc1, const float* __restrict__ sc2,
                                                       int64_t n, float* __restrict__ x0, float* __restrict__ x1,
                                                       float* __restrict__ x2) {
    const int64_t total = n * kXW;
    for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < total; t += int64_t(gridDim.x) * blockDim.x) {
        if (t < n * 128) {
            const float v = o0[(t >> 7) * 224 + (t & 127)];
            x0[t] = v * sigmoid_f(v) + sc0[t];
        } else if (t < n * 320) {
            const int64_t q = t - n * 128, a = q / 192;
            x1[q] = o1[q] * sigmoid_f(o0[a * 224 + 128 + (q & 63)]) + sc1[q];
        } else {
            const int64_t q = t - n * 320, a = q / 160;
            x2[q] = o2[q] * sigmoid_f(o0[a * 224 + 192 + (q & 31)]) + sc2[q];
        }
    }
}

__global__ void __launch_bounds__(256) nq_gate_bwd_kernel(const float* __restrict__ o0, const float* __restrict__ o1,
                                                           const float* __restrict__ o2, const float* __restrict__ dx0,
                                                           const float* __restrict__ dx1,
                                                           const float* __restrict__ dx2, int64_t n,
                                                           float* __restrict__ do0, float* __restrict__ do1,
                                                           float* __restrict__ do2) {
    const int64_t total = n * (224 + 192 + 160);
    for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < total; t += int64_t(gridDim.x) * blockDim.x) {
        if (t < n * 224) {
            const int64_t a = t / 224;
            const int k = int(t - a * 224);
            const float v = o0[t], sg = sigmoid_f(v);
            if (k < 128) {
                do0[t] = dx0[a * 128 + k] * (sg * (1.f + v * (1.f - sg)));
            } else if (k < 192) {
                float acc = 0.f;
#pragma unroll
                for (int m = 0; m < 3; ++m) acc += dx1[a * 192 + m * 64 + (k - 128)] * o1[a * 192 + m * 64 + (k - 128)];
                do0[t] = acc * (sg * (1.f - sg));
            } else {
                float acc = 0.f;
#pragma unroll
                for (int m = 0; m < 5; ++m) acc += dx2[a * 160 + m * 32 + (k - 192)] * o2[a * 160 + m * 32 + (k - 192)];
                do0[t] = acc * (sg * (1.f - sg));
            }
        } else if (t < n * 416) {
            const int64_t q = t - n * 224, a = q / 192;
            do1[q] = dx1[q] * sigmoid_f(o0[a * 224 + 128 + (q & 63)]);
        } else {
            const int64_t q = t - n * 416, a = q / 160;
            do2[q] = dx2[q] * sigmoid_f(o0[a * 224 + 192 + (q & 31)]);
        }
    }
}

// ------------------------------------------------------------------ self-connection
//
// The element-dependent linear of every plane: out[n, m, c] = sum_u x[n, m, u] w_l[z(n), u, c]
// (forward) or sum_u x[n, m, u] w_l[z(n), c, u] (transposed: the input gradient), w_l [elements, U, U].
// One thread per (atom, plane, output channel c) computes the plane's 2l + 1 rows of the atom, so each
// weight load serves every row; the atom's rows are read as float4 (broadcast across the warp, L1),
// the weights across the warp's consecutive c; each output summed in u order.

template <int U, int D, bool T>
__device__ __forceinline__ void sc_plane(const float* __restrict__ x, const float* __restrict__ w, int64_t a, int c,
                                         float* __restrict__ o) {
    const float* xr = x + a * (D * U);
    float acc[D];
#pragma unroll
    for (int m = 0; m < D; ++m) acc[m] = 0.f;
#pragma unroll 4
    for (int u = 0; u < U; u += 4) {
        float wv[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) wv[k] = T ? w[c * U + u + k] : w[(u + k) * U + c];
#pragma unroll
        for (int m = 0; m < D; ++m) {
            const float4 xv = *reinterpret_cast<const float4*>(xr + m * U + u);
            acc[m] = fmaf(xv.x, wv[0], acc[m]);
            acc[m] = fmaf(xv.y, wv[1], acc[m]);
            acc[m] = fmaf(xv.z, wv[2], acc[m]);
            acc[m] = fmaf(xv.w, wv[3], acc[m]);
        }
    }
#pragma unroll
    for (int m = 0; m < D; ++m) o[a * (D * U) + m * U + c] = acc[m];
}

template <bool T>
__global__ void __launch_bounds__(256) nq_self_conn_kernel(const float* __restrict__ x0, const float* __restrict__ x1,
                                                            const float* __restrict__ x2,
                                                            const int64_t* __restrict__ elem,
                                                            const float* __restrict__ w0, const float* __restrict__ w1,
                                                            const float* __restrict__ w2, int64_t n,
                                                            float* __restrict__ o0, float* __restrict__ o1,
                                                            float* __restrict__ o2) {
    const int64_t total = n * (128 + 64 + 32);
    for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < total; t += int64_t(gridDim.x) * blockDim.x) {
        if (t < n * 128) {
            const int64_t a = t >> 7;
            sc_plane<128, 1, T>(x0, w0 + elem[a] * (128 * 128), a, int(t & 127), o0);
        } else if (t < n * 192) {
            const int64_t q = t - n * 128, a = q >> 6;
            sc_plane<64, 3, T>(x1, w1 + elem[a] * (64 * 64), a, int(q & 63), o1);
        } else {
            const int64_t q = t - n * 192, a = q >> 5;
            sc_plane<32, 5, T>(x2, w2 + elem[a] * (32 * 32), a, int(q & 31), o2);
        }
    }
}

// forces[a] = sum of grad_vec over the edges a receives - sum over the edges a sends: a warp per atom,
// lane l takes the run's entries l, l + 32, ..., then a fixed xor tree over the lanes
constexpr int kForceWarpsNq = 8;
__global__ void __launch_bounds__(32 * kForceWarpsNq) nq_edge_forces_kernel(
    const float* __restrict__ g, const int32_t* __restrict__ edge_index, const int64_t* __restrict__ recv_off,
    const int64_t* __restrict__ send_off, const int32_t* __restrict__ send_perm, int64_t n_atoms,
    float* __restrict__ forces) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = int64_t(gridDim.x) * kForceWarpsNq;
    for (int64_t a = blockIdx.x * int64_t(kForceWarpsNq) + (threadIdx.x >> 5); a < n_atoms; a += warps) {
        float r[3] = {0.f, 0.f, 0.f}, t[3] = {0.f, 0.f, 0.f};
        for (int64_t e = recv_off[a] + lane; e < recv_off[a + 1]; e += 32)
#pragma unroll
            for (int c = 0; c < 3; ++c) r[c] += g[3 * e + c];
        for (int64_t k = send_off[a] + lane; k < send_off[a + 1]; k += 32) {
            const int64_t e = send_perm[k];
#pragma unroll
            for (int c = 0; c < 3; ++c) t[c] += g[3 * e + c];
        }
#pragma unroll
        for (int c = 0; c < 3; ++c)
            for (int d = 16; d > 0; d >>= 1) {
                r[c] += __shfl_xor_sync(0xffffffffu, r[c], d);
                t[c] += __shfl_xor_sync(0xffffffffu, t[c], d);
            }
        if (lane < 3) forces[3 * a + lane] = r[lane] - t[lane];
    }
}

bool make_cell3(const float* host, Cell3& c) {
    if (host == nullptr) return false;
    for (int k = 0; k < 9; ++k) c.c[k] = host[k];
    return true;
}

inline int grid_of(int64_t work, int per) {
    const int64_t g = (work + per - 1) / per;
    return int(g < 148 * 32 ? (g > 0 ? g : 1) : 148 * 32);
}


}  // namespace
}  // namespace fmd

using namespace fmd;

extern "C" {

fmd_status fmd_nequip_edge_basis(const float* positions, const float* cell_host, const int32_t* edge_index,
                                 const float* edge_image, const float* override_vec, const int64_t* n_real,
                                 int64_t n_edges, float r_max, int32_t n_basis, int32_t poly_p, float* Y, float* B,
                                 float* geo, void* stream) {
    BasisArgs a{};
    if (n_edges < 0 || !(r_max > 0.f) || n_basis < 1 || n_basis > 32 || poly_p < 2 || !make_cell3(cell_host, a.cell))
        return FMD_ERR_INVALID_ARGUMENT;
    if (n_edges == 0) return FMD_OK;
    if (positions == nullptr || edge_index == nullptr || edge_image == nullptr || Y == nullptr || B == nullptr ||
        geo == nullptr)
        return FMD_ERR_INVALID_ARGUMENT;
    a.pos = positions;
    a.edge_index = edge_index;
    a.edge_image = edge_image;
    a.override_vec = override_vec;
    a.n_real = n_real;
    a.n_edges = n_edges;
    a.r_max = r_max;
    a.n_basis = n_basis;
    a.poly_p = poly_p;
    a.Y = Y;
    a.B = B;
    a.geo = geo;
    nq_basis_kernel<<<grid_of(n_edges, 256), 256, 0, as_stream(stream)>>>(a);
    return check_launch();
}

fmd_status fmd_nequip_edge_basis_bwd(const float* geo, const float* dY, const float* dB, const float* override_vec,
                                     const int64_t* n_real, int64_t n_edges, float r_max, int32_t n_basis,
                                     int32_t poly_p, float* grad_vec, void* stream) {
    BasisArgs a{};
    if (n_edges < 0 || !(r_max > 0.f) || n_basis < 1 || n_basis > 32 || poly_p < 2) return FMD_ERR_INVALID_ARGUMENT;
    if (n_edges == 0) return FMD_OK;
    if (geo == nullptr || dY == nullptr || dB == nullptr || grad_vec == nullptr) return FMD_ERR_INVALID_ARGUMENT;
    a.geo = const_cast<float*>(geo);
    a.override_vec = override_vec;
    a.n_real = n_real;
    a.n_edges = n_edges;
    a.r_max = r_max;
    a.n_basis = n_basis;
    a.poly_p = poly_p;
    nq_basis_bwd_kernel<<<grid_of(n_edges, 256), 256, 0, as_stream(stream)>>>(a, dY, dB, grad_vec);
    return check_launch();
}

static fmd_status conv_args(ConvArgs& a, const float* x, const float* Y, const float* W, const float* cg,
                            const int32_t* edge_index, const int64_t* recv_off, const int64_t* send_off,
                            const int32_t* send_perm, int64_t n_atoms, float inv_avg) {
    if (n_atoms < 0 || !(inv_avg > 0.f)) return FMD_ERR_INVALID_ARGUMENT;
    if (x == nullptr || cg == nullptr || recv_off == nullptr) return FMD_ERR_INVALID_ARGUMENT;
    // rows are staged with 16-byte loads
    if (reinterpret_cast<uintptr_t>(x) % 16 != 0 || reinterpret_cast<uintptr_t>(W) % 16 != 0)
        return FMD_ERR_INVALID_ARGUMENT;
    a = ConvArgs{x, Y, W, cg, edge_index, recv_off, send_off, send_perm, n_atoms, inv_avg};
    return FMD_OK;
}

fmd_status fmd_nequip_conv(const float* x, const float* Y, const float* W, const float* cg,
                           const int32_t* edge_index, const int64_t* recv_off, int64_t n_atoms, float inv_avg,
                           float* messages, void* stream) {
    ConvArgs a;
    fmd_status st = conv_args(a, x, Y, W, cg, edge_index, recv_off, nullptr, nullptr, n_atoms, inv_avg);
    if (st != FMD_OK) return st;
    if (n_atoms == 0) return FMD_OK;
    if (messages == nullptr) return FMD_ERR_INVALID_ARGUMENT;
    const size_t smem = sizeof(float) * kFwdBlock;
    if ((st = grant_dynamic_smem((const void*)nq_conv_kernel, smem)) != FMD_OK) return st;
    nq_conv_kernel<<<grid_of(n_atoms, 1), kRecvThreads, smem, as_stream(stream)>>>(a, messages);
    return check_launch();
}

fmd_status fmd_nequip_conv_bwd(const float* x, const float* Y, const float* W, const float* cg,
                               const int32_t* edge_index, const int64_t* recv_off, const int64_t* send_off,
                               const int32_t* send_perm, int64_t n_atoms, float inv_avg, const float* grad_messages,
                               float* grad_x, float* grad_W, float* grad_Y, int32_t accumulate_grad_y, void* stream) {
    ConvArgs a;
    fmd_status st = conv_args(a, x, Y, W, cg, edge_index, recv_off, send_off, send_perm, n_atoms, inv_avg);
    if (st != FMD_OK) return st;
    if (n_atoms == 0) return FMD_OK;
    if (grad_messages == nullptr || grad_W == nullptr || grad_Y == nullptr || (grad_x != nullptr && send_off == nullptr))
        return FMD_ERR_INVALID_ARGUMENT;
    const size_t smem_e = sizeof(float) * kBwdBlock, smem_x = sizeof(float) * kBxBlock;
    if ((st = grant_dynamic_smem((const void*)nq_conv_bwd_edge_kernel, smem_e)) != FMD_OK) return st;
    if ((st = grant_dynamic_smem((const void*)nq_conv_bwd_x_kernel, smem_x)) != FMD_OK) return st;
    const cudaStream_t s = as_stream(stream);
    nq_conv_bwd_edge_kernel<<<grid_of(n_atoms, 1), kRecvThreads, smem_e, s>>>(a, grad_messages, grad_W,
                                                                                       grad_Y, accumulate_grad_y != 0);
    if ((st = check_launch()) != FMD_OK) return st;
    if (grad_x == nullptr) return FMD_OK;  // the input needs no gradient (the first block's embedding)
    nq_conv_bwd_x_kernel<<<grid_of(n_atoms, 1), kRecvThreads, smem_x, s>>>(a, grad_messages, grad_x);
    return check_launch();
}

fmd_status fmd_edge_forces(const float* grad_vec, const int32_t* edge_index, const int64_t* recv_off,
                           const int64_t* send_off, const int32_t* send_perm, int64_t n_atoms, float* forces,
                           void* stream) {
    if (n_atoms < 0) return FMD_ERR_INVALID_ARGUMENT;
    if (n_atoms == 0) return FMD_OK;
    if (grad_vec == nullptr || recv_off == nullptr || send_off == nullptr || send_perm == nullptr ||
        forces == nullptr)
        return FMD_ERR_INVALID_ARGUMENT;
    (void)edge_index;  // the runs name the edges; kept for the callers' symmetry with the gradient's layout
    const int64_t blocks = (n_atoms + kForceWarpsNq - 1) / kForceWarpsNq;
    nq_edge_forces_kernel<<<int(blocks < 148 * 16 ? blocks : 148 * 16), 32 * kForceWarpsNq, 0, as_stream(stream)>>>(
        grad_vec, edge_index, recv_off, send_off, send_perm, n_atoms, forces);
    return check_launch();
}

fmd_status fmd_nequip_gate(const float* o0, const float* o1, const float* o2, const float* sc0, const float* sc1,
                           const float* sc2, int64_t n_atoms, float* x0, float* x1, float* x2, void* stream) {
    if (n_atoms < 0) return FMD_ERR_INVALID_ARGUMENT;
    if (n_atoms == 0) return FMD_OK;
    if (o0 == nullptr || o1 == nullptr || o2 == nullptr || sc0 == nullptr || sc1 == nullptr || sc2 == nullptr ||
        x0 == nullptr || x1 == nullptr || x2 == nullptr)
        return FMD_ERR_INVALID_ARGUMENT;
    nq_gate_kernel<<<grid_of(n_atoms * kXW, 256), 256, 0, as_stream(stream)>>>(o0, o1, o2, sc0, sc1, sc2, n_atoms, x0,
                                                                                 x1, x2);
    return check_launch();
}

fmd_status fmd_nequip_gate_bwd(const float* o0, const float* o1, const float* o2, const float* dx0, const float* dx1,
                               const float* dx2, int64_t n_atoms, float* do0, float* do1, float* do2, void* stream) {
    if (n_atoms < 0) return FMD_ERR_INVALID_ARGUMENT;
    if (n_atoms == 0) return FMD_OK;
    if (o0 == nullptr || o1 == nullptr || o2 == nullptr || dx0 == nullptr || dx1 == nullptr || dx2 == nullptr ||
        do0 == nullptr || do1 == nullptr || do2 == nullptr)
        return FMD_ERR_INVALID_ARGUMENT;
    nq_gate_bwd_kernel<<<grid_of(n_atoms * 576, 256), 256, 0, as_stream(stream)>>>(o0, o1, o2, dx0, dx1, dx2, n_atoms,
                                                                                     do0, do1, do2);
    return check_launch();
}

fmd_status fmd_nequip_self_connection(const float* x0, const float* x1, const float* x2, const int64_t* elem,
                                      const float* w0, const float* w1, const float* w2, int64_t n_atoms,
                                      int32_t transposed, float* out0, float* out1, float* out2, void* stream) {
    if (n_atoms < 0 || (transposed != 0 && transposed != 1)) return FMD_ERR_INVALID_ARGUMENT;
    if (n_atoms == 0) return FMD_OK;
    if (x0 == nullptr || x1 == nullptr || x2 == nullptr || elem == nullptr || w0 == nullptr || w1 == nullptr ||
        w2 == nullptr || out0 == nullptr || out1 == nullptr || out2 == nullptr)
        return FMD_ERR_INVALID_ARGUMENT;
    // the planes' rows are read as float4
    if (reinterpret_cast<uintptr_t>(x0) % 16 != 0 || reinterpret_cast<uintptr_t>(x1) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(x2) % 16 != 0)
        return FMD_ERR_INVALID_ARGUMENT;
    const int g = grid_of(n_atoms * 224, 256);
    if (transposed)
        nq_self_conn_kernel<true><<<g, 256, 0, as_stream(stream)>>>(x0, x1, x2, elem, w0, w1, w2, n_atoms, out0, out1,
                                                                    out2);
    else
        nq_self_conn_kernel<false><<<g, 256, 0, as_stream(stream)>>>(x0, x1, x2, elem, w0, w1, w2, n_atoms, out0,
                                                                     out1, out2);
    return check_launch();
}

}  // extern "C"
