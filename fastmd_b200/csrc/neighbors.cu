// Neighbour lists of periodic systems: the cell-list candidate build and the
// per-step exact re-filter of FastMD's fixed-capacity builder, and the
// ragged (eager) neighbour list.
//
// Layout: R systems ("replicas") of n atoms each share one cell; atom a of
// system r is global row r*n + a, and no pair crosses systems (the
// disjoint-union graph of replica_batch.py).
//
// Candidate build (cell list):
//   bin:     wrap every atom (the builder's float32 arithmetic), cell index
//            from the fractional coordinates, atomic slot in the cell;
//   scan:    cell starts (CUB exclusive scan over R*ncells counts);
//   scatter: atoms grouped by cell, their wrapped positions as float4;
//   query:   one CTA per home cell stages the atoms of the (2s+1)^3
//            neighbouring (cell, image) pairs in shared memory, each warp
//            tests one home atom against the staged atoms, compacts the hits
//            with a warp ballot into a per-warp list, ranks the list by the
//            canonical key (neighbour, image) and writes it out. The output
//            order is therefore independent of the atomics of the bin pass.
//
// Re-filter (every MD step, inside the whole-step CUDA graph): two kernels,
// a thread-block cluster of 8 CTAs per system, each CTA a slice of the
// centres. The count kernel wraps the positions (wrap delta
// since the candidate refresh, skin test), and counts per atom the
// candidates with dist2 < rc^2 evaluated in the reference's float32
// operation order (fixed_capacity_builder.py:159-163; this file is compiled
// without FMA contraction). The materialize kernel writes the edges with a
// ballot compaction at the global offsets (candidates are sorted once per
// refresh, so the edges come out in canonical order with no per-step sort),
// the receiver CSR, the sender CSR (each run ascending), the padding rows
// (far self-loops) and the status words.

#include <cub/device/device_scan.cuh>

#include <algorithm>
#include <cmath>
#include <mutex>

#include <cooperative_groups.h>

#include "common.cuh"

namespace fmd {

namespace cg = cooperative_groups;

// ------------------------------------------------------------------ geometry

struct Cell9 {
    float c[9];      // row-major lattice vectors
    float inv[9];    // row-major float32 inverse
};

// small_matmul row: out[c] = (a0*m[0][c] + a1*m[1][c]) + a2*m[2][c] (geometry.py:7)
__device__ __forceinline__ float3 row_times(float3 a, const float* m) {
    return make_float3((a.x * m[0] + a.y * m[3]) + a.z * m[6], (a.x * m[1] + a.y * m[4]) + a.z * m[7],
                       (a.x * m[2] + a.y * m[5]) + a.z * m[8]);
}

// build prologue (fixed_capacity_builder.py:2203-2208)
__device__ __forceinline__ void wrap_atom(float3 p, const Cell9& cell, float3& wrapped, int3& wraps,
                                          float3& frac) {
    const float3 fu = row_times(p, cell.inv);
    const float wx = floorf(fu.x), wy = floorf(fu.y), wz = floorf(fu.z);
    wraps = make_int3(int(wx), int(wy), int(wz));
    frac = make_float3(fu.x - wx, fu.y - wy, fu.z - wz);
    wrapped = row_times(frac, cell.c);
}

// dist2 of a candidate in the re-filter's operation order (fixed_capacity_builder.py:159-163)
__device__ __forceinline__ float refilter_dist2(float3 p, float3 q, float sx, float sy, float sz,
                                                const float* c) {
    const float dx = (((q.x - p.x) + sx * c[0]) + sy * c[3]) + sz * c[6];
    const float dy = (((q.y - p.y) + sx * c[1]) + sy * c[4]) + sz * c[7];
    const float dz = (((q.z - p.z) + sx * c[2]) + sy * c[5]) + sz * c[8];
    return (dx * dx + dy * dy) + dz * dz;
}

// distance of the ragged path's re-filter (gpu_graph_builder.py:186-192):
// diff = (q - p) + image @ cell (small_matmul), dist = |diff|
__device__ __forceinline__ float ragged_dist(float3 p, float3 q, int3 s, const float* c) {
    const float3 sh = row_times(make_float3(float(s.x), float(s.y), float(s.z)), c);
    const float dx = (q.x - p.x) + sh.x, dy = (q.y - p.y) + sh.y, dz = (q.z - p.z) + sh.z;
    return sqrtf((dx * dx + dy * dy) + dz * dz);
}

__device__ __forceinline__ float3 ld3(const float* p, int64_t i) {
    return make_float3(p[3 * i], p[3 * i + 1], p[3 * i + 2]);
}

__device__ __forceinline__ int3 ld3i(const int32_t* p, int64_t i) {
    return make_int3(p[3 * i], p[3 * i + 1], p[3 * i + 2]);
}

// canonical key of a candidate of one centre: neighbour, then the image
// (each component offset by 512, 10 bits): unique per (neighbour, image)
__device__ __forceinline__ uint64_t cand_key(int32_t nbr, int3 s) {
    return (uint64_t(uint32_t(nbr)) << 30) | (uint64_t(uint32_t(s.x + 512) & 1023u) << 20) |
           (uint64_t(uint32_t(s.y + 512) & 1023u) << 10) | uint64_t(uint32_t(s.z + 512) & 1023u);
}

__device__ __forceinline__ int floor_div(int a, int b) { return a >= 0 ? a / b : -((-a + b - 1) / b); }

struct Grid {
    int n[3];       // cells per axis
    int s[3];       // search reach in cells per axis
    int ncells;     // n0*n1*n2 (per system)
};

// --------------------------------------------------------------- cell list

__global__ void cell_bin_kernel(const float* __restrict__ positions, int64_t n_atoms, int32_t n_systems,
                                Cell9 cell, Grid grid, float4* __restrict__ wrapped_out,
                                int32_t* __restrict__ atom_cell, int32_t* __restrict__ atom_slot,
                                int32_t* __restrict__ cell_count, int32_t* flags) {
    const int64_t total = n_atoms * n_systems;
    for (int64_t a = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; a < total;
         a += int64_t(gridDim.x) * blockDim.x) {
        const int64_t sys = a / n_atoms;
        float3 w, f;
        int3 wr;
        wrap_atom(ld3(positions, a), cell, w, wr, f);
        const bool finite = isfinite(w.x) && isfinite(w.y) && isfinite(w.z);
        if (!finite) raise_flag(flags, FMD_FLAG_NONFINITE);
        int cx = finite ? int(floorf(f.x * grid.n[0])) : 0;
        int cy = finite ? int(floorf(f.y * grid.n[1])) : 0;
        int cz = finite ? int(floorf(f.z * grid.n[2])) : 0;
        cx = min(max(cx, 0), grid.n[0] - 1);
        cy = min(max(cy, 0), grid.n[1] - 1);
        cz = min(max(cz, 0), grid.n[2] - 1);
        const int c = int(sys * grid.ncells) + (cx * grid.n[1] + cy) * grid.n[2] + cz;
        atom_cell[a] = c;
        atom_slot[a] = atomicAdd(cell_count + c, 1);
        wrapped_out[a] = make_float4(w.x, w.y, w.z, 0.f);
    }
}

__global__ void cell_scatter_kernel(int64_t total, const float4* __restrict__ wrapped,
                                    const int32_t* __restrict__ atom_cell, const int32_t* __restrict__ atom_slot,
                                    const int32_t* __restrict__ cell_start, int32_t* __restrict__ cell_atoms,
                                    float4* __restrict__ cell_pos) {
    for (int64_t a = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; a < total;
         a += int64_t(gridDim.x) * blockDim.x) {
        const int k = cell_start[atom_cell[a]] + atom_slot[a];
        cell_atoms[k] = int32_t(a);
        float4 p = wrapped[a];
        cell_pos[k] = p;
    }
}

constexpr int kQueryWarps = 8;
constexpr int kStageCap = 1024;   // staged (atom, image) entries per chunk
constexpr int kMaxHome = 512;     // home atoms handled per pass over the neighbourhood

struct QueryArgs {
    const int32_t* cell_start;   // [R*ncells + 1]
    const int32_t* cell_atoms;   // grouped by cell
    const float4* cell_pos;      // wrapped positions grouped by cell
    int64_t n_atoms;             // per system
    int32_t n_systems;
    Cell9 cell;
    Grid grid;
    float cutoff;                // candidate cutoff (dist2 < cutoff^2, FP32)
    int32_t bmax;                // slots per atom in the output matrix
    int32_t list_cap;            // per-warp sort buffer (shared memory), >= bmax
    int32_t off_cap;             // (cell, image) offsets the shared memory holds: (2s0+1)(2s1+1)(2s2+1)
    int32_t* nbr_out;            // [R*n, bmax] global neighbour rows
    int32_t* shift_out;          // [R*n, bmax, 3]
    int32_t* count_out;          // [R*n] true candidate count
    int32_t* flags;
};

struct QuerySmem {
    float4* pos;       // [kStageCap] staged positions, shifted by their image
    int32_t* atom;     // [kStageCap]
    int32_t* img;      // [kStageCap] packed image
    int32_t* o_begin;  // [off_cap] first atom of the offset's cell
    int32_t* o_pref;   // [off_cap + 1] exclusive prefix of the offsets' atom counts
    int32_t* o_img;    // [off_cap]
    float* o_shift;    // [off_cap * 3]
    int32_t* hits;     // [kMaxHome]
    uint64_t* list;    // [kQueryWarps * list_cap]
};

// Shared memory of a query CTA for off_cap offsets (sized to the grid's search reach, not to the
// largest one: the 27 offsets of a reach of one cell leave room for twice the resident CTAs).
inline size_t query_smem(int list_cap, int off_cap) {
    return sizeof(float4) * kStageCap + 2 * sizeof(int32_t) * kStageCap + sizeof(int32_t) * off_cap * 3 +
           sizeof(int32_t) * (off_cap + 1) + sizeof(float) * off_cap * 3 + sizeof(int32_t) * kMaxHome +
           sizeof(uint64_t) * size_t(kQueryWarps) * list_cap + 64;
}

__device__ QuerySmem carve_query_smem(unsigned char* raw, int list_cap, int off_cap) {
    QuerySmem m;
    m.pos = reinterpret_cast<float4*>(raw);
    m.list = reinterpret_cast<uint64_t*>(m.pos + kStageCap);
    m.atom = reinterpret_cast<int32_t*>(m.list + size_t(kQueryWarps) * list_cap);
    m.img = m.atom + kStageCap;
    m.o_begin = m.img + kStageCap;
    m.o_pref = m.o_begin + off_cap;
    m.o_img = m.o_pref + off_cap + 1;
    m.hits = m.o_img + off_cap;
    m.o_shift = reinterpret_cast<float*>(m.hits + kMaxHome);
    return m;
}

__global__ void __launch_bounds__(kQueryWarps * 32) cell_query_kernel(QueryArgs q) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const QuerySmem m = carve_query_smem(smem_raw, q.list_cap, q.off_cap);
    __shared__ int s_scan[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ncells = q.grid.ncells;
    const int64_t total_cells = int64_t(ncells) * q.n_systems;
    const float cut2 = q.cutoff * q.cutoff;
    const int r0 = q.grid.s[0], r1 = q.grid.s[1], r2 = q.grid.s[2];
    const int w1 = 2 * r1 + 1, w2 = 2 * r2 + 1;
    const int n_off = (2 * r0 + 1) * w1 * w2;
    const int zero_img = (512 << 20) | (512 << 10) | 512;
    for (int64_t home = blockIdx.x; home < total_cells; home += gridDim.x) {
        const int64_t sys = home / ncells;
        const int32_t sys_base = int32_t(sys * q.n_atoms);
        const int local = int(home - sys * ncells);
        const int hx = local / (q.grid.n[1] * q.grid.n[2]);
        const int hy = (local / q.grid.n[2]) % q.grid.n[1];
        const int hz = local % q.grid.n[2];
        const int h_begin = q.cell_start[home], h_end = q.cell_start[home + 1];
        if (h_begin == h_end) continue;  // uniform per CTA
        // the neighbourhood: (cell, image) per offset, atom counts, prefix
        __syncthreads();
        int running = 0;
        for (int o0 = 0; o0 < n_off; o0 += blockDim.x) {
            const int o = o0 + threadIdx.x;
            int cnt = 0;
            if (o < n_off) {
                const int ox = o / (w1 * w2) - r0, oy = (o / w2) % w1 - r1, oz = o % w2 - r2;
                const int gx = hx + ox, gy = hy + oy, gz = hz + oz;
                const int ix = floor_div(gx, q.grid.n[0]), iy = floor_div(gy, q.grid.n[1]), iz = floor_div(gz, q.grid.n[2]);
                const int cx = gx - ix * q.grid.n[0], cy = gy - iy * q.grid.n[1], cz = gz - iz * q.grid.n[2];
                const int64_t c = sys * ncells + (cx * q.grid.n[1] + cy) * q.grid.n[2] + cz;
                const int b = q.cell_start[c];
                cnt = q.cell_start[c + 1] - b;
                m.o_begin[o] = b;
                m.o_img[o] = ((ix + 512) << 20) | ((iy + 512) << 10) | (iz + 512);
                const float fx = float(ix), fy = float(iy), fz = float(iz);
                m.o_shift[3 * o] = (fx * q.cell.c[0] + fy * q.cell.c[3]) + fz * q.cell.c[6];
                m.o_shift[3 * o + 1] = (fx * q.cell.c[1] + fy * q.cell.c[4]) + fz * q.cell.c[7];
                m.o_shift[3 * o + 2] = (fx * q.cell.c[2] + fy * q.cell.c[5]) + fz * q.cell.c[8];
            }
            // block exclusive scan of cnt
            const int lane_s = threadIdx.x & 31, warp_s = threadIdx.x >> 5;
            int x = cnt;
            for (int d = 1; d < 32; d <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, d);
                if (lane_s >= d) x += y;
            }
            __syncthreads();
            if (lane_s == 31) s_scan[warp_s] = x;
            __syncthreads();
            int before = 0, chunk_total = 0;
            for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
                if (w < warp_s) before += s_scan[w];
                chunk_total += s_scan[w];
            }
            if (o < n_off) m.o_pref[o] = running + before + x - cnt;
            running += chunk_total;
            __syncthreads();
        }
        if (threadIdx.x == 0) m.o_pref[n_off] = running;
        const int staged_total = running;
        // One staging pass holds the whole neighbourhood (the common case): each warp collects a home
        // atom's hit keys in its shared-memory list, ranks them there and writes each slot once.
        if (staged_total <= kStageCap && q.bmax <= q.list_cap) {
            const int ns = staged_total;
            __syncthreads();
            for (int t = threadIdx.x; t < ns; t += blockDim.x) {
                int lo = 0, hi = n_off;  // last offset with o_pref[o] <= t
                while (hi - lo > 1) {
                    const int mid = (lo + hi) >> 1;
                    if (m.o_pref[mid] <= t) lo = mid; else hi = mid;
                }
                const int src = m.o_begin[lo] + (t - m.o_pref[lo]);
                const float4 p = q.cell_pos[src];
                m.pos[t] = make_float4(p.x + m.o_shift[3 * lo], p.y + m.o_shift[3 * lo + 1],
                                       p.z + m.o_shift[3 * lo + 2], 0.f);
                m.atom[t] = q.cell_atoms[src];
                m.img[t] = m.o_img[lo];
            }
            __syncthreads();
            uint64_t* list = m.list + size_t(warp) * q.list_cap;
            for (int h = warp; h < h_end - h_begin; h += kQueryWarps) {
                const float4 hp = q.cell_pos[h_begin + h];
                const int32_t ha = q.cell_atoms[h_begin + h];
                const int64_t row = ha;
                int hits = 0;
                for (int base = 0; base < ns; base += 32) {
                    const int k = base + lane;
                    bool hit = false;
                    int32_t atom = 0;
                    int packed = 0;
                    if (k < ns) {
                        const float4 p = m.pos[k];
                        const float dx = p.x - hp.x, dy = p.y - hp.y, dz = p.z - hp.z;
                        const float d2 = (dx * dx + dy * dy) + dz * dz;
                        atom = m.atom[k];
                        packed = m.img[k];
                        hit = d2 < cut2 && !(atom == ha && packed == zero_img);
                    }
                    const unsigned mask = __ballot_sync(0xffffffffu, hit);
                    if (hit) {  // the first bmax hits in discovery order, as the two-pass path keeps them
                        const int pos = hits + __popc(mask & ((1u << lane) - 1u));
                        if (pos < q.bmax) list[pos] = (uint64_t(uint32_t(atom - sys_base)) << 30) | uint32_t(packed);
                    }
                    hits += __popc(mask);
                }
                __syncwarp();
                const int k_list = min(hits, q.bmax);
                for (int e = lane; e < k_list; e += 32) {
                    const uint64_t key = list[e];
                    int rank = 0;
                    for (int f = 0; f < k_list; ++f) rank += list[f] < key ? 1 : 0;
                    const int64_t slot = row * q.bmax + rank;
                    q.nbr_out[slot] = sys_base + int32_t(key >> 30);
                    q.shift_out[3 * slot] = int32_t((key >> 20) & 1023u) - 512;
                    q.shift_out[3 * slot + 1] = int32_t((key >> 10) & 1023u) - 512;
                    q.shift_out[3 * slot + 2] = int32_t(key & 1023u) - 512;
                }
                if (lane == 0) {
                    q.count_out[row] = hits;
                    if (hits > q.bmax) raise_flag(q.flags, FMD_FLAG_CANDIDATE_OVERFLOW);
                }
                __syncwarp();
            }
            continue;
        }
        for (int hb = h_begin; hb < h_end; hb += kMaxHome) {
            const int n_home = min(kMaxHome, h_end - hb);
            for (int h = threadIdx.x; h < n_home; h += blockDim.x) m.hits[h] = 0;
            for (int c0 = 0; c0 < staged_total; c0 += kStageCap) {
                const int ns = min(kStageCap, staged_total - c0);
                __syncthreads();
                for (int t = threadIdx.x; t < ns; t += blockDim.x) {
                    const int k = c0 + t;
                    int lo = 0, hi = n_off;  // last offset with o_pref[o] <= k
                    while (hi - lo > 1) {
                        const int mid = (lo + hi) >> 1;
                        if (m.o_pref[mid] <= k) lo = mid; else hi = mid;
                    }
                    const int src = m.o_begin[lo] + (k - m.o_pref[lo]);
                    const float4 p = q.cell_pos[src];
                    m.pos[t] = make_float4(p.x + m.o_shift[3 * lo], p.y + m.o_shift[3 * lo + 1],
                                           p.z + m.o_shift[3 * lo + 2], 0.f);
                    m.atom[t] = q.cell_atoms[src];
                    m.img[t] = m.o_img[lo];
                }
                __syncthreads();
                for (int h = warp; h < n_home; h += kQueryWarps) {
                    const float4 hp = q.cell_pos[hb + h];
                    const int32_t ha = q.cell_atoms[hb + h];
                    const int64_t row = ha;
                    int hits = m.hits[h];
                    for (int base = 0; base < ns; base += 32) {
                        const int k = base + lane;
                        bool hit = false;
                        int32_t atom = 0;
                        int packed = 0;
                        if (k < ns) {
                            const float4 p = m.pos[k];
                            const float dx = p.x - hp.x, dy = p.y - hp.y, dz = p.z - hp.z;
                            const float d2 = (dx * dx + dy * dy) + dz * dz;
                            atom = m.atom[k];
                            packed = m.img[k];
                            hit = d2 < cut2 && !(atom == ha && packed == zero_img);
                        }
                        const unsigned mask = __ballot_sync(0xffffffffu, hit);
                        if (hit) {
                            const int pos = hits + __popc(mask & ((1u << lane) - 1u));
                            if (pos < q.bmax) {
                                const int64_t slot = row * q.bmax + pos;
                                q.nbr_out[slot] = atom;
                                q.shift_out[3 * slot] = ((packed >> 20) & 1023) - 512;
                                q.shift_out[3 * slot + 1] = ((packed >> 10) & 1023) - 512;
                                q.shift_out[3 * slot + 2] = (packed & 1023) - 512;
                            }
                        }
                        hits += __popc(mask);
                    }
                    if (lane == 0) m.hits[h] = hits;
                }
            }
            __syncthreads();
            // canonical order of every home row: rank sort by (neighbour, image)
            uint64_t* list = m.list + size_t(warp) * q.list_cap;
            for (int h = warp; h < n_home; h += kQueryWarps) {
                const int32_t ha = q.cell_atoms[hb + h];
                const int64_t row = ha;
                const int hits = m.hits[h];
                const int k_list = min(hits, q.bmax);
                if (k_list > q.list_cap) {  // more than the sort buffer holds: reported, left unsorted
                    if (lane == 0) {
                        q.count_out[row] = hits;
                        raise_flag(q.flags, FMD_FLAG_CANDIDATE_OVERFLOW);
                    }
                    continue;
                }
                for (int e = lane; e < k_list; e += 32) {
                    const int64_t slot = row * q.bmax + e;
                    const int3 s3 = make_int3(q.shift_out[3 * slot], q.shift_out[3 * slot + 1], q.shift_out[3 * slot + 2]);
                    list[e] = cand_key(q.nbr_out[slot] - sys_base, s3);
                }
                __syncwarp();
                for (int e = lane; e < k_list; e += 32) {
                    const uint64_t key = list[e];
                    int rank = 0;
                    for (int f = 0; f < k_list; ++f) rank += list[f] < key ? 1 : 0;
                    const int64_t slot = row * q.bmax + rank;
                    q.nbr_out[slot] = sys_base + int32_t(key >> 30);
                    q.shift_out[3 * slot] = int32_t((key >> 20) & 1023u) - 512;
                    q.shift_out[3 * slot + 1] = int32_t((key >> 10) & 1023u) - 512;
                    q.shift_out[3 * slot + 2] = int32_t(key & 1023u) - 512;
                }
                if (lane == 0) {
                    q.count_out[row] = hits;
                    if (hits > q.bmax) raise_flag(q.flags, FMD_FLAG_CANDIDATE_OVERFLOW);
                }
                __syncwarp();
            }
            __syncthreads();
        }
    }
}

// fill unused candidate slots (neighbour = R*n, shift 0) of every row
__global__ void cand_fill_kernel(int64_t rows, int32_t bmax, int32_t fill, int32_t* __restrict__ nbr,
                                 int32_t* __restrict__ shift, const int32_t* __restrict__ count) {
    const int64_t total = rows * bmax;
    for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < total;
         t += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = t / bmax;
        const int k = int(t - r * bmax);
        if (k >= count[r]) {
            nbr[t] = fill;
            shift[3 * t] = 0;
            shift[3 * t + 1] = 0;
            shift[3 * t + 2] = 0;
        }
    }
}

// reference snapshot of the refresh: positions, wraps; wrap delta reset
__global__ void refresh_reference_kernel(const float* __restrict__ positions, int64_t total, Cell9 cell,
                                         float* __restrict__ ref_pos, int32_t* __restrict__ ref_wraps,
                                         int32_t* __restrict__ wrap_delta) {
    for (int64_t a = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; a < total;
         a += int64_t(gridDim.x) * blockDim.x) {
        float3 p = ld3(positions, a), w, f;
        int3 wr;
        wrap_atom(p, cell, w, wr, f);
        ref_pos[3 * a] = p.x;
        ref_pos[3 * a + 1] = p.y;
        ref_pos[3 * a + 2] = p.z;
        ref_wraps[3 * a] = wr.x;
        ref_wraps[3 * a + 1] = wr.y;
        ref_wraps[3 * a + 2] = wr.z;
        wrap_delta[3 * a] = 0;
        wrap_delta[3 * a + 1] = 0;
        wrap_delta[3 * a + 2] = 0;
    }
}

// ------------------------------------------------------------ re-filter

constexpr int kRefThreads = 512;
constexpr int kRefWarps = kRefThreads / 32;

struct RefilterArgs {
    const float* positions;      // [R*n, 3] float32 (the integrator's float32 copy)
    Cell9 cell;
    const float* ref_pos;        // refresh snapshot
    const int32_t* ref_wraps;
    const int32_t* cand_nbr;     // [R*n, bmax] global rows
    const int32_t* cand_shift;   // [R*n, bmax, 3]
    const int32_t* cand_count;   // [R*n]
    int64_t n_atoms;
    int32_t n_systems;
    int32_t bmax;
    float cutoff2;               // rc^2 (float32)
    float skin_limit;            // skin + 1e-6: an atom may move skin_limit / 2
    int32_t minimum_image;       // a lattice jump of the caller's coordinates is no motion
    int64_t e_cap;               // edge rows of the whole union
    int32_t pad_image[3];        // far self-loop image
    // outputs
    float* wrapped;              // [R*n, 3]
    int32_t* wrap_delta;         // [R*n, 3]
    int32_t* counts;             // [R*n] edges per centre
    int32_t* local_off;          // [R*n] exclusive offsets inside the system
    int32_t* sys_total;          // [R]
    float* max_disp;             // [R]
    int32_t* edge_index;         // [e_cap, 2] (centre, neighbour), global rows
    float* edge_image;           // [e_cap, 3]
    int64_t* recv_off;           // [R*n + 1] receiver CSR (real edges)
    int64_t* send_off;           // [R*n + 1] sender CSR offsets
    int32_t* send_perm;          // [e_cap] edge ids grouped by sender (first n_edges used)
    int64_t* n_edges;            // [1]
    int32_t* flags;              // [1]: FMD_FLAG_* of this build
};

__device__ __forceinline__ int block_scan_exclusive(int v, int* smem, int& total) {
    // blockDim <= 1024; warp scan + warp totals
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, m);
        if (lane >= m) x += y;
    }
    __syncthreads();
    if (lane == 31) smem[warp] = x;
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        int w = lane < nw ? smem[lane] : 0;
#pragma unroll
        for (int m = 1; m < 32; m <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, m);
            if (lane >= m) w += y;
        }
        if (lane < nw) smem[lane] = w;  // inclusive warp prefix
    }
    __syncthreads();
    const int before = warp > 0 ? smem[warp - 1] : 0;
    total = smem[(blockDim.x >> 5) - 1];
    __syncthreads();
    return before + x - v;
}

// Both re-filter kernels run a thread-block cluster of kRefCluster CTAs per system (grid n_systems *
// kRefCluster): CTA `rank` of a system owns the centre slice [rank * per, rank * per + per); the
// per-system steps (the displacement maximum, the offsets of the count scan, the sender CSR) go
// through cluster barriers (release / acquire at cluster scope) and the distributed shared memory of
// the cluster. A 135-atom system so spreads over 8 SMs instead of one. Every CTA of a cluster takes
// every barrier (no early exit), and the last barrier keeps each CTA's shared memory alive while the
// others may still read it.
constexpr int kRefCluster = 8;

__device__ __forceinline__ void slice_of(int n, int rank, int& lo, int& hi) {
    const int per = (n + kRefCluster - 1) / kRefCluster;
    lo = min(n, rank * per);
    hi = min(n, lo + per);
}

// Count kernel: wrap, displacement and skin test, edges per centre, per-system offsets.
__global__ void __cluster_dims__(kRefCluster, 1, 1) __launch_bounds__(kRefThreads)
    refilter_count_kernel(RefilterArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float3* s_w = reinterpret_cast<float3*>(smem_raw);                    // wrapped [n] (the whole system)
    int3* s_wd = reinterpret_cast<int3*>(s_w + a.n_atoms);                // wrap delta [n]
    __shared__ int s_scan[32];
    __shared__ float s_max[32];
    __shared__ float s_cmax;   // this CTA's largest displacement (read by rank 0)
    __shared__ int s_total;    // this CTA's edge count (read by the higher ranks)
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = int(cluster.block_rank());
    const int64_t sys = blockIdx.x / kRefCluster;
    const int64_t base = sys * a.n_atoms;
    const int n = int(a.n_atoms);
    int lo, hi;
    slice_of(n, rank, lo, hi);
    // wrap this CTA's slice
    float my_max = 0.f;
    bool nonfinite = false;
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const int64_t g = base + i;
        float3 p = ld3(a.positions, g), w, f;
        int3 wr;
        wrap_atom(p, a.cell, w, wr, f);
        const int3 rw = ld3i(a.ref_wraps, g);
        int3 wd = make_int3(wr.x - rw.x, wr.y - rw.y, wr.z - rw.z);
        const float3 r = ld3(a.ref_pos, g);
        float dx = p.x - r.x, dy = p.y - r.y, dz = p.z - r.z;
        if (a.minimum_image) {
            // minimum-image displacement; the jump leaves the wrapped row (and the images) unchanged
            // (fixed_capacity_builder.py:2229-2241)
            const float3 fj = row_times(make_float3(dx, dy, dz), a.cell.inv);
            const float jx = rintf(fj.x), jy = rintf(fj.y), jz = rintf(fj.z);
            const float3 lj = row_times(make_float3(jx, jy, jz), a.cell.c);
            dx -= lj.x;
            dy -= lj.y;
            dz -= lj.z;
            wd = make_int3(wd.x - int(jx), wd.y - int(jy), wd.z - int(jz));
        }
        a.wrapped[3 * g] = w.x;
        a.wrapped[3 * g + 1] = w.y;
        a.wrapped[3 * g + 2] = w.z;
        a.wrap_delta[3 * g] = wd.x;
        a.wrap_delta[3 * g + 1] = wd.y;
        a.wrap_delta[3 * g + 2] = wd.z;
        const float d = sqrtf((dx * dx + dy * dy) + dz * dz);
        if (!(d == d) || !isfinite(p.x) || !isfinite(p.y) || !isfinite(p.z)) nonfinite = true;
        my_max = fmaxf(my_max, d);
    }
    // CTA max of the displacement (NaN-safe: nonfinite is flagged separately)
    for (int m = 16; m > 0; m >>= 1) my_max = fmaxf(my_max, __shfl_xor_sync(0xffffffffu, my_max, m));
    if ((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = my_max;
    if (nonfinite) raise_flag(a.flags, FMD_FLAG_NONFINITE);
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = 0.f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, s_max[w]);
        s_cmax = m;
    }
    cluster.sync();  // every slice wrapped: the whole system's rows are visible
    if (rank == 0 && threadIdx.x == 0) {
        float m = 0.f;
        for (int r = 0; r < kRefCluster; ++r) m = fmaxf(m, *cluster.map_shared_rank(&s_cmax, r));
        a.max_disp[sys] = m;
        if (!(m * 2.0f <= a.skin_limit)) raise_flag(a.flags, FMD_FLAG_SKIN);
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) {  // the system's rows, written by the whole cluster
        const int64_t g = base + i;
        s_w[i] = make_float3(__ldcg(a.wrapped + 3 * g), __ldcg(a.wrapped + 3 * g + 1), __ldcg(a.wrapped + 3 * g + 2));
        s_wd[i] = make_int3(__ldcg(a.wrap_delta + 3 * g), __ldcg(a.wrap_delta + 3 * g + 1),
                            __ldcg(a.wrap_delta + 3 * g + 2));
    }
    __syncthreads();
    // counts: one warp per centre of the slice
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = lo + warp; i < hi; i += kRefWarps) {
        const int64_t g = base + i;
        const int cnt = min(a.cand_count[g], a.bmax);
        const float3 p = s_w[i];
        const int3 wdi = s_wd[i];
        int edges = 0;
        for (int k0 = 0; k0 < cnt; k0 += 32) {
            const int k = k0 + lane;
            bool hit = false;
            if (k < cnt) {
                int64_t j = int64_t(a.cand_nbr[g * a.bmax + k]) - base;
                j = j < 0 ? 0 : (j >= n ? n - 1 : j);
                const int3 s = ld3i(a.cand_shift, g * a.bmax + k);
                const int3 wdj = s_wd[j];
                const float sx = float(s.x + wdj.x - wdi.x), sy = float(s.y + wdj.y - wdi.y),
                            sz = float(s.z + wdj.z - wdi.z);
                hit = refilter_dist2(p, s_w[j], sx, sy, sz, a.cell.c) < a.cutoff2;
            }
            edges += __popc(__ballot_sync(0xffffffffu, hit));
        }
        if (lane == 0) a.counts[g] = edges;
    }
    __syncthreads();
    // exclusive scan of the slice's counts (offsets inside the slice for now)
    int running = 0;
    for (int i0 = lo; i0 < hi; i0 += blockDim.x) {
        const int i = i0 + threadIdx.x;
        const int v = i < hi ? a.counts[base + i] : 0;
        int chunk_total;
        const int ex = block_scan_exclusive(v, s_scan, chunk_total);
        if (i < hi) a.local_off[base + i] = running + ex;
        running += chunk_total;
    }
    if (threadIdx.x == 0) s_total = running;
    cluster.sync();  // every slice's total is known
    int prefix = 0;  // edges of the lower ranks' slices
    for (int r = 0; r < rank; ++r) prefix += *cluster.map_shared_rank(&s_total, r);
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) a.local_off[base + i] += prefix;
    if (rank == kRefCluster - 1 && threadIdx.x == 0) a.sys_total[sys] = prefix + running;
    cluster.sync();  // no CTA leaves while another may read its shared memory
}

// Materialize kernel: the edges in canonical order, both CSRs, the padding rows.
__global__ void __cluster_dims__(kRefCluster, 1, 1) __launch_bounds__(kRefThreads)
    refilter_materialize_kernel(RefilterArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float3* s_w = reinterpret_cast<float3*>(smem_raw);
    int3* s_wd = reinterpret_cast<int3*>(s_w + a.n_atoms);
    int32_t* s_cursor = reinterpret_cast<int32_t*>(s_wd + a.n_atoms);      // sender counts, then cursors [n]
    int32_t* s_soff = s_cursor + a.n_atoms;                                // sender offsets [n + 1]
    __shared__ int s_scan[32];
    __shared__ long long s_base, s_grand;
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = int(cluster.block_rank());
    const int64_t sys = blockIdx.x / kRefCluster;
    const int64_t base = sys * a.n_atoms;
    const int n = int(a.n_atoms);
    int lo, hi;
    slice_of(n, rank, lo, hi);
    // the sender arrays of the system live in rank 0's shared memory
    int32_t* cursor0 = cluster.map_shared_rank(s_cursor, 0);
    const int32_t* soff0 = cluster.map_shared_rank(s_soff, 0);
    if (threadIdx.x == 0) {
        long long b = 0, g = 0;
        for (int r = 0; r < a.n_systems; ++r) {
            const int t = a.sys_total[r];
            if (r < sys) b += t;
            g += t;
        }
        s_base = b;
        s_grand = g;
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int64_t g = base + i;
        s_w[i] = ld3(a.wrapped, g);
        s_wd[i] = ld3i(a.wrap_delta, g);
        if (rank == 0) s_cursor[i] = 0;
    }
    cluster.sync();  // rank 0's sender counts are zero before any CTA adds to them
    const int64_t sys_base = s_base;
    const int64_t grand = s_grand;
    const int64_t cap = a.e_cap;
    // receiver CSR over the real edges (global), clipped to the capacity
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const int64_t o = sys_base + a.local_off[base + i];
        a.recv_off[base + i] = o < cap ? o : cap;
    }
    if (sys == a.n_systems - 1 && rank == 0 && threadIdx.x == 0) {
        a.recv_off[int64_t(a.n_systems) * a.n_atoms] = grand < cap ? grand : cap;
        a.n_edges[0] = grand;
        if (grand > cap) raise_flag(a.flags, FMD_FLAG_EDGE_OVERFLOW);
    }
    // edges of the slice's centres: warp per centre, ballot compaction in candidate (= canonical) order
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = lo + warp; i < hi; i += kRefWarps) {
        const int64_t g = base + i;
        const int cnt = min(a.cand_count[g], a.bmax);
        const float3 p = s_w[i];
        const int3 wdi = s_wd[i];
        int64_t out = sys_base + a.local_off[g];
        for (int k0 = 0; k0 < cnt; k0 += 32) {
            const int k = k0 + lane;
            bool hit = false;
            int j = 0;
            int3 img = make_int3(0, 0, 0);
            if (k < cnt) {
                int64_t jj = int64_t(a.cand_nbr[g * a.bmax + k]) - base;
                j = int(jj < 0 ? 0 : (jj >= n ? n - 1 : jj));
                const int3 s = ld3i(a.cand_shift, g * a.bmax + k);
                const int3 wdj = s_wd[j];
                img = make_int3(s.x + wdj.x - wdi.x, s.y + wdj.y - wdi.y, s.z + wdj.z - wdi.z);
                hit = refilter_dist2(p, s_w[j], float(img.x), float(img.y), float(img.z), a.cell.c) < a.cutoff2;
            }
            const unsigned mask = __ballot_sync(0xffffffffu, hit);
            if (hit) {
                const int64_t e = out + __popc(mask & ((1u << lane) - 1u));
                if (e < cap) {
                    a.edge_index[2 * e] = int32_t(g);
                    a.edge_index[2 * e + 1] = int32_t(base + j);
                    a.edge_image[3 * e] = float(img.x);
                    a.edge_image[3 * e + 1] = float(img.y);
                    a.edge_image[3 * e + 2] = float(img.z);
                    atomicAdd(cursor0 + j, 1);  // sender count
                }
            }
            out += __popc(mask);
        }
    }
    cluster.sync();  // every edge written, every sender counted
    // sender CSR offsets of the system: counts -> exclusive scan in rank 0
    if (rank == 0) {
        int running = 0;
        for (int i0 = 0; i0 < n; i0 += blockDim.x) {
            const int i = i0 + threadIdx.x;
            const int v = i < n ? s_cursor[i] : 0;
            int chunk_total;
            const int ex = block_scan_exclusive(v, s_scan, chunk_total);
            if (i < n) s_soff[i] = running + ex;
            running += chunk_total;
        }
        if (threadIdx.x == 0) s_soff[n] = running;
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += blockDim.x) s_cursor[i] = 0;
    }
    cluster.sync();  // offsets known, cursors zero
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const int64_t o = sys_base + soff0[i];
        a.send_off[base + i] = o < cap ? o : cap;
    }
    if (sys == a.n_systems - 1 && rank == 0 && threadIdx.x == 0)
        a.send_off[int64_t(a.n_systems) * a.n_atoms] = grand < cap ? grand : cap;
    const int64_t sys_edges = a.sys_total[sys];
    for (int64_t t = int64_t(rank) * blockDim.x + threadIdx.x; t < sys_edges; t += int64_t(kRefCluster) * blockDim.x) {
        const int64_t e = sys_base + t;
        if (e >= cap) break;
        const int j = int(int64_t(__ldcg(a.edge_index + 2 * e + 1)) - base);
        const int slot = atomicAdd(cursor0 + j, 1);
        const int64_t dst = sys_base + soff0[j] + slot;
        if (dst < cap) a.send_perm[dst] = int32_t(e);
    }
    cluster.sync();  // every sender run filled
    // each sender run of the slice ascending by edge id (rank sort, warp per sender)
    for (int j = lo + warp; j < hi; j += kRefWarps) {
        const int64_t b = sys_base + soff0[j];
        const int len = soff0[j + 1] - soff0[j];
        if (len <= 1 || b + len > cap) continue;
        int vals[8];
        int nv = 0;
        for (int k = lane; k < len && nv < 8; k += 32) vals[nv++] = __ldcg(a.send_perm + b + k);
        __syncwarp();
        int ranks[8];
        for (int v = 0; v < nv; ++v) {
            int r = 0;
            for (int f = 0; f < len; ++f) r += __ldcg(a.send_perm + b + f) < vals[v] ? 1 : 0;
            ranks[v] = r;
        }
        __syncwarp();
        for (int v = 0; v < nv; ++v) a.send_perm[b + ranks[v]] = vals[v];
        if (len > 256 && lane == 0) raise_flag(a.flags, FMD_FLAG_CANDIDATE_OVERFLOW);
        __syncwarp();
    }
    // padding rows [grand, cap): far self-loops round robin over the union's atoms
    const int64_t total_atoms = int64_t(a.n_systems) * a.n_atoms;
    const int64_t first = grand < cap ? grand : cap;
    for (int64_t e = first + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < cap;
         e += int64_t(gridDim.x) * blockDim.x) {
        const int32_t atom = int32_t((e - first) % total_atoms);
        a.edge_index[2 * e] = atom;
        a.edge_index[2 * e + 1] = atom;
        a.edge_image[3 * e] = float(a.pad_image[0]);
        a.edge_image[3 * e + 1] = float(a.pad_image[1]);
        a.edge_image[3 * e + 2] = float(a.pad_image[2]);
    }
    cluster.sync();  // rank 0's sender arrays stay alive until every CTA is done with them
}

// ------------------------------------------------------------- ragged list
//
// Two passes and no candidate matrix of (neighbour, shift) rows:
//   collect: one sweep of the cell list; per centre it counts the pairs the
//            eager path keeps and stores its candidates' keys
//            (neighbour << 12 | image, 32-bit below 2^20 atoms) unsorted in a
//            scratch row;
//   scan:    the kept counts give the row offsets;
//   emit:    a warp per centre sorts its keys by (neighbour, image) with a
//            bitonic network in registers and writes the kept pairs into its
//            output row (consecutive lanes, consecutive edges).
//
// A pair is kept when it is a candidate (dist2 < (rc + 1e-6)^2 in the
// staged arithmetic of the candidate build, gpu_graph_builder.py:161) and
// |(q - p) + image @ cell| < rc (gpu_graph_builder.py:186-192). The two
// distances differ only by float32 rounding, bounded on the host by delta: a
// candidate with dist2 < (rc - delta)^2 passes the second test, so the
// collect sweep evaluates that test only in the thin shell between the two
// radii.

constexpr int kRagWarps = 8;
constexpr int kRagStage = 1024;   // staged (atom, image) entries per chunk
constexpr int kRagHome = 512;     // home atoms per pass of the collect sweep
constexpr int kRagMaxList = 2048; // largest candidate row (bmax + 1)

struct RaggedArgs {
    const int32_t* cell_start;   // [ncells + 1]
    const int32_t* cell_atoms;   // atoms grouped by cell
    const float4* cell_pos;      // wrapped positions grouped by cell
    const float4* wrapped;       // wrapped positions by atom
    Cell9 cell;
    Grid grid;
    float cand_cut;              // rc + 1e-6: candidate iff dist2 < cand_cut^2
    float cutoff;                // rc: kept iff |diff| < rc
    float lo2;                   // a candidate below it passes |diff| < rc
    int32_t bmax;                // more candidates of a centre raise FMD_FLAG_CANDIDATE_OVERFLOW
    int32_t row_cap;             // keys per scratch row: bmax + 1 (the centre itself included)
    int32_t sort_cap;            // emit pass: per-warp shared list for rows over 128 keys (0: none)
    int32_t off_cap;             // (cell, image) offsets of a neighbourhood
    void* keys;                  // [n, row_cap] candidate keys (KeyT)
    int32_t* n_keys;             // [n] candidates per centre (the centre itself included)
    int64_t* counts;             // kept pairs per centre
    const int64_t* offsets;      // row offsets [n + 1]
    int64_t n_atoms;
    int64_t e_cap;
    int64_t* center;
    int64_t* neighbor;
    int32_t* images;
    float* dist;
    int32_t* flags;
};

// an image in 12 bits, 4 per axis offset by 8, ordered as (x, y, z) (|image| <= the search reach <= 5)
__device__ __forceinline__ int32_t pack_image4(int ix, int iy, int iz) {
    return ((ix + 8) << 8) | ((iy + 8) << 4) | (iz + 8);
}

__device__ __forceinline__ int3 unpack_image4(uint32_t v) {
    return make_int3(int((v >> 8) & 15u) - 8, int((v >> 4) & 15u) - 8, int(v & 15u) - 8);
}

struct Hood {
    int32_t* begin;   // [off_cap] first cell-grouped row of the offset's cell
    int32_t* pref;    // [off_cap + 1] exclusive prefix of the offsets' atom counts
    int32_t* img;     // [off_cap] packed image (pack_image4)
    float* shift;     // [off_cap * 3] image @ cell
};

// (cell, image) of offset k of home cell `home`: the offset's atom count, with its row start,
// packed image and image @ cell stored
__device__ __forceinline__ int hood_entry(const Hood& o, const int32_t* __restrict__ cell_start, int home, int k,
                                          const Grid& g, const Cell9& cell) {
    const int w1 = 2 * g.s[1] + 1, w2 = 2 * g.s[2] + 1;
    const int hx = home / (g.n[1] * g.n[2]), hy = (home / g.n[2]) % g.n[1], hz = home % g.n[2];
    const int gx = hx + k / (w1 * w2) - g.s[0], gy = hy + (k / w2) % w1 - g.s[1], gz = hz + k % w2 - g.s[2];
    const int ix = floor_div(gx, g.n[0]), iy = floor_div(gy, g.n[1]), iz = floor_div(gz, g.n[2]);
    const int cx = gx - ix * g.n[0], cy = gy - iy * g.n[1], cz = gz - iz * g.n[2];
    const int c = (cx * g.n[1] + cy) * g.n[2] + cz;
    const int b = cell_start[c];
    o.begin[k] = b;
    o.img[k] = pack_image4(ix, iy, iz);
    const float fx = float(ix), fy = float(iy), fz = float(iz);
    o.shift[3 * k] = (fx * cell.c[0] + fy * cell.c[3]) + fz * cell.c[6];
    o.shift[3 * k + 1] = (fx * cell.c[1] + fy * cell.c[4]) + fz * cell.c[7];
    o.shift[3 * k + 2] = (fx * cell.c[2] + fy * cell.c[5]) + fz * cell.c[8];
    return cell_start[c + 1] - b;
}

// The (cell, image) offsets around home cell `home` and the prefix of their atom counts; returns
// the number of staged entries, with the block synchronised. Up to 32 offsets (a search reach of
// one cell) one warp builds it.
__device__ int load_hood(const Hood& o, const int32_t* __restrict__ cell_start, int home, const Grid& g,
                         const Cell9& cell, int* s_scan) {
    const int n_off = (2 * g.s[0] + 1) * (2 * g.s[1] + 1) * (2 * g.s[2] + 1);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = int(blockDim.x >> 5);
    __syncthreads();  // the previous home cell's readers are done
    if (n_off <= 32) {
        if (warp == 0) {
            const int cnt = lane < n_off ? hood_entry(o, cell_start, home, lane, g, cell) : 0;
            int x = cnt;
            for (int d = 1; d < 32; d <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, d);
                if (lane >= d) x += y;
            }
            if (lane < n_off) o.pref[lane] = x - cnt;
            if (lane == 31) o.pref[n_off] = x;
        }
        __syncthreads();
        return o.pref[n_off];
    }
    int running = 0;
    for (int o0 = 0; o0 < n_off; o0 += blockDim.x) {
        const int k = o0 + threadIdx.x;
        const int cnt = k < n_off ? hood_entry(o, cell_start, home, k, g, cell) : 0;
        int x = cnt;
        for (int d = 1; d < 32; d <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, d);
            if (lane >= d) x += y;
        }
        if (lane == 31) s_scan[warp] = x;
        __syncthreads();
        int before = 0, total = 0;
        for (int w = 0; w < nw; ++w) {
            if (w < warp) before += s_scan[w];
            total += s_scan[w];
        }
        if (k < n_off) o.pref[k] = running + before + x - cnt;
        running += total;
        __syncthreads();
    }
    if (threadIdx.x == 0) o.pref[n_off] = running;
    __syncthreads();
    return running;
}

// the offset of staged entry t: the last o with pref[o] <= t
__device__ __forceinline__ int hood_offset(const int32_t* pref, int n_off, int t) {
    int lo = 0, hi = n_off;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (pref[mid] <= t) lo = mid; else hi = mid;
    }
    return lo;
}

// fn(e, src, k) for every staged entry t in [c0, c0 + ns) (e = t - c0, src its cell-grouped row, k
// its offset): a warp per offset, its lanes over the offset cell's atoms
template <class F>
__device__ __forceinline__ void for_staged(const Hood& o, int n_off, int c0, int ns, F&& fn) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = int(blockDim.x >> 5);
    for (int k = warp; k < n_off; k += nw) {
        const int p0 = o.pref[k];
        const int lo = max(p0, c0), hi = min(o.pref[k + 1], c0 + ns);
        for (int t = lo + lane; t < hi; t += 32) fn(t - c0, o.begin[k] + (t - p0), k);
    }
}

// the eager path's distance |(q - p) + sh| (gpu_graph_builder.py:186-192) for sh = image @ cell
__device__ __forceinline__ float eager_dist(float4 p, float4 q, float sx, float sy, float sz) {
    const float dx = (q.x - p.x) + sx, dy = (q.y - p.y) + sy, dz = (q.z - p.z) + sz;
    return sqrtf((dx * dx + dy * dy) + dz * dz);
}

__device__ __forceinline__ int warp_sum_int(int v) {
    for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
    return v;
}

// a staged entry's candidate distance: (q + image @ cell) - p, squared in the candidate build's order
__device__ __forceinline__ float staged_dist2(float4 s, float4 p) {
    const float dx = s.x - p.x, dy = s.y - p.y, dz = s.z - p.z;
    return (dx * dx + dy * dy) + dz * dz;
}

// KeyT: uint32_t when every atom index is below 2^20, else uint64_t
template <class KeyT>
__global__ void __launch_bounds__(kRagWarps * 32) ragged_nbr_collect_kernel(RaggedArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float4* spos = reinterpret_cast<float4*>(smem_raw);      // [kRagStage] staged position + image shift
    KeyT* skey = reinterpret_cast<KeyT*>(spos + kRagStage);  // [kRagStage] (atom << 12) | image
    Hood o;
    o.begin = reinterpret_cast<int32_t*>(skey + kRagStage);
    o.pref = o.begin + a.off_cap;
    o.img = o.pref + a.off_cap + 1;
    int32_t* kept_n = o.img + a.off_cap;   // [kRagHome] kept pairs (the centre itself included)
    int32_t* cand_n = kept_n + kRagHome;   // [kRagHome] candidates (the centre itself included)
    o.shift = reinterpret_cast<float*>(cand_n + kRagHome);
    __shared__ int s_scan[32];
    KeyT* keys = static_cast<KeyT*>(a.keys);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const unsigned below = (1u << lane) - 1u;
    const Grid& g = a.grid;
    const float cut2 = a.cand_cut * a.cand_cut;
    const int n_off = (2 * g.s[0] + 1) * (2 * g.s[1] + 1) * (2 * g.s[2] + 1);
    for (int home = blockIdx.x; home < g.ncells; home += gridDim.x) {
        const int h_begin = a.cell_start[home], h_end = a.cell_start[home + 1];
        if (h_begin == h_end) continue;  // uniform per CTA
        const int staged = load_hood(o, a.cell_start, home, g, a.cell, s_scan);
        for (int hb = h_begin; hb < h_end; hb += kRagHome) {
            const int n_home = min(kRagHome, h_end - hb);
            for (int h = threadIdx.x; h < n_home; h += blockDim.x) kept_n[h] = cand_n[h] = 0;
            for (int c0 = 0; c0 < staged; c0 += kRagStage) {
                const int ns = min(kRagStage, staged - c0);
                __syncthreads();
                for_staged(o, n_off, c0, ns, [&](int e, int src, int k) {
                    const float4 q = a.cell_pos[src];
                    spos[e] = make_float4(q.x + o.shift[3 * k], q.y + o.shift[3 * k + 1], q.z + o.shift[3 * k + 2], 0.f);
                    skey[e] = (KeyT(uint32_t(a.cell_atoms[src])) << 12) | KeyT(uint32_t(o.img[k]));
                });
                __syncthreads();
                for (int h = warp; h < n_home; h += kRagWarps) {
                    const float4 hp = a.cell_pos[hb + h];
                    KeyT* row = keys + size_t(a.cell_atoms[hb + h]) * a.row_cap;
                    int n = cand_n[h], kept = 0;
                    // the test: lane i keeps the hit mask of staged entries [32 i, 32 i + 32) (ns <= 1024)
                    unsigned mine = 0u;
                    for (int base = 0; base < ns; base += 32) {
                        const int k = base + lane;
                        const bool hit = k < ns && staged_dist2(spos[k], hp) < cut2;
                        const unsigned m = __ballot_sync(0xffffffffu, hit);
                        if (lane == (base >> 5)) mine = m;
                    }
                    // the hits, one per lane: the owning 32-entry group by a search over the groups'
                    // inclusive hit counts, the entry by the rank of the hit inside the group's mask
                    const int c = __popc(mine);
                    int incl = c;
                    for (int d = 1; d < 32; d <<= 1) {
                        const int y = __shfl_up_sync(0xffffffffu, incl, d);
                        if (lane >= d) incl += y;
                    }
                    const int excl = incl - c, total = __shfl_sync(0xffffffffu, incl, 31);
                    for (int j0 = 0; j0 < total; j0 += 32) {
                        const int jj = j0 + lane;
                        int grp = 0;
#pragma unroll
                        for (int step = 16; step >= 1; step >>= 1)
                            if (__shfl_sync(0xffffffffu, incl, grp + step - 1) <= jj) grp += step;
                        const unsigned m = __shfl_sync(0xffffffffu, mine, grp);
                        const int r = jj - __shfl_sync(0xffffffffu, excl, grp);
                        if (jj < total) {
                            const int k = grp * 32 + int(__fns(m, 0, r + 1));
                            const float d2 = staged_dist2(spos[k], hp);
                            const int pos = n + jj;
                            if (pos < a.row_cap) row[pos] = skey[k];
                            if (d2 < a.lo2) {
                                ++kept;
                            } else {  // the shell: the eager path's own distance decides
                                const int lo = hood_offset(o.pref, n_off, c0 + k);
                                const float4 q = a.cell_pos[o.begin[lo] + (c0 + k - o.pref[lo])];
                                kept += eager_dist(hp, q, o.shift[3 * lo], o.shift[3 * lo + 1], o.shift[3 * lo + 2]) <
                                                a.cutoff
                                            ? 1
                                            : 0;
                            }
                        }
                    }
                    n += total;
                    kept = warp_sum_int(kept);
                    if (lane == 0) {
                        kept_n[h] += kept;
                        cand_n[h] = n;
                    }
                }
            }
            __syncthreads();
            for (int h = threadIdx.x; h < n_home; h += blockDim.x) {
                // the centre meets itself once (zero image, distance 0) when its position is finite
                const float4 hp = a.cell_pos[hb + h];
                const int self = (isfinite(hp.x) && isfinite(hp.y) && isfinite(hp.z)) ? 1 : 0;
                const int32_t row = a.cell_atoms[hb + h];
                a.counts[row] = kept_n[h] - self;
                a.n_keys[row] = cand_n[h];
                if (cand_n[h] - self > a.bmax) raise_flag(a.flags, FMD_FLAG_CANDIDATE_OVERFLOW);
            }
        }
    }
}

// ascending bitonic sort of list[0, n) (n a power of two) by one warp, in shared memory
template <class KeyT>
__device__ __forceinline__ void warp_bitonic_sort(KeyT* list, int n, int lane) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int t = lane; t < (n >> 1); t += 32) {
                const int i = 2 * t - (t & (stride - 1));
                const int j = i + stride;
                const KeyT x = list[i], y = list[j];
                if ((x > y) == ((i & size) == 0)) {
                    list[i] = y;
                    list[j] = x;
                }
            }
            __syncwarp();
        }
    }
}

// ascending bitonic sort of 32 * EPL keys held by one warp, element j * 32 + lane in v[j]
template <int EPL, class KeyT>
__device__ __forceinline__ void warp_bitonic_regs(KeyT (&v)[EPL], int lane) {
    constexpr int kN = 32 * EPL;
#pragma unroll
    for (int size = 2; size <= kN; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride >= 32) {  // partners in the same lane
                const int js = stride >> 5;
#pragma unroll
                for (int j = 0; j < EPL; ++j) {
                    if ((j & js) == 0) {
                        const bool up = ((j * 32) & size) == 0;
                        const KeyT x = v[j], y = v[j + js];
                        const bool swap = (x > y) == up;
                        v[j] = swap ? y : x;
                        v[j + js] = swap ? x : y;
                    }
                }
            } else {
                const bool lower = (lane & stride) == 0;
#pragma unroll
                for (int j = 0; j < EPL; ++j) {
                    const KeyT p = __shfl_xor_sync(0xffffffffu, v[j], stride);
                    const bool up = ((j * 32 + lane) & size) == 0;
                    const bool take_min = lower == up;
                    v[j] = (take_min == (p < v[j])) ? p : v[j];
                }
            }
        }
    }
}

template <class KeyT>
struct RowWriter {
    float4 hp;          // the centre's wrapped position
    int32_t row;        // the centre
    KeyT self;          // its own key (zero image)
    int64_t out, end;   // next output edge, end of its row (clipped to e_cap)
};

// one warp: the kept pairs among 32 sorted keys (one per lane, `valid` below the row's key count),
// written at the row's next edges in key order
template <class KeyT>
__device__ __forceinline__ void emit_sorted(const RaggedArgs& a, RowWriter<KeyT>& r, KeyT v, bool valid, int lane) {
    bool keep = false;
    float d = 0.f;
    int32_t j = 0;
    int3 s3 = make_int3(0, 0, 0);
    if (valid) {
        j = int32_t(v >> 12);
        s3 = unpack_image4(uint32_t(v & KeyT(0xFFFu)));
        const float4 q = a.wrapped[j];
        const float3 sh = row_times(make_float3(float(s3.x), float(s3.y), float(s3.z)), a.cell.c);
        // the candidate's staged distance (as the collect sweep computed it) and the eager distance
        const float ex = (q.x + sh.x) - r.hp.x, ey = (q.y + sh.y) - r.hp.y, ez = (q.z + sh.z) - r.hp.z;
        const float d2 = (ex * ex + ey * ey) + ez * ez;
        d = eager_dist(r.hp, q, sh.x, sh.y, sh.z);
        keep = v != r.self && (d2 < a.lo2 || d < a.cutoff);
    }
    const unsigned mask = __ballot_sync(0xffffffffu, keep);
    if (keep) {
        const int64_t e = r.out + __popc(mask & ((1u << lane) - 1u));
        if (e < r.end) {
            a.center[e] = r.row;
            a.neighbor[e] = j;
            a.images[3 * e] = s3.x;
            a.images[3 * e + 1] = s3.y;
            a.images[3 * e + 2] = s3.z;
            a.dist[e] = d;
        }
    }
    r.out += __popc(mask);
}

template <int EPL, class KeyT>
__device__ __forceinline__ void sort_and_emit(const RaggedArgs& a, RowWriter<KeyT>& r, const KeyT (&pre)[4], int k,
                                              int lane) {
    KeyT v[EPL];
#pragma unroll
    for (int j = 0; j < EPL; ++j) v[j] = j * 32 + lane < k ? pre[j] : ~KeyT(0);
    warp_bitonic_regs<EPL, KeyT>(v, lane);
#pragma unroll
    for (int j = 0; j < EPL; ++j)
        if (j * 32 < k) emit_sorted(a, r, v[j], j * 32 + lane < k, lane);
}

// a warp per centre: its candidate keys sorted, its kept pairs written into its output row
template <class KeyT>
__global__ void __launch_bounds__(kRagWarps * 32) ragged_nbr_emit_kernel(RaggedArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];  // [warps][sort_cap] keys of long rows
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    KeyT* list = reinterpret_cast<KeyT*>(smem_raw) + size_t(warp) * a.sort_cap;
    const KeyT* keys = static_cast<const KeyT*>(a.keys);
    const int64_t n_warps = int64_t(gridDim.x) * kRagWarps;
    for (int64_t row = int64_t(blockIdx.x) * kRagWarps + warp; row < a.n_atoms; row += n_warps) {
        const KeyT* src = keys + size_t(row) * a.row_cap;
        KeyT pre[4];  // the row's first 128 key slots, loaded with its count
#pragma unroll
        for (int j = 0; j < 4; ++j) pre[j] = j * 32 + lane < a.row_cap ? src[j * 32 + lane] : ~KeyT(0);
        const int k = min(a.n_keys[row], a.row_cap);
        RowWriter<KeyT> r;
        r.hp = a.wrapped[row];
        r.row = int32_t(row);
        r.self = (KeyT(uint32_t(row)) << 12) | KeyT(uint32_t(pack_image4(0, 0, 0)));
        r.out = a.offsets[row];
        r.end = min(a.offsets[row + 1], a.e_cap);
        if (k <= 32) {
            sort_and_emit<1, KeyT>(a, r, pre, k, lane);
        } else if (k <= 64) {
            sort_and_emit<2, KeyT>(a, r, pre, k, lane);
        } else if (k <= 128) {
            sort_and_emit<4, KeyT>(a, r, pre, k, lane);
        } else {  // a long row: sorted in shared memory
            int n = 256;
            while (n < k) n <<= 1;
            for (int i = lane; i < n; i += 32) list[i] = i < k ? src[i] : ~KeyT(0);
            __syncwarp();
            warp_bitonic_sort(list, n, lane);
            for (int base = 0; base < k; base += 32)
                emit_sorted(a, r, list[min(base + lane, k - 1)], base + lane < k, lane);
            __syncwarp();
        }
    }
}

__global__ void copy_wrapped_kernel(const float4* __restrict__ src, int64_t n, float* __restrict__ dst) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const float4 v = src[i];
        dst[3 * i] = v.x;
        dst[3 * i + 1] = v.y;
        dst[3 * i + 2] = v.z;
    }
}

// float64 model positions of a float64 build (fixed_capacity_builder.py:464
// _float64_prologue_kernel): the float32 wrap of the rounded coordinates gives
// the whole lattice vectors w, removed from the float64 coordinates with the
// float64 cell: out = p - ((w0 c[0] + w1 c[1]) + w2 c[2]), rounded per operation
struct Cell64 {
    double c[9];
};

__global__ void model_positions_f64_kernel(const double* __restrict__ p, int64_t n, Cell9 cell, Cell64 cell64,
                                           double* __restrict__ out) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const double x = p[3 * i], y = p[3 * i + 1], z = p[3 * i + 2];
        float3 w, f;
        int3 wr;
        wrap_atom(make_float3(float(x), float(y), float(z)), cell, w, wr, f);
        const double v0 = double(wr.x), v1 = double(wr.y), v2 = double(wr.z);
        const double* c = cell64.c;
        out[3 * i] = __dsub_rn(x, __dadd_rn(__dadd_rn(__dmul_rn(v0, c[0]), __dmul_rn(v1, c[3])), __dmul_rn(v2, c[6])));
        out[3 * i + 1] =
            __dsub_rn(y, __dadd_rn(__dadd_rn(__dmul_rn(v0, c[1]), __dmul_rn(v1, c[4])), __dmul_rn(v2, c[7])));
        out[3 * i + 2] =
            __dsub_rn(z, __dadd_rn(__dadd_rn(__dmul_rn(v0, c[2]), __dmul_rn(v1, c[5])), __dmul_rn(v2, c[8])));
    }
}

// the edge-vector override of exact-rc loop padding (fixed_capacity_builder.py:324
// _pad_self_loops_kernel, HAS_OVERRIDE): the padded rows' vector, 0 on the real rows
__global__ void pad_vector_override_kernel(const int64_t* __restrict__ n_edges, int64_t e_capacity, float3 v,
                                           float* __restrict__ out) {
    const int64_t total = *n_edges < e_capacity ? *n_edges : e_capacity;
    for (int64_t r = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; r < e_capacity; r += int64_t(gridDim.x) * blockDim.x) {
        const bool pad = r >= total;
        out[3 * r] = pad ? v.x : 0.f;
        out[3 * r + 1] = pad ? v.y : 0.f;
        out[3 * r + 2] = pad ? v.z : 0.f;
    }
}

// ------------------------------------------------------------------ host

inline size_t align_up(size_t x) { return (x + 255) & ~size_t(255); }


inline bool make_grid(const float* cell_host, double cutoff, Grid& g) {
    double c[9];
    for (int k = 0; k < 9; ++k) c[k] = cell_host[k];
    const double cross[3][3] = {
        {c[4] * c[8] - c[5] * c[7], c[5] * c[6] - c[3] * c[8], c[3] * c[7] - c[4] * c[6]},
        {c[7] * c[2] - c[8] * c[1], c[8] * c[0] - c[6] * c[2], c[6] * c[1] - c[7] * c[0]},
        {c[1] * c[5] - c[2] * c[4], c[2] * c[3] - c[0] * c[5], c[0] * c[4] - c[1] * c[3]},
    };
    const double vol = fabs(c[0] * cross[0][0] + c[1] * cross[0][1] + c[2] * cross[0][2]);
    if (!(vol > 0) || !(cutoff > 0)) return false;
    int64_t total = 1;
    for (int k = 0; k < 3; ++k) {
        const double area = sqrt(cross[k][0] * cross[k][0] + cross[k][1] * cross[k][1] + cross[k][2] * cross[k][2]);
        const double h = vol / area;  // perpendicular height along axis k
        int n = int(floor(h / cutoff));
        if (n < 1) n = 1;
        if (n > 256) n = 256;
        g.n[k] = n;
        g.s[k] = int(ceil(cutoff * n / h * (1.0 + 1e-6)));
        if (g.s[k] > 5) return false;  // at most (2 * 5 + 1)^3 neighbour (cell, image) pairs
        total *= n;
    }
    g.ncells = int(total);
    return true;
}

inline bool make_cell(const float* cell_host, Cell9& cell) {
    double c[9];
    for (int k = 0; k < 9; ++k) c[k] = cell_host[k];
    const double det = c[0] * (c[4] * c[8] - c[5] * c[7]) - c[1] * (c[3] * c[8] - c[5] * c[6]) +
                       c[2] * (c[3] * c[7] - c[4] * c[6]);
    if (!(fabs(det) > 0)) return false;
    const double inv[9] = {
        (c[4] * c[8] - c[5] * c[7]) / det, (c[2] * c[7] - c[1] * c[8]) / det, (c[1] * c[5] - c[2] * c[4]) / det,
        (c[5] * c[6] - c[3] * c[8]) / det, (c[0] * c[8] - c[2] * c[6]) / det, (c[2] * c[3] - c[0] * c[5]) / det,
        (c[3] * c[7] - c[4] * c[6]) / det, (c[1] * c[6] - c[0] * c[7]) / det, (c[0] * c[4] - c[1] * c[3]) / det,
    };
    for (int k = 0; k < 9; ++k) {
        cell.c[k] = cell_host[k];
        cell.inv[k] = float(inv[k]);
    }
    return true;
}

struct CellWorkspace {
    float4* wrapped;
    int32_t* atom_cell;
    int32_t* atom_slot;
    int32_t* cell_count;   // [R*ncells + 1]
    int32_t* cell_start;   // [R*ncells + 1]
    int32_t* cell_atoms;
    float4* cell_pos;
    void* scan_temp;
    size_t scan_bytes;
};

inline size_t scan_temp_bytes(int64_t items) {
    size_t bytes = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, bytes, (const int32_t*)nullptr, (int32_t*)nullptr, int(items));
    return bytes;
}

inline size_t cell_workspace_bytes(int64_t atoms, int64_t cells) {
    return align_up(sizeof(float4) * atoms) + 2 * align_up(sizeof(int32_t) * atoms) +
           2 * align_up(sizeof(int32_t) * (cells + 1)) + align_up(sizeof(int32_t) * atoms) +
           align_up(sizeof(float4) * atoms) + align_up(scan_temp_bytes(cells + 1));
}

inline CellWorkspace carve(void* ws, int64_t atoms, int64_t cells) {
    CellWorkspace w{};
    char* p = static_cast<char*>(ws);
    w.wrapped = reinterpret_cast<float4*>(p); p += align_up(sizeof(float4) * atoms);
    w.atom_cell = reinterpret_cast<int32_t*>(p); p += align_up(sizeof(int32_t) * atoms);
    w.atom_slot = reinterpret_cast<int32_t*>(p); p += align_up(sizeof(int32_t) * atoms);
    w.cell_count = reinterpret_cast<int32_t*>(p); p += align_up(sizeof(int32_t) * (cells + 1));
    w.cell_start = reinterpret_cast<int32_t*>(p); p += align_up(sizeof(int32_t) * (cells + 1));
    w.cell_atoms = reinterpret_cast<int32_t*>(p); p += align_up(sizeof(int32_t) * atoms);
    w.cell_pos = reinterpret_cast<float4*>(p); p += align_up(sizeof(float4) * atoms);
    w.scan_temp = p;
    w.scan_bytes = scan_temp_bytes(cells + 1);
    return w;
}

inline int list_cap_for(int32_t bmax) { return bmax < 32 ? 32 : (bmax > 1024 ? 1024 : bmax); }

// bin + scan + scatter: the atoms grouped by cell
inline fmd_status build_cells(const float* positions, int64_t n_atoms, int32_t n_systems, const Cell9& cell,
                              const Grid& grid, const CellWorkspace& w, int32_t* flags, cudaStream_t s) {
    const int64_t atoms = n_atoms * n_systems;
    const int64_t cells = int64_t(grid.ncells) * n_systems;
    cudaError_t err = cudaMemsetAsync(w.cell_count, 0, sizeof(int32_t) * (cells + 1), s);
    if (err != cudaSuccess) return record_cuda_error(err);
    const int threads = 256;
    cell_bin_kernel<<<grid_for(atoms, threads), threads, 0, s>>>(positions, n_atoms, n_systems, cell, grid,
                                                                  w.wrapped, w.atom_cell, w.atom_slot,
                                                                  w.cell_count, flags);
    fmd_status st = check_launch();
    if (st != FMD_OK) return st;
    size_t bytes = w.scan_bytes;
    err = cub::DeviceScan::ExclusiveSum(w.scan_temp, bytes, w.cell_count, w.cell_start, int(cells + 1), s);
    if (err != cudaSuccess) return record_cuda_error(err);
    cell_scatter_kernel<<<grid_for(atoms, threads), threads, 0, s>>>(atoms, w.wrapped, w.atom_cell, w.atom_slot,
                                                                      w.cell_start, w.cell_atoms, w.cell_pos);
    return check_launch();
}

// bin + scan + scatter + query into a candidate matrix
inline fmd_status run_cell_list(const float* positions, int64_t n_atoms, int32_t n_systems, const Cell9& cell,
                                const Grid& grid, float cutoff, int32_t bmax, int32_t* nbr, int32_t* shift,
                                int32_t* count, const CellWorkspace& w, int32_t* flags, cudaStream_t s) {
    const int64_t atoms = n_atoms * n_systems;
    const int64_t cells = int64_t(grid.ncells) * n_systems;
    const int threads = 256;
    fmd_status st = build_cells(positions, n_atoms, n_systems, cell, grid, w, flags, s);
    if (st != FMD_OK) return st;
    QueryArgs q{};
    q.cell_start = w.cell_start;
    q.cell_atoms = w.cell_atoms;
    q.cell_pos = w.cell_pos;
    q.n_atoms = n_atoms;
    q.n_systems = n_systems;
    q.cell = cell;
    q.grid = grid;
    q.cutoff = cutoff;
    q.bmax = bmax;
    q.list_cap = list_cap_for(bmax);
    q.off_cap = (2 * grid.s[0] + 1) * (2 * grid.s[1] + 1) * (2 * grid.s[2] + 1);
    q.nbr_out = nbr;
    q.shift_out = shift;
    q.count_out = count;
    q.flags = flags;
    const size_t smem = query_smem(q.list_cap, q.off_cap);
    if (smem > 227 * 1024) return FMD_ERR_UNSUPPORTED;
    if ((st = grant_dynamic_smem(reinterpret_cast<const void*>(cell_query_kernel), smem)) != FMD_OK) return st;
    const int qgrid = int(cells < int64_t(kNumSMs) * 16 ? cells : int64_t(kNumSMs) * 16);
    cell_query_kernel<<<qgrid, kQueryWarps * 32, smem, s>>>(q);
    if ((st = check_launch()) != FMD_OK) return st;
    cand_fill_kernel<<<grid_for(atoms * bmax, threads), threads, 0, s>>>(atoms, bmax, int32_t(atoms), nbr, shift,
                                                                         count);
    return check_launch();
}

}  // namespace fmd

using namespace fmd;

extern "C" {

fmd_status fmd_cell_list_workspace_bytes(const float* cell_host, float cutoff, int64_t n_atoms,
                                         int32_t n_systems, size_t* bytes) {
    Grid g{};
    if (cell_host == nullptr || bytes == nullptr || n_atoms < 1 || n_systems < 1 ||
        !make_grid(cell_host, cutoff, g))
        return FMD_ERR_INVALID_ARGUMENT;
    *bytes = cell_workspace_bytes(n_atoms * n_systems, int64_t(g.ncells) * n_systems);
    return FMD_OK;
}

fmd_status fmd_candidates_build(const float* positions, const float* cell_host, int64_t n_atoms,
                                int32_t n_systems, float candidate_cutoff, int32_t bmax,
                                int32_t* cand_nbr, int32_t* cand_shift, int32_t* cand_count,
                                float* ref_positions, int32_t* ref_wraps, int32_t* wrap_delta,
                                void* workspace, size_t workspace_bytes, int32_t* flags, void* stream) {
    Cell9 cell{};
    Grid grid{};
    if (positions == nullptr || cand_nbr == nullptr || cand_shift == nullptr || cand_count == nullptr ||
        n_atoms < 1 || n_systems < 1 || bmax < 1 || !make_cell(cell_host, cell) ||
        !make_grid(cell_host, candidate_cutoff, grid) || int64_t(n_atoms) * n_systems >= (int64_t(1) << 31) ||
        n_atoms >= (int64_t(1) << 33))
        return FMD_ERR_INVALID_ARGUMENT;
    const int64_t atoms = n_atoms * n_systems;
    const int64_t cells = int64_t(grid.ncells) * n_systems;
    if (workspace == nullptr || workspace_bytes < cell_workspace_bytes(atoms, cells)) return FMD_ERR_WORKSPACE;
    cudaStream_t s = as_stream(stream);
    const CellWorkspace w = carve(workspace, atoms, cells);
    if (ref_positions != nullptr && ref_wraps != nullptr && wrap_delta != nullptr) {
        refresh_reference_kernel<<<grid_for(atoms, 256), 256, 0, s>>>(positions, atoms, cell, ref_positions,
                                                                       ref_wraps, wrap_delta);
        fmd_status st = check_launch();
        if (st != FMD_OK) return st;
    }
    return run_cell_list(positions, n_atoms, n_systems, cell, grid, candidate_cutoff, bmax, cand_nbr, cand_shift,
                         cand_count, w, flags, s);
}

fmd_status fmd_refilter_workspace_bytes(int64_t n_atoms, int32_t n_systems, size_t* bytes) {
    if (bytes == nullptr || n_atoms < 1 || n_systems < 1) return FMD_ERR_INVALID_ARGUMENT;
    const int64_t atoms = n_atoms * n_systems;
    *bytes = 2 * align_up(sizeof(int32_t) * atoms) + align_up(sizeof(int32_t) * n_systems);
    return FMD_OK;
}

// largest system the re-filter holds in shared memory (every CTA of a system's cluster stages it)
static int64_t refilter_smem_bytes(int64_t n_atoms) {
    return int64_t(sizeof(float3) + sizeof(int3) + 2 * sizeof(int32_t)) * n_atoms + 4;
}

fmd_status fmd_refilter_edges(const float* positions, const float* cell_host, int64_t n_atoms, int32_t n_systems,
                              const float* ref_positions, const int32_t* ref_wraps, const int32_t* cand_nbr,
                              const int32_t* cand_shift, const int32_t* cand_count, int32_t bmax, float cutoff,
                              float skin, int64_t e_capacity, const int32_t* pad_image_host,
                              int32_t minimum_image, float* wrapped, int32_t* wrap_delta, int32_t* edge_index, float* edge_image, int64_t* recv_off,
                              int64_t* send_off, int32_t* send_perm, int64_t* n_edges, float* max_displacement,
                              void* workspace, size_t workspace_bytes, int32_t* flags, void* stream) {
    Cell9 cell{};
    if (positions == nullptr || ref_positions == nullptr || ref_wraps == nullptr || cand_nbr == nullptr ||
        cand_shift == nullptr || cand_count == nullptr || wrapped == nullptr || wrap_delta == nullptr ||
        edge_index == nullptr || edge_image == nullptr || recv_off == nullptr || send_off == nullptr ||
        send_perm == nullptr || n_edges == nullptr || max_displacement == nullptr || flags == nullptr ||
        n_atoms < 1 || n_systems < 1 || bmax < 1 || e_capacity < 0 || !make_cell(cell_host, cell) ||
        int64_t(n_atoms) * n_systems >= (int64_t(1) << 31) || e_capacity >= (int64_t(1) << 31))
        return FMD_ERR_INVALID_ARGUMENT;
    const int64_t smem = refilter_smem_bytes(n_atoms);
    if (smem > 200 * 1024) return FMD_ERR_UNSUPPORTED;  // per-system atoms beyond shared memory
    size_t need = 0;
    fmd_refilter_workspace_bytes(n_atoms, n_systems, &need);
    if (workspace == nullptr || workspace_bytes < need) return FMD_ERR_WORKSPACE;
    const int64_t atoms = n_atoms * n_systems;
    char* ws = static_cast<char*>(workspace);
    RefilterArgs a{};
    a.positions = positions;
    a.cell = cell;
    a.ref_pos = ref_positions;
    a.ref_wraps = ref_wraps;
    a.cand_nbr = cand_nbr;
    a.cand_shift = cand_shift;
    a.cand_count = cand_count;
    a.n_atoms = n_atoms;
    a.n_systems = n_systems;
    a.bmax = bmax;
    a.cutoff2 = cutoff * cutoff;
    a.skin_limit = skin + 1.0e-6f;
    a.minimum_image = minimum_image;
    a.e_cap = e_capacity;
    for (int k = 0; k < 3; ++k) a.pad_image[k] = pad_image_host ? pad_image_host[k] : 0;
    a.wrapped = wrapped;
    a.wrap_delta = wrap_delta;
    a.counts = reinterpret_cast<int32_t*>(ws); ws += align_up(sizeof(int32_t) * atoms);
    a.local_off = reinterpret_cast<int32_t*>(ws); ws += align_up(sizeof(int32_t) * atoms);
    a.sys_total = reinterpret_cast<int32_t*>(ws);
    a.max_disp = max_displacement;
    a.edge_index = edge_index;
    a.edge_image = edge_image;
    a.recv_off = recv_off;
    a.send_off = send_off;
    a.send_perm = send_perm;
    a.n_edges = n_edges;
    a.flags = flags;
    cudaStream_t s = as_stream(stream);
    const size_t smem_count = (sizeof(float3) + sizeof(int3)) * size_t(n_atoms);
    const size_t smem_mat = size_t(smem);
    const int grid = n_systems * kRefCluster;  // a cluster of kRefCluster CTAs per system
    fmd_status st0 = grant_dynamic_smem(reinterpret_cast<const void*>(refilter_count_kernel), smem_count);
    if (st0 != FMD_OK) return st0;
    st0 = grant_dynamic_smem(reinterpret_cast<const void*>(refilter_materialize_kernel), smem_mat);
    if (st0 != FMD_OK) return st0;
    refilter_count_kernel<<<grid, kRefThreads, smem_count, s>>>(a);
    fmd_status st = check_launch();
    if (st != FMD_OK) return st;
    refilter_materialize_kernel<<<grid, kRefThreads, smem_mat, s>>>(a);
    return check_launch();
}

// ---------------------------------------------------------------------------
// Allocation-free re-filter. Some callers cannot allocate device memory at
// all: a C or Fortran MD host that links this library but has no CUDA
// allocator or memory pool of its own to hand out a workspace, or a caller
// running inside another framework whose memory manager owns every byte of
// the device. For them the re-filter's scratch (per-atom edge counts and
// offsets, per-system totals) lives in this file-scope device array instead
// of a caller workspace. It is 1 MiB, held by every GPU that loads the
// library until the process exits, and serves up to 126,976 atoms in total
// (n_atoms * n_systems, with up to 4,096 systems); larger calls are refused
// with FMD_ERR_WORKSPACE before anything is launched.
// ---------------------------------------------------------------------------

constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;
constexpr int64_t kNoAllocMaxAtoms = 126976;   // n_atoms * n_systems
constexpr int32_t kNoAllocMaxSystems = 4096;
constexpr int kNoAllocMaxDevices = 64;
// the largest admitted call fits the array: 2 x 507,904 B of counts/offsets + 16,384 B of totals
static_assert(2 * ((4 * kNoAllocMaxAtoms + 255) / 256 * 256) + (4 * kNoAllocMaxSystems + 255) / 256 * 256 <=
                  int64_t(kNoAllocScratchBytes),
              "the allocation-free re-filter limits must fit its static scratch");

static __device__ __align__(256) unsigned char g_refilter_scratch[kNoAllocScratchBytes];

// Host code must not pass g_refilter_scratch itself to a kernel: on the host
// that name is only a stand-in for the device symbol. The device address is
// looked up once per device (with that device current) and cached.
static void* g_refilter_scratch_ptr[kNoAllocMaxDevices] = {};
static std::mutex g_refilter_scratch_mutex;

static fmd_status refilter_scratch_address(void** out) {
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return record_cuda_error(err);
    if (device < 0 || device >= kNoAllocMaxDevices) return FMD_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_refilter_scratch_mutex);
    if (g_refilter_scratch_ptr[device] == nullptr) {
        void* address = nullptr;
        err = cudaGetSymbolAddress(&address, g_refilter_scratch);
        if (err != cudaSuccess) return record_cuda_error(err);
        g_refilter_scratch_ptr[device] = address;
    }
    *out = g_refilter_scratch_ptr[device];
    return FMD_OK;
}

static size_t ragged_scan_bytes(int64_t n_atoms) {
    size_t cub_bytes = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, cub_bytes, (const int64_t*)nullptr, (int64_t*)nullptr, int(n_atoms + 1));
    return cub_bytes;
}

// candidate keys of the ragged list: 32-bit (atom << 12 | image) below 2^20 atoms, else 64-bit
static size_t ragged_key_bytes(int64_t n_atoms) { return n_atoms <= (int64_t(1) << 20) ? 4 : 8; }

fmd_status fmd_neighbor_list_workspace_bytes(const float* cell_host, float cutoff, int64_t n_atoms,
                                             int32_t bmax, size_t* bytes) {
    Grid g{};
    if (cell_host == nullptr || bytes == nullptr || n_atoms < 1 || bmax < 1 ||
        !make_grid(cell_host, cutoff + 1e-6f, g))
        return FMD_ERR_INVALID_ARGUMENT;
    *bytes = cell_workspace_bytes(n_atoms, g.ncells) + align_up(sizeof(int64_t) * (n_atoms + 1)) +
             align_up(sizeof(int32_t) * n_atoms) + align_up(ragged_key_bytes(n_atoms) * size_t(n_atoms) * (bmax + 1)) +
             align_up(ragged_scan_bytes(n_atoms));
    return FMD_OK;
}

// A candidate closer than rc - delta passes the eager path's |(q - p) + image @ cell| < rc. Both
// distances round each difference component at most twice, on magnitudes of at most
// (3 + reach) C + 2 rc (C: the largest coordinate of a wrapped position, the image shift at most
// reach C), so they differ by less than 2^-23 ((3 + reach) C + 5 rc); delta is 8 times that.
static float eager_shell_lo2(const float* cell_host, const Grid& g, float cutoff) {
    double c_max = 0.0;
    for (int c = 0; c < 3; ++c)
        c_max = fmax(c_max, fabs(double(cell_host[c])) + fabs(double(cell_host[3 + c])) + fabs(double(cell_host[6 + c])));
    const int reach = std::max(g.s[0], std::max(g.s[1], g.s[2]));
    const double delta = ldexp((3.0 + reach) * c_max + 5.0 * double(cutoff), -20);
    const double lo = double(cutoff) - delta;
    if (!(lo > 0.0)) return 0.f;
    return nextafterf(float(lo * lo), 0.f);
}

fmd_status fmd_neighbor_list(const float* positions, const float* cell_host, int64_t n_atoms, float cutoff,
                             int32_t bmax, int64_t e_capacity, float* wrapped, int64_t* center, int64_t* neighbor,
                             int32_t* images, float* dist, int64_t* offsets, void* workspace,
                             size_t workspace_bytes, int32_t* flags, void* stream) {
    Cell9 cell{};
    Grid grid{};
    const float cand_cut = cutoff + 1e-6f;  // candidates at rc + 1e-6 (gpu_graph_builder.py:161)
    if (positions == nullptr || center == nullptr || neighbor == nullptr || images == nullptr ||
        dist == nullptr || offsets == nullptr || n_atoms < 1 || bmax < 1 || e_capacity < 0 ||
        !make_cell(cell_host, cell) || !make_grid(cell_host, cand_cut, grid) || n_atoms >= (int64_t(1) << 31))
        return FMD_ERR_INVALID_ARGUMENT;
    if (bmax >= kRagMaxList) return FMD_ERR_UNSUPPORTED;  // more than 2047 candidates per centre
    size_t need = 0;
    if (fmd_neighbor_list_workspace_bytes(cell_host, cutoff, n_atoms, bmax, &need) != FMD_OK)
        return FMD_ERR_INVALID_ARGUMENT;
    if (workspace == nullptr || workspace_bytes < need) return FMD_ERR_WORKSPACE;
    cudaStream_t s = as_stream(stream);
    char* p = static_cast<char*>(workspace);
    const CellWorkspace w = carve(p, n_atoms, grid.ncells);
    p += cell_workspace_bytes(n_atoms, grid.ncells);
    int64_t* counts64 = reinterpret_cast<int64_t*>(p); p += align_up(sizeof(int64_t) * (n_atoms + 1));
    int32_t* n_keys = reinterpret_cast<int32_t*>(p); p += align_up(sizeof(int32_t) * n_atoms);
    const bool narrow_keys = ragged_key_bytes(n_atoms) == 4;
    void* keys = p; p += align_up(ragged_key_bytes(n_atoms) * size_t(n_atoms) * (bmax + 1));
    void* cub_temp = p;
    size_t cub_bytes = ragged_scan_bytes(n_atoms);
    fmd_status st = build_cells(positions, n_atoms, 1, cell, grid, w, flags, s);
    if (st != FMD_OK) return st;
    RaggedArgs a{};
    a.cell_start = w.cell_start;
    a.cell_atoms = w.cell_atoms;
    a.cell_pos = w.cell_pos;
    a.wrapped = w.wrapped;
    a.cell = cell;
    a.grid = grid;
    a.cand_cut = cand_cut;
    a.cutoff = cutoff;
    a.lo2 = eager_shell_lo2(cell_host, grid, cutoff);
    a.bmax = bmax;
    a.row_cap = bmax + 1;
    a.sort_cap = 0;
    if (a.row_cap > 128) {
        a.sort_cap = 256;
        while (a.sort_cap < a.row_cap) a.sort_cap <<= 1;
    }
    a.off_cap = (2 * grid.s[0] + 1) * (2 * grid.s[1] + 1) * (2 * grid.s[2] + 1);
    a.keys = keys;
    a.n_keys = n_keys;
    a.counts = counts64;
    a.offsets = offsets;
    a.n_atoms = n_atoms;
    a.e_cap = e_capacity;
    a.center = center;
    a.neighbor = neighbor;
    a.images = images;
    a.dist = dist;
    a.flags = flags;
    const size_t key_bytes = ragged_key_bytes(n_atoms);
    const size_t hood = sizeof(int32_t) * (3 * size_t(a.off_cap) + 1) + sizeof(float) * 3 * size_t(a.off_cap);
    const size_t collect_smem = (sizeof(float4) + key_bytes) * kRagStage + 2 * sizeof(int32_t) * kRagHome + hood + 16;
    const size_t emit_smem = key_bytes * size_t(kRagWarps) * a.sort_cap;
    const void* collect = narrow_keys ? reinterpret_cast<const void*>(ragged_nbr_collect_kernel<uint32_t>)
                                      : reinterpret_cast<const void*>(ragged_nbr_collect_kernel<uint64_t>);
    const void* emit = narrow_keys ? reinterpret_cast<const void*>(ragged_nbr_emit_kernel<uint32_t>)
                                   : reinterpret_cast<const void*>(ragged_nbr_emit_kernel<uint64_t>);
    if ((st = grant_dynamic_smem(collect, collect_smem)) != FMD_OK || (st = grant_dynamic_smem(emit, emit_smem)) != FMD_OK)
        return st;
    const int qgrid = grid.ncells < kNumSMs * 16 ? grid.ncells : kNumSMs * 16;
    if (narrow_keys)
        ragged_nbr_collect_kernel<uint32_t><<<qgrid, kRagWarps * 32, collect_smem, s>>>(a);
    else
        ragged_nbr_collect_kernel<uint64_t><<<qgrid, kRagWarps * 32, collect_smem, s>>>(a);
    if ((st = check_launch()) != FMD_OK) return st;
    cudaError_t err = cudaMemsetAsync(counts64 + n_atoms, 0, sizeof(int64_t), s);
    if (err != cudaSuccess) return record_cuda_error(err);
    err = cub::DeviceScan::ExclusiveSum(cub_temp, cub_bytes, counts64, offsets, int(n_atoms + 1), s);
    if (err != cudaSuccess) return record_cuda_error(err);
    const int64_t egrid64 = (n_atoms + kRagWarps - 1) / kRagWarps;
    const int egrid = int(egrid64 < int64_t(kNumSMs) * 64 ? egrid64 : int64_t(kNumSMs) * 64);
    if (narrow_keys)
        ragged_nbr_emit_kernel<uint32_t><<<egrid, kRagWarps * 32, emit_smem, s>>>(a);
    else
        ragged_nbr_emit_kernel<uint64_t><<<egrid, kRagWarps * 32, emit_smem, s>>>(a);
    if ((st = check_launch()) != FMD_OK) return st;
    if (wrapped != nullptr) {
        const int threads = 256;
        copy_wrapped_kernel<<<grid_for(n_atoms, threads), threads, 0, s>>>(w.wrapped, n_atoms, wrapped);
        if ((st = check_launch()) != FMD_OK) return st;
    }
    return FMD_OK;
}

fmd_status fmd_refilter_edges_noalloc(const float* positions, const float* cell_host, int64_t n_atoms,
                                      int32_t n_systems, const float* ref_positions, const int32_t* ref_wraps,
                                      const int32_t* cand_nbr, const int32_t* cand_shift,
                                      const int32_t* cand_count, int32_t bmax, float cutoff, float skin,
                                      int64_t e_capacity, const int32_t* pad_image_host, int32_t minimum_image,
                                      float* wrapped, int32_t* wrap_delta, int32_t* edge_index, float* edge_image,
                                      int64_t* recv_off, int64_t* send_off, int32_t* send_perm, int64_t* n_edges,
                                      float* max_displacement, int32_t* flags, void* stream) {
    if (n_atoms < 1 || n_systems < 1) return FMD_ERR_INVALID_ARGUMENT;
    if (n_systems > kNoAllocMaxSystems || n_atoms > kNoAllocMaxAtoms / n_systems) return FMD_ERR_WORKSPACE;
    size_t need = 0;
    fmd_status st = fmd_refilter_workspace_bytes(n_atoms, n_systems, &need);
    if (st != FMD_OK) return st;
    if (need > kNoAllocScratchBytes) return FMD_ERR_WORKSPACE;  // beyond the static scratch
    void* scratch = nullptr;
    if ((st = refilter_scratch_address(&scratch)) != FMD_OK) return st;
    // Every field of the scratch is written before it is read within the call, so the previous
    // call's contents need no clearing.
    return fmd_refilter_edges(positions, cell_host, n_atoms, n_systems, ref_positions, ref_wraps, cand_nbr,
                              cand_shift, cand_count, bmax, cutoff, skin, e_capacity, pad_image_host, minimum_image,
                              wrapped, wrap_delta, edge_index, edge_image, recv_off, send_off, send_perm, n_edges,
                              max_displacement, scratch, kNoAllocScratchBytes, flags, stream);
}

fmd_status fmd_pad_vector_override(const int64_t* n_edges, int64_t e_capacity, const float* pad_vector_host,
                                   float* edge_vec_override, void* stream) {
    if (e_capacity < 0 || pad_vector_host == nullptr) return FMD_ERR_INVALID_ARGUMENT;
    if (e_capacity == 0) return FMD_OK;
    if (n_edges == nullptr || edge_vec_override == nullptr) return FMD_ERR_INVALID_ARGUMENT;
    constexpr int threads = 256;
    const float3 v = make_float3(pad_vector_host[0], pad_vector_host[1], pad_vector_host[2]);
    pad_vector_override_kernel<<<grid_for(e_capacity, threads), threads, 0, as_stream(stream)>>>(n_edges, e_capacity, v,
                                                                                              edge_vec_override);
    return check_launch();
}

fmd_status fmd_model_positions_f64(const double* positions, int64_t n_atoms, const float* cell_host,
                                   const double* cell64_host, double* out, void* stream) {
    if (n_atoms < 0 || cell_host == nullptr || cell64_host == nullptr) return FMD_ERR_INVALID_ARGUMENT;
    if (n_atoms == 0) return FMD_OK;
    if (positions == nullptr || out == nullptr) return FMD_ERR_INVALID_ARGUMENT;
    Cell9 cell;
    if (!make_cell(cell_host, cell)) return FMD_ERR_INVALID_ARGUMENT;
    Cell64 cell64;
    for (int k = 0; k < 9; ++k) cell64.c[k] = cell64_host[k];
    constexpr int threads = 256;
    model_positions_f64_kernel<<<grid_for(n_atoms, threads), threads, 0, as_stream(stream)>>>(positions, n_atoms, cell,
                                                                                           cell64, out);
    return check_launch();
}

}  // extern "C"
