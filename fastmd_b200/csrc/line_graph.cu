// MatRIS bond graph on the device: reverse-edge pairing (directed <->
// undirected edges) and the line graph of ordered bond pairs (triplets)
// around each centre atom (fastmd/graph/gpu_graph_builder.py:217 _build_d2u,
// :511 _build_line_graph).
//
// Pairing. Every directed edge e = (c, n, image) has the forward key
// (c N + n) V + code(image) and the reverse key (n N + c) V + code(-image),
// V = 21^3, code in radix 21 with offset 10 (images within +-10). The forward
// keys are sorted (a CUB radix sort of (key, edge) pairs, skipped when the
// edges are already in key order), each edge's reverse key is located by a
// lower-bound search (clamped to the last edge), m(e) = min(e, pair(e)), and
// directed2undirected(e) = the rank of m(e) among the distinct minima (a
// scan of their marks); undirected2directed(u) = the smallest edge of u
// (atomicMin: order independent).
//
// Line graph. Short edges (dist < cutoff) are compacted in edge order
// (scan + scatter), stably sorted by centre unless already grouped by centre
// (keys past the short count sort last), the per-atom runs found by lower
// bound, and the k (k - 1) ordered pairs of an atom with k short edges
// numbered by an exclusive scan; row t of the triplet table is
// [atom, u(first), e(first), u(second), e(second)] with first = l / (k - 1),
// second = l % (k - 1) skipping first, l = t - pair_offset(atom). No host
// synchronisation: counts stay on the device, the triplet count is written
// to n_triplets and rows past t_capacity raise FMD_FLAG_TRIPLET_OVERFLOW.

#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>

#include "common.cuh"

namespace fmd {
namespace {

constexpr int kThreads = 256;
constexpr int64_t kMaxImage = 10;
constexpr int64_t kRadix = 2 * kMaxImage + 1;
constexpr int64_t kVolume = kRadix * kRadix * kRadix;

inline size_t align_up(size_t b) { return (b + 255) & ~size_t(255); }

__device__ __forceinline__ uint64_t pair_key(int64_t a, int64_t b, int64_t n_atoms, int64_t ix, int64_t iy,
                                             int64_t iz) {
    return uint64_t((a * n_atoms + b) * kVolume + (ix + kMaxImage) * kRadix * kRadix + (iy + kMaxImage) * kRadix +
                    (iz + kMaxImage));
}

__global__ void forward_keys_kernel(const int64_t* __restrict__ center, const int64_t* __restrict__ neighbor,
                                    const int32_t* __restrict__ images, int64_t n_edges, int64_t n_atoms,
                                    uint64_t* __restrict__ keys, int64_t* __restrict__ ids, int32_t* flags) {
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < n_edges; e += int64_t(gridDim.x) * blockDim.x) {
        int64_t c = center[e], n = neighbor[e];
        int64_t ix = images[3 * e], iy = images[3 * e + 1], iz = images[3 * e + 2];
        if (c < 0 || c >= n_atoms || n < 0 || n >= n_atoms || ix < -kMaxImage || ix > kMaxImage ||
            iy < -kMaxImage || iy > kMaxImage || iz < -kMaxImage || iz > kMaxImage) {
            raise_flag(flags, FMD_FLAG_INDEX_RANGE);
            c = c < 0 ? 0 : (c >= n_atoms ? n_atoms - 1 : c);
            n = n < 0 ? 0 : (n >= n_atoms ? n_atoms - 1 : n);
            ix = ix < -kMaxImage ? -kMaxImage : (ix > kMaxImage ? kMaxImage : ix);
            iy = iy < -kMaxImage ? -kMaxImage : (iy > kMaxImage ? kMaxImage : iy);
            iz = iz < -kMaxImage ? -kMaxImage : (iz > kMaxImage ? kMaxImage : iz);
        }
        keys[e] = pair_key(c, n, n_atoms, ix, iy, iz);
        ids[e] = e;
    }
}

template <typename K>
__device__ __forceinline__ int64_t lower_bound(const K* __restrict__ sorted, int64_t n, K key) {
    int64_t lo = 0, hi = n;
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (sorted[mid] < key)
            lo = mid + 1;
        else
            hi = mid;
    }
    return lo;
}

__global__ void reverse_pair_kernel(const int64_t* __restrict__ center, const int64_t* __restrict__ neighbor,
                                    const int32_t* __restrict__ images, int64_t n_edges, int64_t n_atoms,
                                    const uint64_t* __restrict__ sorted, const int64_t* __restrict__ sort_idx,
                                    int64_t* __restrict__ mins, int32_t* __restrict__ mark) {
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < n_edges; e += int64_t(gridDim.x) * blockDim.x) {
        int64_t c = center[e], n = neighbor[e];
        c = c < 0 ? 0 : (c >= n_atoms ? n_atoms - 1 : c);
        n = n < 0 ? 0 : (n >= n_atoms ? n_atoms - 1 : n);
        int64_t ix = -int64_t(images[3 * e]), iy = -int64_t(images[3 * e + 1]), iz = -int64_t(images[3 * e + 2]);
        ix = ix < -kMaxImage ? -kMaxImage : (ix > kMaxImage ? kMaxImage : ix);
        iy = iy < -kMaxImage ? -kMaxImage : (iy > kMaxImage ? kMaxImage : iy);
        iz = iz < -kMaxImage ? -kMaxImage : (iz > kMaxImage ? kMaxImage : iz);
        int64_t pos = lower_bound(sorted, n_edges, pair_key(n, c, n_atoms, ix, iy, iz));
        if (pos > n_edges - 1) pos = n_edges - 1;
        const int64_t pair = sort_idx != nullptr ? sort_idx[pos] : pos;
        const int64_t m = e < pair ? e : pair;
        mins[e] = m;
        mark[m] = 1;  // benign: every writer stores 1
    }
}

__global__ void undirected_kernel(const int64_t* __restrict__ mins, const int32_t* __restrict__ rank,
                                  const int32_t* __restrict__ mark, int64_t n_edges, int32_t* __restrict__ d2u,
                                  int32_t* __restrict__ u2d, int64_t* __restrict__ n_undirected) {
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < n_edges; e += int64_t(gridDim.x) * blockDim.x) {
        const int32_t u = rank[mins[e]];
        d2u[e] = u;
        atomicMin(u2d + u, int32_t(e));
        if (e == n_edges - 1) *n_undirected = int64_t(rank[e]) + mark[e];
    }
}

__global__ void fill_i32_kernel(int32_t* __restrict__ p, int64_t n, int32_t v) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        p[i] = v;
}

// ----------------------------------------------------------------- line graph

__global__ void short_flags_kernel(const float* __restrict__ dist, int64_t n_edges, float cutoff,
                                   int32_t* __restrict__ flag) {
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < n_edges; e += int64_t(gridDim.x) * blockDim.x)
        flag[e] = dist[e] < cutoff ? 1 : 0;
}

// short edges in edge order, their centres as sort keys (past the short count: keys that sort last)
__global__ void short_compact_kernel(const int32_t* __restrict__ flag, const int32_t* __restrict__ pos,
                                     const int64_t* __restrict__ center, int64_t n_edges, int64_t n_atoms,
                                     uint32_t* __restrict__ keys, int64_t* __restrict__ short_ids, int32_t* flags) {
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < n_edges; e += int64_t(gridDim.x) * blockDim.x) {
        const int64_t n_short = int64_t(pos[n_edges - 1]) + flag[n_edges - 1];
        if (e >= n_short) keys[e] = 0xFFFFFFFFu;  // slot e past the short edges
        if (flag[e]) {
            int64_t c = center[e];
            if (c < 0 || c >= n_atoms) {
                raise_flag(flags, FMD_FLAG_INDEX_RANGE);
                c = c < 0 ? 0 : n_atoms - 1;
            }
            keys[pos[e]] = uint32_t(c);
            short_ids[pos[e]] = e;
        }
    }
}

__global__ void atom_runs_kernel(const uint32_t* __restrict__ sorted_keys, int64_t n_edges, int64_t n_atoms,
                                 int64_t* __restrict__ offsets, int64_t* __restrict__ pair_counts) {
    for (int64_t a = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; a <= n_atoms; a += int64_t(gridDim.x) * blockDim.x) {
        const int64_t lo = lower_bound(sorted_keys, n_edges, uint32_t(a));
        offsets[a] = lo;
        if (a < n_atoms) {
            const int64_t k = lower_bound(sorted_keys, n_edges, uint32_t(a + 1)) - lo;
            pair_counts[a] = k * (k - 1);
        } else {
            pair_counts[a] = 0;
        }
    }
}

__global__ void triplets_kernel(const int64_t* __restrict__ offsets, const int64_t* __restrict__ pair_offsets,
                                const int64_t* __restrict__ short_ids, const int32_t* __restrict__ d2u,
                                int64_t n_atoms, int64_t t_capacity, int32_t* __restrict__ triplets,
                                int64_t* __restrict__ n_triplets, int32_t* flags) {
    const int64_t total = pair_offsets[n_atoms];
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        *n_triplets = total;
        if (total > t_capacity) raise_flag(flags, FMD_FLAG_TRIPLET_OVERFLOW);
    }
    const int64_t rows = total < t_capacity ? total : t_capacity;
    for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < rows; t += int64_t(gridDim.x) * blockDim.x) {
        // the last atom whose pair offset is <= t
        int64_t lo = 0, hi = n_atoms - 1;
        while (lo < hi) {
            const int64_t mid = (lo + hi + 1) >> 1;
            if (pair_offsets[mid] <= t)
                lo = mid;
            else
                hi = mid - 1;
        }
        const int64_t atom = lo;
        const int64_t local = t - pair_offsets[atom];
        const int64_t k = offsets[atom + 1] - offsets[atom];
        const int64_t first = local / (k - 1);
        const int64_t second_raw = local - first * (k - 1);
        const int64_t second = second_raw + (second_raw >= first ? 1 : 0);
        const int64_t e1 = short_ids[offsets[atom] + first], e2 = short_ids[offsets[atom] + second];
        int32_t* row = triplets + 5 * t;
        row[0] = int32_t(atom);
        row[1] = d2u[e1];
        row[2] = int32_t(e1);
        row[3] = d2u[e2];
        row[4] = int32_t(e2);
    }
}

struct PairLayout {
    size_t keys, sorted, ids, sort_idx, mark, rank, temp, total;
};

fmd_status pair_layout(int64_t n_edges, PairLayout* l) {
    size_t sort_temp = 0, scan_temp = 0;
    cudaError_t err = cub::DeviceRadixSort::SortPairs(nullptr, sort_temp, (const uint64_t*)nullptr,
                                                      (uint64_t*)nullptr, (const int64_t*)nullptr, (int64_t*)nullptr,
                                                      n_edges);
    if (err == cudaSuccess)
        err = cub::DeviceScan::ExclusiveSum(nullptr, scan_temp, (const int32_t*)nullptr, (int32_t*)nullptr, n_edges);
    if (err != cudaSuccess) return record_cuda_error(err);
    const size_t e = size_t(n_edges);
    l->keys = 0;
    l->sorted = l->keys + align_up(8 * e);
    l->ids = l->sorted + align_up(8 * e);
    l->sort_idx = l->ids + align_up(8 * e);
    l->mark = l->sort_idx + align_up(8 * e);
    l->rank = l->mark + align_up(4 * e);
    l->temp = l->rank + align_up(4 * e);
    l->total = l->temp + align_up(sort_temp > scan_temp ? sort_temp : scan_temp);
    return FMD_OK;
}

struct LineLayout {
    size_t flag, pos, keys, sorted_keys, ids, sorted_ids, offsets, pair_counts, pair_offsets, temp, total;
    size_t temp_bytes;
};

fmd_status line_layout(int64_t n_edges, int64_t n_atoms, LineLayout* l) {
    size_t sort_temp = 0, scan_temp = 0, scan64_temp = 0;
    cudaError_t err = cub::DeviceRadixSort::SortPairs(nullptr, sort_temp, (const uint32_t*)nullptr,
                                                      (uint32_t*)nullptr, (const int64_t*)nullptr, (int64_t*)nullptr,
                                                      n_edges);
    if (err == cudaSuccess)
        err = cub::DeviceScan::ExclusiveSum(nullptr, scan_temp, (const int32_t*)nullptr, (int32_t*)nullptr, n_edges);
    if (err == cudaSuccess)
        err = cub::DeviceScan::ExclusiveSum(nullptr, scan64_temp, (const int64_t*)nullptr, (int64_t*)nullptr,
                                            n_atoms + 1);
    if (err != cudaSuccess) return record_cuda_error(err);
    size_t temp = sort_temp > scan_temp ? sort_temp : scan_temp;
    temp = temp > scan64_temp ? temp : scan64_temp;
    const size_t e = size_t(n_edges), n1 = size_t(n_atoms) + 1;
    l->flag = 0;
    l->pos = l->flag + align_up(4 * e);
    l->keys = l->pos + align_up(4 * e);
    l->sorted_keys = l->keys + align_up(4 * e);
    l->ids = l->sorted_keys + align_up(4 * e);
    l->sorted_ids = l->ids + align_up(8 * e);
    l->offsets = l->sorted_ids + align_up(8 * e);
    l->pair_counts = l->offsets + align_up(8 * n1);
    l->pair_offsets = l->pair_counts + align_up(8 * n1);
    l->temp = l->pair_offsets + align_up(8 * n1);
    l->temp_bytes = temp;
    l->total = l->temp + align_up(temp);
    return FMD_OK;
}

}  // namespace
}  // namespace fmd

using namespace fmd;

extern "C" {

fmd_status fmd_reverse_pairs_workspace_bytes(int64_t n_edges, size_t* bytes) {
    if (bytes == nullptr || n_edges < 0 || n_edges >= (int64_t(1) << 31)) return FMD_ERR_INVALID_ARGUMENT;
    PairLayout l;
    fmd_status st = pair_layout(n_edges > 0 ? n_edges : 1, &l);
    if (st == FMD_OK) *bytes = l.total;
    return st;
}

fmd_status fmd_reverse_pairs(const int64_t* center, const int64_t* neighbor, const int32_t* images, int64_t n_edges,
                             int64_t n_atoms, int32_t presorted, void* workspace, size_t workspace_bytes,
                             int32_t* directed2undirected, int32_t* undirected2directed, int64_t* n_undirected,
                             int32_t* flags, void* stream) {
    if (n_edges < 0 || n_edges >= (int64_t(1) << 31) || n_atoms < 1 || n_undirected == nullptr ||
        n_atoms > int64_t(1) << 31 ||
        (n_edges > 0 && (center == nullptr || neighbor == nullptr || images == nullptr ||
                         directed2undirected == nullptr || undirected2directed == nullptr)))
        return FMD_ERR_INVALID_ARGUMENT;
    cudaStream_t s = as_stream(stream);
    if (n_edges == 0) {
        cudaError_t err = cudaMemsetAsync(n_undirected, 0, sizeof(int64_t), s);
        return err == cudaSuccess ? FMD_OK : record_cuda_error(err);
    }
    PairLayout l;
    fmd_status st = pair_layout(n_edges, &l);
    if (st != FMD_OK) return st;
    if (workspace == nullptr || workspace_bytes < l.total) return FMD_ERR_WORKSPACE;
    char* ws = static_cast<char*>(workspace);
    uint64_t* keys = reinterpret_cast<uint64_t*>(ws + l.keys);
    uint64_t* sorted = reinterpret_cast<uint64_t*>(ws + l.sorted);
    int64_t* ids = reinterpret_cast<int64_t*>(ws + l.ids);
    int64_t* sort_idx = reinterpret_cast<int64_t*>(ws + l.sort_idx);
    int32_t* mark = reinterpret_cast<int32_t*>(ws + l.mark);
    int32_t* rank = reinterpret_cast<int32_t*>(ws + l.rank);
    void* temp = ws + l.temp;
    size_t temp_bytes = workspace_bytes - l.temp;
    const int grid = grid_for(n_edges, kThreads);
    forward_keys_kernel<<<grid, kThreads, 0, s>>>(center, neighbor, images, n_edges, n_atoms, keys, ids, flags);
    if ((st = check_launch()) != FMD_OK) return st;
    cudaError_t err = cudaSuccess;
    if (!presorted) {
        err = cub::DeviceRadixSort::SortPairs(temp, temp_bytes, keys, sorted, ids, sort_idx, n_edges, 0, 64, s);
        if (err != cudaSuccess) return record_cuda_error(err);
    }
    err = cudaMemsetAsync(mark, 0, sizeof(int32_t) * size_t(n_edges), s);
    if (err != cudaSuccess) return record_cuda_error(err);
    // mins reuse the edge-id buffer (free after the sort)
    reverse_pair_kernel<<<grid, kThreads, 0, s>>>(center, neighbor, images, n_edges, n_atoms,
                                                  presorted ? keys : sorted, presorted ? nullptr : sort_idx, ids,
                                                  mark);
    if ((st = check_launch()) != FMD_OK) return st;
    err = cub::DeviceScan::ExclusiveSum(temp, temp_bytes, mark, rank, n_edges, s);
    if (err != cudaSuccess) return record_cuda_error(err);
    fill_i32_kernel<<<grid, kThreads, 0, s>>>(undirected2directed, n_edges, int32_t(n_edges));
    undirected_kernel<<<grid, kThreads, 0, s>>>(ids, rank, mark, n_edges, directed2undirected, undirected2directed,
                                                n_undirected);
    return check_launch();
}

fmd_status fmd_line_graph_workspace_bytes(int64_t n_edges, int64_t n_atoms, size_t* bytes) {
    if (bytes == nullptr || n_edges < 0 || n_edges >= (int64_t(1) << 31) || n_atoms < 1 ||
        n_atoms >= (int64_t(1) << 32) - 1)
        return FMD_ERR_INVALID_ARGUMENT;
    LineLayout l;
    fmd_status st = line_layout(n_edges > 0 ? n_edges : 1, n_atoms, &l);
    if (st == FMD_OK) *bytes = l.total;
    return st;
}

fmd_status fmd_line_graph(const int64_t* center, const float* dist, const int32_t* directed2undirected,
                          int64_t n_edges, int64_t n_atoms, float cutoff, int32_t presorted, int64_t t_capacity,
                          void* workspace, size_t workspace_bytes, int32_t* triplets, int64_t* n_triplets,
                          int32_t* flags, void* stream) {
    if (n_edges < 0 || n_edges >= (int64_t(1) << 31) || n_atoms < 1 || n_atoms >= (int64_t(1) << 32) - 1 ||
        t_capacity < 0 || n_triplets == nullptr || (t_capacity > 0 && triplets == nullptr) ||
        (n_edges > 0 && (center == nullptr || dist == nullptr || directed2undirected == nullptr)))
        return FMD_ERR_INVALID_ARGUMENT;
    cudaStream_t s = as_stream(stream);
    if (n_edges == 0) {
        cudaError_t err = cudaMemsetAsync(n_triplets, 0, sizeof(int64_t), s);
        return err == cudaSuccess ? FMD_OK : record_cuda_error(err);
    }
    LineLayout l;
    fmd_status st = line_layout(n_edges, n_atoms, &l);
    if (st != FMD_OK) return st;
    if (workspace == nullptr || workspace_bytes < l.total) return FMD_ERR_WORKSPACE;
    char* ws = static_cast<char*>(workspace);
    int32_t* flag = reinterpret_cast<int32_t*>(ws + l.flag);
    int32_t* pos = reinterpret_cast<int32_t*>(ws + l.pos);
    uint32_t* keys = reinterpret_cast<uint32_t*>(ws + l.keys);
    uint32_t* sorted_keys = reinterpret_cast<uint32_t*>(ws + l.sorted_keys);
    int64_t* ids = reinterpret_cast<int64_t*>(ws + l.ids);
    int64_t* sorted_ids = reinterpret_cast<int64_t*>(ws + l.sorted_ids);
    int64_t* offsets = reinterpret_cast<int64_t*>(ws + l.offsets);
    int64_t* pair_counts = reinterpret_cast<int64_t*>(ws + l.pair_counts);
    int64_t* pair_offsets = reinterpret_cast<int64_t*>(ws + l.pair_offsets);
    void* temp = ws + l.temp;
    size_t temp_bytes = l.temp_bytes;
    const int grid = grid_for(n_edges, kThreads);
    short_flags_kernel<<<grid, kThreads, 0, s>>>(dist, n_edges, cutoff, flag);
    cudaError_t err = cub::DeviceScan::ExclusiveSum(temp, temp_bytes, flag, pos, n_edges, s);
    if (err != cudaSuccess) return record_cuda_error(err);
    short_compact_kernel<<<grid, kThreads, 0, s>>>(flag, pos, center, n_edges, n_atoms, keys, ids, flags);
    if ((st = check_launch()) != FMD_OK) return st;
    if (!presorted) {  // stable: equal centres keep edge order
        err = cub::DeviceRadixSort::SortPairs(temp, temp_bytes, keys, sorted_keys, ids, sorted_ids, n_edges, 0, 32, s);
        if (err != cudaSuccess) return record_cuda_error(err);
    } else {
        sorted_keys = keys;
        sorted_ids = ids;
    }
    atom_runs_kernel<<<grid_for(n_atoms + 1, kThreads), kThreads, 0, s>>>(sorted_keys, n_edges, n_atoms, offsets,
                                                                          pair_counts);
    if ((st = check_launch()) != FMD_OK) return st;
    err = cub::DeviceScan::ExclusiveSum(temp, temp_bytes, pair_counts, pair_offsets, n_atoms + 1, s);
    if (err != cudaSuccess) return record_cuda_error(err);
    const int64_t work = t_capacity > 0 ? t_capacity : 1;
    triplets_kernel<<<grid_for(work, kThreads), kThreads, 0, s>>>(offsets, pair_offsets, sorted_ids,
                                                                  directed2undirected, n_atoms, t_capacity, triplets,
                                                                  n_triplets, flags);
    return check_launch();
}

}  // extern "C"
