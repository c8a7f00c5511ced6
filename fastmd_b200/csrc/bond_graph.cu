// Fixed-capacity MatRIS bond graph: undirected pairs and triplets over the
// padded, canonical edge rows of a fixed-capacity build, capture-safe (every
// count stays on the device).
//
// The reference builds it in _materialize_pairs, _materialize_line_graph,
// _line_graph_kernel, _allocate_overflow_topology and
// _substitute_overflow_topology (fastmd/graph/fixed_capacity_builder.py:2001,
// :2101, :681, :1474, :2163) from rows it sorts itself; the re-filter of this
// library already writes the real rows in canonical (centre, neighbour, image)
// order, so here each row finds its reverse by a binary search over them.
//
//   bond_rows     one thread per row: the reverse row (lower bound of the
//                 reverse key among the real rows), the pair-leader bit
//                 (row <= reverse), the short bit (dist2 < line_cutoff^2 in
//                 the re-filter's FP32 operation order), packed as
//                 leader << 32 | short for one scan; padded rows rewritten
//                 by the padding rule (sink atoms: both rows of padded pair p
//                 on sink N + p n_dummy / n_pad_u, image (3, 3, 3); far
//                 self-loops: the two opposite loops of atom p mod N);
//                 undirected2directed prefilled.
//   (scan)        inclusive sum of the packed bits: leader ranks in the high
//                 word, short ranks in the low word.
//   bond_pairs    directed2undirected = leader rank of min(row, reverse)
//                 (padded rows: padded pairs in order); each leader writes
//                 its undirected2directed entry; each short row its slot in
//                 the compacted short-row list; the pair-count check.
//   bond_atoms    one thread per atom: its run of rows (binary search of the
//                 centre column), its short count k and first short slot,
//                 k (k - 1) ordered pairs.
//   (scan)        exclusive sum of the pair counts: pair_offsets [N + 1].
//   bond_finish   the overflow decision (edges >= e_capacity, triplets >
//                 t_capacity, invalid pairs, invalid candidates), then either
//                 the all-padding topology over every row, pair and triplet,
//                 or the triplet rows [atom, u(first), first, u(second),
//                 second] with first = l / (k - 1), second = l % (k - 1)
//                 skipping first, and the padded triplets on padded pairs.
//
// The integer arithmetic of every row, pair and triplet is the reference's,
// so the outputs are equal to its builder's bit for bit (this file is
// compiled without FMA contraction, like the re-filter it follows).

#include <cub/device/device_scan.cuh>

#include "common.cuh"

namespace fmd {
namespace {

constexpr int kThreads = 256;
inline size_t align_up(size_t b) { return (b + 255) & ~size_t(255); }
constexpr int32_t kCandidateInvalid = FMD_FLAG_SKIN | FMD_FLAG_CANDIDATE_OVERFLOW | FMD_FLAG_NONFINITE;

struct BondArgs {
    const float* pos;       // [N, 3] wrapped positions the edges were computed from
    float cell[9];          // row-major lattice vectors
    int64_t n_atoms;
    int32_t* edge_index;    // [E_cap, 2] (centre, neighbour)
    float* edge_image;      // [E_cap, 3] integer images as float
    const int64_t* n_edges; // device: real directed edges (unclamped)
    int64_t e_cap, u_cap, t_cap;
    float line2;
    int32_t sink;
    int64_t n_dummy;
    int32_t pad_image[3];
    int32_t* pair_pos;      // [E_cap] reverse row
    int64_t* bits;          // [E_cap] leader << 32 | short
    int64_t* ranks;         // [E_cap] inclusive scan of bits
    int32_t* short_rows;    // [E_cap] short rows in row order
    int64_t* atom_pairs;    // [N + 1] k (k - 1), last 0
    int64_t* pair_off;      // [N + 1]
    int64_t* short_start;   // [N] first short slot of each atom
    int32_t* short_count;   // [N]
    int32_t* d2u;           // [E_cap]
    int32_t* u2d;           // [U_cap]
    int32_t* line_graph;    // [T_cap, 5]
    int64_t* n_triplets;
    int32_t* flags;
};

struct Row {
    int32_t c, n, x, y, z;
};

__device__ __forceinline__ Row load_row(const BondArgs& a, int64_t e) {
    const int2 cn = *reinterpret_cast<const int2*>(a.edge_index + 2 * e);
    return Row{cn.x, cn.y, __float2int_rn(a.edge_image[3 * e]), __float2int_rn(a.edge_image[3 * e + 1]),
               __float2int_rn(a.edge_image[3 * e + 2])};
}

// lexicographic (centre, neighbour, image) order: the order of the reference's
// sort key (c N + n) V + code(image) for images within its radix
__device__ __forceinline__ bool row_less(const Row& r, const Row& k) {
    if (r.c != k.c) return r.c < k.c;
    if (r.n != k.n) return r.n < k.n;
    if (r.x != k.x) return r.x < k.x;
    if (r.y != k.y) return r.y < k.y;
    return r.z < k.z;
}

__device__ __forceinline__ bool row_equal(const Row& r, const Row& k) {
    return r.c == k.c && r.n == k.n && r.x == k.x && r.y == k.y && r.z == k.z;
}

__device__ __forceinline__ int64_t total_clamped(const BondArgs& a) { return min(*a.n_edges, a.e_cap); }

__device__ __forceinline__ float short_dist2(const BondArgs& a, const Row& r) {
    const float* c = a.cell;
    const float sx = float(r.x), sy = float(r.y), sz = float(r.z);
    const float px = a.pos[3 * int64_t(r.c)], py = a.pos[3 * int64_t(r.c) + 1], pz = a.pos[3 * int64_t(r.c) + 2];
    const float qx = a.pos[3 * int64_t(r.n)], qy = a.pos[3 * int64_t(r.n) + 1], qz = a.pos[3 * int64_t(r.n) + 2];
    const float dx = __fadd_rn(__fadd_rn(__fadd_rn(__fsub_rn(qx, px), __fmul_rn(sx, c[0])), __fmul_rn(sy, c[3])),
                               __fmul_rn(sz, c[6]));
    const float dy = __fadd_rn(__fadd_rn(__fadd_rn(__fsub_rn(qy, py), __fmul_rn(sx, c[1])), __fmul_rn(sy, c[4])),
                               __fmul_rn(sz, c[7]));
    const float dz = __fadd_rn(__fadd_rn(__fadd_rn(__fsub_rn(qz, pz), __fmul_rn(sx, c[2])), __fmul_rn(sy, c[5])),
                               __fmul_rn(sz, c[8]));
    return __fadd_rn(__fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)), __fmul_rn(dz, dz));
}

__device__ __forceinline__ void write_row(const BondArgs& a, int64_t e, int64_t c, int64_t n, int x, int y, int z) {
    *reinterpret_cast<int2*>(a.edge_index + 2 * e) = make_int2(int(c), int(n));
    a.edge_image[3 * e] = float(x);
    a.edge_image[3 * e + 1] = float(y);
    a.edge_image[3 * e + 2] = float(z);
}

__global__ void __launch_bounds__(kThreads) bond_rows_kernel(BondArgs a) {
    const int64_t tc = total_clamped(a);
    const int64_t real_u = tc / 2;
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < a.e_cap; e += int64_t(gridDim.x) * blockDim.x) {
        int64_t bits = 0;
        if (e < tc) {
            const Row r = load_row(a, e);
            const Row rev{r.n, r.c, -r.x, -r.y, -r.z};
            int64_t lo = 0, hi = tc;
            while (lo < hi) {
                const int64_t mid = (lo + hi) >> 1;
                if (row_less(load_row(a, mid), rev))
                    lo = mid + 1;
                else
                    hi = mid;
            }
            const bool match = lo < tc && row_equal(load_row(a, lo), rev);
            const int64_t pos = min(lo, a.e_cap - 1);
            a.pair_pos[e] = int32_t(pos);
            if (!match) raise_flag(a.flags, FMD_FLAG_INVALID_PAIRS);
            const bool leader = match && e <= pos;
            const bool is_short = r.c >= 0 && r.c < a.n_atoms && r.n >= 0 && r.n < a.n_atoms &&
                                  short_dist2(a, r) < a.line2;
            bits = (int64_t(leader) << 32) | int64_t(is_short);
        } else {
            const int64_t pad = e - tc;
            if (a.sink) {
                const int64_t n_pad_u = a.e_cap / 2 - real_u;
                const int64_t sink = a.n_atoms + (pad / 2) * a.n_dummy / max(n_pad_u, int64_t(1));
                write_row(a, e, sink, sink, 3, 3, 3);
            } else {
                const int64_t atom = (pad / 2) % a.n_atoms;
                const int sign = 1 - 2 * int(pad % 2);
                write_row(a, e, atom, atom, sign * a.pad_image[0], sign * a.pad_image[1], sign * a.pad_image[2]);
            }
            a.pair_pos[e] = int32_t(e);
        }
        a.bits[e] = bits;
        if (e < a.u_cap)  // leaders overwrite their entries in bond_pairs
            a.u2d[e] = int32_t(e < real_u ? a.e_cap - 1 : min(tc + 2 * (e - real_u), a.e_cap - 1));
    }
}

__global__ void __launch_bounds__(kThreads) bond_pairs_kernel(BondArgs a) {
    const int64_t total = *a.n_edges;
    const int64_t tc = min(total, a.e_cap);
    const int64_t real_u = tc / 2;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        const int64_t pair_count = a.ranks[a.e_cap - 1] >> 32;
        if (total % 2 != 0 || pair_count != total / 2) raise_flag(a.flags, FMD_FLAG_INVALID_PAIRS);
    }
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < a.e_cap; e += int64_t(gridDim.x) * blockDim.x) {
        int64_t u;
        if (e < tc) {
            const int64_t canonical = min(e, int64_t(a.pair_pos[e]));
            u = (a.ranks[canonical] >> 32) - 1;
            const int64_t bits = a.bits[e];
            if ((bits >> 32) != 0 && u < real_u) a.u2d[u] = int32_t(e);
            if ((bits & 1) != 0) a.short_rows[(a.ranks[e] & 0xffffffffll) - 1] = int32_t(e);
        } else {
            u = real_u + (e - tc) / 2;
        }
        a.d2u[e] = int32_t(min(max(u, int64_t(0)), a.u_cap - 1));
    }
}

__device__ __forceinline__ int64_t centre_lower_bound(const BondArgs& a, int64_t tc, int64_t atom) {
    int64_t lo = 0, hi = tc;
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (a.edge_index[2 * mid] < atom)
            lo = mid + 1;
        else
            hi = mid;
    }
    return lo;
}

__global__ void __launch_bounds__(kThreads) bond_atoms_kernel(BondArgs a) {
    const int64_t tc = total_clamped(a);
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i <= a.n_atoms;
         i += int64_t(gridDim.x) * blockDim.x) {
        if (i == a.n_atoms) {
            a.atom_pairs[i] = 0;
            continue;
        }
        const int64_t s = centre_lower_bound(a, tc, i), t = centre_lower_bound(a, tc, i + 1);
        const int64_t before = s > 0 ? (a.ranks[s - 1] & 0xffffffffll) : 0;
        const int64_t upto = t > 0 ? (a.ranks[t - 1] & 0xffffffffll) : 0;
        const int64_t k = upto - before;
        a.short_start[i] = before;
        a.short_count[i] = int32_t(k);
        a.atom_pairs[i] = k * (k - 1);
    }
}

__global__ void __launch_bounds__(kThreads) bond_finish_kernel(BondArgs a) {
    const int64_t total = *a.n_edges;
    const int64_t tc = min(total, a.e_cap);
    const int64_t n_trip = a.pair_off[a.n_atoms];
    const int32_t seen = *a.flags;
    const bool overflow = total >= a.e_cap || n_trip > a.t_cap ||
                          (seen & (FMD_FLAG_INVALID_PAIRS | kCandidateInvalid)) != 0;
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    const int64_t first_thread = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
    if (first_thread == 0) {
        *a.n_triplets = n_trip;
        if (total >= a.e_cap) raise_flag(a.flags, FMD_FLAG_EDGE_OVERFLOW);
        if (n_trip > a.t_cap) raise_flag(a.flags, FMD_FLAG_TRIPLET_OVERFLOW);
    }
    const int64_t rows = max(a.e_cap, a.t_cap);
    if (overflow) {
        // the all-padding topology: pair p on sink N + p n_dummy / U (or loop atom p mod N)
        auto safe_atom = [&](int64_t u) { return a.sink ? a.n_atoms + u * a.n_dummy / a.u_cap : u % a.n_atoms; };
        for (int64_t e = first_thread; e < rows; e += stride) {
            if (e < a.e_cap) {
                const int64_t u = e / 2, atom = safe_atom(u);
                const int sign = e % 2 == 0 ? 1 : -1;
                if (a.sink)
                    write_row(a, e, atom, atom, 3 * sign, 3 * sign, 3 * sign);
                else
                    write_row(a, e, atom, atom, sign * a.pad_image[0], sign * a.pad_image[1], sign * a.pad_image[2]);
                a.d2u[e] = int32_t(u);
                if (e < a.u_cap) a.u2d[e] = int32_t(2 * e);
            }
            if (e < a.t_cap) {
                int64_t line_u = a.sink ? ((e * a.n_dummy / a.t_cap) * a.u_cap + a.n_dummy - 1) / a.n_dummy
                                        : e * a.u_cap / a.t_cap;
                line_u = min(line_u, a.u_cap - 1);
                const int64_t de = 2 * line_u;
                int32_t* out = a.line_graph + 5 * e;
                out[0] = int32_t(safe_atom(de / 2));
                out[1] = int32_t(line_u);
                out[2] = int32_t(de);
                out[3] = int32_t(line_u);
                out[4] = int32_t(de);
            }
        }
        return;
    }
    const int64_t t_clamped = min(n_trip, a.t_cap);
    const int64_t real_u = tc / 2;
    for (int64_t t = first_thread; t < a.t_cap; t += stride) {
        int32_t* out = a.line_graph + 5 * t;
        if (t < t_clamped) {
            // the last atom whose pair offset is <= t
            int64_t lo = 0, hi = a.n_atoms;
            while (lo < hi) {
                const int64_t mid = (lo + hi + 1) >> 1;
                if (a.pair_off[mid] <= t)
                    lo = mid;
                else
                    hi = mid - 1;
            }
            const int64_t atom = min(lo, a.n_atoms - 1);
            const int64_t local = t - a.pair_off[atom];
            const int64_t denom = max(int64_t(a.short_count[atom]) - 1, int64_t(1));
            const int64_t first = local / denom;
            const int64_t second_raw = local - first * denom;
            const int64_t second = second_raw + (second_raw >= first ? 1 : 0);
            const int32_t e1 = a.short_rows[a.short_start[atom] + first];
            const int32_t e2 = a.short_rows[a.short_start[atom] + second];
            out[0] = int32_t(atom);
            out[1] = a.d2u[e1];
            out[2] = e1;
            out[3] = a.d2u[e2];
            out[4] = e2;
        } else {
            const int64_t pad_id = t - t_clamped;
            const int64_t pad_pair = pad_id % max(a.u_cap - real_u, int64_t(1));
            const int64_t pad_u = real_u + pad_pair, pad_de = tc + 2 * pad_pair;
            const int64_t pad_atom = a.sink ? a.n_atoms + pad_id * a.n_dummy / max(a.t_cap - t_clamped, int64_t(1))
                                            : pad_pair % a.n_atoms;
            out[0] = int32_t(pad_atom);
            out[1] = int32_t(pad_u);
            out[2] = int32_t(pad_de);
            out[3] = int32_t(pad_u);
            out[4] = int32_t(pad_de);
        }
    }
}

struct BondLayout {
    size_t pair_pos, bits, ranks, short_rows, atom_pairs, pair_off, short_start, short_count, temp, temp_bytes, total;
};

fmd_status bond_layout(int64_t n_atoms, int64_t e_cap, BondLayout* l) {
    size_t scan_a = 0, scan_b = 0;
    cudaError_t err = cub::DeviceScan::InclusiveSum(nullptr, scan_a, static_cast<int64_t*>(nullptr),
                                                    static_cast<int64_t*>(nullptr), int(e_cap));
    if (err == cudaSuccess)
        err = cub::DeviceScan::ExclusiveSum(nullptr, scan_b, static_cast<int64_t*>(nullptr),
                                            static_cast<int64_t*>(nullptr), int(n_atoms + 1));
    if (err != cudaSuccess) return record_cuda_error(err);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off += align_up(bytes);
        return at;
    };
    l->pair_pos = take(sizeof(int32_t) * e_cap);
    l->bits = take(sizeof(int64_t) * e_cap);
    l->ranks = take(sizeof(int64_t) * e_cap);
    l->short_rows = take(sizeof(int32_t) * e_cap);
    l->atom_pairs = take(sizeof(int64_t) * (n_atoms + 1));
    l->pair_off = take(sizeof(int64_t) * (n_atoms + 1));
    l->short_start = take(sizeof(int64_t) * n_atoms);
    l->short_count = take(sizeof(int32_t) * n_atoms);
    l->temp_bytes = scan_a > scan_b ? scan_a : scan_b;
    l->temp = take(l->temp_bytes);
    l->total = off;
    return FMD_OK;
}

}  // namespace
}  // namespace fmd

using namespace fmd;

extern "C" {

fmd_status fmd_bond_graph_workspace_bytes(int64_t n_atoms, int64_t e_capacity, size_t* bytes) {
    if (bytes == nullptr || n_atoms < 1 || e_capacity < 2 || e_capacity > INT32_MAX) return FMD_ERR_INVALID_ARGUMENT;
    BondLayout l;
    const fmd_status st = bond_layout(n_atoms, e_capacity, &l);
    if (st != FMD_OK) return st;
    *bytes = l.total;
    return FMD_OK;
}

fmd_status fmd_bond_graph(const float* positions, const float* cell, int64_t n_atoms, int32_t* edge_index,
                          float* edge_image, const int64_t* n_edges, int64_t u_capacity, int64_t t_capacity,
                          float line_cutoff, int32_t padding, int64_t n_dummy, const int32_t* pad_image,
                          void* workspace, size_t workspace_bytes, int32_t* directed2undirected,
                          int32_t* undirected2directed, int32_t* line_graph, int64_t* n_triplets, int32_t* flags,
                          void* stream) {
    const int64_t e_cap = 2 * u_capacity;
    if (positions == nullptr || cell == nullptr || edge_index == nullptr || edge_image == nullptr ||
        n_edges == nullptr || directed2undirected == nullptr || undirected2directed == nullptr ||
        line_graph == nullptr || n_triplets == nullptr || flags == nullptr || n_atoms < 1 || u_capacity < 1 ||
        t_capacity < 1 || e_cap > INT32_MAX || !(line_cutoff >= 0.0f) ||
        (padding != FMD_PAD_SINK_ATOMS && padding != FMD_PAD_FAR_SELF_LOOPS) ||
        (padding == FMD_PAD_SINK_ATOMS && n_dummy < 1) || (padding == FMD_PAD_FAR_SELF_LOOPS && pad_image == nullptr) ||
        n_atoms + n_dummy > INT32_MAX)
        return FMD_ERR_INVALID_ARGUMENT;
    BondLayout l;
    fmd_status st = bond_layout(n_atoms, e_cap, &l);
    if (st != FMD_OK) return st;
    if (workspace == nullptr || workspace_bytes < l.total) return FMD_ERR_WORKSPACE;
    char* ws = static_cast<char*>(workspace);
    BondArgs a;
    a.pos = positions;
    for (int i = 0; i < 9; ++i) a.cell[i] = cell[i];
    a.n_atoms = n_atoms;
    a.edge_index = edge_index;
    a.edge_image = edge_image;
    a.n_edges = n_edges;
    a.e_cap = e_cap;
    a.u_cap = u_capacity;
    a.t_cap = t_capacity;
    a.line2 = line_cutoff * line_cutoff;
    a.sink = padding == FMD_PAD_SINK_ATOMS;
    a.n_dummy = a.sink ? n_dummy : 0;
    for (int i = 0; i < 3; ++i) a.pad_image[i] = a.sink ? 0 : pad_image[i];
    a.pair_pos = reinterpret_cast<int32_t*>(ws + l.pair_pos);
    a.bits = reinterpret_cast<int64_t*>(ws + l.bits);
    a.ranks = reinterpret_cast<int64_t*>(ws + l.ranks);
    a.short_rows = reinterpret_cast<int32_t*>(ws + l.short_rows);
    a.atom_pairs = reinterpret_cast<int64_t*>(ws + l.atom_pairs);
    a.pair_off = reinterpret_cast<int64_t*>(ws + l.pair_off);
    a.short_start = reinterpret_cast<int64_t*>(ws + l.short_start);
    a.short_count = reinterpret_cast<int32_t*>(ws + l.short_count);
    a.d2u = directed2undirected;
    a.u2d = undirected2directed;
    a.line_graph = line_graph;
    a.n_triplets = n_triplets;
    a.flags = flags;
    const cudaStream_t s = as_stream(stream);
    size_t temp_bytes = l.temp_bytes;
    void* temp = ws + l.temp;
    bond_rows_kernel<<<grid_for(e_cap, kThreads), kThreads, 0, s>>>(a);
    cudaError_t err = cub::DeviceScan::InclusiveSum(temp, temp_bytes, a.bits, a.ranks, int(e_cap), s);
    if (err != cudaSuccess) return record_cuda_error(err);
    bond_pairs_kernel<<<grid_for(e_cap, kThreads), kThreads, 0, s>>>(a);
    bond_atoms_kernel<<<grid_for(n_atoms + 1, kThreads), kThreads, 0, s>>>(a);
    temp_bytes = l.temp_bytes;
    err = cub::DeviceScan::ExclusiveSum(temp, temp_bytes, a.atom_pairs, a.pair_off, int(n_atoms + 1), s);
    if (err != cudaSuccess) return record_cuda_error(err);
    const int64_t rows = e_cap > t_capacity ? e_cap : t_capacity;
    bond_finish_kernel<<<grid_for(rows, kThreads), kThreads, 0, s>>>(a);
    return check_launch();
}

}  // extern "C"
