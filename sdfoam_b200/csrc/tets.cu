// Tetrahedra of the Delaunay triangulation: the B200 replacement of the
// reference's Triangulation::tets / tet_adjacency / vert_to_tet
// (src/delaunay/delaunay.h:23-37, filled by find_adjacency,
// src/delaunay/delaunay.cu:32-144; bound as Triangulation.tets() etc. in
// torch_bindings/triangulation_bindings.cpp:59-115).
//
// A Delaunay tet {i, a, b, c} is a vertex of the Voronoi cell of each of its
// four sites, where the bisector planes of a, b and c meet.  Each site's cell
// is rebuilt from its CSR row alone (the box of the adjacency pass, clipped
// by the row's sites nearest first; no search, no vertex checks) and the cell
// emits the tets of the vertices that involve no box plane and whose other
// three sites all have larger indices, so each tet comes from exactly one
// cell, the cell of its smallest site.  Cells in ascending site order, each
// emitting its tets sorted by their other three sites, give the tets sorted by
// their sorted vertex sets: the order of the reference's tet map
// (SortedMap<IndexedTet> keyed by set_less, src/utils/geometry.h:217-232), so
// tet indices agree with the reference's for the same tet set.  Within a tet
// the vertices are ascending with the last two swapped where needed for the
// reference's orientation (IndexedTet::volume > 0, geometry.h:488-494; the
// growth step's swap, growth_iteration.cu:55-60).
//
// Faces: tet t's face j is the triangle opposite vertex j.  A face is filed
// under its smallest vertex; each vertex's bucket is sorted by the other two
// vertices, and a face met twice links its two tets:
// tet_adjacency[4 t + j] = 4 t' + j' of the tet across it, UINT32_MAX on the
// hull (find_adjacency's face_to_tet encoding).  A face met more than twice
// is counted as ambiguous, which the caller reports as the reference does
// ("ambiguous triangulation").  vert_to_tet[v] = the smallest tet index that
// contains v, UINT32_MAX for none (the reference's atomicMin).
#include <cfloat>
#include <cstdint>
#include <cstring>

#include "foam_internal.h"
#include "voronoi_cell.cuh"

namespace sdfoam_b200 {

namespace {

using namespace voronoi;

constexpr uint32_t kTetLargeSlots = 148 * 8;  // large cells for rows past a small cell's room
enum TetStatus { kTsFailed = 0, kTsAmbiguous = 1, kTsTooLong = 2, kTsQueued = 3 };

struct TetParams {
    Tree tree;                 // the sites (boxes unused)
    const uint32_t *adj, *off;
    uint32_t adjacency_size;
    double lo[3], hi[3];       // the box, absolute
    uint32_t *count;           // [n] tets owned by each site
    const uint32_t *first;     // write pass: [n + 1] first tet of each site
    uint32_t *tets;            // write pass: [num_tets][4]
    uint32_t num_tets;
    uint32_t *status;          // TetStatus words
    uint32_t *queue;           // sites whose row needs a large cell
    uint32_t queue_cap;
};

__device__ __forceinline__ bool row_of(const TetParams &P, uint32_t i, uint32_t &b, uint32_t &e) {
    b = i == 0 ? 0u : P.off[i];
    e = P.off[i + 1];
    return b != 0xffffffffu && e != 0xffffffffu && b <= e && e <= P.adjacency_size;
}

// Rebuilds site i's cell from its row and counts (write = false) or writes
// the tets it owns.  Returns false when the row does not fit in Cell.
template <class Cell>
__device__ bool tet_cell(const TetParams &P, uint32_t i, Cell &C, bool write) {
    const Tree &T = P.tree;
    uint32_t b, e;
    if (!row_of(P, i, b, e)) {
        if (!write) P.count[i] = 0;
        return true;
    }
    const uint32_t deg = e - b;
    if (deg + 6 > uint32_t(Cell::kPlanes)) return false;
    const double p[3] = {__ldg(T.points + 3 * size_t(i)), __ldg(T.points + 3 * size_t(i) + 1),
                         __ldg(T.points + 3 * size_t(i) + 2)};
    // the row's sites, nearest first (ties to the lower index)
    double dd[Cell::kPlanes];
    uint32_t ids[Cell::kPlanes];
    for (uint32_t k = 0; k < deg; ++k) {
        const uint32_t j = min(__ldg(P.adj + b + k), T.num_points - 1);
        const double dx = double(__ldg(T.points + 3 * size_t(j))) - p[0];
        const double dy = double(__ldg(T.points + 3 * size_t(j) + 1)) - p[1];
        const double dz = double(__ldg(T.points + 3 * size_t(j) + 2)) - p[2];
        const double d = dx * dx + dy * dy + dz * dz;
        uint32_t m = k;
        while (m > 0 && (dd[m - 1] > d || (dd[m - 1] == d && ids[m - 1] > j))) {
            dd[m] = dd[m - 1];
            ids[m] = ids[m - 1];
            --m;
        }
        dd[m] = d;
        ids[m] = j;
    }
    const double lo[3] = {P.lo[0] - p[0], P.lo[1] - p[1], P.lo[2] - p[2]};
    const double hi[3] = {P.hi[0] - p[0], P.hi[1] - p[1], P.hi[2] - p[2]};
    uint32_t scratch[4] = {0, 0, 0, 0};
    C.bad = false;
    C.guard = scratch;
    init_box(C, lo, hi);
    bool ok = true;
    for (uint32_t k = 0; k < deg && ok; ++k) ok = clip_candidate(C, T, p, ids[k], scratch) >= 0 && !C.bad;
    if (!ok) {
        atomicAdd(P.status + kTsFailed, 1u);
        if (!write) P.count[i] = 0;
        return true;
    }
    // the owned tets: vertices on three site planes whose sites all follow i
    uint32_t owned = 0;
    for (int t = 0; t < C.nt; ++t) {
        const uint32_t x = C.pid[C.tri[t][0]], y = C.pid[C.tri[t][1]], z = C.pid[C.tri[t][2]];
        if (is_box(x) || is_box(y) || is_box(z)) continue;
        if (x > i && y > i && z > i) {
            if (write) {  // the owned triples, each sorted, over the vertex slots already read
                const uint32_t s0 = min(x, min(y, z)), s2 = max(x, max(y, z));
                const uint32_t s1 = x ^ y ^ z ^ s0 ^ s2;
                C.vx[owned] = double(s0);
                C.vy[owned] = double(s1);
                C.vz[owned] = double(s2);
            }
            ++owned;
        }
    }
    if (!write) {
        P.count[i] = owned;
        return true;
    }
    // insertion sort of the owned triples (held exactly as doubles; at most
    // nt of them, and the vertex coordinates are no longer needed)
    for (uint32_t a = 1; a < owned; ++a) {
        const double k0 = C.vx[a], k1 = C.vy[a], k2 = C.vz[a];
        uint32_t m = a;
        while (m > 0 && (C.vx[m - 1] > k0 || (C.vx[m - 1] == k0 && (C.vy[m - 1] > k1 ||
                                                                   (C.vy[m - 1] == k1 && C.vz[m - 1] > k2))))) {
            C.vx[m] = C.vx[m - 1];
            C.vy[m] = C.vy[m - 1];
            C.vz[m] = C.vz[m - 1];
            --m;
        }
        C.vx[m] = k0;
        C.vy[m] = k1;
        C.vz[m] = k2;
    }
    const uint32_t base = P.first[i];
    if (owned != P.first[i + 1] - base || base + owned > P.num_tets) {
        atomicAdd(P.status + kTsFailed, 1u);
        return true;
    }
    for (uint32_t k = 0; k < owned; ++k) {
        uint32_t v1 = uint32_t(C.vx[k]), v2 = uint32_t(C.vy[k]), v3 = uint32_t(C.vz[k]);
        // orientation: det(v1 - v0, v2 - v0, v3 - v0) < 0, i.e. the reference's
        // volume (v2 - v0) x (v1 - v0) . (v3 - v0) / 6 > 0
        double q[3][3];
        const uint32_t vs[3] = {v1, v2, v3};
        for (int r = 0; r < 3; ++r)
            for (int c = 0; c < 3; ++c) q[r][c] = double(__ldg(T.points + 3 * size_t(vs[r]) + c)) - p[c];
        const double det = q[0][0] * (q[1][1] * q[2][2] - q[1][2] * q[2][1]) -
                           q[0][1] * (q[1][0] * q[2][2] - q[1][2] * q[2][0]) +
                           q[0][2] * (q[1][0] * q[2][1] - q[1][1] * q[2][0]);
        if (det > 0.0) {
            const uint32_t s = v2;
            v2 = v3;
            v3 = s;
        }
        uint4 *out = reinterpret_cast<uint4 *>(P.tets) + base + k;
        *out = make_uint4(i, v1, v2, v3);
    }
    return true;
}

__global__ void __launch_bounds__(64) tet_cells_kernel(const TetParams P, bool write) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= P.tree.num_points) return;
    SmallCell C;
    if (!tet_cell(P, i, C, write)) {
        if (write) return;  // the large pass writes it
        const uint32_t slot = atomicAdd(P.status + kTsQueued, 1u);
        if (slot < P.queue_cap) P.queue[slot] = i;
        P.count[i] = 0;
    }
}

__global__ void __launch_bounds__(64) tet_large_cells_kernel(const TetParams P, LargeCell *slots, bool write) {
    const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t queued = min(P.status[kTsQueued], P.queue_cap);
    for (uint32_t k = t; k < queued; k += gridDim.x * blockDim.x) {
        const uint32_t i = P.queue[k];
        if (i >= P.tree.num_points) continue;
        if (!tet_cell(P, i, slots[t], write)) {
            if (!write) {
                atomicAdd(P.status + kTsTooLong, 1u);
                P.count[i] = 0;
            }
        }
    }
}

// the sites' bounding box as order-preserving keys (min in 0..2, max in 3..5)
__device__ __forceinline__ uint32_t order_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u ^ 0x80000000u);
}
float key_float(uint32_t k) {
    const uint32_t u = (k & 0x80000000u) ? (k ^ 0x80000000u) : ~k;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

__global__ void __launch_bounds__(256) bbox_kernel(const float *__restrict__ points, uint32_t n,
                                                   uint32_t *__restrict__ box) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const uint32_t k = order_key(__ldg(points + 3 * size_t(i) + c));
        atomicMin(box + c, k);
        atomicMax(box + 3 + c, k);
    }
}

// faces, filed under their smallest vertex
__device__ __forceinline__ void face_of(const uint4 &t, int j, uint32_t &x, uint32_t &y, uint32_t &z) {
    const uint32_t v[4] = {t.x, t.y, t.z, t.w};
    uint32_t a = v[(j + 1) & 3], b = v[(j + 2) & 3], c = v[(j + 3) & 3];
    x = min(a, min(b, c));
    z = max(a, max(b, c));
    y = a ^ b ^ c ^ x ^ z;
}

__global__ void __launch_bounds__(256) face_count_kernel(const uint4 *__restrict__ tets, uint32_t num_tets,
                                                         uint32_t n, uint32_t *__restrict__ fcount,
                                                         uint32_t *__restrict__ vert_to_tet,
                                                         uint32_t *__restrict__ status) {
    const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= num_tets) return;
    const uint4 q = tets[t];
    if (q.x >= n || q.y >= n || q.z >= n || q.w >= n) {
        atomicAdd(status + kTsFailed, 1u);
        return;
    }
    atomicMin(vert_to_tet + q.x, t);
    atomicMin(vert_to_tet + q.y, t);
    atomicMin(vert_to_tet + q.z, t);
    atomicMin(vert_to_tet + q.w, t);
    for (int j = 0; j < 4; ++j) {
        uint32_t x, y, z;
        face_of(q, j, x, y, z);
        atomicAdd(fcount + x, 1u);
    }
}

__global__ void __launch_bounds__(256) face_fill_kernel(const uint4 *__restrict__ tets, uint32_t num_tets,
                                                        uint32_t n, const uint32_t *__restrict__ fstart,
                                                        uint32_t *__restrict__ fcursor, uint4 *__restrict__ rec) {
    const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= num_tets) return;
    const uint4 q = tets[t];
    if (q.x >= n || q.y >= n || q.z >= n || q.w >= n) return;
    for (int j = 0; j < 4; ++j) {
        uint32_t x, y, z;
        face_of(q, j, x, y, z);
        const uint32_t slot = fstart[x] + atomicAdd(fcursor + x, 1u);
        if (slot < fstart[x + 1]) rec[slot] = make_uint4(y, z, 4 * t + uint32_t(j), 0u);
    }
}

__device__ __forceinline__ bool rec_less(const uint4 &a, const uint4 &b) {
    return a.x < b.x || (a.x == b.x && (a.y < b.y || (a.y == b.y && a.z < b.z)));
}

__global__ void __launch_bounds__(256) face_match_kernel(uint4 *__restrict__ rec, const uint32_t *__restrict__ fstart,
                                                         uint32_t n, uint32_t num_tets,
                                                         uint32_t *__restrict__ tet_adjacency,
                                                         uint32_t *__restrict__ status) {
    const uint32_t x = blockIdx.x * blockDim.x + threadIdx.x;
    if (x >= n) return;
    const uint32_t b = fstart[x], e = fstart[x + 1];
    for (uint32_t a = b + 1; a < e; ++a) {
        const uint4 v = rec[a];
        uint32_t m = a;
        while (m > b && rec_less(v, rec[m - 1])) {
            rec[m] = rec[m - 1];
            --m;
        }
        rec[m] = v;
    }
    const uint32_t limit = 4 * num_tets;
    for (uint32_t a = b; a < e;) {
        uint32_t c = a + 1;
        while (c < e && rec[c].x == rec[a].x && rec[c].y == rec[a].y) ++c;
        const uint32_t f0 = rec[a].z;
        if (c - a == 2) {
            const uint32_t f1 = rec[a + 1].z;
            if (f0 < limit && f1 < limit) {
                tet_adjacency[f0] = f1;
                tet_adjacency[f1] = f0;
            }
        } else {
            if (c - a > 2) atomicAdd(status + kTsAmbiguous, 1u);
            for (uint32_t k = a; k < c; ++k)
                if (rec[k].z < limit) tet_adjacency[rec[k].z] = 0xffffffffu;
        }
        a = c;
    }
}

struct TetLayout {
    size_t count, first, sums, status, box, queue, large, fcount, fstart, fcursor, rec, total;
};

TetLayout tet_layout(uint32_t n, uint32_t num_tets) {
    TetLayout l{};
    l.count = 0;
    l.first = align_up(l.count + (size_t(n) + 1) * 4, 256);
    l.sums = align_up(l.first + (size_t(n) + 1) * 4, 256);
    l.status = align_up(l.sums + scan_partials(n) * 4, 256);
    l.box = align_up(l.status + 64, 256);
    l.queue = align_up(l.box + 64, 256);
    l.large = align_up(l.queue + size_t(n) * 4, 256);
    l.fcount = align_up(l.large + size_t(kTetLargeSlots) * sizeof(LargeCell), 256);
    l.fstart = align_up(l.fcount + (size_t(n) + 1) * 4, 256);
    l.fcursor = align_up(l.fstart + (size_t(n) + 1) * 4, 256);
    l.rec = align_up(l.fcursor + (size_t(n) + 1) * 4, 256);
    l.total = align_up(l.rec + size_t(num_tets) * 4 * 16, 256);
    return l;
}

// The counting passes shared by both entry points: the box, then the owned
// tets of every site; leaves the per-site counts and their prefix in the
// workspace and the status words on the device.
cudaError_t count_pass(const float *points, uint32_t n, const uint32_t *adjacency, uint32_t adjacency_size,
                       const uint32_t *offsets, char *ws, const TetLayout &l, TetParams &P, cudaStream_t stream) {
    uint32_t *status = reinterpret_cast<uint32_t *>(ws + l.status);
    uint32_t *box = reinterpret_cast<uint32_t *>(ws + l.box);
    cudaError_t e = cudaMemsetAsync(status, 0, 64, stream);
    if (e != cudaSuccess) return e;
    const uint32_t init[6] = {0xffffffffu, 0xffffffffu, 0xffffffffu, 0u, 0u, 0u};
    if ((e = cudaMemcpyAsync(box, init, sizeof(init), cudaMemcpyHostToDevice, stream)) != cudaSuccess) return e;
    bbox_kernel<<<(n + 255) / 256, 256, 0, stream>>>(points, n, box);
    uint32_t hb[6];
    if ((e = cudaMemcpyAsync(hb, box, sizeof(hb), cudaMemcpyDeviceToHost, stream)) != cudaSuccess) return e;
    if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return e;
    // the adjacency pass's box: the bounds grown by 10^10 times the extent
    double ext = 0.0;
    for (int k = 0; k < 3; ++k) {
        const double d = double(key_float(hb[3 + k])) - key_float(hb[k]);
        ext = ext > d ? ext : d;
    }
    const double grow = 1e10 * (ext + 1e-3);
    P = TetParams{};
    P.tree.points = points;
    P.tree.num_points = n;
    P.adj = adjacency;
    P.off = offsets;
    P.adjacency_size = adjacency_size;
    for (int k = 0; k < 3; ++k) {
        P.lo[k] = double(key_float(hb[k])) - grow;
        P.hi[k] = double(key_float(hb[3 + k])) + grow;
    }
    P.count = reinterpret_cast<uint32_t *>(ws + l.count);
    P.status = status;
    P.queue = reinterpret_cast<uint32_t *>(ws + l.queue);
    P.queue_cap = n;
    LargeCell *large = reinterpret_cast<LargeCell *>(ws + l.large);
    tet_cells_kernel<<<(n + 63) / 64, 64, 0, stream>>>(P, false);
    tet_large_cells_kernel<<<kTetLargeSlots / 64, 64, 0, stream>>>(P, large, false);
    uint32_t *first = reinterpret_cast<uint32_t *>(ws + l.first);
    if ((e = launch_exclusive_scan(P.count, n, reinterpret_cast<uint32_t *>(ws + l.sums), first, stream)) !=
        cudaSuccess)
        return e;
    P.first = first;
    return cudaGetLastError();
}

}  // namespace

size_t tets_workspace_bytes(uint32_t n, uint32_t num_tets) { return tet_layout(n, num_tets).total; }

cudaError_t launch_tets_count(const float *points, uint32_t n, const uint32_t *adjacency, uint32_t adjacency_size,
                              const uint32_t *offsets, void *workspace, uint32_t *num_tets, uint32_t *status,
                              cudaStream_t stream) {
    const TetLayout l = tet_layout(n, 0);
    char *ws = static_cast<char *>(workspace);
    TetParams P;
    cudaError_t e = count_pass(points, n, adjacency, adjacency_size, offsets, ws, l, P, stream);
    if (e != cudaSuccess) return e;
    if ((e = cudaMemcpyAsync(num_tets, ws + l.first + size_t(n) * 4, 4, cudaMemcpyDeviceToHost, stream)) !=
        cudaSuccess)
        return e;
    if ((e = cudaMemcpyAsync(status, ws + l.status, 16, cudaMemcpyDeviceToHost, stream)) != cudaSuccess) return e;
    return cudaStreamSynchronize(stream);
}

cudaError_t launch_tets(const float *points, uint32_t n, const uint32_t *adjacency, uint32_t adjacency_size,
                        const uint32_t *offsets, void *workspace, uint32_t num_tets, uint32_t *tets,
                        uint32_t *tet_adjacency, uint32_t *vert_to_tet, uint32_t *status, bool *count_mismatch,
                        cudaStream_t stream) {
    *count_mismatch = false;
    const TetLayout l = tet_layout(n, num_tets);
    char *ws = static_cast<char *>(workspace);
    TetParams P;
    cudaError_t e = count_pass(points, n, adjacency, adjacency_size, offsets, ws, l, P, stream);
    if (e != cudaSuccess) return e;
    uint32_t total = 0;
    if ((e = cudaMemcpyAsync(&total, ws + l.first + size_t(n) * 4, 4, cudaMemcpyDeviceToHost, stream)) !=
        cudaSuccess)
        return e;
    if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return e;
    if (total != num_tets) {
        *count_mismatch = true;
        return cudaSuccess;
    }
    P.tets = tets;
    P.num_tets = num_tets;
    LargeCell *large = reinterpret_cast<LargeCell *>(ws + l.large);
    tet_cells_kernel<<<(n + 63) / 64, 64, 0, stream>>>(P, true);
    tet_large_cells_kernel<<<kTetLargeSlots / 64, 64, 0, stream>>>(P, large, true);
    uint32_t *fcount = reinterpret_cast<uint32_t *>(ws + l.fcount);
    uint32_t *fstart = reinterpret_cast<uint32_t *>(ws + l.fstart);
    uint32_t *fcursor = reinterpret_cast<uint32_t *>(ws + l.fcursor);
    uint4 *rec = reinterpret_cast<uint4 *>(ws + l.rec);
    if ((e = cudaMemsetAsync(fcount, 0, size_t(n) * 4, stream)) != cudaSuccess) return e;
    if ((e = cudaMemsetAsync(fcursor, 0, size_t(n) * 4, stream)) != cudaSuccess) return e;
    if ((e = cudaMemsetAsync(vert_to_tet, 0xff, size_t(n) * 4, stream)) != cudaSuccess) return e;
    if (num_tets > 0) {
        const uint32_t g = (num_tets + 255) / 256;
        face_count_kernel<<<g, 256, 0, stream>>>(reinterpret_cast<const uint4 *>(tets), num_tets, n, fcount,
                                                 vert_to_tet, P.status);
        if ((e = launch_exclusive_scan(fcount, n, reinterpret_cast<uint32_t *>(ws + l.sums), fstart, stream)) !=
            cudaSuccess)
            return e;
        face_fill_kernel<<<g, 256, 0, stream>>>(reinterpret_cast<const uint4 *>(tets), num_tets, n, fstart, fcursor,
                                                rec);
        face_match_kernel<<<(n + 255) / 256, 256, 0, stream>>>(rec, fstart, n, num_tets, tet_adjacency, P.status);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((e = cudaMemcpyAsync(status, ws + l.status, 16, cudaMemcpyDeviceToHost, stream)) != cudaSuccess) return e;
    return cudaStreamSynchronize(stream);
}

}  // namespace sdfoam_b200
