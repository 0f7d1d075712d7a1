// Delaunay adjacency of the sites: the B200 replacement of the reference's
// DelaunayTriangulation::rebuild (src/delaunay/delaunay.cu:273-370) and of the
// CSR it derives (find_adjacency, delaunay.cu:32-229).
//
// The Delaunay neighbours of a site are the sites whose bisector planes bound
// its Voronoi cell.  One thread builds one cell by clipping a large box around
// its site with bisector planes, nearest candidate first (the convex-cell
// clipping of "Meshless Voronoi on the GPU", Ray, Sokolov, Lefebvre, Levy,
// 2018), in double precision and in coordinates relative to the site:
//   * the cell is kept as its vertices, each the intersection of three planes,
//     stored as triangles of plane slots whose orientation is consistent
//     (det(n_a, n_b, n_c) > 0); a new plane deletes the vertices on its far
//     side and is stitched to the boundary of the deleted patch;
//   * candidates are the site's nearest sites (64, then 121) from an AABB
//     tree over the sites in Morton order (the caller's sort_points order
//     makes stick-shaped leaf boxes), found by a heap search seeded with the
//     site's index neighbours; the cell is final once the farthest candidate
//     is more than twice the cell's radius away, because no farther site's
//     bisector can reach it;
//   * cells still open after that -- sites on the convex hull, or sites whose
//     nearest sites all lie to one side -- are finished vertex by vertex: a
//     vertex is final when no site is closer to it than the cell's own site
//     (nearest-site search in double).  Any point of the segment from the site
//     to a vertex lies in the cell, so vertices on the box are probed at
//     growing distances along that segment first, which finds the sites that
//     close a one-sided cell with short searches.
// The box is the sites' bounding box grown by 10^10 times its size: every
// Voronoi vertex (Delaunay circumcentre) inside it is found, which covers all
// but hull slivers flatter than about 10^-10 (hull slivers of random sites
// have circumcentres 10^6 and more away); double precision still separates
// the far vertex tests (differences ~10^10, rounding ~10^4).
//
// The neighbour relation is then made symmetric (a pair seen from one side
// only, which only near-degenerate sets such as five cospherical sites can
// produce, is added to the other side) and written as the reference's CSR:
// rows of ascending neighbour ids; offsets[0] = 0, offsets[N] = 2 * edges, and
// offsets[r + 1] = the end of row r when row r is not empty and a later row
// is, else UINT32_MAX (the memset and key-change fill of delaunay.cu:207-226).
#include <cfloat>
#include <cstdint>

#include "foam_device.cuh"
#include "foam_internal.h"
#include "voronoi_cell.cuh"

namespace sdfoam_b200 {

namespace {

using namespace voronoi;

// First pass: one thread per site, the cell in local memory.
__global__ void __launch_bounds__(64) voronoi_cells_kernel(const CellParams P) {
    SmallCell C;
    voronoi_cell(P, blockIdx.x * blockDim.x + threadIdx.x, C, false);
}

// Second pass over the queued sites: each thread owns one large cell in the
// workspace (kLargeSlots of them) and walks the queue with a grid stride.
#ifndef SDFOAM_DELAUNAY_LARGE_SLOTS
#define SDFOAM_DELAUNAY_LARGE_SLOTS (148 * 64)
#endif
constexpr uint32_t kLargeSlots = SDFOAM_DELAUNAY_LARGE_SLOTS;

__global__ void __launch_bounds__(64) voronoi_large_cells_kernel(const CellParams P, LargeCell *slots) {
    const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t queued = min(P.status[kStRetry], P.retry_cap);
    for (uint32_t k = t; k < queued; k += gridDim.x * blockDim.x) voronoi_cell(P, P.retry[k], slots[t], true);
}

// --------------------------------------------------------------------------
// symmetry and CSR
// --------------------------------------------------------------------------

__device__ __forceinline__ bool row_has(const uint32_t *row, uint32_t n, uint32_t v) {
    uint32_t lo = 0, hi = n;
    while (lo < hi) {
        const uint32_t mid = (lo + hi) / 2;
        if (row[mid] < v)
            lo = mid + 1;
        else
            hi = mid;
    }
    return lo < n && row[lo] == v;
}

// pairs (i -> j) whose reverse is missing are recorded as (j, i)
__global__ void __launch_bounds__(256) asymmetry_kernel(const uint32_t *__restrict__ nbr,
                                                        const uint32_t *__restrict__ cnt, uint32_t n, uint32_t cap,
                                                        uint2 *__restrict__ extra, uint32_t extra_cap,
                                                        uint32_t *__restrict__ status) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t *row = nbr + size_t(i) * cap;
    const uint32_t m = cnt[i];
    if (m > cap) {
        vc_record(status + kStGuard, 21, i);
        return;
    }
    for (uint32_t k = 0; k < m; ++k) {
        const uint32_t j = row[k];
        if (j >= n || cnt[j] > cap) {
            vc_record(status + kStGuard, 22, i);
            continue;
        }
        if (!row_has(nbr + size_t(j) * cap, cnt[j], i)) {
            const uint32_t slot = atomicAdd(status + kStAsymmetric, 1u);
            if (slot < extra_cap) extra[slot] = make_uint2(j, i);
        }
    }
}

__global__ void __launch_bounds__(256) add_extra_kernel(const uint2 *__restrict__ extra, uint32_t n,
                                                        const uint32_t *status, uint32_t extra_cap,
                                                        uint32_t *__restrict__ nbr, uint32_t *__restrict__ cnt,
                                                        uint32_t cap, uint32_t *__restrict__ dirty,
                                                        uint32_t *status_out) {
    const uint32_t e = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t total = min(status[kStAsymmetric], extra_cap);
    if (e >= total) return;
    const uint2 x = extra[e];
    if (x.x >= n || x.y >= n) {  // self-check: ids come from the cells kernel
        vc_record(status_out + kStGuard, 20, e);
        return;
    }
    const uint32_t k = atomicAdd(cnt + x.x, 1u);
    if (k < cap) {
        nbr[size_t(x.x) * cap + k] = x.y;
    } else {
        atomicSub(cnt + x.x, 1u);
        atomicAdd(status_out + kStFailed, 1u);
    }
    dirty[x.x] = 1;
}

__global__ void __launch_bounds__(256) sort_dirty_kernel(uint32_t *__restrict__ nbr, const uint32_t *__restrict__ cnt,
                                                         uint32_t n, uint32_t cap, const uint32_t *__restrict__ dirty) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n || !dirty[i]) return;
    uint32_t *row = nbr + size_t(i) * cap;
    const uint32_t m = min(cnt[i], cap);
    for (uint32_t a = 1; a < m; ++a) {
        const uint32_t v = row[a];
        uint32_t b = a;
        while (b > 0 && row[b - 1] > v) {
            row[b] = row[b - 1];
            --b;
        }
        row[b] = v;
    }
}

constexpr int kScanItems = 16;
constexpr int kScanBlock = 256;
constexpr uint32_t kScanTile = kScanItems * kScanBlock;

__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t *warp_sums, uint32_t &total) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= uint32_t(o)) incl += y;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    uint32_t before = 0;
    total = 0;
    for (uint32_t w = 0; w < blockDim.x / 32; ++w) {
        if (w < warp) before += warp_sums[w];
        total += warp_sums[w];
    }
    __syncthreads();
    return before + incl - v;
}

__global__ void __launch_bounds__(kScanBlock) tile_sums_kernel(const uint32_t *__restrict__ cnt, uint32_t n,
                                                               uint32_t *__restrict__ sums) {
    __shared__ uint32_t ws[kScanBlock / 32];
    const size_t base = size_t(blockIdx.x) * kScanTile + size_t(threadIdx.x) * kScanItems;
    uint32_t s = 0;
    for (int k = 0; k < kScanItems; ++k)
        if (base + k < n) s += cnt[base + k];
    uint32_t total;
    block_exclusive_scan(s, ws, total);
    if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

__global__ void __launch_bounds__(1024) scan_sums_kernel(uint32_t *__restrict__ sums, uint32_t m) {
    __shared__ uint32_t ws[32];
    uint32_t carry = 0;
    for (uint32_t base = 0; base < m; base += blockDim.x) {
        const uint32_t i = base + threadIdx.x;
        const uint32_t v = i < m ? sums[i] : 0u;
        uint32_t total;
        const uint32_t ex = block_exclusive_scan(v, ws, total);
        if (i < m) sums[i] = carry + ex;
        carry += total;
    }
}

// prefix[i] = sum of cnt[0..i), prefix[n] = total
__global__ void __launch_bounds__(kScanBlock) tile_scan_kernel(const uint32_t *__restrict__ cnt, uint32_t n,
                                                               const uint32_t *__restrict__ sums,
                                                               uint32_t *__restrict__ prefix) {
    __shared__ uint32_t ws[kScanBlock / 32];
    const size_t base = size_t(blockIdx.x) * kScanTile + size_t(threadIdx.x) * kScanItems;
    uint32_t v[kScanItems];
    uint32_t s = 0;
    for (int k = 0; k < kScanItems; ++k) {
        v[k] = base + k < n ? cnt[base + k] : 0u;
        s += v[k];
    }
    uint32_t total;
    uint32_t run = sums[blockIdx.x] + block_exclusive_scan(s, ws, total);
    for (int k = 0; k < kScanItems; ++k) {
        if (base + k < n) prefix[base + k] = run;
        run += v[k];
        if (base + k + 1 == n) prefix[n] = run;
    }
}

__global__ void __launch_bounds__(256) last_row_kernel(const uint32_t *__restrict__ cnt, uint32_t n,
                                                       uint32_t *__restrict__ last) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n && cnt[i] > 0) atomicMax(last, i + 1);  // 0 = no row
}

__global__ void __launch_bounds__(256) offsets_kernel(const uint32_t *__restrict__ cnt,
                                                      const uint32_t *__restrict__ prefix, uint32_t n,
                                                      const uint32_t *__restrict__ last,
                                                      uint32_t *__restrict__ offsets) {
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r > n) return;
    uint32_t v;
    if (r == 0) {
        v = 0;
    } else if (r == n) {
        v = prefix[n];
    } else {
        const uint32_t row = r - 1;
        v = (cnt[row] > 0 && row + 1 < *last) ? prefix[r] : 0xffffffffu;
    }
    offsets[r] = v;
}

__global__ void __launch_bounds__(256) fill_kernel(const uint32_t *__restrict__ nbr, const uint32_t *__restrict__ cnt,
                                                   const uint32_t *__restrict__ prefix, uint32_t n, uint32_t cap,
                                                   uint32_t *__restrict__ adjacency, uint32_t adjacency_size) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t b = prefix[i];
    const uint32_t m = min(cnt[i], cap);
    for (uint32_t k = 0; k < m && b + k < adjacency_size; ++k) adjacency[b + k] = nbr[size_t(i) * cap + k];
}

__global__ void duplicates_kernel(const float *__restrict__ points, uint32_t n, uint32_t *__restrict__ status) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i + 1 >= n) return;
    const float *a = points + 3 * size_t(i);
    if (a[0] == a[3] && a[1] == a[4] && a[2] == a[5]) atomicAdd(status + kStDuplicate, 1u);
}

// The cells' site order.  A cell's candidates come from a k-nearest search
// over an AABB tree whose leaves pair consecutive sites; the caller's
// sort_points order ends in 1024-site blocks sorted along one axis, whose
// leaf boxes are long sticks, so the cells use the Morton order of the sites
// (21 bits per axis over the sites' bounding box), where a node's sites form
// a compact region and a site's index neighbours are also its spatial ones.
__device__ __forceinline__ uint64_t spread21(uint32_t v) {
    uint64_t x = v & 0x1fffffu;
    x = (x | (x << 32)) & 0x1f00000000ffffull;
    x = (x | (x << 16)) & 0x1f0000ff0000ffull;
    x = (x | (x << 8)) & 0x100f00f00f00f00full;
    x = (x | (x << 4)) & 0x10c30c30c30c30c3ull;
    x = (x | (x << 2)) & 0x1249249249249249ull;
    return x;
}

__global__ void __launch_bounds__(256) morton_kernel(const float *__restrict__ points, uint32_t n, float lox,
                                                     float loy, float loz, float scale, uint32_t *__restrict__ low,
                                                     uint32_t *__restrict__ high, uint32_t *__restrict__ idx) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float lo[3] = {lox, loy, loz};
    uint64_t code = 0;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float q = (__ldg(points + 3 * size_t(i) + k) - lo[k]) * scale;
        const uint32_t c = q > 0.0f ? static_cast<uint32_t>(fminf(q, 2097151.0f)) : 0u;
        code |= spread21(c) << k;
    }
    low[i] = static_cast<uint32_t>(code);
    high[i] = static_cast<uint32_t>(code >> 32);
    idx[i] = i;
}

__global__ void __launch_bounds__(256) gather_keys_kernel(const uint32_t *__restrict__ src,
                                                          const uint32_t *__restrict__ idx, uint32_t n,
                                                          uint32_t *__restrict__ dst) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = src[min(idx[i], n - 1)];
}

__global__ void __launch_bounds__(256) gather_points_kernel(const float *__restrict__ points,
                                                            const uint32_t *__restrict__ idx, uint32_t n,
                                                            float *__restrict__ out) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const size_t j = min(idx[i], n - 1);
#pragma unroll
    for (int k = 0; k < 3; ++k) out[3 * size_t(i) + k] = __ldg(points + 3 * j + k);
}

}  // namespace

DelaunayLayout delaunay_layout(uint32_t n) {
    DelaunayLayout l{};
    const uint32_t cap = kDelaunayCap;
    const uint32_t tiles = (n + kScanTile - 1) / kScanTile;
    l.nbr = 0;
    l.cnt = align_up(l.nbr + size_t(n) * cap * 4, 256);
    l.prefix = align_up(l.cnt + size_t(n) * 4, 256);
    l.sums = align_up(l.prefix + (size_t(n) + 1) * 4, 256);
    l.dirty = align_up(l.sums + size_t(tiles + 1) * 4, 256);
    l.extra = align_up(l.dirty + size_t(n) * 4, 256);
    l.extra_cap = n;
    l.status = align_up(l.extra + size_t(l.extra_cap) * 8, 256);
    l.retry_cap = n;
    l.retry = align_up(l.status + 64, 256);
    l.large = align_up(l.retry + size_t(l.retry_cap) * 4, 256);
    l.order = align_up(l.large + size_t(kLargeSlots) * sizeof(LargeCell), 256);
    l.mpoints = align_up(l.order + size_t(n) * 4, 256);
    l.mtree = align_up(l.mpoints + size_t(n) * 12, 256);
    l.total = align_up(l.mtree + size_t(pow2_round_up(n)) * 24, 256);
    // sort scratch inside the neighbour lists (n * 1 KB)
    const size_t arr = align_up(size_t(n) * 4, 256);
    l.keys_a = l.nbr;
    l.keys_b = l.keys_a + arr;
    l.vals_b = l.keys_b + arr;
    l.high = l.vals_b + arr;
    l.hist = l.high + arr;
    l.totals = align_up(l.hist + radix_hist_entries(n) * 4, 256);
    return l;
}

cudaError_t launch_delaunay_neighbors(const float *points, uint32_t n, const float *tree, void *workspace,
                                      uint32_t *offsets, cudaStream_t stream, const char **failed_stage) {
    const DelaunayLayout l = delaunay_layout(n);
    char *ws = static_cast<char *>(workspace);
    uint32_t *nbr = reinterpret_cast<uint32_t *>(ws + l.nbr);
    uint32_t *cnt = reinterpret_cast<uint32_t *>(ws + l.cnt);
    uint32_t *prefix = reinterpret_cast<uint32_t *>(ws + l.prefix);
    uint32_t *sums = reinterpret_cast<uint32_t *>(ws + l.sums);
    uint32_t *dirty = reinterpret_cast<uint32_t *>(ws + l.dirty);
    uint2 *extra = reinterpret_cast<uint2 *>(ws + l.extra);
    uint32_t *status = reinterpret_cast<uint32_t *>(ws + l.status);
    uint32_t *retry = reinterpret_cast<uint32_t *>(ws + l.retry);
    LargeCell *large = reinterpret_cast<LargeCell *>(ws + l.large);
    cudaError_t e = cudaMemsetAsync(status, 0, 64, stream);
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(dirty, 0, size_t(n) * 4, stream);
    if (e != cudaSuccess) return e;
    duplicates_kernel<<<(n + 255) / 256, 256, 0, stream>>>(points, n, status);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;

    CellParams P{};
    P.tree.points = points;
    P.tree.boxes = tree;
    P.tree.num_points = n;
    P.tree.num_leaves = pow2_round_up(n) / 2;
    P.tree.levels = 0;
    for (uint32_t w = P.tree.num_leaves; w >= 1; w >>= 1) ++P.tree.levels;
    P.cap = kDelaunayCap;
    P.nbr = nbr;
    P.cnt = cnt;
    P.status = status;
    uint32_t *order = reinterpret_cast<uint32_t *>(ws + l.order);
    float *mpoints = reinterpret_cast<float *>(ws + l.mpoints);
    float *mtree = reinterpret_cast<float *>(ws + l.mtree);
    // the box: the root node's bounds (read back once; the tree is tiny next
    // to the cell work) grown by 10^10 times the extent
    float root[6];
    const size_t root_off = 6 * (2 * size_t(P.tree.num_leaves) - 2);
    e = cudaMemcpyAsync(root, tree + root_off, sizeof(root), cudaMemcpyDeviceToHost, stream);
    if (e != cudaSuccess) return e;
    e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return e;
    double ext = 0.0;
    for (int k = 0; k < 3; ++k) ext = ext > double(root[3 + k]) - root[k] ? ext : double(root[3 + k]) - root[k];
    const double grow = 1e10 * (ext + 1e-3);
    for (int k = 0; k < 3; ++k) {
        P.lo[k] = double(root[k]) - grow;
        P.hi[k] = double(root[3 + k]) + grow;
    }
    // each stage is checked before the next starts, so that an error names
    // the stage that raised it (a rebuild already waits for the host twice)
    auto stage = [&](const char *name) -> cudaError_t {
        cudaError_t err = cudaGetLastError();
        if (err == cudaSuccess) err = cudaStreamSynchronize(stream);
        if (err != cudaSuccess && failed_stage) *failed_stage = name;
        return err;
    };
    // the cells' order: Morton codes as (low, high) halves, sorted by the low
    // half and then stably by the high half; the sites gathered in that order
    // and their tree
    {
        uint32_t *keys[2] = {reinterpret_cast<uint32_t *>(ws + l.keys_a), reinterpret_cast<uint32_t *>(ws + l.keys_b)};
        uint32_t *vals[2] = {order, reinterpret_cast<uint32_t *>(ws + l.vals_b)};
        uint32_t *high = reinterpret_cast<uint32_t *>(ws + l.high);
        uint32_t *hist = reinterpret_cast<uint32_t *>(ws + l.hist);
        uint32_t *totals = reinterpret_cast<uint32_t *>(ws + l.totals);
        const float scale = static_cast<float>(2097151.0 / (ext > 0.0 ? ext : 1.0));
        morton_kernel<<<(n + 255) / 256, 256, 0, stream>>>(points, n, root[0], root[1], root[2], scale, keys[0], high,
                                                           vals[0]);
        int cur = 0;
        if ((e = launch_radix_sort_pairs(keys, vals, n, hist, totals, cur, stream)) != cudaSuccess) return e;
        gather_keys_kernel<<<(n + 255) / 256, 256, 0, stream>>>(high, vals[cur], n, keys[cur]);
        if ((e = launch_radix_sort_pairs(keys, vals, n, hist, totals, cur, stream)) != cudaSuccess) return e;
        // eight passes end where they started: the order is in vals[0]
        gather_points_kernel<<<(n + 255) / 256, 256, 0, stream>>>(points, order, n, mpoints);
        if ((e = launch_build_aabb_tree(mpoints, n, mtree, stream)) != cudaSuccess) return e;
        if ((e = stage("site order")) != cudaSuccess) return e;
    }
    P.tree.points = mpoints;
    P.tree.boxes = mtree;
    P.to_out = order;
    P.retry = retry;
    P.retry_cap = l.retry_cap;
    voronoi_cells_kernel<<<(n + 63) / 64, 64, 0, stream>>>(P);
    if ((e = stage("voronoi cells")) != cudaSuccess) return e;
    voronoi_large_cells_kernel<<<kLargeSlots / 64, 64, 0, stream>>>(P, large);
    if ((e = stage("large voronoi cells")) != cudaSuccess) return e;
    asymmetry_kernel<<<(n + 255) / 256, 256, 0, stream>>>(nbr, cnt, n, kDelaunayCap, extra, l.extra_cap, status);
    // the asymmetric count is read on the device by the next two launches
    add_extra_kernel<<<(l.extra_cap + 255) / 256, 256, 0, stream>>>(extra, n, status, l.extra_cap, nbr, cnt,
                                                                      kDelaunayCap, dirty, status);
    sort_dirty_kernel<<<(n + 255) / 256, 256, 0, stream>>>(nbr, cnt, n, kDelaunayCap, dirty);
    if ((e = stage("symmetry")) != cudaSuccess) return e;
    const uint32_t tiles = (n + kScanTile - 1) / kScanTile;
    tile_sums_kernel<<<tiles, kScanBlock, 0, stream>>>(cnt, n, sums);
    scan_sums_kernel<<<1, 1024, 0, stream>>>(sums, tiles);
    tile_scan_kernel<<<tiles, kScanBlock, 0, stream>>>(cnt, n, sums, prefix);
    uint32_t *last = status + kStLastRow;
    last_row_kernel<<<(n + 255) / 256, 256, 0, stream>>>(cnt, n, last);
    offsets_kernel<<<(n + 1 + 255) / 256, 256, 0, stream>>>(cnt, prefix, n, last, offsets);
    return stage("offsets");
}

size_t scan_partials(uint32_t n) { return size_t((n + kScanTile - 1) / kScanTile) + 1; }

cudaError_t launch_exclusive_scan(const uint32_t *cnt, uint32_t n, uint32_t *sums, uint32_t *prefix,
                                  cudaStream_t stream) {
    const uint32_t tiles = (n + kScanTile - 1) / kScanTile;
    if (n == 0) return cudaMemsetAsync(prefix, 0, 4, stream);
    tile_sums_kernel<<<tiles, kScanBlock, 0, stream>>>(cnt, n, sums);
    scan_sums_kernel<<<1, 1024, 0, stream>>>(sums, tiles);
    tile_scan_kernel<<<tiles, kScanBlock, 0, stream>>>(cnt, n, sums, prefix);
    return cudaGetLastError();
}

cudaError_t launch_delaunay_adjacency(const void *workspace, uint32_t n, uint32_t *adjacency,
                                      uint32_t adjacency_size, cudaStream_t stream) {
    const DelaunayLayout l = delaunay_layout(n);
    const char *ws = static_cast<const char *>(workspace);
    fill_kernel<<<(n + 255) / 256, 256, 0, stream>>>(
        reinterpret_cast<const uint32_t *>(ws + l.nbr), reinterpret_cast<const uint32_t *>(ws + l.cnt),
        reinterpret_cast<const uint32_t *>(ws + l.prefix), n, kDelaunayCap, adjacency, adjacency_size);
    return cudaGetLastError();
}

}  // namespace sdfoam_b200
