// sort_points: the site permutation that puts spatially close sites next to
// each other (the reference's sort_points, src/aabb_tree/aabb_tree.cu:62-190,
// run before every Delaunay rebuild and AABB-tree build).
//
// Keys are the float bits of one coordinate made order-preserving as u32
// (sign set -> all bits flipped, else the sign bit flipped; aabb_tree.cu:
// 79-92).  Rounds r = 0, 1, ... use axis r mod 3 and a segment size that
// starts at pow2(N) and halves each round until it reaches 1.  Per round the
// reference sorts stably by that key
//   * all N sites at once while segments exceed 1024 sites and there are at
//     most 1024 of them (aabb_tree.cu:135-152: the segment structure of the
//     previous round is not kept),
//   * within each segment [s seg, min((s+1) seg, N)) while segments exceed
//     1024 sites and there are more than 1024 of them (aabb_tree.cu:107-134),
//   * within each block of 1024 consecutive sites once segments have at most
//     1024 sites (aabb_tree.cu:154-163; whole blocks, whatever the segment
//     size).
// The result is defined by stability alone, so any stable sort reproduces it.
//
// Here: rounds on large units are a least-significant-digit radix sort, four
// passes of 8-bit digits over 2048-site tiles (histogram; scan of each
// digit's tile counts per unit, a warp per digit; ranked scatter, which
// scans the unit's digit totals itself).  Units are whole tiles, so a pass never moves a site out
// of its unit.  All block rounds run in one launch: a 1024-thread block keeps
// its sites in shared memory and sorts (key, position) pairs -- unique, so a
// bitonic network gives the stable order -- once per round.
#include <algorithm>
#include <cstdint>

#include "foam_internal.h"

namespace sdfoam_b200 {

namespace {

constexpr int kThreads = 256;
constexpr int kItems = 8;
constexpr uint32_t kTile = kThreads * kItems;  // 2048 sites per tile
constexpr uint32_t kBlockSort = 1024;          // the reference's SORT_BLOCK_SIZE

__device__ __forceinline__ uint32_t order_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u ^ 0x80000000u);
}

// keys[i] = order key of coordinate dim of site perm[i] (perm NULL: identity,
// and vals[i] = i is written for the first round).
__global__ void __launch_bounds__(256) round_keys_kernel(const float *__restrict__ points,
                                                         const uint32_t *__restrict__ perm, uint32_t n, int dim,
                                                         uint32_t *__restrict__ keys, uint32_t *__restrict__ vals) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t src = i;
    if (perm) {
        src = min(perm[i], n - 1);  // a permutation of [0, n); the clamp keeps every gather in bounds
    } else {
        vals[i] = i;
    }
    keys[i] = order_key(__ldg(points + 3 * size_t(src) + dim));
}

// Digit counts of one tile, stored unit-major then digit-major:
// hist[(unit * 256 + digit) * tiles_per_unit + tile_in_unit].
__global__ void __launch_bounds__(kThreads) radix_hist_kernel(const uint32_t *__restrict__ keys, uint32_t n, int shift,
                                                              uint32_t tiles_per_unit, uint32_t *__restrict__ hist) {
    __shared__ uint32_t cnt[256];
    const uint32_t tid = threadIdx.x;
    cnt[tid] = 0;
    __syncthreads();
    const size_t base = size_t(blockIdx.x) * kTile;
#pragma unroll
    for (int r = 0; r < kItems; ++r) {
        const size_t i = base + r * kThreads + tid;
        if (i < n) atomicAdd(&cnt[(keys[i] >> shift) & 255u], 1u);
    }
    __syncthreads();
    const uint32_t unit = blockIdx.x / tiles_per_unit, t = blockIdx.x % tiles_per_unit;
    hist[(size_t(unit) * 256 + tid) * tiles_per_unit + t] = cnt[tid];
}

// Exclusive scan of each (unit, digit) row of tile counts, one warp per row:
// hist[row * tiles_per_unit + t] becomes the number of sites with that digit
// in the unit's tiles before t, and totals[row] the row's sum.  Counts of
// tiles past the end are zero.
__global__ void __launch_bounds__(256) radix_scan_kernel(uint32_t *__restrict__ hist, uint32_t *__restrict__ totals,
                                                         uint32_t rows, uint32_t num_tiles,
                                                         uint32_t tiles_per_unit) {
    const uint32_t row = blockIdx.x * 8 + (threadIdx.x >> 5);
    const uint32_t lane = threadIdx.x & 31;
    if (row >= rows) return;
    const uint32_t unit = row / 256;
    const uint32_t first_tile = unit * tiles_per_unit;
    const uint32_t valid = min(tiles_per_unit, num_tiles > first_tile ? num_tiles - first_tile : 0u);
    uint32_t *h = hist + size_t(row) * tiles_per_unit;
    const uint32_t per = (valid + 31) / 32;
    const uint32_t beg = min(valid, lane * per), end = min(valid, beg + per);
    uint32_t sum = 0;
    for (uint32_t t = beg; t < end; ++t) sum += h[t];
    uint32_t incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= uint32_t(o)) incl += y;
    }
    uint32_t run = incl - sum;
    for (uint32_t t = beg; t < end; ++t) {
        const uint32_t c = h[t];
        h[t] = run;
        run += c;
    }
    if (lane == 31) totals[row] = incl;
}

// Stable scatter of one tile by its digit: items are taken in site order
// (rows of 256 threads), ranked within a warp by __match_any_sync and across
// the block's warps through shared per-warp digit counts.
__global__ void __launch_bounds__(kThreads) radix_scatter_kernel(const uint32_t *__restrict__ keys_in,
                                                                 const uint32_t *__restrict__ vals_in,
                                                                 uint32_t *__restrict__ keys_out,
                                                                 uint32_t *__restrict__ vals_out,
                                                                 const uint32_t *__restrict__ offsets,
                                                                 const uint32_t *__restrict__ totals, uint32_t n,
                                                                 int shift, uint32_t tiles_per_unit,
                                                                 uint32_t unit_sites) {
    constexpr int kWarps = kThreads / 32;
    __shared__ uint32_t base[256];
    __shared__ uint32_t wcnt[kWarps][256];
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t unit = blockIdx.x / tiles_per_unit, t = blockIdx.x % tiles_per_unit;
    // first slot of digit tid in this tile: the unit's first site, the sites
    // of smaller digits in the unit (block scan of the digit totals), and the
    // sites of this digit in the unit's earlier tiles
    const uint32_t tot = totals[size_t(unit) * 256 + tid];
    uint32_t incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= uint32_t(o)) incl += y;
    }
    if (lane == 31) wcnt[0][warp] = incl;
    __syncthreads();
    uint32_t before = 0;
    for (uint32_t w = 0; w < warp; ++w) before += wcnt[0][w];
    __syncthreads();
    base[tid] = unit * unit_sites + before + (incl - tot) + offsets[(size_t(unit) * 256 + tid) * tiles_per_unit + t];
#pragma unroll
    for (int w = 0; w < kWarps; ++w) wcnt[w][tid] = 0;
    __syncthreads();
    const uint32_t lt = (1u << lane) - 1u;
    const size_t tile0 = size_t(blockIdx.x) * kTile;
    for (int r = 0; r < kItems; ++r) {
        const size_t i = tile0 + r * kThreads + tid;
        const bool valid = i < n;
        const uint32_t k = valid ? keys_in[i] : 0u;
        const uint32_t v = valid ? vals_in[i] : 0u;
        const uint32_t d = (k >> shift) & 255u;
        const uint32_t peers = __match_any_sync(0xffffffffu, valid ? d : 0x100u | lane);
        const uint32_t rank = __popc(peers & lt);
        if (valid && (peers & lt) == 0) wcnt[warp][d] = __popc(peers);
        __syncthreads();
        if (valid) {
            uint32_t pos = base[d] + rank;
            for (uint32_t w = 0; w < warp; ++w) pos += wcnt[w][d];
            if (pos < n) {  // always true for consistent counts; keeps the store in bounds
                keys_out[pos] = k;
                vals_out[pos] = v;
            }
        }
        __syncthreads();
        uint32_t tot = 0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            tot += wcnt[w][tid];
            wcnt[w][tid] = 0;
        }
        base[tid] += tot;
        __syncthreads();
    }
}

// The block rounds: per 1024-site block, `rounds` stable sorts by the axes
// dim0, dim0 + 1, ... (mod 3), then the permutation and the sorted sites.
__global__ void __launch_bounds__(kBlockSort) block_rounds_kernel(const float *__restrict__ points,
                                                                  const uint32_t *__restrict__ perm_in, uint32_t n,
                                                                  int dim0, int rounds, float *__restrict__ sorted,
                                                                  uint32_t *__restrict__ perm_out) {
    __shared__ unsigned long long ck[kBlockSort];
    __shared__ uint32_t pv[kBlockSort];
    const uint32_t tid = threadIdx.x;
    const size_t i = size_t(blockIdx.x) * kBlockSort + tid;
    const bool valid = i < n;
    pv[tid] = valid ? (perm_in ? min(perm_in[i], n - 1) : uint32_t(i)) : 0u;
    __syncthreads();
    for (int r = 0; r < rounds; ++r) {
        const int dim = (dim0 + r) % 3;
        // padding sorts after every site, as the reference's 0xffffffff keys
        // behind the valid threads do
        const uint32_t key = valid ? order_key(__ldg(points + 3 * size_t(pv[tid]) + dim)) : 0xffffffffu;
        ck[tid] = (static_cast<unsigned long long>(key) << 32) | tid;
        __syncthreads();
        for (uint32_t k = 2; k <= kBlockSort; k <<= 1) {
            for (uint32_t j = k >> 1; j > 0; j >>= 1) {
                const uint32_t p = tid ^ j;
                if (p > tid) {
                    const unsigned long long a = ck[tid], b = ck[p];
                    if ((a > b) == ((tid & k) == 0)) {
                        ck[tid] = b;
                        ck[p] = a;
                    }
                }
                __syncthreads();
            }
        }
        const uint32_t moved = pv[ck[tid] & (kBlockSort - 1)];
        __syncthreads();
        pv[tid] = moved;
        __syncthreads();
    }
    if (valid) {
        const uint32_t src = pv[tid];
        perm_out[i] = src;
#pragma unroll
        for (int c = 0; c < 3; ++c) sorted[3 * i + c] = __ldg(points + 3 * size_t(src) + c);
    }
}

uint32_t tiles_of(uint32_t n) { return (n + kTile - 1) / kTile; }

// One round on units of `unit` sites (unit >= 2048, a power of two, or the
// whole array): tiles per unit and number of units.
struct RoundShape {
    uint32_t tiles_per_unit, units, unit_sites;
};

RoundShape round_shape(uint32_t n, uint32_t seg) {
    const uint32_t num_segments = static_cast<uint32_t>((uint64_t(n) + seg - 1) / seg);
    if (num_segments <= 1024) return {tiles_of(n), 1u, 0u};  // one global sort
    return {seg / kTile, num_segments, seg};
}

}  // namespace

SortLayout sort_layout(uint32_t n) {
    SortLayout l{};
    const size_t arr = align_up(size_t(n) * 4, 256);
    l.keys_a = 0;
    l.keys_b = arr;
    l.vals_a = 2 * arr;
    l.vals_b = 3 * arr;
    l.hist = 4 * arr;
    size_t hist_entries = 0, rows = 0;
    for (uint32_t seg = pow2_round_up(n); seg > kBlockSort; seg >>= 1) {
        const RoundShape s = round_shape(n, seg);
        hist_entries = std::max(hist_entries, size_t(256) * s.units * s.tiles_per_unit);
        rows = std::max(rows, size_t(256) * s.units);
    }
    l.totals = align_up(l.hist + hist_entries * 4, 256);
    l.total = align_up(l.totals + rows * 4, 256);
    return l;
}

size_t radix_hist_entries(uint32_t n) { return size_t(256) * tiles_of(n); }

cudaError_t launch_radix_sort_pairs(uint32_t *const keys[2], uint32_t *const vals[2], uint32_t n, uint32_t *hist,
                                    uint32_t *totals, int &cur, cudaStream_t stream) {
    const uint32_t num_tiles = tiles_of(n);
    for (int shift = 0; shift < 32; shift += 8) {
        radix_hist_kernel<<<num_tiles, kThreads, 0, stream>>>(keys[cur], n, shift, num_tiles, hist);
        radix_scan_kernel<<<256 / 8, 256, 0, stream>>>(hist, totals, 256, num_tiles, num_tiles);
        radix_scatter_kernel<<<num_tiles, kThreads, 0, stream>>>(keys[cur], vals[cur], keys[cur ^ 1], vals[cur ^ 1],
                                                                 hist, totals, n, shift, num_tiles, 0u);
        cur ^= 1;
    }
    return cudaGetLastError();
}

cudaError_t launch_sort_points(const float *points, uint32_t n, float *sorted, uint32_t *perm, void *workspace,
                               cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    const SortLayout l = sort_layout(n);
    char *ws = static_cast<char *>(workspace);
    uint32_t *keys[2] = {reinterpret_cast<uint32_t *>(ws + l.keys_a), reinterpret_cast<uint32_t *>(ws + l.keys_b)};
    uint32_t *vals[2] = {reinterpret_cast<uint32_t *>(ws + l.vals_a), reinterpret_cast<uint32_t *>(ws + l.vals_b)};
    uint32_t *hist = reinterpret_cast<uint32_t *>(ws + l.hist);
    uint32_t *totals = reinterpret_cast<uint32_t *>(ws + l.totals);
    const uint32_t num_tiles = tiles_of(n);
    uint32_t seg = pow2_round_up(n);
    int dim = 0;
    const uint32_t *cur_perm = nullptr;  // identity before the first round
    int cur = 0;
    for (; seg > kBlockSort; seg >>= 1) {
        const RoundShape s = round_shape(n, seg);
        round_keys_kernel<<<(n + 255) / 256, 256, 0, stream>>>(points, cur_perm, n, dim, keys[cur], vals[cur]);
        for (int shift = 0; shift < 32; shift += 8) {
            radix_hist_kernel<<<num_tiles, kThreads, 0, stream>>>(keys[cur], n, shift, s.tiles_per_unit, hist);
            const uint32_t rows = 256 * s.units;
            radix_scan_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(hist, totals, rows, num_tiles, s.tiles_per_unit);
            radix_scatter_kernel<<<num_tiles, kThreads, 0, stream>>>(keys[cur], vals[cur], keys[cur ^ 1],
                                                                     vals[cur ^ 1], hist, totals, n, shift,
                                                                     s.tiles_per_unit, s.unit_sites);
            cur ^= 1;
        }
        cur_perm = vals[cur];
        dim = (dim + 1) % 3;
    }
    int rounds = 0;
    for (; seg > 1; seg >>= 1) ++rounds;
    block_rounds_kernel<<<(n + kBlockSort - 1) / kBlockSort, kBlockSort, 0, stream>>>(points, cur_perm, n, dim,
                                                                                      rounds, sorted, perm);
    return cudaGetLastError();
}

}  // namespace sdfoam_b200
