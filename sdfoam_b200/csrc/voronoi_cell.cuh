// One Voronoi cell per call: the per-site work of the Delaunay adjacency
// (delaunay.cu has the method).  Plain C++ apart from the three macros below,
// so the same code also compiles for the host.
#pragma once

#include <cfloat>
#include <cmath>
#include <cstdint>
#include <type_traits>

#ifdef __CUDACC__
#define VC_HD __device__
#define VC_INLINE __forceinline__
template <typename T>
__device__ __forceinline__ T vc_ldg(const T *p) { return __ldg(p); }
__device__ __forceinline__ void vc_count(uint32_t *p) { atomicAdd(p, 1u); }
__device__ __forceinline__ uint32_t vc_fetch_add(uint32_t *p) { return atomicAdd(p, 1u); }
// first self-check failure: guard[0] = code, guard[1] = the index
__device__ __forceinline__ void vc_record(uint32_t *guard, uint32_t code, uint64_t idx) {
    if (atomicCAS(guard, 0u, code) == 0u) guard[1] = static_cast<uint32_t>(idx);
}
#else
#define VC_HD
#define VC_INLINE inline
template <typename T>
inline T vc_ldg(const T *p) { return *p; }
inline void vc_count(uint32_t *p) { ++*p; }
inline uint32_t vc_fetch_add(uint32_t *p) { return (*p)++; }
inline void vc_record(uint32_t *guard, uint32_t code, uint64_t idx) {
    if (guard[0] == 0u) {
        guard[0] = code;
        guard[1] = static_cast<uint32_t>(idx);
    }
}
#endif

#ifndef VC_TRACE
#define VC_TRACE(...) ((void)0)
#endif

namespace sdfoam_b200 {
namespace voronoi {

constexpr uint32_t kNoSite = 0xffffffffu;

constexpr int kSmallPlanes = 128;         // plane slots of a first-pass cell (box included)
constexpr int kLargePlanes = 262;         // ... of a second-pass cell: 256 neighbours + the box
constexpr int kK1 = 64, kK2 = 121;        // candidates of the two tiers
constexpr int kSkip = 16;                 // sites whose clip was a rounding no-op
constexpr uint32_t kBoxId = 0xfffffff0u;  // plane ids of the six box faces: kBoxId + k
constexpr int kStack = 64;

enum Status {
    kStFailed = 0,
    kStDuplicate = 1,
    kStAsymmetric = 2,
    kStOpenCells = 3,
    kStGuard = 4,   // and 5: self-check code and index
    kStRetry = 6,   // cells handed to the second pass
    kStLastRow = 8,
};

// A convex cell with room for P planes: a cell with F faces has 2F - 4
// vertices, and a deleted patch has at most as many boundary edges.
template <int P>
struct CellT {
    static constexpr int kPlanes = P, kTris = 2 * P, kEdges = 2 * P;
    static constexpr int kMaxChecks = 8 * kTris;  // vertex checks of one open cell
    using Idx = typename std::conditional<(P <= 255), unsigned char, uint16_t>::type;
    double nx[P], ny[P], nz[P], w[P];  // n . x <= w
    uint32_t pid[P];
    Idx tri[kTris][3];
    unsigned char flag[kTris];  // bit 0: verified vertex, bit 1: scratch mark
    double vx[kTris], vy[kTris], vz[kTris];
    int np, nt;
    bool bad;         // a self-check failed: the cell is abandoned
    uint32_t *guard;  // where the first failure is recorded
};
using SmallCell = CellT<kSmallPlanes>;
using LargeCell = CellT<kLargePlanes>;

// Self-check of an index before the access it guards: records the failure,
// abandons the cell and tells the caller to skip the access.
template <class Cell>
VC_HD VC_INLINE bool oob(Cell &C, uint32_t code, uint64_t idx, uint64_t limit) {
    if (idx < limit) return false;
    vc_record(C.guard, code, idx);
    C.bad = true;
    return true;
}

VC_HD VC_INLINE bool is_box(uint32_t id) { return id >= kBoxId; }

template <class Cell>
VC_HD void vertex_of(Cell &C, int t) {
    if (oob(C, 1, t, Cell::kTris)) return;
    const int a = C.tri[t][0], b = C.tri[t][1], c = C.tri[t][2];
    if (oob(C, 2, a, C.np) || oob(C, 2, b, C.np) || oob(C, 2, c, C.np)) return;
    // v = (w_a (n_b x n_c) + w_b (n_c x n_a) + w_c (n_a x n_b)) / (n_a . (n_b x n_c))
    const double bcx = C.ny[b] * C.nz[c] - C.nz[b] * C.ny[c];
    const double bcy = C.nz[b] * C.nx[c] - C.nx[b] * C.nz[c];
    const double bcz = C.nx[b] * C.ny[c] - C.ny[b] * C.nx[c];
    const double cax = C.ny[c] * C.nz[a] - C.nz[c] * C.ny[a];
    const double cay = C.nz[c] * C.nx[a] - C.nx[c] * C.nz[a];
    const double caz = C.nx[c] * C.ny[a] - C.ny[c] * C.nx[a];
    const double abx = C.ny[a] * C.nz[b] - C.nz[a] * C.ny[b];
    const double aby = C.nz[a] * C.nx[b] - C.nx[a] * C.nz[b];
    const double abz = C.nx[a] * C.ny[b] - C.ny[a] * C.nx[b];
    const double det = C.nx[a] * bcx + C.ny[a] * bcy + C.nz[a] * bcz;
    const double inv = 1.0 / det;
    C.vx[t] = (C.w[a] * bcx + C.w[b] * cax + C.w[c] * abx) * inv;
    C.vy[t] = (C.w[a] * bcy + C.w[b] * cay + C.w[c] * aby) * inv;
    C.vz[t] = (C.w[a] * bcz + C.w[b] * caz + C.w[c] * abz) * inv;
}

// The box [lo, hi] relative to the site, as the octahedral dual of a cube:
// planes 0..5 = +x, -x, +y, -y, +z, -z; corner (sx, sy, sz) is the triangle of
// its three faces, ordered so that det(n_a, n_b, n_c) > 0.
template <class Cell>
VC_HD void init_box(Cell &C, const double lo[3], const double hi[3]) {
    C.np = 6;
    for (int k = 0; k < 3; ++k) {
        C.nx[2 * k] = C.ny[2 * k] = C.nz[2 * k] = 0.0;
        C.nx[2 * k + 1] = C.ny[2 * k + 1] = C.nz[2 * k + 1] = 0.0;
    }
    C.nx[0] = 1.0;
    C.nx[1] = -1.0;
    C.ny[2] = 1.0;
    C.ny[3] = -1.0;
    C.nz[4] = 1.0;
    C.nz[5] = -1.0;
    C.w[0] = hi[0];
    C.w[1] = -lo[0];
    C.w[2] = hi[1];
    C.w[3] = -lo[1];
    C.w[4] = hi[2];
    C.w[5] = -lo[2];
    for (int k = 0; k < 6; ++k) C.pid[k] = kBoxId + k;
    C.nt = 0;
    for (int s = 0; s < 8; ++s) {
        const int sx = s & 1, sy = (s >> 1) & 1, sz = (s >> 2) & 1;  // 0: +, 1: -
        const int px = sx, py = 2 + sy, pz = 4 + sz;
        const int neg = sx + sy + sz;
        C.tri[C.nt][0] = static_cast<unsigned char>(px);
        if (neg % 2 == 0) {
            C.tri[C.nt][1] = static_cast<unsigned char>(py);
            C.tri[C.nt][2] = static_cast<unsigned char>(pz);
        } else {
            C.tri[C.nt][1] = static_cast<unsigned char>(pz);
            C.tri[C.nt][2] = static_cast<unsigned char>(py);
        }
        C.flag[C.nt] = 0;
        vertex_of(C, C.nt);
        ++C.nt;
    }
}

// Drops plane slots no vertex uses.  Returns the number of slots freed.
template <class Cell>
VC_HD int compact_planes(Cell &C) {
    unsigned char used[Cell::kPlanes];
    typename Cell::Idx remap[Cell::kPlanes];
    for (int s = 0; s < C.np; ++s) used[s] = 0;
    for (int t = 0; t < C.nt; ++t)
        for (int e = 0; e < 3; ++e) {
            if (oob(C, 3, C.tri[t][e], C.np)) return 0;
            used[C.tri[t][e]] = 1;
        }
    int k = 0;
    for (int s = 0; s < C.np; ++s) {
        if (!used[s]) continue;
        remap[s] = static_cast<typename Cell::Idx>(k);
        C.nx[k] = C.nx[s];
        C.ny[k] = C.ny[s];
        C.nz[k] = C.nz[s];
        C.w[k] = C.w[s];
        C.pid[k] = C.pid[s];
        ++k;
    }
    const int freed = C.np - k;
    C.np = k;
    for (int t = 0; t < C.nt; ++t)
        for (int e = 0; e < 3; ++e) C.tri[t][e] = remap[C.tri[t][e]];
    return freed;
}

// Clips the cell by n . x <= w (the bisector of the site and site id).
// Returns 1 if the plane cut the cell, 0 if no vertex lies beyond it, -1 when
// a capacity is exceeded (the cell is then left unchanged).
template <class Cell>
VC_HD int clip(Cell &C, double nx, double ny, double nz, double w, uint32_t id) {
    if (C.bad || oob(C, 4, C.nt, Cell::kTris + 1) || oob(C, 4, C.np, Cell::kPlanes + 1)) return -1;
    int nmark = 0;
    for (int t = 0; t < C.nt; ++t) {
        const bool out = nx * C.vx[t] + ny * C.vy[t] + nz * C.vz[t] > w;
        C.flag[t] = static_cast<unsigned char>((C.flag[t] & 1u) | (out ? 2u : 0u));
        nmark += out;
    }
    if (nmark == 0) return 0;
    VC_TRACE("clip id %u: np %d nt %d nmark %d\n", id, C.np, C.nt, nmark);
    if (nmark == C.nt) return -1;  // impossible for a cell that contains its site
    if (C.np == Cell::kPlanes) {
        compact_planes(C);
        if (C.np == Cell::kPlanes) return -1;
    }
    // boundary of the deleted patch: directed edges of deleted vertices whose
    // reverse is not also an edge of a deleted vertex
    typename Cell::Idx ea[Cell::kEdges], eb[Cell::kEdges];
    int ne = 0;
    for (int t = 0; t < C.nt; ++t) {
        if (!(C.flag[t] & 2u)) continue;
        for (int e = 0; e < 3; ++e) {
            const typename Cell::Idx a = C.tri[t][e], b = C.tri[t][(e + 1) % 3];
            int r = -1;
            for (int k = 0; k < ne; ++k)
                if (ea[k] == b && eb[k] == a) {
                    r = k;
                    break;
                }
            if (r >= 0) {
                --ne;
                ea[r] = ea[ne];
                eb[r] = eb[ne];
            } else {
                if (ne == Cell::kEdges) return -1;
                ea[ne] = a;
                eb[ne] = b;
                ++ne;
            }
        }
    }
    VC_TRACE("   boundary edges %d\n", ne);
    if (C.nt - nmark + ne > Cell::kTris) return -1;
    if (oob(C, 6, C.np, Cell::kPlanes)) return -1;
    const int s = C.np++;
    C.nx[s] = nx;
    C.ny[s] = ny;
    C.nz[s] = nz;
    C.w[s] = w;
    C.pid[s] = id;
    int k = 0;
    for (int t = 0; t < C.nt; ++t) {
        if (C.flag[t] & 2u) continue;
        if (k != t) {
            C.tri[k][0] = C.tri[t][0];
            C.tri[k][1] = C.tri[t][1];
            C.tri[k][2] = C.tri[t][2];
            C.vx[k] = C.vx[t];
            C.vy[k] = C.vy[t];
            C.vz[k] = C.vz[t];
        }
        C.flag[k] = C.flag[t] & 1u;
        ++k;
    }
    C.nt = k;
    for (int e = 0; e < ne; ++e) {
        // the kept neighbour holds (b, a): the new vertex holds (a, b)
        if (oob(C, 5, C.nt, Cell::kTris)) return -1;
        C.tri[C.nt][0] = ea[e];
        C.tri[C.nt][1] = eb[e];
        C.tri[C.nt][2] = static_cast<typename Cell::Idx>(s);
        C.flag[C.nt] = 0;
        vertex_of(C, C.nt);
        ++C.nt;
    }
    return 1;
}

// Clip by the bisector of the site (origin) and q (relative position).
template <class Cell>
VC_HD VC_INLINE int clip_site(Cell &C, double qx, double qy, double qz, uint32_t id) {
    return clip(C, qx, qy, qz, 0.5 * (qx * qx + qy * qy + qz * qz), id);
}

template <class Cell>
VC_HD VC_INLINE double radius2(const Cell &C) {
    double r = 0.0;
    for (int t = 0; t < C.nt; ++t) r = fmax(r, C.vx[t] * C.vx[t] + C.vy[t] * C.vy[t] + C.vz[t] * C.vz[t]);
    return r;
}

// --------------------------------------------------------------------------
// AABB-tree queries (tree layout of aabb.cu: levels leaves first, leaf j
// covers sites 2j, 2j + 1)
// --------------------------------------------------------------------------

struct Tree {
    const float *points;
    const float *boxes;
    uint32_t num_points, num_leaves, levels;
};

VC_HD VC_INLINE uint64_t level_offset(const Tree &T, uint32_t L) {
    uint64_t off = 0;
    for (uint32_t l = 0; l < L; ++l) off += T.num_leaves >> l;
    return off;
}

// Child `child` of a level-L node (it sits on level L - 1) covers the sites
// from child << L on.  Past the last site the leaves are padding whose boxes
// repeat the last site: a search near that site would otherwise walk the whole
// padding subtree (up to half the tree), so such children are never entered.
VC_HD VC_INLINE bool real_child(const Tree &T, uint32_t L, uint32_t child) {
    return (uint64_t(child) << L) < T.num_points;
}

VC_HD VC_INLINE float box_dist2(const float *box, float x, float y, float z) {
    const float gx = fmaxf(fmaxf(vc_ldg(box + 0) - x, x - vc_ldg(box + 3)), 0.0f);
    const float gy = fmaxf(fmaxf(vc_ldg(box + 1) - y, y - vc_ldg(box + 4)), 0.0f);
    const float gz = fmaxf(fmaxf(vc_ldg(box + 2) - z, z - vc_ldg(box + 5)), 0.0f);
    return gx * gx + gy * gy + gz * gz;
}

// Candidate order: nearer first, ties to the lower index.
VC_HD VC_INLINE bool farther(float da, uint32_t ia, float db, uint32_t ib) {
    return da > db || (da == db && ia > ib);
}

// The k candidates kept so far as a max-heap on (distance, index): entry 0 is
// the farthest.  Adds (d, i), dropping the farthest once k are kept.
VC_HD VC_INLINE void heap_offer(float *kd, uint32_t *ki, int &cnt, int k, float d, uint32_t i) {
    int j;
    if (cnt < k) {
        j = cnt++;
        while (j > 0) {
            const int up = (j - 1) >> 1;
            if (!farther(d, i, kd[up], ki[up])) break;
            kd[j] = kd[up];
            ki[j] = ki[up];
            j = up;
        }
    } else {
        if (!farther(kd[0], ki[0], d, i)) return;
        j = 0;
        for (;;) {
            int c = 2 * j + 1;
            if (c >= k) break;
            if (c + 1 < k && farther(kd[c + 1], ki[c + 1], kd[c], ki[c])) ++c;
            if (!farther(kd[c], ki[c], d, i)) break;
            kd[j] = kd[c];
            ki[j] = ki[c];
            j = c;
        }
    }
    kd[j] = d;
    ki[j] = i;
}

// The k nearest sites of site self, sorted nearer first (ties to the lower
// index); returns how many were found (< k only when the foam has fewer
// sites).  The heap starts from the 2k sites next to self in the tree's
// order, which in a spatial order bound the k-th distance closely, so the
// depth-first walk (nearer child first) prunes from its first node; it skips
// those sites when it meets them.  A final heap sort orders the result.
template <class Cell>
VC_HD int knn(Cell &C, const Tree &T, uint32_t self, float x, float y, float z, int k, float *kd, uint32_t *ki) {
    int cnt = 0;
    const uint32_t n = T.num_points;
    const uint32_t span = (uint32_t(2 * k) + 1 < n ? uint32_t(2 * k) + 1 : n);  // seeds + self
    uint32_t lo = self > span / 2 ? self - span / 2 : 0u;
    if (lo + span > n) lo = n - span;
    const uint32_t hi = lo + span;
    for (uint32_t i = lo; i < hi; ++i) {
        if (i == self) continue;
        const float dx = vc_ldg(T.points + 3 * size_t(i)) - x;
        const float dy = vc_ldg(T.points + 3 * size_t(i) + 1) - y;
        const float dz = vc_ldg(T.points + 3 * size_t(i) + 2) - z;
        heap_offer(kd, ki, cnt, k, dx * dx + dy * dy + dz * dz, i);
    }
    uint32_t stack[kStack];
    int sp = 0;
    stack[sp++] = ((T.levels - 1) << 27) | 0u;
    while (sp > 0) {
        const uint32_t e = stack[--sp];
        const uint32_t L = e >> 27, node = e & ((1u << 27) - 1);
        const float worst = cnt < k ? FLT_MAX : kd[0];
        if (L == 0) {
            for (uint32_t i = 2 * node; i < 2 * node + 2 && i < n; ++i) {
                if (i >= lo && i < hi) continue;  // self or a seed
                const float dx = vc_ldg(T.points + 3 * size_t(i)) - x;
                const float dy = vc_ldg(T.points + 3 * size_t(i) + 1) - y;
                const float dz = vc_ldg(T.points + 3 * size_t(i) + 2) - z;
                heap_offer(kd, ki, cnt, k, dx * dx + dy * dy + dz * dz, i);
            }
            continue;
        }
        const uint64_t off = level_offset(T, L - 1);
        if (oob(C, 7, off + 2 * size_t(node) + 1, 2 * size_t(T.num_leaves) - 1)) return 0;
        const float d0 = box_dist2(T.boxes + 6 * (off + 2 * size_t(node)), x, y, z);
        const float d1 = box_dist2(T.boxes + 6 * (off + 2 * size_t(node) + 1), x, y, z);
        const int nearer = d1 < d0 ? 1 : 0;
        const float dn = nearer ? d1 : d0, df = nearer ? d0 : d1;
        if (df <= worst && sp < kStack && real_child(T, L, 2 * node + 1 - nearer))
            stack[sp++] = ((L - 1) << 27) | (2 * node + 1 - nearer);
        if (dn <= worst && sp < kStack && real_child(T, L, 2 * node + nearer))
            stack[sp++] = ((L - 1) << 27) | (2 * node + nearer);
    }
    // heap sort: the farthest moves to the end
    for (int m = cnt - 1; m > 0; --m) {
        const float d = kd[m];
        const uint32_t i = ki[m];
        kd[m] = kd[0];
        ki[m] = ki[0];
        int j = 0;
        for (;;) {
            int c = 2 * j + 1;
            if (c >= m) break;
            if (c + 1 < m && farther(kd[c + 1], ki[c + 1], kd[c], ki[c])) ++c;
            if (!farther(kd[c], ki[c], d, i)) break;
            kd[j] = kd[c];
            ki[j] = ki[c];
            j = c;
        }
        kd[j] = d;
        ki[j] = i;
    }
    return cnt;
}

template <class Cell>
VC_HD VC_INLINE bool in_cell_or_skip(const Cell &C, const uint32_t *skip, int nskip, uint32_t i) {
    for (int s = 0; s < C.np; ++s)
        if (C.pid[s] == i) return true;
    for (int s = 0; s < nskip; ++s)
        if (skip[s] == i) return true;
    return false;
}

// The site nearest to the point p + (x, y, z) among those strictly closer to
// it than the site p itself, or kNoSite.  Double precision throughout.
template <class Cell>
VC_HD uint32_t nearest_closer(const Tree &T, Cell &C, const uint32_t *skip, int nskip, uint32_t self,
                                   const double p[3], double x, double y, double z) {
    double best = x * x + y * y + z * z;
    uint32_t cand = kNoSite;
    const double cx = p[0] + x, cy = p[1] + y, cz = p[2] + z;
    uint32_t stack[kStack];
    int sp = 0;
    stack[sp++] = ((T.levels - 1) << 27) | 0u;
    while (sp > 0) {
        const uint32_t e = stack[--sp];
        const uint32_t L = e >> 27, node = e & ((1u << 27) - 1);
        if (L == 0) {
            for (uint32_t i = 2 * node; i < 2 * node + 2 && i < T.num_points; ++i) {
                if (i == self) continue;
                const double dx = double(vc_ldg(T.points + 3 * size_t(i))) - cx;
                const double dy = double(vc_ldg(T.points + 3 * size_t(i) + 1)) - cy;
                const double dz = double(vc_ldg(T.points + 3 * size_t(i) + 2)) - cz;
                const double d = dx * dx + dy * dy + dz * dz;
                if (d < best && !in_cell_or_skip(C, skip, nskip, i)) {
                    best = d;
                    cand = i;
                }
            }
            continue;
        }
        const uint64_t off = level_offset(T, L - 1);
        if (oob(C, 8, off + 2 * size_t(node) + 1, 2 * size_t(T.num_leaves) - 1)) return kNoSite;
        double dc[2];
        for (int c = 0; c < 2; ++c) {
            const float *box = T.boxes + 6 * (off + 2 * size_t(node) + c);
            const double gx = fmax(fmax(double(vc_ldg(box + 0)) - cx, cx - double(vc_ldg(box + 3))), 0.0);
            const double gy = fmax(fmax(double(vc_ldg(box + 1)) - cy, cy - double(vc_ldg(box + 4))), 0.0);
            const double gz = fmax(fmax(double(vc_ldg(box + 2)) - cz, cz - double(vc_ldg(box + 5))), 0.0);
            dc[c] = gx * gx + gy * gy + gz * gz;
        }
        const int nearer = dc[1] < dc[0] ? 1 : 0;
        if (dc[1 - nearer] < best && sp < kStack && real_child(T, L, 2 * node + 1 - nearer))
            stack[sp++] = ((L - 1) << 27) | (2 * node + 1 - nearer);
        if (dc[nearer] < best && sp < kStack && real_child(T, L, 2 * node + nearer))
            stack[sp++] = ((L - 1) << 27) | (2 * node + nearer);
    }
    return cand;
}

// --------------------------------------------------------------------------
// one Voronoi cell per thread
// --------------------------------------------------------------------------

struct CellParams {
    Tree tree;
    double lo[3], hi[3];  // the box, absolute
    uint32_t cap;         // neighbour slots per site
    uint32_t *nbr;        // [N, cap]
    uint32_t *cnt;        // [N]
    uint32_t *status;     // [4]
    uint32_t *reason;     // optional [N]: why a cell failed (0 = it did not)
    uint32_t *retry;      // first pass: sites whose cell ran out of room, for the second pass
    uint32_t retry_cap;
    const uint32_t *to_out;  // optional [N]: the output index (row of nbr, cnt, reason; neighbour id) of tree site i
};

// Why a cell failed: the reason codes of CellParams::reason.
enum FailReason : uint32_t {
    kFailTierClip = 1,    // a capacity ran out while clipping the nearest candidates
    kFailOpenClip = 2,    // ... while clipping a site found by the vertex checks
    kFailChecks = 3,      // too many vertex checks
    kFailSkip = 4,        // too many sites whose clip was a rounding no-op
    kFailOutput = 5,      // more neighbours than the output row holds
    kFailSelfCheck = 6,   // an index self-check fired
};

template <class Cell>
VC_HD int clip_candidate(Cell &C, const Tree &T, const double p[3], uint32_t i, uint32_t *status) {
    if (oob(C, 9, i, T.num_points)) return -1;
    const double qx = double(vc_ldg(T.points + 3 * size_t(i))) - p[0];
    const double qy = double(vc_ldg(T.points + 3 * size_t(i) + 1)) - p[1];
    const double qz = double(vc_ldg(T.points + 3 * size_t(i) + 2)) - p[2];
    if (qx == 0.0 && qy == 0.0 && qz == 0.0) {
        vc_count(status + kStDuplicate);
        return 0;
    }
    return clip_site(C, qx, qy, qz, i);
}

// The cell of site at p (absolute, double) clipped by its nearest candidates
// in two tiers, closed by the security radius: returns false when a capacity
// ran out (reason set); done = the cell is final; r0 = the distance of the
// farthest candidate.
template <class Cell>
VC_HD bool build_tiers(const CellParams &P, uint32_t site, const double p[3], Cell &C, bool &done, double &r0,
                       uint32_t &reason) {
    const Tree &T = P.tree;
    float kd[kK2];
    uint32_t ki[kK2];
    const double lo[3] = {P.lo[0] - p[0], P.lo[1] - p[1], P.lo[2] - p[2]};
    const double hi[3] = {P.hi[0] - p[0], P.hi[1] - p[1], P.hi[2] - p[2]};
    C.bad = false;
    C.guard = P.status + kStGuard;
    init_box(C, lo, hi);
    bool ok = true;
    done = false;
    int seen = 0;
    const float fx = static_cast<float>(p[0]), fy = static_cast<float>(p[1]), fz = static_cast<float>(p[2]);
    for (int tier = 0; tier < 2 && ok && !done; ++tier) {
        const int k = tier == 0 ? kK1 : kK2;
        const int n = knn(C, T, site, fx, fy, fz, k, kd, ki);
        for (int j = seen; j < n && ok; ++j) ok = clip_candidate(C, T, p, ki[j], P.status) >= 0 && !C.bad;
        ok = ok && !C.bad;
        if (!ok && !reason) reason = kFailTierClip;
        seen = n;
        if (n < k) {
            done = true;  // every other site was a candidate
        } else if (ok) {
            const double r2 = radius2(C);
            done = 4.0 * r2 < double(kd[n - 1]) * (1.0 - 1e-5);
        }
    }
    r0 = seen > 0 ? sqrt(double(kd[seen - 1])) : 0.0;
    return ok;
}

// The site nearest to vertex t of an open cell among those closer to it than
// the cell's own site (skipping the cell's planes and the skip list), or
// kNoSite.  Any point of the segment from the site to a vertex lies in the
// cell, so a vertex on the box is probed first at 2 r0 along that segment,
// then 4 times farther each time up to the vertex itself.
template <class Cell>
VC_HD uint32_t probe_vertex(const Tree &T, Cell &C, const uint32_t *skip, int nskip, uint32_t site,
                            const double p[3], double r0, int t) {
    const bool on_box = is_box(C.pid[C.tri[t][0]]) || is_box(C.pid[C.tri[t][1]]) || is_box(C.pid[C.tri[t][2]]);
    const double vx = C.vx[t], vy = C.vy[t], vz = C.vz[t];
    const double len = sqrt(vx * vx + vy * vy + vz * vz);
    double s = on_box ? fmin(1.0, 2.0 * r0 / len) : 1.0;
    if (!(s > 1e-12)) s = 1.0;  // degenerate radius or vertex: probe the vertex itself
    uint32_t q = kNoSite;
    for (;;) {
        q = nearest_closer(T, C, skip, nskip, site, p, s * vx, s * vy, s * vz);
        if (q != kNoSite || s >= 1.0) break;
        s = fmin(1.0, 4.0 * s);
    }
    return q;
}

// Finishes an open cell vertex by vertex, one thread: a vertex is final when
// no site is closer to it than the cell's site.
template <class Cell>
VC_HD bool verify_serial(const CellParams &P, uint32_t site, const double p[3], double r0, Cell &C,
                         uint32_t &reason) {
    const Tree &T = P.tree;
    uint32_t skip[kSkip];
    int nskip = 0;
    int checks = 0;
    for (;;) {
        int t = 0;
        while (t < C.nt && (C.flag[t] & 1u)) ++t;
        if (t == C.nt) return true;
        if (C.bad || ++checks > Cell::kMaxChecks) {
            reason = C.bad ? kFailSelfCheck : kFailChecks;
            return false;
        }
        const uint32_t q = probe_vertex(T, C, skip, nskip, site, p, r0, t);
        if (q == kNoSite) {
            C.flag[t] |= 1u;
            continue;
        }
        const int r = clip_candidate(C, T, p, q, P.status);
        if (r < 0) {
            reason = kFailOpenClip;
            return false;
        }
        if (r == 0) {  // the exact test and the clip disagree by rounding
            if (nskip == kSkip) {
                reason = kFailSkip;
                return false;
            }
            skip[nskip++] = q;
        }
    }
}

// Writes the neighbour list of a finished cell: the sites of the planes the
// final cell uses, as output indices, ascending.  A cell that failed, or
// whose list does not fit, is queued for the second pass (first pass only)
// or counted as failed.
template <class Cell>
VC_HD void finish_cell(const CellParams &P, uint32_t site, Cell &C, bool ok, uint32_t reason, bool retry_pass) {
    const uint32_t row = P.to_out ? vc_ldg(P.to_out + site) : site;
    uint32_t *out = P.nbr + size_t(row) * P.cap;
    uint32_t n_out = 0;
    ok = ok && !C.bad;
    if (ok) {
        compact_planes(C);
        ok = !C.bad;
    }
    if (ok) {
        for (int s = 0; s < C.np; ++s) {
            if (is_box(C.pid[s])) continue;
            const uint32_t id = P.to_out ? vc_ldg(P.to_out + C.pid[s]) : C.pid[s];
            if (n_out == P.cap) {
                ok = false;
                reason = kFailOutput;
                break;
            }
            uint32_t j = n_out++;
            while (j > 0 && out[j - 1] > id) {
                out[j] = out[j - 1];
                --j;
            }
            out[j] = id;
        }
    }
    if (!ok) {
        n_out = 0;
        if (!reason) reason = C.bad ? kFailSelfCheck : kFailTierClip;
        bool queued = false;
        if (!retry_pass && reason != kFailSelfCheck && P.retry) {
            const uint32_t slot = vc_fetch_add(P.status + kStRetry);
            if (slot < P.retry_cap) {
                P.retry[slot] = site;
                queued = true;
            }
        }
        if (!queued) vc_count(P.status + kStFailed);
    }
    P.cnt[row] = n_out;
    if (P.reason) P.reason[row] = ok ? 0u : reason;
}

// The Voronoi cell of one site and its neighbour list (P.nbr / P.cnt), built
// in C by one thread.  A first-pass cell that fails for lack of room (planes,
// vertices, boundary edges, vertex checks) queues its site in P.retry instead
// of failing; the second pass (retry_pass) rebuilds it in a larger cell.
template <class Cell>
VC_HD void voronoi_cell(const CellParams &P, uint32_t site, Cell &C, bool retry_pass) {
    const Tree &T = P.tree;
    if (site >= T.num_points) return;
    const double p[3] = {vc_ldg(T.points + 3 * size_t(site)), vc_ldg(T.points + 3 * size_t(site) + 1),
                         vc_ldg(T.points + 3 * size_t(site) + 2)};
    bool done = false;
    double r0 = 0.0;
    uint32_t reason = 0;
    bool ok = build_tiers(P, site, p, C, done, r0, reason);
    if (ok && !done) {
        vc_count(P.status + kStOpenCells);
        ok = verify_serial(P, site, p, r0, C, reason);
    }
    finish_cell(P, site, C, ok, reason, retry_pass);
}

}  // namespace voronoi
}  // namespace sdfoam_b200
