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
//   * candidates are the site's nearest sites from the AABB tree (33, then
//     121); the cell is final once the farthest candidate is more than twice
//     the cell's radius away, because no farther site's bisector can reach it;
//   * cells still open after that -- sites on the convex hull, or sites whose
//     nearest sites all lie to one side -- are finished vertex by vertex: a
//     vertex is final when no site is closer to it than the cell's own site
//     (nearest-site search in double).  Any point of the segment from the site
//     to a vertex lies in the cell, so vertices on the box are probed at
//     growing distances along that segment first, which finds the sites that
//     close a one-sided cell with short searches.
// The box is the sites' bounding box grown by 10^6 times its size: every
// Voronoi vertex (Delaunay circumcentre) inside it is exact, which covers
// everything but slivers flatter than 10^-6 on the hull.
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

namespace sdfoam_b200 {

namespace {

constexpr int kMaxPlanes = 128;           // plane slots of one cell (box included)
constexpr int kMaxTris = 2 * kMaxPlanes;  // a cell with F faces has 2F - 4 vertices
constexpr int kMaxEdges = kMaxTris;       // boundary edges of one deleted patch
constexpr int kK1 = 33, kK2 = 121;        // candidates of the two tiers
constexpr int kSkip = 16;                 // sites whose clip was a rounding no-op
constexpr int kMaxChecks = 8 * kMaxTris;  // vertex checks of one open cell
constexpr uint32_t kBoxId = 0xfffffff0u;  // plane ids of the six box faces: kBoxId + k
constexpr int kStack = 64;

enum Status { kStFailed = 0, kStDuplicate = 1, kStAsymmetric = 2, kStOpenCells = 3 };

struct Cell {
    double nx[kMaxPlanes], ny[kMaxPlanes], nz[kMaxPlanes], w[kMaxPlanes];  // n . x <= w
    uint32_t pid[kMaxPlanes];
    unsigned char tri[kMaxTris][3];
    unsigned char flag[kMaxTris];  // bit 0: verified vertex, bit 1: scratch mark
    double vx[kMaxTris], vy[kMaxTris], vz[kMaxTris];
    int np, nt;
};

__device__ __forceinline__ bool is_box(uint32_t id) { return id >= kBoxId; }

__device__ void vertex_of(Cell &C, int t) {
    const int a = C.tri[t][0], b = C.tri[t][1], c = C.tri[t][2];
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
__device__ void init_box(Cell &C, const double lo[3], const double hi[3]) {
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
__device__ int compact_planes(Cell &C) {
    unsigned char used[kMaxPlanes];
    unsigned char remap[kMaxPlanes];
    for (int s = 0; s < C.np; ++s) used[s] = 0;
    for (int t = 0; t < C.nt; ++t)
        for (int e = 0; e < 3; ++e) used[C.tri[t][e]] = 1;
    int k = 0;
    for (int s = 0; s < C.np; ++s) {
        if (!used[s]) continue;
        remap[s] = static_cast<unsigned char>(k);
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
__device__ int clip(Cell &C, double nx, double ny, double nz, double w, uint32_t id) {
    int nmark = 0;
    for (int t = 0; t < C.nt; ++t) {
        const bool out = nx * C.vx[t] + ny * C.vy[t] + nz * C.vz[t] > w;
        C.flag[t] = static_cast<unsigned char>((C.flag[t] & 1u) | (out ? 2u : 0u));
        nmark += out;
    }
    if (nmark == 0) return 0;
    if (nmark == C.nt) return -1;  // impossible for a cell that contains its site
    if (C.np == kMaxPlanes) {
        compact_planes(C);
        if (C.np == kMaxPlanes) return -1;
    }
    // boundary of the deleted patch: directed edges of deleted vertices whose
    // reverse is not also an edge of a deleted vertex
    unsigned char ea[kMaxEdges], eb[kMaxEdges];
    int ne = 0;
    for (int t = 0; t < C.nt; ++t) {
        if (!(C.flag[t] & 2u)) continue;
        for (int e = 0; e < 3; ++e) {
            const unsigned char a = C.tri[t][e], b = C.tri[t][(e + 1) % 3];
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
                if (ne == kMaxEdges) return -1;
                ea[ne] = a;
                eb[ne] = b;
                ++ne;
            }
        }
    }
    if (C.nt - nmark + ne > kMaxTris) return -1;
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
        C.tri[C.nt][0] = ea[e];
        C.tri[C.nt][1] = eb[e];
        C.tri[C.nt][2] = static_cast<unsigned char>(s);
        C.flag[C.nt] = 0;
        vertex_of(C, C.nt);
        ++C.nt;
    }
    return 1;
}

// Clip by the bisector of the site (origin) and q (relative position).
__device__ __forceinline__ int clip_site(Cell &C, double qx, double qy, double qz, uint32_t id) {
    return clip(C, qx, qy, qz, 0.5 * (qx * qx + qy * qy + qz * qz), id);
}

__device__ __forceinline__ double radius2(const Cell &C) {
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

__device__ __forceinline__ uint64_t level_offset(const Tree &T, uint32_t L) {
    uint64_t off = 0;
    for (uint32_t l = 0; l < L; ++l) off += T.num_leaves >> l;
    return off;
}

__device__ __forceinline__ float box_dist2(const float *box, float x, float y, float z) {
    const float gx = fmaxf(fmaxf(__ldg(box + 0) - x, x - __ldg(box + 3)), 0.0f);
    const float gy = fmaxf(fmaxf(__ldg(box + 1) - y, y - __ldg(box + 4)), 0.0f);
    const float gz = fmaxf(fmaxf(__ldg(box + 2) - z, z - __ldg(box + 5)), 0.0f);
    return gx * gx + gy * gy + gz * gz;
}

// The k nearest sites of site self (sorted by float distance, ties by index);
// returns how many were found (< k only when the foam has fewer sites).
__device__ int knn(const Tree &T, uint32_t self, float x, float y, float z, int k, float *kd, uint32_t *ki) {
    int cnt = 0;
    uint32_t stack[kStack];
    int sp = 0;
    stack[sp++] = ((T.levels - 1) << 27) | 0u;
    while (sp > 0) {
        const uint32_t e = stack[--sp];
        const uint32_t L = e >> 27, node = e & ((1u << 27) - 1);
        const float worst = cnt < k ? FLT_MAX : kd[k - 1];
        if (L == 0) {
            for (uint32_t i = 2 * node; i < 2 * node + 2 && i < T.num_points; ++i) {
                if (i == self) continue;
                const float dx = __ldg(T.points + 3 * size_t(i)) - x;
                const float dy = __ldg(T.points + 3 * size_t(i) + 1) - y;
                const float dz = __ldg(T.points + 3 * size_t(i) + 2) - z;
                const float d = dx * dx + dy * dy + dz * dz;
                if (cnt == k && !(d < kd[k - 1] || (d == kd[k - 1] && i < ki[k - 1]))) continue;
                int j = cnt < k ? cnt++ : k - 1;
                while (j > 0 && (kd[j - 1] > d || (kd[j - 1] == d && ki[j - 1] > i))) {
                    kd[j] = kd[j - 1];
                    ki[j] = ki[j - 1];
                    --j;
                }
                kd[j] = d;
                ki[j] = i;
            }
            continue;
        }
        const uint64_t off = level_offset(T, L - 1);
        const float d0 = box_dist2(T.boxes + 6 * (off + 2 * size_t(node)), x, y, z);
        const float d1 = box_dist2(T.boxes + 6 * (off + 2 * size_t(node) + 1), x, y, z);
        const int nearer = d1 < d0 ? 1 : 0;
        const float dn = nearer ? d1 : d0, df = nearer ? d0 : d1;
        if (df <= worst && sp < kStack) stack[sp++] = ((L - 1) << 27) | (2 * node + 1 - nearer);
        if (dn <= worst && sp < kStack) stack[sp++] = ((L - 1) << 27) | (2 * node + nearer);
    }
    return cnt;
}

__device__ __forceinline__ bool in_cell_or_skip(const Cell &C, const uint32_t *skip, int nskip, uint32_t i) {
    for (int s = 0; s < C.np; ++s)
        if (C.pid[s] == i) return true;
    for (int s = 0; s < nskip; ++s)
        if (skip[s] == i) return true;
    return false;
}

// The site nearest to the point p + (x, y, z) among those strictly closer to
// it than the site p itself, or kNone.  Double precision throughout.
__device__ uint32_t nearest_closer(const Tree &T, const Cell &C, const uint32_t *skip, int nskip, uint32_t self,
                                   const double p[3], double x, double y, double z) {
    double best = x * x + y * y + z * z;
    uint32_t cand = kNone;
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
                const double dx = double(__ldg(T.points + 3 * size_t(i))) - cx;
                const double dy = double(__ldg(T.points + 3 * size_t(i) + 1)) - cy;
                const double dz = double(__ldg(T.points + 3 * size_t(i) + 2)) - cz;
                const double d = dx * dx + dy * dy + dz * dz;
                if (d < best && !in_cell_or_skip(C, skip, nskip, i)) {
                    best = d;
                    cand = i;
                }
            }
            continue;
        }
        const uint64_t off = level_offset(T, L - 1);
        double dc[2];
        for (int c = 0; c < 2; ++c) {
            const float *box = T.boxes + 6 * (off + 2 * size_t(node) + c);
            const double gx = fmax(fmax(double(__ldg(box + 0)) - cx, cx - double(__ldg(box + 3))), 0.0);
            const double gy = fmax(fmax(double(__ldg(box + 1)) - cy, cy - double(__ldg(box + 4))), 0.0);
            const double gz = fmax(fmax(double(__ldg(box + 2)) - cz, cz - double(__ldg(box + 5))), 0.0);
            dc[c] = gx * gx + gy * gy + gz * gz;
        }
        const int nearer = dc[1] < dc[0] ? 1 : 0;
        if (dc[1 - nearer] < best && sp < kStack) stack[sp++] = ((L - 1) << 27) | (2 * node + 1 - nearer);
        if (dc[nearer] < best && sp < kStack) stack[sp++] = ((L - 1) << 27) | (2 * node + nearer);
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
};

__device__ int clip_candidate(Cell &C, const Tree &T, const double p[3], uint32_t i, uint32_t *status) {
    const double qx = double(__ldg(T.points + 3 * size_t(i))) - p[0];
    const double qy = double(__ldg(T.points + 3 * size_t(i) + 1)) - p[1];
    const double qz = double(__ldg(T.points + 3 * size_t(i) + 2)) - p[2];
    if (qx == 0.0 && qy == 0.0 && qz == 0.0) {
        atomicAdd(status + kStDuplicate, 1u);
        return 0;
    }
    return clip_site(C, qx, qy, qz, i);
}

__global__ void __launch_bounds__(64) voronoi_cells_kernel(const CellParams P) {
    const uint32_t site = blockIdx.x * blockDim.x + threadIdx.x;
    const Tree &T = P.tree;
    if (site >= T.num_points) return;
    Cell C;
    float kd[kK2];
    uint32_t ki[kK2];
    const float fx = __ldg(T.points + 3 * size_t(site));
    const float fy = __ldg(T.points + 3 * size_t(site) + 1);
    const float fz = __ldg(T.points + 3 * size_t(site) + 2);
    const double p[3] = {fx, fy, fz};
    const double lo[3] = {P.lo[0] - p[0], P.lo[1] - p[1], P.lo[2] - p[2]};
    const double hi[3] = {P.hi[0] - p[0], P.hi[1] - p[1], P.hi[2] - p[2]};
    init_box(C, lo, hi);
    bool ok = true, done = false;
    int seen = 0;
    // tiers of nearest candidates, closed by the security radius
    for (int tier = 0; tier < 2 && ok && !done; ++tier) {
        const int k = tier == 0 ? kK1 : kK2;
        const int n = knn(T, site, fx, fy, fz, k, kd, ki);
        for (int j = seen; j < n && ok; ++j) ok = clip_candidate(C, T, p, ki[j], P.status) >= 0;
        seen = n;
        if (n < k) {
            done = true;  // every other site was a candidate
        } else if (ok) {
            const double r2 = radius2(C);
            done = 4.0 * r2 < double(kd[n - 1]) * (1.0 - 1e-5);
        }
    }
    if (ok && !done) {
        // open cell: verify vertex by vertex
        atomicAdd(P.status + kStOpenCells, 1u);
        uint32_t skip[kSkip];
        int nskip = 0;
        const double r0 = sqrt(double(kd[seen - 1]));
        int checks = 0;
        for (;;) {
            int t = 0;
            while (t < C.nt && (C.flag[t] & 1u)) ++t;
            if (t == C.nt) break;
            if (++checks > kMaxChecks) {
                ok = false;
                break;
            }
            const bool on_box = is_box(C.pid[C.tri[t][0]]) || is_box(C.pid[C.tri[t][1]]) ||
                                is_box(C.pid[C.tri[t][2]]);
            const double vx = C.vx[t], vy = C.vy[t], vz = C.vz[t];
            const double len = sqrt(vx * vx + vy * vy + vz * vz);
            double s = on_box ? fmin(1.0, 2.0 * r0 / len) : 1.0;
            uint32_t q = kNone;
            for (;;) {
                q = nearest_closer(T, C, skip, nskip, site, p, s * vx, s * vy, s * vz);
                if (q != kNone || s >= 1.0) break;
                s = fmin(1.0, 4.0 * s);
            }
            if (q == kNone) {
                C.flag[t] |= 1u;
                continue;
            }
            const int r = clip_candidate(C, T, p, q, P.status);
            if (r < 0) {
                ok = false;
                break;
            }
            if (r == 0) {  // the exact test and the clip disagree by rounding
                if (nskip == kSkip) {
                    ok = false;
                    break;
                }
                skip[nskip++] = q;
            }
        }
    }
    // neighbours: the sites of the planes the final cell uses, ascending
    uint32_t *out = P.nbr + size_t(site) * P.cap;
    uint32_t n_out = 0;
    if (ok) {
        compact_planes(C);
        for (int s = 0; s < C.np; ++s) {
            const uint32_t id = C.pid[s];
            if (is_box(id)) continue;
            if (n_out == P.cap) {
                ok = false;
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
        atomicAdd(P.status + kStFailed, 1u);
        n_out = 0;
    }
    P.cnt[site] = n_out;
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
    for (uint32_t k = 0; k < cnt[i]; ++k) {
        const uint32_t j = row[k];
        if (j >= n) continue;
        if (!row_has(nbr + size_t(j) * cap, cnt[j], i)) {
            const uint32_t slot = atomicAdd(status + kStAsymmetric, 1u);
            if (slot < extra_cap) extra[slot] = make_uint2(j, i);
        }
    }
}

__global__ void __launch_bounds__(256) add_extra_kernel(const uint2 *__restrict__ extra,
                                                        const uint32_t *__restrict__ status, uint32_t extra_cap,
                                                        uint32_t *__restrict__ nbr, uint32_t *__restrict__ cnt,
                                                        uint32_t cap, uint32_t *__restrict__ dirty,
                                                        uint32_t *__restrict__ status_out) {
    const uint32_t e = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t total = min(status[kStAsymmetric], extra_cap);
    if (e >= total) return;
    const uint2 x = extra[e];
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
    l.total = align_up(l.status + 64, 256);
    return l;
}

cudaError_t launch_delaunay_neighbors(const float *points, uint32_t n, const float *tree, void *workspace,
                                      uint32_t *offsets, cudaStream_t stream) {
    const DelaunayLayout l = delaunay_layout(n);
    char *ws = static_cast<char *>(workspace);
    uint32_t *nbr = reinterpret_cast<uint32_t *>(ws + l.nbr);
    uint32_t *cnt = reinterpret_cast<uint32_t *>(ws + l.cnt);
    uint32_t *prefix = reinterpret_cast<uint32_t *>(ws + l.prefix);
    uint32_t *sums = reinterpret_cast<uint32_t *>(ws + l.sums);
    uint32_t *dirty = reinterpret_cast<uint32_t *>(ws + l.dirty);
    uint2 *extra = reinterpret_cast<uint2 *>(ws + l.extra);
    uint32_t *status = reinterpret_cast<uint32_t *>(ws + l.status);
    cudaError_t e = cudaMemsetAsync(status, 0, 64, stream);
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(dirty, 0, size_t(n) * 4, stream);
    if (e != cudaSuccess) return e;
    duplicates_kernel<<<(n + 255) / 256, 256, 0, stream>>>(points, n, status);

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
    // the box: the root node's bounds (read back once; the tree is tiny next
    // to the cell work) grown by 10^6 times the extent
    float root[6];
    const size_t root_off = 6 * (2 * size_t(P.tree.num_leaves) - 2);
    e = cudaMemcpyAsync(root, tree + root_off, sizeof(root), cudaMemcpyDeviceToHost, stream);
    if (e != cudaSuccess) return e;
    e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return e;
    double ext = 0.0;
    for (int k = 0; k < 3; ++k) ext = ext > double(root[3 + k]) - root[k] ? ext : double(root[3 + k]) - root[k];
    const double grow = 1e6 * (ext + 1e-3);
    for (int k = 0; k < 3; ++k) {
        P.lo[k] = double(root[k]) - grow;
        P.hi[k] = double(root[3 + k]) + grow;
    }
    voronoi_cells_kernel<<<(n + 63) / 64, 64, 0, stream>>>(P);
    asymmetry_kernel<<<(n + 255) / 256, 256, 0, stream>>>(nbr, cnt, n, kDelaunayCap, extra, l.extra_cap, status);
    // the asymmetric count is read on the device by the next two launches
    add_extra_kernel<<<(l.extra_cap + 255) / 256, 256, 0, stream>>>(extra, status, l.extra_cap, nbr, cnt,
                                                                      kDelaunayCap, dirty, status);
    sort_dirty_kernel<<<(n + 255) / 256, 256, 0, stream>>>(nbr, cnt, n, kDelaunayCap, dirty);
    const uint32_t tiles = (n + kScanTile - 1) / kScanTile;
    tile_sums_kernel<<<tiles, kScanBlock, 0, stream>>>(cnt, n, sums);
    scan_sums_kernel<<<1, 1024, 0, stream>>>(sums, tiles);
    tile_scan_kernel<<<tiles, kScanBlock, 0, stream>>>(cnt, n, sums, prefix);
    uint32_t *last = status + 8;
    last_row_kernel<<<(n + 255) / 256, 256, 0, stream>>>(cnt, n, last);
    offsets_kernel<<<(n + 1 + 255) / 256, 256, 0, stream>>>(cnt, prefix, n, last, offsets);
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
