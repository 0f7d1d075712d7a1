// Forward and backward Voronoi-foam walk kernels for sm_100a.
//
// One lane walks one ray; its state (origin, direction, SH basis, t0, T,
// colour accumulators) stays in registers for the whole walk.  Per step the
// lane reads the current site's face records (neighbour id + plane offset,
// 128- or 256-bit loads), keeps the first face with the smallest exit
// distance, then reads the next site's 32-byte head (position, face range,
// last attribute channel) with one 256-bit load and the current site's SH row
// with 256-bit loads.
//
// Exit-face search.  The reference computes t = dot(fo - o, off) / dot(off, d)
// with an IEEE division for every face (tracing_utils.cuh:64-88).  Here each
// face gets an approximate quotient num * rcp.approx(dp) whose relative error
// is below 2^-22; a face is accepted, rejected or ordered against the current
// best from that value whenever a 2^-20 relative margin decides the
// comparison, and the exact IEEE quotient is computed only when it does not
// (and once for the chosen face).  The chosen face and its t are therefore
// exactly those of the reference rule: the first face in CSR order with the
// smallest exact t among faces with dp > 0 (and t > t0 in safe mode).
// Faces store h = off / 2 (exact), so dot(w, h) / dot(h, d) equals the
// reference quotient bit for bit (both operands are scaled by 2 exactly).
//
// Semantics follow the reference walk and cell functors:
//   trace()        src/tracing/tracing_utils.cuh:17-109
//   forward        src/tracing/pipeline.cu:36-264
//   backward_sdf   src/tracing/pipeline.cu:267-550  (NeuS mode)
//   backward       src/tracing/pipeline.cu:553-791  (RadFoam density mode,
//                  "unsafe" exit-face rule without the t > t0 test)
// Gradient scatter uses 128-bit vector atomics (red.global.add.v4.f32) into
// 16-byte aligned per-site rows, folded into the caller's [N,A] / [N,3]
// outputs afterwards; the per-step sharpness gradient of the reference (a
// single-address atomic per step) is summed in registers and reduced once per
// block.
#include <cfloat>

#include "foam_device.cuh"
#include "foam_internal.h"

namespace sdfoam_b200 {

namespace {

constexpr int kBlock = 128;

struct RayState {
    float ox, oy, oz, dx, dy, dz;
};

__device__ __forceinline__ RayState load_ray(const float *__restrict__ rays, uint32_t r) {
    const float *src = rays + 6 * size_t(r);
    RayState s;
    s.ox = __ldg(src + 0);
    s.oy = __ldg(src + 1);
    s.oz = __ldg(src + 2);
    float dx = __ldg(src + 3), dy = __ldg(src + 4), dz = __ldg(src + 5);
    const float len = __fsqrt_rn(fmaf(dx, dx, fmaf(dy, dy, __fmul_rn(dz, dz))));
    s.dx = __fdiv_rn(dx, len);
    s.dy = __fdiv_rn(dy, len);
    s.dz = __fdiv_rn(dz, len);
    return s;
}

struct Head {
    float px, py, pz;
    uint32_t beg, end;
    float last;
};

__device__ __forceinline__ Head load_head(const uint32_t *__restrict__ heads, uint32_t c) {
    uint32_t w[8];
    ldg256(heads + 8 * size_t(c), w);
    Head h;
    h.px = __uint_as_float(w[0]);
    h.py = __uint_as_float(w[1]);
    h.pz = __uint_as_float(w[2]);
    h.beg = w[3];
    h.end = w[4];
    h.last = __uint_as_float(w[5]);
    return h;
}

// Running exit-face choice over one site's faces (see the file comment).
// lo/hi bracket the exact quotient; faces whose bracket is unusable carry
// (-inf, +inf) and always take the exact path.
template <bool SAFE>
struct ExitSearch {
    float t0;
    bool have;
    bool bexact;
    float blo, bhi, bnum, bdp, bt;
    uint32_t bid;

    __device__ __forceinline__ explicit ExitSearch(float t0_) : t0(t0_), have(false), bexact(false) {}

    __device__ __forceinline__ void face(const RayState &ray, float px, float py, float pz, uint32_t id,
                                         float hx, float hy, float hz) {
        const float dp = dot3(hx, hy, hz, ray.dx, ray.dy, ray.dz);
        if (!(dp > 0.0f)) return;
        const float wx = __fsub_rn(__fadd_rn(px, hx), ray.ox);
        const float wy = __fsub_rn(__fadd_rn(py, hy), ray.oy);
        const float wz = __fsub_rn(__fadd_rn(pz, hz), ray.oz);
        const float num = dot3(wx, wy, wz, hx, hy, hz);
        const float qa = __fmul_rn(num, rcp_approx(dp));
        const float aq = fabsf(qa);
        const float m = __fmul_rn(aq, 0x1p-20f);
        const bool sure = dp >= 1e-30f && aq >= 1e-30f && aq <= 1e30f;
        const float lo = sure ? __fsub_rn(qa, m) : -__int_as_float(0x7f800000);
        const float hi = sure ? __fadd_rn(qa, m) : __int_as_float(0x7f800000);
        float t = 0.0f;
        bool exact = false;
        if (SAFE) {
            if (!(lo > t0)) {           // not certainly valid
                if (hi <= t0) return;   // certainly t <= t0
                t = __fdiv_rn(num, dp);
                exact = true;
                if (!(t > t0)) return;
            }
        }
        bool take;
        if (!have) {
            if (sure) {
                take = true;
            } else {
                if (!exact) {
                    t = __fdiv_rn(num, dp);
                    exact = true;
                }
                take = t < __int_as_float(0x7f800000);
            }
        } else if (hi < blo) {
            take = true;
        } else if (lo > bhi) {
            take = false;
        } else {
            if (!exact) {
                t = __fdiv_rn(num, dp);
                exact = true;
            }
            if (!bexact) {
                bt = __fdiv_rn(bnum, bdp);
                bexact = true;
            }
            take = t < bt;
        }
        if (take) {
            have = true;
            blo = lo;
            bhi = hi;
            bnum = num;
            bdp = dp;
            bexact = exact;
            bt = t;
            bid = id;
        }
    }

    __device__ __forceinline__ float t1() const { return bexact ? bt : __fdiv_rn(bnum, bdp); }
};

__device__ __forceinline__ void face_rec(const uint32_t *w, uint32_t &id, float &hx, float &hy, float &hz) {
    id = w[0];
    hx = __uint_as_float(w[1]);
    hy = __uint_as_float(w[2]);
    hz = __uint_as_float(w[3]);
}

// Scans the CSR range [beg, end): 256-bit loads of record pairs where the
// pair is 32-byte aligned, 128-bit loads at the ragged ends.
template <bool SAFE>
__device__ __forceinline__ bool find_exit(const uint4 *__restrict__ faces, uint32_t beg, uint32_t end,
                                          const RayState &ray, float px, float py, float pz, float t0,
                                          float &t1, uint32_t &next) {
    ExitSearch<SAFE> s(t0);
    uint32_t j = beg;
    uint32_t id;
    float hx, hy, hz;
    if ((j & 1u) && j < end) {
        const uint4 r = __ldg(faces + j);
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
        face_rec(w, id, hx, hy, hz);
        s.face(ray, px, py, pz, id, hx, hy, hz);
        ++j;
    }
    for (; j + 1 < end; j += 2) {
        uint32_t w[8];
        ldg256(faces + j, w);
        face_rec(w, id, hx, hy, hz);
        s.face(ray, px, py, pz, id, hx, hy, hz);
        face_rec(w + 4, id, hx, hy, hz);
        s.face(ray, px, py, pz, id, hx, hy, hz);
    }
    if (j < end) {
        const uint4 r = __ldg(faces + j);
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
        face_rec(w, id, hx, hy, hz);
        s.face(ray, px, py, pz, id, hx, hy, hz);
    }
    if (!s.have) return false;
    t1 = s.t1();
    next = s.bid;
    return true;
}

// NeuS density s = sha * phi * (1 - phi), phi = 1 / (1 + exp(sha * d))
// (pipeline.cu:149, 386-387).
__device__ __forceinline__ float neus_phi(float sha, float d) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, foam_expf(__fmul_rn(sha, d))));
}

// Attribute channel ch of a site: the last channel lives in the head, the
// others in the SH rows of the cell records.
template <int DEG>
__device__ __forceinline__ float attr_channel(const CellsView &C, uint32_t site, float last, int ch) {
    constexpr int A = AttrLayout<DEG>::kDim;
    if (ch == A - 1) return last;
    return __ldg(C.sh + size_t(site) * AttrLayout<DEG>::kStride + ch);
}

// --------------------------------------------------------------------------
// forward
// --------------------------------------------------------------------------

template <int DEG, bool NEUS>
__global__ void __launch_bounds__(kBlock) forward_kernel(const ForwardParams P) {
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= P.num_rays) return;
    const CellsView &C = P.cells;
    const RayState ray = load_ray(P.rays, r);
    SHBasis Y;
    sh_basis<DEG>(ray.dx, ray.dy, ray.dz, Y);

    const uint32_t Q = P.quantiles ? P.num_quantiles : 0u;
    const float *rq = P.quantiles ? P.quantiles + size_t(r) * P.num_quantiles : nullptr;
    uint32_t qi = 0;
    float q = 0.0f;
    if (rq && P.num_quantiles > 0) q = __ldg(rq);
    const int sdf_ch = P.settings.sdf_channel;
    const bool neus_alpha = NEUS && sdf_ch >= 0;
    const float sha = NEUS ? __ldg(P.sharpness) : 0.0f;
    const float thr = P.settings.weight_threshold;
    const uint32_t max_steps = P.settings.max_intersections;

    float T = 1.0f, ar = 0.0f, ag = 0.0f, ab = 0.0f;
    float t0 = 0.0f;
    uint32_t n = 0;
    uint64_t seq_pos = 0, seq_end = 0;
    if (P.seq_cells) {
        seq_pos = P.seq_offsets[r];
        seq_end = P.seq_offsets[r + 1];
    }
    uint32_t nseq = 0;
    uint32_t faces_seen = 0;

    uint32_t cur = __ldg(P.start + r);
    if (cur < C.num_points) {
        Head h = load_head(C.heads, cur);
        for (;;) {
            ++n;
            if (n > max_steps) break;
            if (h.beg > h.end || h.end > C.adjacency_size) break;
            faces_seen += h.end - h.beg;
            float t1;
            uint32_t nxt = kNone;
            if (!find_exit<true>(C.faces, h.beg, h.end, ray, h.px, h.py, h.pz, t0, t1, nxt)) break;
            if (nxt >= C.num_points) break;
            const Head nh = load_head(C.heads, nxt);
            if (t1 > t0) {
                AttrRow<DEG> row;
                load_row<DEG>(C.sh, cur, row);
                float cr = 0.0f, cg = 0.0f, cb = 0.0f;
                if (NEUS || h.last > 1e-6f) sh_rgb<DEG>(Y, row, cr, cg, cb);
                const float dt = fmaxf(__fsub_rn(t1, t0), 0.0f);
                float s;
                if (neus_alpha) {
                    const float phi = neus_phi(sha, attr_channel<DEG>(C, cur, h.last, sdf_ch));
                    s = __fmul_rn(__fmul_rn(sha, phi), __fsub_rn(1.0f, phi));
                } else {
                    s = h.last;
                }
                const float alpha = __fsub_rn(1.0f, foam_expf(-__fmul_rn(s, dt)));
                const float w = __fmul_rn(T, alpha);
                if (P.alpha) P.alpha[cur] = alpha;
                if (P.contribution) atomicAdd(P.contribution + cur, w);
                ar = fmaf(w, cr, ar);
                ag = fmaf(w, cg, ag);
                ab = fmaf(w, cb, ab);
                const float Tn = __fmul_rn(T, __fsub_rn(1.0f, alpha));
                if (NEUS) {
                    const float drop = __fsub_rn(T, Tn);
                    if (drop > 1e-12f) {
                        while (qi < Q && Tn < q) {
                            float frac = __fdiv_rn(__fsub_rn(T, q), drop);
                            frac = fminf(1.0f, fmaxf(0.0f, frac));
                            P.depth[size_t(r) * Q + qi] = fmaf(frac, __fsub_rn(t1, t0), t0);
                            P.depth_indices[size_t(r) * Q + qi] = cur;
                            ++qi;
                            if (qi < Q) q = __ldg(rq + qi);
                        }
                    }
                } else {
                    while (qi < Q && Tn < q) {
                        P.depth[size_t(r) * Q + qi] = __fadd_rn(t0, __fdiv_rn(logf(__fdiv_rn(T, q)), s));
                        P.depth_indices[size_t(r) * Q + qi] = cur;
                        ++qi;
                        if (qi < Q) q = __ldg(rq + qi);
                    }
                }
                if (seq_pos < seq_end) P.seq_cells[seq_pos++] = cur;
                ++nseq;
                T = Tn;
                if (!(T > thr)) break;
            }
            t0 = fmaxf(t0, t1);
            cur = nxt;
            h = nh;
        }
    }
    while (qi < Q) {
        P.depth[size_t(r) * Q + qi] = -1.0f;
        P.depth_indices[size_t(r) * Q + qi] = kNone;
        ++qi;
    }
    reinterpret_cast<float4 *>(P.rgba)[r] = make_float4(ar, ag, ab, __fsub_rn(1.0f, T));
    if (P.num_intersections) P.num_intersections[r] = n;
    if (P.seq_count) P.seq_count[r] = nseq;
    if (P.face_tests) P.face_tests[r] = faces_seen;
}

// --------------------------------------------------------------------------
// backward
// --------------------------------------------------------------------------

// d t / d primal for the bisector planes of (p, q) and (q, p) at once
// (tracing_utils.cuh:112-124): both share the plane's numerator and ray
// projection up to sign.  Differs from the reference's per-component division
// by one reciprocal (within the gradient tolerance).
__device__ __forceinline__ void cig_pair(float px, float py, float pz, float qx, float qy, float qz,
                                         const RayState &ray, float &gpx, float &gpy, float &gpz, float &gqx,
                                         float &gqy, float &gqz) {
    const float wx = __fsub_rn(__fmul_rn(__fadd_rn(px, qx), 0.5f), ray.ox);
    const float wy = __fsub_rn(__fmul_rn(__fadd_rn(py, qy), 0.5f), ray.oy);
    const float wz = __fsub_rn(__fmul_rn(__fadd_rn(pz, qz), 0.5f), ray.oz);
    const float nx = __fsub_rn(qx, px), ny = __fsub_rn(qy, py), nz = __fsub_rn(qz, pz);
    const float num = dot3(wx, wy, wz, nx, ny, nz);
    const float dp = dot3(nx, ny, nz, ray.dx, ray.dy, ray.dz);
    const float inv = __frcp_rn(__fmul_rn(dp, dp));
    gpx = __fmul_rn(fmaf(num, ray.dx, __fmul_rn(dp, __fsub_rn(ray.ox, px))), inv);
    gpy = __fmul_rn(fmaf(num, ray.dy, __fmul_rn(dp, __fsub_rn(ray.oy, py))), inv);
    gpz = __fmul_rn(fmaf(num, ray.dz, __fmul_rn(dp, __fsub_rn(ray.oz, pz))), inv);
    gqx = __fmul_rn(fmaf(-num, ray.dx, __fmul_rn(-dp, __fsub_rn(ray.ox, qx))), inv);
    gqy = __fmul_rn(fmaf(-num, ray.dy, __fmul_rn(-dp, __fsub_rn(ray.oy, qy))), inv);
    gqz = __fmul_rn(fmaf(-num, ray.dz, __fmul_rn(-dp, __fsub_rn(ray.oz, qz))), inv);
}

// SH gradient row (value Y_k * g_c at channel 3k+c, plus `last` at channel A-1)
// added with 128-bit vector atomics.
template <int DEG>
__device__ __forceinline__ void scatter_row(float4 *__restrict__ dst, const SHBasis &Y, float gr, float gg,
                                            float gb, float last, bool with_last) {
    constexpr int V = AttrLayout<DEG>::kVec4;
    constexpr int NSH = AttrLayout<DEG>::kSH;
    constexpr int A = AttrLayout<DEG>::kDim;
    const float g3[3] = {gr, gg, gb};
#pragma unroll
    for (int v = 0; v < V; ++v) {
        float e[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int i = 4 * v + k;
            e[k] = i < NSH ? __fmul_rn(Y.y[i / 3], g3[i % 3]) : (i == A - 1 && with_last ? last : 0.0f);
        }
        if (4 * v >= NSH && !with_last) continue;  // nothing but padding left
        atomicAdd(dst + v, make_float4(e[0], e[1], e[2], e[3]));
    }
}

template <int DEG, bool NEUS>
__global__ void __launch_bounds__(kBlock) backward_kernel(const BackwardParams P) {
    constexpr int A = AttrLayout<DEG>::kDim;
    constexpr int V = AttrLayout<DEG>::kVec4;
    __shared__ float block_sha[kBlock / 32];
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    float sha_sum = 0.0f;
    if (r < P.num_rays) {
        const CellsView &C = P.cells;
        const RayState ray = load_ray(P.rays, r);
        SHBasis Y;
        sh_basis<DEG>(ray.dx, ray.dy, ray.dz, Y);
        const float4 g = reinterpret_cast<const float4 *>(P.rgba_grad)[r];
        const float4 Cf = reinterpret_cast<const float4 *>(P.rgba)[r];
        const uint32_t Q = P.quantiles ? P.num_quantiles : 0u;
        const float *rq = P.quantiles ? P.quantiles + size_t(r) * P.num_quantiles : nullptr;
        const float *rdg = P.depth_grad ? P.depth_grad + size_t(r) * P.num_quantiles : nullptr;
        const float err = P.ray_error ? __ldg(P.ray_error + r) : 0.0f;
        const float thr = P.settings.weight_threshold;
        const uint32_t max_steps = P.settings.max_intersections;
        const int sdf_set = P.settings.sdf_channel;
        const int sdf_ch = NEUS ? (sdf_set >= 0 ? sdf_set : A - 1) : A - 1;
        const bool sdf_fast = sdf_ch == A - 1;
        const float sha = NEUS ? __ldg(P.sharpness) : 0.0f;
        uint32_t qi = 0;
        float q = 0.0f;
        if (rq && P.num_quantiles > 0) q = __ldg(rq);

        // RadFoam mode: sum of depth_grad / s over the recorded quantile sites
        // (pipeline.cu:620-629)
        float cur_depth_grad = 0.0f;
        if (!NEUS) {
            for (uint32_t i = 0; i < Q; ++i) {
                const uint32_t pi = P.depth_indices[size_t(r) * Q + i];
                if (pi < C.num_points) {  // kNone marks an unfilled quantile
                    const float sv = __uint_as_float(__ldg(C.heads + 8 * size_t(pi) + 5));
                    cur_depth_grad = __fadd_rn(cur_depth_grad, __fdiv_rn(__ldg(rdg + i), sv));
                }
            }
        }

        float g_logT = 0.0f;
        float T = 1.0f, ar = 0.0f, ag = 0.0f, ab = 0.0f;
        uint32_t prev_idx = kNone;
        float qpx = 0.0f, qpy = 0.0f, qpz = 0.0f;          // prev point
        float pgx = 0.0f, pgy = 0.0f, pgz = 0.0f;          // prev point grad
        float cgx = 0.0f, cgy = 0.0f, cgz = 0.0f;          // current point grad
        float t0 = 0.0f;
        uint32_t n = 0;
        uint32_t cur = __ldg(P.start + r);
        if (cur < C.num_points) {
            Head h = load_head(C.heads, cur);
            for (;;) {
                ++n;
                if (n > max_steps) break;
                if (h.beg > h.end || h.end > C.adjacency_size) break;
                float t1;
                uint32_t nxt = kNone;
                if (!find_exit<NEUS>(C.faces, h.beg, h.end, ray, h.px, h.py, h.pz, t0, t1, nxt)) break;
                if (nxt >= C.num_points) break;
                const Head nh = load_head(C.heads, nxt);
                if (t1 > t0) {
                    const float px = h.px, py = h.py, pz = h.pz;
                    AttrRow<DEG> row;
                    load_row<DEG>(C.sh, cur, row);
                    const float last = h.last;
                    float cr = 0.0f, cg = 0.0f, cb = 0.0f;
                    if (NEUS || last > 1e-6f) sh_rgb<DEG>(Y, row, cr, cg, cb);
                    const float dt = fmaxf(__fsub_rn(t1, t0), 0.0f);
                    float s, phi = 0.0f, d = 0.0f;
                    if (NEUS) {
                        d = sdf_fast ? last : attr_channel<DEG>(C, cur, last, sdf_ch);
                        phi = neus_phi(sha, d);
                        s = __fmul_rn(__fmul_rn(sha, phi), __fsub_rn(1.0f, phi));
                    } else {
                        s = last;
                    }
                    const float alpha = __fsub_rn(1.0f, foam_expf(-__fmul_rn(s, dt)));
                    const float oma = __fsub_rn(1.0f, alpha);
                    const float w = __fmul_rn(T, alpha);
                    ar = fmaf(w, cr, ar);
                    ag = fmaf(w, cg, ag);
                    ab = fmaf(w, cb, ab);
                    if (P.point_error) atomicAdd(P.point_error + cur, __fmul_rn(w, err));
                    float gr = __fmul_rn(g.x, w), gg = __fmul_rn(g.y, w), gb = __fmul_rn(g.z, w);
                    const float denom = NEUS ? fmaf(T, oma, 1e-6f) : __fmul_rn(T, __fadd_rn(oma, 1e-6f));
                    const float ux = __fsub_rn(cr, __fdiv_rn(__fsub_rn(Cf.x, ar), denom));
                    const float uy = __fsub_rn(cg, __fdiv_rn(__fsub_rn(Cf.y, ag), denom));
                    const float uz = __fsub_rn(cb, __fdiv_rn(__fsub_rn(Cf.z, ab), denom));
                    float dL_dalpha = __fmul_rn(T, dot3(ux, uy, uz, g.x, g.y, g.z));
                    dL_dalpha = __fadd_rn(dL_dalpha, __fdiv_rn(__fmul_rn(__fsub_rn(1.0f, Cf.w), g.w),
                                                               __fadd_rn(oma, 1e-6f)));
                    const float Tn = __fmul_rn(T, oma);
                    float dL_ds, dL_ddelta, dL_dt0;
                    if (NEUS) {
                        dL_dalpha = __fadd_rn(dL_dalpha, __fdiv_rn(-g_logT, fmaxf(oma, 1e-12f)));
                        dL_ds = __fmul_rn(dL_dalpha, __fmul_rn(dt, oma));
                        dL_ddelta = __fmul_rn(dL_dalpha, __fmul_rn(s, oma));
                        float units = 0.0f;
                        if (rq && P.num_quantiles > 0) {
                            const float drop = __fsub_rn(T, Tn);
                            if (drop > 1e-12f) {
                                while (qi < Q && Tn < q) {
                                    const float gq = __ldg(rdg + qi);
                                    float frac = __fdiv_rn(__fsub_rn(T, q), drop);
                                    frac = fminf(1.0f, fmaxf(0.0f, frac));
                                    units = __fadd_rn(units, gq);
                                    dL_ddelta = fmaf(gq, frac, dL_ddelta);
                                    if (alpha > 1e-12f && T > 1e-20f)
                                        g_logT = fmaf(gq, __fdiv_rn(__fmul_rn(dt, q), __fmul_rn(alpha, T)), g_logT);
                                    ++qi;
                                    if (qi < Q) q = __ldg(rq + qi);
                                }
                            }
                        }
                        dL_dt0 = __fsub_rn(units, dL_ddelta);
                    } else {
                        const float dalpha_ddt = dt > 0.0f ? __fmul_rn(s, oma) : 0.0f;
                        dL_ds = __fmul_rn(dL_dalpha, __fmul_rn(dt, oma));
                        dL_ddelta = __fmul_rn(dL_dalpha, dalpha_ddt);
                        dL_dt0 = 0.0f;
                        while (qi < Q && Tn < q) {
                            const float dgi = __fdiv_rn(__ldg(rdg + qi), s);
                            dL_dt0 = __fadd_rn(dL_dt0, dgi);
                            dL_ds = __fadd_rn(dL_ds, __fdiv_rn(__fmul_rn(-dgi, logf(__fdiv_rn(T, q))), s));
                            cur_depth_grad = __fsub_rn(cur_depth_grad, dgi);
                            ++qi;
                            if (qi < Q) q = __ldg(rq + qi);
                        }
                        if (qi < Q) {
                            dL_ds = fmaf(-dt, cur_depth_grad, dL_ds);
                            dL_ddelta = fmaf(-s, cur_depth_grad, dL_ddelta);
                        }
                        dL_dt0 = __fadd_rn(dL_dt0, -dL_ddelta);
                    }
                    const float dL_dt1 = dL_ddelta;

                    // geometry: bisector-plane derivatives of t0 and t1.  The
                    // reference evaluates d t0 / d current against prev_point
                    // even on the first step, where prev_point is (0,0,0).
                    float a0x, a0y, a0z, b0x, b0y, b0z;
                    cig_pair(qpx, qpy, qpz, px, py, pz, ray, a0x, a0y, a0z, b0x, b0y, b0z);
                    if (prev_idx == kNone) {
                        a0x = 0.0f;
                        a0y = 0.0f;
                        a0z = 0.0f;
                    }
                    float b1x, b1y, b1z, c1x, c1y, c1z;
                    cig_pair(px, py, pz, nh.px, nh.py, nh.pz, ray, b1x, b1y, b1z, c1x, c1y, c1z);
                    pgx = fmaf(dL_dt0, a0x, pgx);
                    pgy = fmaf(dL_dt0, a0y, pgy);
                    pgz = fmaf(dL_dt0, a0z, pgz);
                    cgx = __fadd_rn(cgx, fmaf(dL_dt0, b0x, __fmul_rn(dL_dt1, b1x)));
                    cgy = __fadd_rn(cgy, fmaf(dL_dt0, b0y, __fmul_rn(dL_dt1, b1y)));
                    cgz = __fadd_rn(cgz, fmaf(dL_dt0, b0z, __fmul_rn(dL_dt1, b1z)));
                    const float ngx = __fmul_rn(dL_dt1, c1x);
                    const float ngy = __fmul_rn(dL_dt1, c1y);
                    const float ngz = __fmul_rn(dL_dt1, c1z);
                    if (prev_idx != kNone) atomicAdd(P.point_acc + prev_idx, make_float4(pgx, pgy, pgz, 0.0f));
                    qpx = px;
                    qpy = py;
                    qpz = pz;
                    prev_idx = cur;
                    pgx = cgx;
                    pgy = cgy;
                    pgz = cgz;
                    cgx = ngx;
                    cgy = ngy;
                    cgz = ngz;

                    float last_grad = 0.0f;
                    bool with_last = false;
                    if (NEUS) {
                        const float omtp = fmaf(-2.0f, phi, 1.0f);
                        const float dphi_dd = __fmul_rn(__fmul_rn(-sha, phi), __fsub_rn(1.0f, phi));
                        const float ds_dd = __fmul_rn(__fmul_rn(sha, omtp), dphi_dd);
                        const float ds_dsha = __fmul_rn(__fmul_rn(phi, __fsub_rn(1.0f, phi)),
                                                        fmaf(-__fmul_rn(sha, d), omtp, 1.0f));
                        const float dL_dd = __fmul_rn(dL_ds, ds_dd);
                        sha_sum = __fadd_rn(sha_sum, __fmul_rn(dL_ds, ds_dsha));
                        if (sdf_set >= 0) {
                            if (sdf_fast) {
                                last_grad = dL_dd;
                                with_last = true;
                            } else {
                                atomicAdd(reinterpret_cast<float *>(P.attr_acc + size_t(cur) * V) + sdf_ch, dL_dd);
                            }
                        }
                    } else {
                        last_grad = dL_ds;
                        with_last = true;
                    }
                    if (cr == 0.0f) gr = 0.0f;
                    if (cg == 0.0f) gg = 0.0f;
                    if (cb == 0.0f) gb = 0.0f;
                    scatter_row<DEG>(P.attr_acc + size_t(cur) * V, Y, gr, gg, gb, last_grad, with_last);
                    T = Tn;
                    if (!(T > thr)) break;
                }
                t0 = fmaxf(t0, t1);
                cur = nxt;
                h = nh;
            }
        }
    }
    if (NEUS && P.sharpness_grad) {
        // one atomic per block instead of one per step
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sha_sum += __shfl_xor_sync(0xffffffffu, sha_sum, o);
        if ((threadIdx.x & 31) == 0) block_sha[threadIdx.x >> 5] = sha_sum;
        __syncthreads();
        if (threadIdx.x == 0) {
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < kBlock / 32; ++w) s += block_sha[w];
            atomicAdd(P.sharpness_grad, s);
        }
    }
}

template <int V>
__global__ void __launch_bounds__(256) fold_grads_kernel(uint32_t num_points, int attr_dim,
                                                         const float4 *__restrict__ attr_acc,
                                                         const float4 *__restrict__ point_acc,
                                                         float *__restrict__ attr_grad,
                                                         float *__restrict__ points_grad) {
    const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint64_t na = uint64_t(num_points) * attr_dim;
    if (i < na) {
        const uint64_t c = i / attr_dim;
        const int ch = static_cast<int>(i % attr_dim);
        attr_grad[i] = __ldg(reinterpret_cast<const float *>(attr_acc + c * V) + ch);
    }
    if (i < uint64_t(num_points) * 3) {
        const uint64_t c = i / 3;
        points_grad[i] = __ldg(reinterpret_cast<const float *>(point_acc + c) + (i % 3));
    }
}

template <int DEG>
cudaError_t launch_forward_deg(const ForwardParams &p, cudaStream_t stream) {
    const uint32_t blocks = (p.num_rays + kBlock - 1) / kBlock;
    if (p.settings.alpha_mode == SDFOAM_ALPHA_NEUS)
        forward_kernel<DEG, true><<<blocks, kBlock, 0, stream>>>(p);
    else
        forward_kernel<DEG, false><<<blocks, kBlock, 0, stream>>>(p);
    return cudaGetLastError();
}

template <int DEG>
cudaError_t launch_backward_deg(const BackwardParams &p, cudaStream_t stream) {
    const uint32_t blocks = (p.num_rays + kBlock - 1) / kBlock;
    if (p.settings.alpha_mode == SDFOAM_ALPHA_NEUS)
        backward_kernel<DEG, true><<<blocks, kBlock, 0, stream>>>(p);
    else
        backward_kernel<DEG, false><<<blocks, kBlock, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_forward(uint32_t sh_degree, const ForwardParams &p, cudaStream_t stream) {
    if (p.num_rays == 0) return cudaSuccess;
    switch (sh_degree) {
    case 0: return launch_forward_deg<0>(p, stream);
    case 1: return launch_forward_deg<1>(p, stream);
    case 2: return launch_forward_deg<2>(p, stream);
    case 3: return launch_forward_deg<3>(p, stream);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_backward(uint32_t sh_degree, const BackwardParams &p, cudaStream_t stream) {
    if (p.num_rays == 0) return cudaSuccess;
    switch (sh_degree) {
    case 0: return launch_backward_deg<0>(p, stream);
    case 1: return launch_backward_deg<1>(p, stream);
    case 2: return launch_backward_deg<2>(p, stream);
    case 3: return launch_backward_deg<3>(p, stream);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_fold_grads(uint32_t sh_degree, uint32_t num_points, const float4 *attr_acc,
                              const float4 *point_acc, float *attr_grad, float *points_grad,
                              cudaStream_t stream) {
    if (num_points == 0) return cudaSuccess;
    const int A = attr_dim_of(sh_degree);
    const uint64_t total = uint64_t(num_points) * (A > 3 ? A : 3);
    const uint32_t blocks = static_cast<uint32_t>((total + 255) / 256);
    switch (attr_vec4_of(sh_degree)) {
    case 1: fold_grads_kernel<1><<<blocks, 256, 0, stream>>>(num_points, A, attr_acc, point_acc, attr_grad, points_grad); break;
    case 4: fold_grads_kernel<4><<<blocks, 256, 0, stream>>>(num_points, A, attr_acc, point_acc, attr_grad, points_grad); break;
    case 7: fold_grads_kernel<7><<<blocks, 256, 0, stream>>>(num_points, A, attr_acc, point_acc, attr_grad, points_grad); break;
    case 13: fold_grads_kernel<13><<<blocks, 256, 0, stream>>>(num_points, A, attr_acc, point_acc, attr_grad, points_grad); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace sdfoam_b200
