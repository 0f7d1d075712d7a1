// Forward and backward Voronoi-foam walk kernels for sm_100a.
//
// One lane walks one ray; its state (origin, direction, SH basis, t0, T,
// colour accumulators) stays in registers for the whole walk.  Per step the
// lane reads the current site's plane row (binary16 offsets, four faces per
// 256-bit load), keeps the first face with the smallest exit distance, reads
// that face's record (next site, its CSR start and degree), then the next
// site's 32-byte head (position, face range, last attribute channel) with one
// 256-bit load and the current site's SH row with 256-bit loads.  The walk is
// bound by the L1 data pipeline (one wavefront per lane and load for these
// scattered rows), so loads per step are what counts.
//
// Latency.  A step's loads depend on the previous step's exit face; the
// face record of the winner carries the neighbour's id, first CSR entry
// and degree, and the warps resident on an SM hide the round trips (explicit
// L1 prefetches of the next site's lines measured 1-2 % slower).  The
// backward walk applies the two plane derivatives that need the next site's
// position one iteration later (they only feed gradients that are flushed
// later), so no step waits on a dependent load.
//
// Semantics follow the reference walk and cell functors:
//   trace()        src/tracing/tracing_utils.cuh:17-109
//   forward        src/tracing/pipeline.cu:36-264
//   backward_sdf   src/tracing/pipeline.cu:267-550  (NeuS mode)
//   backward       src/tracing/pipeline.cu:553-791  (RadFoam density mode,
//                  "unsafe" exit-face rule without the t > t0 test)
// Gradient scatter.  The backward walks warp-synchronously (one step per
// iteration for every live lane) so that after each step the lanes whose
// attribute-gradient rows go to the same site are combined in shared memory
// and the sum is added with one 128-bit vector atomic (red.global.add.v4.f32)
// per float4 of the row; coherent rays share sites (2.5 rows per site and
// step on average), and with dense gradients (an SDF from the sdfnet)
// same-address atomics from every lane made the backward 1.8x slower.  Rows are 16-byte aligned per-site
// buffers folded into the caller's [N,A] / [N,3] outputs afterwards.  The
// per-step sharpness gradient of the reference (a single-address atomic per
// step) is summed in registers and reduced once per block.
#include <cfloat>
#include <type_traits>

#include "foam_device.cuh"
#include "foam_internal.h"

namespace sdfoam_b200 {

namespace {

constexpr int kBlock = 128;

// Attribute-typed buffers (float32 or binary16 pipelines).
template <typename AT>
__device__ __forceinline__ float attr_to_f(const void *base, size_t i) {
    if constexpr (std::is_same<AT, __half>::value)
        return __half2float(reinterpret_cast<const __half *>(base)[i]);
    else
        return __ldg(reinterpret_cast<const float *>(base) + i);
}

template <typename AT>
__device__ __forceinline__ float4 load_rgba(const void *base, uint32_t r) {
    if constexpr (std::is_same<AT, __half>::value) {
        const uint2 u = reinterpret_cast<const uint2 *>(base)[r];
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
        return make_float4(a.x, a.y, b.x, b.y);
    } else {
        return reinterpret_cast<const float4 *>(base)[r];
    }
}

template <typename AT>
__device__ __forceinline__ void store_rgba(void *base, uint32_t r, float x, float y, float z, float w) {
    if constexpr (std::is_same<AT, __half>::value) {
        const __half2 a = __floats2half2_rn(x, y), b = __floats2half2_rn(z, w);
        reinterpret_cast<uint2 *>(base)[r] =
            make_uint2(*reinterpret_cast<const uint32_t *>(&a), *reinterpret_cast<const uint32_t *>(&b));
    } else {
        reinterpret_cast<float4 *>(base)[r] = make_float4(x, y, z, w);
    }
}

// atomicAdd(attr_scalar *, (attr_scalar)v) of the reference functors.
template <typename AT>
__device__ __forceinline__ void attr_atomic_add(void *base, size_t i, float v) {
    if constexpr (std::is_same<AT, __half>::value)
        atomicAdd(reinterpret_cast<__half *>(base) + i, __float2half_rn(v));
    else
        atomicAdd(reinterpret_cast<float *>(base) + i, v);
}

// The sharpness as the reference reads it: `*sharpness` of a float buffer
// through an attr_scalar pointer (pipeline.cu:137-141, 381-383), i.e. the
// first two bytes of the float as a binary16 value in the float16 pipeline.
template <typename AT>
__device__ __forceinline__ float read_sharpness(const float *p) {
    if constexpr (std::is_same<AT, __half>::value)
        return __half2float(*reinterpret_cast<const __half *>(p));
    else
        return __ldg(p);
}

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

template <int DEG>
__device__ __forceinline__ const unsigned char *site_ptr(const CellsView &C, uint32_t c) {
    constexpr int SB = (32 + 4 * AttrLayout<DEG>::kStride + 127) / 128 * 128;
    return C.sites + size_t(c) * SB;
}

template <int DEG>
__device__ __forceinline__ Head load_head(const CellsView &C, uint32_t c) {
    uint32_t w[8];
    ldg256(site_ptr<DEG>(C, c), w);
    Head h;
    h.px = __uint_as_float(w[0]);
    h.py = __uint_as_float(w[1]);
    h.pz = __uint_as_float(w[2]);
    h.beg = w[3];
    h.end = w[4];
    h.last = __uint_as_float(w[5]);
    return h;
}

template <int DEG>
__device__ __forceinline__ void load_sh(const CellsView &C, uint32_t c, AttrRow<DEG> &row) {
    const float *src = reinterpret_cast<const float *>(site_ptr<DEG>(C, c) + 32);
#pragma unroll
    for (int i = 0; i < AttrLayout<DEG>::kStride / 8; ++i) ldg256f(src + 8 * i, row.v + 8 * i);
}

// The exit face chosen for one site and what the walk needs about its
// neighbour.
struct Exit {
    float t1;
    uint32_t next, next_beg, next_deg;
    uint32_t face;  // CSR index of the exit face
};

// Face test of trace() (tracing_utils.cuh:64-88) on one binary16 plane
// offset (xy = half(dx) | half(dy) << 16, z = half(dz) in the low half):
// off = half->float, fo = p + off * 0.5, dp = dot(off, d),
// t = dot(fo - o, off) / dp.  SAFE: dp > 0 && t > t0 && t < t1; otherwise
// dp > 0 && t < t1.  Strict '<' keeps the first minimum in CSR order.
template <bool SAFE>
__device__ __forceinline__ void plane_test(const RayState &ray, float px, float py, float pz, float t0, uint32_t xy,
                                           uint32_t z, uint32_t k, float &t1, uint32_t &kbest) {
    const float fx = h2f(xy), fy = h2f(xy >> 16), fz = h2f(z);
    const float wx = __fsub_rn(fmaf(fx, 0.5f, px), ray.ox);
    const float wy = __fsub_rn(fmaf(fy, 0.5f, py), ray.oy);
    const float wz = __fsub_rn(fmaf(fz, 0.5f, pz), ray.oz);
    const float dp = dot3(fx, fy, fz, ray.dx, ray.dy, ray.dz);
    const float t = __fdiv_rn(dot3(wx, wy, wz, fx, fy, fz), dp);
    const bool take = SAFE ? (dp > 0.0f && t > t0 && t < t1) : (dp > 0.0f && t < t1);
    if (take) {
        t1 = t;
        kbest = k;
    }
}

constexpr uint32_t kNoFace = 0xffffffffu;

// The exit face of site `site` (CSR range [beg, end)): the search runs over
// the site's plane row, four faces per 256-bit load (the zero padding never
// wins), then one 128-bit load of the winner's face record gives the next
// site and where its row starts.
template <bool SAFE>
__device__ __forceinline__ bool find_exit(const CellsView &C, uint32_t site, uint32_t beg, uint32_t end,
                                          const RayState &ray, float px, float py, float pz, float t0, Exit &best) {
    const uint2 *row = C.planes + plane_row(site, beg);
    const uint32_t deg = end - beg;
    float t1 = __int_as_float(0x7f800000);
    uint32_t kb = kNoFace;
    for (uint32_t k = 0; k < deg; k += 4) {
        uint32_t w[8];
        ldg256(row + k, w);
        plane_test<SAFE>(ray, px, py, pz, t0, w[0], w[1], k, t1, kb);
        plane_test<SAFE>(ray, px, py, pz, t0, w[2], w[3], k + 1, t1, kb);
        plane_test<SAFE>(ray, px, py, pz, t0, w[4], w[5], k + 2, t1, kb);
        plane_test<SAFE>(ray, px, py, pz, t0, w[6], w[7], k + 3, t1, kb);
    }
    if (kb == kNoFace) return false;
    const uint4 r = __ldg(C.faces + beg + kb);
    best.t1 = t1;
    best.next = r.x;
    best.next_beg = r.y;
    best.next_deg = r.w >> 16;
    best.face = beg + kb;
    return true;
}

// Exit record: per ray one byte per walk iteration that searched for an exit
// face -- its position in the row (0..253), 254 for "no exit (the walk
// ends)", 255 for "not recorded" -- packed eight to a 64-bit word.  The
// forward writes it; the NeuS backward, whose walk takes the same steps,
// replays it with a single face test per step.
constexpr uint32_t kExitNone = 254u, kExitUnknown = 255u;

__device__ __forceinline__ uint32_t exit_code(bool found, const Exit &e, uint32_t beg) {
    if (!found) return kExitNone;
    const uint32_t k = e.face - beg;
    return k < kExitNone ? k : kExitUnknown;
}

// The recorded face's test: the same arithmetic as the search, so the same
// t1 and next site; false if the face does not pass (then the caller
// searches).
template <bool SAFE>
__device__ __forceinline__ bool replay_exit(const uint4 *__restrict__ faces, uint32_t beg, uint32_t end, uint32_t k,
                                            const RayState &ray, float px, float py, float pz, float t0, Exit &best) {
    const uint32_t j = beg + k;
    if (j >= end) return false;
    const uint4 r = __ldg(faces + j);
    float t1 = __int_as_float(0x7f800000);
    uint32_t kb = kNoFace;
    plane_test<SAFE>(ray, px, py, pz, t0, r.z, r.w & 0xffffu, k, t1, kb);
    if (kb == kNoFace) return false;
    best.t1 = t1;
    best.next = r.x;
    best.next_beg = r.y;
    best.next_deg = r.w >> 16;
    best.face = j;
    return true;
}

// CSR range of the site the walk enters, from the exit face's record (or the
// head for very long rows); invalid rows become an empty-and-reversed range
// that the loop head rejects like the reference (beg > end).
__device__ __forceinline__ void next_range(const Exit &e, const Head &nh, uint32_t &beg, uint32_t &end) {
    if (e.next_deg < kDegFromHead) {
        beg = e.next_beg;
        end = e.next_beg + e.next_deg;
    } else if (e.next_deg == kDegFromHead) {
        beg = nh.beg;
        end = nh.end;
    } else {
        beg = 1u;
        end = 0u;
    }
}

// NeuS density s = sha * phi * (1 - phi), phi = 1 / (1 + exp(sha * d))
// (pipeline.cu:149, 386-387).
__device__ __forceinline__ float neus_phi(float sha, float d) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, foam_expf(__fmul_rn(sha, d))));
}

// Attribute channel ch of a site: the last channel lives in the head, the
// others in the SH row of the site record.
template <int DEG>
__device__ __forceinline__ float attr_channel(const CellsView &C, uint32_t site, float last, int ch) {
    constexpr int A = AttrLayout<DEG>::kDim;
    if (ch == A - 1) return last;
    return __ldg(reinterpret_cast<const float *>(site_ptr<DEG>(C, site) + 32) + ch);
}

// --------------------------------------------------------------------------
// forward
// --------------------------------------------------------------------------

template <int DEG, bool NEUS, typename AT>
// Resident blocks per SM the forward is compiled for (its register cap).
#ifndef SDFOAM_FWD_BLOCKS_PER_SM
#define SDFOAM_FWD_BLOCKS_PER_SM 8
#endif
__global__ void __launch_bounds__(kBlock, SDFOAM_FWD_BLOCKS_PER_SM) forward_kernel(const ForwardParams P) {
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= P.num_rays) return;
    const CellsView &C = P.cells;
    const RayState ray = load_ray(P.rays, r);
    // the ray's SH basis in a shared-memory column, read when a step is shaded
    constexpr int NB = AttrLayout<DEG>::kBasis;
    __shared__ float ysh[NB][kBlock];
    {
        SHBasis Y0;
        sh_basis<DEG>(ray.dx, ray.dy, ray.dz, Y0);
#pragma unroll
        for (int k = 0; k < NB; ++k) ysh[k][threadIdx.x] = Y0.y[k];
    }

    const uint32_t Q = P.quantiles ? P.num_quantiles : 0u;
    // per-ray rows (quantiles, exit record, cell sequence) are formed from the
    // kernel parameters where used, not held in registers across the walk
#define RQ (P.quantiles + size_t(r) * P.num_quantiles)
#define REC (P.exits + size_t(r) * P.exits_stride)
    uint32_t qi = 0;
    float q = 0.0f;
    if (P.quantiles && P.num_quantiles > 0) q = __ldg(RQ);
    const int sdf_ch = P.settings.sdf_channel;
    const bool neus_alpha = NEUS && sdf_ch >= 0;
    const float sha = NEUS ? read_sharpness<AT>(P.sharpness) : 0.0f;
    const float thr = P.settings.weight_threshold;
    const uint32_t max_steps = P.settings.max_intersections;

    float T = 1.0f, ar = 0.0f, ag = 0.0f, ab = 0.0f;
    float t0 = 0.0f;
    uint32_t n = 0;
    uint32_t nseq = 0;
    uint32_t faces_seen = 0;

    uint64_t rec_word = 0;
    uint32_t searched = 0;

    uint32_t cur = __ldg(P.start + r);
    if (cur < C.num_points) {
        Head h = load_head<DEG>(C, cur);
        uint32_t beg = h.beg, end = h.end;
        for (;;) {
            ++n;
            if (n > max_steps) break;
            // the step record: the site entered at this step, or kNone where the walk ends
            uint32_t *srec = (P.sites && n - 1 < P.colors_steps) ? P.sites + size_t(n - 1) * P.num_rays + r
                                                                  : nullptr;
            if (beg > end || end > C.adjacency_size) {
                if (srec) __stcs(srec, kNone);
                break;
            }
            faces_seen += end - beg;
            Exit ex;
            const bool found = find_exit<true>(C, cur, beg, end, ray, h.px, h.py, h.pz, t0, ex);
            if (srec) __stcs(srec, (found && ex.next < C.num_points) ? ex.next : kNone);
            if (P.exits && searched < P.exits_stride) {
                rec_word |= uint64_t(exit_code(found, ex, beg)) << (8 * (searched & 7u));
                if ((searched & 7u) == 7u) {
                    *reinterpret_cast<uint64_t *>(REC + (searched & ~7u)) = rec_word;
                    rec_word = 0;
                }
            }
            ++searched;
            if (!found) break;
            if (ex.next >= C.num_points) break;
            const float t1 = ex.t1;
            if (t1 > t0) {
                AttrRow<DEG> row;
                load_sh<DEG>(C, cur, row);
                float cr = 0.0f, cg = 0.0f, cb = 0.0f;
                if (NEUS || h.last > 1e-6f) {
                    SHBasis Y;
                    const volatile float *col = &ysh[0][threadIdx.x];
#pragma unroll
                    for (int k = 0; k < NB; ++k) Y.y[k] = col[k * kBlock];
                    sh_rgb<DEG>(Y, row, cr, cg, cb);
                }
                if (P.colors && n - 1 < P.colors_steps)
                    __stcs(P.colors + size_t(n - 1) * P.num_rays + r, make_float4(cr, cg, cb, t1));
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
                if (P.contribution) attr_atomic_add<AT>(P.contribution, cur, w);
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
                            if (qi < Q) q = __ldg(RQ + qi);
                        }
                    }
                } else {
                    while (qi < Q && Tn < q) {
                        P.depth[size_t(r) * Q + qi] = __fadd_rn(t0, __fdiv_rn(logf(__fdiv_rn(T, q)), s));
                        P.depth_indices[size_t(r) * Q + qi] = cur;
                        ++qi;
                        if (qi < Q) q = __ldg(RQ + qi);
                    }
                }
                if (P.seq_cells) {
                    const uint64_t pos = P.seq_offsets[r] + nseq;
                    if (pos < P.seq_offsets[r + 1]) P.seq_cells[pos] = cur;
                }
                ++nseq;
                T = Tn;
                if (!(T > thr)) break;
            }
            t0 = fmaxf(t0, t1);
            cur = ex.next;
            h = load_head<DEG>(C, cur);
            next_range(ex, h, beg, end);
        }
    }
    while (qi < Q) {
        P.depth[size_t(r) * Q + qi] = -1.0f;
        P.depth_indices[size_t(r) * Q + qi] = kNone;
        ++qi;
    }
    if (P.exits && (searched & 7u) && searched <= P.exits_stride)
        *reinterpret_cast<uint64_t *>(REC + ((searched - 1) & ~7u)) = rec_word;
    store_rgba<AT>(P.rgba, r, ar, ag, ab, __fsub_rn(1.0f, T));
    if (P.num_intersections) P.num_intersections[r] = n;
    if (P.seq_count) P.seq_count[r] = nseq;
    if (P.face_tests) P.face_tests[r] = faces_seen;
}

#undef RQ
#undef REC

// --------------------------------------------------------------------------
// headless render (trace_benchmark)
// --------------------------------------------------------------------------

constexpr float kPi = 3.14159265358979f;  // M_PIf

// cast_ray (camera.h:56-85) followed by the render kernel's own check and
// second normalisation (pipeline.cu:1101-1113).  Vector sums contract like
// the reference's device code: x*a + y*b -> fma(x, a, y*b), then + z*c ->
// fma(z, c, ...).  False for fisheye pixels outside the lens.
__device__ __forceinline__ bool camera_ray(const RenderParams &P, uint32_t i, uint32_t j, RayState &ray) {
    const float x = __fdiv_rn(float(i), float(P.width));
    const float y = __fdiv_rn(float(j), float(P.height));
    const float u = __fmul_rn(__fsub_rn(__fmul_rn(2.0f, x), 1.0f), P.aspect);
    const float v = __fsub_rn(1.0f, __fmul_rn(2.0f, y));
    float d[3];
    float mask = 1.0f;
    if (P.model == SDFOAM_PINHOLE) {
#pragma unroll
        for (int k = 0; k < 3; ++k) d[k] = fmaf(v, P.up[k], fmaf(P.focal, P.forward[k], __fmul_rn(u, P.right[k])));
    } else {
        const float theta = atan2f(v, u);
        float phi = __fmul_rn(P.fov, __fsqrt_rn(fmaf(u, u, __fmul_rn(v, v))));
        if (phi >= kPi) {
            phi = __fsub_rn(kPi, 1e-6f);
            mask = 0.0f;
        }
        const float sp = sinf(phi);
        const float a = __fmul_rn(sp, cosf(theta)), b = __fmul_rn(sp, sinf(theta)), c = cosf(phi);
#pragma unroll
        for (int k = 0; k < 3; ++k) d[k] = fmaf(c, P.forward[k], fmaf(a, P.right[k], __fmul_rn(b, P.up[k])));
    }
    const float n2 = dot3(d[0], d[1], d[2], d[0], d[1], d[2]);
    if (n2 > 0.0f) {
        const float len = __fsqrt_rn(n2);
#pragma unroll
        for (int k = 0; k < 3; ++k) d[k] = __fdiv_rn(d[k], len);
    }
#pragma unroll
    for (int k = 0; k < 3; ++k) d[k] = __fmul_rn(d[k], mask);
    const float norm = __fsqrt_rn(dot3(d[0], d[1], d[2], d[0], d[1], d[2]));
    if (norm < 0.1f) return false;
    ray.ox = P.position[0];
    ray.oy = P.position[1];
    ray.oz = P.position[2];
    ray.dx = __fdiv_rn(d[0], norm);
    ray.dy = __fdiv_rn(d[1], norm);
    ray.dz = __fdiv_rn(d[2], norm);
    return true;
}

// make_rgba8 (tracing_utils.cuh:126-136): clamp (a NaN becomes 1) and
// truncate x * 255.
__device__ __forceinline__ uint32_t rgba8(float r, float g, float b, float a) {
    auto q = [](float x) -> uint32_t {
        x = x < 1.0f ? x : 1.0f;
        x = 0.0f < x ? x : 0.0f;
        return static_cast<uint32_t>(static_cast<int>(__fmul_rn(x, 255.0f)));
    };
    return (q(a) << 24) | (q(b) << 16) | (q(g) << 8) | q(r);
}

constexpr int kTileW = 16, kTileH = 8;  // a block's pixels; each warp an 8 x 4 tile

template <int DEG, bool NEUS, typename AT>
__global__ void __launch_bounds__(kBlock) render_kernel(const RenderParams P) {
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t i = blockIdx.x * kTileW + (warp & 1) * 8 + (lane & 7);
    const uint32_t j = blockIdx.y * kTileH + (warp >> 1) * 4 + (lane >> 3);
    if (i >= P.width || j >= P.height) return;
    const size_t out_idx = size_t(P.height - 1 - j) * P.width + i;
    float bg[3] = {P.bg[0], P.bg[1], P.bg[2]};
    RayState ray;
    if (!camera_ray(P, i, j, ray)) {
        P.rgba8[out_idx] = rgba8(bg[0], bg[1], bg[2], 1.0f);
        return;
    }
    const CellsView &C = P.cells;
    SHBasis Y;
    sh_basis<DEG>(ray.dx, ray.dy, ray.dz, Y);
    const int sdf_ch = P.settings.sdf_channel;
    const bool neus_alpha = NEUS && sdf_ch >= 0;
    const float sha = NEUS ? read_sharpness<AT>(P.sharpness) : 0.0f;
    const float thr = P.settings.weight_threshold;
    const uint32_t max_steps = P.settings.max_intersections;

    float T = 1.0f, ar = 0.0f, ag = 0.0f, ab = 0.0f;
    float t0 = 0.0f;
    uint32_t n = 0;
    uint32_t cur = __ldg(P.start);
    if (cur < C.num_points) {
        Head h = load_head<DEG>(C, cur);
        uint32_t beg = h.beg, end = h.end;
        for (;;) {
            ++n;
            if (n > max_steps) break;
            if (beg > end || end > C.adjacency_size) break;
            Exit ex;
            if (!find_exit<true>(C, cur, beg, end, ray, h.px, h.py, h.pz, t0, ex)) break;
            if (ex.next >= C.num_points) break;
            const float t1 = ex.t1;
            if (t1 > t0) {
                AttrRow<DEG> row;
                load_sh<DEG>(C, cur, row);
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
                ar = fmaf(w, cr, ar);
                ag = fmaf(w, cg, ag);
                ab = fmaf(w, cb, ab);
                T = __fmul_rn(T, __fsub_rn(1.0f, alpha));
                if (!(T > thr)) break;
            }
            t0 = fmaxf(t0, t1);
            cur = ex.next;
            h = load_head<DEG>(C, cur);
            next_range(ex, h, beg, end);
        }
    }
    if (P.checker) {
        const int is = 2 * int((i / 20) % 2) - 1;
        const int js = 2 * int((j / 20) % 2) - 1;
        bg[0] = bg[1] = bg[2] = is * js > 0 ? 0.3f : 0.5f;
    }
    P.rgba8[out_idx] = rgba8(fmaf(T, bg[0], ar), fmaf(T, bg[1], ag), fmaf(T, bg[2], ab), 1.0f);
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

// SH gradient row (value Y_k * g_c at channel 3k+c, plus `last` at channel
// A-1) written to this lane's staging slot for the warp's aggregated scatter.
template <int DEG>
__device__ __forceinline__ void stage_row(float4 *__restrict__ slot, const SHBasis &Y, float gr, float gg, float gb,
                                          float last, bool with_last) {
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
        slot[v] = make_float4(e[0], e[1], e[2], e[3]);
    }
}

__device__ __forceinline__ void red_add_v4(float4 *p, float4 v) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

// Groups of at most this many rows for one site add their rows directly.
// (Measured on the headline workload, backward ms: 99.4 with none, 99.3
// with single rows, 102.8 with up to 3, 118.9 up to 8, 182.9 with all rows
// direct.)
constexpr int kDirectRows = 1;

// Warp-cooperative scatter of one gradient row per lane (Y_k * g_c at
// channel 3k+c, `last` at channel A-1).  Lanes whose rows go to the same
// site form one group (__match_any_sync).  A lane alone with its site adds
// its row with vector atomics straight from registers.  Larger groups stage
// their rows in shared memory; the (group, float4) slots are spread over
// the lanes, each slot sums its group's rows in lane order and issues one
// vector atomic, which turns many same-address atomics of coherent rays
// into one.  All 32 lanes must call it.
template <int DEG>
__device__ __forceinline__ void warp_scatter(float4 (*stage)[AttrLayout<DEG>::kVec4], uint32_t *gmask,
                                             uint32_t *gcell, bool has_row, uint32_t cell, const SHBasis &Y,
                                             float gr, float gg, float gb, float last,
                                             float4 *__restrict__ attr_acc) {
    constexpr int V = AttrLayout<DEG>::kVec4;
    constexpr int NSH = AttrLayout<DEG>::kSH;
    constexpr int A = AttrLayout<DEG>::kDim;
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t any = __ballot_sync(0xffffffffu, has_row);
    if (any == 0u) return;
    const uint32_t key = has_row ? cell : (0xffffffe0u | lane);  // unique keys for lanes without a row
    const uint32_t grp = __match_any_sync(0xffffffffu, key);
    const bool direct = has_row && __popc(grp) <= kDirectRows;
    if (direct) {
        const float g3[3] = {gr, gg, gb};
        float4 *dst = attr_acc + size_t(cell) * V;
#pragma unroll
        for (int v = 0; v < V; ++v) {
            float e[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int i = 4 * v + k;
                e[k] = i < NSH ? __fmul_rn(Y.y[i / 3], g3[i % 3]) : (i == A - 1 ? last : 0.0f);
            }
            if (e[0] != 0.0f || e[1] != 0.0f || e[2] != 0.0f || e[3] != 0.0f)
                red_add_v4(dst + v, make_float4(e[0], e[1], e[2], e[3]));
        }
    }
    const bool staged = has_row && !direct;
    if (__ballot_sync(0xffffffffu, staged) == 0u) return;
    if (staged) stage_row<DEG>(stage[lane], Y, gr, gg, gb, last, true);
    const bool leader = staged && lane == uint32_t(__ffs(grp) - 1);
    const uint32_t leaders = __ballot_sync(0xffffffffu, leader);
    if (leader) {
        const uint32_t k = __popc(leaders & ((1u << lane) - 1u));
        gmask[k] = grp;
        gcell[k] = cell;
    }
    __syncwarp();
    const uint32_t G = __popc(leaders);
    for (uint32_t idx = lane; idx < G * V; idx += 32u) {
        const uint32_t gi = idx / V, v = idx % V;
        uint32_t mem = gmask[gi];
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        while (mem) {
            const uint32_t l = __ffs(mem) - 1;
            mem &= mem - 1u;
            const float4 x = stage[l][v];
            acc.x = __fadd_rn(acc.x, x.x);
            acc.y = __fadd_rn(acc.y, x.y);
            acc.z = __fadd_rn(acc.z, x.z);
            acc.w = __fadd_rn(acc.w, x.w);
        }
        if (acc.x != 0.0f || acc.y != 0.0f || acc.z != 0.0f || acc.w != 0.0f)
            red_add_v4(attr_acc + size_t(gcell[gi]) * V + v, acc);
    }
    __syncwarp();
}

// a / b for the gradient-only quotients of the backward, without the IEEE
// division's special-case branch: the product with an approximate reciprocal
// y of b, refined once with its fused remainder, q = q0 + (a - b q0) y (the
// correction step of P. Markstein, "Computation of elementary functions on
// the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990).  For b
// in the normal range it is within an ulp of the IEEE quotient (on the stress
// foam the gradients came out as with IEEE division); the walk's own
// decisions keep IEEE division.
__device__ __forceinline__ float rcp_approx(float b) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(b));
    return y;
}
__device__ __forceinline__ float div_refined(float a, float b, float y) {
    const float q0 = __fmul_rn(a, y);
    return fmaf(fmaf(-b, q0, a), y, q0);
}

// Resident blocks per SM the backward is compiled for (its register cap).
#ifndef SDFOAM_BWD_BLOCKS_PER_SM
#define SDFOAM_BWD_BLOCKS_PER_SM 5
#endif

template <int DEG, bool NEUS, typename AT>
__global__ void __launch_bounds__(kBlock, SDFOAM_BWD_BLOCKS_PER_SM) backward_kernel(const BackwardParams P) {
    constexpr int A = AttrLayout<DEG>::kDim;
    constexpr int V = AttrLayout<DEG>::kVec4;
    constexpr int W = kBlock / 32;
    __shared__ float4 stage[W][32][V];
    __shared__ uint32_t gmask[W][32];
    __shared__ uint32_t gcell[W][32];
    __shared__ float block_sha[W];
    // the ray's SH basis, kept in shared memory (one column per thread)
    // instead of 16 registers for the whole walk
    constexpr int NB = AttrLayout<DEG>::kBasis;
    __shared__ float ysh[NB][kBlock];
    auto load_basis = [&](SHBasis &Yl) {
        const volatile float *col = &ysh[0][threadIdx.x];
#pragma unroll
        for (int k = 0; k < NB; ++k) Yl.y[k] = col[k * kBlock];
    };
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t lane = threadIdx.x & 31u, wid = threadIdx.x >> 5;
    const CellsView &C = P.cells;
    float sha_sum = 0.0f;
    bool alive = false;

    // per-ray state (rays past the end stay idle but join the warp collectives)
    RayState ray{};
    SHBasis Y0;
    float4 g = make_float4(0.0f, 0.0f, 0.0f, 0.0f), Cf = g;
    uint32_t Q = 0;
    // per-ray rows of the quantile inputs and the exit record, formed from the
    // kernel parameters where used (no registers held across the walk)
    const bool has_q = P.quantiles != nullptr;
#define RQ (P.quantiles + size_t(r) * P.num_quantiles)
#define RDG (P.depth_grad + size_t(r) * P.num_quantiles)
#define REC (P.exits + size_t(r) * P.exits_stride)
    float err = 0.0f;
    const float thr = P.settings.weight_threshold;
    const uint32_t max_steps = P.settings.max_intersections;
    const int sdf_set = P.settings.sdf_channel;
    const int sdf_ch = NEUS ? (sdf_set >= 0 ? sdf_set : A - 1) : A - 1;
    const bool sdf_fast = sdf_ch == A - 1;
    const float sha = NEUS ? read_sharpness<AT>(P.sharpness) : 0.0f;
    uint32_t qi = 0;
    float q = 0.0f;
    float cur_depth_grad = 0.0f;
    float g_logT = 0.0f;
    float T = 1.0f, ar = 0.0f, ag = 0.0f, ab = 0.0f;
    uint32_t prev_idx = kNone;
    float qpx = 0.0f, qpy = 0.0f, qpz = 0.0f;          // prev point
    float pgx = 0.0f, pgy = 0.0f, pgz = 0.0f;          // prev point grad
    float cgx = 0.0f, cgy = 0.0f, cgz = 0.0f;          // current point grad
    float pend_dt1 = 0.0f;                              // deferred dL/dt1 of the last functor call
    bool pending = false;
    float t0 = 0.0f;
    uint32_t n = 0;
    uint32_t cur = kNone, beg = 1u, end = 0u;
    Head h{};
    uint64_t rec_word = 0;
    if (r < P.num_rays) {
        ray = load_ray(P.rays, r);
        sh_basis<DEG>(ray.dx, ray.dy, ray.dz, Y0);
        g = load_rgba<AT>(P.rgba_grad, r);
        Cf = load_rgba<AT>(P.rgba, r);
        Q = P.quantiles ? P.num_quantiles : 0u;
        err = P.ray_error ? attr_to_f<AT>(P.ray_error, r) : 0.0f;
        if (has_q && P.num_quantiles > 0) q = __ldg(RQ);
        // RadFoam mode: sum of depth_grad / s over the recorded quantile sites
        // (pipeline.cu:620-629)
        if (!NEUS) {
            for (uint32_t i = 0; i < Q; ++i) {
                const uint32_t pi = P.depth_indices[size_t(r) * Q + i];
                if (pi < C.num_points) {  // kNone marks an unfilled quantile
                    const float sv = load_head<DEG>(C, pi).last;
                    cur_depth_grad = __fadd_rn(cur_depth_grad, __fdiv_rn(__ldg(RDG + i), sv));
                }
            }
        }
        cur = __ldg(P.start + r);
        if (cur < C.num_points) {
            h = load_head<DEG>(C, cur);
            beg = h.beg;
            end = h.end;
            alive = true;
        }
    }

#pragma unroll
    for (int k = 0; k < NB; ++k) ysh[k][threadIdx.x] = r < P.num_rays ? Y0.y[k] : 0.0f;
    __syncwarp();

    // One walk step per iteration for every live lane of the warp; the
    // gradient rows of the step are scattered together afterwards.
    while (__any_sync(0xffffffffu, alive)) {
        bool has_row = false;
        uint32_t row_cell = 0;
        float row_r = 0.0f, row_g = 0.0f, row_b = 0.0f, row_last = 0.0f;
        if (alive) {
            do {
                ++n;
                // a step the forward recorded: its exit distance, the site it
                // entered and its colour, read coalesced (the warp's lanes are
                // at the same step) -- no face test
                const bool colored = NEUS && P.colors && n - 1 < P.colors_steps;
                const bool recorded = colored && P.sites;
                if (n > max_steps || (!recorded && (beg > end || end > C.adjacency_size))) {
                    alive = false;
                    break;
                }
                Exit ex;
                uint32_t next;
                float t1;
                float4 crec = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (recorded) {
                    const size_t k = size_t(n - 1) * P.num_rays + r;
                    next = __ldcs(P.sites + k);
                    if (next == kNone) {  // the forward's walk ended at this step
                        alive = false;
                        break;
                    }
                    crec = __ldcs(P.colors + k);
                    t1 = crec.w;
                } else {
                    uint32_t code = kExitUnknown;
                    if (NEUS && P.exits && n - 1 < P.exits_stride) {
                        if (((n - 1) & 7u) == 0)
                            rec_word = __ldg(reinterpret_cast<const unsigned long long *>(REC + (n - 1)));
                        code = uint32_t(rec_word >> (8 * ((n - 1) & 7u))) & 0xffu;
                    }
                    bool found;
                    if (code == kExitNone) {
                        found = false;
                    } else if (code < kExitNone &&
                               replay_exit<NEUS>(C.faces, beg, end, code, ray, h.px, h.py, h.pz, t0, ex)) {
                        found = true;
                    } else {
                        found = find_exit<NEUS>(C, cur, beg, end, ray, h.px, h.py, h.pz, t0, ex);
                    }
                    if (!found || ex.next >= C.num_points) {
                        alive = false;
                        break;
                    }
                    next = ex.next;
                    t1 = ex.t1;
                }
                if (t1 > t0) {
                    const float px = h.px, py = h.py, pz = h.pz;
                    const float last = h.last;
                    float cr = 0.0f, cg = 0.0f, cb = 0.0f;
                    if (colored) {
                        // the forward's colour of this step
                        if (!recorded) crec = __ldcs(P.colors + size_t(n - 1) * P.num_rays + r);
                        cr = crec.x;
                        cg = crec.y;
                        cb = crec.z;
                    } else {
                        AttrRow<DEG> row;
                        load_sh<DEG>(C, cur, row);
                        if (NEUS || last > 1e-6f) {
                            SHBasis Yl;
                            load_basis(Yl);
                            sh_rgb<DEG>(Yl, row, cr, cg, cb);
                        }
                    }
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
                    if (P.point_error) attr_atomic_add<AT>(P.point_error, cur, __fmul_rn(w, err));
                    float gr = __fmul_rn(g.x, w), gg = __fmul_rn(g.y, w), gb = __fmul_rn(g.z, w);
                    const float denom = NEUS ? fmaf(T, oma, 1e-6f) : __fmul_rn(T, __fadd_rn(oma, 1e-6f));
                    const float yd = rcp_approx(denom);
                    const float ux = __fsub_rn(cr, div_refined(__fsub_rn(Cf.x, ar), denom, yd));
                    const float uy = __fsub_rn(cg, div_refined(__fsub_rn(Cf.y, ag), denom, yd));
                    const float uz = __fsub_rn(cb, div_refined(__fsub_rn(Cf.z, ab), denom, yd));
                    float dL_dalpha = __fmul_rn(T, dot3(ux, uy, uz, g.x, g.y, g.z));
                    const float om6 = __fadd_rn(oma, 1e-6f);
                    dL_dalpha = __fadd_rn(dL_dalpha, div_refined(__fmul_rn(__fsub_rn(1.0f, Cf.w), g.w), om6,
                                                                 rcp_approx(om6)));
                    const float Tn = __fmul_rn(T, oma);
                    float dL_ds, dL_ddelta, dL_dt0;
                    if (NEUS) {
                        const float om12 = fmaxf(oma, 1e-12f);
                        dL_dalpha = __fadd_rn(dL_dalpha, div_refined(-g_logT, om12, rcp_approx(om12)));
                        dL_ds = __fmul_rn(dL_dalpha, __fmul_rn(dt, oma));
                        dL_ddelta = __fmul_rn(dL_dalpha, __fmul_rn(s, oma));
                        float units = 0.0f;
                        if (has_q && P.num_quantiles > 0) {
                            const float drop = __fsub_rn(T, Tn);
                            if (drop > 1e-12f) {
                                while (qi < Q && Tn < q) {
                                    const float gq = __ldg(RDG + qi);
                                    float frac = __fdiv_rn(__fsub_rn(T, q), drop);
                                    frac = fminf(1.0f, fmaxf(0.0f, frac));
                                    units = __fadd_rn(units, gq);
                                    dL_ddelta = fmaf(gq, frac, dL_ddelta);
                                    if (alpha > 1e-12f && T > 1e-20f)
                                        g_logT = fmaf(gq, __fdiv_rn(__fmul_rn(dt, q), __fmul_rn(alpha, T)), g_logT);
                                    ++qi;
                                    if (qi < Q) q = __ldg(RQ + qi);
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
                            const float dgi = __fdiv_rn(__ldg(RDG + qi), s);
                            dL_dt0 = __fadd_rn(dL_dt0, dgi);
                            dL_ds = __fadd_rn(dL_ds, __fdiv_rn(__fmul_rn(-dgi, logf(__fdiv_rn(T, q))), s));
                            cur_depth_grad = __fsub_rn(cur_depth_grad, dgi);
                            ++qi;
                            if (qi < Q) q = __ldg(RQ + qi);
                        }
                        if (qi < Q) {
                            dL_ds = fmaf(-dt, cur_depth_grad, dL_ds);
                            dL_ddelta = fmaf(-s, cur_depth_grad, dL_ddelta);
                        }
                        dL_dt0 = __fadd_rn(dL_dt0, -dL_ddelta);
                    }

                    // geometry (tracing_utils.cuh:112-124 via pipeline.cu:485-506):
                    // the t0 derivatives now; the t1 derivatives, which need
                    // the next site's position, right after the move below.
                    // The reference evaluates d t0 / d current against
                    // prev_point even on the first step, where it is (0,0,0).
                    float a0x, a0y, a0z, b0x, b0y, b0z;
                    cig_pair(qpx, qpy, qpz, px, py, pz, ray, a0x, a0y, a0z, b0x, b0y, b0z);
                    if (prev_idx == kNone) {
                        a0x = 0.0f;
                        a0y = 0.0f;
                        a0z = 0.0f;
                    }
                    pgx = fmaf(dL_dt0, a0x, pgx);
                    pgy = fmaf(dL_dt0, a0y, pgy);
                    pgz = fmaf(dL_dt0, a0z, pgz);
                    cgx = fmaf(dL_dt0, b0x, cgx);
                    cgy = fmaf(dL_dt0, b0y, cgy);
                    cgz = fmaf(dL_dt0, b0z, cgz);
                    if (prev_idx != kNone) red_add_v4(P.point_acc + prev_idx, make_float4(pgx, pgy, pgz, 0.0f));
                    qpx = px;
                    qpy = py;
                    qpz = pz;
                    prev_idx = cur;
                    pgx = cgx;
                    pgy = cgy;
                    pgz = cgz;
                    cgx = 0.0f;
                    cgy = 0.0f;
                    cgz = 0.0f;
                    pend_dt1 = dL_ddelta;
                    pending = true;

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
                    row_r = cr == 0.0f ? 0.0f : gr;
                    row_g = cg == 0.0f ? 0.0f : gg;
                    row_b = cb == 0.0f ? 0.0f : gb;
                    row_last = with_last ? last_grad : 0.0f;
                    has_row = true;
                    row_cell = cur;
                    T = Tn;
                    if (!(T > thr)) {
                        alive = false;
                        break;
                    }
                }
                t0 = fmaxf(t0, t1);
                cur = next;
                h = load_head<DEG>(C, cur);
                if (recorded) {
                    beg = h.beg;
                    end = h.end;
                } else {
                    next_range(ex, h, beg, end);
                }
                if (pending) {
                    // t1 derivatives of the last functor call: its next site is
                    // the one just entered (prev point = that call's site)
                    float b1x, b1y, b1z, c1x, c1y, c1z;
                    cig_pair(qpx, qpy, qpz, h.px, h.py, h.pz, ray, b1x, b1y, b1z, c1x, c1y, c1z);
                    pgx = fmaf(pend_dt1, b1x, pgx);
                    pgy = fmaf(pend_dt1, b1y, pgy);
                    pgz = fmaf(pend_dt1, b1z, pgz);
                    cgx = __fmul_rn(pend_dt1, c1x);
                    cgy = __fmul_rn(pend_dt1, c1y);
                    cgz = __fmul_rn(pend_dt1, c1z);
                    pending = false;
                }
            } while (false);
        }
        SHBasis Yl;
        load_basis(Yl);
        warp_scatter<DEG>(stage[wid], gmask[wid], gcell[wid], has_row, row_cell, Yl, row_r, row_g, row_b, row_last,
                          P.attr_acc);
    }
    if (NEUS && P.sharpness_grad) {
        // one atomic per block instead of one per step
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sha_sum += __shfl_xor_sync(0xffffffffu, sha_sum, o);
        if (lane == 0) block_sha[wid] = sha_sum;
        __syncthreads();
        if (threadIdx.x == 0) {
            float s = 0.0f;
#pragma unroll
            for (int w2 = 0; w2 < W; ++w2) s += block_sha[w2];
            atomicAdd(P.sharpness_grad, s);
        }
    }
}

template <int V, typename AT>
#undef RQ
#undef RDG
#undef REC

__global__ void __launch_bounds__(256) fold_grads_kernel(uint32_t num_points, int attr_dim,
                                                         const float4 *__restrict__ attr_acc,
                                                         const float4 *__restrict__ point_acc,
                                                         AT *__restrict__ attr_grad,
                                                         float *__restrict__ points_grad) {
    const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint64_t na = uint64_t(num_points) * attr_dim;
    if (i < na) {
        const uint64_t c = i / attr_dim;
        const int ch = static_cast<int>(i % attr_dim);
        const float v = __ldg(reinterpret_cast<const float *>(attr_acc + c * V) + ch);
        if constexpr (std::is_same<AT, __half>::value)
            attr_grad[i] = __float2half_rn(v);
        else
            attr_grad[i] = v;
    }
    if (i < uint64_t(num_points) * 3) {
        const uint64_t c = i / 3;
        points_grad[i] = __ldg(reinterpret_cast<const float *>(point_acc + c) + (i % 3));
    }
}

template <int DEG, typename AT>
cudaError_t launch_forward_deg(const ForwardParams &p, cudaStream_t stream) {
    const uint32_t blocks = (p.num_rays + kBlock - 1) / kBlock;
    if (p.settings.alpha_mode == SDFOAM_ALPHA_NEUS)
        forward_kernel<DEG, true, AT><<<blocks, kBlock, 0, stream>>>(p);
    else
        forward_kernel<DEG, false, AT><<<blocks, kBlock, 0, stream>>>(p);
    return cudaGetLastError();
}

template <int DEG, typename AT>
cudaError_t launch_render_deg(const RenderParams &p, cudaStream_t stream) {
    const dim3 grid((p.width + kTileW - 1) / kTileW, (p.height + kTileH - 1) / kTileH);
    if (p.settings.alpha_mode == SDFOAM_ALPHA_NEUS)
        render_kernel<DEG, true, AT><<<grid, kBlock, 0, stream>>>(p);
    else
        render_kernel<DEG, false, AT><<<grid, kBlock, 0, stream>>>(p);
    return cudaGetLastError();
}

template <typename AT>
cudaError_t launch_render_t(uint32_t sh_degree, const RenderParams &p, cudaStream_t stream) {
    switch (sh_degree) {
    case 0: return launch_render_deg<0, AT>(p, stream);
    case 1: return launch_render_deg<1, AT>(p, stream);
    case 2: return launch_render_deg<2, AT>(p, stream);
    case 3: return launch_render_deg<3, AT>(p, stream);
    default: return cudaErrorInvalidValue;
    }
}

template <int DEG, typename AT>
cudaError_t launch_backward_deg(const BackwardParams &p, cudaStream_t stream) {
    const uint32_t blocks = (p.num_rays + kBlock - 1) / kBlock;
    if (p.settings.alpha_mode == SDFOAM_ALPHA_NEUS)
        backward_kernel<DEG, true, AT><<<blocks, kBlock, 0, stream>>>(p);
    else
        backward_kernel<DEG, false, AT><<<blocks, kBlock, 0, stream>>>(p);
    return cudaGetLastError();
}

template <typename AT>
cudaError_t launch_forward_t(uint32_t sh_degree, const ForwardParams &p, cudaStream_t stream) {
    switch (sh_degree) {
    case 0: return launch_forward_deg<0, AT>(p, stream);
    case 1: return launch_forward_deg<1, AT>(p, stream);
    case 2: return launch_forward_deg<2, AT>(p, stream);
    case 3: return launch_forward_deg<3, AT>(p, stream);
    default: return cudaErrorInvalidValue;
    }
}

template <typename AT>
cudaError_t launch_backward_t(uint32_t sh_degree, const BackwardParams &p, cudaStream_t stream) {
    switch (sh_degree) {
    case 0: return launch_backward_deg<0, AT>(p, stream);
    case 1: return launch_backward_deg<1, AT>(p, stream);
    case 2: return launch_backward_deg<2, AT>(p, stream);
    case 3: return launch_backward_deg<3, AT>(p, stream);
    default: return cudaErrorInvalidValue;
    }
}

template <typename AT>
cudaError_t launch_fold_t(uint32_t sh_degree, uint32_t num_points, const float4 *attr_acc, const float4 *point_acc,
                          void *attr_grad, float *points_grad, cudaStream_t stream) {
    const int A = attr_dim_of(sh_degree);
    const uint64_t total = uint64_t(num_points) * (A > 3 ? A : 3);
    const uint32_t blocks = static_cast<uint32_t>((total + 255) / 256);
    AT *out = static_cast<AT *>(attr_grad);
    switch (attr_vec4_of(sh_degree)) {
    case 1: fold_grads_kernel<1, AT><<<blocks, 256, 0, stream>>>(num_points, A, attr_acc, point_acc, out, points_grad); break;
    case 4: fold_grads_kernel<4, AT><<<blocks, 256, 0, stream>>>(num_points, A, attr_acc, point_acc, out, points_grad); break;
    case 7: fold_grads_kernel<7, AT><<<blocks, 256, 0, stream>>>(num_points, A, attr_acc, point_acc, out, points_grad); break;
    case 13: fold_grads_kernel<13, AT><<<blocks, 256, 0, stream>>>(num_points, A, attr_acc, point_acc, out, points_grad); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_forward(uint32_t sh_degree, uint32_t attr_dtype, const ForwardParams &p, cudaStream_t stream) {
    if (p.num_rays == 0) return cudaSuccess;
    return attr_dtype == SDFOAM_F16 ? launch_forward_t<__half>(sh_degree, p, stream)
                                    : launch_forward_t<float>(sh_degree, p, stream);
}

cudaError_t launch_render(uint32_t sh_degree, uint32_t attr_dtype, const RenderParams &p, cudaStream_t stream) {
    if (p.width == 0 || p.height == 0) return cudaSuccess;
    return attr_dtype == SDFOAM_F16 ? launch_render_t<__half>(sh_degree, p, stream)
                                    : launch_render_t<float>(sh_degree, p, stream);
}

cudaError_t launch_backward(uint32_t sh_degree, uint32_t attr_dtype, const BackwardParams &p, cudaStream_t stream) {
    if (p.num_rays == 0) return cudaSuccess;
    return attr_dtype == SDFOAM_F16 ? launch_backward_t<__half>(sh_degree, p, stream)
                                    : launch_backward_t<float>(sh_degree, p, stream);
}

cudaError_t launch_fold_grads(uint32_t sh_degree, uint32_t attr_dtype, uint32_t num_points, const float4 *attr_acc,
                              const float4 *point_acc, void *attr_grad, float *points_grad, cudaStream_t stream) {
    if (num_points == 0) return cudaSuccess;
    return attr_dtype == SDFOAM_F16
               ? launch_fold_t<__half>(sh_degree, num_points, attr_acc, point_acc, attr_grad, points_grad, stream)
               : launch_fold_t<float>(sh_degree, num_points, attr_acc, point_acc, attr_grad, points_grad, stream);
}

}  // namespace sdfoam_b200
