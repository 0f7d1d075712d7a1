/*
 * sdfoam_oracle.c -- CPU restatement of the SDFoam Voronoi-foam tracer.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * kernels in sdfoam_b200/csrc.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it.  The product
 * path never calls it and has no CPU fallback.
 *
 * PARITY STATUS: unpinned against the reference binary.  The reference
 * (mmlab-cv/SDFoam) cannot be compiled here (its Eigen submodule is empty and
 * Eigen is not installed), it is GPU-only code, and it ships no tests, golden
 * vectors or fixtures.  This oracle restates the reference algorithm from its
 * source, and is checked by finite-difference self-consistency tests
 * (tests/test_oracle.py).
 *
 * What it follows (paths inside the reference project):
 *   walk           src/tracing/tracing_utils.cuh:17-109 (trace), :112-124
 *                  (cell_intersection_grad)
 *   forward        src/tracing/pipeline.cu:36-264
 *   backward NeuS  src/tracing/pipeline.cu:267-550 (backward_sdf)
 *   backward std   src/tracing/pipeline.cu:553-791 (RadFoam backward)
 *   SH             src/tracing/sh_utils.cuh:8-92
 *   diff quantise  src/tracing/pipeline.cu:1202-1224 (half4(q - p, 0), RNE)
 *   settings       src/tracing/pipeline.h:12-40
 *   render         src/tracing/pipeline.cu:1067-1199 (benchmark kernel),
 *                  camera.h:56-85 (cast_ray), tracing_utils.cuh:126-136
 *                  (make_rgba8)
 *
 * Floating-point contract shared with the CUDA kernels (both sides implement
 * it independently; the GPU files are compiled with -fmad=false, this file
 * with -ffp-contract=off, so only the fmaf() calls written out below fuse):
 *   dot3(a,b)       = fmaf(a0,b0, fmaf(a1,b1, a2*b2))   (Eigen's halving
 *                     reduction a0b0 + (a1b1 + a2b2), with the first product
 *                     of each add fused, as nvcc -fmad contracts it)
 *   face test       off = half->float(diff); fo = p + off*0.5; dp = dot3(off,dir)
 *                   t = dot3(fo - o, off) / dp            (IEEE division)
 *   exp             foam_expf(): Cody-Waite reduction + degree-7 Taylor
 *                   polynomial (own implementation).  The reference uses the
 *                   hardware approximation __expf, which no CPU reproduces;
 *                   both sides of this build use foam_expf so that walk lengths
 *                   (hit counts) agree bit for bit.
 *   SH colour       rgb_c = 0.5; rgb_c = fmaf(Y_k, coef[3k+c], rgb_c), k = 0..K-1
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define U32_NONE 0xffffffffu

/* ------------------------------------------------------------------ */
/* scalar helpers                                                      */
/* ------------------------------------------------------------------ */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* IEEE binary32 -> binary16, round to nearest even (the conversion Eigen::half
 * and __float2half_rn perform; pipeline.cu:1222). */
uint16_t oracle_f2h(float f)
{
    uint32_t x = f2u(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t e8 = (x >> 23) & 0xffu;
    uint32_t mant = x & 0x7fffffu;
    if (e8 == 0xffu) /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (mant ? (0x200u | (mant >> 13)) : 0u));
    int e = (int)e8 - 127 + 15;
    if (e >= 31)
        return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) { /* half subnormal (or zero) */
        if (e8 == 0)
            return (uint16_t)sign; /* float zero / subnormal -> 0 */
        uint32_t m = mant | 0x800000u;
        int shift = 14 - e;
        if (shift > 24)
            return (uint16_t)sign;
        uint32_t hm = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (hm & 1u)))
            hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t r = sign | ((uint32_t)e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u)))
        r++;
    return (uint16_t)r;
}

float oracle_h2f(uint16_t h)
{
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e5 = ((uint32_t)h >> 10) & 0x1fu;
    uint32_t m = (uint32_t)h & 0x3ffu;
    if (e5 == 0) {
        float v = (float)m * 5.9604644775390625e-08f; /* m * 2^-24, exact */
        return sign ? -v : v;
    }
    if (e5 == 31)
        return u2f(sign | 0x7f800000u | (m << 13));
    return u2f(sign | ((e5 - 15 + 127) << 23) | (m << 13));
}

/* exp(x) in binary32.  Cody & Waite (1980) argument reduction x = n*ln2 + r,
 * |r| <= ln2/2, with ln2 split into a float head and tail; e^r from its
 * degree-7 Taylor polynomial (truncation error < 6e-9 relative on that
 * interval); the result is scaled by 2^n in two exact power-of-two steps so
 * that overflow gives inf and underflow rounds through subnormals.
 * Measured error against a double-precision exp: see tests/test_oracle.py. */
float oracle_expf(float x)
{
    if (x != x)
        return x;
    if (x > 88.8f)
        return u2f(0x7f800000u);
    if (x < -104.0f)
        return 0.0f;
    const float log2e = 1.44269502162933349609375f;   /* float(1/ln 2) */
    const float ln2_hi = 0.693147182464599609375f;    /* float(ln 2) */
    const float ln2_lo = -1.904654323148236e-09f;     /* float(ln 2 - ln2_hi) */
    float n = rintf(x * log2e);
    float r = fmaf(n, -ln2_hi, x);
    r = fmaf(n, -ln2_lo, r);
    float p = 1.98412698412698413e-04f;                /* 1/5040 */
    p = fmaf(p, r, 1.38888888888888889e-03f);          /* 1/720 */
    p = fmaf(p, r, 8.33333333333333333e-03f);          /* 1/120 */
    p = fmaf(p, r, 4.16666666666666667e-02f);          /* 1/24 */
    p = fmaf(p, r, 1.66666666666666667e-01f);          /* 1/6 */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;
    int n1 = ni / 2;
    int n2 = ni - n1;
    float s1 = u2f((uint32_t)(n1 + 127) << 23);
    float s2 = u2f((uint32_t)(n2 + 127) << 23);
    return (p * s1) * s2;
}

static inline float dot3(const float *a, const float *b)
{
    return fmaf(a[0], b[0], fmaf(a[1], b[1], a[2] * b[2]));
}

/* ------------------------------------------------------------------ */
/* spherical harmonics (sh_utils.cuh:8-83)                             */
/* ------------------------------------------------------------------ */

static const float SH_C0 = 0.28209479177387814f;
static const float SH_C1 = 0.4886025119029199f;
static const float SH_C2[5] = {1.0925484305920792f, -1.0925484305920792f,
                               0.31539156525252005f, -1.0925484305920792f,
                               0.5462742152960396f};
static const float SH_C3[7] = {-0.5900435899266435f, 2.890611442640554f,
                               -0.4570457994644658f, 0.3731763325901154f,
                               -0.4570457994644658f, 1.445305721320277f,
                               -0.5900435899266435f};

/* sh_coefficients<degree> (sh_utils.cuh:34-70); unused entries are zero. */
static void sh_basis(int degree, const float *dir, float *Y)
{
    float x = dir[0], y = dir[1], z = dir[2];
    for (int k = 0; k < 16; ++k)
        Y[k] = 0.0f;
    Y[0] = SH_C0;
    if (degree > 0) {
        Y[1] = (-SH_C1) * y;
        Y[2] = SH_C1 * z;
        Y[3] = (-SH_C1) * x;
    }
    float xx = x * x, yy = y * y, zz = z * z;
    float xy = x * y, yz = y * z, xz = x * z;
    if (degree > 1) {
        Y[4] = SH_C2[0] * xy;
        Y[5] = SH_C2[1] * yz;
        Y[6] = SH_C2[2] * ((2.0f * zz - xx) - yy);
        Y[7] = SH_C2[3] * xz;
        Y[8] = SH_C2[4] * (xx - yy);
    }
    if (degree > 2) {
        Y[9] = (SH_C3[0] * y) * fmaf(3.0f, xx, -yy);
        Y[10] = (SH_C3[1] * xy) * z;
        Y[11] = (SH_C3[2] * y) * ((4.0f * zz - xx) - yy);
        Y[12] = (SH_C3[3] * z) * fmaf(-3.0f, yy, fmaf(-3.0f, xx, 2.0f * zz));
        Y[13] = (SH_C3[4] * x) * ((4.0f * zz - xx) - yy);
        Y[14] = (SH_C3[5] * z) * (xx - yy);
        Y[15] = (SH_C3[6] * x) * fmaf(-3.0f, yy, xx);
    }
}

/* load_sh_as_rgb (sh_utils.cuh:72-83) */
static void sh_rgb(int nbasis, const float *Y, const float *coef, float *rgb)
{
    float r = 0.5f, g = 0.5f, b = 0.5f;
    for (int k = 0; k < nbasis; ++k) {
        r = fmaf(Y[k], coef[3 * k + 0], r);
        g = fmaf(Y[k], coef[3 * k + 1], g);
        b = fmaf(Y[k], coef[3 * k + 2], b);
    }
    rgb[0] = fmaxf(r, 0.0f);
    rgb[1] = fmaxf(g, 0.0f);
    rgb[2] = fmaxf(b, 0.0f);
}

/* ------------------------------------------------------------------ */
/* scene and settings                                                  */
/* ------------------------------------------------------------------ */

typedef struct {
    uint32_t num_points;
    uint32_t adjacency_size;
    uint32_t attr_dim;          /* 1 + 3*(deg+1)^2 */
    int sh_degree;
    const float *points;        /* [N,3] */
    const float *attributes;    /* [N,attr_dim] */
    const uint32_t *adjacency;  /* [E] */
    const uint32_t *offsets;    /* [N+1] */
    const uint16_t *diffs;      /* [E,4] binary16, from oracle_build_diffs */
} oracle_scene;

typedef struct {
    float weight_threshold;     /* pipeline.h:31 default 1e-7 */
    uint32_t max_intersections; /* pipeline.h:32 default 1024 */
    int neus;                   /* alpha_mode == AlphaNeuS */
    int sdf_channel;            /* < 0: none */
    float sharpness;            /* element 0 of the sharpness buffer */
} oracle_settings;

/* prefetch_adjacent_diff_kernel (pipeline.cu:1202-1224): per CSR entry j of
 * site i, half4(points[adj[j]] - points[i], 0).  Rows whose offsets are not
 * ordered are skipped, as are neighbour ids outside [0, N). */
void oracle_build_diffs(uint32_t num_points, const float *points,
                        const uint32_t *adjacency, const uint32_t *offsets,
                        uint32_t adjacency_size, uint16_t *diffs)
{
    memset(diffs, 0, sizeof(uint16_t) * 4 * (size_t)adjacency_size);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)num_points; ++i) {
        uint32_t beg = offsets[i], end = offsets[i + 1];
        if (beg > end || end > adjacency_size)
            continue;
        const float *p = points + 3 * i;
        for (uint32_t j = beg; j < end; ++j) {
            uint32_t a = adjacency[j];
            if (a >= num_points)
                continue;
            const float *q = points + 3 * (size_t)a;
            diffs[4 * (size_t)j + 0] = oracle_f2h(q[0] - p[0]);
            diffs[4 * (size_t)j + 1] = oracle_f2h(q[1] - p[1]);
            diffs[4 * (size_t)j + 2] = oracle_f2h(q[2] - p[2]);
            diffs[4 * (size_t)j + 3] = 0;
        }
    }
}

typedef struct {
    float o[3];
    float d[3];  /* unit direction */
} oracle_ray;

static void load_ray(const float *rays, size_t r, oracle_ray *ray)
{
    const float *src = rays + 6 * r;
    float d[3] = {src[3], src[4], src[5]};
    float len = sqrtf(fmaf(d[0], d[0], fmaf(d[1], d[1], d[2] * d[2])));
    for (int k = 0; k < 3; ++k) {
        ray->o[k] = src[k];
        ray->d[k] = d[k] / len;
    }
}

/* One exit-face search of trace() (tracing_utils.cuh:43-91).  safe != 0 is
 * the forward / NeuS-backward mode (dp > 0 && t > t0 && t < t1); safe == 0 is
 * the RadFoam backward mode (dp > 0 && t < t1).  Strict '<' keeps the first
 * minimum in CSR order.  Returns the face index or U32_NONE, t1 in *t1_out. */
static uint32_t find_exit(const oracle_scene *sc, const oracle_ray *ray,
                          const float *p, uint32_t beg, uint32_t end, float t0,
                          int safe, float *t1_out)
{
    float t1 = u2f(0x7f800000u);
    uint32_t best = U32_NONE;
    for (uint32_t j = beg; j < end; ++j) {
        const uint16_t *h = sc->diffs + 4 * (size_t)j;
        float off[3] = {oracle_h2f(h[0]), oracle_h2f(h[1]), oracle_h2f(h[2])};
        float w[3];
        for (int k = 0; k < 3; ++k)
            w[k] = (p[k] + off[k] * 0.5f) - ray->o[k];
        float dp = dot3(off, ray->d);
        float t = dot3(w, off) / dp;
        if (safe) {
            if (dp > 0.0f && t > t0 && t < t1) {
                t1 = t;
                best = j - beg;
            }
        } else {
            if (dp > 0.0f && t < t1) {
                t1 = t;
                best = j - beg;
            }
        }
    }
    *t1_out = t1;
    return best;
}

/* NeuS density of a site: s = sha * phi * (1 - phi), phi = sigmoid(-sha * d)
 * (pipeline.cu:149, 386-387).  sigmoidf(x) = 1/(1 + exp(-x)), and
 * -(-sha * d) == sha * d exactly. */
static inline float neus_phi(float sha, float d)
{
    return 1.0f / (1.0f + oracle_expf(sha * d));
}

/* ------------------------------------------------------------------ */
/* forward (pipeline.cu:36-264)                                        */
/* ------------------------------------------------------------------ */

typedef struct {
    uint32_t num_rays;
    const float *rays;          /* [R,6] */
    const uint32_t *start;      /* [R] */
    uint32_t num_quantiles;
    const float *quantiles;     /* [R,Q] or NULL */
    float *rgba;                /* [R,4] */
    float *depth;               /* [R,Q] or NULL */
    uint32_t *depth_indices;    /* [R,Q] or NULL */
    uint32_t *num_intersections;/* [R] or NULL */
    float *contribution;        /* [N] or NULL (accumulated, caller zeroes) */
    float *alpha_out;           /* [N] or NULL (racy last-writer store) */
    /* optional debug dump: per ray, the cells handed to the cell functor, in
     * order, with the alpha computed there.  seq_offsets has R+1 entries. */
    const uint64_t *seq_offsets;
    uint32_t *seq_cells;
    float *seq_alpha;
    uint32_t *seq_count;        /* [R] functor calls actually made */
    /* optional [R]: 1 where the ray's termination (T > weight_threshold) or
     * a quantile crossing (Tn < q) could fall on another step under the
     * reference's exp (see exp_interval below), else 0 */
    uint8_t *ambiguous;
} oracle_fwd_io;

/* The reference evaluates every exp of the forward functor with the hardware
 * approximation __expf (pipeline.cu:57, 151, 155), whose documented maximum
 * error is 2 + floor(|1.173 x|) ulp (CUDA C++ Programming Guide, table of
 * single-precision intrinsic functions); oracle_expf is within 2 ulp of exp
 * (tests/test_oracle.py).  exp_interval() widens this oracle's exp(x) = e to
 * an interval that contains the reference's __expf(x): 4 + floor(|1.173 x|)
 * ulp of e on either side, plus one ulp for the roundings that follow.  The
 * interval walk below carries T through these intervals; a ray whose
 * T > weight_threshold (or Tn < q) test has different outcomes at the two
 * ends of the interval is "threshold-ambiguous": its hit count could differ
 * from the reference's even though every face decision is the same. */
static void exp_interval(float x, float e, float *lo, float *hi)
{
    float ulps = 5.0f + floorf(fabsf(1.173f * x));
    float up = nextafterf(e, INFINITY) - e;
    if (!(up > 0.0f) || up != up)
        up = 1.401298464e-45f;
    float w = ulps * up;
    *lo = fmaxf(e - w, 0.0f);
    *hi = e + w;
}

/* s = (sha * phi) * (1 - phi) over phi in [plo, phi_hi]: s is largest at
 * phi = 1/2 and monotone on either side of it. */
static void neus_s_interval(float sha, float plo, float phi_hi, float *slo, float *shi)
{
    float a = (sha * plo) * (1.0f - plo);
    float b = (sha * phi_hi) * (1.0f - phi_hi);
    *slo = fminf(a, b);
    *shi = fmaxf(a, b);
    if (plo <= 0.5f && 0.5f <= phi_hi)
        *shi = fmaxf(*shi, (sha * 0.5f) * 0.5f);
}

static void forward_ray(const oracle_scene *sc, const oracle_settings *st,
                        const oracle_fwd_io *io, size_t r)
{
    const int nb = (sc->sh_degree + 1) * (sc->sh_degree + 1);
    const uint32_t D = sc->attr_dim;
    const int neus_alpha = st->neus && st->sdf_channel >= 0;
    oracle_ray ray;
    load_ray(io->rays, r, &ray);
    float Y[16];
    sh_basis(sc->sh_degree, ray.d, Y);

    const uint32_t Q = io->quantiles ? io->num_quantiles : 0;
    const float *rq = io->quantiles ? io->quantiles + (size_t)r * io->num_quantiles : NULL;
    uint32_t qi = 0;
    float q = 0.0f;
    if (rq && io->num_quantiles > 0)
        q = rq[0];

    float T = 1.0f;
    float Tlo = 1.0f, Thi = 1.0f;   /* interval walk (io->ambiguous) */
    uint8_t amb = 0;
    float acc[3] = {0.0f, 0.0f, 0.0f};
    uint64_t seq_pos = io->seq_offsets ? io->seq_offsets[r] : 0;
    uint64_t seq_end = io->seq_offsets ? io->seq_offsets[r + 1] : 0;
    uint32_t nseq = 0;

    /* trace() (tracing_utils.cuh:17-109) */
    float t0 = 0.0f;
    uint32_t n = 0;
    uint32_t cur = io->start[r];
    if (cur < sc->num_points) {
        float p[3] = {sc->points[3 * (size_t)cur], sc->points[3 * (size_t)cur + 1],
                      sc->points[3 * (size_t)cur + 2]};
        for (;;) {
            ++n;
            if (n > st->max_intersections)
                break;
            uint32_t beg = sc->offsets[cur], end = sc->offsets[cur + 1];
            if (beg > end || end > sc->adjacency_size)
                break;
            float t1;
            uint32_t f = find_exit(sc, &ray, p, beg, end, t0, 1, &t1);
            if (f == U32_NONE)
                break;
            uint32_t nxt = sc->adjacency[beg + f];
            if (nxt >= sc->num_points)
                break;
            const float *qp = sc->points + 3 * (size_t)nxt;
            if (t1 > t0) {
                /* cell functor (pipeline.cu:117-235) */
                const float *attr = sc->attributes + (size_t)cur * D;
                float last = attr[D - 1];
                float rgb[3];
                if (st->neus || last > 1e-6f)
                    sh_rgb(nb, Y, attr, rgb);
                else
                    rgb[0] = rgb[1] = rgb[2] = 0.0f;
                float s, alpha;
                float dt = fmaxf(t1 - t0, 0.0f);
                if (neus_alpha) {
                    float d = attr[st->sdf_channel];
                    float phi = neus_phi(st->sharpness, d);
                    s = (st->sharpness * phi) * (1.0f - phi);
                } else {
                    s = last;
                }
                alpha = 1.0f - oracle_expf(-(s * dt));
                float Tnlo = 0.0f, Tnhi = 0.0f;
                if (io->ambiguous) {
                    float slo = s, shi = s;
                    if (neus_alpha) {
                        float x = st->sharpness * attr[st->sdf_channel];
                        float elo, ehi;
                        exp_interval(x, oracle_expf(x), &elo, &ehi);
                        neus_s_interval(st->sharpness, 1.0f / (1.0f + ehi), 1.0f / (1.0f + elo), &slo, &shi);
                    }
                    float xa = -(shi * dt), xb = -(slo * dt), Elo, Ehi, dummy;
                    exp_interval(xa, oracle_expf(xa), &Elo, &dummy);
                    exp_interval(xb, oracle_expf(xb), &dummy, &Ehi);
                    Tnlo = Tlo * (1.0f - (1.0f - Elo));
                    Tnhi = Thi * (1.0f - (1.0f - fminf(Ehi, 1.0f)));
                }
                float weight = T * alpha;
                if (io->alpha_out)
                    io->alpha_out[cur] = alpha;
                if (io->contribution) {
#pragma omp atomic
                    io->contribution[cur] += weight;
                }
                for (int c = 0; c < 3; ++c)
                    acc[c] = fmaf(weight, rgb[c], acc[c]);
                float Tn = T * (1.0f - alpha);
                if (st->neus) {
                    float drop = T - Tn;
                    if (drop > 1e-12f) {
                        while (qi < Q && Tn < q) {
                            float frac = (T - q) / drop;
                            frac = fminf(1.0f, fmaxf(0.0f, frac));
                            float tq = fmaf(frac, t1 - t0, t0);
                            io->depth[(size_t)r * Q + qi] = tq;
                            io->depth_indices[(size_t)r * Q + qi] = cur;
                            ++qi;
                            if (qi < Q)
                                q = rq[qi];
                        }
                    }
                } else {
                    while (qi < Q && Tn < q) {
                        io->depth[(size_t)r * Q + qi] = t0 + logf(T / q) / s;
                        io->depth_indices[(size_t)r * Q + qi] = cur;
                        ++qi;
                        if (qi < Q)
                            q = rq[qi];
                    }
                }
                if (io->seq_cells && seq_pos < seq_end) {
                    io->seq_cells[seq_pos] = cur;
                    if (io->seq_alpha)
                        io->seq_alpha[seq_pos] = alpha;
                    ++seq_pos;
                }
                ++nseq;
                if (io->ambiguous) {
                    if ((Tnlo > st->weight_threshold) != (Tnhi > st->weight_threshold))
                        amb = 1;
                    for (uint32_t k = 0; k < Q; ++k)
                        if ((Tnlo < rq[k]) != (Tnhi < rq[k]))
                            amb = 1;
                    Tlo = Tnlo;
                    Thi = Tnhi;
                }
                T = Tn;
                if (!(T > st->weight_threshold))
                    break;
            }
            t0 = fmaxf(t0, t1);
            cur = nxt;
            p[0] = qp[0];
            p[1] = qp[1];
            p[2] = qp[2];
        }
    }
    /* epilogue (pipeline.cu:251-263) */
    while (qi < Q) {
        io->depth[(size_t)r * Q + qi] = -1.0f;
        io->depth_indices[(size_t)r * Q + qi] = U32_NONE;
        ++qi;
    }
    io->rgba[4 * r + 0] = acc[0];
    io->rgba[4 * r + 1] = acc[1];
    io->rgba[4 * r + 2] = acc[2];
    io->rgba[4 * r + 3] = 1.0f - T;
    if (io->num_intersections)
        io->num_intersections[r] = n;
    if (io->seq_count)
        io->seq_count[r] = nseq;
    if (io->ambiguous)
        io->ambiguous[r] = amb;
}

void oracle_trace_forward(const oracle_scene *sc, const oracle_settings *st,
                          const oracle_fwd_io *io, int threads)
{
#ifdef _OPENMP
    if (threads > 0)
        omp_set_num_threads(threads);
#else
    (void)threads;
#endif
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t r = 0; r < (int64_t)io->num_rays; ++r)
        forward_ray(sc, st, io, (size_t)r);
}

/* ------------------------------------------------------------------ */
/* headless render (trace_benchmark, pipeline.cu:1067-1199)            */
/* ------------------------------------------------------------------ */

typedef struct {
    float position[3], forward[3], right[3], up[3];
    float fov;
    uint32_t width, height;
    uint32_t model;   /* 0 pinhole, 1 fisheye */
    float bg[3];
    int checker;
} oracle_camera;

/* make_rgba8 (tracing_utils.cuh:126-136): std::min(1, x) then std::max(0, .)
 * (a NaN becomes 1), truncation of x * 255. */
static uint32_t rgba8_channel(float x)
{
    x = x < 1.0f ? x : 1.0f;
    x = 0.0f < x ? x : 0.0f;
    return (uint32_t)(int)(x * 255.0f);
}

/* cast_ray (camera.h:56-85) and the render kernel's check + second
 * normalisation (pipeline.cu:1101-1113); vector sums contracted as
 * x*a + y*b -> fmaf(x, a, y*b), then + z*c -> fmaf(z, c, .).  Returns 0 for
 * fisheye pixels outside the lens. */
static int camera_ray(const oracle_camera *cam, float focal, float aspect, uint32_t i, uint32_t j,
                      oracle_ray *ray)
{
    const float x = (float)i / (float)cam->width;
    const float y = (float)j / (float)cam->height;
    const float u = (2.0f * x - 1.0f) * aspect;
    const float v = 1.0f - 2.0f * y;
    float d[3];
    float mask = 1.0f;
    if (cam->model == 0) {
        for (int k = 0; k < 3; ++k)
            d[k] = fmaf(v, cam->up[k], fmaf(focal, cam->forward[k], u * cam->right[k]));
    } else {
        const float kpi = 3.14159265358979f;
        const float theta = atan2f(v, u);
        float phi = cam->fov * sqrtf(fmaf(u, u, v * v));
        if (phi >= kpi) {
            phi = kpi - 1e-6f;
            mask = 0.0f;
        }
        const float sp = sinf(phi);
        const float a = sp * cosf(theta), b = sp * sinf(theta), c = cosf(phi);
        for (int k = 0; k < 3; ++k)
            d[k] = fmaf(c, cam->forward[k], fmaf(a, cam->right[k], b * cam->up[k]));
    }
    const float n2 = dot3(d, d);
    if (n2 > 0.0f) {
        const float len = sqrtf(n2);
        for (int k = 0; k < 3; ++k)
            d[k] = d[k] / len;
    }
    for (int k = 0; k < 3; ++k)
        d[k] = d[k] * mask;
    const float norm = sqrtf(dot3(d, d));
    if (norm < 0.1f)
        return 0;
    for (int k = 0; k < 3; ++k) {
        ray->o[k] = cam->position[k];
        ray->d[k] = d[k] / norm;
    }
    return 1;
}

static uint32_t render_pixel(const oracle_scene *sc, const oracle_settings *st, const oracle_camera *cam,
                             float focal, float aspect, uint32_t start, uint32_t i, uint32_t j)
{
    float bg[3] = {cam->bg[0], cam->bg[1], cam->bg[2]};
    oracle_ray ray;
    if (!camera_ray(cam, focal, aspect, i, j, &ray))
        return (rgba8_channel(1.0f) << 24) | (rgba8_channel(bg[2]) << 16) | (rgba8_channel(bg[1]) << 8) |
               rgba8_channel(bg[0]);
    const int nb = (sc->sh_degree + 1) * (sc->sh_degree + 1);
    const uint32_t D = sc->attr_dim;
    const int neus_alpha = st->neus && st->sdf_channel >= 0;
    float Y[16];
    sh_basis(sc->sh_degree, ray.d, Y);
    float T = 1.0f;
    float acc[3] = {0.0f, 0.0f, 0.0f};
    float t0 = 0.0f;
    uint32_t n = 0;
    uint32_t cur = start;
    if (cur < sc->num_points) {
        float p[3] = {sc->points[3 * (size_t)cur], sc->points[3 * (size_t)cur + 1],
                      sc->points[3 * (size_t)cur + 2]};
        for (;;) {
            ++n;
            if (n > st->max_intersections)
                break;
            uint32_t beg = sc->offsets[cur], end = sc->offsets[cur + 1];
            if (beg > end || end > sc->adjacency_size)
                break;
            float t1;
            uint32_t f = find_exit(sc, &ray, p, beg, end, t0, 1, &t1);
            if (f == U32_NONE)
                break;
            uint32_t nxt = sc->adjacency[beg + f];
            if (nxt >= sc->num_points)
                break;
            if (t1 > t0) {
                const float *attr = sc->attributes + (size_t)cur * D;
                float last = attr[D - 1];
                float rgb[3];
                if (st->neus || last > 1e-6f)
                    sh_rgb(nb, Y, attr, rgb);
                else
                    rgb[0] = rgb[1] = rgb[2] = 0.0f;
                float s;
                float dt = fmaxf(t1 - t0, 0.0f);
                if (neus_alpha) {
                    float phi = neus_phi(st->sharpness, attr[st->sdf_channel]);
                    s = (st->sharpness * phi) * (1.0f - phi);
                } else {
                    s = last;
                }
                float alpha = 1.0f - oracle_expf(-(s * dt));
                float w = T * alpha;
                for (int c = 0; c < 3; ++c)
                    acc[c] = fmaf(w, rgb[c], acc[c]);
                T = T * (1.0f - alpha);
                if (!(T > st->weight_threshold))
                    break;
            }
            t0 = fmaxf(t0, t1);
            cur = nxt;
            const float *qp = sc->points + 3 * (size_t)nxt;
            p[0] = qp[0];
            p[1] = qp[1];
            p[2] = qp[2];
        }
    }
    if (cam->checker) {
        int is = 2 * (int)((i / 20) % 2) - 1;
        int js = 2 * (int)((j / 20) % 2) - 1;
        bg[0] = bg[1] = bg[2] = is * js > 0 ? 0.3f : 0.5f;
    }
    return (rgba8_channel(1.0f) << 24) | (rgba8_channel(fmaf(T, bg[2], acc[2])) << 16) |
           (rgba8_channel(fmaf(T, bg[1], acc[1])) << 8) | rgba8_channel(fmaf(T, bg[0], acc[0]));
}

/* out[(height - 1 - j) * width + i] = RGBA8 of pixel (i, j). */
void oracle_render(const oracle_scene *sc, const oracle_settings *st, const oracle_camera *cam,
                   uint32_t start, uint32_t *out, int threads)
{
#ifdef _OPENMP
    if (threads > 0)
        omp_set_num_threads(threads);
#else
    (void)threads;
#endif
    const float focal = 1.0f / tanf(cam->fov * 0.5f);
    const float aspect = (float)cam->width / (float)cam->height;
    const int64_t total = (int64_t)cam->width * cam->height;
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t t = 0; t < total; ++t) {
        uint32_t i = (uint32_t)(t % cam->width), j = (uint32_t)(t / cam->width);
        out[(size_t)(cam->height - 1 - j) * cam->width + i] = render_pixel(sc, st, cam, focal, aspect, start, i, j);
    }
}

/* ------------------------------------------------------------------ */
/* backward                                                            */
/* ------------------------------------------------------------------ */

typedef struct {
    uint32_t num_rays;
    const float *rays;
    const uint32_t *start;
    uint32_t num_quantiles;
    const float *quantiles;       /* [R,Q] or NULL */
    const uint32_t *depth_indices;/* [R,Q] or NULL (used by the RadFoam mode) */
    const float *rgba;            /* forward output [R,4] */
    const float *rgba_grad;       /* [R,4] */
    const float *depth_grad;      /* [R,Q] or NULL */
    const float *ray_error;       /* [R] or NULL */
    float *points_grad;           /* [N,3] accumulated */
    float *attr_grad;             /* [N,attr_dim] accumulated */
    float *point_error;           /* [N] or NULL */
    float *sharpness_grad;        /* [1] or NULL */
    /* optional: sum of |term| per accumulated entry, for error bounds */
    float *points_grad_abs;
    float *attr_grad_abs;
} oracle_bwd_io;

/* cell_intersection_grad (tracing_utils.cuh:112-124): d t / d primal for the
 * bisector plane between p (primal) and q (opposite). */
static void cig(const float *p, const float *q, const oracle_ray *ray, float *g)
{
    float w[3], nrm[3];
    for (int k = 0; k < 3; ++k) {
        w[k] = ((p[k] + q[k]) * 0.5f) - ray->o[k];
        nrm[k] = q[k] - p[k];
    }
    float num = dot3(w, nrm);
    float dp = dot3(nrm, ray->d);
    float dp2 = dp * dp;
    for (int k = 0; k < 3; ++k)
        g[k] = fmaf(num, ray->d[k], dp * (ray->o[k] - p[k])) / dp2;
}

static inline void acc_add(float *dst, float *dst_abs, size_t i, float v)
{
#pragma omp atomic
    dst[i] += v;
    if (dst_abs) {
        float a = fabsf(v);
#pragma omp atomic
        dst_abs[i] += a;
    }
}

/* backward_sdf (pipeline.cu:267-550) */
static void backward_neus_ray(const oracle_scene *sc, const oracle_settings *st,
                              const oracle_bwd_io *io, size_t r, double *sha_acc)
{
    const int nb = (sc->sh_degree + 1) * (sc->sh_degree + 1);
    const uint32_t D = sc->attr_dim;
    const int sdf_ch = st->sdf_channel >= 0 ? st->sdf_channel : (int)D - 1;
    const float sha = st->sharpness;
    oracle_ray ray;
    load_ray(io->rays, r, &ray);
    float Y[16];
    sh_basis(sc->sh_degree, ray.d, Y);
    float g[4], C[4];
    for (int k = 0; k < 4; ++k) {
        g[k] = io->rgba_grad[4 * r + k];
        C[k] = io->rgba[4 * r + k];
    }
    const uint32_t Q = io->quantiles ? io->num_quantiles : 0;
    const float *rq = io->quantiles ? io->quantiles + r * io->num_quantiles : NULL;
    const float *rdg = io->depth_grad ? io->depth_grad + r * io->num_quantiles : NULL;
    float err = io->ray_error ? io->ray_error[r] : 0.0f;
    uint32_t qi = 0;
    float q = 0.0f;
    if (rq && io->num_quantiles > 0)
        q = rq[0];
    float g_logT = 0.0f;
    float T = 1.0f;
    float acc[3] = {0.0f, 0.0f, 0.0f};
    uint32_t prev_idx = U32_NONE;
    float prev_pt[3] = {0.0f, 0.0f, 0.0f};
    float prev_grad[3] = {0.0f, 0.0f, 0.0f};
    float cur_grad[3] = {0.0f, 0.0f, 0.0f};
    float next_grad[3] = {0.0f, 0.0f, 0.0f};
    double sha_sum = 0.0;

    float t0 = 0.0f;
    uint32_t n = 0;
    uint32_t cur = io->start[r];
    if (cur >= sc->num_points)
        return;
    float p[3] = {sc->points[3 * (size_t)cur], sc->points[3 * (size_t)cur + 1],
                  sc->points[3 * (size_t)cur + 2]};
    for (;;) {
        ++n;
        if (n > st->max_intersections)
            break;
        uint32_t beg = sc->offsets[cur], end = sc->offsets[cur + 1];
        if (beg > end || end > sc->adjacency_size)
            break;
        float t1;
        uint32_t f = find_exit(sc, &ray, p, beg, end, t0, 1, &t1);
        if (f == U32_NONE)
            break;
        uint32_t nxt = sc->adjacency[beg + f];
        if (nxt >= sc->num_points)
            break;
        const float *qp = sc->points + 3 * (size_t)nxt;
        if (t1 > t0) {
            const float *attr = sc->attributes + (size_t)cur * D;
            float rgb[3];
            sh_rgb(nb, Y, attr, rgb);
            float dt = fmaxf(t1 - t0, 0.0f);
            float d = attr[sdf_ch];
            float phi = neus_phi(sha, d);
            float s = (sha * phi) * (1.0f - phi);
            float alpha = 1.0f - oracle_expf(-(s * dt));
            float weight = T * alpha;
            for (int c = 0; c < 3; ++c)
                acc[c] = fmaf(weight, rgb[c], acc[c]);
            if (io->point_error) {
#pragma omp atomic
                io->point_error[cur] += weight * err;
            }
            float dL_drgb[3];
            for (int c = 0; c < 3; ++c)
                dL_drgb[c] = g[c] * weight;
            float denom = fmaf(T, 1.0f - alpha, 1e-6f);
            float u[3];
            for (int c = 0; c < 3; ++c)
                u[c] = rgb[c] - (C[c] - acc[c]) / denom;
            float dL_dalpha = T * dot3(u, g);
            dL_dalpha = dL_dalpha + ((1.0f - C[3]) * g[3]) / ((1.0f - alpha) + 1e-6f);
            dL_dalpha = dL_dalpha + (-g_logT) / fmaxf(1.0f - alpha, 1e-12f);
            float oma = 1.0f - alpha;
            float dL_ds = dL_dalpha * (dt * oma);
            float dL_ddelta = dL_dalpha * (s * oma);
            float Tn = T * (1.0f - alpha);
            float dL_dt0_units = 0.0f;
            if (rq && io->num_quantiles > 0) {
                float T0 = T;
                float drop = T0 - Tn;
                if (drop > 1e-12f) {
                    while (qi < Q && Tn < q) {
                        float gq = rdg[qi];
                        float frac = (T0 - q) / drop;
                        frac = fminf(1.0f, fmaxf(0.0f, frac));
                        dL_dt0_units = dL_dt0_units + gq;
                        dL_ddelta = fmaf(gq, frac, dL_ddelta);
                        /* the alpha term added to dL_dalpha here in the
                         * reference (pipeline.cu:462-464) is never read again:
                         * dL_ds was already formed above. */
                        if (alpha > 1e-12f && T0 > 1e-20f)
                            g_logT = fmaf(gq, (dt * q) / (alpha * T0), g_logT);
                        ++qi;
                        if (qi < Q)
                            q = rq[qi];
                    }
                }
            }
            float dL_dt0 = dL_dt0_units - dL_ddelta;
            float dL_dt1 = dL_ddelta;
            float dprev[3] = {0.0f, 0.0f, 0.0f};
            if (prev_idx != U32_NONE)
                cig(prev_pt, p, &ray, dprev);
            float d1cur[3], d0cur[3], d1next[3];
            cig(p, qp, &ray, d1cur);
            cig(p, prev_pt, &ray, d0cur);
            cig(qp, p, &ray, d1next);
            for (int k = 0; k < 3; ++k) {
                prev_grad[k] = fmaf(dL_dt0, dprev[k], prev_grad[k]);
                cur_grad[k] = cur_grad[k] + fmaf(dL_dt0, d0cur[k], dL_dt1 * d1cur[k]);
                next_grad[k] = fmaf(dL_dt1, d1next[k], next_grad[k]);
            }
            if (prev_idx != U32_NONE) {
                for (int k = 0; k < 3; ++k)
                    acc_add(io->points_grad, io->points_grad_abs,
                            3 * (size_t)prev_idx + k, prev_grad[k]);
            }
            for (int k = 0; k < 3; ++k) {
                prev_pt[k] = p[k];
                prev_grad[k] = cur_grad[k];
                cur_grad[k] = next_grad[k];
                next_grad[k] = 0.0f;
            }
            prev_idx = cur;
            float omtp = fmaf(-2.0f, phi, 1.0f);
            float dphi_dd = ((-sha) * phi) * (1.0f - phi);
            float ds_dd = (sha * omtp) * dphi_dd;
            float ds_dsha = (phi * (1.0f - phi)) * fmaf(-(sha * d), omtp, 1.0f);
            float dL_dd = dL_ds * ds_dd;
            if (st->sdf_channel >= 0)
                acc_add(io->attr_grad, io->attr_grad_abs,
                        (size_t)cur * D + (size_t)sdf_ch, dL_dd);
            sha_sum += (double)(dL_ds * ds_dsha);
            for (int c = 0; c < 3; ++c)
                if (rgb[c] == 0.0f)
                    dL_drgb[c] = 0.0f;
            for (int i = 0; i < 3 * nb; ++i)
                acc_add(io->attr_grad, io->attr_grad_abs, (size_t)cur * D + i,
                        Y[i / 3] * dL_drgb[i % 3]);
            T = Tn;
            if (!(T > st->weight_threshold))
                break;
        }
        t0 = fmaxf(t0, t1);
        cur = nxt;
        p[0] = qp[0];
        p[1] = qp[1];
        p[2] = qp[2];
    }
    *sha_acc += sha_sum;
}

/* RadFoam backward (pipeline.cu:553-791): density mode, unsafe walk. */
static void backward_std_ray(const oracle_scene *sc, const oracle_settings *st,
                             const oracle_bwd_io *io, size_t r)
{
    const int nb = (sc->sh_degree + 1) * (sc->sh_degree + 1);
    const uint32_t D = sc->attr_dim;
    oracle_ray ray;
    load_ray(io->rays, r, &ray);
    float Y[16];
    sh_basis(sc->sh_degree, ray.d, Y);
    float g[4], C[4];
    for (int k = 0; k < 4; ++k) {
        g[k] = io->rgba_grad[4 * r + k];
        C[k] = io->rgba[4 * r + k];
    }
    const uint32_t Q = io->quantiles ? io->num_quantiles : 0;
    const float *rq = io->quantiles ? io->quantiles + r * io->num_quantiles : NULL;
    const float *rdg = io->depth_grad ? io->depth_grad + r * io->num_quantiles : NULL;
    float err = io->ray_error ? io->ray_error[r] : 0.0f;
    uint32_t qi = 0;
    float q = 0.0f;
    if (rq && io->num_quantiles > 0)
        q = rq[0];
    /* pipeline.cu:620-629: sum of depth_grad / s over the recorded quantile
     * sites */
    float cur_depth_grad = 0.0f;
    for (uint32_t i = 0; i < Q; ++i) {
        uint32_t pi = io->depth_indices[r * Q + i];
        if (pi != U32_NONE) {
            float sv = sc->attributes[(size_t)pi * D + D - 1];
            cur_depth_grad = cur_depth_grad + rdg[i] / sv;
        }
    }
    float T = 1.0f;
    float acc[3] = {0.0f, 0.0f, 0.0f};
    uint32_t prev_idx = U32_NONE;
    float prev_pt[3] = {0.0f, 0.0f, 0.0f};
    float prev_grad[3] = {0.0f, 0.0f, 0.0f};
    float cur_grad[3] = {0.0f, 0.0f, 0.0f};
    float next_grad[3] = {0.0f, 0.0f, 0.0f};

    float t0 = 0.0f;
    uint32_t n = 0;
    uint32_t cur = io->start[r];
    if (cur >= sc->num_points)
        return;
    float p[3] = {sc->points[3 * (size_t)cur], sc->points[3 * (size_t)cur + 1],
                  sc->points[3 * (size_t)cur + 2]};
    for (;;) {
        ++n;
        if (n > st->max_intersections)
            break;
        uint32_t beg = sc->offsets[cur], end = sc->offsets[cur + 1];
        if (beg > end || end > sc->adjacency_size)
            break;
        float t1;
        uint32_t f = find_exit(sc, &ray, p, beg, end, t0, 0, &t1);
        if (f == U32_NONE)
            break;
        uint32_t nxt = sc->adjacency[beg + f];
        if (nxt >= sc->num_points)
            break;
        const float *qp = sc->points + 3 * (size_t)nxt;
        if (t1 > t0) {
            const float *attr = sc->attributes + (size_t)cur * D;
            float s = attr[D - 1];
            float rgb[3];
            if (s > 1e-6f)
                sh_rgb(nb, Y, attr, rgb);
            else
                rgb[0] = rgb[1] = rgb[2] = 0.0f;
            float dt = fmaxf(t1 - t0, 0.0f);
            float alpha = 1.0f - oracle_expf(-(s * dt));
            float weight = T * alpha;
            float dalpha_ds = dt * (1.0f - alpha);
            float dalpha_ddt = 0.0f;
            if (dt > 0.0f)
                dalpha_ddt = s * (1.0f - alpha);
            for (int c = 0; c < 3; ++c)
                acc[c] = fmaf(weight, rgb[c], acc[c]);
            if (io->point_error) {
#pragma omp atomic
                io->point_error[cur] += weight * err;
            }
            float dL_drgb[3];
            for (int c = 0; c < 3; ++c)
                dL_drgb[c] = g[c] * weight;
            float denom = T * ((1.0f - alpha) + 1e-6f);
            float u[3];
            for (int c = 0; c < 3; ++c)
                u[c] = rgb[c] - (C[c] - acc[c]) / denom;
            float dL_dalpha = T * dot3(u, g);
            dL_dalpha = dL_dalpha + ((1.0f - C[3]) * g[3]) / ((1.0f - alpha) + 1e-6f);
            float dL_ds = dL_dalpha * dalpha_ds;
            float dL_ddt = dL_dalpha * dalpha_ddt;
            float dL_dt0 = 0.0f;
            float Tn = T * (1.0f - alpha);
            while (qi < Q && Tn < q) {
                float dgi = rdg[qi] / s;
                dL_dt0 = dL_dt0 + dgi;
                dL_ds = dL_ds + ((-dgi) * logf(T / q)) / s;
                cur_depth_grad = cur_depth_grad - dgi;
                ++qi;
                if (qi < Q)
                    q = rq[qi];
            }
            if (qi < Q) {
                dL_ds = fmaf(-dt, cur_depth_grad, dL_ds);
                dL_ddt = fmaf(-s, cur_depth_grad, dL_ddt);
            }
            dL_dt0 = dL_dt0 + (-dL_ddt);
            float dL_dt1 = dL_ddt;
            float dprev[3] = {0.0f, 0.0f, 0.0f};
            if (prev_idx != U32_NONE)
                cig(prev_pt, p, &ray, dprev);
            float d1cur[3], d0cur[3], d1next[3];
            cig(p, qp, &ray, d1cur);
            cig(p, prev_pt, &ray, d0cur);
            cig(qp, p, &ray, d1next);
            for (int k = 0; k < 3; ++k) {
                prev_grad[k] = fmaf(dL_dt0, dprev[k], prev_grad[k]);
                cur_grad[k] = cur_grad[k] + fmaf(dL_dt0, d0cur[k], dL_dt1 * d1cur[k]);
                next_grad[k] = fmaf(dL_dt1, d1next[k], next_grad[k]);
            }
            if (prev_idx != U32_NONE) {
                for (int k = 0; k < 3; ++k)
                    acc_add(io->points_grad, io->points_grad_abs,
                            3 * (size_t)prev_idx + k, prev_grad[k]);
            }
            for (int k = 0; k < 3; ++k) {
                prev_pt[k] = p[k];
                prev_grad[k] = cur_grad[k];
                cur_grad[k] = next_grad[k];
                next_grad[k] = 0.0f;
            }
            prev_idx = cur;
            T = Tn;
            for (int c = 0; c < 3; ++c)
                if (rgb[c] == 0.0f)
                    dL_drgb[c] = 0.0f;
            for (int i = 0; i < 3 * nb; ++i)
                acc_add(io->attr_grad, io->attr_grad_abs, (size_t)cur * D + i,
                        Y[i / 3] * dL_drgb[i % 3]);
            acc_add(io->attr_grad, io->attr_grad_abs, (size_t)cur * D + D - 1, dL_ds);
            if (!(T > st->weight_threshold))
                break;
        }
        t0 = fmaxf(t0, t1);
        cur = nxt;
        p[0] = qp[0];
        p[1] = qp[1];
        p[2] = qp[2];
    }
}

void oracle_trace_backward(const oracle_scene *sc, const oracle_settings *st,
                           const oracle_bwd_io *io, int threads)
{
#ifdef _OPENMP
    if (threads > 0)
        omp_set_num_threads(threads);
#else
    (void)threads;
#endif
    double sha_total = 0.0;
#pragma omp parallel for schedule(dynamic, 64) reduction(+ : sha_total)
    for (int64_t r = 0; r < (int64_t)io->num_rays; ++r) {
        if (st->neus)
            backward_neus_ray(sc, st, io, (size_t)r, &sha_total);
        else
            backward_std_ray(sc, st, io, (size_t)r);
    }
    if (st->neus && io->sharpness_grad)
        io->sharpness_grad[0] += (float)sha_total;
}

int oracle_version(void) { return 1; }

/* array forms for the accuracy tests */
void oracle_expf_array(const float *x, float *y, size_t n)
{
    for (size_t i = 0; i < n; ++i)
        y[i] = oracle_expf(x[i]);
}

void oracle_f2h_array(const float *x, uint16_t *y, size_t n)
{
    for (size_t i = 0; i < n; ++i)
        y[i] = oracle_f2h(x[i]);
}

void oracle_h2f_array(const uint16_t *x, float *y, size_t n)
{
    for (size_t i = 0; i < n; ++i)
        y[i] = oracle_h2f(x[i]);
}

/* the SH basis of n unit directions [n][3] -> [n][16] (degree 3) */
void oracle_sh_basis_array(const float *dirs, float *Y, size_t n)
{
    for (size_t i = 0; i < n; ++i)
        sh_basis(3, dirs + 3 * i, Y + 16 * i);
}

/* farthest_neighbor_kernel (src/delaunay/triangulation_ops.cu:10-44):
 * distance sqrt(dx*dx + (dy*dy + dz*dz)) with the first product of each sum
 * fused (Eigen norm as nvcc contracts it); sum += 0.5 * distance is done in
 * double by the reference, i.e. one float rounding of sum + 0.5 d. */
void oracle_farthest_neighbor(const float *points, const uint32_t *adjacency, const uint32_t *offsets,
                              uint32_t num_points, uint32_t adjacency_size, uint32_t *indices, float *radius)
{
    for (uint32_t i = 0; i < num_points; ++i) {
        uint32_t beg = offsets[i], end = offsets[i + 1];
        if (beg > end || end > adjacency_size) {
            indices[i] = U32_NONE;
            radius[i] = u2f(0x7fffffffu);
            continue;
        }
        const float *p = points + 3 * (size_t)i;
        uint32_t best = U32_NONE;
        float best_d = 0.0f, sum = 0.0f;
        for (uint32_t j = beg; j < end; ++j) {
            uint32_t a = adjacency[j];
            if (a >= num_points)
                continue;
            const float *q = points + 3 * (size_t)a;
            float dx = q[0] - p[0], dy = q[1] - p[1], dz = q[2] - p[2];
            float d = sqrtf(fmaf(dx, dx, fmaf(dy, dy, dz * dz)));
            sum = (float)((double)sum + 0.5 * (double)d);
            if (d > best_d) {
                best_d = d;
                best = a;
            }
        }
        indices[i] = best;
        radius[i] = sum / (float)(end - beg);
    }
}
