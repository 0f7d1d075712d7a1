// Elementwise stages of the sdfnet MLP around its GEMMs (bf16 activations,
// fp32 math), written so that every GEMM of the network is 8-aligned and
// carries its bias as an extra input column of ones:
//
//   encode      points -> [x - c, sin(2 pi 2^k (x - c)), cos(...), 1, 0 ...]
//               (positional encoding of the reference sdfnet.py:21-40, 48
//               columns: 39 features, the bias column, zero padding)
//   activate    z -> a = softplus_100(z), written into the next layer's input
//               buffer followed by the bias column; the layer feeding the
//               skip connection also appends the encoding and scales by
//               1/sqrt(2) (sdfnet.py:128-134)
//   deactivate  dz = da * sigma(100 z), with the derivative recomputed from
//               the stored activation: e^(100 a) = 1 + e^(100 z), so
//               sigma(100 z) = 1 - e^(-100 a).  The activation is kept for
//               the weight gradient anyway, so no derivative is stored.
//   decode      d points from d encoding (chain rule of sin / cos)
//
// Softplus with beta = 100 (PyTorch: beta z > 20 -> z, else
// log1p(exp(beta z)) / beta), evaluated in the overflow-free form
// max(z, 0) + log1p(exp(-beta |z|)) / beta.  Outputs are bf16, so the fast
// exp / log intrinsics (relative error ~1e-7) and the multiply by 1/beta in
// place of a division are below the output rounding.
#include <cuda_bf16.h>

#include "foam_internal.h"

namespace sdfoam_b200 {

namespace {

constexpr float kBeta = 100.0f;
constexpr float kInvBeta = 0.01f;
constexpr float kTwoPi = 6.283185307179586f;

__global__ void __launch_bounds__(256) encode_kernel(const float *__restrict__ points, const float *__restrict__ center,
                                                     uint32_t n, int multires, int ld, __nv_bfloat16 *__restrict__ out) {
    const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float x[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) x[k] = __ldg(points + 3 * i + k) - (center ? __ldg(center + k) : 0.0f);
    __nv_bfloat16 *row = out + i * ld;
    if (multires == 6 && ld == 48) {
        // the sdfnet's encoding: one sincosf per axis and frequency, the row
        // written as six 16-byte vectors
        float v[48];
#pragma unroll
        for (int k = 0; k < 3; ++k) v[k] = x[k];
#pragma unroll
        for (int f = 0; f < 6; ++f) {
            const float w = kTwoPi * float(1 << f);
#pragma unroll
            for (int k = 0; k < 3; ++k) sincosf(x[k] * w, &v[3 + 6 * f + k], &v[6 + 6 * f + k]);
        }
        v[39] = 1.0f;
#pragma unroll
        for (int c = 40; c < 48; ++c) v[c] = 0.0f;
        uint4 *dst = reinterpret_cast<uint4 *>(row);
#pragma unroll
        for (int q = 0; q < 6; ++q) {
            uint32_t w4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const __nv_bfloat162 h = __floats2bfloat162_rn(v[8 * q + 2 * e], v[8 * q + 2 * e + 1]);
                w4[e] = *reinterpret_cast<const uint32_t *>(&h);
            }
            dst[q] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
        return;
    }
    int c = 0;
#pragma unroll
    for (int k = 0; k < 3; ++k) row[c++] = __float2bfloat16_rn(x[k]);
    for (int f = 0; f < multires; ++f) {
        const float w = kTwoPi * float(1 << f);
#pragma unroll
        for (int k = 0; k < 3; ++k) row[c + k] = __float2bfloat16_rn(sinf(x[k] * w));
#pragma unroll
        for (int k = 0; k < 3; ++k) row[c + 3 + k] = __float2bfloat16_rn(cosf(x[k] * w));
        c += 6;
    }
    row[c++] = __float2bfloat16_rn(1.0f);
    for (; c < ld; ++c) row[c] = __float2bfloat16_rn(0.0f);
}

// 8 consecutive bf16 as one 16-byte vector.
struct alignas(16) Bf8 {
    __nv_bfloat162 h[4];
};

__device__ __forceinline__ void bf8_to_f(const Bf8 &v, float *f) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float2 x = __bfloat1622float2(v.h[k]);
        f[2 * k] = x.x;
        f[2 * k + 1] = x.y;
    }
}

__device__ __forceinline__ Bf8 f_to_bf8(const float *f) {
    Bf8 v;
#pragma unroll
    for (int k = 0; k < 4; ++k) v.h[k] = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
    return v;
}

// One warp per row; lane l covers columns [8l, 8l + 8) of the output row
// (and lane 0 also the chunk at 256 for rows wider than 256).  z [n, zc]
// (leading dim ldz) -> out [n, ld]: scale * softplus(z) for c < zc, then
// scale * enc[:, :enc_cols], then 1, then zeros.  All leading dims are
// multiples of 8.
__global__ void __launch_bounds__(256) activate_kernel(const __nv_bfloat16 *__restrict__ z, int ldz, int zc, uint32_t n,
                                                       const __nv_bfloat16 *__restrict__ enc, int ldenc, int enc_cols,
                                                       float scale, int ld, __nv_bfloat16 *__restrict__ out) {
    const uint32_t row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    const size_t i = row;
    for (int c0 = 8 * lane; c0 < ld; c0 += 256) {
        float zf[8], v[8];
        const bool any_z = c0 < zc;
        if (any_z) bf8_to_f(*reinterpret_cast<const Bf8 *>(z + i * ldz + c0), zf);
        float ef[8];
        const bool any_e = enc_cols > 0 && c0 + 8 > zc && c0 < zc + enc_cols;
        if (any_e) {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int e = c0 + k - zc;
                ef[k] = (e >= 0 && e < enc_cols) ? __bfloat162float(enc[i * ldenc + e]) : 0.0f;
            }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int c = c0 + k;
            if (c < zc) {
                // softplus(z) = max(z, 0) + log1p(e^(-beta |z|)) / beta; past
                // PyTorch's threshold (beta z > 20) the second term is below
                // 2e-11 and vanishes in the bf16 output
                const float e = __expf(-kBeta * fabsf(zf[k]));
                const float l = e < 1e-4f ? e * (1.0f - 0.5f * e) : __logf(1.0f + e);
                v[k] = scale * (fmaxf(zf[k], 0.0f) + l * kInvBeta);
            } else if (c < zc + enc_cols) {
                v[k] = scale * ef[k];
            } else {
                v[k] = c == zc + enc_cols ? 1.0f : 0.0f;
            }
        }
        *reinterpret_cast<Bf8 *>(out + i * ld + c0) = f_to_bf8(v);
    }
}

// dz [n, ldz] = scale * da * (1 - exp(-beta act / scale)) for c < cols, 0
// for cols <= c < ldz; one warp per row, 8 columns per lane.
__global__ void __launch_bounds__(256) deactivate_kernel(const __nv_bfloat16 *__restrict__ da, int lda,
                                                         const __nv_bfloat16 *__restrict__ act, int ld_act,
                                                         float scale, uint32_t n, int cols,
                                                         __nv_bfloat16 *__restrict__ dz, int ldz) {
    const float k_exp = -kBeta / scale;
    const uint32_t row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    const size_t i = row;
    for (int c0 = 8 * lane; c0 < ldz; c0 += 256) {
        float a[8], d[8], v[8];
        bf8_to_f(*reinterpret_cast<const Bf8 *>(da + i * lda + c0), a);
        bf8_to_f(*reinterpret_cast<const Bf8 *>(act + i * ld_act + c0), d);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = c0 + k < cols ? scale * a[k] * (1.0f - __expf(k_exp * d[k])) : 0.0f;
        *reinterpret_cast<Bf8 *>(dz + i * ldz + c0) = f_to_bf8(v);
    }
}

// d points [n, 3] (+=) from d encoding: x term plus w cos(w x) / -w sin(w x)
__global__ void __launch_bounds__(256) decode_kernel(const float *__restrict__ points, const float *__restrict__ center,
                                                     uint32_t n, int multires, const __nv_bfloat16 *__restrict__ denc,
                                                     int ld, float *__restrict__ dpoints) {
    const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const __nv_bfloat16 *row = denc + i * ld;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float x = __ldg(points + 3 * i + k) - (center ? __ldg(center + k) : 0.0f);
        float g = __bfloat162float(row[k]);
        for (int f = 0; f < multires; ++f) {
            const float w = kTwoPi * float(1 << f);
            float s, c;
            sincosf(x * w, &s, &c);
            g += __bfloat162float(row[3 + 6 * f + k]) * w * c - __bfloat162float(row[3 + 6 * f + 3 + k]) * w * s;
        }
        dpoints[3 * i + k] += g;
    }
}

// Tangent of the positional encoding along gbar (the forward-mode
// derivative J_enc gbar): [gbar, w cos(w u) gbar, -w sin(w u) gbar per
// frequency], 0 in the ones column and the padding.
__global__ void __launch_bounds__(256) encode_jvp_kernel(const float *__restrict__ points,
                                                         const float *__restrict__ center, uint32_t n, int multires,
                                                         const float *__restrict__ gbar, int ld,
                                                         __nv_bfloat16 *__restrict__ out) {
    const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float x[3], g[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        x[k] = __ldg(points + 3 * i + k) - (center ? __ldg(center + k) : 0.0f);
        g[k] = __ldg(gbar + 3 * i + k);
    }
    __nv_bfloat16 *row = out + i * ld;
    int c = 0;
#pragma unroll
    for (int k = 0; k < 3; ++k) row[c++] = __float2bfloat16_rn(g[k]);
    for (int f = 0; f < multires; ++f) {
        const float w = kTwoPi * float(1 << f);
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            float sn, cs;
            sincosf(x[k] * w, &sn, &cs);
            row[c + k] = __float2bfloat16_rn(w * cs * g[k]);
            row[c + 3 + k] = __float2bfloat16_rn(-w * sn * g[k]);
        }
        c += 6;
    }
    for (; c < ld; ++c) row[c] = __float2bfloat16_rn(0.0f);
}

// dpoints += J_enc^T denc2 + H_enc[denc](gbar): the encoding's share of the
// eikonal term's input gradient -- the first-order chain applied to the
// second sweep's encoding gradient denc2, plus the encoding's curvature
// contracted with the first-order encoding gradient denc and gbar
// (d^2 sin(w u) / du^2 = -w^2 sin(w u), and likewise for cos).
__global__ void __launch_bounds__(256) decode_hessian_kernel(const float *__restrict__ points,
                                                             const float *__restrict__ center, uint32_t n,
                                                             int multires, const __nv_bfloat16 *__restrict__ denc2,
                                                             const __nv_bfloat16 *__restrict__ denc, int ld,
                                                             const float *__restrict__ gbar,
                                                             float *__restrict__ dpoints) {
    const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const __nv_bfloat16 *r2 = denc2 + i * ld;
    const __nv_bfloat16 *r1 = denc + i * ld;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float x = __ldg(points + 3 * i + k) - (center ? __ldg(center + k) : 0.0f);
        const float gb = __ldg(gbar + 3 * i + k);
        float g = __bfloat162float(r2[k]);
        for (int f = 0; f < multires; ++f) {
            const float w = kTwoPi * float(1 << f);
            float sn, cs;
            sincosf(x * w, &sn, &cs);
            const float ds2 = __bfloat162float(r2[3 + 6 * f + k]), dc2 = __bfloat162float(r2[3 + 6 * f + 3 + k]);
            const float ds1 = __bfloat162float(r1[3 + 6 * f + k]), dc1 = __bfloat162float(r1[3 + 6 * f + 3 + k]);
            g += ds2 * w * cs - dc2 * w * sn;
            g -= (ds1 * sn + dc1 * cs) * w * w * gb;
        }
        dpoints[3 * i + k] += g;
    }
}

}  // namespace

cudaError_t launch_mlp_encode_jvp(const float *points, const float *center, uint32_t n, int multires,
                                  const float *gbar, int ld, void *out, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    encode_jvp_kernel<<<(n + 255) / 256, 256, 0, stream>>>(points, center, n, multires, gbar, ld,
                                                           static_cast<__nv_bfloat16 *>(out));
    return cudaGetLastError();
}

cudaError_t launch_mlp_decode_hessian(const float *points, const float *center, uint32_t n, int multires,
                                      const void *denc2, const void *denc, int ld, const float *gbar, float *dpoints,
                                      cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    decode_hessian_kernel<<<(n + 255) / 256, 256, 0, stream>>>(
        points, center, n, multires, static_cast<const __nv_bfloat16 *>(denc2),
        static_cast<const __nv_bfloat16 *>(denc), ld, gbar, dpoints);
    return cudaGetLastError();
}

cudaError_t launch_mlp_encode(const float *points, const float *center, uint32_t n, int multires, int ld,
                              void *out, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    encode_kernel<<<(n + 255) / 256, 256, 0, stream>>>(points, center, n, multires, ld,
                                                       static_cast<__nv_bfloat16 *>(out));
    return cudaGetLastError();
}

cudaError_t launch_mlp_activate(const void *z, int ldz, int zc, uint32_t n, const void *enc, int ldenc, int enc_cols,
                                float scale, int ld, void *out, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    activate_kernel<<<(n + 7) / 8, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16 *>(z), ldz, zc, n, static_cast<const __nv_bfloat16 *>(enc), ldenc, enc_cols,
        scale, ld, static_cast<__nv_bfloat16 *>(out));
    return cudaGetLastError();
}

cudaError_t launch_mlp_deactivate(const void *da, int lda, const void *act, int ld_act, float scale, uint32_t n,
                                  int cols, void *dz, int ldz, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    deactivate_kernel<<<(n + 7) / 8, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16 *>(da), lda, static_cast<const __nv_bfloat16 *>(act), ld_act, scale, n, cols,
        static_cast<__nv_bfloat16 *>(dz), ldz);
    return cudaGetLastError();
}

cudaError_t launch_mlp_decode(const float *points, const float *center, uint32_t n, int multires, const void *denc,
                              int ld, float *dpoints, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    decode_kernel<<<(n + 255) / 256, 256, 0, stream>>>(points, center, n, multires,
                                                       static_cast<const __nv_bfloat16 *>(denc), ld, dpoints);
    return cudaGetLastError();
}

}  // namespace sdfoam_b200
