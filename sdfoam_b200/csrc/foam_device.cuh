// Device-side arithmetic of the Voronoi-foam walk.
//
// Every expression here follows the floating-point contract that the CPU
// checker states in its header: the library is compiled with -fmad=false, so
// only the fmaf() calls written below fuse, divisions and square roots are the
// IEEE-rounded __fdiv_rn / __fsqrt_rn, and exp is foam_expf (own Cody-Waite
// implementation; the reference's __expf is a hardware approximation that no
// CPU reproduces, so both sides of this build share this one).
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace sdfoam_b200 {

constexpr uint32_t kNone = 0xffffffffu;

// exp(x): x = n ln2 + r (Cody & Waite 1980, ln2 split head/tail, fused
// reductions), e^r by its degree-7 Taylor polynomial (truncation < 6e-9
// relative for |r| <= ln2/2), 2^n applied as two exact power-of-two factors.
__device__ __forceinline__ float foam_expf(float x) {
    if (x != x) return x;
    if (x > 88.8f) return __int_as_float(0x7f800000);
    if (x < -104.0f) return 0.0f;
    const float log2e = 1.44269502162933349609375f;
    const float ln2_hi = 0.693147182464599609375f;
    const float ln2_lo = -1.904654323148236e-09f;
    float n = rintf(__fmul_rn(x, log2e));
    float r = fmaf(n, -ln2_hi, x);
    r = fmaf(n, -ln2_lo, r);
    float p = 1.98412698412698413e-04f;
    p = fmaf(p, r, 1.38888888888888889e-03f);
    p = fmaf(p, r, 8.33333333333333333e-03f);
    p = fmaf(p, r, 4.16666666666666667e-02f);
    p = fmaf(p, r, 1.66666666666666667e-01f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = static_cast<int>(n);
    int n1 = ni / 2;
    int n2 = ni - n1;
    float s1 = __int_as_float((n1 + 127) << 23);
    float s2 = __int_as_float((n2 + 127) << 23);
    return __fmul_rn(__fmul_rn(p, s1), s2);
}

// a0 b0 + (a1 b1 + a2 b2) with the first product of each sum fused.
__device__ __forceinline__ float dot3(float a0, float a1, float a2, float b0, float b1, float b2) {
    return fmaf(a0, b0, fmaf(a1, b1, __fmul_rn(a2, b2)));
}

__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}

// Real SH basis up to degree 3 (reference sh_utils.cuh:8-70).
struct SHBasis {
    float y[16];
};

template <int DEG>
__device__ __forceinline__ void sh_basis(float x, float y, float z, SHBasis &b) {
    constexpr float C0 = 0.28209479177387814f;
    constexpr float C1 = 0.4886025119029199f;
    constexpr float C2_0 = 1.0925484305920792f, C2_1 = -1.0925484305920792f,
                    C2_2 = 0.31539156525252005f, C2_3 = -1.0925484305920792f,
                    C2_4 = 0.5462742152960396f;
    constexpr float C3_0 = -0.5900435899266435f, C3_1 = 2.890611442640554f,
                    C3_2 = -0.4570457994644658f, C3_3 = 0.3731763325901154f,
                    C3_4 = -0.4570457994644658f, C3_5 = 1.445305721320277f,
                    C3_6 = -0.5900435899266435f;
#pragma unroll
    for (int k = 0; k < 16; ++k) b.y[k] = 0.0f;
    b.y[0] = C0;
    if (DEG > 0) {
        b.y[1] = __fmul_rn(-C1, y);
        b.y[2] = __fmul_rn(C1, z);
        b.y[3] = __fmul_rn(-C1, x);
    }
    const float xx = __fmul_rn(x, x), yy = __fmul_rn(y, y), zz = __fmul_rn(z, z);
    const float xy = __fmul_rn(x, y), yz = __fmul_rn(y, z), xz = __fmul_rn(x, z);
    if (DEG > 1) {
        b.y[4] = __fmul_rn(C2_0, xy);
        b.y[5] = __fmul_rn(C2_1, yz);
        b.y[6] = __fmul_rn(C2_2, __fsub_rn(__fsub_rn(__fmul_rn(2.0f, zz), xx), yy));
        b.y[7] = __fmul_rn(C2_3, xz);
        b.y[8] = __fmul_rn(C2_4, __fsub_rn(xx, yy));
    }
    if (DEG > 2) {
        const float t4 = __fsub_rn(__fsub_rn(__fmul_rn(4.0f, zz), xx), yy);
        b.y[9] = __fmul_rn(__fmul_rn(C3_0, y), fmaf(3.0f, xx, -yy));
        b.y[10] = __fmul_rn(__fmul_rn(C3_1, xy), z);
        b.y[11] = __fmul_rn(__fmul_rn(C3_2, y), t4);
        b.y[12] = __fmul_rn(__fmul_rn(C3_3, z), fmaf(-3.0f, yy, fmaf(-3.0f, xx, __fmul_rn(2.0f, zz))));
        b.y[13] = __fmul_rn(__fmul_rn(C3_4, x), t4);
        b.y[14] = __fmul_rn(__fmul_rn(C3_5, z), __fsub_rn(xx, yy));
        b.y[15] = __fmul_rn(__fmul_rn(C3_6, x), fmaf(-3.0f, yy, xx));
    }
}

template <int DEG>
struct AttrLayout {
    static constexpr int kBasis = (DEG + 1) * (DEG + 1);
    static constexpr int kSH = 3 * kBasis;          // SH scalars
    static constexpr int kDim = kSH + 1;            // + last scalar (SDF / density)
    static constexpr int kVec4 = (kDim + 3) / 4;    // float4 per gradient row
    static constexpr int kStride = (kSH + 7) / 8 * 8;  // SH row in the cell records
};

// 256-bit read-only global loads (sm_100: ld.global.nc.v8), 32-byte aligned.
__device__ __forceinline__ void ldg256(const void *p, uint32_t (&w)[8]) {
    asm("ld.global.nc.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7])
        : "l"(p));
}

__device__ __forceinline__ void ldg256f(const float *p, float *v) {
    asm("ld.global.nc.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7])
        : "l"(p));
}

// One site's SH coefficients held in registers.
template <int DEG>
struct AttrRow {
    float v[AttrLayout<DEG>::kStride];
};

// load_sh_as_rgb (reference sh_utils.cuh:72-83): 0.5 + sum_k Y_k c_k, clamped at 0.
template <int DEG>
__device__ __forceinline__ void sh_rgb(const SHBasis &b, const AttrRow<DEG> &row, float &r, float &g, float &bl) {
    r = 0.5f;
    g = 0.5f;
    bl = 0.5f;
#pragma unroll
    for (int k = 0; k < AttrLayout<DEG>::kBasis; ++k) {
        r = fmaf(b.y[k], row.v[3 * k + 0], r);
        g = fmaf(b.y[k], row.v[3 * k + 1], g);
        bl = fmaf(b.y[k], row.v[3 * k + 2], bl);
    }
    r = fmaxf(r, 0.0f);
    g = fmaxf(g, 0.0f);
    bl = fmaxf(bl, 0.0f);
}

}  // namespace sdfoam_b200
