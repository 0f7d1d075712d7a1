// One hidden layer of the sdfnet MLP on the 5th-generation tensor cores:
//
//   out[r, :] = [scale * softplus_100(x[r, :] W^T)[:zc], scale * enc[r, :enc_cols], 1, 0 ...]
//
// x is the layer input [n, K] (bf16, its last used column the constant 1 that
// carries the bias), W the bias-folded weights [N <= 256, K] (bf16), out the
// next layer's input [n, ld] (the same layout, sdfoam_mlp_activate's output).
//
// A persistent CTA per SM walks 128-row tiles with warp-specialised roles:
//   * warp 0 (one lane) loads W once into shared memory (all K, at most
//     5 x 32 KB) and streams 128 x 64 tiles of x through a 3-stage ring with
//     TMA (128-byte swizzle; rows past n, columns past K and weight rows past
//     N read as zero);
//   * warp 1 allocates 512 TMEM columns, i.e. two fp32 accumulators of
//     128 x 256, and one lane issues tcgen05.mma (M 128, N 256, K 16, bf16)
//     into them, releasing ring stages and finished accumulators with
//     tcgen05.commit;
//   * warps 2-17 read an accumulator back with tcgen05.ld (warp w owns TMEM
//     lanes 32 (w % 4) ... and 64 of the 256 columns, one row per thread)
//     while the MMAs fill the other, apply softplus, the skip columns and
//     the bias column, and store bf16 rows.  Sixteen epilogue warps hide the
//     latency of the loads, the exp / log and the stores.
// Every wait on an mbarrier gives up after half a second and raises a shared
// abort flag that unwinds all roles; the CTA then waits (bounded) for its
// own copies and MMAs, writes NaN rows for the tiles it did not finish, sets
// *error and frees its TMEM.
//
// No TMA multicast: every copy reads this GPU's memory into its own CTA.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include "foam_internal.h"

namespace sdfoam_b200 {

namespace {

constexpr int kTileM = 128;
constexpr int kTileN = 256;
constexpr int kTileK = 64;  // 128 bytes of bf16: one swizzle span
constexpr int kMaxKBlocks = 4;  // K <= 256 on the tensor cores (a bias column at 256 is added in the epilogue)
constexpr int kStages = 3;
constexpr uint32_t kABytes = kTileM * kTileK * 2;  // 16 KB
constexpr uint32_t kBBytes = kTileN * kTileK * 2;  // 32 KB per K block of W
constexpr uint32_t kWBytes = kMaxKBlocks * kBBytes;
constexpr int kEpiWarps = 16;  // 4 per TMEM lane quarter, 64 accumulator columns each
constexpr uint32_t kBoxBytes = 32 * 64;  // an epilogue warp's output box: 32 rows x 32 bf16 columns
constexpr uint32_t kSmemBytes = kWBytes + kStages * kABytes + kEpiWarps * kBoxBytes + (2 * kTileN + 8) * 4 + 1024 + 256;
constexpr uint32_t kTmemCols = 512;
constexpr int kThreads = 32 * (2 + kEpiWarps);
constexpr uint32_t kMaxPolls = 1u << 26;
constexpr uint64_t kWaitNs = 500000000ull;  // half a second: a tile's wait is microseconds
constexpr float kBeta = 100.0f;
constexpr float kInvBeta = 0.01f;

// tcgen05 instruction descriptor, kind::f16: D fp32 (bits 4-5 = 1), A and B
// bf16 (bits 7-9, 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at 24.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(kTileN >> 3) << 17) |
                            (uint32_t(kTileM >> 4) << 24);

// Shared-memory matrix descriptor of a K-major tile written by TMA with the
// 128-byte swizzle: start address >> 4, leading offset 1 (unused for this
// layout), stride 1024 bytes between 8-row groups, version 1, layout 2.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
    uint64_t d = uint64_t((smem_addr >> 4) & 0x3fffu);
    d |= uint64_t(1) << 16;
    d |= uint64_t(1024 >> 4) << 32;
    d |= uint64_t(1) << 46;
    d |= uint64_t(2) << 61;
    return d;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Polls the phase of the given parity.  False when *abort is raised or after
// kWaitNs nanoseconds (which raises *abort); abort == nullptr: only the time
// bound (the clean-up waits).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort) {
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0; i < kMaxPolls; ++i) {
        uint32_t done;
        asm volatile(
            "{\n"
            ".reg .pred p;\n"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            "selp.u32 %0, 1, 0, p;\n"
            "}\n"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return true;
        if ((i & 255u) == 255u) {
            if (abort && *abort) return false;
            if (global_ns() - t0 > kWaitNs) break;
        }
    }
    if (abort) *abort = 1;
    return false;
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
        "}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_bf16_id(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
        "}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float *v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int k = 0; k < 32; ++k) v[k] = __uint_as_float(r[k]);
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float lg2_approx(float x) {
    float y;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// scale * softplus_100(z) = scale * (max(z, 0) + log1p(e) / 100), e = 2^(-100 log2(e) |z|):
// log1p(e) = ln 2 * log2(1 + e), or e (1 - e / 2) once 1 + e would round
// (e < 1e-4; error below 1e-8 relative).  The hardware exp2 / log2 carry
// ~2^-22 relative error, far below the bf16 output.
__device__ __forceinline__ float softplus100(float z, float scale) {
    const float e = ex2_approx(-144.26950408889634f * fabsf(z));
    const float big = 0.6931471805599453f * lg2_approx(1.0f + e);
    const float small = e * (1.0f - 0.5f * e);
    return scale * (fmaxf(z, 0.0f) + (e < 1e-4f ? small : big) * kInvBeta);
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return uint32_t(__bfloat16_as_ushort(h.x)) | (uint32_t(__bfloat16_as_ushort(h.y)) << 16);
}

struct LayerParams {
    uint32_t n;         // rows
    int k_blocks;       // ceil(K / 64), at most kMaxKBlocks
    int zc;             // forward: softplus columns; backward: derivative columns
    int enc_cols;       // forward: skip columns appended after them
    int ld;             // output leading dimension (multiple of 8, >= zc + enc_cols + 1)
    int ldenc;
    float scale;
    const __nv_bfloat16 *enc;
    __nv_bfloat16 *out;
    int *error;
    // forward with K > 256: the bias W[:, 256] (stride ldw) over nw rows
    const __nv_bfloat16 *wbias;
    int ldw, nw;
    // backward: the activation the derivative is recomputed from, and the
    // gradient of the skip columns [zc, 256) (scaled), if any
    const __nv_bfloat16 *act;
    int ld_act;
    __nv_bfloat16 *skip;
    int ldskip;
    // forward, optional: the next (output) layer's single row wdot [>= 257,
    // bias at 256] applied to this layer's bf16 output; zdot [n, 4] receives
    // the dot product of each 64-column block times dot_scale (the bias in
    // the last block)
    const __nv_bfloat16 *wdot;
    float *zdot;
    float dot_scale;
    // backward, optional: added to the first add_cols output columns
    const __nv_bfloat16 *add;
    int ldadd, add_cols;
    // backward, eikonal modes (optional):
    //   zout [n, ldzo]: the raw product (before the derivative) as bf16,
    //     columns past zc zero -- the tangent pre-activations;
    //   inj_dz, inj_tz: adds dz * tz * 100 (1 - sigmoid(100 z)) to the first
    //     zc columns (the second derivative of softplus_100 along the
    //     tangent tz, weighted by the first-order gradient dz);
    //   enc / enc_cols: columns [zc, zc + enc_cols) of the output are
    //     scale * enc (the tangent of the skip concatenation)
    __nv_bfloat16 *zout;
    int ldzo;
    const __nv_bfloat16 *inj_dz, *inj_tz;
    int ld_inj_dz, ld_inj_tz;
};

// Stores a warp's 32 x 32 bf16 box (rows y .. y+31, columns x .. x+31; lane
// = row) through the warp's shared-memory staging buffer: every lane writes
// its row's 64 bytes with the 64-byte swizzle of the output tensor map
// (16-byte chunk q of row r at chunk q ^ ((r >> 1) & 3): conflict-free, and
// what the TMA unit reads back), then one lane issues the TMA store.  Rows
// past n and columns past the row width are dropped by the TMA unit.  The
// buffer is reused once the previous store has read it.
__device__ __forceinline__ void store_box(unsigned char *box, const CUtensorMap *map, const uint32_t (&wd)[16], int x,
                                          int y, uint32_t lane) {
    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    __syncwarp();
    unsigned char *row = box + lane * 64u;
    const uint32_t sw = (lane >> 1) & 3u;
#pragma unroll
    for (uint32_t q = 0; q < 4; ++q)
        *reinterpret_cast<uint4 *>(row + ((q ^ sw) << 4)) =
            make_uint4(wd[4 * q], wd[4 * q + 1], wd[4 * q + 2], wd[4 * q + 3]);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) {
        asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                         reinterpret_cast<uint64_t>(map)),
                     "r"(x), "r"(y), "r"(smem_u32(box))
                     : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
}

// Output column c >= zc of a forward row: the skip (encoding) columns, the
// bias column, zero padding.
__device__ __forceinline__ float tail_value(const LayerParams &P, uint32_t row, bool live, int c) {
    if (c < P.zc + P.enc_cols) return live ? P.scale * __bfloat162float(P.enc[size_t(row) * P.ldenc + (c - P.zc)]) : 0.0f;
    return c == P.zc + P.enc_cols ? 1.0f : 0.0f;
}

// Columns [c_beg, c_end) of the warp's 32 output rows row0 + lane from their
// accumulator (TMEM lane = row in the tile), plus the bias column (bias_s,
// fp32, zero when there is none); the warp holding the last block also
// writes the columns past the accumulator (the bias column and padding).
// The bf16 pair of a packed word as floats.
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ void store_row(const LayerParams &P, const CUtensorMap *map_out, unsigned char *box,
                                          const float *bias_s, const float *dot_s, uint32_t taddr, uint32_t row0,
                                          uint32_t lane, int c_beg, int c_end, bool tail) {
    const uint32_t row = row0 + lane;
    const bool live = row < P.n;
    float dot = 0.0f;
    for (int c0 = c_beg; c0 < c_end; c0 += 32) {
        float v[32];
        tmem_ld32(taddr + c0, v);  // every lane of the warp takes part
        if (c0 >= P.ld) continue;  // the same for every lane
        uint32_t wd[16];
        if (c0 + 32 <= P.zc) {
            // the common chunk: softplus only
#pragma unroll
            for (int k = 0; k < 32; k += 4) {
                const float4 b = *reinterpret_cast<const float4 *>(bias_s + c0 + k);
                wd[k / 2] = pack_bf16(softplus100(v[k] + b.x, P.scale), softplus100(v[k + 1] + b.y, P.scale));
                wd[k / 2 + 1] = pack_bf16(softplus100(v[k + 2] + b.z, P.scale), softplus100(v[k + 3] + b.w, P.scale));
            }
            if (P.zdot) {
                // the output layer on the stored (bf16) activations
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    dot = fmaf(bf_lo(wd[k]), dot_s[c0 + 2 * k], dot);
                    dot = fmaf(bf_hi(wd[k]), dot_s[c0 + 2 * k + 1], dot);
                }
            }
        } else {
            // the chunk where softplus ends and the skip / bias columns begin
            // (c is the same for every lane: no divergence)
#pragma unroll
            for (int k = 0; k < 32; k += 2) {
                float y[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int c = c0 + k + e;
                    y[e] = c < P.zc ? softplus100(v[k + e] + bias_s[c], P.scale) : tail_value(P, row, live, c);
                }
                wd[k / 2] = pack_bf16(y[0], y[1]);
            }
            if (P.zdot) {
                for (int k = 0; k < 16; ++k) {
                    const int c = c0 + 2 * k;
                    if (c < P.zc) dot = fmaf(bf_lo(wd[k]), dot_s[c], dot);
                    if (c + 1 < P.zc) dot = fmaf(bf_hi(wd[k]), dot_s[c + 1], dot);
                }
            }
        }
        store_box(box, map_out, wd, c0, int(row0), lane);
    }
    if (P.zdot && live) {
        // + the output layer's bias (the bias column of ones) once per row;
        // each 64-column block writes its own partial (summed in a fixed
        // order by the caller, so the result is the same every run)
        if (tail) dot += dot_s[kTileN];
        P.zdot[size_t(row) * 4 + c_beg / 64] = dot * P.dot_scale;
    }
    if (!tail) return;
    for (int c0 = kTileN; c0 < P.ld; c0 += 32) {
        uint32_t wd[16];
#pragma unroll
        for (int k = 0; k < 32; k += 2)
            wd[k / 2] = pack_bf16(tail_value(P, row, live, c0 + k), tail_value(P, row, live, c0 + k + 1));
        store_box(box, map_out, wd, c0, int(row0), lane);
    }
}

// Backward epilogue: columns [c_beg, c_end) of dz[row] = scale * acc *
// sigmoid(100 z) for the warp's 32 rows row0 + lane, with sigmoid(100 z) =
// 1 - e^(-100 act / scale) from the stored activation act = scale *
// softplus_100(z); columns past zc are the skip gradient (scale * acc into
// P.skip) and leave dz zero.
__device__ __forceinline__ void store_row_backward(const LayerParams &P, const CUtensorMap *map_out,
                                                   unsigned char *box, uint32_t taddr, uint32_t row0, uint32_t lane,
                                                   int c_beg, int c_end) {
    const uint32_t row = row0 + lane;
    const bool live = row < P.n;
    const __nv_bfloat16 *arow = P.act ? P.act + size_t(live ? row : 0u) * P.ld_act : nullptr;
    const float k_exp = -144.26950408889634f / P.scale;  // -100 log2(e) / scale
    for (int c0 = c_beg; c0 < c_end; c0 += 32) {
        float v[32];
        tmem_ld32(taddr + c0, v);  // every lane of the warp takes part
        if (c0 >= P.ld && (c0 + 32 <= P.zc || !P.skip)) continue;  // the same for every lane
        uint32_t wd[16];
        if (!live) {
#pragma unroll
            for (int k = 0; k < 16; ++k) wd[k] = 0u;
        } else if (!arow) {
            // no activation: the plain product (+ the addend), e.g. the
            // gradient of the layer's input
            const __nv_bfloat16 *addr = P.add ? P.add + size_t(row) * P.ldadd : nullptr;
#pragma unroll
            for (int k = 0; k < 32; k += 2) {
                float y[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int c = c0 + k + e;
                    y[e] = c < P.zc ? P.scale * v[k + e] : 0.0f;
                    if (addr && c < P.add_cols) y[e] += __bfloat162float(addr[c]);
                }
                wd[k / 2] = pack_bf16(y[0], y[1]);
            }
        } else if (c0 + 32 <= P.zc) {
            const uint4 *src = reinterpret_cast<const uint4 *>(arow + c0);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint4 a4 = src[q];
                const uint32_t aw[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float a0 = __uint_as_float(aw[e] << 16), a1 = __uint_as_float(aw[e] & 0xffff0000u);
                    const int k = 8 * q + 2 * e;
                    wd[4 * q + e] = pack_bf16(P.scale * v[k] * (1.0f - ex2_approx(k_exp * a0)),
                                              P.scale * v[k + 1] * (1.0f - ex2_approx(k_exp * a1)));
                }
            }
        } else {
#pragma unroll
            for (int k = 0; k < 32; k += 2) {
                float y[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int c = c0 + k + e;  // the same for every lane: no divergence
                    if (c < P.zc) {
                        const float a = __bfloat162float(arow[c]);
                        y[e] = P.scale * v[k + e] * (1.0f - ex2_approx(k_exp * a));
                    } else {
                        y[e] = 0.0f;
                        if (P.skip) P.skip[size_t(row) * P.ldskip + (c - P.zc)] = __float2bfloat16_rn(P.scale * v[k + e]);
                    }
                }
                wd[k / 2] = pack_bf16(y[0], y[1]);
            }
        }
        if (c0 < P.ld) store_box(box, map_out, wd, c0, int(row0), lane);
    }
}

// The eikonal term's sweeps (layer_kernel<kModeEikonal>): columns [c_beg,
// c_end) of out[row] = scale * acc * sigma'(z) (+ dz * tz * 100 (1 -
// sigma'(z)) with the second sweep's addend), the skip columns (the tangent's
// appended encoding, or the second sweep's skip gradient into P.skip), and
// the raw product into P.zout (the tangent pre-activations).
__device__ __forceinline__ void store_row_eikonal(const LayerParams &P, const CUtensorMap *map_out,
                                                  unsigned char *box, uint32_t taddr, uint32_t row0, uint32_t lane,
                                                  int c_beg, int c_end) {
    const uint32_t row = row0 + lane;
    const bool live = row < P.n;
    const size_t r = live ? row : 0u;
    const __nv_bfloat16 *arow = P.act + r * P.ld_act;
    const __nv_bfloat16 *drow = P.inj_dz ? P.inj_dz + r * P.ld_inj_dz : nullptr;
    const __nv_bfloat16 *trow = P.inj_tz ? P.inj_tz + r * P.ld_inj_tz : nullptr;
    const float k_exp = -144.26950408889634f / P.scale;  // -100 log2(e) / scale
    for (int c0 = c_beg; c0 < c_end; c0 += 32) {
        float v[32];
        tmem_ld32(taddr + c0, v);  // every lane of the warp takes part
        if (c0 >= P.ld && (c0 + 32 <= P.zc || !P.skip)) continue;  // the same for every lane
        uint32_t wd[16], zw[16];
        if (!live) {
#pragma unroll
            for (int k = 0; k < 16; ++k) wd[k] = zw[k] = 0u;
        } else if (c0 + 32 <= P.zc) {
            // the common chunk: 16-byte loads of the activation (and of dz, tz)
            const uint4 *asrc = reinterpret_cast<const uint4 *>(arow + c0);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint4 a4 = asrc[q];
                uint4 d4 = make_uint4(0, 0, 0, 0), t4 = d4;
                if (drow) {
                    d4 = reinterpret_cast<const uint4 *>(drow + c0)[q];
                    t4 = reinterpret_cast<const uint4 *>(trow + c0)[q];
                }
                const uint32_t aw[4] = {a4.x, a4.y, a4.z, a4.w};
                const uint32_t dw[4] = {d4.x, d4.y, d4.z, d4.w};
                const uint32_t tw[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int k = 8 * q + 2 * e;
                    const float s0 = 1.0f - ex2_approx(k_exp * bf_lo(aw[e]));
                    const float s1 = 1.0f - ex2_approx(k_exp * bf_hi(aw[e]));
                    float y0 = P.scale * v[k] * s0, y1 = P.scale * v[k + 1] * s1;
                    if (drow) {
                        y0 += bf_lo(dw[e]) * bf_lo(tw[e]) * 100.0f * (1.0f - s0);
                        y1 += bf_hi(dw[e]) * bf_hi(tw[e]) * 100.0f * (1.0f - s1);
                    }
                    wd[4 * q + e] = pack_bf16(y0, y1);
                    zw[4 * q + e] = pack_bf16(v[k], v[k + 1]);
                }
            }
        } else {
            // the chunk where the derivative columns end (c is the same for
            // every lane: no divergence)
#pragma unroll
            for (int k = 0; k < 32; k += 2) {
                float y[2], zr[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int c = c0 + k + e;
                    zr[e] = 0.0f;
                    if (c < P.zc) {
                        const float s1 = 1.0f - ex2_approx(k_exp * __bfloat162float(arow[c]));
                        y[e] = P.scale * v[k + e] * s1;
                        if (drow)
                            y[e] += __bfloat162float(drow[c]) * __bfloat162float(trow[c]) * 100.0f * (1.0f - s1);
                        zr[e] = v[k + e];
                    } else {
                        y[e] = (P.enc && c < P.zc + P.enc_cols)
                                   ? P.scale * __bfloat162float(P.enc[r * P.ldenc + (c - P.zc)])
                                   : 0.0f;
                        if (P.skip) P.skip[r * P.ldskip + (c - P.zc)] = __float2bfloat16_rn(P.scale * v[k + e]);
                    }
                }
                wd[k / 2] = pack_bf16(y[0], y[1]);
                zw[k / 2] = pack_bf16(zr[0], zr[1]);
            }
        }
        if (P.zout && live && c0 < P.ldzo) {
            uint4 *dst = reinterpret_cast<uint4 *>(P.zout + r * P.ldzo + c0);
#pragma unroll
            for (int q = 0; q < 4; ++q) dst[q] = make_uint4(zw[4 * q], zw[4 * q + 1], zw[4 * q + 2], zw[4 * q + 3]);
        }
        if (c0 < P.ld) store_box(box, map_out, wd, c0, int(row0), lane);
    }
}

__device__ __forceinline__ void nan_row(const LayerParams &P, uint32_t row, int c_beg, int c_end) {
    if (row >= P.n) return;
    __nv_bfloat16 *orow = P.out + size_t(row) * P.ld;
    for (int c = c_beg; c < c_end && c < P.ld; ++c) orow[c] = __float2bfloat16_rn(__int_as_float(0x7fc00000));
}

// layer_kernel modes: the forward epilogue, the backward (dgrad / input
// gradient) epilogue, the eikonal sweeps' epilogue.
constexpr int kModeForward = 0, kModeBackward = 1, kModeEikonal = 2;

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) layer_kernel(const __grid_constant__ CUtensorMap map_x,
                                                            const __grid_constant__ CUtensorMap map_w,
                                                            const __grid_constant__ CUtensorMap map_out,
                                                            const LayerParams P) {
    extern __shared__ unsigned char smem_raw[];
    // 1024-byte alignment (of the shared-window address) for the swizzled tiles
    unsigned char *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    unsigned char *w_smem = smem;                          // [k_blocks][256 x 64]
    unsigned char *a_smem = smem + kWBytes;                // [kStages][128 x 64]
    unsigned char *out_smem = a_smem + kStages * kABytes;  // [kEpiWarps][32 x 32] output boxes
    float *bias_s = reinterpret_cast<float *>(out_smem + kEpiWarps * kBoxBytes);  // [256]
    float *dot_s = bias_s + kTileN;                                                // [257]
    uint64_t *bars = reinterpret_cast<uint64_t *>(dot_s + kTileN + 8);
    // bars: w_full, a_full[3], a_empty[3], acc_full[2], acc_empty[2], drain
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 12);
    __shared__ volatile int abort_flag;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t w_full = smem_u32(bars), a_full = w_full + 8, a_empty = a_full + 8 * kStages;
    const uint32_t acc_full = a_empty + 8 * kStages, acc_empty = acc_full + 16, drain = acc_empty + 16;
    const uint32_t num_tiles = (P.n + kTileM - 1) / kTileM;
    const uint32_t my_tiles = blockIdx.x < num_tiles ? (num_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;

    if (threadIdx.x == 0) {
        mbar_init(w_full, 1);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(a_full + 8 * s, 1);
            mbar_init(a_empty + 8 * s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(acc_full + 8 * b, 1);
            mbar_init(acc_empty + 8 * b, kEpiWarps);  // one arrival per epilogue warp
        }
        mbar_init(drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        abort_flag = 0;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // ---- producer ----
        mbar_expect_tx(w_full, uint32_t(P.k_blocks) * kBBytes);
        for (int kb = 0; kb < P.k_blocks; ++kb) tma_load_2d(smem_u32(w_smem + kb * kBBytes), &map_w, kb * kTileK, 0, w_full);
        uint32_t issued = 0;
        bool ok = true;
        for (uint32_t i = 0; i < my_tiles && ok; ++i) {
            const int row0 = int((blockIdx.x + i * gridDim.x) * kTileM);
            for (int kb = 0; kb < P.k_blocks; ++kb, ++issued) {
                const uint32_t s = issued % kStages, u = issued / kStages;
                if (u > 0 && !mbar_wait(a_empty + 8 * s, (u - 1) & 1, &abort_flag)) {
                    ok = false;
                    break;
                }
                mbar_expect_tx(a_full + 8 * s, kABytes);
                tma_load_2d(smem_u32(a_smem + s * kABytes), &map_x, kb * kTileK, row0, a_full + 8 * s);
            }
        }
        // own copies: the weights and the last use of every stage
        mbar_wait(w_full, 0, nullptr);
        for (uint32_t l = issued > kStages ? issued - kStages : 0; l < issued; ++l)
            mbar_wait(a_full + 8 * (l % kStages), (l / kStages) & 1, nullptr);
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer ----
        bool ok = mbar_wait(w_full, 0, &abort_flag);
        uint32_t consumed = 0;
        for (uint32_t i = 0; i < my_tiles && ok; ++i) {
            const uint32_t b = i & 1, v = i >> 1;
            if (v > 0 && !mbar_wait(acc_empty + 8 * b, (v - 1) & 1, &abort_flag)) {
                ok = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;");
            const uint32_t d = tmem + b * kTileN;
            for (int kb = 0; kb < P.k_blocks; ++kb, ++consumed) {
                const uint32_t s = consumed % kStages, u = consumed / kStages;
                if (!mbar_wait(a_full + 8 * s, u & 1, &abort_flag)) {
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint64_t ad = sw128_desc(smem_u32(a_smem + s * kABytes));
                const uint64_t bd = sw128_desc(smem_u32(w_smem + kb * kBBytes));
#pragma unroll
                for (int k = 0; k < kTileK / 16; ++k)
                    mma_bf16(d, ad + uint64_t(2 * k), bd + uint64_t(2 * k), (kb > 0 || k > 0) ? 1u : 0u);
                mma_commit(a_empty + 8 * s);
            }
            if (ok) mma_commit(acc_full + 8 * b);
        }
        // no MMA may still be running when the accumulators are freed
        mma_commit(drain);
        mbar_wait(drain, 0, nullptr);
    } else if (warp >= 2) {
        // ---- epilogue: warp w owns TMEM lane quarter w % 4 and one of four
        // 64-column blocks; the last block also writes the tail columns ----
        const uint32_t quarter = warp & 3;
        const int block = int(warp - 2) / 4;
        const int c_beg = block * (kTileN / 4), c_end = c_beg + kTileN / 4;
        const bool tail = block == 3;
        unsigned char *box = out_smem + (warp - 2) * kBoxBytes;
        if (MODE == kModeForward) {
            // the bias column of W (fp32; zero past nw or without one)
            const uint32_t t = threadIdx.x - 64u;
            if (t < uint32_t(kTileN))
                bias_s[t] = (P.wbias && int(t) < P.nw) ? __bfloat162float(P.wbias[size_t(t) * P.ldw]) : 0.0f;
            if (t <= uint32_t(kTileN)) dot_s[t] = P.wdot ? __bfloat162float(P.wdot[t]) : 0.0f;
            asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
        }
        uint32_t i = 0;
        for (; i < my_tiles; ++i) {
            const uint32_t b = i & 1, v = i >> 1;
            if (!mbar_wait(acc_full + 8 * b, v & 1, &abort_flag)) break;
            asm volatile("tcgen05.fence::after_thread_sync;");
            const uint32_t row0 = (blockIdx.x + i * gridDim.x) * kTileM + quarter * 32;
            if (MODE == kModeBackward)
                store_row_backward(P, &map_out, box, tmem + ((quarter * 32) << 16) + b * kTileN, row0, lane, c_beg,
                                   c_end);
            else if (MODE == kModeEikonal)
                store_row_eikonal(P, &map_out, box, tmem + ((quarter * 32) << 16) + b * kTileN, row0, lane, c_beg,
                                  c_end);
            else
                store_row(P, &map_out, box, bias_s, dot_s, tmem + ((quarter * 32) << 16) + b * kTileN, row0, lane,
                          c_beg, c_end, tail);
            asm volatile("tcgen05.fence::before_thread_sync;");
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + 8 * b);
        }
        // this warp's TMA stores are complete before the rows below and the
        // kernel's end
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        __syncwarp();
        for (; i < my_tiles; ++i)
            nan_row(P, (blockIdx.x + i * gridDim.x) * kTileM + quarter * 32 + lane, c_beg, tail ? P.ld : c_end);
    }
    __syncthreads();
    if (abort_flag && threadIdx.x == 0) atomicExch(P.error, 1);
    if (warp == 1) {
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// --------------------------------------------------------------------------
// weight gradient: dw[m, c] += sum_r dz[r, m] act[r, c]
// --------------------------------------------------------------------------
//
// A GEMM whose reduction runs over the rows (K = n, millions), with both
// operands row-major in HBM: A = dz^T and B = act^T are MN-major for the
// tensor cores.  A persistent CTA per SM takes a contiguous range of 64-row
// chunks:
//   * warp 0 (one lane) streams each chunk's dz columns (up to 4 boxes of
//     64 rows x 64 columns) and act columns (up to 4 boxes) into a 3-stage
//     ring with TMA (128-byte swizzle, rows past n read as zero);
//   * warp 1 holds up to two fp32 accumulators of 128 x 256 in TMEM (the
//     two 128-row halves of dw) and one lane issues tcgen05.mma (M 128,
//     N = 64 x act boxes, K 16, both operands MN-major) over the chunk;
//   * warps 2-3 add up the chunk's dz columns from shared memory: the
//     gradient of a bias column of ones (bias_col);
//   * warps 4-7 read the accumulators back once at the end (tcgen05.ld) and
//     add them to dw with 128-bit vector atomics (fp32, zeroed by the
//     caller): one partial sum per SM.
// Waits are bounded as in layer_kernel; a CTA that gives up sets *error and
// adds nothing from its accumulators.  No TMA multicast.
constexpr int kWgRows = 64;                           // rows (K) per stage
constexpr uint32_t kWgBox = kWgRows * 64 * 2;         // 64 rows x 64 bf16 columns: 8 KB
constexpr int kWgStages = 3;
constexpr uint32_t kWgStageBytes = 8 * kWgBox;        // 4 dz boxes + 4 act boxes
constexpr uint32_t kWgSmemBytes = kWgStages * kWgStageBytes + 1024 + 256;
constexpr int kWgThreads = 256;

struct WgradParams {
    uint32_t n;       // rows (the reduction)
    int a_boxes;      // 64-column boxes of dz per chunk (ceil(m / 64))
    int halves;       // 128-row halves of dw (ceil(m / 128))
    int b_boxes;      // 64-column boxes of act per chunk: MMA N = 64 b_boxes
    int m;            // rows of dw (columns of dz)
    int kcols;        // columns of dw from the MMA (multiple of 4, <= 64 b_boxes)
    int bias_col;     // dw column for the sums of dz's columns, or -1
    float *dw;        // [m, lddw] fp32, 16-byte aligned, accumulated
    int lddw;         // multiple of 4
    int *error;
};

// Shared-memory descriptor of an MN-major operand written by TMA with the
// 128-byte swizzle: 64-element blocks along M (or N) `lbo` bytes apart, 8-row
// groups along K 1024 bytes apart, version 1, layout 2.
__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t smem_addr, uint32_t lbo) {
    uint64_t d = uint64_t((smem_addr >> 4) & 0x3fffu);
    d |= uint64_t((lbo >> 4) & 0x3fffu) << 16;
    d |= uint64_t(1024 >> 4) << 32;
    d |= uint64_t(1) << 46;
    d |= uint64_t(2) << 61;
    return d;
}

// kind::f16 instruction descriptor: D fp32, A and B bf16, both MN-major
// (bits 15 and 16), N >> 3 at bit 17, M = 128.
__device__ __forceinline__ uint32_t wgrad_idesc(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (1u << 16) | (uint32_t(n >> 3) << 17) |
           (uint32_t(kTileM >> 4) << 24);
}

__device__ __forceinline__ void red_add_v4f(float *p, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

__global__ void __launch_bounds__(kWgThreads, 1) wgrad_kernel(const __grid_constant__ CUtensorMap map_dz,
                                                              const __grid_constant__ CUtensorMap map_act,
                                                              const WgradParams P) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    // stage s: dz boxes at smem + s * kWgStageBytes, act boxes 4 boxes further
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kWgStages * kWgStageBytes);
    // bars: a_full[3], a_empty[3], acc_full, drain
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 8);
    __shared__ volatile int abort_flag;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t a_full = smem_u32(bars), a_empty = a_full + 8 * kWgStages;
    const uint32_t acc_full = a_empty + 8 * kWgStages, drain = acc_full + 8;
    const uint32_t chunks = (P.n + kWgRows - 1) / kWgRows;
    const uint32_t per = (chunks + gridDim.x - 1) / gridDim.x;
    const uint32_t c_beg = blockIdx.x * per;
    const uint32_t my = c_beg < chunks ? min(per, chunks - c_beg) : 0u;
    const bool colsum = P.bias_col >= 0;
    const uint32_t tmem_cols = P.halves > 1 ? 512u : 256u;

    // dz boxes that no copy fills (dw with fewer than 256 rows) multiply as
    // zeros: clear them once in every stage
    if (P.a_boxes < 4) {
        const uint32_t per_stage = uint32_t(4 - P.a_boxes) * (kWgBox / 16);
        for (uint32_t i = threadIdx.x; i < kWgStages * per_stage; i += blockDim.x) {
            const uint32_t st = i / per_stage, j = i % per_stage;
            reinterpret_cast<uint4 *>(smem + st * kWgStageBytes + P.a_boxes * kWgBox)[j] = make_uint4(0, 0, 0, 0);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (threadIdx.x == 0) {
        for (int st = 0; st < kWgStages; ++st) {
            mbar_init(a_full + 8 * st, 1);
            mbar_init(a_empty + 8 * st, colsum ? 3 : 1);  // the MMA commit (+ the two column-sum warps)
        }
        mbar_init(acc_full, 1);
        mbar_init(drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        abort_flag = 0;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // ---- producer ----
        const uint32_t bytes = uint32_t(P.a_boxes + P.b_boxes) * kWgBox;
        uint32_t issued = 0;
        for (; issued < my; ++issued) {
            const uint32_t st = issued % kWgStages, u = issued / kWgStages;
            if (u > 0 && !mbar_wait(a_empty + 8 * st, (u - 1) & 1, &abort_flag)) break;
            unsigned char *base = smem + st * kWgStageBytes;
            const int row0 = int((c_beg + issued) * kWgRows);
            mbar_expect_tx(a_full + 8 * st, bytes);
            for (int b = 0; b < P.a_boxes; ++b)
                tma_load_2d(smem_u32(base + b * kWgBox), &map_dz, b * 64, row0, a_full + 8 * st);
            for (int b = 0; b < P.b_boxes; ++b)
                tma_load_2d(smem_u32(base + (4 + b) * kWgBox), &map_act, b * 64, row0, a_full + 8 * st);
        }
        // own copies: the last use of every stage
        for (uint32_t l = issued > kWgStages ? issued - kWgStages : 0; l < issued; ++l)
            mbar_wait(a_full + 8 * (l % kWgStages), (l / kWgStages) & 1, nullptr);
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer ----
        const uint32_t idesc = wgrad_idesc(64 * P.b_boxes);
        bool ok = true;
        for (uint32_t i = 0; i < my; ++i) {
            const uint32_t st = i % kWgStages, u = i / kWgStages;
            if (!mbar_wait(a_full + 8 * st, u & 1, &abort_flag)) {
                ok = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;");
            const uint32_t base = smem_u32(smem + st * kWgStageBytes);
#pragma unroll
            for (int j = 0; j < kWgRows / 16; ++j) {
                const uint64_t bd = sw128_mn_desc(base + 4 * kWgBox + j * 2048, kWgBox);
                for (int h = 0; h < P.halves; ++h) {
                    const uint64_t ad = sw128_mn_desc(base + h * 2 * kWgBox + j * 2048, kWgBox);
                    mma_bf16_id(tmem + h * kTileN, ad, bd, idesc, (i > 0 || j > 0) ? 1u : 0u);
                }
            }
            mma_commit(a_empty + 8 * st);
        }
        if (ok && my > 0) mma_commit(acc_full);
        // no MMA may still be running when the accumulators are freed
        mma_commit(drain);
        mbar_wait(drain, 0, nullptr);
    } else if (warp == 2 || warp == 3) {
        // ---- column sums of dz (the bias column's gradient) ----
        if (colsum) {
            const uint32_t t = threadIdx.x - 64u;
            const uint32_t c = t & 31u;               // 16-byte chunk: columns 8c .. 8c+7
            const uint32_t r_beg = (t >> 5) * 32u;    // rows r_beg .. r_beg+31 of the chunk
            const bool active = c < uint32_t(P.a_boxes) * 8u;
            float acc[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
            for (uint32_t i = 0; i < my; ++i) {
                const uint32_t st = i % kWgStages, u = i / kWgStages;
                if (!mbar_wait(a_full + 8 * st, u & 1, &abort_flag)) break;
                if (active) {
                    const unsigned char *box = smem + st * kWgStageBytes + (c >> 3) * kWgBox;
#pragma unroll 4
                    for (uint32_t r = r_beg; r < r_beg + 32u; ++r) {
                        const uint4 q = *reinterpret_cast<const uint4 *>(box + r * 128u + (((c & 7u) ^ (r & 7u)) << 4));
                        acc[0] += bf_lo(q.x);
                        acc[1] += bf_hi(q.x);
                        acc[2] += bf_lo(q.y);
                        acc[3] += bf_hi(q.y);
                        acc[4] += bf_lo(q.z);
                        acc[5] += bf_hi(q.z);
                        acc[6] += bf_lo(q.w);
                        acc[7] += bf_hi(q.w);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(a_empty + 8 * st);
            }
            if (active && !abort_flag) {
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int col = int(8 * c) + e;
                    if (col < P.m) atomicAdd(P.dw + size_t(col) * P.lddw + P.bias_col, acc[e]);
                }
            }
        }
    } else if (warp >= 4) {
        // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 ----
        const uint32_t quarter = warp & 3;
        if (my > 0 && mbar_wait(acc_full, 0, &abort_flag)) {
            asm volatile("tcgen05.fence::after_thread_sync;");
            const int ncols = 64 * P.b_boxes;
            for (int h = 0; h < P.halves; ++h) {
                const int row = h * kTileM + int(quarter * 32 + lane);
                for (int c0 = 0; c0 < ncols; c0 += 32) {
                    float v[32];
                    tmem_ld32(tmem + ((quarter * 32) << 16) + h * kTileN + c0, v);  // the whole warp
                    if (row < P.m) {
                        float *dst = P.dw + size_t(row) * P.lddw;
#pragma unroll
                        for (int k = 0; k < 32; k += 4)
                            if (c0 + k < P.kcols) red_add_v4f(dst + c0 + k, v[k], v[k + 1], v[k + 2], v[k + 3]);
                    }
                }
            }
        }
    }
    __syncthreads();
    if (abort_flag && threadIdx.x == 0) atomicExch(P.error, 1);
    if (warp == 1) {
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols));
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2-D bf16 map of a row-major [rows, cols] matrix with row stride ld
// elements, box [box_rows, 64 columns], 128-byte swizzle, zero fill.
bool make_map(CUtensorMap *map, const void *base, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
    const cuuint32_t box[2] = {uint32_t(kTileK), box_rows};
    const cuuint32_t elem[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The output map: [rows, cols] bf16 with row stride ld elements, stored in
// 32 x 32 boxes with the 64-byte swizzle (store_box).
bool make_out_map(CUtensorMap *map, void *base, uint32_t rows, uint32_t cols, uint32_t ld) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
    const cuuint32_t box[2] = {32u, 32u};
    const cuuint32_t elem[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

namespace {

template <int MODE>
cudaError_t launch_layer(const CUtensorMap &mx, const CUtensorMap &mw, const CUtensorMap &mo, const LayerParams &P,
                         cudaStream_t stream) {
    static bool attr_set[64] = {};
    static int sm_count[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(layer_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (e != cudaSuccess) return e;
        e = cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    if (P.k_blocks > kMaxKBlocks) return cudaErrorInvalidValue;
    const uint32_t tiles = (P.n + kTileM - 1) / kTileM;
    const uint32_t grid = tiles < uint32_t(sm_count[dev]) ? tiles : uint32_t(sm_count[dev]);
    layer_kernel<MODE><<<grid, kThreads, kSmemBytes, stream>>>(mx, mw, mo, P);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_mlp_layer(const void *x, int ldx, int kx, uint32_t n, const void *w, int ldw, int nw,
                             const void *enc, int ldenc, int enc_cols, int zc, float scale, void *out, int ld,
                             int *error, cudaStream_t stream) {
    return launch_mlp_layer_dot(x, ldx, kx, n, w, ldw, nw, enc, ldenc, enc_cols, zc, scale, out, ld, nullptr,
                                nullptr, 1.0f, error, stream);
}

cudaError_t launch_mlp_layer_dot(const void *x, int ldx, int kx, uint32_t n, const void *w, int ldw, int nw,
                                 const void *enc, int ldenc, int enc_cols, int zc, float scale, void *out, int ld,
                                 const void *wdot, float *zdot, float dot_scale, int *error, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    // columns past 256 of x are the bias column (1) and zeros: the tensor
    // cores take K <= 256 and the epilogue adds W[:, 256]
    const int kmma = kx < kTileN ? kx : kTileN;
    CUtensorMap mx, mw, mo;
    if (!make_map(&mx, x, n, uint32_t(kmma), uint32_t(ldx), kTileM) ||
        !make_map(&mw, w, uint32_t(nw), uint32_t(kmma), uint32_t(ldw), kTileN) ||
        !make_out_map(&mo, out, n, uint32_t(ld), uint32_t(ld)))
        return cudaErrorInvalidValue;
    LayerParams P{};
    P.n = n;
    P.k_blocks = (kmma + kTileK - 1) / kTileK;
    P.wbias = kx > kTileN ? static_cast<const __nv_bfloat16 *>(w) + kTileN : nullptr;
    P.ldw = ldw;
    P.nw = nw;
    P.zc = zc;
    P.enc_cols = enc_cols;
    P.ld = ld;
    P.ldenc = ldenc;
    P.scale = scale;
    P.enc = static_cast<const __nv_bfloat16 *>(enc);
    P.out = static_cast<__nv_bfloat16 *>(out);
    P.error = error;
    P.wdot = static_cast<const __nv_bfloat16 *>(wdot);
    P.zdot = zdot;
    P.dot_scale = dot_scale;
    return launch_layer<kModeForward>(mx, mw, mo, P, stream);
}

cudaError_t launch_mlp_wgrad(const void *dz, int ldz, int m, uint32_t n, const void *act, int lda, int k,
                             float *dw, int lddw, int bias_col, int *error, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    static bool attr_set[64] = {};
    static int sm_count[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(wgrad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kWgSmemBytes);
        if (e != cudaSuccess) return e;
        e = cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    CUtensorMap ma, mb;
    if (!make_map(&ma, dz, n, uint32_t(m), uint32_t(ldz), kWgRows) ||
        !make_map(&mb, act, n, uint32_t(k), uint32_t(lda), kWgRows))
        return cudaErrorInvalidValue;
    WgradParams P{};
    P.n = n;
    P.a_boxes = (m + 63) / 64;
    P.halves = (m + 127) / 128;
    P.b_boxes = (k + 63) / 64;
    P.m = m;
    P.kcols = k;
    P.bias_col = bias_col;
    P.dw = dw;
    P.lddw = lddw;
    P.error = error;
    const uint32_t chunks = (n + kWgRows - 1) / kWgRows;
    const uint32_t grid = chunks < uint32_t(sm_count[dev]) ? chunks : uint32_t(sm_count[dev]);
    wgrad_kernel<<<grid, kWgThreads, kWgSmemBytes, stream>>>(ma, mb, P);
    return cudaGetLastError();
}

cudaError_t launch_mlp_input_grad(const void *dz, int ld, int k, uint32_t n, const void *wt, int ldwt, int nwt,
                                  const void *add, int ldadd, int add_cols, void *out, int ldout, int *error,
                                  cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    CUtensorMap mx, mw, mo;
    if (!make_map(&mx, dz, n, uint32_t(k), uint32_t(ld), kTileM) ||
        !make_map(&mw, wt, uint32_t(nwt), uint32_t(k), uint32_t(ldwt), kTileN) ||
        !make_out_map(&mo, out, n, uint32_t(ldout), uint32_t(ldout)))
        return cudaErrorInvalidValue;
    LayerParams P{};
    P.n = n;
    P.k_blocks = (k + kTileK - 1) / kTileK;
    P.zc = nwt;
    P.ld = ldout;
    P.scale = 1.0f;
    P.out = static_cast<__nv_bfloat16 *>(out);
    P.error = error;
    P.add = static_cast<const __nv_bfloat16 *>(add);
    P.ldadd = ldadd;
    P.add_cols = add ? add_cols : 0;
    return launch_layer<kModeBackward>(mx, mw, mo, P, stream);
}

cudaError_t launch_mlp_layer_tangent(const void *t_in, int ld_in, int k, uint32_t n, const void *w, int ldw, int nw,
                                    const void *act, int ld_act, int cols, float scale, const void *tenc, int ldenc,
                                    int enc_cols, void *out, int ldout, void *zout, int ldzo, int *error,
                                    cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    CUtensorMap mx, mw, mo;
    if (!make_map(&mx, t_in, n, uint32_t(k), uint32_t(ld_in), kTileM) ||
        !make_map(&mw, w, uint32_t(nw), uint32_t(k), uint32_t(ldw), kTileN) ||
        !make_out_map(&mo, out, n, uint32_t(ldout), uint32_t(ldout)))
        return cudaErrorInvalidValue;
    LayerParams P{};
    P.n = n;
    P.k_blocks = (k + kTileK - 1) / kTileK;
    P.zc = cols;
    P.ld = ldout;
    P.scale = scale;
    P.out = static_cast<__nv_bfloat16 *>(out);
    P.error = error;
    P.act = static_cast<const __nv_bfloat16 *>(act);
    P.ld_act = ld_act;
    P.enc = static_cast<const __nv_bfloat16 *>(tenc);
    P.ldenc = ldenc;
    P.enc_cols = tenc ? enc_cols : 0;
    P.zout = static_cast<__nv_bfloat16 *>(zout);
    P.ldzo = ldzo;
    return launch_layer<kModeEikonal>(mx, mw, mo, P, stream);
}

cudaError_t launch_mlp_layer_second(const void *s_next, int ld_next, int k, uint32_t n, const void *wt, int ldwt,
                                    int nwt, const void *act, int ld_act, int cols, float scale, const void *dz,
                                    int lddz, const void *tz, int ldtz, void *out, int ldout, void *skip, int ldskip,
                                    int *error, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    CUtensorMap mx, mw, mo;
    if (!make_map(&mx, s_next, n, uint32_t(k), uint32_t(ld_next), kTileM) ||
        !make_map(&mw, wt, uint32_t(nwt), uint32_t(k), uint32_t(ldwt), kTileN) ||
        !make_out_map(&mo, out, n, uint32_t(ldout), uint32_t(ldout)))
        return cudaErrorInvalidValue;
    LayerParams P{};
    P.n = n;
    P.k_blocks = (k + kTileK - 1) / kTileK;
    P.zc = cols;
    P.ld = ldout;
    P.scale = scale;
    P.out = static_cast<__nv_bfloat16 *>(out);
    P.error = error;
    P.act = static_cast<const __nv_bfloat16 *>(act);
    P.ld_act = ld_act;
    P.skip = static_cast<__nv_bfloat16 *>(skip);
    P.ldskip = ldskip;
    P.inj_dz = static_cast<const __nv_bfloat16 *>(dz);
    P.ld_inj_dz = lddz;
    P.inj_tz = static_cast<const __nv_bfloat16 *>(tz);
    P.ld_inj_tz = ldtz;
    return launch_layer<kModeEikonal>(mx, mw, mo, P, stream);
}

cudaError_t launch_mlp_layer_backward(const void *dz_next, int ld_next, int k, uint32_t n, const void *wt, int ldwt,
                                      int nwt, const void *act, int ld_act, int cols, float scale, void *dz, int ldz,
                                      void *skip, int ldskip, int *error, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    CUtensorMap mx, mw, mo;
    if (!make_map(&mx, dz_next, n, uint32_t(k), uint32_t(ld_next), kTileM) ||
        !make_map(&mw, wt, uint32_t(nwt), uint32_t(k), uint32_t(ldwt), kTileN) ||
        !make_out_map(&mo, dz, n, uint32_t(ldz), uint32_t(ldz)))
        return cudaErrorInvalidValue;
    LayerParams P{};
    P.n = n;
    P.k_blocks = (k + kTileK - 1) / kTileK;
    P.zc = cols;
    P.ld = ldz;
    P.scale = scale;
    P.out = static_cast<__nv_bfloat16 *>(dz);
    P.error = error;
    P.act = static_cast<const __nv_bfloat16 *>(act);
    P.ld_act = ld_act;
    P.skip = static_cast<__nv_bfloat16 *>(skip);
    P.ldskip = ldskip;
    return launch_layer<kModeBackward>(mx, mw, mo, P, stream);
}

}  // namespace sdfoam_b200
