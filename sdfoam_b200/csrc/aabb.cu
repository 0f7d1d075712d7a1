// AABB tree over sorted sites and the nearest-site query that seeds each ray.
//
// Tree layout (the reference's build_aabb_tree, src/aabb_tree/aabb_tree.cu:
// 192-341, and its binding triangulation_bindings.cpp:117-140): a complete
// binary tree stored level by level, leaves first, as [pow2(N)][2][3] floats
// (box min, box max).  Leaf j covers sites 2j and 2j+1, with indices past the
// end clamped to the last site; node j of level L covers leaves
// [j 2^L, (j+1) 2^L).  Boxes are component-wise min / max, so any build order
// gives the same bits.  Here each level is one launch of a streaming kernel.
//
// Query (the reference's nn, aabb_tree.cu:343-415, a warp-cooperative k-NN
// with k = 1): one thread per query walks the tree depth first, nearer child
// first, pruning subtrees whose box is farther than the best site so far.
// Distances are squared Euclidean distances evaluated as
// (dx*dx + dy*dy) + dz*dz without fused multiply-adds; the box distance uses
// the same expression on the per-axis gaps, which never exceed the gaps to a
// site inside the box, so pruning is exact.  Ties go to the lowest site index.
#include <cfloat>

#include "foam_device.cuh"
#include "foam_internal.h"

namespace sdfoam_b200 {

namespace {

__device__ __forceinline__ float dist2(float dx, float dy, float dz) {
    return __fadd_rn(__fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)), __fmul_rn(dz, dz));
}

__global__ void __launch_bounds__(256) aabb_leaves_kernel(const float *__restrict__ points, uint32_t num_points,
                                                          uint32_t num_leaves, float *__restrict__ tree) {
    const uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= num_leaves) return;
    uint32_t a = 2 * j, b = 2 * j + 1;
    if (a >= num_points) a = num_points - 1;
    if (b >= num_points) b = a;
    float lo[3], hi[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float pa = __ldg(points + 3 * size_t(a) + k);
        const float pb = __ldg(points + 3 * size_t(b) + k);
        lo[k] = fminf(pa, pb);
        hi[k] = fmaxf(pa, pb);
    }
    float *out = tree + 6 * size_t(j);
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        out[k] = lo[k];
        out[3 + k] = hi[k];
    }
}

__global__ void __launch_bounds__(256) aabb_level_kernel(const float *__restrict__ below, uint32_t width,
                                                         float *__restrict__ level) {
    const uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= width) return;
    const float *c0 = below + 12 * size_t(j);
    float *out = level + 6 * size_t(j);
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        out[k] = fminf(c0[k], c0[6 + k]);
        out[3 + k] = fmaxf(c0[3 + k], c0[9 + k]);
    }
}

constexpr int kMaxDepth = 40;

__global__ void __launch_bounds__(128) nn_kernel(const float *__restrict__ points, uint32_t num_points,
                                                 const float *__restrict__ tree, uint32_t num_leaves,
                                                 uint32_t levels, const float *__restrict__ queries,
                                                 uint32_t num_queries, uint32_t *__restrict__ indices) {
    const uint32_t qi = blockIdx.x * blockDim.x + threadIdx.x;
    if (qi >= num_queries) return;
    const float qx = __ldg(queries + 3 * size_t(qi) + 0);
    const float qy = __ldg(queries + 3 * size_t(qi) + 1);
    const float qz = __ldg(queries + 3 * size_t(qi) + 2);
    float best = __int_as_float(0x7f800000);
    uint32_t best_i = kNone;
    if (num_leaves == 0) {  // a single site
        indices[qi] = 0;
        return;
    }
    // level offsets: level L starts at sum_{l<L} num_leaves >> l
    // stack of (level, node) packed as level << 27 | node (node < 2^27)
    uint32_t stack[kMaxDepth];
    int sp = 0;
    stack[sp++] = ((levels - 1) << 27) | 0u;
    while (sp > 0) {
        const uint32_t e = stack[--sp];
        const uint32_t L = e >> 27;
        const uint32_t node = e & ((1u << 27) - 1);
        if (L == 0) {
            const uint32_t a = 2 * node;
            for (uint32_t i = a; i < a + 2 && i < num_points; ++i) {
                const float d = dist2(__fsub_rn(qx, __ldg(points + 3 * size_t(i) + 0)),
                                      __fsub_rn(qy, __ldg(points + 3 * size_t(i) + 1)),
                                      __fsub_rn(qz, __ldg(points + 3 * size_t(i) + 2)));
                if (d < best || (d == best && i < best_i)) {
                    best = d;
                    best_i = i;
                }
            }
            continue;
        }
        // children (L-1, 2 node) and (L-1, 2 node + 1)
        uint64_t off = 0;
        for (uint32_t l = 0; l + 1 < L; ++l) off += num_leaves >> l;
        float cd[2];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            const float *box = tree + 6 * (off + 2 * size_t(node) + c);
            const float gx = fmaxf(fmaxf(__fsub_rn(__ldg(box + 0), qx), __fsub_rn(qx, __ldg(box + 3))), 0.0f);
            const float gy = fmaxf(fmaxf(__fsub_rn(__ldg(box + 1), qy), __fsub_rn(qy, __ldg(box + 4))), 0.0f);
            const float gz = fmaxf(fmaxf(__fsub_rn(__ldg(box + 2), qz), __fsub_rn(qz, __ldg(box + 5))), 0.0f);
            cd[c] = dist2(gx, gy, gz);
        }
        // push the farther child first so the nearer one is visited first;
        // a child whose first site (child << L) is past the end holds only
        // padding leaves, whose boxes repeat the last site, and is skipped
        const int nearer = cd[1] < cd[0] ? 1 : 0;
        const int farther = 1 - nearer;
        const bool real[2] = {(uint64_t(2 * node) << L) < num_points, (uint64_t(2 * node + 1) << L) < num_points};
        if (real[farther] && cd[farther] <= best && sp < kMaxDepth) stack[sp++] = ((L - 1) << 27) | (2 * node + farther);
        if (real[nearer] && cd[nearer] <= best && sp < kMaxDepth) stack[sp++] = ((L - 1) << 27) | (2 * node + nearer);
    }
    indices[qi] = best_i;
}

}  // namespace

uint32_t pow2_round_up(uint32_t x) {
    uint32_t p = 1;
    while (p < x) p <<= 1;
    return p;
}

cudaError_t launch_build_aabb_tree(const float *points, uint32_t num_points, float *tree, cudaStream_t stream) {
    if (num_points == 0) return cudaSuccess;
    const uint32_t num_leaves = pow2_round_up(num_points) / 2;
    if (num_leaves == 0) {  // one site: its own box
        cudaError_t e = cudaMemcpyAsync(tree, points, 12, cudaMemcpyDeviceToDevice, stream);
        if (e != cudaSuccess) return e;
        return cudaMemcpyAsync(tree + 3, points, 12, cudaMemcpyDeviceToDevice, stream);
    }
    aabb_leaves_kernel<<<(num_leaves + 255) / 256, 256, 0, stream>>>(points, num_points, num_leaves, tree);
    size_t off = 0;
    uint32_t width = num_leaves;
    while (width > 1) {
        const uint32_t up = width / 2;
        aabb_level_kernel<<<(up + 255) / 256, 256, 0, stream>>>(tree + 6 * off, up, tree + 6 * (off + width));
        off += width;
        width = up;
    }
    return cudaGetLastError();
}

cudaError_t launch_nn(const float *points, uint32_t num_points, const float *tree, const float *queries,
                      uint32_t num_queries, uint32_t *indices, cudaStream_t stream) {
    if (num_queries == 0) return cudaSuccess;
    const uint32_t num_leaves = pow2_round_up(num_points) / 2;
    uint32_t levels = 0;
    for (uint32_t w = num_leaves; w >= 1; w >>= 1) ++levels;
    nn_kernel<<<(num_queries + 127) / 128, 128, 0, stream>>>(points, num_points, tree, num_leaves, levels, queries,
                                                            num_queries, indices);
    return cudaGetLastError();
}

}  // namespace sdfoam_b200
