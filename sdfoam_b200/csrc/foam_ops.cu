// Per-site helpers of the densification step around the tracer.
//
// farthest_neighbor (reference src/delaunay/triangulation_ops.cu:10-44,
// binding triangulation_bindings.cpp:183-217): for each site, the Delaunay
// neighbour at the largest distance (first one in CSR order on ties, none when
// every distance is 0) and the mean half-edge length sum(0.5 |q - p|) / deg.
// |q - p| = sqrt(dx*dx + (dy*dy + dz*dz)) with the first product of each sum
// fused; the reference's `sum += 0.5 * distance` is evaluated in double from
// float operands, which is one float rounding of sum + 0.5 d.  Rows whose
// CSR range is reversed or past the end of the adjacency get no neighbour and
// a NaN radius (the reference would read out of bounds).
#include "foam_device.cuh"
#include "foam_internal.h"

namespace sdfoam_b200 {

namespace {

__global__ void __launch_bounds__(256) farthest_neighbor_kernel(const float *__restrict__ points,
                                                                const uint32_t *__restrict__ adjacency,
                                                                const uint32_t *__restrict__ offsets,
                                                                uint32_t num_points, uint32_t adjacency_size,
                                                                uint32_t *__restrict__ indices,
                                                                float *__restrict__ radius) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= num_points) return;
    const uint32_t beg = __ldg(offsets + i), end = __ldg(offsets + i + 1);
    if (beg > end || end > adjacency_size) {
        indices[i] = kNone;
        radius[i] = __int_as_float(0x7fffffff);
        return;
    }
    const float px = __ldg(points + 3 * size_t(i)), py = __ldg(points + 3 * size_t(i) + 1),
                pz = __ldg(points + 3 * size_t(i) + 2);
    uint32_t best = kNone;
    float best_d = 0.0f, sum = 0.0f;
    for (uint32_t j = beg; j < end; ++j) {
        const uint32_t a = __ldg(adjacency + j);
        if (a >= num_points) continue;
        const float dx = __fsub_rn(__ldg(points + 3 * size_t(a)), px);
        const float dy = __fsub_rn(__ldg(points + 3 * size_t(a) + 1), py);
        const float dz = __fsub_rn(__ldg(points + 3 * size_t(a) + 2), pz);
        const float d = __fsqrt_rn(fmaf(dx, dx, fmaf(dy, dy, __fmul_rn(dz, dz))));
        sum = __fadd_rn(sum, __fmul_rn(0.5f, d));
        if (d > best_d) {
            best_d = d;
            best = a;
        }
    }
    indices[i] = best;
    radius[i] = __fdiv_rn(sum, static_cast<float>(end - beg));
}

}  // namespace

cudaError_t launch_farthest_neighbor(const float *points, const uint32_t *adjacency, const uint32_t *offsets,
                                     uint32_t num_points, uint32_t adjacency_size, uint32_t *indices,
                                     float *radius, cudaStream_t stream) {
    if (num_points == 0) return cudaSuccess;
    farthest_neighbor_kernel<<<(num_points + 255) / 256, 256, 0, stream>>>(points, adjacency, offsets, num_points,
                                                                          adjacency_size, indices, radius);
    return cudaGetLastError();
}

}  // namespace sdfoam_b200
