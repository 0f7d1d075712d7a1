// Cell-record builder: the B200 replacement of the reference's per-call
// prefetch_adjacent_diff_kernel (src/tracing/pipeline.cu:1202-1224).
//
// The reference writes half4(q - p, 0) per CSR entry into a fresh buffer
// before every forward and every backward.  Here one build produces:
//   * per site a 32-byte head (position, CSR range, last attribute channel),
//     read with one 256-bit load when the walk steps into the site;
//   * per CSR entry a 16-byte face record: the neighbour id next to half of
//     the reference's binary16 offset, h = fp16(q - p) / 2, stored as fp32
//     (exact), so the walk needs no conversions and no * 0.5;
//   * the SH coefficients in 32-byte aligned rows for 256-bit loads.
// The build is streaming work (the neighbour positions it gathers fit in L2).
#include "foam_device.cuh"
#include "foam_internal.h"

namespace sdfoam_b200 {

namespace {

constexpr int kFaceLanes = 16;  // half a warp per site: mean degree is ~15

__global__ void __launch_bounds__(256) build_faces_kernel(const float *__restrict__ points,
                                                          const float *__restrict__ attributes, int attr_dim,
                                                          const uint32_t *__restrict__ adjacency,
                                                          const uint32_t *__restrict__ offsets,
                                                          uint32_t num_points, uint32_t adjacency_size,
                                                          uint4 *__restrict__ heads, uint4 *__restrict__ faces) {
    const uint64_t gtid = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint64_t site64 = gtid / kFaceLanes;
    const uint32_t lane = threadIdx.x % kFaceLanes;
    if (site64 >= num_points) return;
    const uint32_t c = static_cast<uint32_t>(site64);
    const uint32_t beg = __ldg(offsets + c);
    const uint32_t end = __ldg(offsets + c + 1);
    const float px = __ldg(points + 3 * size_t(c) + 0);
    const float py = __ldg(points + 3 * size_t(c) + 1);
    const float pz = __ldg(points + 3 * size_t(c) + 2);
    if (lane == 0) {
        const float last = __ldg(attributes + size_t(c) * attr_dim + (attr_dim - 1));
        heads[2 * size_t(c) + 0] = make_uint4(__float_as_uint(px), __float_as_uint(py), __float_as_uint(pz), beg);
        heads[2 * size_t(c) + 1] = make_uint4(end, __float_as_uint(last), 0u, 0u);
    }
    if (beg > end || end > adjacency_size) return;  // rows the walk never enters
    for (uint32_t j = beg + lane; j < end; j += kFaceLanes) {
        const uint32_t a = __ldg(adjacency + j);
        uint4 rec = make_uint4(kNone, 0u, 0u, 0u);
        if (a < num_points) {
            const float qx = __ldg(points + 3 * size_t(a) + 0);
            const float qy = __ldg(points + 3 * size_t(a) + 1);
            const float qz = __ldg(points + 3 * size_t(a) + 2);
            // diff = q - p in float32, round-to-nearest-even binary16, back to
            // float32 (exact), halved (exact)
            const float hx = __fmul_rn(__half2float(__float2half_rn(__fsub_rn(qx, px))), 0.5f);
            const float hy = __fmul_rn(__half2float(__float2half_rn(__fsub_rn(qy, py))), 0.5f);
            const float hz = __fmul_rn(__half2float(__float2half_rn(__fsub_rn(qz, pz))), 0.5f);
            rec = make_uint4(a, __float_as_uint(hx), __float_as_uint(hy), __float_as_uint(hz));
        }
        faces[j] = rec;
    }
}

// SH coefficients (channels 0..A-2) into rows of `stride` floats, zero padded.
__global__ void __launch_bounds__(256) pack_sh_kernel(const float *__restrict__ attributes, uint32_t num_points,
                                                      int attr_dim, int stride, float *__restrict__ out) {
    const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= uint64_t(num_points) * stride) return;
    const uint64_t c = i / stride;
    const int ch = static_cast<int>(i % stride);
    out[i] = ch < attr_dim - 1 ? __ldg(attributes + c * attr_dim + ch) : 0.0f;
}

}  // namespace

cudaError_t launch_build_cells(const sdfoam_foam &foam, void *cells, cudaStream_t stream) {
    if (foam.num_points == 0) return cudaSuccess;
    const CellsLayout L = CellsLayout::make(foam.num_points, foam.adjacency_size, foam.sh_degree);
    char *base = static_cast<char *>(cells);
    uint4 *heads = reinterpret_cast<uint4 *>(base + L.heads_off);
    uint4 *faces = reinterpret_cast<uint4 *>(base + L.faces_off);
    float *sh = reinterpret_cast<float *>(base + L.sh_off);
    const int A = attr_dim_of(foam.sh_degree);
    const float *attrs = static_cast<const float *>(foam.attributes);
    {
        const uint64_t threads = uint64_t(foam.num_points) * kFaceLanes;
        const uint32_t blocks = static_cast<uint32_t>((threads + 255) / 256);
        build_faces_kernel<<<blocks, 256, 0, stream>>>(foam.points, attrs, A, foam.point_adjacency,
                                                       foam.point_adjacency_offsets, foam.num_points,
                                                       foam.adjacency_size, heads, faces);
    }
    {
        const int S = sh_stride_of(foam.sh_degree);
        const uint64_t total = uint64_t(foam.num_points) * S;
        const uint32_t blocks = static_cast<uint32_t>((total + 255) / 256);
        pack_sh_kernel<<<blocks, 256, 0, stream>>>(attrs, foam.num_points, A, S, sh);
    }
    return cudaGetLastError();
}

}  // namespace sdfoam_b200
