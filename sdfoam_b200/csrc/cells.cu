// Cell-record builder: the B200 replacement of the reference's per-call
// prefetch_adjacent_diff_kernel (src/tracing/pipeline.cu:1202-1224).
//
// The reference writes half4(q - p, 0) per CSR entry into a fresh buffer
// before every forward and every backward.  Here one build produces, per site,
// a 16-byte head (position + first CSR entry) and, per CSR entry, a 16-byte
// face record holding the neighbour id next to the same binary16 offset, so
// that the walk reads a face's id and plane with one 128-bit load and reaches
// the next site's position and face range with one more.  Attributes are
// repacked into 16-byte aligned rows for 128-bit loads.  The build is HBM-bound
// streaming work (the neighbour positions it gathers fit in L2).
#include "foam_device.cuh"
#include "foam_internal.h"

namespace sdfoam_b200 {

namespace {

constexpr int kFaceLanes = 16;  // half a warp per site: mean degree is ~15

// heads[c] and the face records of site c, half a warp per site.
__global__ void __launch_bounds__(256) build_faces_kernel(const float *__restrict__ points,
                                                          const uint32_t *__restrict__ adjacency,
                                                          const uint32_t *__restrict__ offsets,
                                                          uint32_t num_points, uint32_t adjacency_size,
                                                          float4 *__restrict__ heads,
                                                          uint4 *__restrict__ faces) {
    const uint64_t gtid = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint64_t site64 = gtid / kFaceLanes;
    const uint32_t lane = threadIdx.x % kFaceLanes;
    if (site64 > num_points) return;
    const uint32_t c = static_cast<uint32_t>(site64);
    const uint32_t beg = __ldg(offsets + c);
    if (c == num_points) {
        if (lane == 0) heads[c] = make_float4(0.0f, 0.0f, 0.0f, __uint_as_float(beg));
        return;
    }
    const float px = __ldg(points + 3 * size_t(c) + 0);
    const float py = __ldg(points + 3 * size_t(c) + 1);
    const float pz = __ldg(points + 3 * size_t(c) + 2);
    if (lane == 0) heads[c] = make_float4(px, py, pz, __uint_as_float(beg));
    const uint32_t end = __ldg(offsets + c + 1);
    if (beg > end || end > adjacency_size) return;  // rows the walk never enters
    for (uint32_t j = beg + lane; j < end; j += kFaceLanes) {
        const uint32_t a = __ldg(adjacency + j);
        uint4 rec = make_uint4(kNone, 0u, 0u, 0u);
        if (a < num_points) {
            const float qx = __ldg(points + 3 * size_t(a) + 0);
            const float qy = __ldg(points + 3 * size_t(a) + 1);
            const float qz = __ldg(points + 3 * size_t(a) + 2);
            // diff = q - p in float32, then round-to-nearest-even binary16
            const uint32_t hx = __half_as_ushort(__float2half_rn(__fsub_rn(qx, px)));
            const uint32_t hy = __half_as_ushort(__float2half_rn(__fsub_rn(qy, py)));
            const uint32_t hz = __half_as_ushort(__float2half_rn(__fsub_rn(qz, pz)));
            rec = make_uint4(a, hx | (hy << 16), hz, 0u);
        }
        faces[j] = rec;
    }
}

// Attribute rows repacked to V float4 per site (channels beyond A are zero).
template <int V>
__global__ void __launch_bounds__(256) pack_attrs_kernel(const float *__restrict__ attributes,
                                                         uint32_t num_points, int attr_dim,
                                                         float4 *__restrict__ out) {
    const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= uint64_t(num_points) * V) return;
    const uint64_t c = i / V;
    const int v = static_cast<int>(i % V);
    const float *row = attributes + c * attr_dim;
    float q[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int ch = 4 * v + k;
        q[k] = ch < attr_dim ? __ldg(row + ch) : 0.0f;
    }
    out[i] = make_float4(q[0], q[1], q[2], q[3]);
}

}  // namespace

cudaError_t launch_build_cells(const sdfoam_foam &foam, void *cells, cudaStream_t stream) {
    const CellsLayout L = CellsLayout::make(foam.num_points, foam.adjacency_size, foam.sh_degree);
    char *base = static_cast<char *>(cells);
    float4 *heads = reinterpret_cast<float4 *>(base + L.heads_off);
    uint4 *faces = reinterpret_cast<uint4 *>(base + L.faces_off);
    float4 *attrs = reinterpret_cast<float4 *>(base + L.attrs_off);
    {
        const uint64_t threads = uint64_t(foam.num_points + 1) * kFaceLanes;
        const uint32_t blocks = static_cast<uint32_t>((threads + 255) / 256);
        build_faces_kernel<<<blocks, 256, 0, stream>>>(foam.points, foam.point_adjacency,
                                                       foam.point_adjacency_offsets, foam.num_points,
                                                       foam.adjacency_size, heads, faces);
    }
    if (foam.num_points > 0) {
        const int V = attr_vec4_of(foam.sh_degree);
        const int A = attr_dim_of(foam.sh_degree);
        const uint64_t total = uint64_t(foam.num_points) * V;
        const uint32_t blocks = static_cast<uint32_t>((total + 255) / 256);
        const float *src = static_cast<const float *>(foam.attributes);
        switch (V) {
        case 1: pack_attrs_kernel<1><<<blocks, 256, 0, stream>>>(src, foam.num_points, A, attrs); break;
        case 4: pack_attrs_kernel<4><<<blocks, 256, 0, stream>>>(src, foam.num_points, A, attrs); break;
        case 7: pack_attrs_kernel<7><<<blocks, 256, 0, stream>>>(src, foam.num_points, A, attrs); break;
        case 13: pack_attrs_kernel<13><<<blocks, 256, 0, stream>>>(src, foam.num_points, A, attrs); break;
        default: return cudaErrorInvalidValue;
        }
    }
    return cudaGetLastError();
}

}  // namespace sdfoam_b200
