// Internal declarations shared by the C-ABI layer and the kernels.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <cuda_runtime.h>

#include "../../include/sdfoam_b200.h"

namespace sdfoam_b200 {

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

inline int attr_dim_of(uint32_t sh_degree) { return 1 + 3 * int((sh_degree + 1) * (sh_degree + 1)); }
inline int attr_vec4_of(uint32_t sh_degree) { return (attr_dim_of(sh_degree) + 3) / 4; }
// SH scalars per site padded to whole 32-byte chunks (8 floats).
inline int sh_stride_of(uint32_t sh_degree) { return (3 * int((sh_degree + 1) * (sh_degree + 1)) + 7) / 8 * 8; }

// Cell-record workspace layout (all sections 256-byte aligned):
//   heads  [N] x 32 B  (p.x, p.y, p.z, first CSR entry, end CSR entry, last
//                       attribute channel, 0, 0) -- one 256-bit load
//   faces  uint4 [E]   (neighbour id, hx, hy, hz): h = fp16(q - p) / 2 as fp32
//   sh     float [N * sh_stride] SH coefficients (channels 0..A-2), zero padded
struct CellsLayout {
    size_t heads_off, faces_off, sh_off, total;
    static CellsLayout make(uint32_t n, uint32_t e, uint32_t sh_degree) {
        CellsLayout L;
        L.heads_off = 0;
        L.faces_off = align_up(L.heads_off + size_t(n) * 32, 256);
        L.sh_off = align_up(L.faces_off + size_t(e) * 16, 256);
        L.total = align_up(L.sh_off + size_t(n) * sh_stride_of(sh_degree) * 4, 256);
        return L;
    }
};

// Gradient workspace layout:
//   attr_acc   float4 [N * V]   per-site attribute gradient rows
//   point_acc  float4 [N]       per-site position gradient (x, y, z, 0)
struct GradLayout {
    size_t attr_off, point_off, total;
    static GradLayout make(uint32_t n, uint32_t sh_degree) {
        GradLayout L;
        L.attr_off = 0;
        L.point_off = align_up(size_t(n) * attr_vec4_of(sh_degree) * 16, 256);
        L.total = align_up(L.point_off + size_t(n) * 16, 256);
        return L;
    }
};

struct CellsView {
    const uint32_t *heads;  // 8 words per site
    const uint4 *faces;
    const float *sh;
    uint32_t num_points;
    uint32_t adjacency_size;
};

struct ForwardParams {
    CellsView cells;
    sdfoam_trace_settings settings;
    uint32_t num_rays;
    const float *rays;
    const uint32_t *start;
    uint32_t num_quantiles;
    const float *quantiles;
    const float *sharpness;
    float *rgba;
    float *depth;
    uint32_t *depth_indices;
    uint32_t *num_intersections;
    float *contribution;
    float *alpha;
    const uint64_t *seq_offsets;
    uint32_t *seq_cells;
    uint32_t *seq_count;
    uint32_t *face_tests;
};

struct BackwardParams {
    CellsView cells;
    sdfoam_trace_settings settings;
    uint32_t num_rays;
    const float *rays;
    const uint32_t *start;
    uint32_t num_quantiles;
    const float *quantiles;
    const uint32_t *depth_indices;
    const float *rgba;
    const float *rgba_grad;
    const float *depth_grad;
    const float *ray_error;
    const float *sharpness;
    float4 *attr_acc;
    float4 *point_acc;
    float *point_error;
    float *sharpness_grad;
};

// Sets the message sdfoam_last_error() returns on this thread.
void set_last_error(const std::string &msg);

cudaError_t launch_build_cells(const sdfoam_foam &foam, void *cells, cudaStream_t stream);
uint32_t pow2_round_up(uint32_t x);
cudaError_t launch_build_aabb_tree(const float *points, uint32_t num_points, float *tree, cudaStream_t stream);
cudaError_t launch_nn(const float *points, uint32_t num_points, const float *tree, const float *queries,
                      uint32_t num_queries, uint32_t *indices, cudaStream_t stream);
cudaError_t launch_forward(uint32_t sh_degree, const ForwardParams &p, cudaStream_t stream);
cudaError_t launch_backward(uint32_t sh_degree, const BackwardParams &p, cudaStream_t stream);
cudaError_t launch_fold_grads(uint32_t sh_degree, uint32_t num_points, const float4 *attr_acc,
                              const float4 *point_acc, float *attr_grad, float *points_grad,
                              cudaStream_t stream);

inline CellsView cells_view(const sdfoam_foam &foam, const void *cells) {
    CellsLayout L = CellsLayout::make(foam.num_points, foam.adjacency_size, foam.sh_degree);
    const char *base = static_cast<const char *>(cells);
    CellsView v;
    v.heads = reinterpret_cast<const uint32_t *>(base + L.heads_off);
    v.faces = reinterpret_cast<const uint4 *>(base + L.faces_off);
    v.sh = reinterpret_cast<const float *>(base + L.sh_off);
    v.num_points = foam.num_points;
    v.adjacency_size = foam.adjacency_size;
    return v;
}

}  // namespace sdfoam_b200
