// extern "C" entry points declared in include/sdfoam_b200.h.
//
// The layer validates arguments (the checks the reference's pybind binding
// performs on tensors, pipeline_bindings.cpp:12-75, 176-210, 399-505, restated
// on raw pointers and sizes), resolves the dispatch table of create_pipeline
// (pipeline.cu:1477-1506: {float32, float16} x SH degree 0..3), and launches
// on the caller's stream.  It allocates nothing.
#include <cstdio>
#include <cstring>
#include <cmath>
#include <string>

#include "foam_internal.h"

using namespace sdfoam_b200;

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string &msg) {
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char *where) {
    return fail(SDFOAM_ERR_CUDA, std::string(where) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

int check_foam(const sdfoam_foam *foam) {
    if (!foam) return fail(SDFOAM_ERR_INVALID, "foam is NULL");
    if (foam->sh_degree > 3) return fail(SDFOAM_ERR_UNSUPPORTED, "Unsupported SH degree");
    if (foam->attr_dtype != SDFOAM_F32 && foam->attr_dtype != SDFOAM_F16)
        return fail(SDFOAM_ERR_UNSUPPORTED, "Unsupported attribute type");
    if (foam->num_points > 0 && (!foam->points || !foam->attributes))
        return fail(SDFOAM_ERR_INVALID, "points and attributes must be non-NULL");
    if (!foam->point_adjacency_offsets) return fail(SDFOAM_ERR_INVALID, "point_adjacency_offsets is NULL");
    if (foam->adjacency_size > 0 && !foam->point_adjacency)
        return fail(SDFOAM_ERR_INVALID, "point_adjacency is NULL");
    if (!CellsLayout::fits(foam->num_points, foam->adjacency_size))
        return fail(SDFOAM_ERR_INVALID, "foam too large: adjacency_size + 3 * num_points must stay below 2^32");
    return SDFOAM_OK;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// [R,4] attribute-typed rows: 16 bytes (float32) or 8 bytes (float16) each.
bool rgba_aligned(const void *p, uint32_t attr_dtype) {
    return (reinterpret_cast<uintptr_t>(p) & (attr_dtype == SDFOAM_F16 ? 7u : 15u)) == 0;
}

int check_settings(const sdfoam_foam *foam, const sdfoam_trace_settings *s) {
    if (!s) return fail(SDFOAM_ERR_INVALID, "settings is NULL");
    if (s->alpha_mode != SDFOAM_ALPHA_STANDARD && s->alpha_mode != SDFOAM_ALPHA_NEUS)
        return fail(SDFOAM_ERR_INVALID, "alpha_mode must be SDFOAM_ALPHA_STANDARD or SDFOAM_ALPHA_NEUS");
    if (s->sdf_channel >= attr_dim_of(foam->sh_degree))
        return fail(SDFOAM_ERR_INVALID, "sdf_channel must be smaller than the attribute dimension " +
                                            std::to_string(attr_dim_of(foam->sh_degree)));
    return SDFOAM_OK;
}

int check_cells(const sdfoam_foam *foam, const void *cells) {
    if (!cells) return fail(SDFOAM_ERR_INVALID, "cells is NULL (build them with sdfoam_build_cells)");
    if (reinterpret_cast<uintptr_t>(cells) & 31u) return fail(SDFOAM_ERR_INVALID, "cells must be 32-byte aligned");
    (void)foam;
    return SDFOAM_OK;
}

}  // namespace

void sdfoam_b200::set_last_error(const std::string &msg) { g_last_error = msg; }

extern "C" {

size_t sdfoam_cells_bytes(uint32_t num_points, uint32_t adjacency_size, uint32_t sh_degree) {
    if (sh_degree > 3 || !CellsLayout::fits(num_points, adjacency_size)) return 0;
    return CellsLayout::make(num_points, adjacency_size, sh_degree).total;
}

int sdfoam_build_cells(const sdfoam_foam *foam, void *cells, size_t cells_bytes, sdfoam_stream_t stream) {
    if (int rc = check_foam(foam)) return rc;
    if (int rc = check_cells(foam, cells)) return rc;
    const size_t need = sdfoam_cells_bytes(foam->num_points, foam->adjacency_size, foam->sh_degree);
    if (cells_bytes < need)
        return fail(SDFOAM_ERR_INVALID, "cells workspace too small: " + std::to_string(cells_bytes) + " < " +
                                            std::to_string(need));
    cudaError_t e = launch_build_cells(*foam, nullptr, cells, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "sdfoam_build_cells");
    return SDFOAM_OK;
}

int sdfoam_build_cells_from_diffs(const sdfoam_foam *foam, const void *adjacent_diff, void *cells,
                                  size_t cells_bytes, sdfoam_stream_t stream) {
    if (int rc = check_foam(foam)) return rc;
    if (int rc = check_cells(foam, cells)) return rc;
    if (foam->adjacency_size > 0 && (!adjacent_diff || (reinterpret_cast<uintptr_t>(adjacent_diff) & 7u)))
        return fail(SDFOAM_ERR_INVALID, "adjacent_diff must be non-NULL and 8-byte aligned");
    const size_t need = sdfoam_cells_bytes(foam->num_points, foam->adjacency_size, foam->sh_degree);
    if (cells_bytes < need)
        return fail(SDFOAM_ERR_INVALID, "cells workspace too small: " + std::to_string(cells_bytes) + " < " +
                                            std::to_string(need));
    cudaError_t e = launch_build_cells(*foam, adjacent_diff, cells, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "sdfoam_build_cells_from_diffs");
    return SDFOAM_OK;
}

int sdfoam_trace_benchmark(const sdfoam_foam *foam, const void *cells, const sdfoam_trace_settings *settings,
                           const sdfoam_camera *camera, const uint32_t *start_point, const float *sharpness,
                           const float *bg_color, int checker_bg, uint32_t *output_rgba, sdfoam_stream_t stream) {
    if (int rc = check_foam(foam)) return rc;
    if (int rc = check_cells(foam, cells)) return rc;
    if (int rc = check_settings(foam, settings)) return rc;
    if (!camera) return fail(SDFOAM_ERR_INVALID, "camera is NULL");
    if (camera->model != SDFOAM_PINHOLE && camera->model != SDFOAM_FISHEYE)
        return fail(SDFOAM_ERR_INVALID, "Invalid camera model");
    if (camera->width == 0 || camera->height == 0) return SDFOAM_OK;
    if (uint64_t(camera->width) * camera->height > 0xffffffffull)
        return fail(SDFOAM_ERR_INVALID, "too many pixels");
    if (!start_point || !output_rgba) return fail(SDFOAM_ERR_INVALID, "start_point and output_rgba must be non-NULL");
    if (settings->alpha_mode == SDFOAM_ALPHA_NEUS && !sharpness)
        return fail(SDFOAM_ERR_INVALID, "sharpness must be non-NULL in NeuS mode");
    RenderParams p{};
    p.cells = cells_view(*foam, cells);
    p.settings = *settings;
    p.sharpness = sharpness;
    p.start = start_point;
    for (int k = 0; k < 3; ++k) {
        p.position[k] = camera->position[k];
        p.forward[k] = camera->forward[k];
        p.right[k] = camera->right[k];
        p.up[k] = camera->up[k];
        p.bg[k] = bg_color ? bg_color[k] : 1.0f;
    }
    p.fov = camera->fov;
    // cast_ray's per-frame constants (camera.h:59, 67), once on the host
    p.focal = 1.0f / std::tan(camera->fov * 0.5f);
    p.aspect = static_cast<float>(camera->width) / static_cast<float>(camera->height);
    p.width = camera->width;
    p.height = camera->height;
    p.model = camera->model;
    p.checker = checker_bg ? 1u : 0u;
    p.rgba8 = output_rgba;
    cudaError_t e = launch_render(foam->sh_degree, foam->attr_dtype, p, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "sdfoam_trace_benchmark");
    return SDFOAM_OK;
}

int sdfoam_trace_forward(const sdfoam_foam *foam, const void *cells, const sdfoam_trace_settings *settings,
                         const sdfoam_forward_io *io, sdfoam_stream_t stream) {
    if (int rc = check_foam(foam)) return rc;
    if (int rc = check_cells(foam, cells)) return rc;
    if (int rc = check_settings(foam, settings)) return rc;
    if (!io) return fail(SDFOAM_ERR_INVALID, "io is NULL");
    if (io->num_rays > 0) {
        if (!io->rays || !io->start_point) return fail(SDFOAM_ERR_INVALID, "rays and start_point must be non-NULL");
        if (!io->ray_rgba || !rgba_aligned(io->ray_rgba, foam->attr_dtype))
            return fail(SDFOAM_ERR_INVALID, "ray_rgba must be non-NULL and aligned to one rgba row");
        if (settings->alpha_mode == SDFOAM_ALPHA_NEUS && !io->sharpness)
            return fail(SDFOAM_ERR_INVALID, "sharpness must be non-NULL in NeuS mode");
        if (io->depth_quantiles && io->num_depth_quantiles > 0 && (!io->depth || !io->depth_indices))
            return fail(SDFOAM_ERR_INVALID, "depth and depth_indices are required with depth_quantiles");
        if (io->seq_cells && !io->seq_offsets) return fail(SDFOAM_ERR_INVALID, "seq_cells needs seq_offsets");
    }
    ForwardParams p{};
    p.cells = cells_view(*foam, cells);
    p.settings = *settings;
    p.num_rays = io->num_rays;
    p.rays = io->rays;
    p.start = io->start_point;
    p.num_quantiles = io->depth_quantiles ? io->num_depth_quantiles : 0;
    p.quantiles = p.num_quantiles ? io->depth_quantiles : nullptr;
    p.sharpness = io->sharpness;
    p.rgba = io->ray_rgba;
    p.depth = io->depth;
    p.depth_indices = io->depth_indices;
    p.num_intersections = io->num_intersections;
    p.contribution = io->point_contribution;
    p.alpha = io->alpha;
    p.seq_offsets = io->seq_offsets;
    p.seq_cells = io->seq_cells;
    p.seq_count = io->seq_count;
    p.face_tests = io->face_tests;
    if (io->exits && io->num_rays > 0) {
        if (io->exits_stride == 0 || io->exits_stride % 8 || (reinterpret_cast<uintptr_t>(io->exits) & 7u))
            return fail(SDFOAM_ERR_INVALID, "exits needs a stride that is a multiple of 8 and 8-byte alignment");
        p.exits = io->exits;
        p.exits_stride = io->exits_stride;
    }
    if (io->step_colors && io->num_rays > 0) {
        if (io->step_colors_steps == 0 || (reinterpret_cast<uintptr_t>(io->step_colors) & 15u))
            return fail(SDFOAM_ERR_INVALID, "step_colors needs at least one step and 16-byte alignment");
        p.colors = reinterpret_cast<float4 *>(io->step_colors);
        p.colors_steps = io->step_colors_steps;
        p.sites = io->step_sites;
    }
    cudaError_t e = launch_forward(foam->sh_degree, foam->attr_dtype, p, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "sdfoam_trace_forward");
    return SDFOAM_OK;
}

size_t sdfoam_backward_workspace_bytes(uint32_t num_points, uint32_t sh_degree) {
    if (sh_degree > 3) return 0;
    return GradLayout::make(num_points, sh_degree).total;
}

int sdfoam_trace_backward(const sdfoam_foam *foam, const void *cells, const sdfoam_trace_settings *settings,
                          const sdfoam_backward_io *io, sdfoam_stream_t stream) {
    if (int rc = check_foam(foam)) return rc;
    if (int rc = check_cells(foam, cells)) return rc;
    if (int rc = check_settings(foam, settings)) return rc;
    if (!io) return fail(SDFOAM_ERR_INVALID, "io is NULL");
    const size_t need = sdfoam_backward_workspace_bytes(foam->num_points, foam->sh_degree);
    if (!io->workspace || !aligned16(io->workspace) || io->workspace_bytes < need)
        return fail(SDFOAM_ERR_INVALID, "backward workspace must be 16-byte aligned and at least " +
                                            std::to_string(need) + " bytes");
    if (foam->num_points > 0 && (!io->points_grad || !io->attr_grad))
        return fail(SDFOAM_ERR_INVALID, "points_grad and attr_grad must be non-NULL");
    const bool quant = io->depth_quantiles && io->num_depth_quantiles > 0;
    if (io->num_rays > 0) {
        if (!io->rays || !io->start_point) return fail(SDFOAM_ERR_INVALID, "rays and start_point must be non-NULL");
        if (!io->ray_rgba || !io->ray_rgba_grad || !rgba_aligned(io->ray_rgba, foam->attr_dtype) ||
            !rgba_aligned(io->ray_rgba_grad, foam->attr_dtype))
            return fail(SDFOAM_ERR_INVALID, "rgb_out and grad_in must be non-NULL and aligned to one rgba row");
        if (settings->alpha_mode == SDFOAM_ALPHA_NEUS && !io->sharpness)
            return fail(SDFOAM_ERR_INVALID, "sharpness must be non-NULL in NeuS mode");
        if (quant && !io->depth_grad)
            return fail(SDFOAM_ERR_INVALID, "depth_grad must be provided if depth_quantiles is provided");
        if (quant && !io->depth_indices)
            return fail(SDFOAM_ERR_INVALID, "depth_indices must be provided if depth_quantiles is provided");
        if (io->ray_error && !io->point_error)
            return fail(SDFOAM_ERR_INVALID, "point_error must be non-NULL when ray_error is given");
    }
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const GradLayout G = GradLayout::make(foam->num_points, foam->sh_degree);
    char *ws = static_cast<char *>(io->workspace);
    float4 *attr_acc = reinterpret_cast<float4 *>(ws + G.attr_off);
    float4 *point_acc = reinterpret_cast<float4 *>(ws + G.point_off);
    cudaError_t e = cudaMemsetAsync(ws, 0, G.total, s);
    if (e != cudaSuccess) return cuda_fail(e, "sdfoam_trace_backward (workspace clear)");
    BackwardParams p{};
    p.cells = cells_view(*foam, cells);
    p.settings = *settings;
    p.num_rays = io->num_rays;
    p.rays = io->rays;
    p.start = io->start_point;
    p.num_quantiles = quant ? io->num_depth_quantiles : 0;
    p.quantiles = quant ? io->depth_quantiles : nullptr;
    p.depth_indices = quant ? io->depth_indices : nullptr;
    p.rgba = io->ray_rgba;
    p.rgba_grad = io->ray_rgba_grad;
    p.depth_grad = quant ? io->depth_grad : nullptr;
    p.ray_error = io->ray_error;
    p.sharpness = io->sharpness;
    p.attr_acc = attr_acc;
    p.point_acc = point_acc;
    p.point_error = io->ray_error ? io->point_error : nullptr;
    p.sharpness_grad = io->sharpness_grad;
    if (io->exits && io->num_rays > 0) {
        if (io->exits_stride == 0 || io->exits_stride % 8 || (reinterpret_cast<uintptr_t>(io->exits) & 7u))
            return fail(SDFOAM_ERR_INVALID, "exits needs a stride that is a multiple of 8 and 8-byte alignment");
        p.exits = io->exits;
        p.exits_stride = io->exits_stride;
    }
    if (io->step_colors && io->num_rays > 0) {
        if (io->step_colors_steps == 0 || (reinterpret_cast<uintptr_t>(io->step_colors) & 15u))
            return fail(SDFOAM_ERR_INVALID, "step_colors needs at least one step and 16-byte alignment");
        p.colors = reinterpret_cast<const float4 *>(io->step_colors);
        p.colors_steps = io->step_colors_steps;
        p.sites = io->step_sites;
    }
    e = launch_backward(foam->sh_degree, foam->attr_dtype, p, s);
    if (e != cudaSuccess) return cuda_fail(e, "sdfoam_trace_backward");
    e = launch_fold_grads(foam->sh_degree, foam->attr_dtype, foam->num_points, attr_acc, point_acc, io->attr_grad,
                          io->points_grad, s);
    if (e != cudaSuccess) return cuda_fail(e, "sdfoam_trace_backward (fold)");
    return SDFOAM_OK;
}

uint32_t sdfoam_aabb_tree_nodes(uint32_t num_points) { return num_points ? pow2_round_up(num_points) : 0; }

int sdfoam_build_aabb_tree(const float *points, uint32_t num_points, float *tree, sdfoam_stream_t stream) {
    if (num_points > 0 && (!points || !tree)) return fail(SDFOAM_ERR_INVALID, "points and tree must be non-NULL");
    if (num_points > (1u << 31)) return fail(SDFOAM_ERR_INVALID, "too many points");
    cudaError_t e = launch_build_aabb_tree(points, num_points, tree, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "sdfoam_build_aabb_tree");
    return SDFOAM_OK;
}

int sdfoam_nn(const float *points, uint32_t num_points, const float *tree, const float *queries,
              uint32_t num_queries, uint32_t *indices, sdfoam_stream_t stream) {
    if (num_points == 0) return fail(SDFOAM_ERR_INVALID, "number of points must be at least 1");
    if (num_points > (1u << 27)) return fail(SDFOAM_ERR_INVALID, "too many points for the tree query");
    if (!points || !tree || (num_queries > 0 && (!queries || !indices)))
        return fail(SDFOAM_ERR_INVALID, "points, tree, queries and indices must be non-NULL");
    cudaError_t e = launch_nn(points, num_points, tree, queries, num_queries, indices,
                              reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "sdfoam_nn");
    return SDFOAM_OK;
}

int sdfoam_farthest_neighbor(const float *points, const uint32_t *point_adjacency,
                             const uint32_t *point_adjacency_offsets, uint32_t num_points, uint32_t adjacency_size,
                             uint32_t *indices, float *cell_radius, sdfoam_stream_t stream) {
    if (num_points > 0 && (!points || !point_adjacency_offsets || !indices || !cell_radius ||
                           (adjacency_size > 0 && !point_adjacency)))
        return fail(SDFOAM_ERR_INVALID, "points, adjacency, offsets and outputs must be non-NULL");
    cudaError_t e = launch_farthest_neighbor(points, point_adjacency, point_adjacency_offsets, num_points,
                                             adjacency_size, indices, cell_radius,
                                             reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "sdfoam_farthest_neighbor");
    return SDFOAM_OK;
}

size_t sdfoam_sort_points_workspace_bytes(uint32_t num_points) {
    return num_points && num_points <= (1u << 31) ? sort_layout(num_points).total : 0;
}

int sdfoam_sort_points(const float *points, uint32_t num_points, float *sorted_points, uint32_t *permutation,
                       void *workspace, size_t workspace_bytes, sdfoam_stream_t stream) {
    if (num_points == 0) return SDFOAM_OK;
    if (num_points > (1u << 31)) return fail(SDFOAM_ERR_INVALID, "too many points");
    if (!points || !sorted_points || !permutation)
        return fail(SDFOAM_ERR_INVALID, "points, sorted_points and permutation must be non-NULL");
    const uintptr_t a = reinterpret_cast<uintptr_t>(points), b = reinterpret_cast<uintptr_t>(sorted_points);
    const uintptr_t bytes = uintptr_t(num_points) * 12;
    if (a < b + bytes && b < a + bytes) return fail(SDFOAM_ERR_INVALID, "sorted_points must not overlap points");
    const size_t need = sort_layout(num_points).total;
    if (!workspace || !aligned16(workspace) || workspace_bytes < need)
        return fail(SDFOAM_ERR_INVALID, "sort workspace must be 16-byte aligned and at least " +
                                            std::to_string(need) + " bytes");
    cudaError_t e = launch_sort_points(points, num_points, sorted_points, permutation, workspace,
                                       reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SDFOAM_OK : cuda_fail(e, "sdfoam_sort_points");
}

size_t sdfoam_delaunay_workspace_bytes(uint32_t num_points) {
    return num_points >= 32 && num_points <= (1u << 27) ? delaunay_layout(num_points).total : 0;
}

int sdfoam_delaunay_neighbors(const float *points, uint32_t num_points, const float *tree, void *workspace,
                              size_t workspace_bytes, uint32_t *point_adjacency_offsets, sdfoam_stream_t stream) {
    if (num_points < 32) return fail(SDFOAM_ERR_INVALID, "Delaunay triangulation does not support less than 32 points");
    if (num_points > (1u << 27)) return fail(SDFOAM_ERR_INVALID, "too many points");
    if (!points || !tree || !point_adjacency_offsets)
        return fail(SDFOAM_ERR_INVALID, "points, tree and point_adjacency_offsets must be non-NULL");
    const size_t need = delaunay_layout(num_points).total;
    if (!workspace || !aligned16(workspace) || workspace_bytes < need)
        return fail(SDFOAM_ERR_INVALID, "Delaunay workspace must be 16-byte aligned and at least " +
                                            std::to_string(need) + " bytes");
    const char *stage = "launch";
    cudaError_t e = launch_delaunay_neighbors(points, num_points, tree, workspace, point_adjacency_offsets,
                                              reinterpret_cast<cudaStream_t>(stream), &stage);
    return e == cudaSuccess ? SDFOAM_OK : cuda_fail(e, (std::string("sdfoam_delaunay_neighbors (") + stage + ")").c_str());
}

int sdfoam_delaunay_status(const void *workspace, uint32_t num_points, uint32_t *status, sdfoam_stream_t stream) {
    if (num_points < 32 || !workspace || !status) return fail(SDFOAM_ERR_INVALID, "bad arguments");
    const char *ws = static_cast<const char *>(workspace) + delaunay_layout(num_points).status;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(status, ws, 6 * sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return e == cudaSuccess ? SDFOAM_OK : cuda_fail(e, "sdfoam_delaunay_status");
}

int sdfoam_delaunay_adjacency(const void *workspace, uint32_t num_points, uint32_t *point_adjacency,
                              uint32_t adjacency_size, sdfoam_stream_t stream) {
    if (num_points < 32 || !workspace) return fail(SDFOAM_ERR_INVALID, "bad arguments");
    if (adjacency_size > 0 && !point_adjacency) return fail(SDFOAM_ERR_INVALID, "point_adjacency must be non-NULL");
    cudaError_t e = launch_delaunay_adjacency(workspace, num_points, point_adjacency, adjacency_size,
                                              reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SDFOAM_OK : cuda_fail(e, "sdfoam_delaunay_adjacency");
}

size_t sdfoam_delaunay_tets_workspace_bytes(uint32_t num_points, uint32_t num_tets) {
    return num_points >= 32 && num_points <= (1u << 27) && num_tets <= (1u << 30)
               ? tets_workspace_bytes(num_points, num_tets)
               : 0;
}

static int check_tets_args(const float *points, uint32_t n, const uint32_t *adjacency, uint32_t adjacency_size,
                           const uint32_t *offsets, const void *workspace, size_t workspace_bytes, uint32_t num_tets,
                           const uint32_t *status) {
    if (n < 32 || n > (1u << 27)) return fail(SDFOAM_ERR_INVALID, "Delaunay triangulation needs 32 to 2^27 points");
    if (!points || !offsets || !status || (adjacency_size > 0 && !adjacency))
        return fail(SDFOAM_ERR_INVALID, "points, offsets, status (and adjacency) must be non-NULL");
    const size_t need = sdfoam_delaunay_tets_workspace_bytes(n, num_tets);
    if (!workspace || !aligned16(workspace) || need == 0 || workspace_bytes < need)
        return fail(SDFOAM_ERR_INVALID, "workspace too small or unaligned");
    return SDFOAM_OK;
}

int sdfoam_delaunay_tets_count(const float *points, uint32_t num_points, const uint32_t *point_adjacency,
                               uint32_t adjacency_size, const uint32_t *point_adjacency_offsets, void *workspace,
                               size_t workspace_bytes, uint32_t *num_tets, uint32_t *status, sdfoam_stream_t stream) {
    int rc = check_tets_args(points, num_points, point_adjacency, adjacency_size, point_adjacency_offsets, workspace,
                             workspace_bytes, 0, status);
    if (rc != SDFOAM_OK) return rc;
    if (!num_tets) return fail(SDFOAM_ERR_INVALID, "num_tets must be non-NULL");
    cudaError_t e = launch_tets_count(points, num_points, point_adjacency, adjacency_size, point_adjacency_offsets,
                                      workspace, num_tets, status, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SDFOAM_OK : cuda_fail(e, "sdfoam_delaunay_tets_count");
}

int sdfoam_delaunay_tets(const float *points, uint32_t num_points, const uint32_t *point_adjacency,
                         uint32_t adjacency_size, const uint32_t *point_adjacency_offsets, void *workspace,
                         size_t workspace_bytes, uint32_t num_tets, uint32_t *tets, uint32_t *tet_adjacency,
                         uint32_t *vert_to_tet, uint32_t *status, sdfoam_stream_t stream) {
    int rc = check_tets_args(points, num_points, point_adjacency, adjacency_size, point_adjacency_offsets, workspace,
                             workspace_bytes, num_tets, status);
    if (rc != SDFOAM_OK) return rc;
    if (!vert_to_tet || (num_tets > 0 && (!tets || !tet_adjacency)))
        return fail(SDFOAM_ERR_INVALID, "tets, tet_adjacency and vert_to_tet must be non-NULL");
    if (!aligned16(tets)) return fail(SDFOAM_ERR_INVALID, "tets must be 16-byte aligned");
    bool mismatch = false;
    cudaError_t e = launch_tets(points, num_points, point_adjacency, adjacency_size, point_adjacency_offsets,
                                workspace, num_tets, tets, tet_adjacency, vert_to_tet, status, &mismatch,
                                reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "sdfoam_delaunay_tets");
    return mismatch ? fail(SDFOAM_ERR_INVALID, "num_tets is not the triangulation's tet count") : SDFOAM_OK;
}

int sdfoam_mlp_layer(const void *x, int ldx, int kx, uint32_t n, const void *w, int ldw, int nw, const void *enc,
                     int ldenc, int enc_cols, int zc, float scale, void *out, int ld, int *error,
                     sdfoam_stream_t stream) {
    if (n > 0 && (!x || !w || !out || !error || (enc_cols > 0 && !enc)))
        return fail(SDFOAM_ERR_INVALID, "x, w, out, error (and enc) must be non-NULL");
    if (kx <= 0 || kx > 320 || kx > ldx || kx > ldw || nw <= 0 || nw > 256 || zc < 0 || zc > 256 || enc_cols < 0 ||
        zc + enc_cols + 1 > ld || (enc_cols > 0 && enc_cols > ldenc))
        return fail(SDFOAM_ERR_INVALID, "inconsistent layer shapes");
    if (ldx % 8 || ldw % 8 || ld % 8 || !aligned16(x) || !aligned16(w) || !aligned16(out))
        return fail(SDFOAM_ERR_INVALID, "rows must be multiples of 8 and 16-byte aligned");
    cudaError_t e = launch_mlp_layer(x, ldx, kx, n, w, ldw, nw, enc, ldenc, enc_cols, zc, scale, out, ld, error,
                                     reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SDFOAM_OK : cuda_fail(e, "sdfoam_mlp_layer");
}

int sdfoam_mlp_layer_backward(const void *dz_next, int ld_next, int k, uint32_t n, const void *wt, int ldwt, int nwt,
                              const void *act, int ld_act, int cols, float scale, void *dz, int ldz, void *skip,
                              int ldskip, int *error, sdfoam_stream_t stream) {
    if (n > 0 && (!dz_next || !wt || !act || !dz || !error))
        return fail(SDFOAM_ERR_INVALID, "dz_next, wt, act, dz and error must be non-NULL");
    if (k <= 0 || k > 256 || k > ld_next || k > ldwt || nwt <= 0 || nwt > 256 || cols < 0 || cols > 256 || cols > ldz ||
        cols > ld_act || !(scale > 0.0f) || (cols < 256 && skip && ldskip < 256 - cols))
        return fail(SDFOAM_ERR_INVALID, "inconsistent layer shapes");
    if (ld_next % 8 || ldwt % 8 || ld_act % 8 || ldz % 8 || !aligned16(dz_next) || !aligned16(wt) ||
        !aligned16(act) || !aligned16(dz))
        return fail(SDFOAM_ERR_INVALID, "rows must be multiples of 8 and 16-byte aligned");
    cudaError_t e = launch_mlp_layer_backward(dz_next, ld_next, k, n, wt, ldwt, nwt, act, ld_act, cols, scale, dz,
                                              ldz, skip, ldskip, error, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SDFOAM_OK : cuda_fail(e, "sdfoam_mlp_layer_backward");
}

int sdfoam_mlp_layer_dot(const void *x, int ldx, int kx, uint32_t n, const void *w, int ldw, int nw,
                         const void *enc, int ldenc, int enc_cols, int zc, float scale, void *out, int ld,
                         const void *wdot, float *zdot, float dot_scale, int *error, sdfoam_stream_t stream) {
    if (n > 0 && (!x || !w || !out || !error || !wdot || !zdot || (enc_cols > 0 && !enc)))
        return fail(SDFOAM_ERR_INVALID, "x, w, out, wdot, zdot, error (and enc) must be non-NULL");
    if (zc != 256 || enc_cols != 0)
        return fail(SDFOAM_ERR_INVALID, "the output dot needs 256 softplus columns and no skip columns");
    if (kx <= 0 || kx > 320 || kx > ldx || kx > ldw || nw <= 0 || nw > 256 || zc < 0 || zc > 256 || enc_cols < 0 ||
        zc + enc_cols + 1 > ld || (enc_cols > 0 && enc_cols > ldenc))
        return fail(SDFOAM_ERR_INVALID, "inconsistent layer shapes");
    if (ldx % 8 || ldw % 8 || ld % 8 || !aligned16(x) || !aligned16(w) || !aligned16(out))
        return fail(SDFOAM_ERR_INVALID, "rows must be multiples of 8 and 16-byte aligned");
    cudaError_t e = launch_mlp_layer_dot(x, ldx, kx, n, w, ldw, nw, enc, ldenc, enc_cols, zc, scale, out, ld, wdot,
                                         zdot, dot_scale, error, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SDFOAM_OK : cuda_fail(e, "sdfoam_mlp_layer_dot");
}

int sdfoam_mlp_wgrad(const void *dz, int ldz, int m, uint32_t n, const void *act, int lda, int k, float *dw,
                     int lddw, int bias_col, int *error, sdfoam_stream_t stream) {
    if (n > 0 && (!dz || !act || !dw || !error))
        return fail(SDFOAM_ERR_INVALID, "dz, act, dw and error must be non-NULL");
    if (m <= 0 || m > 256 || m > ldz || k <= 0 || k > 256 || k > lda || k % 4 || k > lddw || lddw % 4 ||
        bias_col >= lddw || (bias_col >= 0 && bias_col < k))
        return fail(SDFOAM_ERR_INVALID, "inconsistent weight-gradient shapes");
    if (ldz % 8 || lda % 8 || !aligned16(dz) || !aligned16(act) || !aligned16(dw))
        return fail(SDFOAM_ERR_INVALID, "rows must be multiples of 8 and 16-byte aligned");
    cudaError_t e = launch_mlp_wgrad(dz, ldz, m, n, act, lda, k, dw, lddw, bias_col, error,
                                     reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SDFOAM_OK : cuda_fail(e, "sdfoam_mlp_wgrad");
}

int sdfoam_mlp_input_grad(const void *dz, int ld, int k, uint32_t n, const void *wt, int ldwt, int nwt,
                          const void *add, int ldadd, int add_cols, void *out, int ldout, int *error,
                          sdfoam_stream_t stream) {
    if (n > 0 && (!dz || !wt || !out || !error || (add_cols > 0 && !add)))
        return fail(SDFOAM_ERR_INVALID, "dz, wt, out, error (and add) must be non-NULL");
    if (k <= 0 || k > 256 || k > ld || k > ldwt || nwt <= 0 || nwt > 256 || nwt > ldout || add_cols < 0 ||
        (add_cols > 0 && (add_cols > ldadd || add_cols > ldout)))
        return fail(SDFOAM_ERR_INVALID, "inconsistent input-gradient shapes");
    if (ld % 8 || ldwt % 8 || ldout % 8 || (add_cols > 0 && ldadd % 8) || !aligned16(dz) || !aligned16(wt) ||
        !aligned16(out))
        return fail(SDFOAM_ERR_INVALID, "rows must be multiples of 8 and 16-byte aligned");
    cudaError_t e = launch_mlp_input_grad(dz, ld, k, n, wt, ldwt, nwt, add, ldadd, add_cols, out, ldout, error,
                                          reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SDFOAM_OK : cuda_fail(e, "sdfoam_mlp_input_grad");
}

int sdfoam_mlp_layer_tangent(const void *t_in, int ld_in, int k, uint32_t n, const void *w, int ldw, int nw,
                             const void *act, int ld_act, int cols, float scale, const void *tenc, int ldenc,
                             int enc_cols, void *out, int ldout, void *zout, int ldzo, int *error,
                             sdfoam_stream_t stream) {
    if (n > 0 && (!t_in || !w || !act || !out || !zout || !error || (enc_cols > 0 && !tenc)))
        return fail(SDFOAM_ERR_INVALID, "t_in, w, act, out, zout, error (and tenc) must be non-NULL");
    if (k <= 0 || k > 256 || k > ld_in || k > ldw || nw <= 0 || nw > 256 || cols < 0 || cols > nw ||
        cols > ld_act || enc_cols < 0 || cols + enc_cols > ldout || (enc_cols > 0 && enc_cols > ldenc) ||
        ldzo < cols || ldout > 256 || !(scale > 0.0f))
        return fail(SDFOAM_ERR_INVALID, "inconsistent tangent-layer shapes");
    if (ld_in % 8 || ldw % 8 || ld_act % 8 || ldout % 8 || ldzo % 8 || !aligned16(t_in) || !aligned16(w) ||
        !aligned16(act) || !aligned16(out) || !aligned16(zout))
        return fail(SDFOAM_ERR_INVALID, "rows must be multiples of 8 and 16-byte aligned");
    cudaError_t e = launch_mlp_layer_tangent(t_in, ld_in, k, n, w, ldw, nw, act, ld_act, cols, scale, tenc, ldenc,
                                             enc_cols, out, ldout, zout, ldzo, error,
                                             reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SDFOAM_OK : cuda_fail(e, "sdfoam_mlp_layer_tangent");
}

int sdfoam_mlp_layer_second(const void *s_next, int ld_next, int k, uint32_t n, const void *wt, int ldwt, int nwt,
                            const void *act, int ld_act, int cols, float scale, const void *dz, int lddz,
                            const void *tz, int ldtz, void *out, int ldout, void *skip, int ldskip, int *error,
                            sdfoam_stream_t stream) {
    if (n > 0 && (!s_next || !wt || !act || !dz || !tz || !out || !error))
        return fail(SDFOAM_ERR_INVALID, "s_next, wt, act, dz, tz, out and error must be non-NULL");
    if (k <= 0 || k > 256 || k > ld_next || k > ldwt || nwt <= 0 || nwt > 256 || cols < 0 || cols > 256 ||
        cols > ldout || cols > ld_act || cols > lddz || cols > ldtz || !(scale > 0.0f) ||
        (cols < 256 && skip && ldskip < 256 - cols))
        return fail(SDFOAM_ERR_INVALID, "inconsistent second-sweep shapes");
    if (ld_next % 8 || ldwt % 8 || ld_act % 8 || ldout % 8 || !aligned16(s_next) || !aligned16(wt) ||
        !aligned16(act) || !aligned16(out))
        return fail(SDFOAM_ERR_INVALID, "rows must be multiples of 8 and 16-byte aligned");
    cudaError_t e = launch_mlp_layer_second(s_next, ld_next, k, n, wt, ldwt, nwt, act, ld_act, cols, scale, dz, lddz,
                                            tz, ldtz, out, ldout, skip, ldskip, error,
                                            reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SDFOAM_OK : cuda_fail(e, "sdfoam_mlp_layer_second");
}

int sdfoam_mlp_encode_jvp(const float *points, const float *center, uint32_t n, int multires, const float *gbar,
                          int ld, void *out, sdfoam_stream_t stream) {
    if (n > 0 && (!points || !gbar || !out)) return fail(SDFOAM_ERR_INVALID, "points, gbar and out must be non-NULL");
    if (multires < 0 || ld < 3 + 6 * multires) return fail(SDFOAM_ERR_INVALID, "ld too small for the encoding");
    cudaError_t e = launch_mlp_encode_jvp(points, center, n, multires, gbar, ld, out,
                                          reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SDFOAM_OK : cuda_fail(e, "sdfoam_mlp_encode_jvp");
}

int sdfoam_mlp_decode_hessian(const float *points, const float *center, uint32_t n, int multires, const void *denc2,
                              const void *denc, int ld, const float *gbar, float *dpoints, sdfoam_stream_t stream) {
    if (n > 0 && (!points || !denc2 || !denc || !gbar || !dpoints))
        return fail(SDFOAM_ERR_INVALID, "points, denc2, denc, gbar and dpoints must be non-NULL");
    if (multires < 0 || ld < 3 + 6 * multires) return fail(SDFOAM_ERR_INVALID, "ld too small for the encoding");
    cudaError_t e = launch_mlp_decode_hessian(points, center, n, multires, denc2, denc, ld, gbar, dpoints,
                                              reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SDFOAM_OK : cuda_fail(e, "sdfoam_mlp_decode_hessian");
}

int sdfoam_mlp_encode(const float *points, const float *center, uint32_t n, int multires, int ld, void *out,
                      sdfoam_stream_t stream) {
    if (n > 0 && (!points || !out)) return fail(SDFOAM_ERR_INVALID, "points and out must be non-NULL");
    if (multires < 0 || ld < 3 + 6 * multires + 1) return fail(SDFOAM_ERR_INVALID, "encoding row too short");
    if (ld % 8 || !aligned16(out)) return fail(SDFOAM_ERR_INVALID, "rows must be multiples of 8 and 16-byte aligned");
    cudaError_t e = launch_mlp_encode(points, center, n, multires, ld, out, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SDFOAM_OK : cuda_fail(e, "sdfoam_mlp_encode");
}

int sdfoam_mlp_activate(const void *z, int ldz, int zc, uint32_t n, const void *enc, int ldenc, int enc_cols,
                        float scale, int ld, void *out, sdfoam_stream_t stream) {
    if (n > 0 && (!z || !out || (enc_cols > 0 && !enc)))
        return fail(SDFOAM_ERR_INVALID, "z, out (and enc) must be non-NULL");
    if (zc < 0 || enc_cols < 0 || zc + enc_cols + 1 > ld || zc > ldz || (enc_cols > 0 && enc_cols > ldenc))
        return fail(SDFOAM_ERR_INVALID, "inconsistent row widths");
    if (ld % 8 || ldz % 8 || !aligned16(z) || !aligned16(out))
        return fail(SDFOAM_ERR_INVALID, "rows must be multiples of 8 and 16-byte aligned");
    cudaError_t e = launch_mlp_activate(z, ldz, zc, n, enc, ldenc, enc_cols, scale, ld, out,
                                        reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SDFOAM_OK : cuda_fail(e, "sdfoam_mlp_activate");
}

int sdfoam_mlp_deactivate(const void *da, int lda, const void *act, int ld_act, float scale, uint32_t n, int cols,
                          void *dz, int ldz, sdfoam_stream_t stream) {
    if (n > 0 && (!da || !act || !dz)) return fail(SDFOAM_ERR_INVALID, "da, act and dz must be non-NULL");
    if (cols < 0 || cols > ldz || ldz > lda || ldz > ld_act || !(scale > 0.0f))
        return fail(SDFOAM_ERR_INVALID, "inconsistent row widths");
    if (lda % 8 || ld_act % 8 || ldz % 8 || !aligned16(da) || !aligned16(act) || !aligned16(dz))
        return fail(SDFOAM_ERR_INVALID, "rows must be multiples of 8 and 16-byte aligned");
    cudaError_t e =
        launch_mlp_deactivate(da, lda, act, ld_act, scale, n, cols, dz, ldz, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SDFOAM_OK : cuda_fail(e, "sdfoam_mlp_deactivate");
}

int sdfoam_mlp_decode(const float *points, const float *center, uint32_t n, int multires, const void *denc, int ld,
                      float *dpoints, sdfoam_stream_t stream) {
    if (n > 0 && (!points || !denc || !dpoints)) return fail(SDFOAM_ERR_INVALID, "points, denc, dpoints non-NULL");
    cudaError_t e =
        launch_mlp_decode(points, center, n, multires, denc, ld, dpoints, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SDFOAM_OK : cuda_fail(e, "sdfoam_mlp_decode");
}

const char *sdfoam_last_error(void) { return g_last_error.c_str(); }

int sdfoam_abi_version(void) { return 5; }

}  // extern "C"
