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
// Bytes of one site record (32-byte head + SH row), rounded to 128-byte lines.
inline int site_bytes_of(uint32_t sh_degree) { return (32 + 4 * sh_stride_of(sh_degree) + 127) / 128 * 128; }

// Degree field of a face record: the neighbour's CSR row length, or one of
constexpr uint32_t kDegFromHead = 0xfffeu;  // row too long: read the head
constexpr uint32_t kDegInvalid = 0xffffu;   // row the walk never enters

// Cell-record workspace layout (sections 256-byte aligned):
//   sites  [N] x site_bytes: head (p.x, p.y, p.z, first CSR entry, end CSR
//          entry, last attribute channel, 0, 0) then the SH coefficients
//          (channels 0..A-2, zero padded); line aligned so a site is
//          prefetched with whole 128-byte lines
//   faces  uint4 [E] per CSR entry: (neighbour id, neighbour's first CSR
//          entry, half(dx) | half(dy) << 16, half(dz) | degree << 16), the
//          binary16 offset q - p of the reference's prefetch plus what the
//          walk needs to prefetch the neighbour before entering it
//   planes uint2 per face: (half(dx) | half(dy) << 16, half(dz)) -- only the
//          offsets the exit-face search reads, four to a 32-byte load.  Site
//          c's row starts at plane_row(c, beg) (a multiple of 4, so no
//          prefix sum is needed) and is zero-padded to a multiple of 4
//          faces; a zero offset has dp = 0 and never wins the search.
//          Row c spans at most [beg + 3c, beg + d + 3c + 6), so E + 3N + 8
//          slots hold every row.
__host__ __device__ inline uint32_t plane_row(uint32_t site, uint32_t beg) { return (beg + 3u * site + 3u) & ~3u; }

struct CellsLayout {
    size_t sites_off, faces_off, planes_off, total;
    static CellsLayout make(uint32_t n, uint32_t e, uint32_t sh_degree) {
        CellsLayout L;
        L.sites_off = 0;
        L.faces_off = align_up(L.sites_off + size_t(n) * site_bytes_of(sh_degree), 256);
        L.planes_off = align_up(L.faces_off + size_t(e) * 16, 256);
        L.total = align_up(L.planes_off + plane_slots(n, e) * 8, 256);
        return L;
    }
    static size_t plane_slots(uint32_t n, uint32_t e) { return align_up(size_t(e) + 3 * size_t(n) + 8, 4); }
    // plane_row() works in 32 bits
    static bool fits(uint32_t n, uint32_t e) { return size_t(e) + 3 * size_t(n) + 8 <= size_t(0xffffffffu); }
};

// Delaunay neighbour workspace: per-site neighbour lists of kDelaunayCap
// slots and their counts, the CSR prefix, scan partials, symmetry repairs and
// status words (failed cells, duplicate sites, asymmetric pairs, open cells,
// self-check code and index, cells queued for the second pass, the last
// non-empty row), the second pass's queue and its large cells, and the cells'
// own site order: the Morton order of the sites (order[i] = the caller's index
// of the i-th site), the sites in that order and their AABB tree.
constexpr uint32_t kDelaunayCap = 256;
struct DelaunayLayout {
    size_t nbr, cnt, prefix, sums, dirty, extra, status, retry, large, order, mpoints, mtree, total;
    // the Morton sort's scratch, inside the neighbour lists (free until the cells are built)
    size_t keys_a, keys_b, vals_b, high, hist, totals;
    uint32_t extra_cap, retry_cap;
};
DelaunayLayout delaunay_layout(uint32_t n);

// sort_points workspace: ping-pong keys / permutation arrays, the per-tile
// digit counts and the per-unit digit totals of the largest round.
struct SortLayout {
    size_t keys_a, keys_b, vals_a, vals_b, hist, totals, total;
};
SortLayout sort_layout(uint32_t n);

// Stable LSD radix sort of n (key, value) pairs by the whole 32-bit key: four
// 8-bit passes over one unit.  keys[cur] / vals[cur] hold the input; on return
// cur names the pair of buffers holding the result.  hist holds
// radix_hist_entries(n) words, totals 256.
size_t radix_hist_entries(uint32_t n);
cudaError_t launch_radix_sort_pairs(uint32_t *const keys[2], uint32_t *const vals[2], uint32_t n, uint32_t *hist,
                                    uint32_t *totals, int &cur, cudaStream_t stream);

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
    const unsigned char *sites;  // site_bytes per site
    const uint4 *faces;
    const uint2 *planes;
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
    void *rgba;             // attribute type
    float *depth;
    uint32_t *depth_indices;
    uint32_t *num_intersections;
    void *contribution;     // attribute type
    float *alpha;
    const uint64_t *seq_offsets;
    uint32_t *seq_cells;
    uint32_t *seq_count;
    uint32_t *face_tests;
    unsigned char *exits;   // optional exit record [R][exits_stride]
    uint32_t exits_stride;
    float4 *colors;         // optional step record [colors_steps][R]: colour, t1
    uint32_t colors_steps;
    uint32_t *sites;        // optional, with colors: the site entered per step
};

// Headless render of one camera (trace_benchmark): per pixel the pinhole or
// fisheye ray of cast_ray, the forward walk from one start site, composited
// over the background and packed as RGBA8.
struct RenderParams {
    CellsView cells;
    sdfoam_trace_settings settings;
    const float *sharpness;
    const uint32_t *start;   // one site for every pixel (device)
    float position[3], forward[3], right[3], up[3];
    float fov;
    float focal;             // 1 / tan(fov / 2), pinhole
    float aspect;            // width / height
    uint32_t width, height, model;
    float bg[3];
    uint32_t checker;
    uint32_t *rgba8;         // [height * width], rows bottom-up
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
    const void *rgba;       // attribute type
    const void *rgba_grad;  // attribute type
    const float *depth_grad;
    const void *ray_error;  // attribute type
    const float *sharpness;
    float4 *attr_acc;
    float4 *point_acc;
    void *point_error;      // attribute type
    float *sharpness_grad;
    const unsigned char *exits;  // optional exit record of the forward (NeuS)
    uint32_t exits_stride;
    const float4 *colors;        // optional step record of the forward (NeuS)
    uint32_t colors_steps;
    const uint32_t *sites;       // optional, with colors: the site entered per step
};

// Sets the message sdfoam_last_error() returns on this thread.
void set_last_error(const std::string &msg);

// diffs: NULL (computed from the positions) or the caller's binary16 [E][4]
cudaError_t launch_build_cells(const sdfoam_foam &foam, const void *diffs, void *cells, cudaStream_t stream);
uint32_t pow2_round_up(uint32_t x);
cudaError_t launch_sort_points(const float *points, uint32_t n, float *sorted, uint32_t *perm, void *workspace,
                               cudaStream_t stream);
cudaError_t launch_delaunay_neighbors(const float *points, uint32_t n, const float *tree, void *workspace,
                                      uint32_t *offsets, cudaStream_t stream, const char **failed_stage);
cudaError_t launch_delaunay_adjacency(const void *workspace, uint32_t n, uint32_t *adjacency,
                                      uint32_t adjacency_size, cudaStream_t stream);
// prefix[i] = sum of cnt[0..i), prefix[n] = the total; sums holds scan_partials(n) words
size_t scan_partials(uint32_t n);
cudaError_t launch_exclusive_scan(const uint32_t *cnt, uint32_t n, uint32_t *sums, uint32_t *prefix,
                                  cudaStream_t stream);
// Tetrahedra of a triangulation from its sites (sort_points order) and CSR
// adjacency; workspace tets_workspace_bytes(n, num_tets).  The count pass
// writes the total to *num_tets (host, after a stream sync); the write pass
// recomputes the counts and sets *count_mismatch (writing nothing) if the
// total is not num_tets.  status (host, 4 words): cells that failed, faces shared by
// more than two tets, rows too long for any cell, 0.
size_t tets_workspace_bytes(uint32_t n, uint32_t num_tets);
cudaError_t launch_tets_count(const float *points, uint32_t n, const uint32_t *adjacency, uint32_t adjacency_size,
                              const uint32_t *offsets, void *workspace, uint32_t *num_tets, uint32_t *status,
                              cudaStream_t stream);
cudaError_t launch_tets(const float *points, uint32_t n, const uint32_t *adjacency, uint32_t adjacency_size,
                        const uint32_t *offsets, void *workspace, uint32_t num_tets, uint32_t *tets,
                        uint32_t *tet_adjacency, uint32_t *vert_to_tet, uint32_t *status, bool *count_mismatch,
                        cudaStream_t stream);
cudaError_t launch_mlp_layer(const void *x, int ldx, int kx, uint32_t n, const void *w, int ldw, int nw,
                             const void *enc, int ldenc, int enc_cols, int zc, float scale, void *out, int ld,
                             int *error, cudaStream_t stream);
cudaError_t launch_mlp_layer_dot(const void *x, int ldx, int kx, uint32_t n, const void *w, int ldw, int nw,
                                 const void *enc, int ldenc, int enc_cols, int zc, float scale, void *out, int ld,
                                 const void *wdot, float *zdot, float dot_scale, int *error, cudaStream_t stream);
cudaError_t launch_mlp_wgrad(const void *dz, int ldz, int m, uint32_t n, const void *act, int lda, int k,
                             float *dw, int lddw, int bias_col, int *error, cudaStream_t stream);
cudaError_t launch_mlp_input_grad(const void *dz, int ld, int k, uint32_t n, const void *wt, int ldwt, int nwt,
                                  const void *add, int ldadd, int add_cols, void *out, int ldout, int *error,
                                  cudaStream_t stream);
cudaError_t launch_mlp_layer_tangent(const void *t_in, int ld_in, int k, uint32_t n, const void *w, int ldw, int nw,
                                    const void *act, int ld_act, int cols, float scale, const void *tenc, int ldenc,
                                    int enc_cols, void *out, int ldout, void *zout, int ldzo, int *error,
                                    cudaStream_t stream);
cudaError_t launch_mlp_layer_second(const void *s_next, int ld_next, int k, uint32_t n, const void *wt, int ldwt,
                                    int nwt, const void *act, int ld_act, int cols, float scale, const void *dz,
                                    int lddz, const void *tz, int ldtz, void *out, int ldout, void *skip, int ldskip,
                                    int *error, cudaStream_t stream);
cudaError_t launch_mlp_encode_jvp(const float *points, const float *center, uint32_t n, int multires,
                                  const float *gbar, int ld, void *out, cudaStream_t stream);
cudaError_t launch_mlp_decode_hessian(const float *points, const float *center, uint32_t n, int multires,
                                      const void *denc2, const void *denc, int ld, const float *gbar, float *dpoints,
                                      cudaStream_t stream);
cudaError_t launch_mlp_layer_backward(const void *dz_next, int ld_next, int k, uint32_t n, const void *wt, int ldwt,
                                      int nwt, const void *act, int ld_act, int cols, float scale, void *dz, int ldz,
                                      void *skip, int ldskip, int *error, cudaStream_t stream);
cudaError_t launch_mlp_encode(const float *points, const float *center, uint32_t n, int multires, int ld,
                              void *out, cudaStream_t stream);
cudaError_t launch_mlp_activate(const void *z, int ldz, int zc, uint32_t n, const void *enc, int ldenc, int enc_cols,
                                float scale, int ld, void *out, cudaStream_t stream);
cudaError_t launch_mlp_deactivate(const void *da, int lda, const void *act, int ld_act, float scale, uint32_t n,
                                  int cols, void *dz, int ldz, cudaStream_t stream);
cudaError_t launch_mlp_decode(const float *points, const float *center, uint32_t n, int multires, const void *denc,
                              int ld, float *dpoints, cudaStream_t stream);
cudaError_t launch_farthest_neighbor(const float *points, const uint32_t *adjacency, const uint32_t *offsets,
                                     uint32_t num_points, uint32_t adjacency_size, uint32_t *indices,
                                     float *radius, cudaStream_t stream);
cudaError_t launch_build_aabb_tree(const float *points, uint32_t num_points, float *tree, cudaStream_t stream);
cudaError_t launch_nn(const float *points, uint32_t num_points, const float *tree, const float *queries,
                      uint32_t num_queries, uint32_t *indices, cudaStream_t stream);
cudaError_t launch_forward(uint32_t sh_degree, uint32_t attr_dtype, const ForwardParams &p, cudaStream_t stream);
cudaError_t launch_render(uint32_t sh_degree, uint32_t attr_dtype, const RenderParams &p, cudaStream_t stream);
cudaError_t launch_backward(uint32_t sh_degree, uint32_t attr_dtype, const BackwardParams &p, cudaStream_t stream);
cudaError_t launch_fold_grads(uint32_t sh_degree, uint32_t attr_dtype, uint32_t num_points, const float4 *attr_acc,
                              const float4 *point_acc, void *attr_grad, float *points_grad, cudaStream_t stream);

inline CellsView cells_view(const sdfoam_foam &foam, const void *cells) {
    CellsLayout L = CellsLayout::make(foam.num_points, foam.adjacency_size, foam.sh_degree);
    const char *base = static_cast<const char *>(cells);
    CellsView v;
    v.sites = reinterpret_cast<const unsigned char *>(base + L.sites_off);
    v.faces = reinterpret_cast<const uint4 *>(base + L.faces_off);
    v.planes = reinterpret_cast<const uint2 *>(base + L.planes_off);
    v.num_points = foam.num_points;
    v.adjacency_size = foam.adjacency_size;
    return v;
}

}  // namespace sdfoam_b200
