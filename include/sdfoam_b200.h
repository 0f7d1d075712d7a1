/*
 * sdfoam_b200.h -- C ABI of the B200 Voronoi-foam tracer.
 *
 * Drop-in boundary for SDFoam's tracing pipeline.  Every entry point takes
 * plain device pointers and sizes, launches asynchronously on the given CUDA
 * stream (NULL = legacy default stream, which is what the reference uses) and
 * returns SDFOAM_OK or an error code; sdfoam_last_error() returns the
 * message of the last failing call on the calling thread.  The library never
 * allocates device memory: workspaces are sized by the *_bytes queries and
 * owned by the caller.
 *
 * Reference interfaces replaced (paths inside mmlab-cv/SDFoam):
 *   sdfoam_build_cells          prefetch_adjacent_diff    src/tracing/pipeline.h:71-77
 *                               (prefetch_adjacent_diff_kernel, pipeline.cu:1202-1224)
 *   sdfoam_trace_forward        Pipeline::trace_forward   src/tracing/pipeline.h:83-101
 *   sdfoam_trace_backward       Pipeline::trace_backward  src/tracing/pipeline.h:104-126
 *   (sh_degree / attr_dtype     create_pipeline           src/tracing/pipeline.h:163,
 *    arguments)                 dispatch table            pipeline.cu:1477-1506
 *   sdfoam_trace_settings       TraceSettings             src/tracing/pipeline.h:12-40
 *   sdfoam_trace_benchmark      Pipeline::trace_benchmark src/tracing/pipeline.h:144-156
 *                               (benchmark kernel, pipeline.cu:1067-1199)
 *   sdfoam_camera               Camera / cast_ray         src/tracing/camera.h:7-85
 *   sdfoam_sort_points, sdfoam_build_aabb_tree, sdfoam_nn,
 *   sdfoam_farthest_neighbor    the triangulation module  (see each declaration)
 *
 * Data layout (all row-major, contiguous):
 *   points           float32 [N,3]
 *   attributes       [N,A] of attr_dtype, A = 1 + 3*(sh_degree+1)^2; channel
 *                    3k+c is SH coefficient k of colour c, channel A-1 is the
 *                    SDF (NeuS mode) or density (standard mode)
 *   point_adjacency  uint32 [E], CSR rows of ascending neighbour ids
 *   offsets          uint32 [N+1]
 *   rays             float32 [R,6] = origin, direction (normalised inside)
 *   start_point      uint32 [R]
 */
#ifndef SDFOAM_B200_H
#define SDFOAM_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SDFOAM_API __attribute__((visibility("default")))
#else
#define SDFOAM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *sdfoam_stream_t; /* same type as cudaStream_t */

enum {
    SDFOAM_OK = 0,
    SDFOAM_ERR_INVALID = 1,     /* bad argument (message says which) */
    SDFOAM_ERR_UNSUPPORTED = 2, /* dtype / SH degree outside the dispatch table */
    SDFOAM_ERR_CUDA = 3         /* a CUDA runtime call failed */
};

enum { SDFOAM_F32 = 0, SDFOAM_F16 = 1 };
enum { SDFOAM_ALPHA_STANDARD = 0, SDFOAM_ALPHA_NEUS = 1 };
enum { SDFOAM_PINHOLE = 0, SDFOAM_FISHEYE = 1 };

/* TraceSettings (pipeline.h:12-27).  Defaults (pipeline.h:29-40):
 * weight_threshold 1e-7, max_intersections 1024, alpha_mode standard.
 * sdf_channel < 0 means "none"; the NeuS alpha is used only when alpha_mode is
 * NeuS and sdf_channel >= 0 (pipeline.cu:129). eps is carried but, as in the
 * reference kernels, unused. */
typedef struct {
    float weight_threshold;
    uint32_t max_intersections;
    uint32_t alpha_mode;
    int32_t sdf_channel;
    float eps;
} sdfoam_trace_settings;

/* The foam a pipeline traces. */
typedef struct {
    uint32_t num_points;      /* N */
    uint32_t adjacency_size;  /* E */
    uint32_t sh_degree;       /* 0..3 */
    uint32_t attr_dtype;      /* SDFOAM_F32 or SDFOAM_F16: type of attributes and of the
                                 attribute-typed buffers marked [attr] below */
    const float *points;
    const void *attributes;
    const uint32_t *point_adjacency;
    const uint32_t *point_adjacency_offsets;
} sdfoam_foam;

/* Bytes of the cell-record workspace for a foam: per site a line-aligned
 * record (position, CSR range, last attribute channel, SH coefficients as
 * float32), per CSR entry a 16-byte face record (neighbour id, the
 * neighbour's CSR start and degree, and the binary16 offset q - p that the
 * reference's prefetch computes), and per site a zero-padded row of 8-byte
 * plane records (the offsets alone, read by the exit-face search).  0 for an
 * unsupported SH degree or a foam with adjacency_size + 3 * num_points +
 * 8 >= 2^32.  The workspace must be 32-byte aligned. */
SDFOAM_API size_t sdfoam_cells_bytes(uint32_t num_points, uint32_t adjacency_size,
                          uint32_t sh_degree);

/* Builds the cell records (replaces prefetch_adjacent_diff).  The records
 * stay valid while points, attributes and adjacency are unchanged, so a
 * forward and its backward can share one build. */
SDFOAM_API int sdfoam_build_cells(const sdfoam_foam *foam, void *cells, size_t cells_bytes,
                       sdfoam_stream_t stream);

/* Pipeline::trace_forward outputs (pipeline.h:83-101).  Optional pointers may
 * be NULL: depth_quantiles (then depth / depth_indices are not written),
 * num_intersections, point_contribution (accumulated: caller zeroes it),
 * alpha (per-site alpha of some ray's visit: the reference's racy store).
 * sharpness: device float, element 0 is the NeuS sharpness inv_s.
 * ray_rgba: [R,4] [attr], 8-byte aligned (16 for float32).
 * In float16 NeuS mode the sharpness is read the way the reference reads it:
 * the first two bytes of the float buffer as a binary16 value
 * (pipeline.cu:137-141 with the float32 buffer of pipeline_bindings.cpp:124-136). */
typedef struct {
    uint32_t num_rays;
    const float *rays;
    const uint32_t *start_point;
    uint32_t num_depth_quantiles;
    const float *depth_quantiles;
    const float *sharpness;
    void *ray_rgba;               /* [attr] */
    float *depth;
    uint32_t *depth_indices;
    uint32_t *num_intersections;
    void *point_contribution;     /* [attr] */
    float *alpha;
    /* debug dump of the walk (NULL to disable): for ray r, the sites handed
     * to the cell functor are written to seq_cells[seq_offsets[r] ..
     * seq_offsets[r+1]) and their count to seq_count[r]. */
    const uint64_t *seq_offsets;
    uint32_t *seq_cells;
    uint32_t *seq_count;
    /* optional per-ray count of face records examined (the sum of the
     * degrees of the sites the walk entered); NULL to disable. */
    uint32_t *face_tests;
    /* optional exit record [R][exits_stride] bytes (stride a multiple of 8,
     * 8-byte aligned rows): the position of each step's exit face in its
     * CSR row, for the first exits_stride steps.  Pass the same buffer to
     * sdfoam_trace_backward (NeuS mode, same rays and foam) and its walk
     * replays the steps with one face test each instead of a search; the
     * results are the same.  NULL to disable. */
    uint8_t *exits;
    uint32_t exits_stride;
    /* optional step record, step-major, for walk steps n <= step_colors_steps
     * of ray r at index (n - 1) * num_rays + r:
     *   step_colors: (r, g, b, t1) -- the SH colour the forward evaluated at
     *     the step and the step's exit distance (16-byte aligned float4);
     *   step_sites (optional, with step_colors): the site the walk entered
     *     at the step, or 0xffffffff where the walk ended there.
     * Pass them to sdfoam_trace_backward (NeuS mode) and the backward reads
     * each recorded step -- the lanes of a warp are at the same step, so the
     * reads are coalesced -- instead of testing the exit face again
     * (step_sites) and gathering and evaluating the site's SH row
     * (step_colors); the results are the same.  NULL to disable. */
    float *step_colors;
    uint32_t step_colors_steps;
    uint32_t *step_sites;
} sdfoam_forward_io;

SDFOAM_API int sdfoam_trace_forward(const sdfoam_foam *foam, const void *cells,
                         const sdfoam_trace_settings *settings,
                         const sdfoam_forward_io *io, sdfoam_stream_t stream);

/* sdfoam_build_cells with the caller's binary16 neighbour offsets: adjacent_diff
 * is [E][4] binary16 (q - p, 0) per CSR entry, 8-byte aligned -- the
 * adjacent_diff argument of the reference's trace_benchmark
 * (pipeline_bindings.cpp:614, 725), used as given instead of recomputed. */
SDFOAM_API int sdfoam_build_cells_from_diffs(const sdfoam_foam *foam, const void *adjacent_diff, void *cells,
                                             size_t cells_bytes, sdfoam_stream_t stream);

/* Camera (camera.h:17-26): host values.  Rays follow cast_ray (camera.h:
 * 56-85): u = (2 i / width - 1) * width / height, v = 1 - 2 j / height, no
 * half-pixel offset; pinhole direction = forward / tan(fov / 2) + u right +
 * v up, fisheye by angle fov * |(u, v)|; then normalised. */
typedef struct sdfoam_camera {
    float position[3];
    float forward[3];
    float right[3];
    float up[3];
    float fov;          /* radians */
    uint32_t width;
    uint32_t height;
    uint32_t model;     /* SDFOAM_PINHOLE or SDFOAM_FISHEYE */
} sdfoam_camera;

/* Pipeline::trace_benchmark (pipeline.h:144-156, kernel pipeline.cu:
 * 1067-1199): renders one frame headless.  Every pixel walks from the single
 * site *start_point (device) with the forward's cell arithmetic (no
 * contributions, alpha or quantiles), composites over bg_color (host, 3
 * floats; NULL = white, the reference's default visualisation settings) or a
 * 20-pixel checkerboard, and stores RGBA8 (r | g << 8 | b << 16 | a << 24,
 * each channel clamped to [0, 1] and truncated from x * 255) at
 * output_rgba[(height - 1 - j) * width + i].  Fisheye pixels outside the
 * lens get the background. */
SDFOAM_API int sdfoam_trace_benchmark(const sdfoam_foam *foam, const void *cells,
                                      const sdfoam_trace_settings *settings, const sdfoam_camera *camera,
                                      const uint32_t *start_point, const float *sharpness,
                                      const float *bg_color, int checker_bg, uint32_t *output_rgba,
                                      sdfoam_stream_t stream);

/* Bytes of the gradient accumulation workspace (16-byte aligned per-site
 * rows, zeroed and folded into attr_grad / points_grad by the call). */
SDFOAM_API size_t sdfoam_backward_workspace_bytes(uint32_t num_points, uint32_t sh_degree);

/* Pipeline::trace_backward (pipeline.h:104-126).  points_grad [N,3] and
 * attr_grad [N,A] are overwritten (the reference's binding hands the kernel
 * zeroed buffers).  sharpness_grad (float, element 0) and point_error [N]
 * are accumulated into.  depth_quantiles / depth_indices / depth_grad are
 * used together or not at all; ray_error enables point_error. */
typedef struct {
    uint32_t num_rays;
    const float *rays;
    const uint32_t *start_point;
    uint32_t num_depth_quantiles;
    const float *depth_quantiles;
    const uint32_t *depth_indices;
    const void *ray_rgba;         /* [attr] */
    const void *ray_rgba_grad;    /* [attr] */
    const float *depth_grad;
    const void *ray_error;        /* [attr] */
    const float *sharpness;
    float *points_grad;
    void *attr_grad;              /* [attr] */
    void *point_error;            /* [attr] */
    float *sharpness_grad;
    void *workspace;
    size_t workspace_bytes;
    /* optional: the exit record the forward wrote for these rays (NeuS mode;
     * ignored in standard mode, whose backward walk uses another exit rule) */
    const uint8_t *exits;
    uint32_t exits_stride;
    /* optional: the step record the forward wrote for these rays (NeuS mode;
     * see sdfoam_forward_io) */
    const float *step_colors;
    uint32_t step_colors_steps;
    const uint32_t *step_sites;
} sdfoam_backward_io;

SDFOAM_API int sdfoam_trace_backward(const sdfoam_foam *foam, const void *cells,
                          const sdfoam_trace_settings *settings,
                          const sdfoam_backward_io *io, sdfoam_stream_t stream);

/* Nodes of the AABB tree over num_points sites: pow2_round_up(num_points);
 * the tree is float32 [nodes][2][3] (box min, box max), level by level with
 * the leaves (site pairs) first -- the layout of the reference's
 * build_aabb_tree (src/aabb_tree/aabb_tree.h:10-13, aabb_tree.cu:192-341,
 * binding triangulation_bindings.cpp:117-140). */
SDFOAM_API uint32_t sdfoam_aabb_tree_nodes(uint32_t num_points);

/* build_aabb_tree: the tree over sites that are already in sorted order. */
SDFOAM_API int sdfoam_build_aabb_tree(const float *points, uint32_t num_points, float *tree,
                                      sdfoam_stream_t stream);

/* nn (src/aabb_tree/aabb_tree.h:15-23, aabb_tree.cu:343-415): index of the
 * site nearest to each query point (float32 [Q,3]) by squared Euclidean
 * distance, ties to the lowest index.  Used to seed each ray's start site. */
SDFOAM_API int sdfoam_nn(const float *points, uint32_t num_points, const float *tree,
                         const float *queries, uint32_t num_queries, uint32_t *indices,
                         sdfoam_stream_t stream);

/* sort_points (src/aabb_tree/aabb_tree.cu:62-190, run by the reference's
 * DelaunayTriangulation::rebuild before it triangulates; the permutation is
 * what Triangulation.permutation() returns, triangulation_bindings.cpp:
 * 219-237): rounds of stable sorts of the sites by the order-preserving u32
 * bits of one coordinate, axes x, y, z, x, ..., on segments of pow2(N) sites
 * halving each round.  permutation[i] = original index of the i-th sorted
 * site; sorted_points[i] = points[permutation[i]] (bit for bit).  sorted_points
 * must not overlap points.  Workspace: sdfoam_sort_points_workspace_bytes. */
SDFOAM_API size_t sdfoam_sort_points_workspace_bytes(uint32_t num_points);
SDFOAM_API int sdfoam_sort_points(const float *points, uint32_t num_points, float *sorted_points,
                                  uint32_t *permutation, void *workspace, size_t workspace_bytes,
                                  sdfoam_stream_t stream);

/* Delaunay adjacency of sorted sites: the point adjacency of the reference's
 * DelaunayTriangulation::rebuild (src/delaunay/delaunay.cu:273-370) as its
 * find_adjacency writes it (delaunay.cu:32-229): CSR rows of ascending
 * neighbour ids, offsets[0] = 0, offsets[N] = 2 * edges, and a row that
 * follows an empty row starting at UINT32_MAX.  Three calls:
 *   sdfoam_delaunay_neighbors  per-site Voronoi cells on the GPU (points in
 *                              sort_points order and their AABB tree), then
 *                              the offsets [N+1];
 *   sdfoam_delaunay_status     waits for the stream and copies 6 words to the
 *                              host: cells that failed, duplicate sites,
 *                              asymmetric pairs repaired, cells finished
 *                              vertex by vertex, and the code and index of the
 *                              first failed self-check of an index (0 if
 *                              none).  Failed cells, duplicates or a failed
 *                              self-check make the rebuild fail
 *                              (TriangulationFailedError);
 *   sdfoam_delaunay_adjacency  the adjacency [offsets[N]] once the caller has
 *                              read offsets[N] and allocated it.
 * At least 32 sites, as the reference requires. */
SDFOAM_API size_t sdfoam_delaunay_workspace_bytes(uint32_t num_points);
SDFOAM_API int sdfoam_delaunay_neighbors(const float *points, uint32_t num_points, const float *tree,
                                         void *workspace, size_t workspace_bytes,
                                         uint32_t *point_adjacency_offsets, sdfoam_stream_t stream);
SDFOAM_API int sdfoam_delaunay_status(const void *workspace, uint32_t num_points, uint32_t *status,
                                      sdfoam_stream_t stream);
SDFOAM_API int sdfoam_delaunay_adjacency(const void *workspace, uint32_t num_points, uint32_t *point_adjacency,
                                         uint32_t adjacency_size, sdfoam_stream_t stream);

/* Tetrahedra of a triangulation: the reference's Triangulation::tets,
 * tet_adjacency and vert_to_tet (src/delaunay/delaunay.h:23-37, filled by
 * find_adjacency, src/delaunay/delaunay.cu:32-144; bound in
 * torch_bindings/triangulation_bindings.cpp:59-115), from the sorted sites and
 * the CSR adjacency sdfoam_delaunay_adjacency wrote.  Two calls:
 *   sdfoam_delaunay_tets_count  the number of tets T (written to *num_tets on
 *                               the host; waits for the stream), with the
 *                               workspace sdfoam_delaunay_tets_workspace_bytes(N, 0);
 *   sdfoam_delaunay_tets        tets [T][4] (16-byte aligned), tet_adjacency
 *                               [T][4] and vert_to_tet [N], with the workspace
 *                               sdfoam_delaunay_tets_workspace_bytes(N, T).
 * Tets are sorted by their sorted vertex sets (the reference's tet order) and
 * oriented as the reference's (IndexedTet::volume > 0); tet_adjacency[4t + j]
 * is 4t' + j' of the tet across the face opposite vertex j, UINT32_MAX on the
 * hull; vert_to_tet[v] is the smallest tet containing v, UINT32_MAX for none.
 * status (host, 4 words, either call): cells that failed, faces shared by
 * more than two tets (the reference's "ambiguous triangulation"), rows too
 * long for any cell, 0.  SDFOAM_ERR_INVALID if T is not the count. */
SDFOAM_API size_t sdfoam_delaunay_tets_workspace_bytes(uint32_t num_points, uint32_t num_tets);
SDFOAM_API int sdfoam_delaunay_tets_count(const float *points, uint32_t num_points, const uint32_t *point_adjacency,
                                          uint32_t adjacency_size, const uint32_t *point_adjacency_offsets,
                                          void *workspace, size_t workspace_bytes, uint32_t *num_tets,
                                          uint32_t *status, sdfoam_stream_t stream);
SDFOAM_API int sdfoam_delaunay_tets(const float *points, uint32_t num_points, const uint32_t *point_adjacency,
                                    uint32_t adjacency_size, const uint32_t *point_adjacency_offsets,
                                    void *workspace, size_t workspace_bytes, uint32_t num_tets, uint32_t *tets,
                                    uint32_t *tet_adjacency, uint32_t *vert_to_tet, uint32_t *status,
                                    sdfoam_stream_t stream);

/* farthest_neighbor (src/delaunay/triangulation_ops.h:8-16,
 * triangulation_ops.cu:10-87): per site, the farthest Delaunay neighbour
 * (uint32, UINT32_MAX if none) and the mean half-edge length (float). */
SDFOAM_API int sdfoam_farthest_neighbor(const float *points, const uint32_t *point_adjacency,
                                        const uint32_t *point_adjacency_offsets, uint32_t num_points,
                                        uint32_t adjacency_size, uint32_t *indices, float *cell_radius,
                                        sdfoam_stream_t stream);

/* Elementwise stages of the sdfnet MLP (the reference's
 * sdfoam_model/sdfnet.py:43-152 is plain PyTorch, so these have no binding
 * counterpart; sdfoam_b200/sdfnet.py drives them around its GEMMs).  All
 * activation buffers are bf16 rows with the given leading dimensions.
 *   encode:     positional encoding of points - center (center may be NULL),
 *               3 + 6*multires features, a 1.0 bias column, zero padding to ld
 *   activate:   out = [scale*softplus_100(z[:, :zc]), scale*enc[:, :enc_cols],
 *               1, 0...]
 *   deactivate: dz = scale * da * sigmoid(100 z) over cols columns (zero up
 *               to ldz), with the sigmoid recomputed from the activation out
 *               that activate wrote: sigmoid(100 z) = 1 - exp(-100 out/scale)
 *   decode:     dpoints += d/dpoints of the encoding given its gradient
 * Leading dimensions are multiples of 8 and rows start 16-byte aligned. */
/* One hidden layer on the tcgen05 tensor cores (a GEMM with its activation
 * fused): out = [scale*softplus_100(x W^T)[:, :zc], scale*enc[:, :enc_cols],
 * 1, 0 ...] -- sdfoam_mlp_activate applied to x W^T without materialising
 * it.  x [n, kx] (leading dimension ldx) ends with the bias column of ones,
 * W [nw <= 256, kx] (ldw) is the bias-folded weight, out [n, ld].  kx <= 320;
 * when kx > 256 the columns of x past 255 must be the bias column (1 at
 * column 256) and zeros: the tensor cores multiply the first 256 columns and
 * the epilogue adds W[:, 256].  All bf16, leading dimensions multiples of 8,
 * 16-byte aligned.  *error (device int) is set to 1 if a tile gave up
 * waiting for its copies or MMAs. */
SDFOAM_API int sdfoam_mlp_layer(const void *x, int ldx, int kx, uint32_t n, const void *w, int ldw, int nw,
                                const void *enc, int ldenc, int enc_cols, int zc, float scale, void *out, int ld,
                                int *error, sdfoam_stream_t stream);
/* The backward of a hidden layer on tcgen05, fused with its activation's
 * derivative: dz = scale * (dz_next Wt^T)[:, :cols] * sigmoid(100 z), where
 * dz_next [n, k <= 256] is the next layer's pre-activation gradient, Wt [nwt
 * <= 256, k] the next layer's bias-folded weight transposed (rows = its inputs), and
 * sigmoid(100 z) is recomputed from this layer's stored output act = scale *
 * softplus_100(z) [n, ld_act].  dz [n, ldz] is zero past cols; when skip is
 * given, scale * (dz_next Wt^T)[:, cols:256] goes to skip [n, ldskip] (the
 * gradient of the skip columns).  Layout rules and *error as
 * sdfoam_mlp_layer. */
SDFOAM_API int sdfoam_mlp_layer_backward(const void *dz_next, int ld_next, int k, uint32_t n, const void *wt,
                                         int ldwt, int nwt, const void *act, int ld_act, int cols, float scale,
                                         void *dz, int ldz, void *skip, int ldskip, int *error,
                                         sdfoam_stream_t stream);
/* sdfoam_mlp_layer whose epilogue also applies the next layer when that layer
 * has a single output (sdfnet's last linear layer, sdfoam_model/sdfnet.py:
 * 120-136): zdot[r, b] = dot_scale * sum_c out[r, c] wdot[c] over the bf16
 * outputs c of the 64-column block b (zc = 256, no skip columns), plus
 * dot_scale * wdot[256] (the bias) in block 3; wdot is bf16 [>= 257], zdot
 * fp32 [n, 4] and the output is zdot[r, 0] + zdot[r, 1] + zdot[r, 2] +
 * zdot[r, 3] (a fixed order: the same bits every run).  Replaces the
 * reference's lin8 GEMM on the last hidden activation. */
SDFOAM_API int sdfoam_mlp_layer_dot(const void *x, int ldx, int kx, uint32_t n, const void *w, int ldw, int nw,
                                    const void *enc, int ldenc, int enc_cols, int zc, float scale, void *out, int ld,
                                    const void *wdot, float *zdot, float dot_scale, int *error,
                                    sdfoam_stream_t stream);
/* Weight gradient of one sdfnet layer on the tcgen05 tensor cores (the
 * reference's autograd of F.linear, sdfoam_model/sdfnet.py:120-136):
 * dw[i, c] += sum_r dz[r, i] act[r, c] for i < m <= 256 and c < k <= 256, and,
 * when bias_col >= 0, dw[i, bias_col] += sum_r dz[r, i] (the gradient of a
 * bias column of ones).  dz [n, ldz] and act [n, lda] bf16 (leading dimensions
 * multiples of 8, rows 16-byte aligned), dw fp32 [m, lddw] accumulated
 * (zeroed by the caller; lddw and k multiples of 4).  Each SM adds one partial
 * sum with fp32 atomics, so the order of the sum varies between calls.
 * *error as sdfoam_mlp_layer. */
SDFOAM_API int sdfoam_mlp_wgrad(const void *dz, int ldz, int m, uint32_t n, const void *act, int lda, int k,
                                float *dw, int lddw, int bias_col, int *error, sdfoam_stream_t stream);
/* Gradient of a layer's input on tcgen05: out[:, :nwt] = dz Wt^T (+ add[:,
 * :add_cols]), zero up to ldout, with dz [n, k <= 256], Wt [nwt <= 256, k] the
 * layer's weight transposed (rows = its inputs) and add an optional bf16
 * addend (the skip connection's gradient).  The sdfnet's encoding gradient
 * (sdfoam_model/sdfnet.py:120-128).  Layout rules and *error as
 * sdfoam_mlp_layer. */
SDFOAM_API int sdfoam_mlp_input_grad(const void *dz, int ld, int k, uint32_t n, const void *wt, int ldwt, int nwt,
                                     const void *add, int ldadd, int add_cols, void *out, int ldout, int *error,
                                     sdfoam_stream_t stream);
/* The eikonal term's double backward (sdfoam_model/sdfnet.py:144-152 with
 * create_graph=True, used by train.py:293-326), as sweeps of the same tcgen05
 * layer kernel:
 *   tangent: out[:, :cols] = scale * (t_in W^T)[:, :cols] * sigmoid(100 z) with
 *     the sigmoid recomputed from this layer's stored activation act (as in
 *     sdfoam_mlp_layer_backward), out[:, cols:cols+enc_cols] = scale * tenc
 *     (the skip concatenation's tangent), zero up to ldout (<= 256); zout
 *     [n, ldzo] receives the raw product t_in W^T (the tangent
 *     pre-activations).  W [nw, k] is the layer's bias-folded weight (its
 *     bias column is not used: a tangent has no constant term).
 *   second: out = sdfoam_mlp_layer_backward's result on s_next plus
 *     dz * tz * 100 (1 - sigmoid(100 z)) on the first cols columns, where dz
 *     is the first-order gradient of this layer's pre-activation and tz its
 *     tangent (zout of the tangent sweep): the softplus's second derivative
 *     along the tangent.
 *   encode_jvp: out = J_enc gbar, the positional encoding's tangent along
 *     gbar [n, 3] (fp32), with 0 in the ones column.
 *   decode_hessian: dpoints += J_enc^T denc2 + H_enc[denc](gbar).
 * Layout rules and *error as sdfoam_mlp_layer. */
SDFOAM_API int sdfoam_mlp_layer_tangent(const void *t_in, int ld_in, int k, uint32_t n, const void *w, int ldw,
                                        int nw, const void *act, int ld_act, int cols, float scale, const void *tenc,
                                        int ldenc, int enc_cols, void *out, int ldout, void *zout, int ldzo,
                                        int *error, sdfoam_stream_t stream);
SDFOAM_API int sdfoam_mlp_layer_second(const void *s_next, int ld_next, int k, uint32_t n, const void *wt, int ldwt,
                                       int nwt, const void *act, int ld_act, int cols, float scale, const void *dz,
                                       int lddz, const void *tz, int ldtz, void *out, int ldout, void *skip,
                                       int ldskip, int *error, sdfoam_stream_t stream);
SDFOAM_API int sdfoam_mlp_encode_jvp(const float *points, const float *center, uint32_t n, int multires,
                                     const float *gbar, int ld, void *out, sdfoam_stream_t stream);
SDFOAM_API int sdfoam_mlp_decode_hessian(const float *points, const float *center, uint32_t n, int multires,
                                         const void *denc2, const void *denc, int ld, const float *gbar,
                                         float *dpoints, sdfoam_stream_t stream);
SDFOAM_API int sdfoam_mlp_encode(const float *points, const float *center, uint32_t n, int multires, int ld,
                                 void *out, sdfoam_stream_t stream);
SDFOAM_API int sdfoam_mlp_activate(const void *z, int ldz, int zc, uint32_t n, const void *enc, int ldenc,
                                   int enc_cols, float scale, int ld, void *out, sdfoam_stream_t stream);
SDFOAM_API int sdfoam_mlp_deactivate(const void *da, int lda, const void *act, int ld_act, float scale, uint32_t n,
                                     int cols, void *dz, int ldz, sdfoam_stream_t stream);
SDFOAM_API int sdfoam_mlp_decode(const float *points, const float *center, uint32_t n, int multires,
                                 const void *denc, int ld, float *dpoints, sdfoam_stream_t stream);

/* Allocation-free sdfoam_trace_forward.  No counterpart in the reference: it
 * exists for callers that cannot allocate device memory -- hosts reaching this
 * library through the C ABI without a device allocator of their own, and frame
 * loops (an interactive viewer) that must not call cudaMalloc / cudaFree, which
 * can synchronise the device.  It builds the cell records into a 64 MiB
 * file-scope device array that every GPU loading the library holds until exit,
 * then traces like sdfoam_trace_forward with the same io.  Foams whose records
 * exceed 64 MiB (sdfoam_cells_bytes; about 100k sites at SH degree 3 with 15
 * neighbours per site) are
 * rejected with SDFOAM_ERR_INVALID; an SH degree or foam size that no entry
 * point takes gets sdfoam_build_cells' code and message.  All calls share the
 * array: calls whose GPU work overlaps race and must be serialised by the
 * caller.  Every call looks up the array's device address on the current
 * device (so it stays valid after cudaDeviceReset); the first call on a device
 * also loads the library's module there, so make it before any stream
 * capture. */
SDFOAM_API int sdfoam_trace_forward_noalloc(const sdfoam_foam *foam,
                                            const sdfoam_trace_settings *settings,
                                            const sdfoam_forward_io *io,
                                            sdfoam_stream_t stream);

/* Message of the last failing call on this thread ("" if none). */
SDFOAM_API const char *sdfoam_last_error(void);

/* ABI version of this header. */
SDFOAM_API int sdfoam_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* SDFOAM_B200_H */
