/*
 * hexel_b200.h — C-ABI of the B200 (sm_100a) hexel / Image-GS rasteriser.
 *
 * Every entry point takes plain device pointers, element counts and a CUDA
 * stream, launches hand-written sm_100a kernels on that stream and returns an
 * hx_status.  None of them allocates device memory: outputs are written into
 * caller buffers and any scratch space is passed in as a "workspace" whose
 * size is reported by the matching *_workspace_bytes() query.  Layouts are the
 * reference's: row-major, fp32 unless stated, int32 ids, int64 intersection
 * keys.  Where a reference launcher returns zero-initialised tensors that its
 * kernel only partly writes, the kernel here writes every element itself, so
 * output buffers need no prior clearing unless the comment says so.
 *
 * Each declaration names the reference interface it replaces
 * (honeycomb-surfels/hexel-kernel, path:line).  Optional pointer arguments
 * are "absent" when NULL, mirroring the reference's empty-tensor convention.
 */
#ifndef HEXEL_B200_H
#define HEXEL_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#if defined(__GNUC__)
#define HX_API __attribute__((visibility("default")))
#else
#define HX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define HX_ABI_VERSION 1

enum hx_status {
    HX_OK = 0,
    HX_ERR_INVALID_ARGUMENT = 1, /* bad size, pointer or option */
    HX_ERR_CUDA = 2,             /* a CUDA runtime call or launch failed */
    HX_ERR_WORKSPACE = 3,        /* workspace missing or too small */
    HX_ERR_OVERFLOW = 4          /* a count does not fit in int32 */
};

/* ---- library ---------------------------------------------------------- */
HX_API int hx_abi_version(void);
/* Message describing the last failure on the calling host thread. */
HX_API const char* hx_last_error(void);
HX_API void hx_clear_error(void);
/* Number of kernels this library has launched since it was loaded. */
HX_API unsigned long long hx_launch_count(void);

/* ---- S1: 2D Gaussian projection ---------------------------------------- */

/* Replaces project_gaussians_2d_scale_rot_forward_tensor
 * (gsplat/cuda/csrc/bindings.cu:2746-2797) and its kernel
 * (gsplat/cuda/csrc/foward2d.cu:9-59).  means2d, scales2d: (N,2); rotation:
 * (N,).  Writes xys (N,2), radii (N,), conics (N,3), num_tiles_hit (N,); all
 * elements are written (zeros where the reference leaves its zero fill). */
HX_API int hx_project_gaussians_2d_scale_rot_forward(
    int num_points, const float* means2d, const float* scales2d, const float* rotation,
    unsigned img_height, unsigned img_width, int tiles_x, int tiles_y,
    float* xys, int32_t* radii, float* conics, int32_t* num_tiles_hit, cudaStream_t stream);

/* Replaces project_gaussians_2d_scale_rot_backward_tensor
 * (gsplat/cuda/csrc/bindings.cu:2800-2846; kernel backward2d.cu:53-100).
 * Writes v_cov2d (N,3), v_mean2d (N,2), v_scale (N,2), v_rot (N,); zeros for
 * culled points (radii <= 0). */
HX_API int hx_project_gaussians_2d_scale_rot_backward(
    int num_points, const float* means2d, const float* scales2d, const float* rotation,
    unsigned img_height, unsigned img_width, const int32_t* radii, const float* conics,
    const float* v_xy, const float* v_conic,
    float* v_cov2d, float* v_mean2d, float* v_scale, float* v_rot, cudaStream_t stream);

/* Replaces compute_cov2d_bounds_tensor (gsplat/cuda/csrc/bindings.cu:20-60).
 * covs2d (N,3) upper triangle -> conics (N,3), radii (N,) as float.  Rows
 * with a zero determinant get zeros (the reference leaves them undefined). */
HX_API int hx_compute_cov2d_bounds(int num_points, const float* covs2d, float* conics, float* radii,
                            cudaStream_t stream);

/* ---- S2 / S7: scan, intersection keys, radix sort, tile ranges ---------- */

/* Inclusive int32 prefix sum; replaces torch.cumsum(num_tiles_hit, int32)
 * (gsplat/utils.py:113) and cub::DeviceScan::InclusiveSum
 * (gsplat/cuda_hexels3d/csrc/hexels3d_forward.cu:2975-2981).  total_out
 * (device int64, may be NULL) receives the sum computed in 64 bits so that an
 * int32 overflow of the running sum can be detected by the caller. */
HX_API size_t hx_scan_workspace_bytes(int n);
HX_API int hx_inclusive_scan_i32(const int32_t* in, int32_t* out, int n, int64_t* total_out,
                          void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* hx_inclusive_scan_i32 without a workspace; it has no counterpart in the
 * reference.  For callers that cannot allocate device memory at the call
 * site: an FFI binding of this C-ABI that owns no device allocator, a process
 * whose device memory is held by a caching allocator (a raw cudaMalloc can
 * fail there although cached blocks are free), or code that must not
 * synchronise the device (cudaMalloc/cudaFree do).  The per-block partial
 * sums live in a fixed 64 KiB file-scope device array, so n is limited to
 * 67,108,864; larger n is rejected with HX_ERR_INVALID_ARGUMENT.  The first
 * call on each device (with that device current) looks the array's address
 * up once with cudaGetSymbolAddress and caches it; make that first call
 * before any stream capture.  All calls on a device share the array: calls
 * that overlap on one device (other streams or host threads) race and must be
 * serialised by the caller.  Nothing in the array needs clearing: each call
 * writes every entry it reads. */
HX_API int hx_inclusive_scan_i32_noalloc(const int32_t* in, int32_t* out, int n,
                                         int64_t* total_out, cudaStream_t stream);

/* Replaces map_gaussian_to_intersects_tensor (gsplat/cuda/csrc/bindings.cu:62-97;
 * kernel forward.cu:13-44).  Writes isect_ids (I,) = (tile << 32) | 0 and
 * gaussian_ids (I,) in Gaussian-major, tile-row-major order.  Writes are
 * bounded by num_intersects. */
HX_API int hx_map_gaussian_to_intersects(
    int num_points, int num_intersects, const float* xys, const int32_t* radii,
    const int32_t* cum_tiles_hit, int tiles_x, int tiles_y,
    int64_t* isect_ids, int32_t* gaussian_ids, cudaStream_t stream);

/* Stable LSD radix sort of (uint64 key, int32 value) pairs on key bits
 * [begin_bit, end_bit).  Replaces torch.sort + torch.gather of the 2D path
 * (gsplat/utils.py:159-160) and cub::DeviceRadixSort::SortPairs of the 3D
 * path (hexels3d_forward.cu:3011-3035).  Inputs are not modified. */
HX_API size_t hx_sort_pairs_workspace_bytes(int n, int key_bytes);
HX_API int hx_sort_pairs_u64(const uint64_t* keys_in, const int32_t* vals_in, uint64_t* keys_out,
                      int32_t* vals_out, int n, int begin_bit, int end_bit,
                      void* workspace, size_t workspace_bytes, cudaStream_t stream);
HX_API int hx_sort_pairs_u32(const uint32_t* keys_in, const int32_t* vals_in, uint32_t* keys_out,
                      int32_t* vals_out, int n, int begin_bit, int end_bit,
                      void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* Replaces get_tile_bin_edges_tensor (gsplat/cuda/csrc/bindings.cu:99-116;
 * kernel forward.cu:49-71).  tile_bins (num_tiles,2) is fully written:
 * [first, last+1) for occupied tiles, (0,0) for empty ones. */
HX_API int hx_get_tile_bin_edges(int num_intersects, int num_tiles, const int64_t* isect_ids_sorted,
                          int32_t* tile_bins, cudaStream_t stream);

/* Fused 2D binning used by rasterize_gaussians_sum: the composition of
 * map_gaussian_to_intersects, a stable sort by tile and get_tile_bin_edges
 * (gsplat/utils.py:118-162) without materialising 64-bit keys.  Produces
 * gaussian_ids_sorted (I,), tile_bins (num_tiles,2) and, if isect_ids_sorted
 * is not NULL, the sorted 64-bit keys.  Results are identical to the
 * reference's sorted lists (within a tile: ascending Gaussian id).
 * tile_row_begin/tile_row_end restrict emission to a horizontal stripe of
 * tile rows (pass 0 and tiles_y for the whole image); cum_tiles_hit must then
 * count only the stripe's tiles (see hx_count_tiles_2d). */
HX_API size_t hx_bin_gaussians_2d_workspace_bytes(int num_intersects, int num_tiles);
HX_API int hx_bin_gaussians_2d(
    int num_points, int num_intersects, const float* xys, const int32_t* radii,
    const int32_t* cum_tiles_hit, int tiles_x, int tiles_y, int tile_row_begin, int tile_row_end,
    int32_t* gaussian_ids_sorted, int32_t* tile_bins, int64_t* isect_ids_sorted,
    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* Per-Gaussian count of tiles in rows [tile_row_begin, tile_row_end) of its
 * tile rectangle (the same rectangle as map_gaussian_to_intersects); used to
 * shard an image into horizontal stripes of tile rows. */
HX_API int hx_count_tiles_2d(int num_points, const float* xys, const int32_t* radii, int tiles_x,
                      int tiles_y, int tile_row_begin, int tile_row_end, int32_t* counts,
                      cudaStream_t stream);

/* ---- S3: Image-GS compositing ------------------------------------------ */

/* Compositing kernels take num_points (N) and num_intersects (length of
 * gaussian_ids_sorted): tile ranges are clipped to the list and ids clamped
 * into [0, N), so malformed bins cannot make a kernel read out of bounds. */

/* Replaces nd_rasterize_forward_tensor (gsplat/cuda/csrc/bindings.cu:175-232;
 * kernel forward.cu:76-170) and rasterize_forward_tensor (bindings.cu:118-173,
 * channels == 3).  Plain sum of colour * exp(-sigma) per pixel.  channels <= 12.
 * out_img (H,W,C). */
HX_API int hx_nd_rasterize_forward(
    int tiles_x, int tiles_y, unsigned img_width, unsigned img_height, int channels,
    int num_points, int num_intersects, const int32_t* gaussian_ids_sorted, const int32_t* tile_bins, const float* xys,
    const float* conics, const float* colors, float* out_img, cudaStream_t stream);

/* Replaces nd_rasterize_backward_tensor (bindings.cu:234-308; kernel
 * backward.cu:23-157) and rasterize_backward_tensor (bindings.cu:2683-2744).
 * v_xy (N,2), v_conic (N,3), v_colors (N,C) are ACCUMULATED into: clear them
 * first. */
HX_API int hx_nd_rasterize_backward(
    int tiles_x, int tiles_y, unsigned img_width, unsigned img_height, int channels,
    int num_points, int num_intersects, const int32_t* gaussian_ids_sorted, const int32_t* tile_bins, const float* xys,
    const float* conics, const float* colors, const float* v_output,
    float* v_xy, float* v_conic, float* v_colors, cudaStream_t stream);

/* Replaces nd_rasterize_forward_topk_norm_tensor and _stats_tensor
 * (bindings.cu:310-444; kernel forward.cu:172-320).  Top-10 normalised
 * weighted sum.  out_img (H,W,C), pixel_topk (H,W,10) int32 (-1 = empty);
 * weights_sum (H,W) and entropy (H,W) are optional. */
HX_API int hx_nd_rasterize_forward_topk_norm(
    int tiles_x, int tiles_y, unsigned img_width, unsigned img_height, int channels,
    int num_points, int num_intersects, const int32_t* gaussian_ids_sorted, const int32_t* tile_bins, const float* xys,
    const float* conics, const float* colors, float* out_img, int32_t* pixel_topk,
    float* weights_sum, float* entropy, cudaStream_t stream);

/* Replaces nd_rasterize_backward_topk_norm_tensor and _stats_tensor
 * (bindings.cu:446-565; kernel backward.cu:159-316).  v_weights_sum and
 * v_entropy (H,W) are optional.  Gradients are ACCUMULATED: clear them first. */
HX_API int hx_nd_rasterize_backward_topk_norm(
    unsigned img_width, unsigned img_height, int channels, int num_points, const float* xys,
    const float* conics, const float* colors, const float* v_output,
    const float* v_weights_sum, const float* v_entropy, const int32_t* pixel_topk,
    float* v_xy, float* v_conic, float* v_colors, cudaStream_t stream);

/* hx_nd_rasterize_backward_topk_norm over pixel rows [row_begin, row_end)
 * only (no reference counterpart; 0 <= row_begin <= row_end <= H): the
 * backward of one stripe of tile rows (rasterize_gaussians_sum(tile_rows=)),
 * which reads none of the per-pixel inputs outside the stripe.  Buffers are
 * the whole image's, as above. */
HX_API int hx_nd_rasterize_backward_topk_norm_rows(
    unsigned img_width, unsigned img_height, int channels, int num_points, const float* xys,
    const float* conics, const float* colors, const float* v_output,
    const float* v_weights_sum, const float* v_entropy, const int32_t* pixel_topk,
    int row_begin, int row_end, float* v_xy, float* v_conic, float* v_colors,
    cudaStream_t stream);

/* ---- S4: tile-less Image-GS -------------------------------------------- */

/* Replaces nd_rasterize_forward_no_tiles_tensor (bindings.cu:2459-2510;
 * kernel forward.cu:322-410). */
HX_API int hx_nd_rasterize_forward_no_tiles(
    unsigned img_width, unsigned img_height, int channels, int num_points, const float* xys,
    const float* conics, const float* colors, float* out_img, int32_t* pixel_topk,
    cudaStream_t stream);

/* Replaces nd_rasterize_backward_no_tiles_tensor (bindings.cu:2512-2565;
 * kernel backward.cu:318-438).  Gradients are ACCUMULATED: clear them first. */
HX_API int hx_nd_rasterize_backward_no_tiles(
    unsigned img_width, unsigned img_height, int channels, int num_points, const float* xys,
    const float* conics, const float* colors, const float* v_output, const int32_t* pixel_topk,
    float* v_xy, float* v_conic, float* v_colors, cudaStream_t stream);

/* ---- S5: 2D image hexels ------------------------------------------------ */

/* One entry point for the eight forward variants
 * nd_rasterize_forward_topk_norm_hexels[_color_grad][_affine][_softness]
 * (gsplat/cuda/csrc/bindings.cu:566-2457; kernels hexels_forward.cu:169-859).
 * Geometry: scales (N,2) + rotation (N,) when affines is NULL, else affines
 * (N,2,2) in the row-vector convention.  color_grads (N,2,C) selects the
 * linear colour-gradient variant.  softnesses (N,) or (N,3) with
 * softness_stride 1 or 3, or NULL to use softness_default.  sharpness (N,) and
 * emission (N,C) optional.  Writes out_img (H,W,C), pixel_topk (H,W,10) and,
 * if given, weights_sum and entropy (H,W). */
HX_API int hx_hexels2d_forward(
    int tiles_x, int tiles_y, unsigned img_width, unsigned img_height, int channels,
    int num_points, int num_intersects, const int32_t* gaussian_ids_sorted, const int32_t* tile_bins,
    const float* xys, const float* scales, const float* rotation, const float* affines,
    const float* colors, const float* color_grads, float color_grad_scale, float aa_kernel_size,
    const float* softnesses, int softness_stride, float softness_default, const float* sharpness,
    const float* emission, float* out_img, int32_t* pixel_topk, float* weights_sum,
    float* entropy, cudaStream_t stream);

/* One entry point for the eight backward variants (bindings.cu:911-2457;
 * kernels hexels_backward.cu:233-1387).  Gradient outputs are ACCUMULATED
 * (clear them first): v_xy (N,2); v_scale (N,2) + v_rot (N,) or v_affines
 * (N,4); v_colors (N,C); v_color_grads (N,2,C) with color_grads; v_emission
 * (N,C) with emission; v_sharpness (N,) with sharpness; v_softnesses shaped
 * like softnesses. */
HX_API int hx_hexels2d_backward(
    unsigned img_width, unsigned img_height, int channels, int num_points, const float* xys,
    const float* scales, const float* rotation, const float* affines, const float* colors,
    const float* color_grads, float color_grad_scale, const float* emission,
    const float* v_output, const float* v_weights_sum, const float* v_entropy,
    const int32_t* pixel_topk, float aa_kernel_size, const float* softnesses, int softness_stride,
    float softness_default, const float* sharpness, float* v_xy, float* v_scale, float* v_rot,
    float* v_affines, float* v_colors, float* v_color_grads, float* v_emission,
    float* v_sharpness, float* v_softnesses, cudaStream_t stream);

/* ---- S6-S8: 3D hexel surfels ------------------------------------------- */

/* Per-surfel preprocessing; replaces the kernel preprocess_hexels3d and its
 * launch (gsplat/cuda_hexels3d/csrc/hexels3d_forward.cu:372-551, 2940-2972).
 * rotations are WXYZ quaternions (P,4); softnesses (P,) or (P,3) with
 * softness_stride 1 or 3, or NULL to use softness_default (stride 1).
 * Writes radii (P,), tile_radii (P,2), points_xy_image (P,2),
 * points_xy_center (P,2; only with prefilter_edge_on, else may be NULL),
 * depths (P,), transMats (P,9), tiles_touched (P,), opacities_out (P,),
 * softnesses_out (P,) or (P,3), view_dirs (P,3) and, if not NULL, normals
 * (P,3).  Every element is written (zeros for culled surfels). */
HX_API int hx_hexels3d_preprocess(
    int P, const float* means3d, const float* scales, float scale_modifier,
    const float* rotations, const float* opacities, const float* softnesses,
    float softness_default, int softness_stride, const float* viewmatrix,
    const float* projmatrix, const float* campos, int image_width, int image_height,
    int prefilter_edge_on, int conservative_bounds, int32_t* radii, int32_t* tile_radii,
    float* points_xy_image, float* points_xy_center, float* depths, float* transMats,
    int32_t* tiles_touched, float* opacities_out, float* softnesses_out, float* view_dirs,
    float* normals, cudaStream_t stream);

/* Depth-ordered binning, the same sorted lists as hx_hexels3d_bin with far
 * less sorting; together the two calls replace the scan, duplicate_with_keys,
 * cub::DeviceRadixSort::SortPairs and identify_tile_ranges
 * (hexels3d_forward.cu:553-604, 2972-3043).
 * hx_hexels3d_depth_order: order (P,) = surfel ids stably sorted by depth
 * bits; offsets (P,) = inclusive scan of tiles_touched taken in that order;
 * total_out (device int64) = num_rendered.
 * hx_hexels3d_bin_ordered: emits each surfel's tiles in that order, stably
 * sorts the tile indices and writes point_list (I,) and ranges (tiles,2)
 * (zeros for empty tiles); keys_sorted (I,) int64 (tile << 32 | depth bits)
 * is optional (NULL to skip; needs depths).  Within a tile the order is
 * depth bits then surfel id -- the reference's stable (tile, depth) order. */
HX_API size_t hx_hexels3d_depth_order_workspace_bytes(int P);
HX_API int hx_hexels3d_depth_order(int P, const float* depths, const int32_t* tiles_touched,
                                   int32_t* order, int32_t* offsets, int64_t* total_out,
                                   void* workspace, size_t workspace_bytes, cudaStream_t stream);
HX_API size_t hx_hexels3d_bin_ordered_workspace_bytes(int num_rendered);
HX_API int hx_hexels3d_bin_ordered(int P, int num_rendered, int image_width, int image_height,
                                   const float* points_xy_image, const int32_t* order,
                                   const int32_t* offsets, const int32_t* radii,
                                   const int32_t* tile_radii, const float* depths,
                                   int64_t* keys_sorted, int32_t* point_list, int32_t* ranges,
                                   void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* Depth order and binning of a group of V views of one scene at once (no
 * reference counterpart: the reference bins one view per call,
 * hexels3d_forward.cu:2972-3043).  Inputs are the preprocess outputs of the
 * V views stacked view-major ((V, P) arrays).  depth_order_views sorts all
 * V x P entries by (view, depth bits), stable, so each view's entries are
 * contiguous and in that view's own depth order; order holds
 * view * P + surfel; offsets and total_out are the inclusive prefix sum of
 * the tile counts in that order over all views (one read-back per group).
 * bin_views then emits key view * tiles + tile for every tile of each entry's
 * rectangle with the surfel index within its view as value, sorts stably
 * and writes ranges (V, tiles, 2) as offsets into the group's point_list:
 * view v's lists are exactly those hx_hexels3d_bin_ordered gives for v
 * alone, shifted by the entries of views 0..v-1, so the compositing calls of
 * view v take ranges + 2 * v * tiles, the whole point_list and its total as
 * num_rendered. */
HX_API size_t hx_hexels3d_depth_order_views_workspace_bytes(int views, int P);
HX_API int hx_hexels3d_depth_order_views(int views, int P, const float* depths,
                                         const int32_t* tiles_touched, int32_t* order,
                                         int32_t* offsets, int64_t* total_out, void* workspace,
                                         size_t workspace_bytes, cudaStream_t stream);
HX_API size_t hx_hexels3d_bin_views_workspace_bytes(int num_rendered);
HX_API int hx_hexels3d_bin_views(int views, int P, int num_rendered, int image_width,
                                 int image_height, const float* points_xy_image,
                                 const int32_t* order, const int32_t* offsets,
                                 const int32_t* radii, const int32_t* tile_radii,
                                 int32_t* point_list, int32_t* ranges, void* workspace,
                                 size_t workspace_bytes, cudaStream_t stream);

/* Intersection emission, stable sort and tile ranges; replaces
 * duplicate_with_keys + cub::DeviceRadixSort::SortPairs + identify_tile_ranges
 * (hexels3d_forward.cu:553-604, 2990-3043).  offsets = inclusive scan of
 * tiles_touched; num_rendered its total.  Writes keys_sorted (I,) int64
 * (tile << 32 | depth bits), point_list (I,) and ranges (tiles,2) (zeros for
 * empty tiles). */
HX_API size_t hx_hexels3d_bin_workspace_bytes(int num_rendered);
HX_API int hx_hexels3d_bin(int P, int num_rendered, int image_width, int image_height,
                           const float* points_xy_image, const float* depths,
                           const int32_t* offsets, const int32_t* radii,
                           const int32_t* tile_radii, int64_t* keys_sorted,
                           int32_t* point_list, int32_t* ranges, void* workspace,
                           size_t workspace_bytes, cudaStream_t stream);

/* Front-to-back compositing; replaces render_hexels3d<S,F,O> and its launches
 * (hexels3d_forward.cu:610-1011, 3047-3467).  out_color (3,H,W).  Optional
 * outputs (NULL = not requested): contrib (P,), overdraw and overdraw_hits
 * (H,W); surface outputs out_depth, out_alpha (H,W) and out_surface (4 or 5,
 * H,W) (needs normals); owner outputs (owner_id int64, weight, uv (2,H,W),
 * sdf, depth, total alpha); final_T and last_index (H,W) for the RGB
 * backward; final_T_surf, last_index_surf, m1_surf, m2_surf, median_index
 * (H,W) for the surface backward.  points_xy_center non-NULL selects the
 * prefilter path.  contrib_count (2,H,W int32, may be NULL; no reference
 * counterpart) receives per pixel the number of blended (pixel, surfel)
 * pairs (plane 0, the work unit of the backward traversal) and of the pairs
 * evaluated after the warp's box cull (plane 1, the forward's work).
 * records (may be NULL) are hx_hexels3d_surfel_records' output for the same
 * inputs and settings.  blend_mask (num_rendered uint8,
 * may be NULL; no reference counterpart) receives, per sorted intersection of
 * every list entry the traversal staged, bit w (w = 2 * (y / 4) + x / 8 for
 * the pixel (x, y) within its 16x16 tile) set when a pixel of that 8x4 block
 * still compositing met the surfel with alpha >= (1 - 1e-4) / 255: a superset
 * of the pairs the backward blends, which hx_hexels3d_render_backward uses to
 * skip the others. */
HX_API int hx_hexels3d_render_forward(
    int P, int num_rendered, const int32_t* ranges, const int32_t* point_list,
    const float* points_xy_center, int image_width, int image_height, const float* colors,
    const float* color_grads, const float* color_quads, const float* view_grads,
    const float* specular_ks, const float* specular_log_s, const float* view_dirs,
    const float* transMats, const float* opacities, const float* softnesses,
    int softness_stride, const float* background, const float* normals, int overdraw_base_count,
    int color_model, int view_model, int use_view_grads, int return_median_depth,
    float* out_color, float* contrib, float* overdraw, float* overdraw_hits, float* out_depth,
    float* out_alpha, float* out_surface, int64_t* owner_id, float* owner_weight,
    float* owner_uv, float* owner_sdf, float* owner_depth, float* total_alpha, float* final_T,
    int32_t* last_index, float* final_T_surf, int32_t* last_index_surf, float* m1_surf,
    float* m2_surf, int32_t* median_index, int32_t* contrib_count, uint8_t* blend_mask,
    const void* records, cudaStream_t stream);

/* Exact-sort and pixel-risk diagnostics; together with the library's
 * preprocess and binning they replace rasterize_hexels3d_exact_sort_forward
 * and rasterize_hexels3d_pixel_risk_forward (hexels3d_forward.cu:4217-4880)
 * and their kernels (1069-1747).  Shared arguments: the binned view (P,
 * num_rendered, ranges, point_list), the per-surfel arrays of the
 * compositing (colors ... softnesses; normals for the lobe view model),
 * background (3), center_depths (P; the preprocess depths), selected_mask (P
 * uint8, may be NULL), pixel_mask (H x W uint8, exact_mode 5 only), the
 * colour and view models, exact_mode 0..5 (centre replay, hybrid, selected
 * all, crop all, boundary tail, pixel mask) and the crop [x0,x1) x [y0,y1).
 * exact_count: per crop pixel the number of hits (alpha >= 1/255),
 * record_counts (the hits of enabled pixels, else 0) and enabled; with
 * risk_map (H x W float, may be NULL) also the inversion risk of the list
 * order.  The caller scans record_counts (inclusive, record_offsets) and
 * calls exact_resolve with the total: it sorts each enabled pixel's hit
 * records by (pixel, depth at the pixel or centre depth, per mode) stably,
 * writes order_changed (H x W uint8) and the colour composited in that
 * order into out_color (3 x H x W; other pixels untouched). */
HX_API int hx_hexels3d_exact_count(
    int P, int num_rendered, const int32_t* ranges, const int32_t* point_list, int image_width,
    int image_height, const float* colors, const float* color_grads, const float* color_quads,
    const float* view_grads, const float* specular_ks, const float* specular_log_s,
    const float* view_dirs, const float* normals, const float* transMats,
    const float* opacities, const float* softnesses, int softness_stride,
    const float* background, const float* center_depths, const uint8_t* selected_mask,
    const uint8_t* pixel_mask, int color_model, int view_model, int use_view_grads,
    int exact_mode, int crop_x0, int crop_y0, int crop_x1, int crop_y1, int32_t* hit_counts,
    int32_t* record_counts, uint8_t* enabled, float* risk_map, cudaStream_t stream);
HX_API size_t hx_hexels3d_exact_resolve_workspace_bytes(int num_records);
HX_API int hx_hexels3d_exact_resolve(
    int P, int num_rendered, const int32_t* ranges, const int32_t* point_list, int image_width,
    int image_height, const float* colors, const float* color_grads, const float* color_quads,
    const float* view_grads, const float* specular_ks, const float* specular_log_s,
    const float* view_dirs, const float* normals, const float* transMats,
    const float* opacities, const float* softnesses, int softness_stride,
    const float* background, const float* center_depths, const uint8_t* selected_mask,
    const uint8_t* pixel_mask, int color_model, int view_model, int use_view_grads,
    int exact_mode, int crop_x0, int crop_y0, int crop_x1, int crop_y1, const uint8_t* enabled,
    const int32_t* record_counts, const int32_t* record_offsets, int num_records,
    float* out_color, uint8_t* order_changed, void* workspace, size_t workspace_bytes,
    cudaStream_t stream);

/* Per-surfel staged records for the compositing pair (no reference
 * counterpart: the reference gathers every field from its arrays for every
 * list entry, hexels3d_forward.cu:673-760).  Writes, for each of the P
 * surfels, the 128-byte record the compositing kernels stage into shared
 * memory -- transform rows, opacity, softnesses, base colour, linear view
 * colour, colour gradients, viewer-facing normal (surface), the pixel box
 * outside which alpha < 1/255 (or the prefilter centre) and the id -- into
 * `records` (P x 128 bytes, 16-byte aligned).  Passing it as `records` to
 * hx_hexels3d_render_forward / _backward lets each list entry be staged with
 * asynchronous 16-byte copies instead of gathered and recomputed; the
 * records must come from the same per-surfel inputs, colour model,
 * use_view_grads, surface and prefilter settings as those calls (both may
 * also be given NULL, gathering as before). */
HX_API int hx_hexels3d_surfel_records(
    int P, int image_width, int image_height, const float* transMats, const float* opacities,
    const float* softnesses, int softness_stride, const float* colors, const float* color_grads,
    const float* view_grads, const float* view_dirs, const float* normals,
    const float* points_xy_center, int color_model, int use_view_grads, int surface,
    void* records, cudaStream_t stream);

/* Reverse traversal VJP; replaces render_hexels3d_backward<S,F> and its
 * launches (hexels3d_forward.cu:1749-2492, 5323-5505).  Uses the forward's
 * saved final_T/last_index (and the surface state when surface gradients are
 * given).  All gradient outputs are ACCUMULATED (clear them first);
 * grad_transMats (P,9), grad_view_dirs (P,3) and grad_normals (P,3) are
 * intermediates for hx_hexels3d_geometry_backward.  blend_mask (may be NULL)
 * is the forward's per-intersection mask of the same call's lists: list
 * entries whose bits are clear for a warp's pixel block are skipped. */
HX_API int hx_hexels3d_render_backward(
    int P, int num_rendered, const int32_t* ranges, const int32_t* point_list,
    const float* points_xy_center, float* grad_points_xy_center, int image_width,
    int image_height, const float* colors, const float* color_grads, const float* color_quads,
    const float* view_grads, const float* specular_ks, const float* specular_log_s,
    int view_model, const float* view_dirs, const float* transMats, const float* opacities,
    const float* softnesses, int softness_stride, const float* background,
    const float* grad_out_color, const float* grad_out_overdraw,
    const float* grad_out_surf_depth, const float* grad_out_surf_alpha,
    const float* grad_out_surf_normals, int has_median_grad, const float* normals,
    float* grad_colors, float* grad_color_grads, float* grad_color_quads, float* grad_view_grads,
    float* grad_specular_ks, float* grad_specular_log_s, float* grad_opacities,
    float* grad_softnesses, float* grad_transMats, float* abs_means2d, float* grad_view_dirs,
    float* grad_normals, int overdraw_base_count, int color_model, int use_view_grads,
    const float* final_T, const int32_t* last_index, const float* final_T_surf,
    const int32_t* last_index_surf, const float* m1_surf, const float* m2_surf,
    const int32_t* median_index, const uint8_t* blend_mask, const void* records,
    cudaStream_t stream);

/* VJP from transforms (and view directions / normals) to means3d, scales and
 * WXYZ rotations, plus the screen-gradient proxy for means2d and the
 * prefilter-centre VJP; replaces transmat_to_geometry_backward,
 * transmat_to_means2d_backward and points_xy_center_to_means3d_backward
 * (hexels3d_forward.cu:2494-2664).  grad_means3d, grad_scales and
 * grad_rotations are written for visible surfels and must be zeroed first;
 * grad_means2d (P, means2d_stride) may be NULL.  With accumulate != 0 the
 * gradients are added to the buffers' contents instead (gradient
 * accumulation over views; no reference counterpart). */
HX_API int hx_hexels3d_geometry_backward(
    int P, int num_rendered, const float* means3d, const float* scales, float scale_modifier,
    const float* rotations, const float* projmatrix, const float* campos, int image_width,
    int image_height, const int32_t* radii, const float* transMats, const float* grad_transMats,
    const float* grad_view_dirs, const float* grad_normals, const float* grad_points_xy_center,
    float* grad_means3d, float* grad_means2d, int means2d_stride, float* grad_scales,
    float* grad_rotations, int accumulate, cudaStream_t stream);

/* Mean-squared-error loss of a fit step in one pass (no reference
 * counterpart; the reference's training loops form it with torch ops):
 * grad[i] = (pred[i] - target[i]) * 2 inv_n, and sum_i (pred[i] - target[i])^2
 * inv_n is ADDED to *loss (clear it first; the order of the float additions
 * across CTAs is not fixed).  n >= 0; 16-byte aligned inputs take a vector path. */
HX_API int hx_l2_loss_grad(const float* pred, const float* target, int64_t n, float inv_n,
                           float* grad, float* loss, cudaStream_t stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* HEXEL_B200_H */
