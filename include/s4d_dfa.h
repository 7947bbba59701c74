/*
 * s4d_dfa.h -- C ABI of the B200 (sm_100a) DeformableFeatureAggregation hot path.
 *
 * Three operators, each a set of hand-written CUDA kernels:
 *
 *   s4d_kps_project            anchor decode -> 7 fixed + N learnable keypoints -> yaw rotation
 *                              -> per-camera lidar2img projection -> depth clamp and
 *                              normalisation -> depth mask, frustum mask and the compacted
 *                              list of visible (batch, anchor, camera, point) indices.
 *   s4d_deformable_aggregation softmax of the weight logits over camera x level x point per
 *                              group, fused with the multi-camera, multi-scale bilinear gather
 *                              (zeros padding, align_corners=False) and the weighted sum over
 *                              cameras, levels and points.
 *   s4d_dfa_weights_fc /       the dense linears before and after the gather on the tensor
 *   s4d_dfa_output_proj        cores (tcgen05), with the embed add and the residual fused.
 *
 * Conventions
 *   - Every pointer is a DEVICE pointer of the current CUDA device unless stated otherwise.
 *     The library never allocates or frees: the caller owns every input, output and workspace.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).  Calls are
 *     asynchronous and stream-ordered; nothing here synchronises the host.  Calls on different
 *     streams from different host threads are safe.  Small launches of s4d_dfa_weights_fc,
 *     s4d_dfa_output_proj(_sum) and the gathers (one frame: one wave of CTAs) use programmatic
 *     dependent launch.  Their CTAs may start before the preceding kernel in the stream ends,
 *     but they touch no global memory until it has completed, so stream order still holds for
 *     every read and write.
 *   - Every entry point returns an s4d_status; nothing throws and no kernel traps.  Shapes are
 *     checked on the host before any launch.  The text of the last failure on the calling
 *     thread is returned by s4d_last_error().
 *   - Integer sizes are int64_t; element counts of one call must stay below 2^31.
 */
#ifndef S4D_DFA_H_
#define S4D_DFA_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define S4D_API __attribute__((visibility("default")))
#else
#define S4D_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum s4d_status {
  S4D_OK = 0,
  S4D_ERR_INVALID_ARG = 1,       /* null pointer, negative size, bad enum value */
  S4D_ERR_UNSUPPORTED_SHAPE = 2, /* valid but outside what the kernels implement */
  S4D_ERR_CUDA = 3,              /* a CUDA runtime call or launch failed */
  S4D_ERR_DEVICE_FAULT = 4       /* a kernel reported bad device-side data via error_flag */
} s4d_status;

/* Feature element types of mc_ms_feat. */
enum { S4D_DTYPE_F32 = 0, S4D_DTYPE_BF16 = 1 };

/* Index layouts of sample_location and weights.
 *   CAM_MAJOR (native):  sample_location [bs, A, Ncam, P, 2]; weights [bs, A, Ncam, L, P, G]
 *                        (the order weights_fc produces, test/dfa_pcc.py:314-318).
 *   PT_MAJOR (upstream Sparse4D deformable_aggregation op order):
 *                        sample_location [bs, A, P, Ncam, 2]; weights [bs, A, P, Ncam, L, G].
 *   GRID (s4d_kps_project output only): grid [Ncam, bs*A, P, 2] holding 2*uv - 1 clamped to
 *                        [-2, 2], the output page order of ttnn.kps_project_fused
 *                        (tt-metal/ops/kps_project_fused/device/kernels/dataflow/
 *                        writer_kps_project.cpp:43-45). */
enum { S4D_LAYOUT_CAM_MAJOR = 0, S4D_LAYOUT_PT_MAJOR = 1, S4D_LAYOUT_GRID = 2 };

/* Bits of the optional device error_flag (OR-ed by kernels, never cleared by them). */
enum {
  S4D_FLAG_BAD_LEVEL = 1,   /* a (camera, level) spatial_shape / scale_start_index entry lies
                               outside mc_ms_feat; its samples were skipped */
  S4D_FLAG_WAIT_TIMEOUT = 2, /* a tensor-core kernel gave up waiting on one of its own pipeline
                               barriers (after 2 s, or the limit set by s4d_set_tc_wait_limit_ns);
                               its outputs were not written.  Never expected at the default limit. */
  S4D_FLAG_PEER_TIMEOUT = 4  /* s4d_peer_signal_wait gave up waiting for a peer's epoch; what the
                               launches after it read from that peer is not that epoch's data */
};

/* Layouts of the per-level maps s4d_pack_feature_maps reads. */
enum { S4D_MAPS_NCHW = 0 /* [bs, Ncam, C, H, W] */, S4D_MAPS_NHWC = 1 /* [bs, Ncam, H, W, C] */ };

/* Residual modes of s4d_dfa_output_proj (the reference module's residual_mode). */
enum { S4D_RESIDUAL_NONE = 0, S4D_RESIDUAL_ADD = 1, S4D_RESIDUAL_CAT = 2 };

/* Human-readable name of a status code. */
S4D_API const char* s4d_status_string(int status);

/* Text of the last non-OK status returned on the calling thread ("" if none). */
S4D_API const char* s4d_last_error(void);

/* Version of this ABI (major * 100 + minor). */
S4D_API int s4d_abi_version(void);

/*
 * Failure detection of the tensor-core kernels (s4d_dfa_weights_fc, s4d_dfa_output_proj).  Their
 * pipeline barrier waits (the TMA producer on a free stage, the MMA issuer on a loaded stage, the
 * epilogue on the accumulator) give up after this many nanoseconds, set S4D_FLAG_WAIT_TIMEOUT in
 * the call's error_flag and leave the outputs unwritten; the CTA still waits (up to 2 s) for the
 * copies and MMAs it already issued before it frees tensor memory and exits, so the context stays
 * usable.  Applies to launches from the calling host thread; default 2,000,000,000 (2 s).  A test
 * sets it to 0 to make the waits run out.  Returns the previous limit.  No counterpart in the
 * reference (its device waits have no limit).
 */
S4D_API uint64_t s4d_set_tc_wait_limit_ns(uint64_t limit_ns);

/* Bytes of device workspace s4d_kps_project needs when it compacts visible indices
 * (visible_idx or visible_count non-NULL).  Host-only, launches nothing. */
S4D_API size_t s4d_kps_workspace_bytes(int64_t bs, int64_t num_anchor, int64_t num_cams, int64_t num_pts);

/*
 * Keypoint generation + projection + visibility compaction.
 *
 * Replaces ttnn.kps_project_fused (tt-metal/ops/kps_project_fused/kps_project_fused.hpp:12-22)
 * together with the keypoint generator it consumes (model/deformable_feature_aggregation.py:
 * 651-677) and the reference's PyTorch _KPSGenerator + project_points
 * (test/dfa_pcc.py:225-247,322-333).
 *
 * Inputs
 *   anchor          [bs, A, anchor_dim] f32, anchor_dim >= 8: x y z log(w) log(l) log(h) sin cos ...
 *   fix_scale       [num_fix, 3] f32 fixed keypoint scales (may be NULL when num_fix == 0)
 *   learnable       [bs, A, num_learnable * 3] f32 learnable_fc outputs BEFORE the sigmoid
 *                   (may be NULL when num_learnable == 0)
 *   projection_mat  [bs, Ncam, 4, 4] f32 lidar2img
 *   image_wh        [bs, Ncam, 2] f32 (width, height)
 *   P = num_fix + num_learnable keypoints per anchor.
 * Outputs (each may be NULL to skip it)
 *   key_points      [bs, A, P, 3] f32
 *   sample_location CAM_MAJOR [bs, A, Ncam, P, 2] / PT_MAJOR [bs, A, P, Ncam, 2]: (u, v) =
 *                   xy / max(z, 1e-5) / image_wh, unclamped; or GRID layout (see above)
 *   depth_mask      [bs, A, Ncam, P] u8: 1 where z > 1e-5
 *   visible_idx     [bs*A*Ncam*P, 4] i32 rows (b, a, cam, pt) of every visible point
 *                   (z > 1e-5 and 0 <= u, v <= 1), lexicographic like torch.nonzero; only the
 *                   first *visible_count rows are written
 *   visible_count   [1] i32
 *   workspace       >= s4d_kps_workspace_bytes(...) bytes, 16-byte aligned; required when
 *                   visible_idx or visible_count is non-NULL, otherwise may be NULL
 */
S4D_API int s4d_kps_project(const float* anchor, int64_t anchor_dim, const float* fix_scale, int64_t num_fix,
                    const float* learnable, int64_t num_learnable, const float* projection_mat,
                    const float* image_wh, int64_t bs, int64_t num_anchor, int64_t num_cams, int layout,
                    float* key_points, float* sample_location, uint8_t* depth_mask, int32_t* visible_idx,
                    int32_t* visible_count, void* workspace, size_t workspace_bytes, void* stream);

/* s4d_kps_project with the learnable keypoint logits computed in the kernel from the instance
 * feature: logit[n, o] = learnable_fc_bias[o] + instance_feature[n, :] . learnable_fc_weight[o, :]
 * (fp32), the keypoint generator's learnable_fc (model/deformable_feature_aggregation.py:651-677,
 * test/dfa_pcc.py:231-233) fused with the projection.  The call then depends only on the layer's
 * inputs, not on another linear's output.
 *   instance_feature    [bs * A, embed_dims] rows of stride instance_ld (floats), 16-byte aligned
 *   learnable_fc_weight [num_learnable * 3, embed_dims], 16-byte aligned; learnable_fc_bias or NULL
 * instance_ld is a multiple of 4.  Implemented: embed_dims 256, num_learnable <= 10,
 * Ncam * P >= 57 (Sparse4D: 6 * 13).  Other arguments as s4d_kps_project. */
S4D_API int s4d_kps_project_linear(const float* anchor, int64_t anchor_dim, const float* fix_scale, int64_t num_fix,
                                   const float* instance_feature, int64_t instance_ld,
                                   const float* learnable_fc_weight, const float* learnable_fc_bias,
                                   int64_t num_learnable, int64_t embed_dims, const float* projection_mat,
                                   const float* image_wh, int64_t bs, int64_t num_anchor, int64_t num_cams,
                                   int layout, float* key_points, float* sample_location, uint8_t* depth_mask,
                                   int32_t* visible_idx, int32_t* visible_count, void* workspace,
                                   size_t workspace_bytes, void* stream);

/*
 * s4d_kps_project without a workspace, for callers that cannot allocate device memory (an FFI
 * host without a CUDA allocator, a fixed device-memory budget, a loop that must not allocate
 * after start-up).  No counterpart in the reference.
 *
 * Same arguments and results as s4d_kps_project minus workspace/workspace_bytes.  The
 * compaction scratch is a 528 KiB array compiled into the library (held on every GPU that
 * loads the library until exit), so bs*A*Ncam*P is limited to 4,194,304 elements; larger calls
 * return S4D_ERR_UNSUPPORTED_SHAPE.  Every call looks the array's device address up
 * (cudaGetSymbolAddress) on the current device, so nothing goes stale across a device reset;
 * the first call in a context may load the library's device code there, so make it before
 * any stream capture.  All calls share the array: calls that overlap on the GPU race.
 * Allocates nothing.
 */
S4D_API int s4d_kps_project_noalloc(const float* anchor, int64_t anchor_dim, const float* fix_scale,
                                    int64_t num_fix, const float* learnable, int64_t num_learnable,
                                    const float* projection_mat, const float* image_wh, int64_t bs,
                                    int64_t num_anchor, int64_t num_cams, int layout, float* key_points,
                                    float* sample_location, uint8_t* depth_mask, int32_t* visible_idx,
                                    int32_t* visible_count, void* stream);

/*
 * Drop-in of ttnn.kps_project_fused in its standard mode
 * (tt-metal/ops/kps_project_fused/kps_project_fused.hpp:12-22, kernel
 * .../dataflow/reader_kps_project.cpp:255-289): pre-rotation keypoints in, normalised grid out.
 *
 *   key_points      [n, P, 3] f32 pre-rotation keypoints (fixed and learnable, times size)
 *   anchor          [n, anchor_dim] f32 (yaw and centre are read from it)
 *   projection_mat  [Ncam, 4, 4] f32, image_wh [Ncam, 2] f32
 *   grid            [Ncam, n, P, 2] f32 = clamp(2 * uv - 1, -2, 2)
 * The reference reads keypoints and anchors as bf16; this reads and computes in f32.
 */
S4D_API int s4d_kps_project_fused(const float* key_points, const float* anchor, int64_t anchor_dim,
                          const float* projection_mat, const float* image_wh, int64_t n, int64_t num_cams,
                          int64_t num_pts, float* grid, void* stream);

/*
 * Fused softmax + multi-camera multi-scale bilinear gather + weighted sum.
 *
 * Replaces ttnn.grid_sample + ttnn.transposed_s2i
 * (tt-metal/ops/transposed_s2i/transposed_s2i.hpp:10-13) + ttnn.grouped_weighted_sum
 * (tt-metal/ops/grouped_weighted_sum/grouped_weighted_sum.hpp:11-16) + the ttnn.softmax of
 * model/deformable_feature_aggregation.py:791-796, i.e. the reference's PyTorch
 * feature_sampling + multi_view_level_fusion + sum over points (test/dfa_pcc.py:298,335-358).
 * Argument meaning follows upstream Sparse4D's deformable_aggregation(mc_ms_feat,
 * spatial_shape, scale_start_index, sample_location, weights).
 *
 *   mc_ms_feat        [bs, num_feat, C] channels-last features, f32 or bf16 (feat_dtype);
 *                     pixel (y, x) of camera c, level l is row scale_start_index[c, l] + y*W + x
 *   spatial_shape     [Ncam, L, 2] i32 (H, W)
 *   scale_start_index [Ncam, L] i32
 *   sample_location   see layout; (u, v) in [0, 1] inside the image
 *   weights           see layout.  With weights_cam != NULL (CAM_MAJOR only) the logits are
 *                     split: weights [bs, A, L, P, G] is the per-anchor term and weights_cam
 *                     [bs, Ncam, L, P, G] the per-camera term; logit = weights + weights_cam.
 *   weights_are_logits 1: softmax over (cam, level, pt) per group first (over ALL Ncam cameras
 *                     even when [cam_begin, cam_end) is a sub-range); 0: use as given;
 *                     2: as 1, split logits whose per-frame camera factors are already in the
 *                     workspace (from s4d_dfa_camera_factors; the Sparse4D v3 shape only)
 *   cam_begin/cam_end only cameras in [cam_begin, cam_end) are sampled (camera sharding)
 *   out               [bs, A, C] f32, summed over points
 *   error_flag        optional [1] i32, OR-ed with S4D_FLAG_* bits
 *   workspace         optional, >= s4d_dfa_workspace_bytes(...) bytes, 16-byte aligned.  With
 *                     split logits it holds the per-frame camera softmax factors, which lets the
 *                     kernel factorise the softmax (fewer exps per anchor); without it (NULL)
 *                     the result is the same up to fp32 rounding, computed without that saving.
 * Implemented: C == 256, G in {1, 2, 4, 8, 16, 32}, Ncam*L*P*G <= 12288.  The Sparse4D v3
 * shape (Ncam 6, L 4, P 13, G 8, cam-major logits) runs shape-specialised kernels.
 */
S4D_API int s4d_deformable_aggregation(const void* mc_ms_feat, int feat_dtype, int64_t num_feat,
                               const int32_t* spatial_shape, const int32_t* scale_start_index,
                               const float* sample_location, const float* weights, const float* weights_cam,
                               int weights_are_logits, int layout, int64_t bs, int64_t num_anchor,
                               int64_t num_cams, int64_t num_levels, int64_t num_pts, int64_t num_groups,
                               int64_t embed_dims, int64_t cam_begin, int64_t cam_end, float* out,
                               int32_t* error_flag, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Per-level feature maps -> the packed mc_ms_feat layout of s4d_deformable_aggregation, with
 * the element type cast fused in: mc_ms_feat[b, c * sum(HW) + start(l) + y * W(l) + x, ch],
 * start(l) = sum of H*W of the levels before l (the scale_start_index of s4d / ops.level_tables).
 * Replaces the per-level reshape + typecast the reference applies to its FPN outputs before the
 * DFA (model/sparse4d.py:549-558; FPN output format model/fpn.py:90-98).
 *   levels       HOST array of num_levels DEVICE pointers, level l [bs, Ncam, C, H, W] (NCHW) or
 *                [bs, Ncam, H, W, C] (NHWC; the reference's [1, 1, N*H*W, C] levels are NHWC with
 *                bs * Ncam = N), element type src_dtype, contiguous, 16-byte aligned
 *   level_hw     HOST array [num_levels][2] of (H, W)
 *   mc_ms_feat   [bs, Ncam * sum(HW), C] of dst_dtype, 16-byte aligned
 * Implemented: 1 <= num_levels <= 8, C a multiple of 64.
 */
S4D_API int s4d_pack_feature_maps(const void* const* levels, int layout, int src_dtype, int64_t bs, int64_t num_cams,
                                  int64_t num_levels, const int32_t* level_hw, int64_t embed_dims, int dst_dtype,
                                  void* mc_ms_feat, void* stream);

/* ---- InstanceBank (inference): temporal projection and confidence top-k -------------------
 * Anchors are 11 fp32: x y z, log w l h, sin cos, vx vy vz.  Every array is contiguous. */

/* anchor_out = the cached anchors moved by -velocity * time_interval[b] and transformed by
 * T_temp2cur[b] (centre and velocity rotated by T[:3, :3], centre translated by T[:3, 3]; the
 * [cos, sin] pair rotated by T[:2, :2] and stored in the (sin, cos) slots, as the reference does).
 * Replaces InstanceBank._anchor_projection and its device form in InstanceBank.get()
 * (model/instance_bank.py:322-369, :116-161).  The reference's get() passes -(t_now - t_cached).
 *   anchor [bs, num, 11], T_temp2cur [bs, 4, 4], time_interval [bs] or NULL (no motion term),
 *   anchor_out [bs, num, 11] (may equal anchor). */
S4D_API int s4d_instance_bank_project(const float* anchor, const float* T_temp2cur, const float* time_interval,
                                      int64_t bs, int64_t num, float* anchor_out, void* stream);

/* InstanceBank.cache() (model/instance_bank.py:248-306): score = sigmoid(max over classes of
 * confidence) (evaluated in double, rounded once), for the first num_temp anchors
 * max(prev_conf * decay, score); the num_temp best anchors (scores descending, ties by ascending
 * index, NaN last) are gathered.
 *   feature [bs, A, C], anchor [bs, A, 11], confidence [bs, A, num_cls], prev_conf [bs, num_temp]
 *   or NULL (first frame); outputs cached_feature [bs, num_temp, C], cached_anchor
 *   [bs, num_temp, 11], cached_conf [bs, num_temp] (may be NULL), top_idx [bs, num_temp] i32
 *   (may be NULL).  Outputs must not overlap inputs.  Implemented: A <= 4096. */
S4D_API int s4d_instance_bank_cache(const float* feature, const float* anchor, const float* confidence,
                                    const float* prev_conf, float decay, int64_t bs, int64_t num_anchor,
                                    int64_t num_cls, int64_t embed_dims, int64_t num_temp, float* cached_feature,
                                    float* cached_anchor, float* cached_conf, int32_t* top_idx, void* stream);

/* InstanceBank.update() (model/instance_bank.py:188-246): for every frame whose mask byte is
 * non-zero (|time gap| within the limit), out = [cached rows | the A - num_temp best new rows by
 * max-over-classes confidence (same order rule as cache)]; for the others out = the frame's own
 * rows.
 *   feature [bs, A, C], anchor [bs, A, 11], confidence [bs, A, num_cls], cached_feature
 *   [bs, num_temp, C], cached_anchor [bs, num_temp, 11], mask [bs] u8 or NULL (all merge);
 *   out_feature [bs, A, C], out_anchor [bs, A, 11], new_idx [bs, A - num_temp] i32 or NULL.
 *   Outputs must not overlap inputs.  Implemented: A <= 4096. */
S4D_API int s4d_instance_bank_update(const float* feature, const float* anchor, const float* confidence,
                                     const float* cached_feature, const float* cached_anchor, const uint8_t* mask,
                                     int64_t bs, int64_t num_anchor, int64_t num_cls, int64_t embed_dims,
                                     int64_t num_temp, float* out_feature, float* out_anchor, int32_t* new_idx,
                                     void* stream);

/* The per-frame camera factors of the split-logit softmax, written into the workspace that
 * s4d_deformable_aggregation then reads with weights_are_logits = 2: per frame and (level, point,
 * group) column, exp(weights_cam - M2[group]) for every camera and their sum over cameras
 * (M2 = the frame's per-group maximum).  They depend only on the per-camera term, so they can be
 * computed once per frame, e.g. next to s4d_dfa_camera_logits on another stream.  The launch
 * also zeroes the workspace's anchor counter (see s4d_dfa_workspace_bytes).
 *   weights_cam [bs, Ncam, L, P, G]; workspace >= s4d_dfa_workspace_bytes(..., split_logits=1)
 *   bytes, 16-byte aligned.  Implemented: Ncam 6, L 4, P 13, G 8. */
S4D_API int s4d_dfa_camera_factors(const float* weights_cam, int64_t bs, int64_t num_cams, int64_t num_levels,
                                   int64_t num_pts, int64_t num_groups, void* workspace, size_t workspace_bytes,
                                   void* stream);

/* s4d_deformable_aggregation with the sample locations computed inside the gather from the
 * anchors instead of read from a sample_location buffer: the keypoints and their projection of
 * s4d_kps_project (same arithmetic, so the same (u, v) bits) followed by the gather, in one
 * launch.  Replaces ttnn.kps_project_fused
 * (tt-metal/ops/kps_project_fused/kps_project_fused.hpp:12-22) fed by
 * _kps_generator_pre_rotation (model/deformable_feature_aggregation.py:651-677) together with
 * the ops s4d_deformable_aggregation replaces; the sample locations are never written.
 *   anchor            [bs * A, anchor_dim] f32 (anchor_dim >= 8: x, y, z, log w, log l, log h,
 *                     sin, cos, ...)
 *   fix_scale         [num_fix, 3] f32
 *   learnable         [bs * A, (P - num_fix) * 3] f32 keypoint logits (learnable_fc output, e.g.
 *                     the learnable columns of s4d_dfa_weights_fc), contiguous
 *   projection_mat    [bs, Ncam, 4, 4] f32, 16-byte aligned; image_wh [bs, Ncam, 2] f32, 8-byte
 *                     aligned
 * The other arguments as s4d_deformable_aggregation with CAM_MAJOR split logits and prepared
 * camera factors (weights_are_logits = 2: the workspace written by s4d_dfa_camera_factors).
 * Implemented: Ncam 6, L 4, P 13, G 8, C 256. */
S4D_API int s4d_deformable_aggregation_anchors(const void* mc_ms_feat, int feat_dtype, int64_t num_feat,
                                               const int32_t* spatial_shape, const int32_t* scale_start_index,
                                               const float* anchor, int64_t anchor_dim, const float* fix_scale,
                                               int64_t num_fix, const float* learnable, const float* projection_mat,
                                               const float* image_wh, const float* weights, const float* weights_cam,
                                               int64_t bs, int64_t num_anchor, int64_t num_cams, int64_t num_levels,
                                               int64_t num_pts, int64_t num_groups, int64_t embed_dims,
                                               int64_t cam_begin, int64_t cam_end, float* out, int32_t* error_flag,
                                               void* workspace, size_t workspace_bytes, void* stream);

/* s4d_deformable_aggregation_anchors with its output rows routed: the flattened (frame, anchor)
 * rows in [peer_row_begin, peer_row_end) are written to out_peer + row * C (the other GPU's
 * receive buffer of a camera-sharded pair, mapped by s4d_ipc_open, [bs * A, C] rows with the
 * same indexing as out), the others to out.  So the partial sums the other GPU projects cross
 * NVLink as the gather produces them, and that GPU's s4d_dfa_output_proj_sum reads both of its
 * sources from its own memory.  Every block fences its stores at system scope before it exits;
 * the flag exchange that follows (s4d_peer_signal_wait*) orders them before the other GPU's
 * reads.  out and out_peer 16-byte aligned when rows are routed; an empty range routes nothing.
 * Replaces the mesh all_reduce of the partial sums (model/deformable_feature_aggregation.py:
 * 925-931) for the transfer half. */
S4D_API int s4d_deformable_aggregation_anchors_peer(const void* mc_ms_feat, int feat_dtype, int64_t num_feat,
                                                    const int32_t* spatial_shape, const int32_t* scale_start_index,
                                                    const float* anchor, int64_t anchor_dim, const float* fix_scale,
                                                    int64_t num_fix, const float* learnable,
                                                    const float* projection_mat, const float* image_wh,
                                                    const float* weights, const float* weights_cam, int64_t bs,
                                                    int64_t num_anchor, int64_t num_cams, int64_t num_levels,
                                                    int64_t num_pts, int64_t num_groups, int64_t embed_dims,
                                                    int64_t cam_begin, int64_t cam_end, float* out, float* out_peer,
                                                    int64_t peer_row_begin, int64_t peer_row_end,
                                                    int32_t* error_flag, void* workspace, size_t workspace_bytes,
                                                    void* stream);

/* Bytes of the optional workspace of s4d_deformable_aggregation (split logits only: the
 * per-frame camera softmax factors, bs * (Ncam + 1) * L * P * G floats rounded up to 16 bytes,
 * then 16 bytes for the gather's anchor counter; 0 otherwise).  Host-only, launches nothing.
 * The counter is zeroed when the factors are written (s4d_dfa_camera_factors, or the gather
 * itself with weights_are_logits = 1) and every gather launch leaves it at zero, so a prepared
 * workspace serves any number of calls in stream order; calls that share one workspace must not
 * overlap on the GPU. */
S4D_API size_t s4d_dfa_workspace_bytes(int64_t bs, int64_t num_cams, int64_t num_levels, int64_t num_pts,
                                       int64_t num_groups, int split_logits);

/* ---- the DFA linears on the tensor cores (tcgen05, TF32 operands, fp32 accumulation) ------
 *
 * TF32 keeps 10 mantissa bits of every operand (the reference's TT path runs these linears in
 * bf16, 7 bits); products are accumulated in fp32.  Matrices are fp32, row-major, with row
 * strides ("ld") in floats; every matrix pointer and bias must be 16-byte aligned and every
 * ld a multiple of 4.  Implemented: embed_dims == 256. */

/* The two linears that read the instance feature, in one tensor-core pass over 128-row tiles:
 *   logits    [rows, num_logits]    = (instance_feature + anchor_embed) . weights_fc^T
 *   learnable [rows, num_learnable] = instance_feature . learnable_fc^T + learnable_bias
 * The sum instance_feature + anchor_embed is formed tile by tile in shared memory and never
 * written to HBM.  logits is the per-anchor term of the split logits of
 * s4d_deformable_aggregation (the weights_fc bias belongs to the per-camera term).
 * Replaces weights_fc(instance_feature + anchor_embed + camera_embed) of
 * model/deformable_feature_aggregation.py:719-798 (test/dfa_pcc.py:306-320) for its
 * per-anchor part, and the keypoint generator's learnable_fc
 * (model/deformable_feature_aggregation.py:651-677, test/dfa_pcc.py:231-233).
 *   instance_feature, anchor_embed  [rows, embed_dims] with row strides instance_ld, embed_ld
 *   weights_fc_weight   [num_logits, embed_dims] contiguous (out, in)
 *   learnable_fc_weight [num_learnable, embed_dims] contiguous, or NULL when num_learnable == 0
 *   learnable_bias      [num_learnable] or NULL (zero)
 *   logits              [rows, num_logits] contiguous
 *   learnable           [rows, num_learnable] contiguous (4-byte aligned is enough), or NULL
 *                       when num_learnable == 0
 *   error_flag          optional [1] i32, OR-ed with S4D_FLAG_WAIT_TIMEOUT
 * Implemented: num_logits == 416 (4 levels x 13 points x 8 groups), num_learnable <= 32. */
S4D_API int s4d_dfa_weights_fc(const float* instance_feature, int64_t instance_ld, const float* anchor_embed,
                               int64_t embed_ld, int64_t rows, const float* weights_fc_weight,
                               const float* learnable_fc_weight, const float* learnable_bias, int64_t num_logits,
                               int64_t num_learnable, int64_t embed_dims, float* logits, float* learnable,
                               int32_t* error_flag, void* stream);

/* The per-frame camera terms, one CTA per frame (fp32):
 *   camera_embed [bs, Ncam, C]          = LN2(ReLU(W2 LN1(ReLU(W1 x + b1)) + b2)),
 *                                         x = projection_mat[b, c, :3, :4] (12 values)
 *   camera_logits [bs, Ncam, num_logits] = weights_fc(camera_embed) with its bias, the
 *                                         per-camera term of the split logits of
 *                                         s4d_deformable_aggregation
 * LayerNorms use eps 1e-5 and the biased variance.  Replaces the camera encoder
 * (Linear-ReLU-LN-Linear-ReLU-LN) of model/deformable_feature_aggregation.py:679-717
 * (test/dfa_pcc.py:272-279,309-312) and weights_fc on its output (:719-798).
 *   projection_mat       [bs, Ncam, 4, 4]
 *   cam_linear1_weight   [C, 12], cam_linear1_bias [C]; cam_ln1_weight/bias [C]
 *   cam_linear2_weight   [C, C] (16-byte aligned), cam_linear2_bias [C]; cam_ln2_weight/bias [C]
 *   weights_fc_weight    [num_logits, C] (16-byte aligned), weights_fc_bias [num_logits]
 *   camera_embed         [bs, Ncam, C] or NULL (not needed by the split-logit gather)
 *   camera_logits        [bs, Ncam, num_logits]
 *   workspace            >= s4d_dfa_camera_workspace_bytes(bs, Ncam, C) bytes, 4-byte aligned
 *                        (the hidden layer between the two launches)
 * Implemented: 1 <= Ncam <= 8, C == 256. */
S4D_API int s4d_dfa_camera_logits(const float* projection_mat, int64_t bs, int64_t num_cams,
                                  const float* cam_linear1_weight, const float* cam_linear1_bias,
                                  const float* cam_ln1_weight, const float* cam_ln1_bias,
                                  const float* cam_linear2_weight, const float* cam_linear2_bias,
                                  const float* cam_ln2_weight, const float* cam_ln2_bias,
                                  const float* weights_fc_weight, const float* weights_fc_bias, int64_t num_logits,
                                  int64_t embed_dims, float* camera_embed, float* camera_logits, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* Bytes of the workspace of s4d_dfa_camera_logits (bs * Ncam * C floats).  Host-only. */
S4D_API size_t s4d_dfa_camera_workspace_bytes(int64_t bs, int64_t num_cams, int64_t embed_dims);

/* The per-frame camera terms in one launch: the outputs of s4d_dfa_camera_logits and, when a
 * workspace is given, the softmax factors of s4d_dfa_camera_factors (with the anchor counter
 * zeroed), bitwise equal to those two calls.  One cluster of 8 CTAs per frame exchanges the
 * hidden layer through distributed shared memory, so no scratch is needed.  Replaces the camera
 * encoder of model/deformable_feature_aggregation.py:679-717, weights_fc on its output (:719-798)
 * and the camera part of the softmax over the weights (:800-805).
 *   arguments as s4d_dfa_camera_logits, with
 *   workspace  NULL (no factors), or the gather workspace of s4d_dfa_workspace_bytes(bs, Ncam,
 *              L, P, G, 1) with L * P * G == num_logits and G == 8, 16-byte aligned
 * Implemented: 1 <= Ncam <= 8, C == 256, num_logits <= 512 (a multiple of 8 with a workspace). */
S4D_API int s4d_dfa_camera_terms(const float* projection_mat, int64_t bs, int64_t num_cams,
                                 const float* cam_linear1_weight, const float* cam_linear1_bias,
                                 const float* cam_ln1_weight, const float* cam_ln1_bias,
                                 const float* cam_linear2_weight, const float* cam_linear2_bias,
                                 const float* cam_ln2_weight, const float* cam_ln2_bias,
                                 const float* weights_fc_weight, const float* weights_fc_bias, int64_t num_logits,
                                 int64_t embed_dims, float* camera_embed, float* camera_logits, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* output_proj with the residual fused into its epilogue:
 *   out[:, :C] = features . weight^T + bias                        (residual_mode NONE)
 *   out[:, :C] = features . weight^T + bias + instance_feature     (ADD)
 *   out[:, :C] = features . weight^T + bias, out[:, C:2C] = instance_feature   (CAT)
 * Replaces output_proj + the residual cat/add of model/deformable_feature_aggregation.py:934-950
 * (test/dfa_pcc.py:299-304).
 *   features          [rows, C] contiguous (the s4d_deformable_aggregation output)
 *   weight            [C, C] (out, in) contiguous; bias [C] or NULL
 *   instance_feature  [rows, C] with row stride instance_ld (ADD and CAT only; must not
 *                     overlap out)
 *   out               [rows, out_ld], out_ld >= 2C for CAT, >= C otherwise
 *   error_flag        optional [1] i32, OR-ed with S4D_FLAG_WAIT_TIMEOUT */
S4D_API int s4d_dfa_output_proj(const float* features, int64_t rows, const float* weight, const float* bias,
                                const float* instance_feature, int64_t instance_ld, int residual_mode, float* out,
                                int64_t out_ld, int64_t embed_dims, int32_t* error_flag, void* stream);

/* output_proj of the sum of two partial-feature sources (the two camera halves of a camera-
 * sharded layer), rows row0 .. row0 + rows - 1 of each:
 *   out[:, :C] = (features + features2)[row0 : row0 + rows] . weight^T + bias  (+ residual)
 * Both sources are [feature_rows, C] contiguous; features2 may be a peer GPU's buffer mapped by
 * s4d_ipc_open (read over NVLink by the kernel's tensor-memory-access loads).  The sum is formed
 * in the tensor-core accumulator, never in memory.  instance_feature (ADD / CAT), out and the
 * residual modes are those of s4d_dfa_output_proj, for the `rows` output rows.  Replaces the
 * mesh all-reduce of the partial sums plus output_proj
 * (model/deformable_feature_aggregation.py:925-950). */
S4D_API int s4d_dfa_output_proj_sum(const float* features, const float* features2, int64_t feature_rows,
                                    int64_t row0, int64_t rows, const float* weight, const float* bias,
                                    const float* instance_feature, int64_t instance_ld, int residual_mode,
                                    float* out, int64_t out_ld, int64_t embed_dims, int32_t* error_flag,
                                    void* stream);

/*
 * Peer memory between the GPUs of a camera group (one process per GPU).  No counterpart in the
 * reference, whose mesh all-reduce hides the transfer (ttnn.all_reduce).
 *
 * s4d_ipc_handle_bytes   size of the opaque handle s4d_ipc_export writes (64).
 * s4d_ipc_export         handle of the cudaMalloc allocation holding the device pointer `ptr`,
 *                        and the byte offset of `ptr` in it.  Host-only.
 * s4d_ipc_open           maps a handle exported by ANOTHER process into this one; *base is the
 *                        allocation's base (add the exporter's offset).  Host-only.
 * s4d_ipc_close          unmaps a base returned by s4d_ipc_open.
 * s4d_peer_signal_wait   one launch: publishes `epoch` in slot `rank` of every peer's slot
 *                        array (peer_slots[r], a mapped device pointer; entry `rank` unused) and
 *                        waits until every peer r has published an epoch >= `epoch` (modulo
 *                        2^32) in own_slots[r].  Work of earlier launches on `stream` is visible
 *                        to the peers' later launches; the peers' earlier work is visible to
 *                        this stream's later launches.  The wait gives up after limit_ns, ORs
 *                        S4D_FLAG_PEER_TIMEOUT into error_flag and returns.  1 <= world <= 8.
 *                        Every rank must call it with the same epoch sequence; the ranks must be
 *                        on different GPUs (waiting launches on one GPU may never run together).
 * s4d_peer_signal_wait_counter
 *                        the same with the epoch kept on the device: epoch = *epoch_counter +
 *                        advance (advance 0 or 1), read when the launch runs, and stored back in
 *                        *epoch_counter when advance is 1; so a CUDA graph that captured the call
 *                        moves to the next epoch at every replay.  epoch_counter is a device u32
 *                        of this rank, zero before the first call.
 */
S4D_API size_t s4d_ipc_handle_bytes(void);
S4D_API int s4d_ipc_export(const void* ptr, void* handle, uint64_t* offset);
S4D_API int s4d_ipc_open(const void* handle, void** base);
S4D_API int s4d_ipc_close(void* base);
S4D_API int s4d_peer_signal_wait(uint32_t* own_slots, uint32_t* const* peer_slots, int rank, int world,
                                 uint32_t epoch, uint64_t limit_ns, int32_t* error_flag, void* stream);
S4D_API int s4d_peer_signal_wait_counter(uint32_t* own_slots, uint32_t* const* peer_slots, int rank, int world,
                                         uint32_t* epoch_counter, int advance, uint64_t limit_ns,
                                         int32_t* error_flag, void* stream);

/* LayerNorm over the last dimension for the decoder layers around the DFA (nn.LayerNorm of the
 * head's "norm" operations, the asymmetric FFN's pre-norm and the linear_relu_ln blocks of the
 * refinement and anchor-encoder MLPs: model/sparse4d_head.py, model/asymmetric_ffn.py,
 * model/refinement_module.py):
 *   y[r, :] = (x[r, :] - mean) / sqrt(var + eps) * weight + bias   (biased variance)
 *   x, y      [rows, width] f32 contiguous, not overlapping
 *   weight    [width] or NULL (no affine); bias [width] or NULL
 * One warp per row.  Implemented: width 32, 64, 128, 256 or 512.  No reference counterpart as
 * a separate op (the reference calls ttnn / torch LayerNorm). */
S4D_API int s4d_layer_norm(const float* x, const float* weight, const float* bias, float* y, int64_t rows,
                           int64_t width, float eps, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* S4D_DFA_H_ */
