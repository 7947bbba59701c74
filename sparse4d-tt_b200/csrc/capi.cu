// extern "C" entry points of include/s4d_dfa.h: argument validation on the host, then the
// launches of kps_project.cu, dfa_gather.cu and linear_tc.cu.  Nothing here allocates, frees or
// synchronises.
#include <stdarg.h>
#include <stdio.h>

#include "params.cuh"

namespace s4d {

static thread_local char g_last_error[512] = "";
static thread_local unsigned long long g_tc_wait_limit_ns = 2000000000ull;

unsigned long long tc_wait_limit_ns() { return g_tc_wait_limit_ns; }

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

}  // namespace s4d

using namespace s4d;

namespace {

constexpr int64_t kMaxElems = (int64_t)1 << 31;

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Shared checks and launch of s4d_dfa_output_proj and s4d_dfa_output_proj_sum (fn names the
// entry point in the error text); rows row0 .. row0 + rows - 1 of [feature_rows, C] sources.
int output_proj_checked(const char* fn, const float* features, const float* features2, int64_t feature_rows,
                        int64_t row0, int64_t rows, const float* weight, const float* bias,
                        const float* instance_feature, int64_t instance_ld, int residual_mode, float* out,
                        int64_t out_ld, int64_t embed_dims, int32_t* error_flag, void* stream);

}  // namespace

extern "C" {

const char* s4d_status_string(int status) {
  switch (status) {
    case S4D_OK: return "S4D_OK";
    case S4D_ERR_INVALID_ARG: return "S4D_ERR_INVALID_ARG";
    case S4D_ERR_UNSUPPORTED_SHAPE: return "S4D_ERR_UNSUPPORTED_SHAPE";
    case S4D_ERR_CUDA: return "S4D_ERR_CUDA";
    case S4D_ERR_DEVICE_FAULT: return "S4D_ERR_DEVICE_FAULT";
    default: return "S4D_ERR_UNKNOWN";
  }
}

const char* s4d_last_error(void) { return g_last_error; }

int s4d_abi_version(void) { return 109; }

uint64_t s4d_set_tc_wait_limit_ns(uint64_t limit_ns) {
  const uint64_t prev = g_tc_wait_limit_ns;
  g_tc_wait_limit_ns = limit_ns;
  return prev;
}

size_t s4d_kps_workspace_bytes(int64_t bs, int64_t num_anchor, int64_t num_cams, int64_t num_pts) {
  int64_t total = 0;
  if (bs <= 0 || num_anchor <= 0 || num_cams <= 0 || num_pts <= 0 ||
      !size_product({bs, num_anchor, num_cams, num_pts}, kMaxElems, &total))
    return 0;  // nothing to compact, or a size s4d_kps_project rejects
  return kps_workspace_bytes(total);
}

int s4d_dfa_camera_factors(const float* weights_cam, int64_t bs, int64_t num_cams, int64_t num_levels,
                           int64_t num_pts, int64_t num_groups, void* workspace, size_t workspace_bytes, void* stream) {
  set_error("%s", "");
  if (bs < 0 || num_cams <= 0 || num_levels <= 0 || num_pts <= 0 || num_groups <= 0)
    return fail(S4D_ERR_INVALID_ARG, "s4d_dfa_camera_factors: bad sizes");
  int64_t n_w = 0;
  if (bs >= (1 << 24) || !size_product({num_cams, num_levels, num_pts, num_groups}, kGatherMaxWeights + 1, &n_w))
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_dfa_camera_factors: too many frames or Ncam*L*P*G > 12288");
  if (bs == 0) return S4D_OK;
  if (weights_cam == nullptr || workspace == nullptr || !aligned(workspace, 16))
    return fail(S4D_ERR_INVALID_ARG, "s4d_dfa_camera_factors: null weights_cam or missing / misaligned workspace");
  if (workspace_bytes < gather_workspace_bytes(bs, (int)num_cams, (int)num_levels, (int)num_pts, (int)num_groups))
    return fail(S4D_ERR_INVALID_ARG, "s4d_dfa_camera_factors: workspace smaller than s4d_dfa_workspace_bytes()");
  return launch_cam_factors(weights_cam, static_cast<float*>(workspace), (int)bs, (int)num_cams, (int)num_levels,
                            (int)num_pts, (int)num_groups, static_cast<cudaStream_t>(stream));
}

size_t s4d_dfa_workspace_bytes(int64_t bs, int64_t num_cams, int64_t num_levels, int64_t num_pts,
                               int64_t num_groups, int split_logits) {
  int64_t n_w = 0;
  if (!split_logits || bs <= 0 || num_cams <= 0 || num_levels <= 0 || num_pts <= 0 || num_groups <= 0 ||
      bs >= (1 << 24) || !size_product({num_cams, num_levels, num_pts, num_groups}, kGatherMaxWeights + 1, &n_w))
    return 0;  // no workspace needed, or a size the gather rejects
  return gather_workspace_bytes(bs, (int)num_cams, (int)num_levels, (int)num_pts, (int)num_groups);
}

// The learnable_fc inputs of s4d_kps_project_linear (null for s4d_kps_project).
struct KpsLinear {
  const float* inst;
  int64_t inst_ld;
  const float* w;
  const float* b;
  int64_t embed_dims;
};

static int kps_entry(const KpsLinear* lin, const float* anchor, int64_t anchor_dim, const float* fix_scale,
                     int64_t num_fix, const float* learnable, int64_t num_learnable, const float* projection_mat,
                     const float* image_wh, int64_t bs, int64_t num_anchor, int64_t num_cams, int layout,
                     float* key_points, float* sample_location, uint8_t* depth_mask, int32_t* visible_idx,
                     int32_t* visible_count, void* workspace, size_t workspace_bytes, void* stream) {
  set_error("%s", "");
  if (bs < 0 || num_anchor < 0 || num_cams < 0 || num_fix < 0 || num_learnable < 0)
    return fail(S4D_ERR_INVALID_ARG, "s4d_kps_project: negative size");
  if (layout != S4D_LAYOUT_CAM_MAJOR && layout != S4D_LAYOUT_PT_MAJOR && layout != S4D_LAYOUT_GRID)
    return fail(S4D_ERR_INVALID_ARG, "s4d_kps_project: unknown layout");
  if (anchor_dim < 8) return fail(S4D_ERR_INVALID_ARG, "s4d_kps_project: anchor_dim must be >= 8");
  const int64_t num_pts = num_fix + num_learnable;
  if (num_pts == 0) return fail(S4D_ERR_INVALID_ARG, "s4d_kps_project: no keypoints");
  if (num_pts > 64) return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_kps_project: at most 64 keypoints per anchor");
  int64_t total = 0, cam_pts = 0;
  if (!size_product({bs, num_anchor, num_cams, num_pts}, kMaxElems, &total) ||
      !size_product({num_cams, num_pts}, 1 << 24, &cam_pts))
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_kps_project: bs*A*Ncam*P must be < 2^31");
  const bool compact = visible_idx != nullptr || visible_count != nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (total == 0) {
    if (visible_count != nullptr)
      return cuda_check(cudaMemsetAsync(visible_count, 0, sizeof(int32_t), st), "cudaMemsetAsync(visible_count)");
    return S4D_OK;
  }
  if (anchor == nullptr || projection_mat == nullptr || image_wh == nullptr)
    return fail(S4D_ERR_INVALID_ARG, "s4d_kps_project: null input pointer");
  if ((num_fix > 0 && fix_scale == nullptr) || (num_learnable > 0 && learnable == nullptr && lin == nullptr))
    return fail(S4D_ERR_INVALID_ARG, "s4d_kps_project: null fix_scale / learnable with a non-zero count");
  if (lin != nullptr && num_learnable > 0) {
    if (lin->inst == nullptr || lin->w == nullptr)
      return fail(S4D_ERR_INVALID_ARG, "s4d_kps_project_linear: null instance_feature / learnable_fc_weight");
    if (lin->embed_dims != 256)
      return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_kps_project_linear: embed_dims must be 256");
    if (num_learnable * 3 > kKpsMaxFusedLogits)
      return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_kps_project_linear: at most 10 learnable keypoints");
    if (lin->inst_ld < lin->embed_dims || lin->inst_ld % 4 != 0)
      return fail(S4D_ERR_INVALID_ARG, "s4d_kps_project_linear: instance_ld must be >= embed_dims and a multiple of 4");
    if (!aligned(lin->inst, 16) || !aligned(lin->w, 16) || (lin->b != nullptr && !aligned(lin->b, 4)))
      return fail(S4D_ERR_INVALID_ARG, "s4d_kps_project_linear: instance_feature and learnable_fc_weight must be "
                                       "16-byte aligned");
    // the anchors one block of 1024 elements can touch must fit the kernel's staging
    if (1024 / (num_cams * num_pts) + 2 > kKpsMaxFusedAnchors)
      return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_kps_project_linear: needs Ncam * P >= 57 (at most 20 anchors per "
                                             "1024 elements)");
  }
  if (sample_location != nullptr && !aligned(sample_location, 8))
    return fail(S4D_ERR_INVALID_ARG, "s4d_kps_project: sample_location must be 8-byte aligned");
  if (visible_idx != nullptr && !aligned(visible_idx, 16))
    return fail(S4D_ERR_INVALID_ARG, "s4d_kps_project: visible_idx must be 16-byte aligned");
  if (compact) {
    if (workspace == nullptr || !aligned(workspace, 16))
      return fail(S4D_ERR_INVALID_ARG, "s4d_kps_project: compaction needs a 16-byte aligned workspace");
    if (workspace_bytes < kps_workspace_bytes(total))
      return fail(S4D_ERR_INVALID_ARG, "s4d_kps_project: workspace smaller than s4d_kps_workspace_bytes()");
  }
  KpsParams k{};
  k.anchor = anchor;
  k.anchor_dim = (int)anchor_dim;
  k.fix_scale = fix_scale;
  k.num_fix = (int)num_fix;
  k.learnable = learnable;
  k.num_learnable = (int)num_learnable;
  k.kp_pre = nullptr;
  k.proj = projection_mat;
  k.wh = image_wh;
  k.bs = (int)bs;
  k.num_anchor = (int)num_anchor;
  k.num_cams = (int)num_cams;
  k.num_pts = (int)num_pts;
  k.layout = layout;
  k.total = total;
  k.key_points = key_points;
  k.loc = sample_location;
  k.mask = depth_mask;
  if (lin != nullptr && num_learnable > 0) {
    k.learnable = nullptr;
    k.inst = lin->inst;
    k.inst_ld = lin->inst_ld;
    k.w_kps = lin->w;
    k.b_kps = lin->b;
    k.embed_dims = (int)lin->embed_dims;
  }
  return launch_kps_project(k, visible_idx, visible_count, workspace, st);
}

int s4d_kps_project(const float* anchor, int64_t anchor_dim, const float* fix_scale, int64_t num_fix,
                    const float* learnable, int64_t num_learnable, const float* projection_mat,
                    const float* image_wh, int64_t bs, int64_t num_anchor, int64_t num_cams, int layout,
                    float* key_points, float* sample_location, uint8_t* depth_mask, int32_t* visible_idx,
                    int32_t* visible_count, void* workspace, size_t workspace_bytes, void* stream) {
  return kps_entry(nullptr, anchor, anchor_dim, fix_scale, num_fix, learnable, num_learnable, projection_mat,
                   image_wh, bs, num_anchor, num_cams, layout, key_points, sample_location, depth_mask, visible_idx,
                   visible_count, workspace, workspace_bytes, stream);
}

int s4d_kps_project_linear(const float* anchor, int64_t anchor_dim, const float* fix_scale, int64_t num_fix,
                           const float* instance_feature, int64_t instance_ld, const float* learnable_fc_weight,
                           const float* learnable_fc_bias, int64_t num_learnable, int64_t embed_dims,
                           const float* projection_mat, const float* image_wh, int64_t bs, int64_t num_anchor,
                           int64_t num_cams, int layout, float* key_points, float* sample_location,
                           uint8_t* depth_mask, int32_t* visible_idx, int32_t* visible_count, void* workspace,
                           size_t workspace_bytes, void* stream) {
  const KpsLinear lin{instance_feature, instance_ld, learnable_fc_weight, learnable_fc_bias, embed_dims};
  return kps_entry(&lin, anchor, anchor_dim, fix_scale, num_fix, nullptr, num_learnable, projection_mat, image_wh,
                   bs, num_anchor, num_cams, layout, key_points, sample_location, depth_mask, visible_idx,
                   visible_count, workspace, workspace_bytes, stream);
}

int s4d_kps_project_fused(const float* key_points, const float* anchor, int64_t anchor_dim,
                          const float* projection_mat, const float* image_wh, int64_t n, int64_t num_cams,
                          int64_t num_pts, float* grid, void* stream) {
  set_error("%s", "");
  if (n < 0 || num_cams < 0 || num_pts < 0) return fail(S4D_ERR_INVALID_ARG, "s4d_kps_project_fused: negative size");
  if (num_pts > 64) return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_kps_project_fused: at most 64 keypoints per anchor");
  if (anchor_dim < 8) return fail(S4D_ERR_INVALID_ARG, "s4d_kps_project_fused: anchor_dim must be >= 8");
  int64_t total = 0;
  if (!size_product({n, num_cams, num_pts}, kMaxElems, &total))
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_kps_project_fused: n*Ncam*P must be < 2^31");
  if (total == 0) return S4D_OK;
  if (key_points == nullptr || anchor == nullptr || projection_mat == nullptr || image_wh == nullptr ||
      grid == nullptr)
    return fail(S4D_ERR_INVALID_ARG, "s4d_kps_project_fused: null pointer");
  if (!aligned(grid, 8)) return fail(S4D_ERR_INVALID_ARG, "s4d_kps_project_fused: grid must be 8-byte aligned");
  KpsParams k{};
  k.anchor = anchor;
  k.anchor_dim = (int)anchor_dim;
  k.kp_pre = key_points;
  k.proj = projection_mat;
  k.wh = image_wh;
  k.bs = 1;
  k.num_anchor = (int)n;
  k.num_cams = (int)num_cams;
  k.num_pts = (int)num_pts;
  k.layout = S4D_LAYOUT_GRID;
  k.total = total;
  k.loc = grid;
  return launch_kps_project(k, nullptr, nullptr, nullptr, static_cast<cudaStream_t>(stream));
}

// Keypoint inputs of s4d_deformable_aggregation_anchors.
struct GatherAnchors {
  const float* anchor;
  int64_t anchor_dim;
  const float* fix_scale;
  int64_t num_fix;
  const float* learnable;
  const float* proj;
  const float* wh;
};

// Shared by s4d_deformable_aggregation (kps == null: sample_location given) and
// s4d_deformable_aggregation_anchors (sample locations computed in the gather).
static int gather_entry(const void* mc_ms_feat, int feat_dtype, int64_t num_feat, const int32_t* spatial_shape,
                        const int32_t* scale_start_index, const float* sample_location, const GatherAnchors* kps,
                        const float* weights, const float* weights_cam, int weights_are_logits, int layout, int64_t bs,
                        int64_t num_anchor, int64_t num_cams, int64_t num_levels, int64_t num_pts,
                        int64_t num_groups, int64_t embed_dims, int64_t cam_begin, int64_t cam_end, float* out,
                        int32_t* error_flag, void* workspace, size_t workspace_bytes, void* stream,
                        float* out_peer = nullptr, int64_t peer_row_begin = 0, int64_t peer_row_end = 0) {
  if (bs < 0 || num_anchor < 0 || num_cams <= 0 || num_levels <= 0 || num_pts <= 0 || num_groups <= 0 ||
      embed_dims <= 0 || num_feat < 0)
    return fail(S4D_ERR_INVALID_ARG, "s4d_deformable_aggregation: sizes must be positive");
  if (feat_dtype != S4D_DTYPE_F32 && feat_dtype != S4D_DTYPE_BF16)
    return fail(S4D_ERR_INVALID_ARG, "s4d_deformable_aggregation: unknown feat_dtype");
  if (layout != S4D_LAYOUT_CAM_MAJOR && layout != S4D_LAYOUT_PT_MAJOR)
    return fail(S4D_ERR_INVALID_ARG, "s4d_deformable_aggregation: layout must be CAM_MAJOR or PT_MAJOR");
  if (cam_begin < 0 || cam_end > num_cams || cam_begin > cam_end)
    return fail(S4D_ERR_INVALID_ARG, "s4d_deformable_aggregation: need 0 <= cam_begin <= cam_end <= num_cams");
  if (weights_cam != nullptr && layout != S4D_LAYOUT_CAM_MAJOR)
    return fail(S4D_ERR_INVALID_ARG, "s4d_deformable_aggregation: split logits (weights_cam) need CAM_MAJOR");
  if (weights_are_logits < 0 || weights_are_logits > 2)
    return fail(S4D_ERR_INVALID_ARG, "s4d_deformable_aggregation: weights_are_logits must be 0, 1 or 2");
  if (weights_cam != nullptr && !weights_are_logits)
    return fail(S4D_ERR_INVALID_ARG, "s4d_deformable_aggregation: split weights are only defined for logits");
  if (weights_are_logits == 2 && (weights_cam == nullptr || workspace == nullptr))
    return fail(S4D_ERR_INVALID_ARG, "s4d_deformable_aggregation: prepared camera factors (weights_are_logits 2) "
                                     "need weights_cam and the workspace they were written to");
  if (weights_are_logits == 2 && !(num_cams == 6 && num_levels == 4 && num_pts == 13 && num_groups == 8 &&
                                   layout == S4D_LAYOUT_CAM_MAJOR))
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_deformable_aggregation: prepared camera factors are implemented "
                                           "for 6 cameras, 4 levels, 13 points, 8 groups");
  if (embed_dims != 256)
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_deformable_aggregation: embed_dims must be 256");
  if (num_groups > 32 || (num_groups & (num_groups - 1)) != 0)
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_deformable_aggregation: num_groups must be 1, 2, 4, 8, 16 or 32");
  int64_t n_w = 0, anchors = 0, rows = 0;
  if (!size_product({num_cams, num_levels, num_pts, num_groups}, kGatherMaxWeights + 1, &n_w))
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_deformable_aggregation: Ncam*L*P*G must be <= 12288");
  if (!size_product({bs, num_anchor}, kMaxElems, &anchors) || !size_product({bs, num_feat}, (int64_t)1 << 40, &rows))
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_deformable_aggregation: too many anchors or feature rows");
  if (num_feat >= kMaxElems)
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_deformable_aggregation: num_feat must be < 2^31");
  if (anchors == 0) return S4D_OK;
  if (mc_ms_feat == nullptr || spatial_shape == nullptr || scale_start_index == nullptr ||
      (kps == nullptr && sample_location == nullptr) || weights == nullptr || out == nullptr)
    return fail(S4D_ERR_INVALID_ARG, "s4d_deformable_aggregation: null pointer");
  if (!aligned(mc_ms_feat, 16))
    return fail(S4D_ERR_INVALID_ARG, "s4d_deformable_aggregation: mc_ms_feat must be 16-byte aligned");
  if (peer_row_begin < 0 || peer_row_end < peer_row_begin || peer_row_end > anchors)
    return fail(S4D_ERR_INVALID_ARG, "s4d_deformable_aggregation: need 0 <= peer_row_begin <= peer_row_end <= bs*A");
  if (peer_row_end > peer_row_begin && (out_peer == nullptr || !aligned(out_peer, 16) || !aligned(out, 16)))
    return fail(S4D_ERR_INVALID_ARG, "s4d_deformable_aggregation: out_peer null, or out / out_peer not 16-byte aligned");
  if ((kps == nullptr && !aligned(sample_location, 8)) || !aligned(weights, 4) || !aligned(out, 4))
    return fail(S4D_ERR_INVALID_ARG, "s4d_deformable_aggregation: misaligned sample_location/weights/out");
  GatherParams p{};
  p.feat = mc_ms_feat;
  p.num_feat = num_feat;
  p.spatial_shape = spatial_shape;
  p.scale_start = scale_start_index;
  p.loc = sample_location;
  p.weights = weights;
  p.weights_cam = weights_cam;
  p.out = out;
  if (peer_row_end > peer_row_begin) {
    p.out_peer = out_peer;
    p.peer_row_begin = peer_row_begin;
    p.peer_row_end = peer_row_end;
  }
  p.error_flag = error_flag;
  p.bs = (int)bs;
  p.num_anchor = (int)num_anchor;
  p.num_cams = (int)num_cams;
  p.num_levels = (int)num_levels;
  p.num_pts = (int)num_pts;
  p.num_groups = (int)num_groups;
  p.cam_begin = (int)cam_begin;
  p.cam_end = (int)cam_end;
  p.logits = weights_are_logits ? 1 : 0;
  p.factors_ready = weights_are_logits == 2 ? 1 : 0;
  p.layout = layout;
  p.cam_ws = nullptr;
  if (weights_cam != nullptr && workspace != nullptr) {
    if (!aligned(workspace, 16))
      return fail(S4D_ERR_INVALID_ARG, "s4d_deformable_aggregation: workspace must be 16-byte aligned");
    if (workspace_bytes < gather_workspace_bytes(bs, (int)num_cams, (int)num_levels, (int)num_pts, (int)num_groups))
      return fail(S4D_ERR_INVALID_ARG, "s4d_deformable_aggregation: workspace smaller than s4d_dfa_workspace_bytes()");
    p.cam_ws = static_cast<float*>(workspace);
  }
  if (gather_smem_bytes(p.num_cams, p.num_levels, p.num_pts, p.num_groups, p.cam_begin, p.cam_end) > 200 * 1024)
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_deformable_aggregation: per-anchor staging exceeds shared memory");
  if (kps != nullptr) {
    p.kps_anchor = kps->anchor;
    p.kps_anchor_dim = (int)kps->anchor_dim;
    p.kps_fix_scale = kps->fix_scale;
    p.kps_num_fix = (int)kps->num_fix;
    p.kps_learnable = kps->learnable;
    p.kps_proj = kps->proj;
    p.kps_wh = kps->wh;
  }
  return launch_gather(p, feat_dtype, static_cast<cudaStream_t>(stream));
}

int s4d_deformable_aggregation(const void* mc_ms_feat, int feat_dtype, int64_t num_feat,
                               const int32_t* spatial_shape, const int32_t* scale_start_index,
                               const float* sample_location, const float* weights, const float* weights_cam,
                               int weights_are_logits, int layout, int64_t bs, int64_t num_anchor,
                               int64_t num_cams, int64_t num_levels, int64_t num_pts, int64_t num_groups,
                               int64_t embed_dims, int64_t cam_begin, int64_t cam_end, float* out,
                               int32_t* error_flag, void* workspace, size_t workspace_bytes, void* stream) {
  set_error("%s", "");
  return gather_entry(mc_ms_feat, feat_dtype, num_feat, spatial_shape, scale_start_index, sample_location, nullptr,
                      weights, weights_cam, weights_are_logits, layout, bs, num_anchor, num_cams, num_levels, num_pts,
                      num_groups, embed_dims, cam_begin, cam_end, out, error_flag, workspace, workspace_bytes, stream);
}

int s4d_deformable_aggregation_anchors_peer(const void* mc_ms_feat, int feat_dtype, int64_t num_feat,
                                            const int32_t* spatial_shape, const int32_t* scale_start_index,
                                            const float* anchor, int64_t anchor_dim, const float* fix_scale,
                                            int64_t num_fix, const float* learnable, const float* projection_mat,
                                            const float* image_wh, const float* weights, const float* weights_cam,
                                            int64_t bs, int64_t num_anchor, int64_t num_cams, int64_t num_levels,
                                            int64_t num_pts, int64_t num_groups, int64_t embed_dims,
                                            int64_t cam_begin, int64_t cam_end, float* out, float* out_peer,
                                            int64_t peer_row_begin, int64_t peer_row_end, int32_t* error_flag,
                                            void* workspace, size_t workspace_bytes, void* stream) {
  set_error("%s", "");
  if (!(num_cams == 6 && num_levels == 4 && num_pts == 13 && num_groups == 8))
    return fail(S4D_ERR_UNSUPPORTED_SHAPE,
                "s4d_deformable_aggregation_anchors: implemented for 6 cameras, 4 levels, 13 points, 8 groups");
  if (anchor_dim < 8 || num_fix < 0 || num_fix > num_pts)
    return fail(S4D_ERR_INVALID_ARG, "s4d_deformable_aggregation_anchors: need anchor_dim >= 8, 0 <= num_fix <= P");
  if (bs > 0 && num_anchor > 0) {
    if (anchor == nullptr || projection_mat == nullptr || image_wh == nullptr ||
        (num_fix > 0 && fix_scale == nullptr) || (num_fix < num_pts && learnable == nullptr))
      return fail(S4D_ERR_INVALID_ARG, "s4d_deformable_aggregation_anchors: null pointer");
    if (!aligned(anchor, 4) || !aligned(projection_mat, 16) || !aligned(image_wh, 8) ||
        (fix_scale != nullptr && !aligned(fix_scale, 4)) || (learnable != nullptr && !aligned(learnable, 4)) ||
        !aligned(weights, 16) || !aligned(weights_cam, 16))
      return fail(S4D_ERR_INVALID_ARG, "s4d_deformable_aggregation_anchors: misaligned pointer (weights, weights_cam "
                                       "and projection_mat need 16 bytes, image_wh 8)");
  }
  const GatherAnchors kps{anchor, anchor_dim, fix_scale, num_fix, learnable, projection_mat, image_wh};
  return gather_entry(mc_ms_feat, feat_dtype, num_feat, spatial_shape, scale_start_index, nullptr, &kps, weights,
                      weights_cam, 2, S4D_LAYOUT_CAM_MAJOR, bs, num_anchor, num_cams, num_levels, num_pts,
                      num_groups, embed_dims, cam_begin, cam_end, out, error_flag, workspace, workspace_bytes, stream,
                      out_peer, peer_row_begin, peer_row_end);
}

int s4d_deformable_aggregation_anchors(const void* mc_ms_feat, int feat_dtype, int64_t num_feat,
                                       const int32_t* spatial_shape, const int32_t* scale_start_index,
                                       const float* anchor, int64_t anchor_dim, const float* fix_scale,
                                       int64_t num_fix, const float* learnable, const float* projection_mat,
                                       const float* image_wh, const float* weights, const float* weights_cam,
                                       int64_t bs, int64_t num_anchor, int64_t num_cams, int64_t num_levels,
                                       int64_t num_pts, int64_t num_groups, int64_t embed_dims, int64_t cam_begin,
                                       int64_t cam_end, float* out, int32_t* error_flag, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  return s4d_deformable_aggregation_anchors_peer(mc_ms_feat, feat_dtype, num_feat, spatial_shape, scale_start_index,
                                                 anchor, anchor_dim, fix_scale, num_fix, learnable, projection_mat,
                                                 image_wh, weights, weights_cam, bs, num_anchor, num_cams, num_levels,
                                                 num_pts, num_groups, embed_dims, cam_begin, cam_end, out, nullptr, 0,
                                                 0, error_flag, workspace, workspace_bytes, stream);
}

int s4d_dfa_weights_fc(const float* instance_feature, int64_t instance_ld, const float* anchor_embed,
                       int64_t embed_ld, int64_t rows, const float* weights_fc_weight,
                       const float* learnable_fc_weight, const float* learnable_bias, int64_t num_logits,
                       int64_t num_learnable, int64_t embed_dims, float* logits, float* learnable,
                       int32_t* error_flag, void* stream) {
  set_error("%s", "");
  if (rows < 0 || num_logits <= 0 || num_learnable < 0)
    return fail(S4D_ERR_INVALID_ARG, "s4d_dfa_weights_fc: bad sizes");
  if (embed_dims != 256) return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_dfa_weights_fc: embed_dims must be 256");
  if (num_logits != 416 || num_learnable > 32)
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_dfa_weights_fc: implemented for num_logits 416, num_learnable <= 32");
  if (rows >= kMaxElems) return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_dfa_weights_fc: rows must be < 2^31");
  if (rows == 0) return S4D_OK;
  if (instance_feature == nullptr || anchor_embed == nullptr || weights_fc_weight == nullptr || logits == nullptr ||
      (num_learnable > 0 && (learnable == nullptr || learnable_fc_weight == nullptr)))
    return fail(S4D_ERR_INVALID_ARG, "s4d_dfa_weights_fc: null pointer");
  if (instance_ld < embed_dims || embed_ld < embed_dims || instance_ld % 4 != 0 || embed_ld % 4 != 0)
    return fail(S4D_ERR_INVALID_ARG, "s4d_dfa_weights_fc: row strides must be >= embed_dims and multiples of 4");
  if (!aligned(instance_feature, 16) || !aligned(anchor_embed, 16) || !aligned(weights_fc_weight, 16) ||
      !aligned(logits, 16) || (learnable_fc_weight != nullptr && !aligned(learnable_fc_weight, 16)) ||
      (learnable_bias != nullptr && !aligned(learnable_bias, 4)) || (learnable != nullptr && !aligned(learnable, 4)))
    return fail(S4D_ERR_INVALID_ARG, "s4d_dfa_weights_fc: misaligned pointer");
  WfcParams p{};
  p.inst = instance_feature;
  p.inst_ld = instance_ld;
  p.embed = anchor_embed;
  p.embed_ld = embed_ld;
  p.w_fc = weights_fc_weight;
  p.w_kps = num_learnable > 0 ? learnable_fc_weight : weights_fc_weight;
  p.learn_bias = num_learnable > 0 ? learnable_bias : nullptr;
  p.logits = logits;
  p.learnable = learnable;
  p.rows = rows;
  p.n_logits = (int)num_logits;
  p.n_learn = (int)num_learnable;
  p.k = (int)embed_dims;
  p.error_flag = error_flag;
  p.wait_limit_ns = tc_wait_limit_ns();
  return launch_weights_fc(p, static_cast<cudaStream_t>(stream));
}

int s4d_pack_feature_maps(const void* const* levels, int layout, int src_dtype, int64_t bs, int64_t num_cams,
                          int64_t num_levels, const int32_t* level_hw, int64_t embed_dims, int dst_dtype,
                          void* mc_ms_feat, void* stream) {
  set_error("%s", "");
  if (layout != S4D_MAPS_NCHW && layout != S4D_MAPS_NHWC)
    return fail(S4D_ERR_INVALID_ARG, "s4d_pack_feature_maps: unknown layout");
  if ((src_dtype != S4D_DTYPE_F32 && src_dtype != S4D_DTYPE_BF16) ||
      (dst_dtype != S4D_DTYPE_F32 && dst_dtype != S4D_DTYPE_BF16))
    return fail(S4D_ERR_INVALID_ARG, "s4d_pack_feature_maps: unknown dtype");
  if (bs < 0 || num_cams <= 0 || num_levels <= 0 || embed_dims <= 0)
    return fail(S4D_ERR_INVALID_ARG, "s4d_pack_feature_maps: bad sizes");
  if (num_levels > kMaxPackLevels || embed_dims % 64 != 0)
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_pack_feature_maps: implemented for <= 8 levels, C a multiple of 64");
  if (bs * num_cams > 65535) return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_pack_feature_maps: bs * Ncam must be <= 65535");
  if (bs == 0) return S4D_OK;
  if (levels == nullptr || level_hw == nullptr || mc_ms_feat == nullptr)
    return fail(S4D_ERR_INVALID_ARG, "s4d_pack_feature_maps: null pointer");
  if (!aligned(mc_ms_feat, 16)) return fail(S4D_ERR_INVALID_ARG, "s4d_pack_feature_maps: mc_ms_feat must be 16-byte aligned");
  PackParams p{};
  int64_t per_cam = 0;
  for (int64_t l = 0; l < num_levels; ++l) {
    const int64_t h = level_hw[2 * l], w = level_hw[2 * l + 1];
    if (h <= 0 || w <= 0) return fail(S4D_ERR_INVALID_ARG, "s4d_pack_feature_maps: level sizes must be positive");
    if (levels[l] == nullptr || !aligned(levels[l], 16))
      return fail(S4D_ERR_INVALID_ARG, "s4d_pack_feature_maps: null or misaligned level pointer");
    p.src[l] = levels[l];
    p.h[l] = (int)h;
    p.w[l] = (int)w;
    per_cam += h * w;
  }
  int64_t elems = 0, cam_elems = 0;
  if (!size_product({per_cam, num_cams, bs, embed_dims}, (int64_t)1 << 40, &elems) ||
      !size_product({per_cam, embed_dims}, kMaxElems, &cam_elems))
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_pack_feature_maps: maps too large");
  p.num_levels = (int)num_levels;
  p.bs = (int)bs;
  p.num_cams = (int)num_cams;
  p.channels = (int)embed_dims;
  p.layout = layout;
  p.src_dtype = src_dtype;
  p.dst_dtype = dst_dtype;
  p.dst = mc_ms_feat;
  return launch_pack_maps(p, static_cast<cudaStream_t>(stream));
}

int s4d_instance_bank_project(const float* anchor, const float* T_temp2cur, const float* time_interval, int64_t bs,
                              int64_t num, float* anchor_out, void* stream) {
  set_error("%s", "");
  if (bs < 0 || num < 0) return fail(S4D_ERR_INVALID_ARG, "s4d_instance_bank_project: negative size");
  int64_t total = 0;
  if (!size_product({bs, num}, kMaxElems, &total))
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_instance_bank_project: too many anchors");
  if (total == 0) return S4D_OK;
  if (anchor == nullptr || T_temp2cur == nullptr || anchor_out == nullptr)
    return fail(S4D_ERR_INVALID_ARG, "s4d_instance_bank_project: null pointer");
  IbProjectParams p{anchor, T_temp2cur, time_interval, anchor_out, (int)bs, (int)num, 11};
  return launch_ib_project(p, static_cast<cudaStream_t>(stream));
}

static int ib_check(const char* fn, int64_t bs, int64_t num_anchor, int64_t num_cls, int64_t embed_dims,
                    int64_t num_temp) {
  if (bs < 0 || num_anchor <= 0 || num_cls <= 0 || embed_dims <= 0 || num_temp <= 0 || num_temp > num_anchor) {
    set_error("%s: need bs >= 0, num_anchor, num_cls, embed_dims > 0 and 0 < num_temp <= num_anchor", fn);
    return S4D_ERR_INVALID_ARG;
  }
  int64_t elems = 0;
  if (num_anchor > 4096 || bs >= 65536 || !size_product({bs, num_anchor, embed_dims}, (int64_t)1 << 40, &elems)) {
    set_error("%s: implemented for num_anchor <= 4096 and bs < 65536", fn);
    return S4D_ERR_UNSUPPORTED_SHAPE;
  }
  return S4D_OK;
}

int s4d_instance_bank_cache(const float* feature, const float* anchor, const float* confidence, const float* prev_conf,
                            float decay, int64_t bs, int64_t num_anchor, int64_t num_cls, int64_t embed_dims,
                            int64_t num_temp, float* cached_feature, float* cached_anchor, float* cached_conf,
                            int32_t* top_idx, void* stream) {
  set_error("%s", "");
  int st = ib_check("s4d_instance_bank_cache", bs, num_anchor, num_cls, embed_dims, num_temp);
  if (st != S4D_OK || bs == 0) return st;
  if (feature == nullptr || anchor == nullptr || confidence == nullptr || cached_feature == nullptr ||
      cached_anchor == nullptr)
    return fail(S4D_ERR_INVALID_ARG, "s4d_instance_bank_cache: null pointer");
  IbSelectParams p{};
  p.feature = feature;
  p.anchor = anchor;
  p.confidence = confidence;
  p.prev_conf = prev_conf;
  p.decay = decay;
  p.out_feature = cached_feature;
  p.out_anchor = cached_anchor;
  p.out_conf = cached_conf;
  p.out_idx = top_idx;
  p.bs = (int)bs;
  p.num_anchor = (int)num_anchor;
  p.num_cls = (int)num_cls;
  p.embed_dims = (int)embed_dims;
  p.anchor_dim = 11;
  p.num_temp = (int)num_temp;
  return launch_ib_select(p, true, static_cast<cudaStream_t>(stream));
}

int s4d_instance_bank_update(const float* feature, const float* anchor, const float* confidence,
                             const float* cached_feature, const float* cached_anchor, const uint8_t* mask, int64_t bs,
                             int64_t num_anchor, int64_t num_cls, int64_t embed_dims, int64_t num_temp,
                             float* out_feature, float* out_anchor, int32_t* new_idx, void* stream) {
  set_error("%s", "");
  int st = ib_check("s4d_instance_bank_update", bs, num_anchor, num_cls, embed_dims, num_temp);
  if (st != S4D_OK || bs == 0) return st;
  if (feature == nullptr || anchor == nullptr || confidence == nullptr || cached_feature == nullptr ||
      cached_anchor == nullptr || out_feature == nullptr || out_anchor == nullptr)
    return fail(S4D_ERR_INVALID_ARG, "s4d_instance_bank_update: null pointer");
  IbSelectParams p{};
  p.feature = feature;
  p.anchor = anchor;
  p.confidence = confidence;
  p.cached_feature = cached_feature;
  p.cached_anchor = cached_anchor;
  p.mask = mask;
  p.out_feature = out_feature;
  p.out_anchor = out_anchor;
  p.out_idx = new_idx;
  p.bs = (int)bs;
  p.num_anchor = (int)num_anchor;
  p.num_cls = (int)num_cls;
  p.embed_dims = (int)embed_dims;
  p.anchor_dim = 11;
  p.num_temp = (int)num_temp;
  return launch_ib_select(p, false, static_cast<cudaStream_t>(stream));
}

size_t s4d_dfa_camera_workspace_bytes(int64_t bs, int64_t num_cams, int64_t embed_dims) {
  int64_t elems = 0;
  if (bs <= 0 || num_cams <= 0 || embed_dims <= 0 || !size_product({bs, num_cams, embed_dims}, (int64_t)1 << 40, &elems))
    return 0;  // nothing to compute, or a size s4d_dfa_camera_logits rejects
  return size_t(elems) * sizeof(float);
}

int s4d_dfa_camera_logits(const float* projection_mat, int64_t bs, int64_t num_cams, const float* cam_linear1_weight,
                          const float* cam_linear1_bias, const float* cam_ln1_weight, const float* cam_ln1_bias,
                          const float* cam_linear2_weight, const float* cam_linear2_bias, const float* cam_ln2_weight,
                          const float* cam_ln2_bias, const float* weights_fc_weight, const float* weights_fc_bias,
                          int64_t num_logits, int64_t embed_dims, float* camera_embed, float* camera_logits,
                          void* workspace, size_t workspace_bytes, void* stream) {
  set_error("%s", "");
  if (bs < 0 || num_cams <= 0 || num_logits <= 0) return fail(S4D_ERR_INVALID_ARG, "s4d_dfa_camera_logits: bad sizes");
  if (num_cams > 8 || embed_dims != 256)
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_dfa_camera_logits: implemented for 1..8 cameras and embed_dims 256");
  if (bs >= (1 << 30) || num_logits >= (1 << 24))
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_dfa_camera_logits: too many frames or logits");
  if (bs == 0) return S4D_OK;
  if (projection_mat == nullptr || cam_linear1_weight == nullptr || cam_linear1_bias == nullptr ||
      cam_ln1_weight == nullptr || cam_ln1_bias == nullptr || cam_linear2_weight == nullptr ||
      cam_linear2_bias == nullptr || cam_ln2_weight == nullptr || cam_ln2_bias == nullptr ||
      weights_fc_weight == nullptr || weights_fc_bias == nullptr || camera_logits == nullptr)
    return fail(S4D_ERR_INVALID_ARG, "s4d_dfa_camera_logits: null pointer");
  if (!aligned(cam_linear2_weight, 16) || !aligned(weights_fc_weight, 16))
    return fail(S4D_ERR_INVALID_ARG, "s4d_dfa_camera_logits: the C x C and weights_fc matrices must be 16-byte aligned");
  if (workspace == nullptr || !aligned(workspace, 4) ||
      workspace_bytes < s4d_dfa_camera_workspace_bytes(bs, num_cams, embed_dims))
    return fail(S4D_ERR_INVALID_ARG, "s4d_dfa_camera_logits: workspace missing or smaller than "
                                     "s4d_dfa_camera_workspace_bytes()");
  CamEncParams p{};
  p.proj = projection_mat;
  p.w1 = cam_linear1_weight;
  p.b1 = cam_linear1_bias;
  p.ln1_w = cam_ln1_weight;
  p.ln1_b = cam_ln1_bias;
  p.w2 = cam_linear2_weight;
  p.b2 = cam_linear2_bias;
  p.ln2_w = cam_ln2_weight;
  p.ln2_b = cam_ln2_bias;
  p.w_fc = weights_fc_weight;
  p.b_fc = weights_fc_bias;
  p.camera_embed = camera_embed;
  p.logits = camera_logits;
  p.hidden = static_cast<float*>(workspace);
  p.bs = (int)bs;
  p.num_cams = (int)num_cams;
  p.num_logits = (int)num_logits;
  p.embed_dims = (int)embed_dims;
  return launch_camera_logits(p, static_cast<cudaStream_t>(stream));
}

int s4d_dfa_camera_terms(const float* projection_mat, int64_t bs, int64_t num_cams, const float* cam_linear1_weight,
                         const float* cam_linear1_bias, const float* cam_ln1_weight, const float* cam_ln1_bias,
                         const float* cam_linear2_weight, const float* cam_linear2_bias, const float* cam_ln2_weight,
                         const float* cam_ln2_bias, const float* weights_fc_weight, const float* weights_fc_bias,
                         int64_t num_logits, int64_t embed_dims, float* camera_embed, float* camera_logits,
                         void* workspace, size_t workspace_bytes, void* stream) {
  set_error("%s", "");
  if (bs < 0 || num_cams <= 0 || num_logits <= 0) return fail(S4D_ERR_INVALID_ARG, "s4d_dfa_camera_terms: bad sizes");
  if (num_cams > 8 || embed_dims != 256 || num_logits > 512)
    return fail(S4D_ERR_UNSUPPORTED_SHAPE,
                "s4d_dfa_camera_terms: implemented for 1..8 cameras, embed_dims 256 and at most 512 logits");
  if (bs >= (1 << 30)) return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_dfa_camera_terms: too many frames");
  if (workspace != nullptr && num_logits % 8 != 0)
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_dfa_camera_terms: the softmax factors need 8 groups "
                                           "(num_logits a multiple of 8)");
  if (bs == 0) return S4D_OK;
  if (projection_mat == nullptr || cam_linear1_weight == nullptr || cam_linear1_bias == nullptr ||
      cam_ln1_weight == nullptr || cam_ln1_bias == nullptr || cam_linear2_weight == nullptr ||
      cam_linear2_bias == nullptr || cam_ln2_weight == nullptr || cam_ln2_bias == nullptr ||
      weights_fc_weight == nullptr || weights_fc_bias == nullptr || camera_logits == nullptr)
    return fail(S4D_ERR_INVALID_ARG, "s4d_dfa_camera_terms: null pointer");
  if (!aligned(cam_linear2_weight, 16) || !aligned(weights_fc_weight, 16))
    return fail(S4D_ERR_INVALID_ARG, "s4d_dfa_camera_terms: the C x C and weights_fc matrices must be 16-byte aligned");
  // the factors and the anchor counter pair sit where the gather expects them: the workspace of
  // s4d_dfa_workspace_bytes(bs, num_cams, L, P, 8, 1) for any L * P * 8 == num_logits
  const size_t need = gather_workspace_bytes(bs, (int)num_cams, 1, 1, (int)num_logits);
  if (workspace != nullptr && (!aligned(workspace, 16) || workspace_bytes < need))
    return fail(S4D_ERR_INVALID_ARG, "s4d_dfa_camera_terms: workspace misaligned or smaller than "
                                     "s4d_dfa_workspace_bytes()");
  CamEncParams p{};
  p.proj = projection_mat;
  p.w1 = cam_linear1_weight;
  p.b1 = cam_linear1_bias;
  p.ln1_w = cam_ln1_weight;
  p.ln1_b = cam_ln1_bias;
  p.w2 = cam_linear2_weight;
  p.b2 = cam_linear2_bias;
  p.ln2_w = cam_ln2_weight;
  p.ln2_b = cam_ln2_bias;
  p.w_fc = weights_fc_weight;
  p.b_fc = weights_fc_bias;
  p.camera_embed = camera_embed;
  p.logits = camera_logits;
  if (workspace != nullptr) {
    p.factors = static_cast<float*>(workspace);
    p.anchor_counter = reinterpret_cast<unsigned*>(static_cast<char*>(workspace) + need - 16);
  }
  p.bs = (int)bs;
  p.num_cams = (int)num_cams;
  p.num_logits = (int)num_logits;
  p.embed_dims = (int)embed_dims;
  return launch_camera_terms(p, static_cast<cudaStream_t>(stream));
}

int s4d_dfa_output_proj(const float* features, int64_t rows, const float* weight, const float* bias,
                        const float* instance_feature, int64_t instance_ld, int residual_mode, float* out,
                        int64_t out_ld, int64_t embed_dims, int32_t* error_flag, void* stream) {
  set_error("%s", "");
  if (rows < 0) return fail(S4D_ERR_INVALID_ARG, "s4d_dfa_output_proj: negative rows");
  return output_proj_checked("s4d_dfa_output_proj", features, nullptr, rows, 0, rows, weight, bias, instance_feature,
                             instance_ld, residual_mode, out, out_ld, embed_dims, error_flag, stream);
}

int s4d_dfa_output_proj_sum(const float* features, const float* features2, int64_t feature_rows, int64_t row0,
                            int64_t rows, const float* weight, const float* bias, const float* instance_feature,
                            int64_t instance_ld, int residual_mode, float* out, int64_t out_ld, int64_t embed_dims,
                            int32_t* error_flag, void* stream) {
  set_error("%s", "");
  if (rows < 0 || row0 < 0 || feature_rows < 0)
    return fail(S4D_ERR_INVALID_ARG, "s4d_dfa_output_proj_sum: negative rows, row0 or feature_rows");
  if (feature_rows >= kMaxElems) return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_dfa_output_proj_sum: feature_rows must be < 2^31");
  if (row0 > feature_rows || rows > feature_rows - row0)
    return fail(S4D_ERR_INVALID_ARG, "s4d_dfa_output_proj_sum: rows row0 .. row0 + rows - 1 outside the sources");
  if (rows > 0 && (features2 == nullptr || !aligned(features2, 16)))
    return fail(S4D_ERR_INVALID_ARG, "s4d_dfa_output_proj_sum: null or misaligned features2");
  return output_proj_checked("s4d_dfa_output_proj_sum", features, features2, feature_rows, row0, rows, weight, bias,
                             instance_feature, instance_ld, residual_mode, out, out_ld, embed_dims, error_flag, stream);
}

}  // extern "C"

namespace {

int output_proj_checked(const char* fn, const float* features, const float* features2, int64_t feature_rows,
                        int64_t row0, int64_t rows, const float* weight, const float* bias,
                        const float* instance_feature, int64_t instance_ld, int residual_mode, float* out,
                        int64_t out_ld, int64_t embed_dims, int32_t* error_flag, void* stream) {
  char msg[160];
  auto bad = [&](int status, const char* what) {
    snprintf(msg, sizeof(msg), "%s: %s", fn, what);
    return fail(status, msg);
  };
  if (residual_mode != S4D_RESIDUAL_NONE && residual_mode != S4D_RESIDUAL_ADD && residual_mode != S4D_RESIDUAL_CAT)
    return bad(S4D_ERR_INVALID_ARG, "unknown residual_mode");
  if (embed_dims != 256) return bad(S4D_ERR_UNSUPPORTED_SHAPE, "embed_dims must be 256");
  if (rows >= kMaxElems) return bad(S4D_ERR_UNSUPPORTED_SHAPE, "rows must be < 2^31");
  const bool res = residual_mode != S4D_RESIDUAL_NONE;
  if (out_ld < (residual_mode == S4D_RESIDUAL_CAT ? 2 : 1) * embed_dims || out_ld % 4 != 0)
    return bad(S4D_ERR_INVALID_ARG, "out_ld too small or not a multiple of 4");
  if (res && (instance_ld < embed_dims || instance_ld % 4 != 0))
    return bad(S4D_ERR_INVALID_ARG, "instance_ld must be >= embed_dims and a multiple of 4");
  if (rows == 0) return S4D_OK;
  if (features == nullptr || weight == nullptr || out == nullptr || (res && instance_feature == nullptr))
    return bad(S4D_ERR_INVALID_ARG, "null pointer");
  if (!aligned(features, 16) || !aligned(weight, 16) || !aligned(out, 16) || (bias != nullptr && !aligned(bias, 16)) ||
      (res && !aligned(instance_feature, 16)))
    return bad(S4D_ERR_INVALID_ARG, "misaligned pointer");
  OprojParams p{};
  p.feat = features;
  p.feat2 = features2;
  p.feat_rows = feature_rows;
  p.feat_row0 = row0;
  p.w = weight;
  p.bias = bias;
  p.res = res ? instance_feature : nullptr;
  p.res_ld = instance_ld;
  p.res_mode = residual_mode;
  p.out = out;
  p.out_ld = out_ld;
  p.rows = rows;
  p.k = (int)embed_dims;
  p.error_flag = error_flag;
  p.wait_limit_ns = tc_wait_limit_ns();
  return launch_output_proj(p, static_cast<cudaStream_t>(stream));
}

}  // namespace
