// Launch parameters and launcher declarations shared by the kernel translation units and the
// C-ABI layer (capi.cu).
#pragma once

#include "common.cuh"

namespace s4d {

struct KpsParams {
  const float* anchor;
  int anchor_dim;
  const float* fix_scale;
  int num_fix;
  const float* learnable;  // [n, num_learnable*3] logits, or null
  int num_learnable;
  const float* kp_pre;  // [n, P, 3] pre-rotation keypoints (kps_project_fused mode), or null
  const float* proj;    // [bs, ncam, 4, 4]
  const float* wh;      // [bs, ncam, 2]
  int bs, num_anchor, num_cams, num_pts;
  int layout;
  int64_t total;  // bs * A * ncam * P
  float* key_points;
  float* loc;
  uint8_t* mask;
  int32_t* block_counts;  // [num_blocks] (compaction only)
  uint32_t* vis_words;    // [num_blocks * 32] (compaction only)
  FastDiv div_anchor_elems;  // by num_cams * num_pts (element -> linear anchor)
  FastDiv div_pts;           // by num_pts
  FastDiv div_anchors;       // by num_anchor (linear anchor -> batch)
  // Learnable keypoint logits computed in the kernel from the instance feature (instead of
  // `learnable`): logit[o] = b_kps[o] + inst[n, :] . w_kps[o, :].
  const float* inst;  // [n, embed_dims] rows of stride inst_ld, or null
  int64_t inst_ld;
  const float* w_kps;  // [num_learnable * 3, embed_dims]
  const float* b_kps;  // [num_learnable * 3] or null
  int embed_dims;
};

// In-kernel learnable logits of kps_project_kernel: at most this many anchors per block (their
// instance rows are staged in shared memory), embed_dims 256, at most 32 logits per anchor.
constexpr int kKpsMaxFusedAnchors = 20;
constexpr int kKpsMaxFusedLogits = 32;

// Largest Ncam*L*P*G the gather stages per anchor in shared memory (48 KiB of fp32).
constexpr int kGatherMaxWeights = 12288;

struct GatherParams {
  const void* feat;
  int64_t num_feat;  // pixel rows per batch item
  const int32_t* spatial_shape;
  const int32_t* scale_start;
  const float* loc;
  const float* weights;
  const float* weights_cam;
  float* out;
  int32_t* error_flag;
  float* cam_ws;  // split logits: per-frame camera softmax factors, or null
  int bs, num_anchor, num_cams, num_levels, num_pts, num_groups;
  int cam_begin, cam_end;
  int logits;
  int layout;
  int factors_ready;  // split logits: cam_ws already holds the camera factors (no prep launch)
  unsigned* anchor_counter;  // warp kernel: next anchor to take (in the workspace, zeroed per launch)
  FastDiv div_anchor;        // warp kernel: by num_anchor (linear anchor -> frame)
  // Sample locations computed in the gather from the anchors (kps_anchor != null; loc unused):
  // keypoints as kps_project's, projected with kps_proj [bs, Ncam, 4, 4] and kps_wh [bs, Ncam, 2].
  const float* kps_anchor;     // [bs * A, kps_anchor_dim]
  int kps_anchor_dim;
  const float* kps_fix_scale;  // [kps_num_fix, 3]
  int kps_num_fix;
  const float* kps_learnable;  // [bs * A, (P - kps_num_fix) * 3] logits
  const float* kps_proj;
  const float* kps_wh;
  // Output routing (warp and cooperative kernels): the rows (flattened anchors) in
  // [peer_row_begin, peer_row_end) go to out_peer + row * 256 (another GPU's buffer, mapped)
  // instead of out + row * 256.
  float* out_peer;
  int64_t peer_row_begin, peer_row_end;
};

// Tensor-core linears (linear_tc.cu).  Row strides are in floats.
struct WfcParams {
  const float* inst;  // [rows, k], row stride inst_ld
  int64_t inst_ld;
  const float* embed;  // [rows, k], row stride embed_ld
  int64_t embed_ld;
  const float* w_fc;        // [n_logits, k]
  const float* w_kps;       // [n_learn, k] or null
  const float* learn_bias;  // [n_learn] or null
  float* logits;            // [rows, n_logits]
  float* learnable;         // [rows, n_learn]
  int64_t rows;
  int n_logits, n_learn, k;
  int32_t* error_flag;
  unsigned long long wait_limit_ns;  // limit of the pipeline's barrier waits (tc_wait_limit_ns())
};

struct OprojParams {
  const float* feat;   // [feat_rows, k]: rows feat_row0 ... feat_row0 + rows - 1 are used
  const float* feat2;  // null, or a second [feat_rows, k] source added to feat (may be a peer's memory)
  int64_t feat_rows;   // rows of the feature sources (0: rows)
  int64_t feat_row0;
  const float* w;     // [k, k]
  const float* bias;  // [k] or null
  const float* res;   // residual rows, row stride res_ld (add / cat)
  int64_t res_ld;
  int res_mode;
  float* out;  // [rows, out_ld]
  int64_t out_ld;
  int64_t rows;
  int k;
  int32_t* error_flag;
  unsigned long long wait_limit_ns;  // limit of the pipeline's barrier waits (tc_wait_limit_ns())
};

// Camera encoder + per-camera logit term (camera_encoder.cu).
struct CamEncParams {
  const float* proj;  // [bs, num_cams, 4, 4]
  const float *w1, *b1, *ln1_w, *ln1_b;  // Linear 12 -> C, LayerNorm
  const float *w2, *b2, *ln2_w, *ln2_b;  // Linear C -> C, LayerNorm
  const float *w_fc, *b_fc;              // weights_fc [num_logits, C], [num_logits]
  float* camera_embed;                   // [bs, num_cams, C] or null
  float* logits;                         // [bs, num_cams, num_logits]
  float* hidden;                         // [bs, num_cams, C] scratch (workspace); unused by camera_terms
  float* factors;                        // camera_terms: softmax factors [bs, num_cams + 1, num_logits] or null
  unsigned* anchor_counter;              // camera_terms: the gather's anchor counter pair, zeroed with factors
  int bs, num_cams, num_logits, embed_dims;
};

int launch_camera_logits(const CamEncParams& p, cudaStream_t stream);
int launch_camera_terms(const CamEncParams& p, cudaStream_t stream);

// Packing of per-level feature maps (pack_maps.cu).
constexpr int kMaxPackLevels = 8;
struct PackParams {
  const void* src[kMaxPackLevels];
  int h[kMaxPackLevels], w[kMaxPackLevels];
  int num_levels, bs, num_cams, channels;
  int layout, src_dtype, dst_dtype;
  void* dst;
};

int launch_pack_maps(const PackParams& p, cudaStream_t stream);

// InstanceBank (instance_bank.cu).
struct IbProjectParams {
  const float* anchor;         // [bs, num, 11]
  const float* T;              // [bs, 4, 4]
  const float* time_interval;  // [bs] or null (no motion term)
  float* out;                  // [bs, num, 11]
  int bs, num, anchor_dim;
};

struct IbSelectParams {
  const float* feature;     // [bs, A, C]
  const float* anchor;      // [bs, A, D]
  const float* confidence;  // [bs, A, num_cls]
  const float* prev_conf;   // CACHE: [bs, num_temp] or null
  float decay;
  const float* cached_feature;  // UPDATE: [bs, num_temp, C]
  const float* cached_anchor;   // UPDATE: [bs, num_temp, D]
  const uint8_t* mask;          // UPDATE: [bs] or null (all frames merge)
  float* out_feature;           // CACHE: [bs, num_temp, C]; UPDATE: [bs, A, C]
  float* out_anchor;            // CACHE: [bs, num_temp, D]; UPDATE: [bs, A, D]
  float* out_conf;              // CACHE: [bs, num_temp] or null
  int32_t* out_idx;             // CACHE: [bs, num_temp]; UPDATE: [bs, A - num_temp]; or null
  int bs, num_anchor, num_cls, embed_dims, anchor_dim, num_temp, sort_size;
};

// Limit of the tensor-core kernels' pipeline waits for launches from this host thread (2 s
// unless s4d_set_tc_wait_limit_ns changed it).
unsigned long long tc_wait_limit_ns();

int launch_ib_project(const IbProjectParams& p, cudaStream_t stream);
int launch_ib_select(IbSelectParams p, bool cache, cudaStream_t stream);
int launch_weights_fc(const WfcParams& p, cudaStream_t stream);
int launch_output_proj(const OprojParams& p, cudaStream_t stream);

int launch_kps_project(KpsParams k, int32_t* visible_idx, int32_t* visible_count, void* workspace,
                       cudaStream_t stream);
size_t kps_workspace_bytes(int64_t total);

int launch_gather(const GatherParams& p, int feat_dtype, cudaStream_t stream);
int launch_cam_factors(const float* weights_cam, float* cam_ws, int bs, int ncam, int nl, int np, int G,
                       cudaStream_t stream);
size_t gather_workspace_bytes(int64_t bs, int ncam, int nl, int np, int G);
size_t gather_smem_bytes(int ncam, int nl, int np, int G, int cam_begin, int cam_end);

}  // namespace s4d
