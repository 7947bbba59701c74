// Keypoint generation and projection arithmetic shared by the keypoint kernel (kps_project.cu)
// and the gather that computes its own sample locations (dfa_gather.cu), so both produce the
// same bits.
//
// Follows the reference's _KPSGenerator.forward (test/dfa_pcc.py:225-247) and project_points
// (test/dfa_pcc.py:322-333); in TT-NN ttnn.kps_project_fused
// (tt-metal/ops/kps_project_fused/device/kernels/dataflow/reader_kps_project.cpp:255-289) fed by
// _kps_generator_pre_rotation (model/deformable_feature_aggregation.py:651-677).
//
// Arithmetic order is fixed and fused multiply-add is disabled on every line that decides a
// mask bit (the __f*_rn intrinsics):
//   X_r = ((P[r][0]*px + P[r][1]*py) + P[r][2]*pz) + P[r][3];   z = X_2 < 1e-5 ? 1e-5 : X_2
//   u = (X_0 / z) / w;   v = (X_1 / z) / h
// u and v are first formed with one fast division each; where either lies within 1e-5 of 0 or 1
// (or is not finite) the correctly rounded divisions above are used instead, so the visibility
// decisions are those of the exact expression and the sample locations are within a few ulp.
#pragma once

#include "common.cuh"

namespace s4d {

__device__ __forceinline__ float kps_sigmoid_rn(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }

// Keypoint p of one anchor before rotation: fix_scale[p] * exp(size) for the first num_fix
// points, (sigmoid(logit) - 0.5) * exp(size) for the learnable ones (lg: the anchor's
// num_learnable * 3 logits).
__device__ __forceinline__ void kps_scaled(const float* a, const float* fix_scale, int num_fix, const float* lg, int p,
                                           float& kx, float& ky, float& kz) {
  const float sx = expf(a[3]), sy = expf(a[4]), sz = expf(a[5]);
  if (p < num_fix) {
    const float* fs = fix_scale + p * 3;
    kx = __fmul_rn(fs[0], sx);
    ky = __fmul_rn(fs[1], sy);
    kz = __fmul_rn(fs[2], sz);
  } else {
    const float* l = lg + (p - num_fix) * 3;
    kx = __fmul_rn(__fsub_rn(kps_sigmoid_rn(l[0]), 0.5f), sx);
    ky = __fmul_rn(__fsub_rn(kps_sigmoid_rn(l[1]), 0.5f), sy);
    kz = __fmul_rn(__fsub_rn(kps_sigmoid_rn(l[2]), 0.5f), sz);
  }
}

// Yaw rotation by the anchor's (sin, cos) = (a[6], a[7]) and translation to its centre a[0..2].
__device__ __forceinline__ void kps_place(const float* a, float kx, float ky, float kz, float& px, float& py,
                                          float& pz) {
  const float s = a[6], c = a[7];
  const float rx = __fsub_rn(__fmul_rn(c, kx), __fmul_rn(s, ky));
  const float ry = __fadd_rn(__fmul_rn(s, kx), __fmul_rn(c, ky));
  px = __fadd_rn(rx, a[0]);
  py = __fadd_rn(ry, a[1]);
  pz = __fadd_rn(kz, a[2]);
}

__device__ __forceinline__ float kps_proj_row(float4 r, float px, float py, float pz) {
  return __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(r.x, px), __fmul_rn(r.y, py)), __fmul_rn(r.z, pz)), r.w);
}

// Normalised image coordinates of a world point in one camera (r0..r2: the first three rows of
// its 4x4 lidar2img; w, h: image width and height); in_front = depth > 1e-5.
__device__ __forceinline__ void kps_uv(float4 r0, float4 r1, float4 r2, float w, float h, float px, float py, float pz,
                                       float& u, float& v, bool& in_front) {
  const float X0 = kps_proj_row(r0, px, py, pz);
  const float X1 = kps_proj_row(r1, px, py, pz);
  const float X2 = kps_proj_row(r2, px, py, pz);
  in_front = X2 > 1e-5f;
  const float z = X2 < 1e-5f ? 1e-5f : X2;  // torch.clamp(min=1e-5): NaN stays NaN
  u = __fdividef(X0, z * w);
  v = __fdividef(X1, z * h);
  if (fabsf(u) < 1e-5f || fabsf(u - 1.0f) < 1e-5f || fabsf(v) < 1e-5f || fabsf(v - 1.0f) < 1e-5f ||
      !(fabsf(u) < 1e30f && fabsf(v) < 1e30f)) {
    u = __fdiv_rn(__fdiv_rn(X0, z), w);
    v = __fdiv_rn(__fdiv_rn(X1, z), h);
  }
}

}  // namespace s4d
