// Per-level FPN outputs -> the packed channels-last feature buffer the gather reads,
// mc_ms_feat[b, c * sum(HW) + level_start + y * W + x, ch], with the cast to the gather's
// element type fused in.  Replaces the reshape + typecast the reference applies to every FPN
// level before its grid_sample (model/sparse4d.py:549-558, FPN output format model/fpn.py:90-98).
//
//   NCHW sources [bs, Ncam, C, H, W] (a PyTorch FPN):   a tiled transpose through shared memory,
//       64 channels x 64 pixels per CTA, read along pixels (4-pixel vectors) and written along
//       channels (channel pairs), both coalesced.
//   channels-last sources [bs, Ncam, H, W, C] (the reference's [1, 1, N*H*W, C] levels): a
//       straight copy + cast of each (batch, camera, level) block, 8 channels per thread.
// HBM-bound: 4 (fp32) or 2 (bf16) bytes read and 2 or 4 bytes written per element.
#include "params.cuh"

namespace s4d {
namespace {

constexpr int kTile = 64;

template <typename S>
__device__ __forceinline__ float to_f32(S v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

// Two channels as one 4- (bf16) or 8-byte (fp32) store.
__device__ __forceinline__ void store2(float* p, float a, float b) { *reinterpret_cast<float2*>(p) = make_float2(a, b); }
__device__ __forceinline__ void store2(__nv_bfloat16* p, float a, float b) {
  *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
}

// grid (ceil(HW / 64), C / 64, bs * Ncam), block 256 (8 warps).  Loads: with HW % 4 == 0 each
// thread reads 4 float4-sized runs of 4 pixels (rows t / 16 + 16 k, pixels 4 (t % 16) ..), else
// one element at a time; stores: warp w writes pixels w, w + 8, ..., lane l channels 2l, 2l + 1,
// so one store instruction writes one pixel's 64 channels.
template <typename S, typename D, bool VEC>
__global__ void __launch_bounds__(256) pack_nchw_kernel(const S* __restrict__ src, D* __restrict__ dst, int hw,
                                                        int channels, int num_cams, int64_t rows_per_item,
                                                        int64_t cam_rows, int64_t level_start) {
  __shared__ float tile[kTile][kTile + 1];
  const int p0 = blockIdx.x * kTile, c0 = blockIdx.y * kTile;
  const int bc = blockIdx.z;  // b * Ncam + cam
  const int b = bc / num_cams, cam = bc - b * num_cams;
  const S* s = src + ((int64_t)bc * channels + c0) * hw + p0;
  const int t = threadIdx.x;
  if (VEC) {
    const int q = t & 15;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int r = (t >> 4) + 16 * k;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (p0 + 4 * q < hw) {  // hw % 4 == 0: the whole run is inside
        if (sizeof(S) == 4) {
          const float4 f = __ldg(reinterpret_cast<const float4*>(s + (int64_t)r * hw) + q);
          v[0] = f.x, v[1] = f.y, v[2] = f.z, v[3] = f.w;
        } else {
          const uint2 u = __ldg(reinterpret_cast<const uint2*>(s + (int64_t)r * hw) + q);
          v[0] = __uint_as_float(u.x << 16), v[1] = __uint_as_float(u.x & 0xffff0000u);
          v[2] = __uint_as_float(u.y << 16), v[3] = __uint_as_float(u.y & 0xffff0000u);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) tile[r][4 * q + j] = v[j];
    }
  } else {
    const int tx = t & 63, ty = t >> 6;
    for (int r = ty; r < kTile; r += 4) tile[r][tx] = p0 + tx < hw ? to_f32<S>(s[(int64_t)r * hw + tx]) : 0.f;
  }
  __syncthreads();
  const int warp = t >> 5, lane = t & 31;
  D* d = dst + ((int64_t)b * rows_per_item + cam * cam_rows + level_start + p0) * channels + c0;
#pragma unroll
  for (int r = warp; r < kTile; r += 8)
    if (p0 + r < hw) store2(d + (int64_t)r * channels + 2 * lane, tile[2 * lane][r], tile[2 * lane + 1][r]);
}

// 8 consecutive elements as fp32 (16- or 32-byte vector loads) and back.
__device__ __forceinline__ void load8(const float* p, float (&f)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w, f[4] = b.x, f[5] = b.y, f[6] = b.z, f[7] = b.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
  bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(p)), f);
}
__device__ __forceinline__ void store8(float* p, const float (&f)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 v;
  uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
    w[k] = *reinterpret_cast<const uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(p) = v;
}

// grid (ceil(HW * C / 8 / 256), bs * Ncam), block 256: 8 channels per thread.
template <typename S, typename D>
__global__ void __launch_bounds__(256) pack_nhwc_kernel(const S* __restrict__ src, D* __restrict__ dst, int hw,
                                                        int channels, int num_cams, int64_t rows_per_item,
                                                        int64_t cam_rows, int64_t level_start) {
  const int bc = blockIdx.y;
  const int b = bc / num_cams, cam = bc - b * num_cams;
  const int64_t n = (int64_t)hw * channels;
  const int64_t i = ((int64_t)blockIdx.x * 256 + threadIdx.x) * 8;
  if (i >= n) return;
  float f[8];
  load8(src + (int64_t)bc * n + i, f);
  store8(dst + ((int64_t)b * rows_per_item + cam * cam_rows + level_start) * channels + i, f);
}

template <typename S, typename D>
int launch_levels(const PackParams& p, cudaStream_t stream) {
  int64_t per_cam = 0;
  for (int l = 0; l < p.num_levels; ++l) per_cam += (int64_t)p.h[l] * p.w[l];
  const int64_t rows_per_item = per_cam * p.num_cams;
  int64_t start = 0;
  for (int l = 0; l < p.num_levels; ++l) {
    const int hw = p.h[l] * p.w[l];
    const S* src = static_cast<const S*>(p.src[l]);
    D* dst = static_cast<D*>(p.dst);
    if (p.layout == S4D_MAPS_NCHW) {
      const dim3 grid((hw + kTile - 1) / kTile, p.channels / kTile, p.bs * p.num_cams);
      if (hw % 4 == 0)  // rows of whole 4-pixel runs, 16-byte aligned given an aligned level base
        pack_nchw_kernel<S, D, true><<<grid, 256, 0, stream>>>(src, dst, hw, p.channels, p.num_cams, rows_per_item,
                                                                per_cam, start);
      else
        pack_nchw_kernel<S, D, false><<<grid, 256, 0, stream>>>(src, dst, hw, p.channels, p.num_cams,
                                                                 rows_per_item, per_cam, start);
    } else {
      const int64_t n = (int64_t)hw * p.channels;
      const dim3 grid((unsigned)((n / 8 + 255) / 256), p.bs * p.num_cams);
      pack_nhwc_kernel<S, D><<<grid, 256, 0, stream>>>(src, dst, hw, p.channels, p.num_cams, rows_per_item, per_cam,
                                                        start);
    }
    const int st = cuda_check(cudaGetLastError(), "pack kernel launch");
    if (st != S4D_OK) return st;
    start += hw;
  }
  return S4D_OK;
}

}  // namespace

int launch_pack_maps(const PackParams& p, cudaStream_t stream) {
  const bool sf = p.src_dtype == S4D_DTYPE_F32, df = p.dst_dtype == S4D_DTYPE_F32;
  if (sf && df) return launch_levels<float, float>(p, stream);
  if (sf && !df) return launch_levels<float, __nv_bfloat16>(p, stream);
  if (!sf && df) return launch_levels<__nv_bfloat16, float>(p, stream);
  return launch_levels<__nv_bfloat16, __nv_bfloat16>(p, stream);
}

}  // namespace s4d
