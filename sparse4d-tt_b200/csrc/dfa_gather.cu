// Kernels (b)+(c): group softmax of the weight logits fused with the multi-camera,
// multi-scale bilinear gather and the weighted sum over cameras, levels and points.
//
// Computes, for every (batch b, anchor a) and channel ch = g*D + d,
//   out[b, a, ch] = sum_{c, l, p} softmax_{c,l,p}(logit[b, a, :, :, :, g]) *
//                   bilinear(feat[b, camera c, level l], uv[b, a, c, p])[ch]
// which is the reference's feature_sampling + multi_view_level_fusion + sum over points
// (test/dfa_pcc.py:298,335-358: F.grid_sample, zeros padding, align_corners=False) and, in
// TT-NN, ttnn.softmax + grid_sample + transposed_s2i + grouped_weighted_sum
// (model/deformable_feature_aggregation.py:791-796,877-899).  The [cams*levels*pts, A, C]
// intermediate of the reference is never materialised.
//
// One CTA of 256 threads (8 warps) per anchor:
//   1. stage the anchor's logits (Ncam*L*P*G fp32) and sample locations in shared memory,
//      together with the (H, W, start) of every (camera, level);
//   2. per-group max and sum of exp over the Ncam*L*P entries: block reductions in which
//      thread t only ever touches group t % G (256 % G == 0), exp values written back;
//   3. build the list of in-bounds samples (any of the 4 taps inside the map) with a
//      deterministic ballot compaction: tap pixel indices, bilinear weights, entry index;
//   4. the 8 warps stride over the list; lane l holds channels 8l..8l+7 (group l*8/D) and
//      reads each tap as one 16-byte vector (bf16) or two (fp32): a tap is one coalesced
//      512-byte row (1 KiB for fp32).  The 4 taps of a sample are in flight together and
//      accumulate in fp32 registers; 32 resident warps per SM keep enough loads in flight;
//   5. the 8 warps' partial sums are added through shared memory and scaled by 1/sum_exp.
// No tensor cores: this is a gather with ~0.1 flop per byte.
#include "params.cuh"

namespace s4d {

constexpr int kGatherThreads = 256;
constexpr int kGatherWarps = kGatherThreads / 32;
constexpr int kChannels = 256;      // embed dims: one warp row of 32 lanes x 8 channels

struct GatherSmem {
  int n_w;       // Ncam*L*P*G
  int n_samp;    // (cam_end-cam_begin)*L*P
  int off_w, off_loc, off_lvl, off_pix, off_bw, off_clp, off_red;
  size_t bytes;
};

__host__ __device__ inline GatherSmem gather_smem_layout(int ncam, int nl, int np, int G, int cam_begin, int cam_end) {
  GatherSmem s;
  s.n_w = ncam * nl * np * G;
  s.n_samp = (cam_end - cam_begin) * nl * np;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = (o + bytes + 15) & ~(size_t)15;
    return (int)at;
  };
  s.off_w = take((size_t)s.n_w * 4);
  s.off_loc = take((size_t)ncam * np * 2 * 4);
  s.off_lvl = take((size_t)ncam * nl * 4 * 4);
  // sample list (pix int4, bw float4, entry int); reused for the cross-warp reduction
  const size_t list = (size_t)s.n_samp * 36 + 48;
  const size_t red = (size_t)kGatherWarps * kChannels * 4;
  const size_t region = list > red ? list : red;
  s.off_pix = take(region);
  s.off_bw = s.off_pix + (int)(((size_t)s.n_samp * 16 + 15) & ~(size_t)15);
  s.off_clp = s.off_bw + (int)(((size_t)s.n_samp * 16 + 15) & ~(size_t)15);
  s.off_red = s.off_pix;
  s.bytes = o;
  return s;
}

template <typename T>
struct FeatLoad;

template <>
struct FeatLoad<__nv_bfloat16> {
  using Vec = uint4;  // 8 channels
  static __device__ __forceinline__ Vec load(const __nv_bfloat16* row, int lane) {
    return ldg_nc_v4(row + lane * 8);
  }
  static __device__ __forceinline__ void widen(const Vec& v, float (&f)[8]) { bf16x8_to_f32(v, f); }
};

struct F32x8 {
  float4 a, b;
};

template <>
struct FeatLoad<float> {
  using Vec = F32x8;
  static __device__ __forceinline__ Vec load(const float* row, int lane) {
    F32x8 v;
    v.a = ldg_nc_f4(row + lane * 8);
    v.b = ldg_nc_f4(row + lane * 8 + 4);
    return v;
  }
  static __device__ __forceinline__ void widen(const Vec& v, float (&f)[8]) {
    f[0] = v.a.x; f[1] = v.a.y; f[2] = v.a.z; f[3] = v.a.w;
    f[4] = v.b.x; f[5] = v.b.y; f[6] = v.b.z; f[7] = v.b.w;
  }
};

// Reduction over the threads that share a group (t % G) of the whole block.
template <bool kMax>
__device__ __forceinline__ void group_reduce(float v, int G, float* s_tmp, float* s_out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = G; o < 32; o <<= 1) {
    const float t = __shfl_xor_sync(0xffffffffu, v, o);
    v = kMax ? fmaxf(v, t) : v + t;
  }
  if (lane < G) s_tmp[warp * 32 + lane] = v;
  __syncthreads();
  if (threadIdx.x < G) {
    float r = s_tmp[threadIdx.x];
#pragma unroll
    for (int w = 1; w < kGatherWarps; ++w) {
      const float t = s_tmp[w * 32 + threadIdx.x];
      r = kMax ? fmaxf(r, t) : r + t;
    }
    s_out[threadIdx.x] = r;
  }
  __syncthreads();
}

template <typename T>
__global__ void __launch_bounds__(kGatherThreads, 4) dfa_gather_kernel(GatherParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ float s_tmp[kGatherWarps * 32];
  __shared__ float s_gmax[32];
  __shared__ float s_gsum[32];
  __shared__ float s_ginv[32];
  __shared__ int s_wcnt[kGatherWarps];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = p.num_groups, ncam = p.num_cams, nl = p.num_levels, np = p.num_pts;
  const GatherSmem L = gather_smem_layout(ncam, nl, np, G, p.cam_begin, p.cam_end);
  float* s_w = reinterpret_cast<float*>(smem + L.off_w);
  float* s_loc = reinterpret_cast<float*>(smem + L.off_loc);
  int4* s_lvl = reinterpret_cast<int4*>(smem + L.off_lvl);  // (H, W, start, ok)
  int4* s_pix = reinterpret_cast<int4*>(smem + L.off_pix);
  float4* s_bw = reinterpret_cast<float4*>(smem + L.off_bw);
  int* s_clp = reinterpret_cast<int*>(smem + L.off_clp);
  float* s_red = reinterpret_cast<float*>(smem + L.off_red);

  const int64_t anchor_lin = blockIdx.x;  // b * A + a
  const int b = (int)(anchor_lin / p.num_anchor);

  // ---- 1. stage levels, logits, locations -------------------------------------------------
  for (int i = tid; i < ncam * nl; i += kGatherThreads) {
    const int H = p.spatial_shape[2 * i], W = p.spatial_shape[2 * i + 1], st = p.scale_start[i];
    const bool ok = H > 0 && W > 0 && st >= 0 && (int64_t)st + (int64_t)H * W <= p.num_feat;
    const int c = i / nl;
    if (!ok && c >= p.cam_begin && c < p.cam_end && p.error_flag != nullptr && blockIdx.x == 0)
      atomicOr(p.error_flag, S4D_FLAG_BAD_LEVEL);
    s_lvl[i] = make_int4(H, W, st, ok ? 1 : 0);
  }
  const int n_w = L.n_w;
  if (p.weights_cam != nullptr) {
    const int lpg = nl * np * G;
    const float* wa = p.weights + anchor_lin * lpg;
    const float* wc = p.weights_cam + (int64_t)b * ncam * lpg;
    for (int i = tid; i < n_w; i += kGatherThreads) s_w[i] = __ldg(wa + i % lpg) + __ldg(wc + i);
  } else if (p.layout == S4D_LAYOUT_CAM_MAJOR) {
    const float* src = p.weights + anchor_lin * n_w;
    if ((n_w & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
      const float4* s4 = reinterpret_cast<const float4*>(src);
      float4* d4 = reinterpret_cast<float4*>(s_w);
      for (int i = tid; i < (n_w >> 2); i += kGatherThreads) d4[i] = ldg_nc_f4(s4 + i);
    } else {
      for (int i = tid; i < n_w; i += kGatherThreads) s_w[i] = __ldg(src + i);
    }
  } else {  // PT_MAJOR: [P, Ncam, L, G] -> [Ncam, L, P, G]
    const float* src = p.weights + anchor_lin * n_w;
    for (int i = tid; i < n_w; i += kGatherThreads) {
      const int g = i % G;
      int r = i / G;
      const int l = r % nl;
      r /= nl;
      const int c = r % ncam;
      const int pt = r / ncam;
      s_w[((c * nl + l) * np + pt) * G + g] = __ldg(src + i);
    }
  }
  {
    const int n_loc = ncam * np;
    const float2* src = reinterpret_cast<const float2*>(p.loc) + anchor_lin * n_loc;
    for (int i = tid; i < n_loc; i += kGatherThreads) {
      const float2 v = __ldg(src + i);
      int dst = i;
      if (p.layout == S4D_LAYOUT_PT_MAJOR) {  // i = pt * ncam + c
        const int pt = i / ncam, c = i - pt * ncam;
        dst = c * np + pt;
      }
      s_loc[2 * dst] = v.x;
      s_loc[2 * dst + 1] = v.y;
    }
  }
  __syncthreads();

  // ---- 2. softmax statistics per group ------------------------------------------------------
  if (p.logits) {
    float m = -INFINITY;
    for (int i = tid; i < n_w; i += kGatherThreads) m = fmaxf(m, s_w[i]);
    group_reduce<true>(m, G, s_tmp, s_gmax);
    const float mg = s_gmax[tid % G];
    float sum = 0.0f;
    for (int i = tid; i < n_w; i += kGatherThreads) {
      const float e = expf(s_w[i] - mg);
      s_w[i] = e;
      sum += e;
    }
    group_reduce<false>(sum, G, s_tmp, s_gsum);
    if (tid < G) s_ginv[tid] = 1.0f / s_gsum[tid];
  } else {
    if (tid < G) s_ginv[tid] = 1.0f;
  }

  // ---- 3. in-bounds sample list -----------------------------------------------------------
  const int lp = nl * np;
  int n_valid = 0;
  for (int base = 0; base < L.n_samp; base += kGatherThreads) {
    const int i = base + tid;
    bool valid = false;
    int4 pix = make_int4(-1, -1, -1, -1);
    float4 bw = make_float4(0.f, 0.f, 0.f, 0.f);
    int clp = 0;
    if (i < L.n_samp) {
      const int c = p.cam_begin + i / lp;
      const int r = i - (i / lp) * lp;
      const int l = r / np, pt = r - l * np;
      const int4 lv = s_lvl[c * nl + l];
      const float u = s_loc[2 * (c * np + pt)], v = s_loc[2 * (c * np + pt) + 1];
      // grid_sample un-normalisation (align_corners=False) of the grid value 2u - 1
      const float Wf = (float)lv.y, Hf = (float)lv.x;
      const float ix = ((u * 2.0f - 1.0f + 1.0f) * Wf - 1.0f) * 0.5f;
      const float iy = ((v * 2.0f - 1.0f + 1.0f) * Hf - 1.0f) * 0.5f;
      if (lv.w && ix > -1.0f && ix < Wf && iy > -1.0f && iy < Hf) {
        const float x0f = floorf(ix), y0f = floorf(iy);
        const int x0 = (int)x0f, y0 = (int)y0f;
        const float x1f = x0f + 1.0f, y1f = y0f + 1.0f;
        const bool vx0 = x0 >= 0, vx1 = x0 + 1 < lv.y, vy0 = y0 >= 0, vy1 = y0 + 1 < lv.x;
        const int p00 = lv.z + y0 * lv.y + x0;
        pix = make_int4(vx0 && vy0 ? p00 : -1, vx1 && vy0 ? p00 + 1 : -1, vx0 && vy1 ? p00 + lv.y : -1,
                        vx1 && vy1 ? p00 + lv.y + 1 : -1);
        bw = make_float4((x1f - ix) * (y1f - iy), (ix - x0f) * (y1f - iy), (x1f - ix) * (iy - y0f),
                         (ix - x0f) * (iy - y0f));
        clp = (c * nl + l) * np + pt;
        valid = true;
      }
    }
    const uint32_t ball = __ballot_sync(0xffffffffu, valid);
    if (lane == 0) s_wcnt[warp] = __popc(ball);
    __syncthreads();
    int off = n_valid;
    int tot = 0;
#pragma unroll
    for (int w = 0; w < kGatherWarps; ++w) {
      const int cw = s_wcnt[w];
      off += w < warp ? cw : 0;
      tot += cw;
    }
    if (valid) {
      const int pos = off + __popc(ball & ((1u << lane) - 1u));
      s_pix[pos] = pix;
      s_bw[pos] = bw;
      s_clp[pos] = clp;
    }
    n_valid += tot;
    __syncthreads();
  }

  // ---- 4. weighted gather ------------------------------------------------------------------
  using LD = FeatLoad<T>;
  const int D = kChannels / G;
  const int g = (lane * 8) / D;
  const T* fb = static_cast<const T*>(p.feat) + (int64_t)b * p.num_feat * kChannels;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.0f;

  for (int s = warp; s < n_valid; s += kGatherWarps) {
    const int4 pa = s_pix[s];
    const int ia[4] = {pa.x, pa.y, pa.z, pa.w};
    typename LD::Vec va[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (ia[k] >= 0) va[k] = LD::load(fb + (int64_t)ia[k] * kChannels, lane);
    const float4 wa4 = s_bw[s];
    const float wa[4] = {wa4.x, wa4.y, wa4.z, wa4.w};
    const float sa = s_w[s_clp[s] * G + g];
    float ta[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) ta[j] = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (ia[k] >= 0) {
        float f[8];
        LD::widen(va[k], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) ta[j] += wa[k] * f[j];
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] += sa * ta[j];
  }

  // ---- 5. cross-warp reduction -------------------------------------------------------------
  __syncthreads();  // every warp is done with the sample list that s_red aliases
  float4* r4 = reinterpret_cast<float4*>(s_red + warp * kChannels + lane * 8);
  r4[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  r4[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  __syncthreads();
  {
    const int ch = tid;  // kGatherThreads == kChannels
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kGatherWarps; ++w) v += s_red[w * kChannels + ch];
    p.out[anchor_lin * kChannels + ch] = v * s_ginv[ch / D];
  }
}

size_t gather_smem_bytes(int ncam, int nl, int np, int G, int cam_begin, int cam_end) {
  return gather_smem_layout(ncam, nl, np, G, cam_begin, cam_end).bytes;
}

int launch_gather(const GatherParams& p, int feat_dtype, cudaStream_t stream) {
  const size_t smem = gather_smem_bytes(p.num_cams, p.num_levels, p.num_pts, p.num_groups, p.cam_begin, p.cam_end);
  const unsigned grid = (unsigned)((int64_t)p.bs * p.num_anchor);
  if (feat_dtype == S4D_DTYPE_BF16) {
    auto k = dfa_gather_kernel<__nv_bfloat16>;
    if (smem > 48 * 1024) {
      int st = cuda_check(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                          "cudaFuncSetAttribute(gather bf16)");
      if (st) return st;
    }
    k<<<grid, kGatherThreads, smem, stream>>>(p);
  } else {
    auto k = dfa_gather_kernel<float>;
    if (smem > 48 * 1024) {
      int st = cuda_check(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                          "cudaFuncSetAttribute(gather f32)");
      if (st) return st;
    }
    k<<<grid, kGatherThreads, smem, stream>>>(p);
  }
  return cuda_check(cudaGetLastError(), "dfa_gather_kernel launch");
}

}  // namespace s4d
