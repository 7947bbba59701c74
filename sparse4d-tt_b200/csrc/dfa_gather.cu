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
// Kernels, chosen by launch_gather():
//   dfa_gather_warp_kernel   Sparse4D v3 shape (6 cams, 4 levels, 13 points, 8 groups), split
//                            logits with the per-frame camera factors (cam_softmax_prep_kernel)
//                            in the workspace: one warp per anchor, factorised softmax.
//   dfa_gather_coop_kernel   the same with fewer anchors than warp slots (a single frame): 2, 4
//                            or 8 warps per anchor, the anchor's work divided between them.
//   dfa_gather_fast_kernel   Sparse4D v3 shape, cam-major logits (full or split, no workspace):
//                            one CTA per anchor with compile-time dimensions.
//   dfa_gather_kernel        every other shape / layout (generic, described below).
//
// dfa_gather_kernel -- one CTA of 256 threads (8 warps) per anchor:
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
#include <type_traits>

#include "kps_math.cuh"
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

// -----------------------------------------------------------------------------------------------
// Shape-specialised kernel for the Sparse4D v3 layout (compile-time Ncam, L, P, G; cam-major
// logits, full or split).  Same five phases as dfa_gather_kernel, with the fixed per-anchor
// work cut down so that the kernel is bound by memory rather than by instruction issue:
//   * logits staged as float4 (split logits: per-anchor row + per-camera row, both float4)
//     with the running max fused into the staging loop.  Element 4i+k of the staged row
//     belongs to group (4i + k) % G, and with a 256-thread stride i = t (mod 256), so every
//     thread only ever sees the 4 groups (4t + k) % G: 4 register "slots" per thread, reduced
//     across lanes with equal t mod G/4 by xor shuffles and across warps in shared memory;
//   * exp as ex2.approx of a fused (x - max) * log2(e), unnormalised; 1/sum applied once per
//     output channel at the end;
//   * candidate (camera, level, point) indices decoded with compile-time divisors; both
//     candidates of a thread compacted with one block prefix;
//   * taps widened bf16 -> fp32 by shift/mask and accumulated with packed fp32x2 FMA
//     (__ffma2_rn), 4 instructions per 8 channels.
// -----------------------------------------------------------------------------------------------
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
struct TapFma;

template <>
struct TapFma<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* fb, int pix, int lane, uint4& v) {
    v = ldg_nc_v4(fb + (int64_t)pix * kChannels + lane * 8);
  }
  static __device__ __forceinline__ void fma(const uint4& v, float w, float2 (&acc)[4]) {
    const float2 ww = make_float2(w, w);
    const uint32_t q[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = make_float2(__uint_as_float(q[i] << 16), __uint_as_float(q[i] & 0xffff0000u));
      acc[i] = __ffma2_rn(ww, f, acc[i]);
    }
  }
};

template <>
struct TapFma<float> {
  struct V {
    float4 a, b;
  };
  static __device__ __forceinline__ void load(const float* fb, int pix, int lane, V& v) {
    const float* row = fb + (int64_t)pix * kChannels + lane * 8;
    v.a = ldg_nc_f4(row);
    v.b = ldg_nc_f4(row + 4);
  }
  static __device__ __forceinline__ void fma(const V& v, float w, float2 (&acc)[4]) {
    const float2 ww = make_float2(w, w);
    acc[0] = __ffma2_rn(ww, make_float2(v.a.x, v.a.y), acc[0]);
    acc[1] = __ffma2_rn(ww, make_float2(v.a.z, v.a.w), acc[1]);
    acc[2] = __ffma2_rn(ww, make_float2(v.b.x, v.b.y), acc[2]);
    acc[3] = __ffma2_rn(ww, make_float2(v.b.z, v.b.w), acc[3]);
  }
};

// End of a gather launch that took anchors from `counter` (counter[0]: next ticket, counter[1]:
// blocks done): called once per block by one thread after the block has taken its last ticket.
// The last block to get here resets both words, so the next launch on the same workspace starts
// from zero without a memset.  The fence orders this block's ticket atomics before its done
// count, so the last block sees every other block's tickets taken before it resets.
__device__ __forceinline__ void release_anchor_counter(unsigned* counter) {
  __threadfence();
  if (atomicAdd(counter + 1, 1u) == gridDim.x - 1) {
    atomicExch(counter, 0u);
    atomicExch(counter + 1, 0u);
  }
}

// A hint to bring the line holding p into L1; no register is written.
__device__ __forceinline__ void prefetch_l1(const void* p) { asm volatile("prefetch.global.L1 [%0];" ::"l"(p)); }

template <typename T>
struct TapVec {
  using type = uint4;
};
template <>
struct TapVec<float> {
  using type = TapFma<float>::V;
};

// Slot reduction: after it, s_out[g] holds the max (kMax) or sum over every thread's slot
// values of group g, where slot k of thread t belongs to group (4t + k) % G.
template <int G, bool kMax>
__device__ __forceinline__ void slot_reduce(float (&v)[4], float (*s_part)[8][4], float* s_out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = G / 4; o < 32; o <<= 1) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float t = __shfl_xor_sync(0xffffffffu, v[k], o);
      v[k] = kMax ? fmaxf(v[k], t) : v[k] + t;
    }
  }
  if (lane < G / 4) {
#pragma unroll
    for (int k = 0; k < 4; ++k) s_part[warp][lane][k] = v[k];
  }
  __syncthreads();
  if (threadIdx.x < G) {
    const int l = threadIdx.x >> 2, k = threadIdx.x & 3;
    float r = s_part[0][l][k];
#pragma unroll
    for (int w = 1; w < kGatherWarps; ++w) r = kMax ? fmaxf(r, s_part[w][l][k]) : r + s_part[w][l][k];
    s_out[threadIdx.x] = r;
  }
  __syncthreads();
}

template <typename T, int NC, int NL, int NP, int G>
__global__ void __launch_bounds__(kGatherThreads, 4) dfa_gather_fast_kernel(GatherParams p) {
  constexpr int NCLP = NC * NL * NP;
  constexpr int LPG = NL * NP * G;
  constexpr int NW4 = NC * LPG / 4;
  constexpr int LPG4 = LPG / 4;
  constexpr int D = kChannels / G;
  constexpr float kLog2e = 1.4426950408889634f;
  static_assert(LPG % 4 == 0 && G >= 4 && G <= 32 && (G & (G - 1)) == 0, "fast gather shape");
  static_assert(NCLP <= 2 * kGatherThreads, "two candidates per thread");
  static_assert(NCLP * 32 >= kGatherWarps * kChannels * 4, "reduction buffer aliases the sample list");

  __shared__ __align__(16) float4 s_w4[NW4];
  __shared__ __align__(16) float2 s_loc[NC * NP];
  __shared__ __align__(16) int4 s_lvl[NC * NL];  // (H, W, start, ok)
  __shared__ __align__(16) unsigned char s_list[NCLP * 32];
  __shared__ int s_clp[NCLP];
  __shared__ float s_part[kGatherWarps][8][4];
  __shared__ float s_gmax[G];
  __shared__ float s_ginv[G];
  __shared__ int s_wcnt[2][kGatherWarps];

  int4* s_pix = reinterpret_cast<int4*>(s_list);
  float4* s_bw = reinterpret_cast<float4*>(s_list + NCLP * 16);
  float* s_red = reinterpret_cast<float*>(s_list);
  const float* s_w = reinterpret_cast<const float*>(s_w4);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t anchor_lin = blockIdx.x;
  const int b = (int)(anchor_lin / p.num_anchor);

  // ---- 1. stage levels, locations and logits (running max in 4 slots) --------------------
  if (tid < NC * NL) {
    const int H = p.spatial_shape[2 * tid], W = p.spatial_shape[2 * tid + 1], st = p.scale_start[tid];
    const bool ok = H > 0 && W > 0 && st >= 0 && (int64_t)st + (int64_t)H * W <= p.num_feat;
    const int c = tid / NL;
    if (!ok && c >= p.cam_begin && c < p.cam_end && p.error_flag != nullptr && blockIdx.x == 0)
      atomicOr(p.error_flag, S4D_FLAG_BAD_LEVEL);
    s_lvl[tid] = make_int4(H, W, st, ok ? 1 : 0);
  }
  if (tid < NC * NP) s_loc[tid] = __ldg(reinterpret_cast<const float2*>(p.loc) + anchor_lin * (NC * NP) + tid);
  float m[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  if (p.weights_cam != nullptr) {
    const float4* wa = reinterpret_cast<const float4*>(p.weights) + anchor_lin * LPG4;
    const float4* wc = reinterpret_cast<const float4*>(p.weights_cam) + (int64_t)b * NW4;
#pragma unroll
    for (int i = tid; i < NW4; i += kGatherThreads) {
      const int c = i / LPG4;
      const float4 x = __ldg(wa + (i - c * LPG4)), y = __ldg(wc + i);
      const float4 v = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
      s_w4[i] = v;
      m[0] = fmaxf(m[0], v.x);
      m[1] = fmaxf(m[1], v.y);
      m[2] = fmaxf(m[2], v.z);
      m[3] = fmaxf(m[3], v.w);
    }
  } else {
    const float4* src = reinterpret_cast<const float4*>(p.weights) + anchor_lin * NW4;
#pragma unroll
    for (int i = tid; i < NW4; i += kGatherThreads) {
      const float4 v = ldg_nc_f4(src + i);
      s_w4[i] = v;
      m[0] = fmaxf(m[0], v.x);
      m[1] = fmaxf(m[1], v.y);
      m[2] = fmaxf(m[2], v.z);
      m[3] = fmaxf(m[3], v.w);
    }
  }
  slot_reduce<G, true>(m, s_part, s_gmax);  // its barriers also publish s_w4 / s_loc / s_lvl

  // ---- 2. unnormalised exp + 3. candidate validity -----------------------------------------
  float sum[4] = {0.f, 0.f, 0.f, 0.f};
  {
    float mg[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) mg[k] = s_gmax[(4 * tid + k) % G] * kLog2e;
#pragma unroll
    for (int i = tid; i < NW4; i += kGatherThreads) {
      const float4 v = s_w4[i];
      const float4 e = make_float4(ex2_approx(fmaf(v.x, kLog2e, -mg[0])), ex2_approx(fmaf(v.y, kLog2e, -mg[1])),
                                   ex2_approx(fmaf(v.z, kLog2e, -mg[2])), ex2_approx(fmaf(v.w, kLog2e, -mg[3])));
      s_w4[i] = e;
      sum[0] += e.x;
      sum[1] += e.y;
      sum[2] += e.z;
      sum[3] += e.w;
    }
  }
  bool valid[2];
  int4 pix[2];
  float4 bw[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int i = tid + r * kGatherThreads;
    valid[r] = false;
    pix[r] = make_int4(-1, -1, -1, -1);
    bw[r] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < NCLP) {
      const int c = i / (NL * NP);
      const int rem = i - c * (NL * NP);
      const int l = rem / NP, pt = rem - l * NP;
      if (c >= p.cam_begin && c < p.cam_end) {
        const int4 lv = s_lvl[c * NL + l];
        const float2 uv = s_loc[c * NP + pt];
        const float Wf = (float)lv.y, Hf = (float)lv.x;
        const float ix = ((uv.x * 2.0f - 1.0f + 1.0f) * Wf - 1.0f) * 0.5f;
        const float iy = ((uv.y * 2.0f - 1.0f + 1.0f) * Hf - 1.0f) * 0.5f;
        if (lv.w && ix > -1.0f && ix < Wf && iy > -1.0f && iy < Hf) {
          const float x0f = floorf(ix), y0f = floorf(iy);
          const int x0 = (int)x0f, y0 = (int)y0f;
          const float x1f = x0f + 1.0f, y1f = y0f + 1.0f;
          const bool vx0 = x0 >= 0, vx1 = x0 + 1 < lv.y, vy0 = y0 >= 0, vy1 = y0 + 1 < lv.x;
          const int p00 = lv.z + y0 * lv.y + x0;
          pix[r] = make_int4(vx0 && vy0 ? p00 : -1, vx1 && vy0 ? p00 + 1 : -1, vx0 && vy1 ? p00 + lv.y : -1,
                             vx1 && vy1 ? p00 + lv.y + 1 : -1);
          bw[r] = make_float4((x1f - ix) * (y1f - iy), (ix - x0f) * (y1f - iy), (x1f - ix) * (iy - y0f),
                              (ix - x0f) * (iy - y0f));
          valid[r] = true;
        }
      }
    }
  }
  const uint32_t ball0 = __ballot_sync(0xffffffffu, valid[0]);
  const uint32_t ball1 = __ballot_sync(0xffffffffu, valid[1]);
  if (lane == 0) {
    s_wcnt[0][warp] = __popc(ball0);
    s_wcnt[1][warp] = __popc(ball1);
  }
  slot_reduce<G, false>(sum, s_part, s_gmax);  // s_gmax now holds the sums; barriers publish s_wcnt
  if (tid < G) s_ginv[tid] = 1.0f / s_gmax[tid];
  int n_valid = 0, off0 = 0, off1 = 0;
#pragma unroll
  for (int w = 0; w < kGatherWarps; ++w) {
    off0 += w < warp ? s_wcnt[0][w] : 0;
    n_valid += s_wcnt[0][w];
  }
  off1 = n_valid;
#pragma unroll
  for (int w = 0; w < kGatherWarps; ++w) {
    off1 += w < warp ? s_wcnt[1][w] : 0;
    n_valid += s_wcnt[1][w];
  }
  const uint32_t lt = (1u << lane) - 1u;
  if (valid[0]) {
    const int pos = off0 + __popc(ball0 & lt);
    s_pix[pos] = pix[0];
    s_bw[pos] = bw[0];
    s_clp[pos] = tid;
  }
  if (valid[1]) {
    const int pos = off1 + __popc(ball1 & lt);
    s_pix[pos] = pix[1];
    s_bw[pos] = bw[1];
    s_clp[pos] = tid + kGatherThreads;
  }
  __syncthreads();

  // ---- 4. weighted gather -------------------------------------------------------------------
  const int g = lane / (D / 8);
  const T* fb = static_cast<const T*>(p.feat) + (int64_t)b * p.num_feat * kChannels;
  float2 acc[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] = make_float2(0.f, 0.f);
  using V = typename TapVec<T>::type;
  for (int s = warp; s < n_valid; s += kGatherWarps) {
    const int4 px = s_pix[s];
    const float4 w4 = s_bw[s];
    const float sw = s_w[s_clp[s] * G + g];
    V v0, v1, v2, v3;
    if (px.x >= 0) TapFma<T>::load(fb, px.x, lane, v0);
    if (px.y >= 0) TapFma<T>::load(fb, px.y, lane, v1);
    if (px.z >= 0) TapFma<T>::load(fb, px.z, lane, v2);
    if (px.w >= 0) TapFma<T>::load(fb, px.w, lane, v3);
    if (px.x >= 0) TapFma<T>::fma(v0, w4.x * sw, acc);
    if (px.y >= 0) TapFma<T>::fma(v1, w4.y * sw, acc);
    if (px.z >= 0) TapFma<T>::fma(v2, w4.z * sw, acc);
    if (px.w >= 0) TapFma<T>::fma(v3, w4.w * sw, acc);
  }

  // ---- 5. cross-warp reduction -------------------------------------------------------------
  __syncthreads();
  float4* r4 = reinterpret_cast<float4*>(s_red + warp * kChannels + lane * 8);
  r4[0] = make_float4(acc[0].x, acc[0].y, acc[1].x, acc[1].y);
  r4[1] = make_float4(acc[2].x, acc[2].y, acc[3].x, acc[3].y);
  __syncthreads();
  float v = 0.0f;
#pragma unroll
  for (int w = 0; w < kGatherWarps; ++w) v += s_red[w * kChannels + tid];
  p.out[anchor_lin * kChannels + tid] = v * s_ginv[tid / D];
}

// -----------------------------------------------------------------------------------------------
// Split logits, factorised softmax.  With logit[c, lp, g] = wa[lp, g] + wc[c, lp, g] (anchor
// term + camera term, lp = (level, point)):
//   exp(logit - M) = exp(wa - M1[g]) * exp(wc - M2[g])      (M = M1 + M2 cancels in the ratio)
//   sum_{c,lp} exp(logit - M) = sum_lp ea[lp, g] * EC[lp, g],  EC = sum_c exp(wc - M2)
// The camera factors (ec, EC) depend only on the frame, so cam_softmax_prep_kernel computes
// them once per frame into the workspace; each anchor then needs LPG exps and an LPG-term dot
// product (one warp, while the other warps build the sample list) instead of Ncam*LPG exps.
// M1 and M2 are the per-group maxima of each term, so every factor is <= 1.  When a group's
// sum falls below 1e-20 (the largest logit sits > ~46 below M1 + M2, where factors could
// underflow) the anchor switches to the exact two-pass softmax over wa + wc.
// -----------------------------------------------------------------------------------------------
// cam_softmax_prep_kernel also resets the workspace's anchor counter pair (ticket, blocks done)
// that the warp and cooperative gather kernels take anchors from, so that a freshly prepared workspace starts at
// zero; every gather launch then leaves the pair at zero again when its last block exits
// (release_anchor_counter), and no memset has to run between the join of this kernel's stream
// and the gather.
template <int NC, int LPG, int G>
__global__ void __launch_bounds__(kGatherThreads) cam_softmax_prep_kernel(const float* __restrict__ wc,
                                                                          float* __restrict__ ws,
                                                                          unsigned* __restrict__ anchor_counter) {
  constexpr float kLog2e = 1.4426950408889634f;
  static_assert(kGatherThreads % G == 0, "thread t only sees group t % G");
  __shared__ float s_tmp[kGatherWarps * 32];
  __shared__ float s_m[32];
  const int b = blockIdx.x, tid = threadIdx.x;
  if (b == 0 && tid < 2) anchor_counter[tid] = 0u;
  const float* w = wc + (int64_t)b * NC * LPG;
  float* ec = ws + (int64_t)b * (NC + 1) * LPG;
  float m = -INFINITY;
  for (int e = tid; e < NC * LPG; e += kGatherThreads) m = fmaxf(m, w[e]);
  group_reduce<true>(m, G, s_tmp, s_m);
  const float mg = s_m[tid % G] * kLog2e;
  for (int j = tid; j < LPG; j += kGatherThreads) {
    float s = 0.0f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const float e = ex2_approx(fmaf(w[c * LPG + j], kLog2e, -mg));
      ec[c * LPG + j] = e;
      s += e;
    }
    ec[NC * LPG + j] = s;
  }
}

// -----------------------------------------------------------------------------------------------
// One warp per anchor.  The per-anchor work is short (a few hundred instructions of softmax and
// candidate bookkeeping, then ~50 in-bounds samples of 4 taps), so the kernel is limited by
// latency unless many anchors are in flight per SM.  A warp per anchor needs no block barrier,
// keeps the per-anchor state in registers (plus LPG floats of shared memory for the anchor's
// softmax factors), and lets 40 anchors share an SM.
//
//   softmax   each lane owns the logits lane + 32k of the anchor row: always group lane % G.
//             MODE 1 (split logits + per-frame camera factors in the workspace): factorised,
//             LPG exps per anchor (see cam_softmax_prep_kernel).  MODE 0 (full logits) and
//             MODE 2 (split logits, no workspace), and MODE 1 when its guard trips: exact
//             two-pass max / sum over the full Ncam*LPG logits, read from L1.
//   samples   the (camera, point) pairs whose (u, v) can touch a map ((u, v) in (-0.5, 1.5)) are
//             kept, each expanded to its NL levels across the lanes; the in-bounds ones are
//             broadcast by shuffle, one at a time, to the whole warp, which gathers the 4 taps
//             (lane l: channels 8l..8l+7) and accumulates with packed fp32x2 FMA.
//   output    normalised in registers (1 / sum of the lane's group) and stored by each lane.
// -----------------------------------------------------------------------------------------------
// One in-bounds sample of a warp's anchor, as the merging step shares it between lanes.
template <int G>
struct SampleRec {
  int4 pix;     // the 4 taps' feature rows (all in bounds; a tap outside the map has weight 0)
  float4 bw;    // their bilinear weights
  float sw[G];  // per group: unnormalised softmax weight (factorised mode), or the logit (exact mode)
};

// Resident one-warp blocks per SM the register allocator must allow (for bf16 maps): the kernel
// is bound by how many anchors are in flight.  Reading sample locations, 28 (72 registers)
// measured fastest (25 / 80 registers: 311 vs 231 us per 32-frame launch; 32 / 64 registers:
// 181 vs 178 us); computing them from the anchors, 32 (64 registers, the most one-warp blocks
// an SM holds) measured fastest (187 vs 191 us).
#ifndef S4D_GATHER_MIN_BLOCKS_BF16
#define S4D_GATHER_MIN_BLOCKS_BF16 28
#endif
#ifndef S4D_GATHER_KPS_MIN_BLOCKS_BF16
#define S4D_GATHER_KPS_MIN_BLOCKS_BF16 32
#endif
// Resident warps per SM the register allocator must allow, for a block of WARPS warps.
template <typename T, bool KPS, int WARPS>
constexpr int warp_kernel_min_blocks() {
  constexpr int warps =
      sizeof(T) == 2 ? (KPS ? S4D_GATHER_KPS_MIN_BLOCKS_BF16 : S4D_GATHER_MIN_BLOCKS_BF16) : 24;
  return warps / WARPS > 0 ? warps / WARPS : 1;
}

// Each warp of the block takes its own anchors (WARPS anchors in flight per block).  Launches of
// fewer anchors than warp slots use dfa_gather_coop_kernel instead (several warps per anchor).
template <typename T, int NC, int NL, int NP, int G, int MODE, int WARPS, bool KPS>
__global__ void __launch_bounds__(WARPS * 32, (warp_kernel_min_blocks<T, KPS, WARPS>()))
    dfa_gather_warp_kernel(GatherParams p) {
  constexpr int NLP = NL * NP;
  constexpr int LPG = NLP * G;
  constexpr int NW = NC * LPG;
  constexpr int NPAIR = NC * NP;
  constexpr int D = kChannels / G;
  constexpr float kLog2e = 1.4426950408889634f;
  static_assert(LPG % 32 == 0 && 32 % G == 0 && G >= 4 && (G & (G - 1)) == 0, "warp gather shape");
  __shared__ __align__(16) int4 s_lvl[NC * NL];  // (H, W, start, ok)
  __shared__ __align__(16) float4 s_win[NC];     // per camera: (u_lo, u_hi, v_lo, v_hi)
  __shared__ __align__(16) float s_ea[MODE == 1 ? WARPS * LPG : 1];
  __shared__ unsigned char s_surv[WARPS][32];
  // per sub-round: the block leaders' records at 0..nlead-1 (lane order), the other members'
  // after them; s_xm[k] = lane bits of leader k's other members
  __shared__ __align__(16) SampleRec<G> s_rec[WARPS][32];
  __shared__ uint32_t s_xm[WARPS][32];
  __shared__ __align__(16) float4 s_kpt[KPS ? WARPS : 1][KPS ? NP : 1];  // KPS: the anchor's keypoints
  __shared__ float s_kc[KPS ? WARPS : 1][KPS ? NP * 3 : 1];               // KPS: their scaled coordinates

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  griddep_wait();  // launched with programmatic serialisation: the kernels ahead of this one are done
  griddep_launch_dependents();
  for (int i = tid; i < NC * NL; i += WARPS * 32) {
    const int H = p.spatial_shape[2 * i], W = p.spatial_shape[2 * i + 1], st = p.scale_start[i];
    const bool ok = H > 0 && W > 0 && st >= 0 && (int64_t)st + (int64_t)H * W <= p.num_feat;
    const int c = i / NL;
    if (!ok && c >= p.cam_begin && c < p.cam_end && p.error_flag != nullptr && blockIdx.x == 0)
      atomicOr(p.error_flag, S4D_FLAG_BAD_LEVEL);
    s_lvl[i] = make_int4(H, W, st, ok ? 1 : 0);
    // A sample of level l has an in-bounds tap iff u in (-0.5 / W, 1 + 0.5 / W) (v likewise), so
    // the union over the camera's valid levels is the window of its narrowest level.  The
    // survivor test below uses it (1e-3 wider, a superset of the exact per-level test).
    if (i % NL == NL - 1) {
      int wmin = 0, hmin = 0;
      for (int l = 0; l < NL; ++l) {
        const int j = c * NL + l;
        const int Hl = p.spatial_shape[2 * j], Wl = p.spatial_shape[2 * j + 1], sl = p.scale_start[j];
        if (Hl > 0 && Wl > 0 && sl >= 0 && (int64_t)sl + (int64_t)Hl * Wl <= p.num_feat) {
          wmin = wmin == 0 || Wl < wmin ? Wl : wmin;
          hmin = hmin == 0 || Hl < hmin ? Hl : hmin;
        }
      }
      s_win[c] = wmin == 0 ? make_float4(1.0f, 0.0f, 1.0f, 0.0f)  // no valid level: empty window
                           : make_float4(-0.5f / wmin - 1e-3f, 1.0f + 0.5f / wmin + 1e-3f, -0.5f / hmin - 1e-3f,
                                         1.0f + 0.5f / hmin + 1e-3f);
    }
  }
  __syncthreads();  // the only block barrier: every thread reaches it before any warp leaves
  // Persistent warps: each takes anchors from the launch's counter until none is left, so the
  // level tables above are staged once per block and uneven anchors balance out.
  const int64_t total_anchors = (int64_t)p.bs * p.num_anchor;
  for (;;) {
  unsigned ticket = 0;
  if (lane == 0) ticket = atomicAdd(p.anchor_counter, 1u);
  ticket = __shfl_sync(0xffffffffu, ticket, 0);
  const int64_t anchor_lin = ticket;
  if (anchor_lin >= total_anchors) break;
  const int b = (int)p.div_anchor.div((uint32_t)anchor_lin);  // anchors < 2^31
  const int gch = lane / (D / 8);  // group of this lane's output channels

  const float* wrow = p.weights + anchor_lin * (MODE == 0 ? NW : LPG);
  const float* wcam = MODE == 0 ? nullptr : p.weights_cam + (int64_t)b * NW;
  const float* ec_tab = MODE == 1 ? p.cam_ws + (int64_t)b * (NC + 1) * LPG : nullptr;
  float* ea = s_ea + (MODE == 1 ? warp * LPG : 0);

  if (KPS) {  // the anchor's keypoints (kps_project's arithmetic)
    const float* a = p.kps_anchor + anchor_lin * p.kps_anchor_dim;
    const int nf = p.kps_num_fix, nlc = (NP - nf) * 3;
    const float* lg = p.kps_learnable + anchor_lin * nlc;
    // one scaled coordinate per lane, the learnable ones (a sigmoid each) first, so only the
    // first of the two passes has sigmoids
    for (int t = lane; t < NP * 3; t += 32) {
      const bool learn = t < nlc;
      const int u = learn ? t : t - nlc;
      const int pt = (learn ? nf : 0) + u / 3, ax = u - (u / 3) * 3;
      const float sc = expf(a[3 + ax]);
      s_kc[warp][3 * pt + ax] = learn ? __fmul_rn(__fsub_rn(kps_sigmoid_rn(lg[u]), 0.5f), sc)
                                      : __fmul_rn(p.kps_fix_scale[u], sc);
    }
    __syncwarp();
    if (lane < NP) {
      float px, py, pz;
      kps_place(a, s_kc[warp][3 * lane], s_kc[warp][3 * lane + 1], s_kc[warp][3 * lane + 2], px, py, pz);
      s_kpt[warp][lane] = make_float4(px, py, pz, 0.0f);
    }
    __syncwarp();
  }

  // ---- 1. softmax statistics of group lane % G ----------------------------------------------
  float m_l = -INFINITY, s_l = 0.0f;
  bool exact = MODE != 1;
  if (MODE == 1) {
    float x[LPG / 32];
#pragma unroll
    for (int k = 0; k < LPG / 32; ++k) x[k] = __ldg(wrow + lane + 32 * k);
#pragma unroll
    for (int k = 0; k < LPG / 32; ++k) m_l = fmaxf(m_l, x[k]);
#pragma unroll
    for (int o = G; o < 32; o <<= 1) m_l = fmaxf(m_l, __shfl_xor_sync(0xffffffffu, m_l, o));
    const float ml = m_l * kLog2e;
#pragma unroll
    for (int k = 0; k < LPG / 32; ++k) {
      const float e = ex2_approx(fmaf(x[k], kLog2e, -ml));
      ea[lane + 32 * k] = e;
      s_l = fmaf(e, __ldg(ec_tab + NW + lane + 32 * k), s_l);
    }
#pragma unroll
    for (int o = G; o < 32; o <<= 1) s_l += __shfl_xor_sync(0xffffffffu, s_l, o);
    exact = __any_sync(0xffffffffu, !(s_l >= 1e-20f));
    __syncwarp();
  }
  if (exact) {
    auto logit = [&](int e) { return MODE == 0 ? __ldg(wrow + e) : __ldg(wrow + e % LPG) + __ldg(wcam + e); };
    m_l = -INFINITY;
    for (int e = lane; e < NW; e += 32) m_l = fmaxf(m_l, logit(e));
#pragma unroll
    for (int o = G; o < 32; o <<= 1) m_l = fmaxf(m_l, __shfl_xor_sync(0xffffffffu, m_l, o));
    const float ml = m_l * kLog2e;
    s_l = 0.0f;
    for (int e = lane; e < NW; e += 32) s_l += ex2_approx(fmaf(logit(e), kLog2e, -ml));
#pragma unroll
    for (int o = G; o < 32; o <<= 1) s_l += __shfl_xor_sync(0xffffffffu, s_l, o);
  }
  // lanes 0..G-1 hold the statistics of groups 0..G-1
  const float inv = __shfl_sync(0xffffffffu, 1.0f / s_l, gch);
  const float mlg = __shfl_sync(0xffffffffu, m_l, gch) * kLog2e;

  // ---- 2. candidates and weighted gather -----------------------------------------------------
  const float2* locp = reinterpret_cast<const float2*>(p.loc) + anchor_lin * NPAIR;
  const T* fb = static_cast<const T*>(p.feat) + (int64_t)b * p.num_feat * kChannels;
  const uint32_t lt = (1u << lane) - 1u;
  float2 acc[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] = make_float2(0.f, 0.f);
  using V = typename TapVec<T>::type;

#pragma unroll 1
  for (int base = 0; base < NPAIR; base += 32) {
    const int q = base + lane;
    const int cq = q / NP;
    float2 uv = make_float2(-4.0f, -4.0f);
    bool maybe = false;
    if (q < NPAIR) {
      if (KPS) {  // project keypoint q % NP into camera cq
        const float4 kp = s_kpt[warp][q - cq * NP];
        const float4* P = reinterpret_cast<const float4*>(p.kps_proj) + ((int64_t)b * NC + cq) * 4;
        const float2 wh = __ldg(reinterpret_cast<const float2*>(p.kps_wh) + (int64_t)b * NC + cq);
        bool front;
        kps_uv(__ldg(P), __ldg(P + 1), __ldg(P + 2), wh.x, wh.y, kp.x, kp.y, kp.z, uv.x, uv.y, front);
      } else {
        uv = __ldg(locp + q);
      }
      const float4 wn = s_win[cq];
      maybe = cq >= p.cam_begin && cq < p.cam_end && uv.x > wn.x && uv.x < wn.y && uv.y > wn.z && uv.y < wn.w;
    }
    const uint32_t keep = __ballot_sync(0xffffffffu, maybe);
    if (keep == 0u) continue;
    if (maybe) s_surv[warp][__popc(keep & lt)] = (unsigned char)lane;
    __syncwarp();
    // Candidates (survivor, level), level-major so that one camera's points at one level sit in
    // the same 32-lane sub-round: samples whose 2x2 tap block coincides are merged there.
    const int nsurv = __popc(keep);
    const int n = nsurv * NL;
    // idx / nsurv for idx < 4 * 32 as (idx * ceil(2^16 / nsurv)) >> 16 (exact for nsurv <= 32)
    const uint32_t inv_surv = (65536u + nsurv - 1) / (uint32_t)nsurv;
#pragma unroll 1
    for (int sub = 0; sub < n; sub += 32) {
      const int idx = sub + lane;
      const int l = (int)(((uint32_t)idx * inv_surv) >> 16), k = idx - l * nsurv;
      const int src = idx < n ? s_surv[warp][k] : 0;
      const float2 uvs = make_float2(__shfl_sync(0xffffffffu, uv.x, src), __shfl_sync(0xffffffffu, uv.y, src));
      const int qs = base + src;
      const int cs = qs / NP, ps = qs - (qs / NP) * NP;
      uint64_t key = 0xffffffff00000000ull | (uint32_t)lane;  // invalid lanes only match themselves
      bool valid = false;
      SampleRec<G> rec;
      if (idx < n) {
        const int4 lv = s_lvl[cs * NL + l];
        const float Wf = (float)lv.y, Hf = (float)lv.x;
        const float ix = ((uvs.x * 2.0f - 1.0f + 1.0f) * Wf - 1.0f) * 0.5f;
        const float iy = ((uvs.y * 2.0f - 1.0f + 1.0f) * Hf - 1.0f) * 0.5f;
        if (lv.w && ix > -1.0f && ix < Wf && iy > -1.0f && iy < Hf) {
          const float x0f = floorf(ix), y0f = floorf(iy);
          const int x0 = (int)x0f, y0 = (int)y0f;
          const float x1f = x0f + 1.0f, y1f = y0f + 1.0f;
          const bool vx0 = x0 >= 0, vx1 = x0 + 1 < lv.y, vy0 = y0 >= 0, vy1 = y0 + 1 < lv.x;
          const int p00 = lv.z + y0 * lv.y + x0;
          // A tap outside the map is given the row of an in-bounds tap of the same block (a valid
          // sample has one) and weight 0, so the gather loop loads and accumulates all 4 taps
          // without tests; the extra load hits L1.
          const bool t00 = vx0 && vy0, t01 = vx1 && vy0, t10 = vx0 && vy1, t11 = vx1 && vy1;
          const int any = t00 ? p00 : t01 ? p00 + 1 : t10 ? p00 + lv.y : p00 + lv.y + 1;
          rec.pix = make_int4(t00 ? p00 : any, t01 ? p00 + 1 : any, t10 ? p00 + lv.y : any, t11 ? p00 + lv.y + 1 : any);
          rec.bw = make_float4(t00 ? (x1f - ix) * (y1f - iy) : 0.0f, t01 ? (ix - x0f) * (y1f - iy) : 0.0f,
                               t10 ? (x1f - ix) * (iy - y0f) : 0.0f, t11 ? (ix - x0f) * (iy - y0f) : 0.0f);
          const int lp = l * NP + ps;
          const int e1 = lp * G, e2 = cs * LPG + lp * G;  // anchor-term and camera-term offsets
          // This sample's weight for every group, computed once here rather than by every lane of
          // every block it joins: exp(wa - M1) * exp(wc - M2) from the per-anchor table and the
          // per-frame camera factors, or (exact mode) the logit itself.
          if (!exact && G % 4 == 0) {  // e1, e2 are multiples of G: 16-byte vectors
#pragma unroll
            for (int g = 0; g < G; g += 4) {
              const float4 a = *reinterpret_cast<const float4*>(ea + e1 + g);
              const float4 c = __ldg(reinterpret_cast<const float4*>(ec_tab + e2 + g));
              rec.sw[g] = a.x * c.x, rec.sw[g + 1] = a.y * c.y, rec.sw[g + 2] = a.z * c.z, rec.sw[g + 3] = a.w * c.w;
            }
          } else {
#pragma unroll
            for (int g = 0; g < G; ++g) {
              if (!exact) {
                rec.sw[g] = ea[e1 + g] * __ldg(ec_tab + e2 + g);
              } else {
                rec.sw[g] = MODE == 0 ? __ldg(wrow + e2 + g) : __ldg(wrow + e1 + g) + __ldg(wcam + e2 + g);
              }
            }
          }
          // (camera, level) and the top-left tap (x0, y0 >= -1) identify the 2x2 block
          key = ((uint64_t)(cs * NL + l) << 32) | (uint32_t)((y0 + 1) * (lv.y + 1) + (x0 + 1));
          valid = true;
        }
      }
      const uint32_t grp = __match_any_sync(0xffffffffu, key);
      const bool lead = valid && lane == __ffs(grp) - 1;
      const uint32_t leaders = __ballot_sync(0xffffffffu, lead);
      const uint32_t extras = __ballot_sync(0xffffffffu, valid && !lead);
      const int nlead = __popc(leaders);
      __syncwarp();  // the previous sub-round's records have been read
      if (valid) {
        const int slot = lead ? __popc(leaders & lt) : nlead + __popc(extras & lt);
        s_rec[warp][slot] = rec;
        if (lead) s_xm[warp][slot] = grp & ~(1u << lane);
      }
      __syncwarp();
      // the tap loop, instantiated for the two softmax modes (exact is fixed per anchor)
      auto tap_loop = [&](auto ex) {
        constexpr bool EX = decltype(ex)::value;
        // unrolled so that the next blocks' loads are scheduled among this block's FMAs (4 fits
        // the 64 registers of the variant that computes its sample locations without spilling)
        constexpr int kTapUnroll = KPS ? 4 : 2;
#pragma unroll kTapUnroll
        for (int k = 0; k < nlead; ++k) {
          const int4 px = s_rec[warp][k].pix;
          V v0, v1, v2, v3;  // every tap row is in bounds (see the record): no tests
          TapFma<T>::load(fb, px.x, lane, v0);
          TapFma<T>::load(fb, px.y, lane, v1);
          TapFma<T>::load(fb, px.z, lane, v2);
          TapFma<T>::load(fb, px.w, lane, v3);
          if (k + 1 < nlead) {  // the next block's rows towards L1 (no registers held)
            const int4 pn = s_rec[warp][k + 1].pix;
            const T* r = fb + lane * (kChannels / 32);
            prefetch_l1(r + (int64_t)pn.x * kChannels);
            prefetch_l1(r + (int64_t)pn.y * kChannels);
            prefetch_l1(r + (int64_t)pn.z * kChannels);
            prefetch_l1(r + (int64_t)pn.w * kChannels);
          }
          // the block's weight for this lane's group: sum over its member samples (the leader's
          // first, then the others in lane order) of bilinear weight x unnormalised softmax weight
          const float4 bw = s_rec[warp][k].bw;
          float sw = s_rec[warp][k].sw[gch];
          if (EX) sw = ex2_approx(fmaf(sw, kLog2e, -mlg));
          float4 w4 = make_float4(bw.x * sw, bw.y * sw, bw.z * sw, bw.w * sw);
          uint32_t xm = s_xm[warp][k];
          while (xm != 0u) {  // warp-uniform: most blocks have a single sample
            const int j = __ffs(xm) - 1;
            xm &= xm - 1u;
            const int e = nlead + __popc(extras & ((1u << j) - 1u));
            const float4 bwe = s_rec[warp][e].bw;
            float swe = s_rec[warp][e].sw[gch];
            if (EX) swe = ex2_approx(fmaf(swe, kLog2e, -mlg));
            w4.x = fmaf(bwe.x, swe, w4.x);
            w4.y = fmaf(bwe.y, swe, w4.y);
            w4.z = fmaf(bwe.z, swe, w4.z);
            w4.w = fmaf(bwe.w, swe, w4.w);
          }
          TapFma<T>::fma(v0, w4.x, acc);
          TapFma<T>::fma(v1, w4.y, acc);
          TapFma<T>::fma(v2, w4.z, acc);
          TapFma<T>::fma(v3, w4.w, acc);
        }
      };
      if (exact)
        tap_loop(std::true_type{});
      else
        tap_loop(std::false_type{});
    }
    __syncwarp();  // s_surv is rewritten by the next pair round
  }

  // ---- 3. normalise and store ------------------------------------------------------------------
  float* dst = anchor_lin >= p.peer_row_begin && anchor_lin < p.peer_row_end ? p.out_peer : p.out;
  float4* o = reinterpret_cast<float4*>(dst + anchor_lin * kChannels + lane * 8);
  o[0] = make_float4(acc[0].x * inv, acc[0].y * inv, acc[1].x * inv, acc[1].y * inv);
  o[1] = make_float4(acc[2].x * inv, acc[2].y * inv, acc[3].x * inv, acc[3].y * inv);
  __syncwarp();  // this anchor's shared-memory state is read before the next one writes it
  }
  if (p.out_peer != nullptr) __threadfence_system();  // the rows stored to the other GPU are performed
  if (WARPS == 1) {
    if (lane == 0) release_anchor_counter(p.anchor_counter);
  } else {
    __syncthreads();  // every warp of the block has taken its last ticket
    if (tid == 0) release_anchor_counter(p.anchor_counter);
  }
}

// -----------------------------------------------------------------------------------------------
// Few anchors (fewer than the resident warp slots, e.g. a single frame): a block of WARPS warps
// per anchor, the anchor's work divided between the warps instead of repeated by each of them.
//   phase 1  warp 0: the softmax statistics (factorised, or the exact fallback) and the anchor's
//            exp table; warp 1: the anchor's keypoints (KPS); the remaining warps (warp 1 as
//            well when WARPS is 2) stage the frame's camera factors, and (KPS) its projection
//            matrices and image sizes, in shared memory.
//   phase 2  the (camera, point) pairs in chunks of CHUNK (<= 32), chunk c to warp c % WARPS:
//            projection (or the stored location), survivor test and the records of the chunk's
//            (survivor, level) candidates with coinciding 2x2 tap blocks merged, 32 candidates
//            per round; after each round every warp gathers every WARPS-th merged block of each
//            warp's records.
//   phase 3  warp 0 adds the WARPS partial sums in warp order, normalises and stores.
// Block barriers (all in uniform control flow): 3 per anchor plus 2 per round after the first.  Every sample's location,
// bilinear weights and softmax weight come from the same arithmetic as in
// dfa_gather_warp_kernel; only the grouping of samples into merged blocks and the order of the
// final sum differ (the result is deterministic).
// -----------------------------------------------------------------------------------------------
template <typename T, int NC, int NL, int NP, int G, int WARPS, bool KPS>
__global__ void __launch_bounds__(WARPS * 32, (sizeof(T) == 2 ? 28 : 20) / WARPS)
    dfa_gather_coop_kernel(GatherParams p) {
  constexpr int NLP = NL * NP;
  constexpr int LPG = NLP * G;
  constexpr int NW = NC * LPG;
  constexpr int NPAIR = NC * NP;
  constexpr int D = kChannels / G;
  constexpr int CHUNK = (NPAIR + WARPS - 1) / WARPS < 32 ? (NPAIR + WARPS - 1) / WARPS : 32;
  constexpr int NCHUNK = (NPAIR + CHUNK - 1) / CHUNK;
  constexpr int STAGER0 = WARPS > 2 ? 2 : 1;  // first warp that stages the frame's tables
  constexpr float kLog2e = 1.4426950408889634f;
  static_assert(WARPS >= 2 && WARPS <= 8, "coop gather: 2 to 8 warps per anchor");
  static_assert(LPG % 32 == 0 && 32 % G == 0 && G >= 4 && (G & (G - 1)) == 0 && NW % 4 == 0, "coop gather shape");
  __shared__ __align__(16) int4 s_lvl[NC * NL];  // (H, W, start, ok)
  __shared__ __align__(16) float4 s_win[NC];     // per camera: (u_lo, u_hi, v_lo, v_hi)
  __shared__ __align__(16) float s_ea[LPG];      // the anchor's exp(wa - M1) per (level, point, group)
  __shared__ __align__(16) float s_ec[NW];       // the frame's camera factors exp(wc - M2)
  __shared__ __align__(16) float4 s_proj[KPS ? NC * 3 : 1];  // KPS: rows 0..2 of each camera's matrix
  __shared__ __align__(16) float2 s_wh[KPS ? NC : 1];
  __shared__ __align__(16) float4 s_kpt[KPS ? NP : 1];
  __shared__ float s_kc[KPS ? NP * 3 : 1];
  __shared__ float s_stat[2][G];  // per group: max x log2(e) (exact mode) and 1 / sum
  __shared__ int s_exact;
  __shared__ unsigned char s_surv[WARPS][32];
  __shared__ __align__(16) SampleRec<G> s_rec[WARPS][32];
  __shared__ uint32_t s_xm[WARPS][32];
  __shared__ __align__(16) float4 s_part[WARPS][64];
  __shared__ int s_nlead[WARPS];       // per round: the warp's merged blocks,
  __shared__ uint32_t s_extras[WARPS];  // the lanes of their other member samples,
  __shared__ int s_more[WARPS];         // whether the warp has candidates left
  __shared__ unsigned s_ticket;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  griddep_wait();  // launched with programmatic serialisation: the kernels ahead of this one are done
  griddep_launch_dependents();
  for (int i = tid; i < NC * NL; i += WARPS * 32) {
    const int H = p.spatial_shape[2 * i], W = p.spatial_shape[2 * i + 1], st = p.scale_start[i];
    const bool ok = H > 0 && W > 0 && st >= 0 && (int64_t)st + (int64_t)H * W <= p.num_feat;
    const int c = i / NL;
    if (!ok && c >= p.cam_begin && c < p.cam_end && p.error_flag != nullptr && blockIdx.x == 0)
      atomicOr(p.error_flag, S4D_FLAG_BAD_LEVEL);
    s_lvl[i] = make_int4(H, W, st, ok ? 1 : 0);
    if (i % NL == NL - 1) {  // the camera's survivor window: that of its narrowest valid level
      int wmin = 0, hmin = 0;
      for (int l = 0; l < NL; ++l) {
        const int j = c * NL + l;
        const int Hl = p.spatial_shape[2 * j], Wl = p.spatial_shape[2 * j + 1], sl = p.scale_start[j];
        if (Hl > 0 && Wl > 0 && sl >= 0 && (int64_t)sl + (int64_t)Hl * Wl <= p.num_feat) {
          wmin = wmin == 0 || Wl < wmin ? Wl : wmin;
          hmin = hmin == 0 || Hl < hmin ? Hl : hmin;
        }
      }
      s_win[c] = wmin == 0 ? make_float4(1.0f, 0.0f, 1.0f, 0.0f)
                           : make_float4(-0.5f / wmin - 1e-3f, 1.0f + 0.5f / wmin + 1e-3f, -0.5f / hmin - 1e-3f,
                                         1.0f + 0.5f / hmin + 1e-3f);
    }
  }
  const int64_t total_anchors = (int64_t)p.bs * p.num_anchor;
  const int gch = lane / (D / 8);  // group of this lane's output channels
  const uint32_t lt = (1u << lane) - 1u;
  using V = typename TapVec<T>::type;
  for (;;) {
    if (tid == 0) s_ticket = atomicAdd(p.anchor_counter, 1u);
    // (A) the ticket and the level tables are visible; the previous anchor is finished
    __syncthreads();
    const int64_t anchor_lin = s_ticket;
    if (anchor_lin >= total_anchors) break;  // block-uniform
    const int b = (int)p.div_anchor.div((uint32_t)anchor_lin);
    const float* wrow = p.weights + anchor_lin * LPG;
    const float* wcam = p.weights_cam + (int64_t)b * NW;
    const float* ec_tab = p.cam_ws + (int64_t)b * (NC + 1) * LPG;

    // ---- phase 1 ------------------------------------------------------------------------------
    if (warp == 0) {  // softmax statistics of group lane % G, the warp kernel's arithmetic
      float x[LPG / 32];
#pragma unroll
      for (int k = 0; k < LPG / 32; ++k) x[k] = __ldg(wrow + lane + 32 * k);
      float m_l = -INFINITY, s_l = 0.0f;
#pragma unroll
      for (int k = 0; k < LPG / 32; ++k) m_l = fmaxf(m_l, x[k]);
#pragma unroll
      for (int o = G; o < 32; o <<= 1) m_l = fmaxf(m_l, __shfl_xor_sync(0xffffffffu, m_l, o));
      const float ml = m_l * kLog2e;
#pragma unroll
      for (int k = 0; k < LPG / 32; ++k) {
        const float e = ex2_approx(fmaf(x[k], kLog2e, -ml));
        s_ea[lane + 32 * k] = e;
        s_l = fmaf(e, __ldg(ec_tab + NW + lane + 32 * k), s_l);
      }
#pragma unroll
      for (int o = G; o < 32; o <<= 1) s_l += __shfl_xor_sync(0xffffffffu, s_l, o);
      const bool exact = __any_sync(0xffffffffu, !(s_l >= 1e-20f));
      if (exact) {  // the factorised sum underflowed: exact two-pass max / sum over all logits
        auto logit = [&](int e) { return __ldg(wrow + e % LPG) + __ldg(wcam + e); };
        m_l = -INFINITY;
        for (int e = lane; e < NW; e += 32) m_l = fmaxf(m_l, logit(e));
#pragma unroll
        for (int o = G; o < 32; o <<= 1) m_l = fmaxf(m_l, __shfl_xor_sync(0xffffffffu, m_l, o));
        const float ml2 = m_l * kLog2e;
        s_l = 0.0f;
        for (int e = lane; e < NW; e += 32) s_l += ex2_approx(fmaf(logit(e), kLog2e, -ml2));
#pragma unroll
        for (int o = G; o < 32; o <<= 1) s_l += __shfl_xor_sync(0xffffffffu, s_l, o);
      }
      if (lane < G) {
        s_stat[0][lane] = m_l * kLog2e;
        s_stat[1][lane] = 1.0f / s_l;
      }
      if (lane == 0) s_exact = exact ? 1 : 0;
    } else if (KPS && warp == 1) {  // the anchor's keypoints (kps_project's arithmetic)
      const float* a = p.kps_anchor + anchor_lin * p.kps_anchor_dim;
      const int nf = p.kps_num_fix, nlc = (NP - nf) * 3;
      const float* lg = p.kps_learnable + anchor_lin * nlc;
      for (int t = lane; t < NP * 3; t += 32) {
        const bool learn = t < nlc;
        const int u = learn ? t : t - nlc;
        const int pt = (learn ? nf : 0) + u / 3, ax = u - (u / 3) * 3;
        const float sc = expf(a[3 + ax]);
        s_kc[3 * pt + ax] = learn ? __fmul_rn(__fsub_rn(kps_sigmoid_rn(lg[u]), 0.5f), sc)
                                  : __fmul_rn(p.kps_fix_scale[u], sc);
      }
      __syncwarp();
      if (lane < NP) {
        float px, py, pz;
        kps_place(a, s_kc[3 * lane], s_kc[3 * lane + 1], s_kc[3 * lane + 2], px, py, pz);
        s_kpt[lane] = make_float4(px, py, pz, 0.0f);
      }
    }
    if (warp >= STAGER0) {  // the frame's tables
      const int t0 = tid - STAGER0 * 32, nt = (WARPS - STAGER0) * 32;
      const float4* ec4 = reinterpret_cast<const float4*>(ec_tab);
      for (int i = t0; i < NW / 4; i += nt) reinterpret_cast<float4*>(s_ec)[i] = __ldg(ec4 + i);
      if (KPS) {
        for (int i = t0; i < NC * 3; i += nt)
          s_proj[i] = __ldg(reinterpret_cast<const float4*>(p.kps_proj) + ((int64_t)b * NC + i / 3) * 4 + i % 3);
        for (int i = t0; i < NC; i += nt)
          s_wh[i] = __ldg(reinterpret_cast<const float2*>(p.kps_wh) + (int64_t)b * NC + i);
      }
    }
    __syncthreads();  // (B) phase 1's tables are visible

    // ---- phase 2 ------------------------------------------------------------------------------
    // Rounds: every warp builds the records of its next sub-round (up to 32 candidates of its
    // current chunk), then all warps gather the merged blocks of every warp's sub-round, warp w
    // taking every WARPS-th block of each, so the tap work is shared out evenly whichever cameras
    // see the anchor.
    const bool exact = s_exact != 0;
    const float inv = s_stat[1][gch];
    const float mlg = s_stat[0][gch];
    const float2* locp = reinterpret_cast<const float2*>(p.loc) + anchor_lin * NPAIR;
    const T* fb = static_cast<const T*>(p.feat) + (int64_t)b * p.num_feat * kChannels;
    float2 acc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] = make_float2(0.f, 0.f);

    // this warp's candidate stream over its chunks (warp-uniform state)
    int chunk = warp - WARPS, base = 0, sub = 0, n = 0, nsurv = 1;
    uint32_t inv_surv = 1;
    float2 uv = make_float2(-4.0f, -4.0f);
    auto next_chunk = [&]() -> bool {  // the warp's next chunk with survivors, if any
      for (chunk += WARPS; chunk < NCHUNK; chunk += WARPS) {
        base = chunk * CHUNK;
        const int q = base + lane;
        const int cq = q / NP;
        uv = make_float2(-4.0f, -4.0f);
        bool maybe = false;
        if (lane < CHUNK && q < NPAIR) {
          if (KPS) {  // project keypoint q % NP into camera cq
            const float4 kp = s_kpt[q - cq * NP];
            const float2 wh = s_wh[cq];
            bool front;
            kps_uv(s_proj[3 * cq], s_proj[3 * cq + 1], s_proj[3 * cq + 2], wh.x, wh.y, kp.x, kp.y, kp.z, uv.x,
                   uv.y, front);
          } else {
            uv = __ldg(locp + q);
          }
          const float4 wn = s_win[cq];
          maybe = cq >= p.cam_begin && cq < p.cam_end && uv.x > wn.x && uv.x < wn.y && uv.y > wn.z && uv.y < wn.w;
        }
        const uint32_t keep = __ballot_sync(0xffffffffu, maybe);
        if (keep == 0u) continue;  // warp-uniform
        __syncwarp();              // the previous chunk's survivor list has been read
        if (maybe) s_surv[warp][__popc(keep & lt)] = (unsigned char)lane;
        __syncwarp();
        nsurv = __popc(keep);
        n = nsurv * NL;  // candidates (survivor, level), level-major, as in the warp kernel
        inv_surv = (65536u + nsurv - 1) / (uint32_t)nsurv;
        sub = 0;
        return true;
      }
      return false;
    };
    bool have = next_chunk();
#pragma unroll 1
    for (;;) {
      int my_nlead = 0;
      uint32_t my_extras = 0u;
      if (have) {  // the records of candidates sub .. sub + 31 of the current chunk
        const int idx = sub + lane;
        const int l = (int)(((uint32_t)idx * inv_surv) >> 16), k = idx - l * nsurv;
        const int src = idx < n ? s_surv[warp][k] : 0;
        const float2 uvs = make_float2(__shfl_sync(0xffffffffu, uv.x, src), __shfl_sync(0xffffffffu, uv.y, src));
        const int qs = base + src;
        const int cs = qs / NP, ps = qs - (qs / NP) * NP;
        uint64_t key = 0xffffffff00000000ull | (uint32_t)lane;  // invalid lanes only match themselves
        bool valid = false;
        SampleRec<G> rec;
        if (idx < n) {
          const int4 lv = s_lvl[cs * NL + l];
          const float Wf = (float)lv.y, Hf = (float)lv.x;
          const float ix = ((uvs.x * 2.0f - 1.0f + 1.0f) * Wf - 1.0f) * 0.5f;
          const float iy = ((uvs.y * 2.0f - 1.0f + 1.0f) * Hf - 1.0f) * 0.5f;
          if (lv.w && ix > -1.0f && ix < Wf && iy > -1.0f && iy < Hf) {
            const float x0f = floorf(ix), y0f = floorf(iy);
            const int x0 = (int)x0f, y0 = (int)y0f;
            const float x1f = x0f + 1.0f, y1f = y0f + 1.0f;
            const bool vx0 = x0 >= 0, vx1 = x0 + 1 < lv.y, vy0 = y0 >= 0, vy1 = y0 + 1 < lv.x;
            const int p00 = lv.z + y0 * lv.y + x0;
            const bool t00 = vx0 && vy0, t01 = vx1 && vy0, t10 = vx0 && vy1, t11 = vx1 && vy1;
            const int any = t00 ? p00 : t01 ? p00 + 1 : t10 ? p00 + lv.y : p00 + lv.y + 1;
            rec.pix = make_int4(t00 ? p00 : any, t01 ? p00 + 1 : any, t10 ? p00 + lv.y : any,
                                t11 ? p00 + lv.y + 1 : any);
            rec.bw = make_float4(t00 ? (x1f - ix) * (y1f - iy) : 0.0f, t01 ? (ix - x0f) * (y1f - iy) : 0.0f,
                                 t10 ? (x1f - ix) * (iy - y0f) : 0.0f, t11 ? (ix - x0f) * (iy - y0f) : 0.0f);
            const int lp = l * NP + ps;
            const int e1 = lp * G, e2 = cs * LPG + lp * G;
            if (!exact && G % 4 == 0) {
#pragma unroll
              for (int g = 0; g < G; g += 4) {
                const float4 a = *reinterpret_cast<const float4*>(s_ea + e1 + g);
                const float4 c = *reinterpret_cast<const float4*>(s_ec + e2 + g);
                rec.sw[g] = a.x * c.x, rec.sw[g + 1] = a.y * c.y, rec.sw[g + 2] = a.z * c.z, rec.sw[g + 3] = a.w * c.w;
              }
            } else {
#pragma unroll
              for (int g = 0; g < G; ++g)
                rec.sw[g] = exact ? __ldg(wrow + e1 + g) + __ldg(wcam + e2 + g) : s_ea[e1 + g] * s_ec[e2 + g];
            }
            key = ((uint64_t)(cs * NL + l) << 32) | (uint32_t)((y0 + 1) * (lv.y + 1) + (x0 + 1));
            valid = true;
          }
        }
        const uint32_t grp = __match_any_sync(0xffffffffu, key);
        const bool lead = valid && lane == __ffs(grp) - 1;
        const uint32_t leaders = __ballot_sync(0xffffffffu, lead);
        my_extras = __ballot_sync(0xffffffffu, valid && !lead);
        my_nlead = __popc(leaders);
        if (valid) {
          const int slot = lead ? __popc(leaders & lt) : my_nlead + __popc(my_extras & lt);
          s_rec[warp][slot] = rec;
          if (lead) s_xm[warp][slot] = grp & ~(1u << lane);
        }
        sub += 32;
        if (sub >= n) have = next_chunk();
      }
      if (lane == 0) {
        s_nlead[warp] = my_nlead;
        s_extras[warp] = my_extras;
        s_more[warp] = have ? 1 : 0;
      }
      __syncthreads();  // (R) every warp's records of this round are visible
      int more = 0;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) more |= s_more[w];
      auto tap_loop = [&](auto ex) {
        constexpr bool EX = decltype(ex)::value;
        constexpr int kTapUnroll = KPS ? 4 : 2;
#pragma unroll 1
        for (int w = 0; w < WARPS; ++w) {
          const int nlead = s_nlead[w];
          const uint32_t extras = s_extras[w];
#pragma unroll kTapUnroll
          for (int k = warp; k < nlead; k += WARPS) {
            const int4 px = s_rec[w][k].pix;
            V v0, v1, v2, v3;  // every tap row is in bounds (see the record): no tests
            TapFma<T>::load(fb, px.x, lane, v0);
            TapFma<T>::load(fb, px.y, lane, v1);
            TapFma<T>::load(fb, px.z, lane, v2);
            TapFma<T>::load(fb, px.w, lane, v3);
            if (k + WARPS < nlead) {  // this warp's next block of the same records towards L1
              const int4 pn = s_rec[w][k + WARPS].pix;
              const T* r = fb + lane * (kChannels / 32);
              prefetch_l1(r + (int64_t)pn.x * kChannels);
              prefetch_l1(r + (int64_t)pn.y * kChannels);
              prefetch_l1(r + (int64_t)pn.z * kChannels);
              prefetch_l1(r + (int64_t)pn.w * kChannels);
            }
            const float4 bw = s_rec[w][k].bw;
            float sw = s_rec[w][k].sw[gch];
            if (EX) sw = ex2_approx(fmaf(sw, kLog2e, -mlg));
            float4 w4 = make_float4(bw.x * sw, bw.y * sw, bw.z * sw, bw.w * sw);
            uint32_t xm = s_xm[w][k];
            while (xm != 0u) {  // warp-uniform: most blocks have a single sample
              const int j = __ffs(xm) - 1;
              xm &= xm - 1u;
              const int e = nlead + __popc(extras & ((1u << j) - 1u));
              const float4 bwe = s_rec[w][e].bw;
              float swe = s_rec[w][e].sw[gch];
              if (EX) swe = ex2_approx(fmaf(swe, kLog2e, -mlg));
              w4.x = fmaf(bwe.x, swe, w4.x);
              w4.y = fmaf(bwe.y, swe, w4.y);
              w4.z = fmaf(bwe.z, swe, w4.z);
              w4.w = fmaf(bwe.w, swe, w4.w);
            }
            TapFma<T>::fma(v0, w4.x, acc);
            TapFma<T>::fma(v1, w4.y, acc);
            TapFma<T>::fma(v2, w4.z, acc);
            TapFma<T>::fma(v3, w4.w, acc);
          }
        }
      };
      if (exact)
        tap_loop(std::true_type{});
      else
        tap_loop(std::false_type{});
      if (!more) break;  // block-uniform
      __syncthreads();   // this round's records are read before the next round writes its own
    }

    // ---- phase 3 ------------------------------------------------------------------------------
    s_part[warp][2 * lane] = make_float4(acc[0].x, acc[0].y, acc[1].x, acc[1].y);
    s_part[warp][2 * lane + 1] = make_float4(acc[2].x, acc[2].y, acc[3].x, acc[3].y);
    __syncthreads();  // (C) every warp's partial sum is in shared memory
    if (warp == 0) {
      float4 a0 = s_part[0][2 * lane], a1 = s_part[0][2 * lane + 1];
#pragma unroll
      for (int w = 1; w < WARPS; ++w) {
        const float4 b0 = s_part[w][2 * lane], b1 = s_part[w][2 * lane + 1];
        a0 = make_float4(a0.x + b0.x, a0.y + b0.y, a0.z + b0.z, a0.w + b0.w);
        a1 = make_float4(a1.x + b1.x, a1.y + b1.y, a1.z + b1.z, a1.w + b1.w);
      }
      float* dst = anchor_lin >= p.peer_row_begin && anchor_lin < p.peer_row_end ? p.out_peer : p.out;
      float4* o = reinterpret_cast<float4*>(dst + anchor_lin * kChannels + lane * 8);
      o[0] = make_float4(a0.x * inv, a0.y * inv, a0.z * inv, a0.w * inv);
      o[1] = make_float4(a1.x * inv, a1.y * inv, a1.z * inv, a1.w * inv);
    }
  }
  if (p.out_peer != nullptr) __threadfence_system();  // the rows stored to the other GPU are performed
  if (tid == 0) release_anchor_counter(p.anchor_counter);
}


// The Sparse4D v3 shape the fast kernels are compiled for.
constexpr int kFastNC = 6, kFastNL = 4, kFastNP = 13, kFastG = 8;
// anchors (warps) per block of dfa_gather_warp_kernel: small blocks retire as soon as their own
// anchors are done, so uneven anchors do not leave finished warps waiting for block-mates
constexpr int kWarpBlock = 1;

// Workspace: the per-frame camera factors, then (16-byte aligned) the anchor counter of the
// persistent warp kernel.
static size_t factor_bytes(int64_t bs, int ncam, int nl, int np, int G) {
  return ((size_t)bs * (ncam + 1) * nl * np * G * sizeof(float) + 15) & ~(size_t)15;
}

size_t gather_workspace_bytes(int64_t bs, int ncam, int nl, int np, int G) {
  return factor_bytes(bs, ncam, nl, np, G) + 16;
}

// One-warp blocks of the warp kernel that fit on the current device at once, cached per device
// and feature type (index `which`).
template <typename K>
static int resident_warp_blocks(K kernel, int which, int warps_per_block = kWarpBlock) {
  static int cache[16][64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148 * 28 / warps_per_block;
  if (cache[which][dev] > 0) return cache[which][dev];
  int per_sm = 0, sms = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, warps_per_block * 32, 0) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || per_sm <= 0 || sms <= 0) {
    cudaGetLastError();
    return 148 * 28 / warps_per_block;
  }
  cache[which][dev] = per_sm * sms;
  return cache[which][dev];
}

// Warps that share one anchor in the warp kernel for `anchors` anchors: the largest of 1, 2, 4, 8
// (at most S4D_GATHER_MAX_SPLIT) that keeps anchors x warps within S4D_GATHER_SPLIT_SLOTS warps
// per SM (28: the warp slots of the cooperative instances), so that a launch of few anchors still fills
// the SMs in one wave.  It depends only on the anchor count and the SM count, so every instance
// family (feature type, keypoints in the kernel or not) sums a given anchor in the same order.
#ifndef S4D_GATHER_SPLIT_SLOTS
#define S4D_GATHER_SPLIT_SLOTS 28
#endif
#ifndef S4D_GATHER_MAX_SPLIT
#define S4D_GATHER_MAX_SPLIT 8
#endif
int gather_split_warps(int64_t anchors) {
  static int sms_cache[64] = {};
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64) {
    if (sms_cache[dev] == 0 && cudaDeviceGetAttribute(&sms_cache[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      cudaGetLastError();
      sms_cache[dev] = 148;
    }
    sms = sms_cache[dev];
  }
  const int64_t slots = (int64_t)sms * S4D_GATHER_SPLIT_SLOTS;
  int s = 1;
  while (s < S4D_GATHER_MAX_SPLIT && s < 8 && anchors * (2 * s) <= slots) s *= 2;
  return s;
}

static bool fast_path_ok(const GatherParams& p) {
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  return p.layout == S4D_LAYOUT_CAM_MAJOR && p.logits && p.num_cams == kFastNC && p.num_levels == kFastNL &&
         p.num_pts == kFastNP && p.num_groups == kFastG && al16(p.weights) &&
         (p.weights_cam == nullptr || al16(p.weights_cam));
}

size_t gather_smem_bytes(int ncam, int nl, int np, int G, int cam_begin, int cam_end) {
  return gather_smem_layout(ncam, nl, np, G, cam_begin, cam_end).bytes;
}

int launch_cam_factors(const float* weights_cam, float* cam_ws, int bs, int ncam, int nl, int np, int G,
                       cudaStream_t stream) {
  if (ncam != kFastNC || nl != kFastNL || np != kFastNP || G != kFastG)
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "camera factors: implemented for 6 cameras, 4 levels, 13 points, 8 groups");
  if (bs <= 0) return S4D_OK;
  constexpr int LPG = kFastNL * kFastNP * kFastG;
  unsigned* counter = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(cam_ws) + factor_bytes(bs, ncam, nl, np, G));
  cam_softmax_prep_kernel<kFastNC, LPG, kFastG><<<(unsigned)bs, kGatherThreads, 0, stream>>>(weights_cam, cam_ws,
                                                                                           counter);
  return cuda_check(cudaGetLastError(), "cam_softmax_prep_kernel launch");
}

int launch_gather(const GatherParams& p, int feat_dtype, cudaStream_t stream) {
  const size_t smem = gather_smem_bytes(p.num_cams, p.num_levels, p.num_pts, p.num_groups, p.cam_begin, p.cam_end);
  const unsigned grid = (unsigned)((int64_t)p.bs * p.num_anchor);
  if (fast_path_ok(p) && p.weights_cam != nullptr && p.cam_ws != nullptr) {
    // split logits with a workspace: per-frame camera factors (unless already there), then one
    // warp per anchor
    if (!p.factors_ready) {
      int st = launch_cam_factors(p.weights_cam, p.cam_ws, p.bs, p.num_cams, p.num_levels, p.num_pts, p.num_groups,
                                  stream);
      if (st) return st;
    }
    GatherParams q = p;
    q.div_anchor = FastDiv((uint32_t)p.num_anchor);
    // the counter pair is zero: reset by cam_softmax_prep_kernel when the workspace was prepared,
    // and by the last block of every gather launch on it since
    q.anchor_counter = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(p.cam_ws) +
                                                   factor_bytes(p.bs, p.num_cams, p.num_levels, p.num_pts, p.num_groups));
    const int64_t anchors = (int64_t)p.bs * p.num_anchor;
    const bool bf = feat_dtype == S4D_DTYPE_BF16;
    const int which = (p.kps_anchor != nullptr ? 2 : 0) + (bf ? 0 : 1);  // index of the one-warp instance
    // The instances of one (feature type, KPS) pair: one-warp blocks (S = 1) and blocks of S warps
    // sharing an anchor (S = 2, 4, 8); `which` + 4 * log2(S) indexes the occupancy cache.
    auto launch_family = [&](auto k1, auto k2, auto k4, auto k8) {
      const int split = gather_split_warps(anchors);
      auto go = [&](auto kernel, int warps, int slot) {
        const int64_t fit = resident_warp_blocks(kernel, which + 4 * slot, warps);
        launch_pdl(warps > 1, kernel, dim3(static_cast<unsigned>(anchors < fit ? anchors : fit)), dim3(warps * 32), 0,
                   stream, q);
      };
      if (split == 8)
        go(k8, 8, 3);
      else if (split == 4)
        go(k4, 4, 2);
      else if (split == 2)
        go(k2, 2, 1);
      else
        go(k1, kWarpBlock, 0);
    };
#define S4D_WARP_FAMILY(T, KPS)                                                                 \
  launch_family(dfa_gather_warp_kernel<T, kFastNC, kFastNL, kFastNP, kFastG, 1, kWarpBlock, KPS>, \
                dfa_gather_coop_kernel<T, kFastNC, kFastNL, kFastNP, kFastG, 2, KPS>,             \
                dfa_gather_coop_kernel<T, kFastNC, kFastNL, kFastNP, kFastG, 4, KPS>,             \
                dfa_gather_coop_kernel<T, kFastNC, kFastNL, kFastNP, kFastG, 8, KPS>)
    if (p.kps_anchor != nullptr) {
      if (bf)
        S4D_WARP_FAMILY(__nv_bfloat16, true);
      else
        S4D_WARP_FAMILY(float, true);
    } else if (bf) {
      S4D_WARP_FAMILY(__nv_bfloat16, false);
    } else {
      S4D_WARP_FAMILY(float, false);
    }
#undef S4D_WARP_FAMILY
    return cuda_check(cudaGetLastError(), "dfa_gather_warp_kernel launch");
  }
  if (p.kps_anchor != nullptr)  // only the warp kernel computes sample locations; the others read p.loc
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "gather from anchors: needs the split-logit warp path");
  if (p.out_peer != nullptr)  // output routing exists in the warp kernels only
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "gather output routing: needs the split-logit warp path");
  if (fast_path_ok(p)) {
    if (feat_dtype == S4D_DTYPE_BF16)
      dfa_gather_fast_kernel<__nv_bfloat16, kFastNC, kFastNL, kFastNP, kFastG><<<grid, kGatherThreads, 0, stream>>>(p);
    else
      dfa_gather_fast_kernel<float, kFastNC, kFastNL, kFastNP, kFastG><<<grid, kGatherThreads, 0, stream>>>(p);
    return cuda_check(cudaGetLastError(), "dfa_gather_fast_kernel launch");
  }
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
