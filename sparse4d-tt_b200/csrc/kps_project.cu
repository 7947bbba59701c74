// Kernel (a): keypoint generation, projection, depth/frustum masks and lexicographic
// compaction of the visible (batch, anchor, camera, point) indices.
//
// Follows the reference's _KPSGenerator.forward (test/dfa_pcc.py:225-247) and project_points
// (test/dfa_pcc.py:322-333); in TT-NN the same work is ttnn.kps_project_fused
// (tt-metal/ops/kps_project_fused/device/kernels/dataflow/reader_kps_project.cpp:255-289)
// fed by _kps_generator_pre_rotation (model/deformable_feature_aggregation.py:651-677).
//
// Work split: one thread per (batch, anchor, camera, point) element, elements in
// lexicographic order, so every output store is coalesced and the visibility bits of a warp
// are 32 consecutive elements.  A block owns kElemsPerBlock consecutive elements (4 rounds of
// 256).  Compaction is count -> scatter with no inter-block waits: the project kernel writes
// one ballot word per 32 elements and one visible count per block; the scatter kernel sums the
// counts of the blocks before it, scans its own 32 words and writes the rows.
//
// The keypoint and projection arithmetic (fixed order, no fused multiply-add on any line that
// decides a mask bit, so the integer outputs reproduce a CPU evaluation of the same expression
// order bit for bit) is in kps_math.cuh, shared with the gather that computes its own sample
// locations.
#include "kps_math.cuh"
#include "params.cuh"

namespace s4d {

constexpr int kKpsThreads = 256;
constexpr int kKpsRounds = 4;
constexpr int kElemsPerBlock = kKpsThreads * kKpsRounds;  // 1024
constexpr int kWordsPerBlock = kElemsPerBlock / 32;        // 32
constexpr int kMaxPts = 64;                                // keypoints per anchor supported
// anchors touched by one block's elements x keypoints: <= (1024 / (Ncam*P) + 2) * P
constexpr int kMaxBlockKeypoints = kElemsPerBlock + 2 * kMaxPts;


// Rotated + translated keypoint p of anchor n (fp32, fixed order); `lg` holds the anchor's
// learnable logits (global memory, or the block's shared-memory copy).
__device__ __forceinline__ void keypoint(const KpsParams& k, uint32_t n, int p, const float* lg_anchor, float& px,
                                         float& py, float& pz) {
  const float* a = k.anchor + (int64_t)n * k.anchor_dim;
  float kx, ky, kz;
  if (k.kp_pre != nullptr) {
    const float* q = k.kp_pre + ((int64_t)n * k.num_pts + p) * 3;
    kx = q[0];
    ky = q[1];
    kz = q[2];
  } else {
    kps_scaled(a, k.fix_scale, k.num_fix, lg_anchor, p, kx, ky, kz);
  }
  kps_place(a, kx, ky, kz, px, py, pz);
}

template <bool FUSED>
__global__ void __launch_bounds__(kKpsThreads) kps_project_kernel(KpsParams k) {
  // Keypoints of the anchors this block's elements belong to, computed once each (not once per
  // camera) and shared through shared memory.
  __shared__ float s_kp[kMaxBlockKeypoints * 3];
  // Index arithmetic in 32 bits (the host guarantees total < 2^31) with multiply-high divisions.
  const int lane = threadIdx.x & 31;
  const uint32_t total = (uint32_t)k.total;
  const uint32_t block_base = blockIdx.x * kElemsPerBlock;
  const uint32_t per_anchor = k.num_cams * k.num_pts;
  const uint32_t n0 = k.div_anchor_elems.div(block_base);
  const uint32_t last = block_base + kElemsPerBlock - 1 < total ? block_base + kElemsPerBlock - 1 : total - 1;
  const int nkp = (int)(k.div_anchor_elems.div(last) - n0 + 1) * k.num_pts;
  const int nl3 = k.num_learnable * 3;
  // In-kernel learnable logits (the keypoint generator's learnable_fc, fp32) of the block's
  // anchors: their instance rows are staged in shared memory in 8 chunks of 32 floats (chunk
  // stride 36 floats, so the 8 chunks a warp reads at once sit in different banks); thread
  // t = 8 o + kc keeps learnable_fc row o, chunk kc in registers and sums that chunk for every
  // anchor; the 8 chunk sums of (anchor, o) meet by shuffles.  The weights are read once per block.
  __shared__ __align__(16) float s_x[1][FUSED ? kKpsMaxFusedAnchors * 8 * 36 : 4];
  __shared__ float s_lg[FUSED ? kKpsMaxFusedAnchors * kKpsMaxFusedLogits : 1];
  if (FUSED) {
    const int n_anc = nkp / k.num_pts;
    for (int idx = threadIdx.x; idx < n_anc * 64; idx += kKpsThreads) {
      const int j = idx >> 6, q = idx & 63;
      const float4 v = __ldg(reinterpret_cast<const float4*>(k.inst + (int64_t)(n0 + j) * k.inst_ld) + q);
      *reinterpret_cast<float4*>(&s_x[0][j * 288 + (q >> 3) * 36 + (q & 7) * 4]) = v;
    }
    const int o = threadIdx.x >> 3, kc = threadIdx.x & 7;
    const bool active = o < nl3;
    float w[32];
    const float4* wr = reinterpret_cast<const float4*>(k.w_kps + (int64_t)(active ? o : 0) * 256 + kc * 32);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 v = __ldg(wr + i);
      w[4 * i] = v.x, w[4 * i + 1] = v.y, w[4 * i + 2] = v.z, w[4 * i + 3] = v.w;
    }
    const float bias = active && k.b_kps != nullptr ? __ldg(k.b_kps + o) : 0.f;
    __syncthreads();
    for (int j = 0; j < n_anc; ++j) {
      const float4* x = reinterpret_cast<const float4*>(&s_x[0][j * 288 + kc * 36]);
      float a0 = 0.f, a1 = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 v = x[i];
        a0 = fmaf(v.x, w[4 * i], a0);
        a1 = fmaf(v.y, w[4 * i + 1], a1);
        a0 = fmaf(v.z, w[4 * i + 2], a0);
        a1 = fmaf(v.w, w[4 * i + 3], a1);
      }
      float acc = a0 + a1;
      acc += __shfl_xor_sync(0xffffffffu, acc, 4);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      if (active && kc == 0) s_lg[j * nl3 + o] = acc + bias;
    }
    __syncthreads();
  }
  for (int i = threadIdx.x; i < nkp; i += kKpsThreads) {
    const uint32_t j = k.div_pts.div(i);
    const uint32_t n = n0 + j;
    const int p = i - (int)j * k.num_pts;
    const float* lg = FUSED ? s_lg + j * nl3 : (k.learnable != nullptr ? k.learnable + (int64_t)n * nl3 : nullptr);
    float px, py, pz;
    keypoint(k, n, p, lg, px, py, pz);
    s_kp[3 * i] = px;
    s_kp[3 * i + 1] = py;
    s_kp[3 * i + 2] = pz;
    if (k.key_points != nullptr) {  // anchors shared by two blocks are written twice, identically
      float* kp = k.key_points + ((int64_t)n * k.num_pts + p) * 3;
      kp[0] = px;
      kp[1] = py;
      kp[2] = pz;
    }
  }
  __syncthreads();
  int count = 0;
#pragma unroll
  for (int r = 0; r < kKpsRounds; ++r) {
    const uint32_t e = block_base + r * kKpsThreads + threadIdx.x;
    bool vis = false;
    if (e < total) {
      const uint32_t n = k.div_anchor_elems.div(e);  // linear anchor index b * A + a
      const uint32_t rem = e - n * per_anchor;
      const uint32_t c = k.div_pts.div(rem);
      const int p = (int)(rem - c * k.num_pts);
      const uint32_t b = k.div_anchors.div(n);
      const int ik = (int)(n - n0) * k.num_pts + p;
      const float px = s_kp[3 * ik], py = s_kp[3 * ik + 1], pz = s_kp[3 * ik + 2];
      float u, v;
      bool in_front;
      const float* P = k.proj + (b * k.num_cams + c) * 16;
      const float* wh = k.wh + (b * k.num_cams + c) * 2;
      kps_uv(make_float4(P[0], P[1], P[2], P[3]), make_float4(P[4], P[5], P[6], P[7]),
             make_float4(P[8], P[9], P[10], P[11]), wh[0], wh[1], px, py, pz, u, v, in_front);
      vis = in_front && u >= 0.0f && u <= 1.0f && v >= 0.0f && v <= 1.0f;
      if (k.mask != nullptr) k.mask[e] = in_front ? 1 : 0;
      if (k.loc != nullptr) {
        if (k.layout == S4D_LAYOUT_CAM_MAJOR) {
          reinterpret_cast<float2*>(k.loc)[e] = make_float2(u, v);
        } else if (k.layout == S4D_LAYOUT_PT_MAJOR) {
          reinterpret_cast<float2*>(k.loc)[((int64_t)n * k.num_pts + p) * k.num_cams + c] = make_float2(u, v);
        } else {  // GRID: [ncam, n_total, P, 2], 2*uv - 1 clamped to [-2, 2]
          const int64_t n_total = (int64_t)k.bs * k.num_anchor;
          const float gx = fminf(fmaxf(__fsub_rn(__fmul_rn(u, 2.0f), 1.0f), -2.0f), 2.0f);
          const float gy = fminf(fmaxf(__fsub_rn(__fmul_rn(v, 2.0f), 1.0f), -2.0f), 2.0f);
          reinterpret_cast<float2*>(k.loc)[((int64_t)c * n_total + n) * k.num_pts + p] = make_float2(gx, gy);
        }
      }
    }
    if (k.vis_words != nullptr) {
      const uint32_t word = __ballot_sync(0xffffffffu, vis);
      if (lane == 0) {
        k.vis_words[(int64_t)blockIdx.x * kWordsPerBlock + r * (kKpsThreads / 32) + (threadIdx.x >> 5)] = word;
        count += __popc(word);
      }
    }
  }
  if (k.block_counts != nullptr) {
    __shared__ int s_cnt[kKpsThreads / 32];
    if (lane == 0) s_cnt[threadIdx.x >> 5] = count;
    __syncthreads();
    if (threadIdx.x == 0) {
      int t = 0;
#pragma unroll
      for (int w = 0; w < kKpsThreads / 32; ++w) t += s_cnt[w];
      k.block_counts[blockIdx.x] = t;
    }
  }
}

// Writes the (b, a, cam, pt) rows of the visible elements of this block at their global
// lexicographic position.  The block's offset is the sum of the counts of all earlier blocks,
// read directly (no inter-block waiting; the project kernel has finished in stream order).
__global__ void __launch_bounds__(kKpsThreads) kps_compact_kernel(const int32_t* __restrict__ block_counts,
                                                                  const uint32_t* __restrict__ vis_words,
                                                                  int num_blocks, FastDiv div_anchor_elems,
                                                                  FastDiv div_pts, FastDiv div_anchors,
                                                                  int4* __restrict__ idx,
                                                                  int32_t* __restrict__ count_out) {
  __shared__ int s_part[kKpsThreads / 32];
  __shared__ int s_word_off[kWordsPerBlock];
  __shared__ uint32_t s_words[kWordsPerBlock];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  int part = 0;
  for (int j = threadIdx.x; j < (int)blockIdx.x; j += kKpsThreads) part += block_counts[j];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if (lane == 0) s_part[warp] = part;
  if (warp == 0) {
    const uint32_t w = vis_words[(int64_t)blockIdx.x * kWordsPerBlock + lane];
    s_words[lane] = w;
    int c = __popc(w);
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    s_word_off[lane] = incl - c;
  }
  __syncthreads();
  int block_off = 0;
#pragma unroll
  for (int w = 0; w < kKpsThreads / 32; ++w) block_off += s_part[w];
  if (count_out != nullptr && blockIdx.x == num_blocks - 1 && threadIdx.x == 0) {
    *count_out = block_off + s_word_off[kWordsPerBlock - 1] + __popc(s_words[kWordsPerBlock - 1]);
  }
  if (idx == nullptr) return;
#pragma unroll
  for (int r = 0; r < kKpsRounds; ++r) {
    const int word_id = r * (kKpsThreads / 32) + warp;
    const uint32_t w = s_words[word_id];
    if ((w >> lane) & 1u) {
      const uint32_t e = blockIdx.x * kElemsPerBlock + r * kKpsThreads + threadIdx.x;
      const int pos = block_off + s_word_off[word_id] + __popc(w & ((1u << lane) - 1u));
      const uint32_t n = div_anchor_elems.div(e);
      const uint32_t rem = e - n * div_anchor_elems.d;
      const uint32_t c = div_pts.div(rem);
      const uint32_t b = div_anchors.div(n);
      idx[pos] = make_int4((int)b, (int)(n - b * div_anchors.d), (int)c, (int)(rem - c * div_pts.d));
    }
  }
}

int64_t kps_num_blocks(int64_t total) { return (total + kElemsPerBlock - 1) / kElemsPerBlock; }

size_t kps_workspace_bytes(int64_t total) {
  const int64_t nb = kps_num_blocks(total);
  const size_t counts = ((size_t)nb * sizeof(int32_t) + 255) & ~(size_t)255;
  return counts + (size_t)nb * kWordsPerBlock * sizeof(uint32_t);
}

int launch_kps_project(KpsParams k, int32_t* visible_idx, int32_t* visible_count, void* workspace,
                       cudaStream_t stream) {
  const int64_t nb = kps_num_blocks(k.total);
  const bool compact = visible_idx != nullptr || visible_count != nullptr;
  if (compact) {
    k.block_counts = static_cast<int32_t*>(workspace);
    const size_t counts = ((size_t)nb * sizeof(int32_t) + 255) & ~(size_t)255;
    k.vis_words = reinterpret_cast<uint32_t*>(static_cast<char*>(workspace) + counts);
  } else {
    k.block_counts = nullptr;
    k.vis_words = nullptr;
  }
  k.div_anchor_elems = FastDiv((uint32_t)(k.num_cams * k.num_pts));
  k.div_pts = FastDiv((uint32_t)k.num_pts);
  k.div_anchors = FastDiv((uint32_t)k.num_anchor);
  if (k.inst != nullptr)
    kps_project_kernel<true><<<(unsigned)nb, kKpsThreads, 0, stream>>>(k);
  else
    kps_project_kernel<false><<<(unsigned)nb, kKpsThreads, 0, stream>>>(k);
  int st = cuda_check(cudaGetLastError(), "kps_project_kernel launch");
  if (st != S4D_OK || !compact) return st;
  kps_compact_kernel<<<(unsigned)nb, kKpsThreads, 0, stream>>>(
      k.block_counts, k.vis_words, (int)nb, k.div_anchor_elems, k.div_pts, k.div_anchors,
      reinterpret_cast<int4*>(visible_idx), visible_count);
  return cuda_check(cudaGetLastError(), "kps_compact_kernel launch");
}

}  // namespace s4d
