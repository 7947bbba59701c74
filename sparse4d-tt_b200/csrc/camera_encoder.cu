// Per-frame camera terms of the DFA layer: the camera encoder
//   x = projection_mat[:3, :4] (12 values per camera)
//   h = LN(ReLU(W1 x + b1)); g = LN(ReLU(W2 h + b2))           (camera_embed)
// (model/deformable_feature_aggregation.py:679-717; test/dfa_pcc.py:272-279,309-312) and the
// per-camera term of the split weight logits, wc = W_fc g + b_fc, i.e. weights_fc applied to
// the camera embedding (model/deformable_feature_aggregation.py:719-798; test/dfa_pcc.py:313-316).
//
// Two launches, each CTA one frame (all its cameras share every weight load) and one slice of
// 32 output channels, so that the weight matrices are spread over many SMs:
//   camera_hidden_kernel  grid (bs, C / 32): layer 1 + LayerNorm (recomputed per CTA, 12 inputs),
//                         then its 32 channels of ReLU(W2 h + b2) to a [bs, Ncam, C] scratch;
//   camera_logits_kernel  grid (bs, ceil(n / 32)): LayerNorm 2 of the scratch rows, then its 32
//                         logit columns of W_fc g + b_fc (the first slice also writes g).
// Within a slice, lane group (o = t / 8, kp = t % 8) sums output o over inputs [32 kp, 32 kp + 32)
// and the 8 partial sums are combined by shuffles.  fp32 throughout; LayerNorm with eps 1e-5
// and the biased variance, mean and variance in two passes over the row.
//
// camera_terms_kernel does the same work, and the per-frame softmax factors of the gather, in
// one launch: a cluster of 8 CTAs per frame.  CTA r computes hidden channels [32 r, 32 r + 32)
// into its shared memory, every CTA then reads all 256 channels from the 8 CTAs' shared memory
// (distributed shared memory, no global scratch), normalises them (LayerNorm 2) and computes its
// share of the logit columns; for the factors the CTAs exchange their per-group column maxima
// the same way.  Every value is computed by the same functions in the same order as the
// two-launch path and the factor kernel of the gather, so the results are bitwise equal.
#include <cooperative_groups.h>

#include "params.cuh"

namespace s4d {
namespace {

constexpr int kC = 256;
constexpr int kMaxCams = 8;

// Mean and variance of the rows held one value per thread (v[c] for camera c), then the
// normalised, scaled and shifted value of this thread's channel.
__device__ __forceinline__ void layer_norm_rows(float (&v)[kMaxCams], int nc, float gamma, float beta,
                                                float (*s_red)[kC / 32]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float mean[kMaxCams];
#pragma unroll
  for (int c = 0; c < kMaxCams; ++c) {
    float s = c < nc ? v[c] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) s_red[c][warp] = s;
  }
  __syncthreads();
#pragma unroll
  for (int c = 0; c < kMaxCams; ++c) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kC / 32; ++w) s += s_red[c][w];
    mean[c] = s * (1.0f / kC);
  }
  __syncthreads();
#pragma unroll
  for (int c = 0; c < kMaxCams; ++c) {
    const float d = c < nc ? v[c] - mean[c] : 0.f;
    float s = d * d;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) s_red[c][warp] = s;
  }
  __syncthreads();
#pragma unroll
  for (int c = 0; c < kMaxCams; ++c) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kC / 32; ++w) s += s_red[c][w];
    v[c] = (v[c] - mean[c]) * rsqrtf(s * (1.0f / kC) + 1e-5f) * gamma + beta;
  }
  __syncthreads();
}

// Loads the frame's 12 camera inputs, then layer 1 + LayerNorm 1 for every channel into s_h.
__device__ __forceinline__ void camera_layer1(const CamEncParams& p, int f, float (*s_x)[12], float (*s_h)[kC],
                                              float (*s_red)[kC / 32]) {
  const int t = threadIdx.x, nc = p.num_cams;
  for (int i = t; i < nc * 12; i += kC) s_x[i / 12][i % 12] = p.proj[(int64_t(f) * nc + i / 12) * 16 + i % 12];
  __syncthreads();
  float v[kMaxCams];
  float w[12];
#pragma unroll
  for (int k = 0; k < 12; ++k) w[k] = __ldg(p.w1 + t * 12 + k);
  const float b = __ldg(p.b1 + t);
#pragma unroll
  for (int c = 0; c < kMaxCams; ++c) {
    float a = b;
    if (c < nc) {
#pragma unroll
      for (int k = 0; k < 12; ++k) a = fmaf(w[k], s_x[c][k], a);
    }
    v[c] = fmaxf(a, 0.f);
  }
  layer_norm_rows(v, nc, __ldg(p.ln1_w + t), __ldg(p.ln1_b + t), s_red);
#pragma unroll
  for (int c = 0; c < kMaxCams; ++c)
    if (c < nc) s_h[c][t] = v[c];
  __syncthreads();
}

// Output o = t / 8 of this CTA's 32-row weight slice W[row0 .. row0 + 32) applied to every
// camera row of s_in: lane group kp = t % 8 covers inputs [32 kp, 32 kp + 32), visiting its 8
// float4 chunks in the order (i + kp) mod 8 so that the 8 lanes of a shared-memory phase read
// different banks; the partial sums meet by shuffles.  Returns the sums (valid on every lane
// of the group) in acc[c].
__device__ __forceinline__ void slice_dot(const float* __restrict__ w, int row0, int nrows, const float (*s_in)[kC],
                                          int nc, float (&acc)[kMaxCams]) {
  const int t = threadIdx.x, o = t >> 3, kp = t & 7;
#pragma unroll
  for (int c = 0; c < kMaxCams; ++c) acc[c] = 0.f;
  if (row0 + o < nrows) {
    const float4* w4 = reinterpret_cast<const float4*>(w + int64_t(row0 + o) * kC + kp * 32);
    float4 wv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) wv[i] = __ldg(w4 + ((i + kp) & 7));
#pragma unroll
    for (int c = 0; c < kMaxCams; ++c) {
      if (c < nc) {
        const float4* h4 = reinterpret_cast<const float4*>(s_in[c] + kp * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 h = h4[(i + kp) & 7];
          acc[c] = fmaf(wv[i].x, h.x, acc[c]);
          acc[c] = fmaf(wv[i].y, h.y, acc[c]);
          acc[c] = fmaf(wv[i].z, h.z, acc[c]);
          acc[c] = fmaf(wv[i].w, h.w, acc[c]);
        }
      }
    }
  }
#pragma unroll
  for (int c = 0; c < kMaxCams; ++c) {
    acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], 1);
    acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], 2);
    acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], 4);
  }
}

__global__ void __launch_bounds__(kC) camera_hidden_kernel(const CamEncParams p) {
  __shared__ float s_x[kMaxCams][12];
  __shared__ __align__(16) float s_h[kMaxCams][kC];
  __shared__ float s_red[kMaxCams][kC / 32];
  const int f = blockIdx.x, row0 = blockIdx.y * 32, nc = p.num_cams;
  camera_layer1(p, f, s_x, s_h, s_red);
  float acc[kMaxCams];
  slice_dot(p.w2, row0, kC, s_h, nc, acc);
  const int t = threadIdx.x, o = t >> 3, kp = t & 7;
  const float b = __ldg(p.b2 + row0 + o);
#pragma unroll
  for (int c = 0; c < kMaxCams; ++c)
    if (c < nc && kp == c) p.hidden[(int64_t(f) * nc + c) * kC + row0 + o] = fmaxf(acc[c] + b, 0.f);
}

__global__ void __launch_bounds__(kC) camera_logits_kernel(const CamEncParams p) {
  __shared__ __align__(16) float s_g[kMaxCams][kC];
  __shared__ float s_red[kMaxCams][kC / 32];
  const int f = blockIdx.x, row0 = blockIdx.y * 32, t = threadIdx.x, nc = p.num_cams;
  float v[kMaxCams];
#pragma unroll
  for (int c = 0; c < kMaxCams; ++c) v[c] = c < nc ? p.hidden[(int64_t(f) * nc + c) * kC + t] : 0.f;
  layer_norm_rows(v, nc, __ldg(p.ln2_w + t), __ldg(p.ln2_b + t), s_red);
#pragma unroll
  for (int c = 0; c < kMaxCams; ++c)
    if (c < nc) {
      s_g[c][t] = v[c];
      if (p.camera_embed != nullptr && blockIdx.y == 0) p.camera_embed[(int64_t(f) * nc + c) * kC + t] = v[c];
    }
  __syncthreads();
  float acc[kMaxCams];
  slice_dot(p.w_fc, row0, p.num_logits, s_g, nc, acc);
  const int o = t >> 3, kp = t & 7;
  if (row0 + o < p.num_logits) {
    const float b = __ldg(p.b_fc + row0 + o);
#pragma unroll
    for (int c = 0; c < kMaxCams; ++c)
      if (c < nc && kp == c) p.logits[(int64_t(f) * nc + c) * p.num_logits + row0 + o] = acc[c] + b;
  }
}

constexpr int kSlices = 8;         // CTAs per frame in camera_terms_kernel (one cluster)
constexpr int kMaxSliceCols = 64;  // logit columns per CTA there: num_logits <= 512
constexpr int kFactorGroups = 8;   // softmax groups of the factors: column j is group j % 8

__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Split cluster barrier: arrive (release this thread's earlier writes) and wait (acquire).
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// One cluster of kSlices CTAs per frame (grid (bs, kSlices)).  Barrier phases of the cluster:
//   1  every CTA has written its hidden slice          (full barrier, then the remote reads)
//   2  every CTA has read the others' slices           (arrive after the reads, wait later)
//   3  every CTA has published its group maxima        (factors only)
//   4  every CTA has read the others' maxima           (arrive after the reads, wait at exit)
// A CTA leaves only after the last phase it takes part in, so no CTA's shared memory goes away
// while another CTA reads it.
__global__ void __cluster_dims__(1, kSlices, 1) __launch_bounds__(kC) camera_terms_kernel(const CamEncParams p) {
  namespace cg = cooperative_groups;
  constexpr float kLog2e = 1.4426950408889634f;
  __shared__ float s_x[kMaxCams][12];
  __shared__ __align__(16) float s_h[kMaxCams][kC];  // layer 1 output, then LayerNorm 2 output
  __shared__ float s_red[kMaxCams][kC / 32];
  __shared__ float s_slice[kMaxCams][32];            // this CTA's hidden channels, read by the cluster
  __shared__ float s_wc[kMaxCams][kMaxSliceCols];    // this CTA's logit columns
  __shared__ float s_gmax[kFactorGroups];            // their per-group maxima, read by the cluster
  __shared__ float s_m2[kFactorGroups];              // the frame's per-group maxima x log2(e)
  cg::cluster_group cluster = cg::this_cluster();
  const int f = blockIdx.x, r = int(cluster.block_rank()), t = threadIdx.x, nc = p.num_cams, n = p.num_logits;
  const int o = t >> 3, kp = t & 7, lane = t & 31, warp = t >> 5;

  camera_layer1(p, f, s_x, s_h, s_red);
  float acc[kMaxCams];
  slice_dot(p.w2, r * 32, kC, s_h, nc, acc);
  const float b2 = __ldg(p.b2 + r * 32 + o);
#pragma unroll
  for (int c = 0; c < kMaxCams; ++c)
    if (c < nc && kp == c) s_slice[c][o] = fmaxf(acc[c] + b2, 0.f);
  cluster.sync();  // phase 1; also ends this CTA's reads of s_h
  float v[kMaxCams];
  {
    const float* src = cluster.map_shared_rank(&s_slice[0][0], t >> 5);  // channel t lives in CTA t / 32
#pragma unroll
    for (int c = 0; c < kMaxCams; ++c) v[c] = c < nc ? src[c * 32 + lane] : 0.f;
  }
  cluster_arrive();  // phase 2
  layer_norm_rows(v, nc, __ldg(p.ln2_w + t), __ldg(p.ln2_b + t), s_red);
#pragma unroll
  for (int c = 0; c < kMaxCams; ++c)
    if (c < nc) {
      s_h[c][t] = v[c];
      if (p.camera_embed != nullptr && r == 0) p.camera_embed[(int64_t(f) * nc + c) * kC + t] = v[c];
    }
  __syncthreads();

  // logit columns [col0, col1): a multiple of 8 per CTA, so that column col0 + jj is group jj % 8
  const int per = (n + 8 * kSlices - 1) / (8 * kSlices) * 8;
  const int col0 = r * per, col1 = min(n, col0 + per), cols = max(0, col1 - col0);
  for (int row0 = col0; row0 < col1; row0 += 32) {
    slice_dot(p.w_fc, row0, col1, s_h, nc, acc);
    if (row0 + o < col1) {
      const float b = __ldg(p.b_fc + row0 + o);
#pragma unroll
      for (int c = 0; c < kMaxCams; ++c)
        if (c < nc && kp == c) {
          const float x = acc[c] + b;
          p.logits[(int64_t(f) * nc + c) * n + row0 + o] = x;
          s_wc[c][row0 - col0 + o] = x;
        }
    }
  }
  if (p.factors == nullptr) {
    cluster_wait();  // phase 2
    return;
  }
  __syncthreads();
  // per-group maximum of this CTA's columns: element e = c * cols + jj is group e % 8 = t % 8
  float m = -INFINITY;
  for (int e = t; e < nc * cols; e += kC) m = fmaxf(m, s_wc[e / cols][e % cols]);
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
  if (lane < kFactorGroups) s_red[warp][lane] = m;
  __syncthreads();
  if (t < kFactorGroups) {
    float g = s_red[0][t];
#pragma unroll
    for (int w = 1; w < kC / 32; ++w) g = fmaxf(g, s_red[w][t]);
    s_gmax[t] = g;
  }
  cluster_wait();    // phase 2
  cluster_arrive();  // phase 3: s_gmax published
  cluster_wait();
  if (t < kFactorGroups) {
    float g = -INFINITY;
    for (int q = 0; q < kSlices; ++q) g = fmaxf(g, *cluster.map_shared_rank(&s_gmax[t], q));
    s_m2[t] = g * kLog2e;
  }
  cluster_arrive();  // phase 4
  __syncthreads();
  // factors of this CTA's columns: ec[c][j] = exp(wc[c][j] - M2[g]) and their sum over the cameras
  float* ec = p.factors + int64_t(f) * (nc + 1) * n;
  for (int jj = t; jj < cols; jj += kC) {
    const float mg = s_m2[jj % kFactorGroups];
    float s = 0.0f;
    for (int c = 0; c < nc; ++c) {
      const float e = ex2_fast(fmaf(s_wc[c][jj], kLog2e, -mg));
      ec[c * n + col0 + jj] = e;
      s += e;
    }
    ec[nc * n + col0 + jj] = s;
  }
  if (f == 0 && r == 0 && t < 2) p.anchor_counter[t] = 0u;
  cluster_wait();  // phase 4
}

}  // namespace

int launch_camera_terms(const CamEncParams& p, cudaStream_t stream) {
  if (p.bs <= 0) return S4D_OK;
  if (p.num_cams < 1 || p.num_cams > kMaxCams || p.embed_dims != kC || p.num_logits < 1 ||
      p.num_logits > kSlices * kMaxSliceCols)
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "camera_terms: implemented for 1..8 cameras, embed_dims 256 and 1..512 logits");
  if (p.factors != nullptr && (p.num_logits % kFactorGroups != 0 || p.anchor_counter == nullptr))
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "camera_terms: the factors need 8 groups (num_logits a multiple of 8)");
  camera_terms_kernel<<<dim3(unsigned(p.bs), kSlices), kC, 0, stream>>>(p);
  return cuda_check(cudaGetLastError(), "camera_terms_kernel launch");
}

int launch_camera_logits(const CamEncParams& p, cudaStream_t stream) {
  if (p.bs <= 0) return S4D_OK;
  if (p.num_cams < 1 || p.num_cams > kMaxCams || p.embed_dims != kC)
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "camera_logits: implemented for 1..8 cameras and embed_dims 256");
  if (p.hidden == nullptr) return fail(S4D_ERR_INVALID_ARG, "camera_logits: no scratch for the hidden layer");
  camera_hidden_kernel<<<dim3(unsigned(p.bs), kC / 32), kC, 0, stream>>>(p);
  int st = cuda_check(cudaGetLastError(), "camera_hidden_kernel launch");
  if (st != S4D_OK) return st;
  camera_logits_kernel<<<dim3(unsigned(p.bs), unsigned((p.num_logits + 31) / 32)), kC, 0, stream>>>(p);
  return cuda_check(cudaGetLastError(), "camera_logits_kernel launch");
}

}  // namespace s4d
