// InstanceBank kernels (inference): the temporal projection of the cached anchors and the
// confidence top-k selections that build the next frame's 600 cached + 300 new instances
// (model/instance_bank.py:95-306, projection model/instance_bank.py:322-369).
//
//   ib_project_kernel  one thread per cached anchor: centre moved by -velocity * dt, then
//                      centre, [cos, sin] yaw pair and velocity rotated by T (the reference
//                      stores the rotated [cos', sin'] in the (sin, cos) slots; kept as is).
//   ib_select_kernel   one CTA per frame.  Score per anchor = max over classes (CACHE: its
//                      sigmoid, evaluated in double and rounded once, then max with the decayed
//                      previous confidence for the first num_temp anchors).  Keys
//                      (order(score) << 32 | index) are sorted ascending in shared memory by a
//                      bitonic network: scores descending, ties by ascending index, NaN last.
//                      CACHE writes the top num_temp rows (feature, anchor) and scores; UPDATE
//                      writes [cached rows | top (A - num_temp) new rows], or the frame's own
//                      rows when its time gap exceeded the limit.
#include "params.cuh"

namespace s4d {
namespace {

constexpr int kSelectThreads = 512;

// Anchor layout (11 floats): x y z, log w l h, sin cos, vx vy vz.
__global__ void __launch_bounds__(256) ib_project_kernel(IbProjectParams p) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)p.bs * p.num) return;
  const int b = (int)(i / p.num);
  const float* a = p.anchor + i * p.anchor_dim;
  float* o = p.out + i * p.anchor_dim;
  const float* T = p.T + (int64_t)b * 16;
  const float dt = p.time_interval != nullptr ? p.time_interval[b] : 0.f;
  const float v[3] = {a[8], a[9], a[10]};
  const float c[3] = {a[0] - v[0] * dt, a[1] - v[1] * dt, a[2] - v[2] * dt};
  for (int r = 0; r < 3; ++r) o[r] = fmaf(T[4 * r + 2], c[2], fmaf(T[4 * r + 1], c[1], T[4 * r] * c[0])) + T[4 * r + 3];
  o[3] = a[3], o[4] = a[4], o[5] = a[5];
  const float cy = a[7], sy = a[6];
  o[6] = fmaf(T[1], sy, T[0] * cy);  // rotated [cos, sin] -> slots 6, 7 as in the reference
  o[7] = fmaf(T[5], sy, T[4] * cy);
  for (int r = 0; r < 3; ++r) o[8 + r] = fmaf(T[4 * r + 2], v[2], fmaf(T[4 * r + 1], v[1], T[4 * r] * v[0]));
}

// Ascending order of the key = descending order of the score; -0 == +0; NaN last.
__device__ __forceinline__ uint32_t desc_key(float v) {
  if (v != v) return 0xffffffffu;
  if (v == 0.f) v = 0.f;
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ~u;
}

// max that propagates NaN, as torch.max / torch.maximum do (fmaxf would drop it).
__device__ __forceinline__ float nan_max(float a, float b) { return (a != a || b != b) ? __int_as_float(0x7fffffff) : fmaxf(a, b); }

__device__ __forceinline__ void copy_row(float* dst, const float* src, int n, int lane) {
  if ((n & 3) == 0 && ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0) {
    for (int i = lane; i < n / 4; i += 32)
      reinterpret_cast<float4*>(dst)[i] = __ldg(reinterpret_cast<const float4*>(src) + i);
  } else {
    for (int i = lane; i < n; i += 32) dst[i] = __ldg(src + i);
  }
}

template <bool CACHE>
__global__ void __launch_bounds__(kSelectThreads) ib_select_kernel(IbSelectParams p) {
  extern __shared__ unsigned long long s_key[];  // [n2]
  const int b = blockIdx.x, tid = threadIdx.x;
  const int A = p.num_anchor, n2 = p.sort_size;
  const float* conf = p.confidence + (int64_t)b * A * p.num_cls;
  for (int a = tid; a < n2; a += kSelectThreads) {
    unsigned long long key = ~0ull;
    if (a < A) {
      float m = conf[(int64_t)a * p.num_cls];
      for (int k = 1; k < p.num_cls; ++k) m = nan_max(m, conf[(int64_t)a * p.num_cls + k]);
      if (CACHE) {
        m = (float)(1.0 / (1.0 + exp(-(double)m)));
        if (p.prev_conf != nullptr && a < p.num_temp) m = nan_max(p.prev_conf[(int64_t)b * p.num_temp + a] * p.decay, m);
      }
      key = ((unsigned long long)desc_key(m) << 32) | (unsigned)a;
    }
    s_key[a] = key;
  }
  __syncthreads();
  for (int k = 2; k <= n2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < n2; i += kSelectThreads) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long x = s_key[i], y = s_key[ixj];
          if ((x > y) == ((i & k) == 0)) {
            s_key[i] = y;
            s_key[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  }
  const int warp = tid >> 5, lane = tid & 31, nwarps = kSelectThreads / 32;
  const int C = p.embed_dims, D = p.anchor_dim;
  const float* feat = p.feature + (int64_t)b * A * C;
  const float* anc = p.anchor + (int64_t)b * A * D;
  if (CACHE) {
    const int K = p.num_temp;
    for (int r = warp; r < K; r += nwarps) {
      const int src = (int)(s_key[r] & 0xffffffffu);
      copy_row(p.out_feature + ((int64_t)b * K + r) * C, feat + (int64_t)src * C, C, lane);
      copy_row(p.out_anchor + ((int64_t)b * K + r) * D, anc + (int64_t)src * D, D, lane);
    }
    for (int r = tid; r < K; r += kSelectThreads) {
      const unsigned long long key = s_key[r];
      const int src = (int)(key & 0xffffffffu);
      if (p.out_idx != nullptr) p.out_idx[(int64_t)b * K + r] = src;
      if (p.out_conf != nullptr) {
        // invert desc_key: the score of this row
        uint32_t u = ~(uint32_t)(key >> 32);
        u = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;
        p.out_conf[(int64_t)b * K + r] = __uint_as_float(u);
      }
    }
  } else {
    const int K0 = p.num_temp, N = A - K0;
    float* of = p.out_feature + (int64_t)b * A * C;
    float* oa = p.out_anchor + (int64_t)b * A * D;
    const bool merge = p.mask == nullptr || p.mask[b] != 0;
    for (int r = warp; r < A; r += nwarps) {
      const float *sf, *sa;
      if (!merge) {
        sf = feat + (int64_t)r * C, sa = anc + (int64_t)r * D;
      } else if (r < K0) {
        sf = p.cached_feature + ((int64_t)b * K0 + r) * C, sa = p.cached_anchor + ((int64_t)b * K0 + r) * D;
      } else {
        const int src = (int)(s_key[r - K0] & 0xffffffffu);
        sf = feat + (int64_t)src * C, sa = anc + (int64_t)src * D;
      }
      copy_row(of + (int64_t)r * C, sf, C, lane);
      copy_row(oa + (int64_t)r * D, sa, D, lane);
    }
    if (p.out_idx != nullptr)
      for (int r = tid; r < N; r += kSelectThreads) p.out_idx[(int64_t)b * N + r] = (int)(s_key[r] & 0xffffffffu);
  }
}

}  // namespace

int launch_ib_project(const IbProjectParams& p, cudaStream_t stream) {
  const int64_t n = (int64_t)p.bs * p.num;
  if (n == 0) return S4D_OK;
  ib_project_kernel<<<unsigned((n + 255) / 256), 256, 0, stream>>>(p);
  return cuda_check(cudaGetLastError(), "ib_project_kernel launch");
}

int launch_ib_select(IbSelectParams p, bool cache, cudaStream_t stream) {
  if (p.bs == 0) return S4D_OK;
  int n2 = 1;
  while (n2 < p.num_anchor) n2 <<= 1;
  p.sort_size = n2;
  const size_t smem = size_t(n2) * sizeof(unsigned long long);
  if (cache) {
    ib_select_kernel<true><<<unsigned(p.bs), kSelectThreads, smem, stream>>>(p);
    return cuda_check(cudaGetLastError(), "ib_select_kernel (cache) launch");
  }
  ib_select_kernel<false><<<unsigned(p.bs), kSelectThreads, smem, stream>>>(p);
  return cuda_check(cudaGetLastError(), "ib_select_kernel (update) launch");
}

}  // namespace s4d
