// LayerNorm over the last dimension, one warp per row, for the decoder layers around the DFA
// (the norms of model/sparse4d_head.py's operation order, the pre-norm of the asymmetric FFN and
// the linear_relu_ln blocks of the refinement and anchor-encoder MLPs: nn.LayerNorm with
// eps 1e-5 over 32 to 512 features).  The decoder's rows are many (frames x 900 anchors) and
// narrow, so a warp holds a whole row in registers (width / 32 values per lane): one read, the
// mean and then the variance of the deviations from it reduced by shuffles, one write.
#include "common.cuh"

namespace s4d {
namespace {

constexpr int kLnWarps = 8;  // rows per block

template <int PER_LANE>
__global__ void __launch_bounds__(kLnWarps * 32)
    layer_norm_kernel(const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ b,
                      float* __restrict__ y, int64_t rows, float eps) {
  constexpr int N = PER_LANE * 32;
  const int lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * kLnWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* xr = x + row * N;
  float v[PER_LANE];
#pragma unroll
  for (int j = 0; j < PER_LANE; ++j) v[j] = __ldg(xr + j * 32 + lane);
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < PER_LANE; ++j) s += v[j];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s * (1.0f / N);
  float q = 0.0f;
#pragma unroll
  for (int j = 0; j < PER_LANE; ++j) {
    const float d = v[j] - mean;
    q = fmaf(d, d, q);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rstd = rsqrtf(q * (1.0f / N) + eps);
  float* yr = y + row * N;
#pragma unroll
  for (int j = 0; j < PER_LANE; ++j) {
    const int c = j * 32 + lane;
    const float n = (v[j] - mean) * rstd;
    yr[c] = w != nullptr ? fmaf(n, __ldg(w + c), b != nullptr ? __ldg(b + c) : 0.0f) : n;
  }
}

bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3) == 0; }

}  // namespace
}  // namespace s4d

using namespace s4d;

extern "C" int s4d_layer_norm(const float* x, const float* weight, const float* bias, float* y, int64_t rows,
                              int64_t width, float eps, void* stream) {
  set_error("%s", "");
  if (rows < 0) return fail(S4D_ERR_INVALID_ARG, "s4d_layer_norm: negative rows");
  if (width != 32 && width != 64 && width != 128 && width != 256 && width != 512)
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_layer_norm: width must be 32, 64, 128, 256 or 512");
  int64_t total = 0;
  if (!size_product({rows, width}, int64_t(1) << 40, &total))
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_layer_norm: too many elements");
  if (!(eps >= 0.0f)) return fail(S4D_ERR_INVALID_ARG, "s4d_layer_norm: eps must be >= 0");
  if (rows == 0) return S4D_OK;
  if (x == nullptr || y == nullptr) return fail(S4D_ERR_INVALID_ARG, "s4d_layer_norm: null pointer");
  if (bias != nullptr && weight == nullptr)
    return fail(S4D_ERR_INVALID_ARG, "s4d_layer_norm: a bias needs a weight");
  if (!aligned4(x) || !aligned4(y) || (weight != nullptr && !aligned4(weight)) || (bias != nullptr && !aligned4(bias)))
    return fail(S4D_ERR_INVALID_ARG, "s4d_layer_norm: misaligned pointer");
  const int64_t blocks = (rows + kLnWarps - 1) / kLnWarps;
  if (blocks > 0x7fffffff) return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_layer_norm: too many rows");
  const dim3 grid{static_cast<unsigned>(blocks)};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (width) {
    case 32: layer_norm_kernel<1><<<grid, kLnWarps * 32, 0, st>>>(x, weight, bias, y, rows, eps); break;
    case 64: layer_norm_kernel<2><<<grid, kLnWarps * 32, 0, st>>>(x, weight, bias, y, rows, eps); break;
    case 128: layer_norm_kernel<4><<<grid, kLnWarps * 32, 0, st>>>(x, weight, bias, y, rows, eps); break;
    case 256: layer_norm_kernel<8><<<grid, kLnWarps * 32, 0, st>>>(x, weight, bias, y, rows, eps); break;
    default: layer_norm_kernel<16><<<grid, kLnWarps * 32, 0, st>>>(x, weight, bias, y, rows, eps); break;
  }
  return cuda_check(cudaGetLastError(), "layer_norm_kernel launch");
}
