// Shared helpers of the DFA kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <initializer_list>
#include <utility>

#include "s4d_dfa.h"

namespace s4d {

// Records the text of the last failure on this host thread (read by s4d_last_error()).
void set_error(const char* fmt, ...);

inline int fail(int status, const char* msg) {
  set_error("%s", msg);
  return status;
}

inline int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return S4D_OK;
  set_error("%s: %s", what, cudaGetErrorString(e));
  return S4D_ERR_CUDA;
}

// Product of sizes passed through the C ABI, computed without signed overflow: true and *out set
// when every factor is >= 0 and the product is < limit; false when a factor is negative, the
// product overflows int64_t or it reaches limit.
inline bool size_product(std::initializer_list<int64_t> factors, int64_t limit, int64_t* out) {
  int64_t r = 1;
  for (int64_t v : factors) {
    if (v < 0 || __builtin_mul_overflow(r, v, &r)) return false;
  }
  *out = r;
  return r < limit;
}

// Quotient of a non-negative integer n < 2^31 by a runtime divisor d >= 1 with one multiply-high
// and a shift, by the round-up method of Granlund & Montgomery ("Division by invariant integers
// using multiplication", PLDI 1994): with l = ceil(log2 d) and m = floor(2^32 (2^l - d) / d) + 1,
// floor(n / d) == (umulhi(n, m) + n) >> l for every n < 2^32 whose sum does not overflow, which
// n < 2^31 guarantees.
struct FastDiv {
  uint32_t d = 1, m = 1, l = 0;
  FastDiv() = default;
  __host__ explicit FastDiv(uint32_t div) : d(div) {
    l = 0;
    while ((uint64_t(1) << l) < div) ++l;
    m = uint32_t(((uint64_t(1) << 32) * ((uint64_t(1) << l) - div)) / div + 1);
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const { return (__umulhi(n, m) + n) >> l; }
};

// 8 consecutive bf16 channels (one 16-byte vector) widened to fp32.
__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // bf16 is the top half of an fp32: shifting the bits into place is exact.
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float4 ldg_nc_f4(const void* p) {
  float4 r;
  asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}

// Programmatic dependent launch.  The DFA layer's chain weights_fc -> gather -> output_proj is
// serial and, for one frame, short; launched with programmatic stream serialisation, a kernel's
// CTAs may start (barrier init, tensor-memory allocation) while the kernel ahead of it in the
// stream is still finishing.  griddep_wait() returns once every kernel this one depends on has
// completed and its memory operations are visible, so each kernel calls it before its first
// global-memory access; griddep_launch_dependents() lets the kernel behind this one be scheduled
// (once every CTA of this launch has called it or exited).  For a launch without the attribute
// both are no-ops.
#ifndef S4D_PDL
#define S4D_PDL 1
#endif
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launches `kernel` on `stream`, with programmatic stream serialisation when `pdl` and S4D_PDL
// are set.  The callers ask for it on the launches of one frame (one wave of CTAs, where CTA
// start-up is a visible share of the kernel); a launch of many waves gains nothing from it.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = S4D_PDL && pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace s4d
