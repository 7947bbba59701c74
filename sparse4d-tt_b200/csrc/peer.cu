// Peer memory between the GPUs of a camera group: CUDA IPC export / import of device buffers and
// a bounded flag exchange over NVLink.
//
// The camera-sharded DFA sums the per-camera-half partial features of two GPUs.  Instead of an
// NCCL reduce-scatter followed by a separate output_proj pass, each GPU maps the other's
// partial-sum buffer (s4d_ipc_export / s4d_ipc_open), the two GPUs raise a flag in each other's
// memory once their gather has finished (s4d_peer_signal_wait), and output_proj reads its own
// rows of both partial sums -- the peer's over NVLink -- and adds them inside its tensor-core
// accumulation (s4d_dfa_output_proj_sum).  The reference combines the same partial sums with a
// mesh all-reduce (model/deformable_feature_aggregation.py:925-931).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace s4d {
namespace {

using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(f);
  });
  return fn;
}

constexpr int kMaxPeers = 8;

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

struct SignalParams {
  uint32_t* own;               // [world] slots of this GPU, slot r written by rank r
  uint32_t* peer[kMaxPeers];   // rank r's slot array (mapped from its GPU); this rank's entry unused
  int rank, world;
  uint32_t epoch;              // used when counter is null
  uint32_t* counter;           // or: epoch = *counter + advance, read when the launch runs
  int advance;                 // 0 or 1; with 1 the launch stores the new epoch back in *counter
  unsigned long long limit_ns;
  int32_t* error_flag;
};

__device__ __forceinline__ unsigned long long timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void store_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One thread per peer: publish `epoch` in the peer's slot for this rank, then wait until the
// peer has published an epoch at least as new in this GPU's slot for it.  Everything the earlier
// launches of the stream wrote (the gather's partial sums) is visible at system scope before the
// peer can see the epoch; the launches after this one see the peer's writes that preceded its
// epoch.  The wait gives up after limit_ns, sets S4D_FLAG_PEER_TIMEOUT and returns.
__global__ void peer_signal_wait_kernel(const SignalParams p) {
  const int r = int(threadIdx.x);
  // a device-side epoch (counter) lets a CUDA graph replay the launch: every replay advances it
  const uint32_t epoch = p.counter != nullptr ? *p.counter + uint32_t(p.advance) : p.epoch;
  __syncthreads();  // every thread has read the counter
  if (r == 0 && p.counter != nullptr && p.advance) *p.counter = epoch;
  if (r >= p.world || r == p.rank) return;
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  store_release_sys(p.peer[r] + p.rank, epoch);
  const unsigned long long t0 = timer_ns();
  while (int32_t(load_acquire_sys(p.own + r) - epoch) < 0) {
    if (timer_ns() - t0 > p.limit_ns) {
      if (p.error_flag != nullptr) atomicOr(p.error_flag, S4D_FLAG_PEER_TIMEOUT);
      return;
    }
    __nanosleep(100);
  }
}

}  // namespace
}  // namespace s4d

using namespace s4d;

extern "C" {

size_t s4d_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int s4d_ipc_export(const void* ptr, void* handle, uint64_t* offset) {
  set_error("%s", "");
  if (ptr == nullptr || handle == nullptr || offset == nullptr) return fail(S4D_ERR_INVALID_ARG, "s4d_ipc_export: null pointer");
  AddressRangeFn range = address_range();
  if (range == nullptr) return fail(S4D_ERR_CUDA, "s4d_ipc_export: cuMemGetAddressRange is not available from the CUDA driver");
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = range(&base, &size, CUdeviceptr(reinterpret_cast<uintptr_t>(ptr)));
  if (r != CUDA_SUCCESS) {
    set_error("s4d_ipc_export: cuMemGetAddressRange failed (CUresult %d): not device memory of this context", int(r));
    return S4D_ERR_INVALID_ARG;
  }
  cudaIpcMemHandle_t h;
  const int st = cuda_check(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(uintptr_t(base))),
                            "s4d_ipc_export: cudaIpcGetMemHandle (the allocation must come from cudaMalloc)");
  if (st != S4D_OK) return st;
  std::memcpy(handle, &h, sizeof(h));
  *offset = uint64_t(reinterpret_cast<uintptr_t>(ptr) - uintptr_t(base));
  return S4D_OK;
}

int s4d_ipc_open(const void* handle, void** base) {
  set_error("%s", "");
  if (handle == nullptr || base == nullptr) return fail(S4D_ERR_INVALID_ARG, "s4d_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *base = nullptr;
  return cuda_check(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess), "s4d_ipc_open: cudaIpcOpenMemHandle");
}

int s4d_ipc_close(void* base) {
  set_error("%s", "");
  if (base == nullptr) return fail(S4D_ERR_INVALID_ARG, "s4d_ipc_close: null pointer");
  return cuda_check(cudaIpcCloseMemHandle(base), "s4d_ipc_close: cudaIpcCloseMemHandle");
}

}  // extern "C"

namespace {

int signal_wait(const char* fn, uint32_t* own_slots, uint32_t* const* peer_slots, int rank, int world, uint32_t epoch,
                uint32_t* counter, int advance, uint64_t limit_ns, int32_t* error_flag, void* stream) {
  char msg[128];
  auto bad = [&](int status, const char* what) {
    snprintf(msg, sizeof(msg), "%s: %s", fn, what);
    return fail(status, msg);
  };
  if (world < 1 || world > kMaxPeers) return bad(S4D_ERR_UNSUPPORTED_SHAPE, "world must be 1..8");
  if (rank < 0 || rank >= world) return bad(S4D_ERR_INVALID_ARG, "rank outside [0, world)");
  if (own_slots == nullptr || peer_slots == nullptr) return bad(S4D_ERR_INVALID_ARG, "null pointer");
  if (!aligned(own_slots, 4)) return bad(S4D_ERR_INVALID_ARG, "misaligned slots");
  if (advance != 0 && advance != 1) return bad(S4D_ERR_INVALID_ARG, "advance must be 0 or 1");
  if (counter != nullptr && !aligned(counter, 4)) return bad(S4D_ERR_INVALID_ARG, "misaligned epoch counter");
  SignalParams p{};
  p.own = own_slots;
  for (int r = 0; r < world; ++r) {
    if (r == rank) continue;
    if (peer_slots[r] == nullptr || !aligned(peer_slots[r], 4))
      return bad(S4D_ERR_INVALID_ARG, "null or misaligned peer slots");
    p.peer[r] = peer_slots[r];
  }
  if (world == 1 && (counter == nullptr || !advance)) return S4D_OK;
  p.rank = rank;
  p.world = world;
  p.epoch = epoch;
  p.counter = counter;
  p.advance = advance;
  p.limit_ns = limit_ns;
  p.error_flag = error_flag;
  peer_signal_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return cuda_check(cudaGetLastError(), "peer_signal_wait_kernel launch");
}

}  // namespace

extern "C" {

int s4d_peer_signal_wait(uint32_t* own_slots, uint32_t* const* peer_slots, int rank, int world, uint32_t epoch,
                         uint64_t limit_ns, int32_t* error_flag, void* stream) {
  set_error("%s", "");
  return signal_wait("s4d_peer_signal_wait", own_slots, peer_slots, rank, world, epoch, nullptr, 0, limit_ns,
                     error_flag, stream);
}

int s4d_peer_signal_wait_counter(uint32_t* own_slots, uint32_t* const* peer_slots, int rank, int world,
                                 uint32_t* epoch_counter, int advance, uint64_t limit_ns, int32_t* error_flag,
                                 void* stream) {
  set_error("%s", "");
  if (epoch_counter == nullptr) return fail(S4D_ERR_INVALID_ARG, "s4d_peer_signal_wait_counter: null epoch counter");
  return signal_wait("s4d_peer_signal_wait_counter", own_slots, peer_slots, rank, world, 0, epoch_counter, advance,
                     limit_ns, error_flag, stream);
}

}  // extern "C"
