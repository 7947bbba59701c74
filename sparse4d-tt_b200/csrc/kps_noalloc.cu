// s4d_kps_project_noalloc: the keypoint projection + visibility compaction of s4d_kps_project
// for callers that cannot allocate device memory.
//
// Who needs it: a host program that drives the library through a plain FFI (Go, Java, Rust,
// a C runtime) often has no CUDA allocator of its own, and a process that runs under a fixed
// device-memory budget, or a real-time loop that forbids allocation once it has started, must
// not call cudaMalloc per frame either.  s4d_kps_project needs a caller-provided workspace
// whenever it compacts the visible indices; this entry point supplies that workspace from a
// fixed array compiled into the library instead, so the caller only passes its inputs and
// outputs.
//
// The scratch array (kScratchBytes, 528 KiB) lives in this file as a static __device__ array:
// every GPU that loads the library holds it until the process exits.  Host code cannot use the
// array's name as a device address, so every call looks the address up with
// cudaGetSymbolAddress on the current device.  Nothing is cached between calls, so a device
// reset or a new primary context between calls cannot leave a stale address behind.  The
// first call in a context may load the library's device code there (lazy module loading);
// make that first call before any stream capture.  All calls share the one array and it keeps
// the previous call's contents; nothing in it has to start at zero, because the projection
// kernel writes every count and ballot word the compaction kernel then reads.  Two calls that
// overlap on the GPU (different streams, or different host threads without ordering) race on
// the array.
#include "params.cuh"

namespace s4d {
namespace {

// Largest bs * A * Ncam * P accepted: 4,194,304 elements (e.g. 32 frames x 900 anchors x 6
// cameras x 13 points = 2,246,400).  The compaction needs one count per 1024 elements (256-byte
// aligned block) plus one 32-bit ballot word per 32 elements.
constexpr int64_t kMaxElements = (int64_t)1 << 22;
constexpr size_t kBlocks = (size_t)((kMaxElements + 1023) / 1024);
constexpr size_t kScratchBytes = ((kBlocks * sizeof(int32_t) + 255) & ~(size_t)255) + kBlocks * 32 * sizeof(uint32_t);

static __device__ __align__(256) unsigned char g_kps_scratch[kScratchBytes];

// Device address of g_kps_scratch in the current device's context.
int scratch_address(void** out) {
  void* p = nullptr;
  const int st = cuda_check(cudaGetSymbolAddress(&p, g_kps_scratch), "s4d_kps_project_noalloc: cudaGetSymbolAddress");
  if (st) return st;
  *out = p;
  return S4D_OK;
}

}  // namespace
}  // namespace s4d

using namespace s4d;

extern "C" int s4d_kps_project_noalloc(const float* anchor, int64_t anchor_dim, const float* fix_scale,
                                       int64_t num_fix, const float* learnable, int64_t num_learnable,
                                       const float* projection_mat, const float* image_wh, int64_t bs,
                                       int64_t num_anchor, int64_t num_cams, int layout, float* key_points,
                                       float* sample_location, uint8_t* depth_mask, int32_t* visible_idx,
                                       int32_t* visible_count, void* stream) {
  set_error("%s", "");
  if (bs < 0 || num_anchor < 0 || num_cams < 0 || num_fix < 0 || num_learnable < 0)
    return fail(S4D_ERR_INVALID_ARG, "s4d_kps_project_noalloc: negative size");
  if (num_fix > 64 || num_learnable > 64)  // s4d_kps_project takes at most 64 keypoints per anchor
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "s4d_kps_project_noalloc: at most 64 keypoints per anchor");
  int64_t total = 0;
  if (!size_product({bs, num_anchor, num_cams, num_fix + num_learnable}, kMaxElements + 1, &total)) {
    set_error("s4d_kps_project_noalloc: bs*A*Ncam*P exceeds the built-in scratch limit of %lld elements; "
              "use s4d_kps_project with a workspace",
              (long long)kMaxElements);
    return S4D_ERR_UNSUPPORTED_SHAPE;
  }
  void* scratch = nullptr;
  int st = scratch_address(&scratch);
  if (st) return st;
  return s4d_kps_project(anchor, anchor_dim, fix_scale, num_fix, learnable, num_learnable, projection_mat, image_wh,
                         bs, num_anchor, num_cams, layout, key_points, sample_location, depth_mask, visible_idx,
                         visible_count, scratch, kScratchBytes, stream);
}
