// Dense linears of the DFA layer on the 5th-generation tensor cores (tcgen05, TF32 operands,
// fp32 accumulation in tensor memory), with the layer's elementwise work fused around them.
//
//   weights_fc   logits = (inst + embed) . W_fc^T and learnable = inst . W_kps^T + b_kps in one
//                pass over 128-row tiles (model/deformable_feature_aggregation.py:651-677,719-798;
//                test/dfa_pcc.py:231-233,306-320).  The sum is formed in shared memory, stage by
//                stage, by the epilogue warps (idle during the K loop): one MMA per K step reads
//                it, instead of one for inst and one for embed.
//   output_proj  feats . W_o^T + b_o written straight into the residual output, the instance
//                feature copied beside it (cat) or added to it (add)
//                (model/deformable_feature_aggregation.py:934-950; test/dfa_pcc.py:299-304).
//
// Both kernels: one CTA per 128-row tile, 6 warps.
//   warp 0     TMA producer: A and B tiles of 16 fp32 (64-byte rows, 64-byte swizzle, zero
//              fill past the last row) into a 4-stage shared-memory ring;
//   warp 1     allocates the tensor-memory accumulator (128 lanes x N fp32 columns); one thread
//              issues tcgen05.mma (M 128, K 8, N <= 256 per instruction) and commits each stage
//              back to the producer;
//   warps 2-5  during the main loop: weights_fc adds each stage's inst tile into its embed tile
//              (the MMA issuer waits for that); output_proj copies the instance rows for the
//              residual cat.  After it: tcgen05.ld of their 32 TMEM lanes (warp
//              index mod 4), bias / residual in registers, the tile staged in shared memory
//              with the 128-byte swizzle and written by TMA bulk-tensor stores.
// Every barrier wait is bounded: after 2 s the CTA raises S4D_FLAG_WAIT_TIMEOUT, lets its copies
// and MMAs finish, frees tensor memory and returns without writing its outputs.
#include <cuda.h>

#include <mutex>

#include "params.cuh"

namespace s4d {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 16;  // fp32 per stage row: 64 bytes, one 64-byte swizzle span
constexpr int kThreads = 192;
constexpr int kStages = 4;
constexpr int kATile = kBM * kBK * 4;  // 8 KiB
constexpr int kStageChunk = 32 * 32 * 4;  // one 32x32 fp32 output box (4 KiB)
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

// ---- PTX wrappers ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits until the phase with `parity` has completed.  Returns false without waiting further
// once another role of the CTA has given up (abort_flag set), or after limit_ns, in which case it
// sets abort_flag itself.  With abort_flag == nullptr only the time limit applies.
//
// Two kinds of waits use it.  The pipeline waits (TMA producer on an empty stage, MMA issuer on a
// full stage, epilogue on the accumulator) pass the CTA's abort flag and the launch's limit
// (WfcParams / OprojParams::wait_limit_ns, 2 s unless a caller lowered it through
// s4d_set_tc_wait_limit_ns).  The teardown waits -- the producer's drain of the loads it issued
// and the MMA issuer's wait for the MMAs it issued -- pass no flag and always kWaitLimitNs: they
// are what guarantees that no copy is still landing in shared memory and no MMA still writing
// tensor memory when the CTA frees it and exits, whatever the pipeline waits decided.
__device__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                          unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_test(bar, parity)) return true;
  const unsigned long long t0 = now_ns();
  for (;;) {
    if (mbar_test(bar, parity)) return true;
    if (abort_flag != nullptr && *abort_flag) return false;
    if (now_ns() - t0 > limit_ns) {
      if (abort_flag != nullptr) *abort_flag = 1;
      return false;
    }
  }
}

// 2-D tiled TMA load of one box of `map` at (x, y), completion counted on `bar`.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// 2-D tiled TMA store of one box from shared memory to `map` at (x, y); rows and columns
// outside the map are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_le1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Generic-proxy shared-memory writes become visible to the async proxy (TMA, tensor cores).
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(cols) : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] . B[smem]^T, both K-major TF32, fp32 accumulate.
__device__ __forceinline__ void mma_tf32(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// Shared-memory matrix descriptor of a K-major tile of 64-byte rows stored with the 64-byte
// swizzle (what a TMA box of 16 fp32 x rows with CU_TENSOR_MAP_SWIZZLE_64B writes, from a
// 512-byte aligned base): start address >> 4 in bits 0-13; leading-dimension offset 16 B
// (not used by swizzled K-major layouts) in bits 16-29; 512 B between 8-row groups in bits
// 32-45; descriptor version 1 in bits 46-47; swizzle mode 4 (64 B) in bits 61-63.  Adding 2
// to the descriptor advances the start by 32 bytes, i.e. by the 8 fp32 of one MMA's K step.
__device__ __forceinline__ uint64_t sw64_desc(uint32_t saddr) {
  return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t(1) << 16) | (uint64_t(512 >> 4) << 32) | (uint64_t(1) << 46) |
         (uint64_t(4) << 61);
}

// Instruction descriptor of kind::tf32: D f32 (bits 4-5 = 1), A and B TF32 (bits 7-9 and
// 10-12 = 2), both K-major (bits 15, 16 = 0), N >> 3 in bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t tf32_idesc(int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(kBM >> 4) << 24);
}

// 32 consecutive accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- shared pieces of the two kernels ------------------------------------------------------

// First column of the kb-th K step a CTA loads.  Every CTA reads the same weight matrix; with
// S4D_TC_STAGGER_K each starts its K loop at a different step (blockIdx.x mod kbs), so that the
// CTAs of a wave do not all fetch the same weight tile from the same L2 lines at once.  The sum
// over K is the same up to the order of the fp32 additions, which is fixed per tile.
#ifndef S4D_TC_STAGGER_K
#define S4D_TC_STAGGER_K 1
#endif
__device__ __forceinline__ int k_column(int kb, int kbs) {
  if (!S4D_TC_STAGGER_K || kbs != 16) return kb * kBK;  // both kernels run K = 256: 16 steps
  const int k = kb + int(blockIdx.x & 15u);
  return (k >= 16 ? k - 16 : k) * kBK;
}

struct Ctl {
  uint64_t* bars;
  uint32_t* tmem_slot;
  volatile int* abort_flag;
};

// Barrier block after the stages: full[S], aux[S] (weights_fc: stage summed), empty[S], acc, then the TMEM slot and the
// abort flag.
template <int STAGE_BYTES>
__device__ __forceinline__ Ctl carve(unsigned char* smem) {
  Ctl c;
  c.bars = reinterpret_cast<uint64_t*>(smem + kStages * STAGE_BYTES);
  c.tmem_slot = reinterpret_cast<uint32_t*>(c.bars + 3 * kStages + 1);
  c.abort_flag = reinterpret_cast<volatile int*>(c.tmem_slot + 1);
  return c;
}

__device__ __forceinline__ unsigned char* aligned_smem(unsigned char* raw) {
  return reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
}

// Bytes of dynamic shared memory for a given stage size (1 KiB alignment slack + control).
constexpr size_t smem_bytes(int stage_bytes) { return size_t(kStages) * stage_bytes + 1024 + 8 * (3 * kStages + 1) + 16; }

// Writes 32 fp32 of this thread's row into a 32x32 staging box laid out as the 128-byte
// swizzled TMA box: 16-byte chunk j of row r lands at chunk j ^ (r & 7), so the 8 rows a
// quarter-warp writes hit 8 different bank groups.
__device__ __forceinline__ void stage_row(unsigned char* box, int r, const float (&f)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<float4*>(box + r * 128 + ((j ^ (r & 7)) << 4)) =
        make_float4(f[4 * j], f[4 * j + 1], f[4 * j + 2], f[4 * j + 3]);
}

// The epilogue warp `q` streams accumulator columns [0, ncols) of its 32 rows to columns
// [col0, col0 + ncols) of `map` (a 32x32-box, 128-byte swizzle store map) through two 4 KiB
// staging boxes at `stage`, adding bias[col0 + col] and, when res != null,
// res[row * res_ld + col0 + col].
__device__ __forceinline__ void store_columns(uint32_t tmem, int q, int lane, int64_t tile_row0, int col0, int ncols,
                                              const CUtensorMap* map, unsigned char* stage, const float* bias,
                                              const float* res, int64_t res_ld, int64_t rows) {
  const int64_t row = tile_row0 + q * 32 + lane;
  for (int c = 0; c < ncols / 32; ++c) {
    uint32_t v[32];
    tmem_ld32(tmem + (uint32_t(q * 32) << 16) + uint32_t(c * 32), v);
    float f[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(v[i]);
    if (bias != nullptr) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 b = __ldg(reinterpret_cast<const float4*>(bias + col0 + c * 32) + i);
        f[4 * i] += b.x, f[4 * i + 1] += b.y, f[4 * i + 2] += b.z, f[4 * i + 3] += b.w;
      }
    }
    if (res != nullptr && row < rows) {
      const float4* r4 = reinterpret_cast<const float4*>(res + row * res_ld + col0 + c * 32);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 r = ldg_nc_f4(r4 + i);
        f[4 * i] += r.x, f[4 * i + 1] += r.y, f[4 * i + 2] += r.z, f[4 * i + 3] += r.w;
      }
    }
    unsigned char* box = stage + (c & 1) * kStageChunk;
    if (lane == 0 && c >= 2) bulk_wait_read_le1();  // the store that last used this box has read it
    __syncwarp();
    stage_row(box, lane, f);
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(map, smem_u32(box), col0 + c * 32, int(tile_row0 + q * 32));
      bulk_commit();
    }
  }
  if (lane == 0) bulk_wait_all();
  __syncwarp();
}

// Common prologue: barrier init, TMEM allocation, hand-off of the TMEM address.
__device__ __forceinline__ uint32_t prologue(const Ctl& c, uint32_t cols, int aux_count) {
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    const uint32_t b0 = smem_u32(c.bars);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(b0 + 8 * s, 1);                                    // full: TMA bytes landed
      mbar_init(b0 + 8 * (kStages + s), aux_count > 0 ? aux_count : 1);  // aux: aux_count arrivals (0: unused)
      mbar_init(b0 + 8 * (2 * kStages + s), 1);                    // empty: MMAs of the stage done
    }
    mbar_init(b0 + 8 * (3 * kStages), 1);  // acc: accumulator complete
    *c.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(smem_u32(c.tmem_slot), cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  return *c.tmem_slot;
}

__device__ __forceinline__ void epilogue_teardown(const Ctl& c, uint32_t tmem, uint32_t cols, int32_t* error_flag) {
  tc_fence_before();
  __syncthreads();
  if ((threadIdx.x >> 5) == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, cols);
  }
  if (threadIdx.x == 0 && *c.abort_flag && error_flag != nullptr) atomicOr(error_flag, S4D_FLAG_WAIT_TIMEOUT);
}

// Producer drain: no copy may still be landing in shared memory when the CTA exits.
__device__ __forceinline__ void drain_loads(uint32_t full0, int issued) {
  for (int kb = issued > kStages ? issued - kStages : 0; kb < issued; ++kb)
    mbar_wait(full0 + 8 * (kb % kStages), (kb / kStages) & 1, nullptr);
}

// Warp-uniform wait for the accumulator (tcgen05.ld is warp-collective).
__device__ __forceinline__ bool wait_accumulator(const Ctl& c, uint32_t acc_bar, unsigned long long limit_ns) {
  const bool done = __all_sync(0xffffffffu, mbar_wait(acc_bar, 0, c.abort_flag, limit_ns));
  const int aborted = __shfl_sync(0xffffffffu, *c.abort_flag, 0);
  tc_fence_after();
  return done && !aborted;
}

// ---- weights_fc -----------------------------------------------------------------------------

template <int NW>
struct Wfc {
  static constexpr int kSplit = NW > 256 ? 2 : 1;  // MMAs per K step for the logits
  static constexpr int kNmma = NW / kSplit;
  static constexpr int kNL = 32;                     // learnable columns (one N-32 MMA)
  static constexpr int kBW = NW * kBK * 4;
  static constexpr int kBL = kNL * kBK * 4;
  static constexpr int kStage = 2 * kATile + kBW + kBL;  // inst, embed, W_fc, W_kps
  // tensor-memory columns: the logits and the learnable columns, rounded up to a power of 2
  static constexpr uint32_t kCols = NW + kNL <= 64 ? 64 : NW + kNL <= 128 ? 128 : NW + kNL <= 256 ? 256 : 512;
  static constexpr size_t kSmem = smem_bytes(kStage);
  static_assert(NW % 32 == 0 && kNmma % 16 == 0 && kNmma <= 256 && NW + kNL <= 512, "logit columns");
  static_assert(kBW % 512 == 0 && kStage % 1024 == 0 && (kNmma * kBK * 4) % 512 == 0, "swizzle alignment");
  static_assert(4 * 2 * kStageChunk <= kStages * kStage, "epilogue staging fits in the stages");
};

template <int NW>
__global__ void __launch_bounds__(kThreads, 1)
    weights_fc_kernel(const __grid_constant__ CUtensorMap map_inst, const __grid_constant__ CUtensorMap map_embed,
                      const __grid_constant__ CUtensorMap map_wfc, const __grid_constant__ CUtensorMap map_wkps,
                      const __grid_constant__ CUtensorMap map_logits, const WfcParams p) {
  using S = Wfc<NW>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = aligned_smem(smem_raw);
  const Ctl c = carve<S::kStage>(smem);
  // full[s]: the stage's TMA bytes landed; summed[s] (the aux slots): the 128 epilogue threads have
  // added its inst tile into its embed tile; empty[s]: its MMAs are done
  const uint32_t full0 = smem_u32(c.bars), summed0 = full0 + 8 * kStages, empty0 = full0 + 16 * kStages,
                 acc_bar = full0 + 24 * kStages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kbs = p.k / kBK;
  const int64_t row0 = int64_t(blockIdx.x) * kBM;
  // Column group: logits [col0, col0 + NW); the learnable columns ride with group 0.
  const int col0 = int(blockIdx.y) * NW;
  const bool learn = blockIdx.y == 0;
  const uint32_t tmem = prologue(c, S::kCols, kThreads - 64);
  griddep_wait();  // the kernels ahead of this one (which write inst, or read this launch's outputs) are done
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      int issued = 0;
      for (int kb = 0; kb < kbs; ++kb) {
        const int s = kb % kStages;
        if (kb >= kStages && !mbar_wait(empty0 + 8 * s, ((kb / kStages) - 1) & 1, c.abort_flag, p.wait_limit_ns)) break;
        const uint32_t st = smem_u32(smem + s * S::kStage), fb = full0 + 8 * s;
        const int kx = k_column(kb, kbs);
        mbar_expect_tx(fb, learn ? S::kStage : S::kStage - S::kBL);
        tma_load_2d(st, &map_inst, fb, kx, int(row0));
        tma_load_2d(st + kATile, &map_embed, fb, kx, int(row0));
#pragma unroll
        for (int j = 0; j < S::kSplit; ++j)
          tma_load_2d(st + 2 * kATile + j * S::kNmma * kBK * 4, &map_wfc, fb, kx, col0 + j * S::kNmma);
        if (learn) tma_load_2d(st + 2 * kATile + S::kBW, &map_wkps, fb, kx, 0);
        issued = kb + 1;
      }
      drain_loads(full0, issued);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      for (int kb = 0; kb < kbs; ++kb) {
        const int s = kb % kStages;
        if (!mbar_wait(summed0 + 8 * s, (kb / kStages) & 1, c.abort_flag, p.wait_limit_ns)) break;
        tc_fence_after();
        const uint32_t st = smem_u32(smem + s * S::kStage);
        const uint64_t a_inst = sw64_desc(st), a_sum = sw64_desc(st + kATile);
        const uint64_t b_kps = sw64_desc(st + 2 * kATile + S::kBW);
#pragma unroll
        for (int k = 0; k < kBK / 8; ++k) {
          const uint32_t acc = (kb | k) != 0;
#pragma unroll
          for (int j = 0; j < S::kSplit; ++j) {
            const uint64_t b = sw64_desc(st + 2 * kATile + j * S::kNmma * kBK * 4) + 2 * k;
            mma_tf32(tmem + j * S::kNmma, a_sum + 2 * k, b, tf32_idesc(S::kNmma), acc);
          }
          if (learn) mma_tf32(tmem + NW, a_inst + 2 * k, b_kps + 2 * k, tf32_idesc(S::kNL), acc);
        }
        mma_commit(empty0 + 8 * s);
      }
      mma_commit(acc_bar);  // also on the abort path: nothing may run once tensor memory is freed
      mbar_wait(acc_bar, 0, nullptr);
    }
  } else {
    // K loop: (inst + embed) of every stage, in place in its embed tile.  The two tiles come from
    // the same kind of tensor map (box, swizzle, zero fill), so element i of one lies at the
    // same byte offset as element i of the other and a flat add over the bytes pairs them up.
    const int et = threadIdx.x - 64;
    for (int kb = 0; kb < kbs; ++kb) {
      const int s = kb % kStages;
      if (!mbar_wait(full0 + 8 * s, (kb / kStages) & 1, c.abort_flag, p.wait_limit_ns)) break;
      const float4* a4 = reinterpret_cast<const float4*>(smem + s * S::kStage);
      float4* e4 = reinterpret_cast<float4*>(smem + s * S::kStage + kATile);
#pragma unroll
      for (int j = 0; j < kATile / 16 / (kThreads - 64); ++j) {
        const int x = et + j * (kThreads - 64);
        const float4 a = a4[x];
        float4 e = e4[x];
        e.x = a.x + e.x, e.y = a.y + e.y, e.z = a.z + e.z, e.w = a.w + e.w;
        e4[x] = e;
      }
      fence_proxy_async();  // the tensor cores read the sum through the async proxy
      mbar_arrive(summed0 + 8 * s);
    }
    // Epilogue: logits through TMA stores, learnable columns (not 16-byte rows) by plain stores.
    const int q = warp & 3;
    if (wait_accumulator(c, acc_bar, p.wait_limit_ns)) {
      store_columns(tmem, q, lane, row0, col0, NW, &map_logits, smem + q * 2 * kStageChunk, nullptr, nullptr, 0,
                    p.rows);
      uint32_t v[32];
      if (learn) tmem_ld32(tmem + (uint32_t(q * 32) << 16) + uint32_t(NW), v);
      const int64_t row = row0 + q * 32 + lane;
      if (learn && row < p.rows && p.n_learn > 0) {
        float* dst = p.learnable + row * p.n_learn;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < p.n_learn) dst[i] = __uint_as_float(v[i]) + (p.learn_bias != nullptr ? __ldg(p.learn_bias + i) : 0.f);
      }
    }
  }
  epilogue_teardown(c, tmem, S::kCols, p.error_flag);
}

// ---- output_proj ----------------------------------------------------------------------------

// A CTA computes output columns [col0, col0 + NO) of a 128-row tile (NO = 256: all of them;
// fewer when a launch has few row tiles, so that more SMs share it).
template <int NO, bool TWO = false>
struct Oproj {
  static constexpr int kK = 256;  // input features (embed_dims)
  static constexpr int kN = NO;
  static constexpr int kA = TWO ? 2 : 1;                     // feature sources summed by the MMAs
  static constexpr int kStage = kA * kATile + kN * kBK * 4;  // feats tile(s), W_o tile
  static constexpr uint32_t kCols = NO <= 32 ? 32 : NO <= 64 ? 64 : NO <= 128 ? 128 : 256;
  static constexpr size_t kSmem = smem_bytes(kStage);
  static_assert(NO % 32 == 0 && NO <= 256 && kStage % 1024 == 0, "swizzle alignment");
  static_assert(4 * 2 * kStageChunk <= kStages * kStage, "epilogue staging fits in the stages");
};

// TWO: out = (feat + feat2) . W^T + ... with feat2 another [rows, k] source (the other camera
// half's partial sums, which may live on a peer GPU): both tiles of a K step are multiplied by the
// same W tile into one accumulator, so the sum is never formed in memory.
template <int NO, bool TWO = false>
__global__ void __launch_bounds__(kThreads, 2)
    output_proj_kernel(const __grid_constant__ CUtensorMap map_feat, const __grid_constant__ CUtensorMap map_feat2,
                       const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_out,
                       const OprojParams p) {
  using S = Oproj<NO, TWO>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = aligned_smem(smem_raw);
  const Ctl c = carve<S::kStage>(smem);
  const uint32_t full0 = smem_u32(c.bars), empty0 = full0 + 16 * kStages, acc_bar = full0 + 24 * kStages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kbs = S::kK / kBK;
  const int64_t row0 = int64_t(blockIdx.x) * kBM;
  const int col0 = int(blockIdx.y) * NO;
  const uint32_t tmem = prologue(c, S::kCols, 0);
  griddep_wait();  // the gather that wrote the features (and any reader of this launch's outputs) is done
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < kbs; ++kb) {
        const int s = kb % kStages;
        if (kb >= kStages && !mbar_wait(empty0 + 8 * s, ((kb / kStages) - 1) & 1, c.abort_flag, p.wait_limit_ns)) break;
        const uint32_t st = smem_u32(smem + s * S::kStage), fb = full0 + 8 * s;
        const int kx = k_column(kb, kbs);
        mbar_expect_tx(fb, S::kStage);
        tma_load_2d(st, &map_feat, fb, kx, int(p.feat_row0 + row0));
        if (TWO) tma_load_2d(st + kATile, &map_feat2, fb, kx, int(p.feat_row0 + row0));
        tma_load_2d(st + S::kA * kATile, &map_w, fb, kx, col0);
        issued = kb + 1;
      }
      drain_loads(full0, issued);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      for (int kb = 0; kb < kbs; ++kb) {
        const int s = kb % kStages;
        if (!mbar_wait(full0 + 8 * s, (kb / kStages) & 1, c.abort_flag, p.wait_limit_ns)) break;
        tc_fence_after();
        const uint32_t st = smem_u32(smem + s * S::kStage);
        const uint64_t a = sw64_desc(st), a2 = sw64_desc(st + kATile), b = sw64_desc(st + S::kA * kATile);
#pragma unroll
        for (int k = 0; k < kBK / 8; ++k) {
          mma_tf32(tmem, a + 2 * k, b + 2 * k, tf32_idesc(S::kN), (kb | k) != 0);
          if (TWO) mma_tf32(tmem, a2 + 2 * k, b + 2 * k, tf32_idesc(S::kN), 1);
        }
        mma_commit(empty0 + 8 * s);
      }
      mma_commit(acc_bar);
      mbar_wait(acc_bar, 0, nullptr);
    }
  } else {
    const int q = warp & 3;
    if (p.res_mode == S4D_RESIDUAL_CAT) {
      // The residual half of the output (this CTA's columns of it) is a plain copy: done while
      // the tensor cores run, 8 float4 per lane in flight per step, consecutive lanes on
      // consecutive 16-byte pieces of a row.
      constexpr int kF4 = NO / 4;          // float4 per row of this CTA's columns
      constexpr int kTotal = 32 * kF4;     // ... over the warp's 32 rows
      const int64_t r_begin = row0 + q * 32;
      for (int base = 0; base < kTotal; base += 8 * 32) {
        float4 buf[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int idx = base + i * 32 + lane;
          const int64_t r = r_begin + idx / kF4;
          if (idx < kTotal && r < p.rows)
            buf[i] = ldg_nc_f4(reinterpret_cast<const float4*>(p.res + r * p.res_ld + col0) + idx % kF4);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int idx = base + i * 32 + lane;
          const int64_t r = r_begin + idx / kF4;
          if (idx < kTotal && r < p.rows)
            reinterpret_cast<float4*>(p.out + r * p.out_ld + S::kK + col0)[idx % kF4] = buf[i];
        }
      }
    }
    if (wait_accumulator(c, acc_bar, p.wait_limit_ns))
      store_columns(tmem, q, lane, row0, col0, NO, &map_out, smem + q * 2 * kStageChunk, p.bias,
                    p.res_mode == S4D_RESIDUAL_ADD ? p.res : nullptr, p.res_ld, p.rows);
  }
  epilogue_teardown(c, tmem, S::kCols, p.error_flag);
}

// ---- host side ----------------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

// Tensor map of an fp32 row-major matrix [rows, cols] with row stride ld (floats), zero fill
// outside the matrix: operand loads use boxes of kBK (16) columns x box_rows rows with the
// 64-byte swizzle; `store` maps (the epilogue's) boxes of 32 columns with the 128-byte swizzle.
int make_map(CUtensorMap* map, const float* base, int64_t rows, int64_t cols, int64_t ld, int box_rows,
             bool store = false) {
  EncodeTiledFn fn = encode_tiled();
  if (fn == nullptr) return fail(S4D_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the CUDA driver");
  const cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(ld) * 4};
  const cuuint32_t box[2] = {uint32_t(store ? 32 : kBK), uint32_t(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, store ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (CUresult %d) for a [%lld, %lld] matrix, ld %lld", int(r),
              (long long)rows, (long long)cols, (long long)ld);
    return S4D_ERR_CUDA;
  }
  return S4D_OK;
}

// The dynamic shared-memory limit of `kernel`, set once per device (the attribute persists in the
// context); `done` is the caller's per-instantiation record of the devices already set.
template <typename K>
int set_smem(K kernel, size_t bytes, const char* what, bool (&done)[64]) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
  if (dev >= 0 && dev < 64 && done[dev]) return S4D_OK;
  const int st = cuda_check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes)), what);
  if (st == S4D_OK && dev >= 0 && dev < 64) done[dev] = true;
  return st;
}

// Column groups for launches of few row tiles (1 = always whole rows per CTA).
#ifndef S4D_TC_COLUMN_GROUPS
#define S4D_TC_COLUMN_GROUPS 1
#endif

// SMs of the current device (148 on B200 if the query fails), cached per device.
int sm_count() {
  static int cache[64] = {};
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 148;
  }
  if (dev >= 0 && dev < 64 && cache[dev] > 0) return cache[dev];
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
    cudaGetLastError();
    return 148;
  }
  if (dev >= 0 && dev < 64) cache[dev] = sms;
  return sms;
}

// Column groups per row tile of a launch with `tiles` row tiles: the most of `choices` (widest
// first) that still fits the launch in one wave on the SMs, so that a launch of few rows (bs = 1:
// 8 tiles) spreads over many SMs; launches of more tiles than SMs keep whole rows per CTA.
int column_groups(int64_t tiles, std::initializer_list<int> choices) {
  const int64_t sms = sm_count();
  int best = 1;
  for (int g : choices)
    if (tiles * g <= sms && g > best) best = g;
  return best;
}

template <int NW>
int launch_weights_fc_cols(const WfcParams& p, cudaStream_t stream, int groups) {
  using S = Wfc<NW>;
  CUtensorMap mi, me, mw, mk, mo;
  int st = make_map(&mi, p.inst, p.rows, p.k, p.inst_ld, kBM);
  if (st == S4D_OK) st = make_map(&me, p.embed, p.rows, p.k, p.embed_ld, kBM);
  if (st == S4D_OK) st = make_map(&mw, p.w_fc, p.n_logits, p.k, p.k, S::kNmma);
  if (st == S4D_OK) st = make_map(&mk, p.w_kps, p.n_learn > 0 ? p.n_learn : 1, p.k, p.k, S::kNL);
  if (st == S4D_OK) st = make_map(&mo, p.logits, p.rows, p.n_logits, p.n_logits, 32, true);
  static bool smem_set[64] = {};
  if (st == S4D_OK) st = set_smem(weights_fc_kernel<NW>, S::kSmem, "cudaFuncSetAttribute(weights_fc_kernel)", smem_set);
  if (st != S4D_OK) return st;
  const dim3 grid(unsigned((p.rows + kBM - 1) / kBM), unsigned(groups));
  return cuda_check(
      launch_pdl(groups > 1, weights_fc_kernel<NW>, grid, dim3(kThreads), S::kSmem, stream, mi, me, mw, mk, mo, p),
      "weights_fc_kernel launch");
}

template <int NO, bool TWO>
int launch_output_proj_cols(const OprojParams& p, cudaStream_t stream, int groups) {
  using S = Oproj<NO, TWO>;
  CUtensorMap mf, mf2, mw, mo;
  const int64_t feat_rows = p.feat_rows > 0 ? p.feat_rows : p.rows;
  int st = make_map(&mf, p.feat, feat_rows, p.k, p.k, kBM);
  if (st == S4D_OK) st = TWO ? make_map(&mf2, p.feat2, feat_rows, p.k, p.k, kBM) : make_map(&mf2, p.feat, feat_rows, p.k, p.k, kBM);
  if (st == S4D_OK) st = make_map(&mw, p.w, p.k, p.k, p.k, NO);
  if (st == S4D_OK) st = make_map(&mo, p.out, p.rows, p.k, p.out_ld, 32, true);
  static bool smem_set[64] = {};
  if (st == S4D_OK)
    st = set_smem(output_proj_kernel<NO, TWO>, S::kSmem, "cudaFuncSetAttribute(output_proj_kernel)", smem_set);
  if (st != S4D_OK) return st;
  const dim3 grid(unsigned((p.rows + kBM - 1) / kBM), unsigned(groups));
  return cuda_check(
      launch_pdl(groups > 1, output_proj_kernel<NO, TWO>, grid, dim3(kThreads), S::kSmem, stream, mf, mf2, mw, mo, p),
      "output_proj_kernel launch");
}

}  // namespace

int launch_weights_fc(const WfcParams& p, cudaStream_t stream) {
  if (p.rows <= 0) return S4D_OK;
  if (p.n_logits != 416 || p.k != 256 || p.n_learn > 32)
    return fail(S4D_ERR_UNSUPPORTED_SHAPE, "weights_fc: implemented for 416 logit columns, embed_dims 256, "
                                           "<= 32 learnable columns");
  // 416 logit columns in 1 or 13 groups (the epilogue stores 32-column boxes: 416 = 13 x 32)
  const int groups = S4D_TC_COLUMN_GROUPS ? column_groups((p.rows + kBM - 1) / kBM, {13}) : 1;
  if (groups == 13) return launch_weights_fc_cols<32>(p, stream, 13);
  return launch_weights_fc_cols<416>(p, stream, 1);
}

int launch_output_proj(const OprojParams& p, cudaStream_t stream) {
  if (p.rows <= 0) return S4D_OK;
  if (p.k != 256) return fail(S4D_ERR_UNSUPPORTED_SHAPE, "output_proj: implemented for embed_dims 256");
  // 256 output columns in 1, 2 (128 each) or 8 (32 each) groups
  const int groups = S4D_TC_COLUMN_GROUPS ? column_groups((p.rows + kBM - 1) / kBM, {2, 8}) : 1;
  if (p.feat2 != nullptr) {
    if (groups == 8) return launch_output_proj_cols<32, true>(p, stream, 8);
    if (groups == 2) return launch_output_proj_cols<128, true>(p, stream, 2);
    return launch_output_proj_cols<256, true>(p, stream, 1);
  }
  if (groups == 8) return launch_output_proj_cols<32, false>(p, stream, 8);
  if (groups == 2) return launch_output_proj_cols<128, false>(p, stream, 2);
  return launch_output_proj_cols<256, false>(p, stream, 1);
}

}  // namespace s4d
