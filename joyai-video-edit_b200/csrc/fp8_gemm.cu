// FP8 (e4m3) row/column-scaled GEMM on the 5th-generation tensor cores.
//
//   D[m, n] = out( scale_a[m] * (sum_k A[m, k] * B[k, n]) * scale_b[n] (+ bias[n]) )
//
// Replaces joyomni_ops::fp8_scaled_mm (joyomni_ops/csrc/fp8_gemm.cu:1450-1546),
// whose sm100 path is a CUTLASS collective on 2x2x1 thread-block clusters
// (:1015-1159).  This kernel is written directly against the sm_100a
// instructions; every CTA loads its own operand tiles (no cross-CTA broadcast):
//
//   * CTA pairs (fp8_gemm_pair_kernel, below) for M > 128: 256 x 256 tiles per
//     pair of SMs with tcgen05.mma.cta_group::2; the single-CTA kernel here
//     takes M <= 128;
//   * persistent: one CTA per SM walks output tiles of 128 x 256;
//   * warp 0, one lane: TMA producer.  A tile 128 x 128 B and B tile 256 x 128 B
//     per k-block (128-byte swizzle, K-major), kStages-deep mbarrier ring;
//   * warp 1, one lane: issues tcgen05.mma.cta_group::1.kind::f8f6f4
//     (128 x 256 x 32 per instruction, fp32 accumulator in tensor memory) and
//     tcgen05.commit to release smem stages / publish finished accumulators;
//     warp 1 also owns the 512-column TMEM allocation (two 256-column
//     accumulators, so the epilogue of tile i overlaps the mainloop of tile i+1);
//   * warps 2-5: epilogue.  tcgen05.ld 32 lanes x 32 columns at a time, apply
//     the EVT order of the reference ((acc * sB) * sA (+ bias), fp32), round to
//     bf16/fp16 and store 64 contiguous bytes per thread.
//
// Every mbarrier wait is bounded (kWaitNs of wall time, pipeline.cuh); on
// expiry the kernel records the fault in the per-device counter (read by
// jo_device_fault_count), stops issuing work, drains its own TMA copies, frees
// its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "pipeline.cuh"
#include "quant.cuh"

namespace jo {
namespace {

constexpr int kBM = 128;       // UMMA M (one CTA)
constexpr int kBN = 256;       // UMMA N
constexpr int kBK = 128;       // bytes of K per stage = one 128-byte swizzle row
constexpr int kUmmaK = 32;     // K per tcgen05.mma kind::f8f6f4
constexpr int kStages = 4;
constexpr int kThreads = 192;  // 6 warps
constexpr int kTmemCols = 512;  // 2 accumulators x 256 fp32 columns
constexpr int kStageA = kBM * kBK;  // 16 KB
constexpr int kStageB = kBN * kBK;  // 32 KB
constexpr int kSmemBytes = kStages * (kStageA + kStageB) + 1024 /*align*/ + 256 /*barriers*/;

// ------------------------------------------------------------------ PTX helpers
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
// D(tmem) (+)= A(smem) * B(smem)^T, both K-major
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, 8-row
// groups 1024 B apart (SBO), LBO unused (1), sm100 descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;              // leading byte offset (ignored for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;    // stride byte offset
  d |= (uint64_t)1 << 46;              // descriptor version (sm100)
  d |= (uint64_t)2 << 61;              // SWIZZLE_128B
  return d;
}

// Instruction descriptor: e4m3 x e4m3 -> f32, both K-major, M = 128, N = 256.
constexpr uint32_t kIdesc = (1u << 4)                       // D format f32
                            | (0u << 7) | (0u << 10)          // A, B: e4m3
                            | ((uint32_t)(kBN >> 3) << 17)    // N >> 3
                            | ((uint32_t)(kBM >> 4) << 24);   // M >> 4

struct GemmArgs {
  void* d;
  int64_t ldd;
  const float* sa;
  const float* sb;
  const void* bias;
  const void* res;   // kEpiResid: residual [M, N] (row stride ldr), same dtype as D
  int64_t ldr;
  const void* gate;  // kEpiResid: gate [N], same dtype as D
  uint32_t* amax;    // kEpiGelu: per-row max |GELU| as 16-bit magnitude bits (zeroed before)
  int m, n, k;
  int tiles_m, tiles_n;
  unsigned int* fault;
};

// Epilogue variants: + bias[n]; gated residual D = res + gate[n] * (GEMM result)
// (torch.addcmul(res, x, gate) of sgl_fused_ops.py:302-305 applied to the fp32
// result, dit.py:536-538) instead of rounding the product to D's dtype first;
// GELU-tanh of the rounded result (the MLP's fc1 -> GELU, dit.py:508-513) with
// a per-row running max of |GELU| for the per-token FP8 quantisation that
// follows.
enum GemmEpi { kEpiBias = 1, kEpiResid = 2, kEpiGelu = 4 };

template <typename OutT>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  return pack_bf16x2(a, b);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  return pack_f16x2(a, b);
}

// Epilogue of one thread's 32 accumulator columns [n0, n0 + 32) of its row:
// (acc * sB) * sA (+ bias) in fp32, then either the gated residual or, for
// kEpiGelu, the rounding to OutT that the Linear's output holds, GELU-tanh of
// that value rounded to OutT again (the elementwise kernel's arithmetic) and a
// running |GELU| maximum; stored 16 bytes at a time.
template <typename OutT, int kEpi>
__device__ __forceinline__ void epi_chunk(const uint32_t* r, int n0, const GemmArgs& args, float s_a, bool row_ok,
                                          OutT* drow, const OutT* rrow, uint32_t& amax16) {
  constexpr bool kBias = (kEpi & kEpiBias) != 0, kResid = (kEpi & kEpiResid) != 0;
  constexpr bool kGelu = (kEpi & kEpiGelu) != 0;
  const OutT* bias = reinterpret_cast<const OutT*>(args.bias);
  const OutT* gate = reinterpret_cast<const OutT*>(args.gate);
#pragma unroll
  for (int g = 0; g < 4; ++g) {  // 8 columns per 16-byte store
    const int ng = n0 + g * 8;
    if (ng >= args.n) break;
    const float4 sb0 = __ldg(reinterpret_cast<const float4*>(args.sb + ng));
    const float4 sb1 = __ldg(reinterpret_cast<const float4*>(args.sb + ng + 4));
    const float sb[8] = {sb0.x, sb0.y, sb0.z, sb0.w, sb1.x, sb1.y, sb1.z, sb1.w};
    float bv[8];
    if constexpr (kBias) {
      float t[8];
      Elt<OutT>::unpack(__ldg(reinterpret_cast<const uint4*>(bias + ng)), t);
#pragma unroll
      for (int e = 0; e < 8; ++e) bv[e] = t[e];
    }
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float t = __uint_as_float(r[g * 8 + e]) * sb[e];
      o[e] = kBias ? fmaf(s_a, t, bv[e]) : s_a * t;
    }
    if (row_ok) {
      if constexpr (kResid) {
        float rv[8], gv[8];
        // plain (coherent) load: D may alias the residual
        Elt<OutT>::unpack(*reinterpret_cast<const uint4*>(rrow + ng), rv);
        Elt<OutT>::unpack(__ldg(reinterpret_cast<const uint4*>(gate + ng)), gv);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = fmaf(gv[e], o[e], rv[e]);
      }
      uint4 v = make_uint4(pack2<OutT>(o[0], o[1]), pack2<OutT>(o[2], o[3]), pack2<OutT>(o[4], o[5]),
                           pack2<OutT>(o[6], o[7]));
      if constexpr (kGelu) {
        v = gelu_vec<OutT>(v);
        amax16 = absmax16x2<OutT>(absmax16x2<OutT>(amax16, v.x), v.y);
        amax16 = absmax16x2<OutT>(absmax16x2<OutT>(amax16, v.z), v.w);
      }
      *reinterpret_cast<uint4*>(drow + ng) = v;
    }
  }
}
// One atomic per thread and tile: the row's |GELU| maximum over its columns.
template <int kEpi>
__device__ __forceinline__ void epi_row_done(const GemmArgs& args, int row, bool row_ok, uint32_t amax16) {
  if constexpr ((kEpi & kEpiGelu) != 0)
    if (row_ok) atomicMax(args.amax + row, amax16_bits(amax16));
}

template <typename OutT, int kEpi>
__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                    const GemmArgs args) {
  unsigned int* const fault = args.fault;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw_base);
  const uint32_t sA = base;                        // kStages x 16 KB
  const uint32_t sB = base + kStages * kStageA;    // kStages x 32 KB
  const uint32_t bars = sB + kStages * kStageB;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (kStages + s); };
  auto tfull_bar = [&](int b) { return bars + 8u * (2 * kStages + b); };
  auto tempty_bar = [&](int b) { return bars + 8u * (2 * kStages + 2 + b); };
  const uint32_t done_bar = bars + 8u * (2 * kStages + 4);  // all MMAs of this CTA retired
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + (bars - base) + 8 * (2 * kStages + 5));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = args.tiles_m * args.tiles_n;
  const int kblocks = (args.k + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), 4 * 32);
    }
    mbar_init(done_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued_phase[kStages];
      bool issued[kStages];
      for (int s = 0; s < kStages; ++s) issued[s] = false;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int tm = tile / args.tiles_n, tn = tile - tm * args.tiles_n;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, fault)) {
            ok = false;
            break;
          }
          mbar_expect_tx(full_bar(stage), kStageA + kStageB);
          tma_load_2d(sA + stage * kStageA, &map_a, kb * kBK, tm * kBM, full_bar(stage));
          tma_load_2d(sB + stage * kStageB, &map_b, kb * kBK, tn * kBN, full_bar(stage));
          issued[stage] = true;
          issued_phase[stage] = phase;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // drain: every copy this thread issued must have landed before the CTA exits
      for (int s = 0; s < kStages; ++s)
        if (issued[s]) mbar_wait(full_bar(s), issued_phase[s], fault);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, fault)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * kBN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, fault)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = sA + stage * kStageA, b0 = sB + stage * kStageB;
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk)
            tc_mma(d_tmem, sw128_desc(a0 + kk * kUmmaK), sw128_desc(b0 + kk * kUmmaK), kIdesc,
                   (kb | kk) != 0);
          tc_commit(empty_bar(stage));  // stage reusable once these MMAs have read it
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        tc_commit(tfull_bar(acc));  // accumulator complete
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // TMEM is freed below: wait until every MMA this thread issued has retired
      tc_commit(done_bar);
      mbar_wait(done_bar, 0, fault);
    }
  } else {
    // ---------------- epilogue: warps 2..5, TMEM lanes 32*(warp%4) .. +31
    const int q = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    OutT* D = reinterpret_cast<OutT*>(args.d);
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int tm = tile / args.tiles_n, tn = tile - tm * args.tiles_n;
      if (!mbar_wait(tfull_bar(acc), acc_phase, fault)) break;
      tc_fence_after();
      const int row = tm * kBM + q * 32 + lane;
      const bool row_ok = row < args.m;
      const float s_a = row_ok ? __ldg(args.sa + row) : 0.f;
      OutT* drow = D + (int64_t)(row_ok ? row : 0) * args.ldd;
      const OutT* rrow = reinterpret_cast<const OutT*>(args.res) + (int64_t)(row_ok ? row : 0) * args.ldr;
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * kBN);
      uint32_t amax16 = 0;
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        const int n0 = tn * kBN + c * 32;
        uint32_t r[32];
        tmem_ld32(t_row + (uint32_t)(c * 32), r);
        if (n0 >= args.n) continue;  // whole chunk past N (uniform across the warp)
        epi_chunk<OutT, kEpi>(r, n0, args, s_a, row_ok, drow, rrow, amax16);
      }
      epi_row_done<kEpi>(args, row, row_ok, amax16);
      tc_fence_before();
      mbar_arrive(tempty_bar(acc));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                 : "memory");
  }
}

// ------------------------------------------------------------------ CTA-pair kernel
// Two CTAs of a (2,1,1) cluster share one 256 x 256 output tile through
// tcgen05.mma.cta_group::2 (M = 256): CTA rank r loads A rows [128r, 128r+128)
// and B columns [128r, 128r+128) of the tile (32 KB per k-block instead of the
// 48 KB a single CTA needs for 128 x 256), the leader CTA (rank 0) issues the
// MMAs, and each CTA's tensor memory receives its 128 rows x 256 columns.
//   * both producers wait on their own `empty` barrier, then load with the
//     .cta_group::2 TMA form, completing bytes on the LEADER's `full` barrier;
//     the leader's producer alone expects the pair's 64 KB per stage;
//   * the leader's MMA thread releases a stage / publishes an accumulator with
//     one tcgen05.commit per CTA (its own barrier and the peer's, by cluster
//     address);
//   * the epilogue threads of both CTAs arrive on the leader's `tmem empty`
//     barrier (256 arrivals), the peer's remotely.
// Every load is a plain (non-broadcast) TMA load of this GPU's memory.
constexpr int kP_BM = 128;                  // A rows per CTA (pair tile: 256)
constexpr int kP_BN = 256;                  // pair tile N (128 B columns per CTA)
constexpr int kP_Stages = 6;
constexpr int kP_StageA = kP_BM * kBK;      // 16 KB
constexpr int kP_StageB = (kP_BN / 2) * kBK;  // 16 KB
constexpr int kP_SmemBytes = kP_Stages * (kP_StageA + kP_StageB) + 1024 /*align*/ + 256 /*barriers*/;
constexpr uint32_t kIdescPair = (1u << 4)                              // D format f32
                                | ((uint32_t)(kP_BN >> 3) << 17)        // N >> 3
                                | ((uint32_t)((2 * kP_BM) >> 4) << 24);  // M >> 4 (M = 256)

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t cluster_addr(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA tile load into this CTA's shared memory, bytes completed on `bar`, which
// may be the peer CTA's barrier (cluster address)
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on `bar` (cluster address) once this thread's prior pair MMAs complete
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

constexpr int kP_EpiWarps = 8;                     // 2 per TMEM lane quadrant, 128 columns each
constexpr int kP_Threads = 64 + 32 * kP_EpiWarps;  // producer warp, MMA warp, epilogue warps

template <typename OutT, int kEpi>
__global__ void __launch_bounds__(kP_Threads, 1)
    fp8_gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                         const GemmArgs args) {
  unsigned int* const fault = args.fault;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;  // identical offsets in both CTAs
  uint8_t* gbase = smem_raw + (base - raw_base);
  const uint32_t sA = base;                           // kP_Stages x 16 KB
  const uint32_t sB = base + kP_Stages * kP_StageA;   // kP_Stages x 16 KB
  const uint32_t bars = sB + kP_Stages * kP_StageB;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (kP_Stages + s); };
  auto tfull_bar = [&](int b) { return bars + 8u * (2 * kP_Stages + b); };
  auto tempty_bar = [&](int b) { return bars + 8u * (2 * kP_Stages + 2 + b); };
  const uint32_t done_bar = bars + 8u * (2 * kP_Stages + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + (bars - base) + 8 * (2 * kP_Stages + 5));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int cluster = (int)(blockIdx.x >> 1), nclusters = (int)(gridDim.x >> 1);
  const int num_tiles = args.tiles_m * args.tiles_n;  // pair tiles of 256 x 256
  const int kblocks = (args.k + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kP_Stages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), 2 * kP_EpiWarps * 32);  // the epilogue threads of both CTAs
    }
    mbar_init(done_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {  // same warp in both CTAs: the pair allocation is collective
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  cluster_sync();  // both CTAs' barriers initialised before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the previous kernel's outputs (our operands) are complete from here on
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs)
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued_phase[kP_Stages];
      bool issued[kP_Stages];
      for (int s = 0; s < kP_Stages; ++s) issued[s] = false;
      for (int tile = cluster; tile < num_tiles && ok; tile += nclusters) {
        const int tm = tile / args.tiles_n, tn = tile - tm * args.tiles_n;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, fault)) {
            ok = false;
            break;
          }
          const uint32_t fb = cluster_addr(full_bar(stage), 0);
          if (leader) mbar_expect_tx(full_bar(stage), 2 * (kP_StageA + kP_StageB));
          tma_load_2d_pair(sA + stage * kP_StageA, &map_a, kb * kBK, tm * (2 * kP_BM) + (int)rank * kP_BM, fb);
          tma_load_2d_pair(sB + stage * kP_StageB, &map_b, kb * kBK, tn * kP_BN + (int)rank * (kP_BN / 2), fb);
          issued[stage] = true;
          issued_phase[stage] = phase;
          if (++stage == kP_Stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // drain (leader): the pair's copies into every issued stage must have landed
      // (the leader's full barriers count both CTAs' bytes); the peer is held by
      // the final cluster barrier until then
      if (leader)
        for (int s = 0; s < kP_Stages; ++s)
          if (issued[s]) mbar_wait(full_bar(s), issued_phase[s], fault);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (leader CTA only)
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = cluster; tile < num_tiles && ok; tile += nclusters) {
        if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, fault)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * kP_BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, fault)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = sA + stage * kP_StageA, b0 = sB + stage * kP_StageB;
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk)
            tc_mma_pair(d_tmem, sw128_desc(a0 + kk * kUmmaK), sw128_desc(b0 + kk * kUmmaK), kIdescPair,
                        (kb | kk) != 0);
          // the stage is reusable in both CTAs once these MMAs have read it
          tc_commit_pair(empty_bar(stage));
          tc_commit_pair(cluster_addr(empty_bar(stage), 1));
          if (++stage == kP_Stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        tc_commit_pair(tfull_bar(acc));  // accumulator complete, in both CTAs
        tc_commit_pair(cluster_addr(tfull_bar(acc), 1));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // TMEM is freed below and the peer's shared memory is read by these
      // MMAs: wait until every one of them has retired
      tc_commit_pair(done_bar);
      mbar_wait(done_bar, 0, fault);
    }
  } else {
    // ---------------- epilogue: warps 2..9 of both CTAs; warp w reads TMEM lanes
    // 32*(w%4) .. +31 (the lane quadrant its warp slot may access) and column half
    // (w-2)/4 of the accumulator
    const int q = warp & 3, half = (warp - 2) >> 2;
    int acc = 0;
    uint32_t acc_phase = 0;
    OutT* D = reinterpret_cast<OutT*>(args.d);
    for (int tile = cluster; tile < num_tiles; tile += nclusters) {
      const int tm = tile / args.tiles_n, tn = tile - tm * args.tiles_n;
      if (!mbar_wait(tfull_bar(acc), acc_phase, fault)) break;
      tc_fence_after();
      const int row = tm * (2 * kP_BM) + (int)rank * kP_BM + q * 32 + lane;
      const bool row_ok = row < args.m;
      const float s_a = row_ok ? __ldg(args.sa + row) : 0.f;
      OutT* drow = D + (int64_t)(row_ok ? row : 0) * args.ldd;
      const OutT* rrow = reinterpret_cast<const OutT*>(args.res) + (int64_t)(row_ok ? row : 0) * args.ldr;
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * kP_BN);
      uint32_t amax16 = 0;
#pragma unroll 1
      for (int c = half * (kP_BN / 64); c < (half + 1) * (kP_BN / 64); ++c) {
        const int n0 = tn * kP_BN + c * 32;
        uint32_t r[32];
        tmem_ld32(t_row + (uint32_t)(c * 32), r);
        if (n0 >= args.n) continue;  // whole chunk past N (uniform across the warp)
        epi_chunk<OutT, kEpi>(r, n0, args, s_a, row_ok, drow, rrow, amax16);
      }
      epi_row_done<kEpi>(args, row, row_ok, amax16);
      tc_fence_before();
      if (leader)
        mbar_arrive(tempty_bar(acc));
      else
        mbar_arrive_cluster(cluster_addr(tempty_bar(acc), 0));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }
  __syncthreads();
  // neither CTA leaves while the other may still signal its barriers or have
  // its shared memory read by the pair's MMAs
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                 : "memory");
  }
}

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D K-major fp8 operand [rows, K] (row stride ld bytes), box kBK x box_rows, 128-byte swizzle.
int make_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t k, int64_t ld, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(JO_ERR_CUDA, "fp8_scaled_mm: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(JO_ERR_CUDA, "fp8_scaled_mm: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return JO_OK;
}

template <typename OutT, int kEpi>
int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& a, cudaStream_t st,
                const DeviceInfo* di) {
  auto kern = fp8_gemm_kernel<OutT, kEpi>;
  static std::atomic<uint64_t> reserved{0};
  if (int s = reserve_smem((const void*)kern, kSmemBytes, reserved, di, "fp8_scaled_mm")) return s;
  const int tiles = a.tiles_m * a.tiles_n;
  const int grid = tiles < di->sm_count ? tiles : di->sm_count;
  kern<<<grid, kThreads, kSmemBytes, st>>>(ma, mb, a);
  return after_launch("fp8_gemm_kernel");
}

// CTA-pair launch: clusters of (2,1,1), as many as can be resident at once.
template <typename OutT, int kEpi>
int launch_gemm_pair(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& a, cudaStream_t st,
                     const DeviceInfo* di) {
  auto kern = fp8_gemm_pair_kernel<OutT, kEpi>;
  static std::atomic<uint64_t> reserved{0};
  if (int s = reserve_smem((const void*)kern, kP_SmemBytes, reserved, di, "fp8_scaled_mm")) return s;
  static std::atomic<int> resident[64];  // resident CTA pairs, per device (0 = not queried yet)
  int max_clusters = resident[di->ordinal].load(std::memory_order_relaxed);
  if (!max_clusters) {
    cudaLaunchConfig_t qc = {};
    qc.gridDim = dim3(2, 1, 1);
    qc.blockDim = dim3(kP_Threads, 1, 1);
    qc.dynamicSmemBytes = kP_SmemBytes;
    cudaLaunchAttribute qa[1];
    qa[0].id = cudaLaunchAttributeClusterDimension;
    qa[0].val.clusterDim.x = 2;
    qa[0].val.clusterDim.y = 1;
    qa[0].val.clusterDim.z = 1;
    qc.attrs = qa;
    qc.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, (const void*)kern, &qc) != cudaSuccess || n < 1)
      return fail(JO_ERR_CUDA, "fp8_scaled_mm: no resident CTA pair");
    max_clusters = n;
    resident[di->ordinal].store(n, std::memory_order_relaxed);
  }
  const int tiles = a.tiles_m * a.tiles_n;
  const int clusters = tiles < max_clusters ? tiles : max_clusters;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  cfg.blockDim = dim3(kP_Threads, 1, 1);
  cfg.dynamicSmemBytes = kP_SmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see launch_pdl
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  if (cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ma, mb, a)) return launch_failed(e, "fp8_scaled_mm");
  return after_launch("fp8_gemm_pair_kernel");
}

// ------------------------------------------------------------------ GELU -> FP8
// Second pass of the MLP's fc1 -> GELU -> per-token FP8: the GEMM epilogue has
// stored y = GELU(fc1) as OutT and the per-row max |y| (16-bit magnitude bits);
// this pass is the quantisation alone, with the row quant kernels' arithmetic
// (scale = max(amax, 1e-8) / 448, q = e4m3(y / scale) with the correctly rounded
// quotient, satfinite), so q and scale equal sgl_per_token_quant_fp8(y) bit for
// bit.  One CTA per row; each thread holds its kApplyVPT 16-byte vectors in
// flight before converting them.
constexpr int kApplyThreads = 256;
constexpr int kApplyVPT = 6;  // 12288 bf16 = 1536 vectors per row: one pass

template <typename T>
__global__ void __launch_bounds__(kApplyThreads) gelu_quant_apply_kernel(const T* __restrict__ y, int64_t ldy,
                                                                         const uint32_t* __restrict__ amax,
                                                                         uint8_t* __restrict__ q, int64_t ldq,
                                                                         float* __restrict__ s_out, int nvec) {
  pdl_wait();  // y and amax are the GEMM's outputs
  const int64_t row = blockIdx.x;
  const float s = quant_scale(bits16_to_f<T>(amax[row]));
  const float2 ns2 = f2(-s), rc2 = f2(__frcp_rn(s));
  const uint8_t* yr = reinterpret_cast<const uint8_t*>(y + row * ldy);
  uint8_t* qr = q + row * ldq;
  for (int base = threadIdx.x; base < nvec; base += kApplyThreads * kApplyVPT) {
    uint4 v[kApplyVPT];
#pragma unroll
    for (int u = 0; u < kApplyVPT; ++u) {
      const int idx = base + u * kApplyThreads;
      if (idx < nvec) v[u] = ld_stream(yr + (int64_t)idx * 16);
    }
#pragma unroll
    for (int u = 0; u < kApplyVPT; ++u) {
      const int idx = base + u * kApplyThreads;
      if (idx >= nvec) continue;
      float2 p[4], qq[4];
      to_pairs<T>(v[u], p);
#pragma unroll
      for (int e = 0; e < 4; ++e) qq[e] = div2_ms(p[e], ns2, rc2);
      const uint32_t w0 = ((uint32_t)e4m3x2(qq[0].x, qq[0].y) | ((uint32_t)e4m3x2(qq[1].x, qq[1].y) << 16)) |
                          e4m3_signs(v[u].x, v[u].y);
      const uint32_t w1 = ((uint32_t)e4m3x2(qq[2].x, qq[2].y) | ((uint32_t)e4m3x2(qq[3].x, qq[3].y) << 16)) |
                          e4m3_signs(v[u].z, v[u].w);
      *reinterpret_cast<uint2*>(qr + (int64_t)idx * 8) = make_uint2(w0, w1);
    }
  }
  if (threadIdx.x == 0) s_out[row] = s;
  pdl_trigger();
}

template <typename T>
int launch_gelu_quant_apply(uint8_t* q, int64_t ldq, float* s, const void* y, int64_t ldy, const uint32_t* amax,
                            int64_t m, int64_t n, cudaStream_t st) {
  auto kern = gelu_quant_apply_kernel<T>;
  if (cudaError_t e = launch_pdl(kern, dim3((unsigned)m), dim3(kApplyThreads), 0, st, reinterpret_cast<const T*>(y),
                                 ldy, amax, q, ldq, s, (int)(n / 8)))
    return launch_failed(e, "fp8_scaled_mm_gelu_quant");
  return after_launch("gelu_quant_apply_kernel");
}

}  // namespace
}  // namespace jo

namespace jo {
namespace {

template <int kEpi>
int dispatch_gemm(bool pair, int out_dtype, const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& g,
                  cudaStream_t st, const DeviceInfo* di) {
  if (pair)
    return out_dtype == JO_BF16 ? launch_gemm_pair<__nv_bfloat16, kEpi>(ma, mb, g, st, di)
                                : launch_gemm_pair<__half, kEpi>(ma, mb, g, st, di);
  return out_dtype == JO_BF16 ? launch_gemm<__nv_bfloat16, kEpi>(ma, mb, g, st, di)
                              : launch_gemm<__half, kEpi>(ma, mb, g, st, di);
}

int gemm_entry(const char* op, void* d, int64_t ldd, const void* a, int64_t lda, const void* b, int64_t ldb,
               const float* scale_a, const float* scale_b, const void* bias, const void* res, int64_t ldr,
               const void* gate, uint32_t* amax, int64_t m, int64_t n, int64_t k, int out_dtype, void* stream) {
  const DeviceInfo* di;
  if (int s = device_info(&di)) return s;
  if (m < 0 || n < 0 || k < 0) return fail(JO_ERR_SHAPE, "%s: negative size", op);
  if (m == 0 || n == 0) return JO_OK;
  if (out_dtype != JO_BF16 && out_dtype != JO_F16) return fail(JO_ERR_DTYPE, "%s: out dtype must be bf16/fp16", op);
  if (!d || !a || !b || !scale_a || !scale_b) return fail(JO_ERR_INVALID, "%s: null operand", op);
  if (k == 0) return fail(JO_ERR_SHAPE, "%s: K must be positive", op);
  if (k % 16 || lda % 16 || ldb % 16) return fail(JO_ERR_ALIGN, "%s: K, lda, ldb must be multiples of 16", op);
  if (n % 8 || ldd % 8) return fail(JO_ERR_ALIGN, "%s: N and ldd must be multiples of 8", op);
  if (lda < k || ldb < k || ldd < n) return fail(JO_ERR_SHAPE, "%s: leading dimension smaller than the row", op);
  if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX) return fail(JO_ERR_SHAPE, "%s: size too large", op);
  if (!aligned16(d) || !aligned16(a) || !aligned16(b) || !aligned16(scale_b) || (bias && !aligned16(bias)))
    return fail(JO_ERR_ALIGN, "%s: D, A, B, scale_b and bias must be 16-byte aligned", op);
  // CTA pairs (256 x 256 tiles) unless A is a single 128-row tile
  const bool pair = m > kBM;
  CUtensorMap ma, mb;
  if (int s = make_map(&ma, a, m, k, lda, pair ? kP_BM : kBM)) return s;
  if (int s = make_map(&mb, b, n, k, ldb, pair ? kP_BN / 2 : kBN)) return s;
  GemmArgs g{};
  g.d = d;
  g.ldd = ldd;
  g.sa = scale_a;
  g.sb = scale_b;
  g.bias = bias;
  g.res = res;
  g.ldr = ldr;
  g.gate = gate;
  g.amax = amax;
  g.m = (int)m;
  g.n = (int)n;
  g.k = (int)k;
  g.tiles_m = (int)cdiv(m, pair ? 2 * kP_BM : kBM);
  g.tiles_n = (int)cdiv(n, pair ? kP_BN : kBN);
  g.fault = di->fault;
  if ((int64_t)g.tiles_m * g.tiles_n > INT32_MAX) return fail(JO_ERR_SHAPE, "%s: too many tiles", op);
  cudaStream_t st = (cudaStream_t)stream;
  const int epi = (bias ? kEpiBias : 0) | (res ? kEpiResid : 0) | (amax ? kEpiGelu : 0);
  if ((epi & kEpiResid) && (epi & kEpiGelu)) return fail(JO_ERR_INVALID, "%s: residual and GELU epilogues are exclusive", op);
  // the GELU epilogue's row maxima accumulate by atomicMax: reset them once every check has passed
  if (amax)
    if (cudaError_t e = cudaMemsetAsync(amax, 0, (size_t)m * sizeof(uint32_t), st))
      return launch_failed(e, "fp8_scaled_mm_gelu_quant (amax reset)");
  switch (epi) {
    case 0: return dispatch_gemm<0>(pair, out_dtype, ma, mb, g, st, di);
    case kEpiBias: return dispatch_gemm<kEpiBias>(pair, out_dtype, ma, mb, g, st, di);
    case kEpiResid: return dispatch_gemm<kEpiResid>(pair, out_dtype, ma, mb, g, st, di);
    case kEpiBias | kEpiResid: return dispatch_gemm<kEpiBias | kEpiResid>(pair, out_dtype, ma, mb, g, st, di);
    case kEpiGelu: return dispatch_gemm<kEpiGelu>(pair, out_dtype, ma, mb, g, st, di);
    case kEpiBias | kEpiGelu: return dispatch_gemm<kEpiBias | kEpiGelu>(pair, out_dtype, ma, mb, g, st, di);
    default: return fail(JO_ERR_INVALID, "%s: unsupported epilogue combination", op);
  }
}

}  // namespace
}  // namespace jo

using namespace jo;

extern "C" {

int jo_fp8_scaled_mm(void* d, int64_t ldd, const void* a, int64_t lda, const void* b, int64_t ldb,
                     const float* scale_a, const float* scale_b, const void* bias, int64_t m, int64_t n,
                     int64_t k, int out_dtype, void* stream) {
  return gemm_entry("fp8_scaled_mm", d, ldd, a, lda, b, ldb, scale_a, scale_b, bias, nullptr, 0, nullptr, nullptr, m,
                    n, k, out_dtype, stream);
}

int jo_fp8_scaled_mm_gated_residual(void* d, int64_t ldd, const void* a, int64_t lda, const void* b, int64_t ldb,
                                    const float* scale_a, const float* scale_b, const void* bias,
                                    const void* residual, int64_t ldr, const void* gate, int64_t m, int64_t n,
                                    int64_t k, int out_dtype, void* stream) {
  const char* op = "fp8_scaled_mm_gated_residual";
  if (!residual || !gate) return fail(JO_ERR_INVALID, "%s: null residual or gate", op);
  if (ldr < n || ldr % 8) return fail(JO_ERR_ALIGN, "%s: residual row stride must be >= N and a multiple of 8", op);
  if (!aligned16(residual) || !aligned16(gate)) return fail(JO_ERR_ALIGN, "%s: residual and gate must be 16-byte aligned", op);
  return gemm_entry(op, d, ldd, a, lda, b, ldb, scale_a, scale_b, bias, residual, ldr, gate, nullptr, m, n, k,
                    out_dtype, stream);
}

int jo_fp8_scaled_mm_gelu_quant(void* out_q, int64_t ldq, float* out_s, void* y, int64_t ldy, uint32_t* amax,
                                const void* a, int64_t lda, const void* b, int64_t ldb, const float* scale_a,
                                const float* scale_b, const void* bias, int64_t m, int64_t n, int64_t k,
                                int y_dtype, void* stream) {
  const char* op = "fp8_scaled_mm_gelu_quant";
  if (m < 0 || n < 0) return fail(JO_ERR_SHAPE, "%s: negative size", op);
  if (m == 0) return JO_OK;
  if (n == 0) return fail(JO_ERR_SHAPE, "%s: N must be positive (per-token amax of an empty row)", op);
  if (m > INT32_MAX) return fail(JO_ERR_SHAPE, "%s: size too large", op);
  if (!out_q || !out_s || !y || !amax) return fail(JO_ERR_INVALID, "%s: null output or workspace", op);
  if (ldq < n || ldq % 8 || (reinterpret_cast<uintptr_t>(out_q) & 7))
    return fail(JO_ERR_ALIGN, "%s: out_q must be 8-byte aligned with a row stride >= N, a multiple of 8", op);
  if (reinterpret_cast<uintptr_t>(amax) & 3) return fail(JO_ERR_ALIGN, "%s: amax workspace must be 4-byte aligned", op);
  cudaStream_t st = (cudaStream_t)stream;
  if (int s = gemm_entry(op, y, ldy, a, lda, b, ldb, scale_a, scale_b, bias, nullptr, 0, nullptr, amax, m, n, k,
                         y_dtype, stream))
    return s;
  return y_dtype == JO_BF16 ? launch_gelu_quant_apply<__nv_bfloat16>((uint8_t*)out_q, ldq, out_s, y, ldy, amax, m, n, st)
                            : launch_gelu_quant_apply<__half>((uint8_t*)out_q, ldq, out_s, y, ldy, amax, m, n, st);
}

}  // extern "C"
