// Timestep conditioning MLP: the whole WanTimeTextImageEmbedding timestep
// branch (deploy/xvideo/models/dit/dit.py:574-579, 605-620) in three launches.
//
//   e   = bf16(Timesteps(freq_dim, flip_sin_to_cos=True, shift=0)(t))   (dit.py:614-618)
//   s1  = bf16(silu(bf16(e  @ W1^T + b1)))     time_embedder.linear_1 + act   [B, dim]
//   s2  = bf16(silu(bf16(s1 @ W2^T + b2)))     time_embedder.linear_2, act_fn (dit.py:619-620)
//   vec = bf16(s2 @ W3^T + b3)                 time_proj                      [B, proj_dim]
//
// Each Linear is the reference's bf16 nn.Linear: fp32 accumulation, bias added
// in fp32, one rounding to bf16; SiLU is evaluated in fp32 on the bf16 value
// and rounded again (the unfused modules materialise both tensors).
//
// Design (B200): at the model's batch (1-2 timesteps) every layer is a GEMV
// bound by the weight read (W3 alone is 113 MB at dim 3072), so each layer is
// one HBM stream: each CTA (one per SM) owns a contiguous block of output rows,
// its 16 warps stream ~6 KB units of consecutive weight rows through their own
// shared-memory slots with TMA bulk copies (bounded mbarrier waits), and
// multiply them against the batch's input rows staged once per CTA in shared
// memory; one warp shuffle reduction per output row and batch row.  The two intermediates live in caller-owned
// scratch (4 * B * dim bytes) between the launches; the sinusoid is computed in
// the first layer's prologue.
#include <math.h>

#include <algorithm>
#include <mutex>

#include "pipeline.cuh"

namespace jo {
namespace {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxK = 4096;                 // input features per layer
constexpr int kMaxB = 8;                    // batch rows per launch
constexpr uint32_t kBudget = 216u * 1024u;  // shared memory: batch rows + weight slots
// Shared memory a layer aims to stay within.  At half an SM (110 KB) the next
// layer's CTAs, launched early (programmatic dependent launch), fit beside this
// layer's and stream their first weight rows while it runs; measured at batch 1
// that is slower than the whole budget (35.2 vs 33.6 us: the big last layer keeps
// fewer rows in flight), so each layer takes the whole budget.
#ifndef JO_TEMB_LAYER_SMEM
#define JO_TEMB_LAYER_SMEM (216u * 1024u)
#endif
constexpr uint32_t kLayerSmem = JO_TEMB_LAYER_SMEM;

struct TembLayer {
  const __nv_bfloat16* x;  // [B, K] input rows (null for the sinusoid layer)
  const float* t;          // [B] timesteps (sinusoid layer)
  const __nv_bfloat16* w;  // [N, K] row-major
  const __nv_bfloat16* bias;  // [N] or null
  __nv_bfloat16* y;        // [B, N]
  int K, N, B;
  float neg_log_period;    // -ln(max_period) rounded to fp32
  // time_proj only: ModulateWan tables [T, N] added to the rounded output,
  // mods[t, b, n] = bf16(tables[t, n] + y[b, n]) (null / 0: none)
  const __nv_bfloat16* tables;
  __nv_bfloat16* mods;
  int T;
  // L2 prefetch of the next layer's first weight rows (null: none): rows
  // c * pf_per + [0, pf_rows) of pf_w for c < pf_ctas, pf_row_bytes each
  const __nv_bfloat16* pf_w;
  int64_t pf_per;
  int pf_rows, pf_ctas, pf_row_bytes, pf_n;
};

// Overlap of time_proj with the two small layers (measured at batch 1, graph replay of the
// three launches: 29.3 us without any of these, 28.6 us with all three):
//  JO_TEMB_CARVEOUT       the small layers run with the whole shared-memory carveout, so an SM
//                         need not drain to change it before time_proj's CTAs can land there
//  JO_TEMB_EARLY_TRIGGER  layer 2 lets time_proj launch before its own wait, so time_proj's
//                         first weight copies go out while layer 2 finishes
//  JO_TEMB_PF_ROWS        layer 2 prefetches into L2, after its wait, the first rows of every
//                         time_proj CTA's block (16 rows: 14.5 MB; 32 rows measured 31.6 us,
//                         prefetches issued before the wait 29.5 us, 4 CTAs per SM for layer 2
//                         29.7 us)
#ifndef JO_TEMB_PF_ROWS
#define JO_TEMB_PF_ROWS 16
#endif
#ifndef JO_TEMB_PF_EARLY
#define JO_TEMB_PF_EARLY 0
#endif
#ifndef JO_TEMB_EARLY_TRIGGER
#define JO_TEMB_EARLY_TRIGGER 1
#endif
#ifndef JO_TEMB_CARVEOUT
#define JO_TEMB_CARVEOUT 1
#endif

// L2 prefetch (no destination) of the next layer's first rows, one bulk prefetch per warp.
__device__ __forceinline__ void temb_prefetch_next(const TembLayer& a) {
  if (a.pf_w == nullptr || (threadIdx.x & 31) != 0) return;
  const int nw = gridDim.x * (blockDim.x >> 5);
  const int total = a.pf_ctas * a.pf_rows;
  for (int idx = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); idx < total; idx += nw) {
    const int c = idx / a.pf_rows, j = idx - c * a.pf_rows;
    const int64_t row = (int64_t)c * a.pf_per + j;
    if (j >= a.pf_per || row >= a.pf_n) continue;
    const char* src = reinterpret_cast<const char*>(a.pf_w) + row * (int64_t)a.pf_row_bytes;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(a.pf_row_bytes) : "memory");
  }
}

struct TembCfg {
  int rows_per_unit;    // consecutive weight rows per bulk copy
  int m;                // slots per warp
  uint32_t slot_bytes;  // rows_per_unit * K * 2, rounded up to 128
  uint32_t x_off;       // byte offset of the staged batch rows
  uint32_t data_off;    // byte offset of slot 0
};

__device__ __forceinline__ float silu_exact(float v) { return v / (1.f + expf(-v)); }

// One layer for batch rows [b0, b0 + kB) (rows >= B are skipped).  Weight rows
// stream through per-warp shared-memory slots filled with 1-D TMA bulk copies
// (each warp keeps its next m units in flight; the copy engine holds the bytes,
// not registers), as in the staged row kernels.
template <int kB, bool kSinIn, bool kSilu>
__global__ void __launch_bounds__(kThreads, 1)
    temb_layer_kernel(const TembLayer a, const TembCfg cfg, int b0, unsigned int* fault) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int K = a.K;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = smem_u32(smem_raw);
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem_raw + cfg.x_off);  // [kB, K]
  const int m = cfg.m, R = cfg.rows_per_unit;
  const int64_t per = (a.N + gridDim.x - 1) / gridDim.x;  // rows of this CTA
  const int64_t r0 = (int64_t)blockIdx.x * per;
  const int64_t rend = r0 + per < a.N ? r0 + per : a.N;
  const int nrows = rend > r0 ? (int)(rend - r0) : 0;
  const int units = (nrows + R - 1) / R;
  if (threadIdx.x < kWarps * m) mbar_init(base + 8u * threadIdx.x, 1);
  if (threadIdx.x == 0) mbar_init_fence();
  __syncthreads();
  const uint32_t bar0 = base + 8u * (uint32_t)(warp * m);
  const uint32_t slot0 = base + cfg.data_off + (uint32_t)(warp * m) * cfg.slot_bytes;
  auto unit_rows = [&](int u) { return min(R, nrows - u * R); };
  // unit k of this warp is unit warp + k * kWarps of the CTA, in slot k % m
  auto issue = [&](int k) {
    const int u = warp + k * kWarps;
    if (u >= units) return;
    const uint32_t bytes = (uint32_t)unit_rows(u) * (uint32_t)K * 2u;
    const uint32_t bar = bar0 + 8u * (uint32_t)(k % m);
    mbar_expect_tx(bar, bytes);
    bulk_load(slot0 + (uint32_t)(k % m) * cfg.slot_bytes, a.w + (r0 + (int64_t)u * R) * K, bytes, bar);
  };
  // Layers 2 and 3 follow a layer of this MLP, which never writes weights, and
  // are launched only once that layer has passed its own wait (so every kernel
  // before it has completed): their first weight copies go out before the wait
  // and overlap the previous layer.  Layer 1 follows the caller's work and
  // waits first.
  constexpr bool kEarly = !kSinIn;
  if (kEarly && lane == 0)
    for (int k = 0; k < m; ++k) issue(k);
  pdl_wait();  // the previous layer's output (our input) is complete from here on
  pdl_trigger();
  if (!kEarly && lane == 0)
    for (int k = 0; k < m; ++k) issue(k);

  // ---- stage the batch's input rows while the first weight rows are in flight
  if constexpr (kSinIn) {
    // diffusers get_timestep_embedding with flip_sin_to_cos=True, shift 0:
    // [cos(t f_i), sin(t f_i)], f_i = exp(-ln(P) * i / half), fp32, then bf16
    const int half = K / 2;
    for (int idx = threadIdx.x; idx < kB * half; idx += blockDim.x) {
      const int b = idx / half, i = idx - b * half;
      float c = 0.f, s = 0.f;
      if (b0 + b < a.B) {
        const float ex = __fdiv_rn(__fmul_rn(a.neg_log_period, (float)i), (float)half);
        const float arg = __fmul_rn(a.t[b0 + b], expf(ex));
        sincosf(arg, &s, &c);
      }
      xs[b * K + i] = __float2bfloat16_rn(c);
      xs[b * K + half + i] = __float2bfloat16_rn(s);
    }
  } else {
    const int nv = K / 8;
    for (int idx = threadIdx.x; idx < kB * nv; idx += blockDim.x) {
      const int b = idx / nv, v = idx - b * nv;
      uint4 u = make_uint4(0, 0, 0, 0);
      if (b0 + b < a.B) u = *reinterpret_cast<const uint4*>(a.x + (int64_t)(b0 + b) * K + v * 8);
      *reinterpret_cast<uint4*>(xs + b * K + v * 8) = u;
    }
  }
  __syncthreads();

  int k = 0;
  for (; warp + k * kWarps < units; ++k) {
    const int u = warp + k * kWarps;
    const uint32_t sl = slot0 + (uint32_t)(k % m) * cfg.slot_bytes;
    if (!mbar_wait(bar0 + 8u * (uint32_t)(k % m), (uint32_t)((k / m) & 1), fault)) break;
    const int nr = unit_rows(u);
    for (int r = 0; r < nr; ++r) {
      float acc[kB];
#pragma unroll
      for (int b = 0; b < kB; ++b) acc[b] = 0.f;
      for (int kk = lane * 8; kk < K; kk += 256) {
        float wf[8];
        Elt<__nv_bfloat16>::unpack(lds128(sl + (uint32_t)(r * K + kk) * 2u), wf);
#pragma unroll
        for (int b = 0; b < kB; ++b) {
          float xf[8];
          Elt<__nv_bfloat16>::unpack(*reinterpret_cast<const uint4*>(xs + b * K + kk), xf);
          float p0 = wf[0] * xf[0], p1 = wf[1] * xf[1];
          p0 = fmaf(wf[2], xf[2], p0);
          p1 = fmaf(wf[3], xf[3], p1);
          p0 = fmaf(wf[4], xf[4], p0);
          p1 = fmaf(wf[5], xf[5], p1);
          p0 = fmaf(wf[6], xf[6], p0);
          p1 = fmaf(wf[7], xf[7], p1);
          acc[b] += p0 + p1;
        }
      }
      const int64_t n = r0 + (int64_t)u * R + r;
      const float bias = a.bias ? __bfloat162float(a.bias[n]) : 0.f;
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        const float h = warp_sum(acc[b]) + bias;  // every lane holds the sum
        if (lane == b && b0 + b < a.B) {
          float y = __bfloat162float(__float2bfloat16_rn(h));
          if constexpr (kSilu) y = silu_exact(y);
          a.y[(int64_t)(b0 + b) * a.N + n] = __float2bfloat16_rn(y);
        }
        if constexpr (!kSilu) {
          if (a.T > 0 && b0 + b < a.B) {  // ModulateWan: bf16(table + bf16(vec)), tables spread over the lanes
            const float y = __bfloat162float(__float2bfloat16_rn(h));
            for (int t = lane; t < a.T; t += 32)
              a.mods[((int64_t)t * a.B + b0 + b) * a.N + n] =
                  __float2bfloat16_rn(__bfloat162float(a.tables[(int64_t)t * a.N + n]) + y);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // slot reads before the refill
      issue(k + m);
    }
  }
  // error path only (a wait expired at unit k): every copy issued, unit k's
  // included, must have landed (or its wait expired too) before the CTA exits
  if (lane == 0 && warp + k * kWarps < units)
    for (int j = k; j < k + m && warp + j * kWarps < units; ++j)
      mbar_wait(bar0 + 8u * (uint32_t)(j % m), (uint32_t)((j / m) & 1), fault);
}

// Small layers (the first two at the model's shape: 1.5 MB and 19 MB of weights)
// are bound by latency, not bandwidth: one warp per output row loads its whole
// weight row into registers with direct 16-byte loads -- before the wait on the
// previous layer when that layer is one of ours (kEarly), so the loads overlap it;
// the CTAs use no dynamic shared memory and fit beside the previous layer's --
// then the batch rows.  The per-lane summation order is the staged kernel's
// (elements lane*8 + j*256, two fma chains per vector), so the bits are the same.
constexpr int kDirectWarps = 8;
constexpr int kDirectMaxB = 2;

template <int kB, int kV, bool kSinIn, bool kSilu, bool kEarly>
#ifndef JO_TEMB_DIRECT_MINB
#define JO_TEMB_DIRECT_MINB 1
#endif
__global__ void __launch_bounds__(kDirectWarps * 32, JO_TEMB_DIRECT_MINB)
    temb_direct_kernel(const TembLayer a, int b0) {
  __shared__ __align__(16) __nv_bfloat16 xs[kB * kV * 256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = a.K;
  const int64_t n = (int64_t)blockIdx.x * kDirectWarps + warp;
  const bool row_ok = n < a.N;
  uint4 w[kV];
  auto load_w = [&]() {
#pragma unroll
    for (int j = 0; j < kV; ++j) {
      const int kk = lane * 8 + j * 256;
      w[j] = (row_ok && kk < K) ? ld_stream(a.w + n * K + kk) : make_uint4(0, 0, 0, 0);
    }
  };
  if constexpr (kEarly) {
    load_w();
    // Layer 2 was launched only once layer 1 had passed its own wait (every kernel
    // before the MLP has completed), so time_proj may start its weight copies now;
    // it reads its input only after its own wait (this layer complete).
    if (JO_TEMB_EARLY_TRIGGER) pdl_trigger();
    if (JO_TEMB_PF_EARLY) temb_prefetch_next(a);
  }
  pdl_wait();  // the previous layer's output (our input) is complete from here on
  pdl_trigger();
  if constexpr (!kEarly) load_w();
  if (!JO_TEMB_PF_EARLY) temb_prefetch_next(a);
  if constexpr (kSinIn) {  // the sinusoid, with the staged kernel's arithmetic
    const int half = K / 2;
    for (int idx = threadIdx.x; idx < kB * half; idx += blockDim.x) {
      const int b = idx / half, i = idx - b * half;
      float c = 0.f, s = 0.f;
      if (b0 + b < a.B) {
        const float ex = __fdiv_rn(__fmul_rn(a.neg_log_period, (float)i), (float)half);
        const float arg = __fmul_rn(a.t[b0 + b], expf(ex));
        sincosf(arg, &s, &c);
      }
      xs[b * K + i] = __float2bfloat16_rn(c);
      xs[b * K + half + i] = __float2bfloat16_rn(s);
    }
  } else {
    const int nv = K / 8;
    for (int idx = threadIdx.x; idx < kB * nv; idx += blockDim.x) {
      const int b = idx / nv, v = idx - b * nv;
      uint4 u = make_uint4(0, 0, 0, 0);
      if (b0 + b < a.B) u = *reinterpret_cast<const uint4*>(a.x + (int64_t)(b0 + b) * K + v * 8);
      *reinterpret_cast<uint4*>(xs + b * K + v * 8) = u;
    }
  }
  __syncthreads();
  if (!row_ok) return;
  float acc[kB];
#pragma unroll
  for (int b = 0; b < kB; ++b) acc[b] = 0.f;
#pragma unroll
  for (int j = 0; j < kV; ++j) {
    const int kk = lane * 8 + j * 256;
    if (kk >= K) break;  // uniform per j across lanes only when K % 256 == 0; per lane otherwise
    float wf[8];
    Elt<__nv_bfloat16>::unpack(w[j], wf);
#pragma unroll
    for (int b = 0; b < kB; ++b) {
      float xf[8];
      Elt<__nv_bfloat16>::unpack(*reinterpret_cast<const uint4*>(xs + b * K + kk), xf);
      float p0 = wf[0] * xf[0], p1 = wf[1] * xf[1];
      p0 = fmaf(wf[2], xf[2], p0);
      p1 = fmaf(wf[3], xf[3], p1);
      p0 = fmaf(wf[4], xf[4], p0);
      p1 = fmaf(wf[5], xf[5], p1);
      p0 = fmaf(wf[6], xf[6], p0);
      p1 = fmaf(wf[7], xf[7], p1);
      acc[b] += p0 + p1;
    }
  }
  const float bias = a.bias ? __bfloat162float(a.bias[n]) : 0.f;
#pragma unroll
  for (int b = 0; b < kB; ++b) {
    const float h = warp_sum(acc[b]) + bias;
    if (lane == b && b0 + b < a.B) {
      float y = __bfloat162float(__float2bfloat16_rn(h));
      if constexpr (kSilu) y = silu_exact(y);
      a.y[(int64_t)(b0 + b) * a.N + n] = __float2bfloat16_rn(y);
    }
  }
}

template <int kB, int kV, bool kSinIn, bool kSilu>
int launch_direct(const TembLayer& a, int b0, cudaStream_t st, const DeviceInfo* di) {
  const int64_t grid = cdiv(a.N, kDirectWarps);
  if (JO_TEMB_CARVEOUT) {
    static std::atomic<uint64_t> carved{0};  // one per kernel instantiation
    if (int s = prefer_max_carveout((const void*)temb_direct_kernel<kB, kV, kSinIn, kSilu, !kSinIn>, carved, di,
                                    "timestep_mlp"))
      return s;
  }
  if (cudaError_t e = launch_pdl(temb_direct_kernel<kB, kV, kSinIn, kSilu, !kSinIn>, dim3((unsigned)grid),
                                 dim3(kDirectWarps * 32), 0, st, a, b0))
    return launch_failed(e, "timestep_mlp");
  return after_launch("temb_direct_kernel");
}

// The direct kernel for layers whose weights are at most kDirectBytes (and batch
// chunks of at most kDirectMaxB rows): returns true when it took the layer.
constexpr int64_t kDirectBytes = 32ll << 20;
template <bool kSinIn, bool kSilu>
bool try_direct(const TembLayer& a, cudaStream_t st, const DeviceInfo* di, int& status) {
  if ((int64_t)a.N * a.K * 2 > kDirectBytes || a.K > kMaxK) return false;
  status = JO_OK;
  for (int b0 = 0; b0 < a.B && status == JO_OK; b0 += kDirectMaxB) {  // one launch at the model's batch
    const bool one = a.B - b0 == 1;
    const int kv = (a.K + 255) / 256;
    if (kv <= 1)
      status = one ? launch_direct<1, 1, kSinIn, kSilu>(a, b0, st, di) : launch_direct<2, 1, kSinIn, kSilu>(a, b0, st, di);
    else if (kv <= 4)
      status = one ? launch_direct<1, 4, kSinIn, kSilu>(a, b0, st, di) : launch_direct<2, 4, kSinIn, kSilu>(a, b0, st, di);
    else if (kv <= 12)
      status = one ? launch_direct<1, 12, kSinIn, kSilu>(a, b0, st, di) : launch_direct<2, 12, kSinIn, kSilu>(a, b0, st, di);
    else
      status = one ? launch_direct<1, 16, kSinIn, kSilu>(a, b0, st, di) : launch_direct<2, 16, kSinIn, kSilu>(a, b0, st, di);
  }
  return true;
}

template <int kB, bool kSinIn, bool kSilu>
int launch_one(const TembLayer& a, const TembCfg& cfg, int b0, int64_t grid, size_t smem, cudaStream_t st,
               const DeviceInfo* di) {
  auto kern = temb_layer_kernel<kB, kSinIn, kSilu>;
  static std::atomic<uint64_t> reserved{0};  // one per kernel instantiation
  if (int s = reserve_smem((const void*)kern, (int)kBudget, reserved, di, "timestep_mlp")) return s;
  if (cudaError_t e = launch_pdl(kern, dim3((unsigned)grid), dim3(kThreads), smem, st, a, cfg, b0, di->fault))
    return launch_failed(e, "timestep_mlp");
  return JO_OK;
}

template <bool kSinIn, bool kSilu>
int launch_layer(const TembLayer& a, cudaStream_t st, const DeviceInfo* di) {
  // the time_proj layer (ModulateWan tables in its epilogue) always streams
  if (kSilu && a.B <= kDirectMaxB) {
    int s = JO_OK;
    if (try_direct<kSinIn, kSilu>(a, st, di, s)) return s;
  }
  for (int b0 = 0; b0 < a.B; b0 += kMaxB) {
    const int nb = std::min(kMaxB, a.B - b0);
    const int kb = nb <= 1 ? 1 : (nb <= 2 ? 2 : (nb <= 4 ? 4 : 8));
    TembCfg cfg{};
    const uint32_t row_bytes = (uint32_t)a.K * 2u;
    cfg.rows_per_unit = std::max(1, (int)(6144u / row_bytes));  // ~6 KB per bulk copy
    cfg.slot_bytes = ((uint32_t)cfg.rows_per_unit * row_bytes + 127u) & ~127u;
    cfg.x_off = 1024;  // after the warps' mbarriers
    cfg.data_off = (cfg.x_off + (uint32_t)kb * row_bytes + 127u) & ~127u;
    const uint32_t half = kLayerSmem > cfg.data_off ? kLayerSmem - cfg.data_off : 0u;
    cfg.m = (int)std::min<uint32_t>(3u, half / (kWarps * cfg.slot_bytes));
    if (cfg.m < 1)  // rows too wide for half an SM: the whole budget, one CTA per SM
      cfg.m = (int)std::min<uint32_t>(3u, (kBudget - cfg.data_off) / (kWarps * cfg.slot_bytes));
    if (cfg.m < 1) return fail(JO_ERR_SHAPE, "timestep_mlp: rows too large to stage");
    const size_t smem = cfg.data_off + (size_t)kWarps * cfg.m * cfg.slot_bytes;
    // CTAs: one per SM (fewer only when there are fewer units than SMs)
    const int64_t units = cdiv(a.N, cfg.rows_per_unit);
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(di->sm_count, units));
    int s = JO_OK;
    switch (kb) {
      case 1: s = launch_one<1, kSinIn, kSilu>(a, cfg, b0, grid, smem, st, di); break;
      case 2: s = launch_one<2, kSinIn, kSilu>(a, cfg, b0, grid, smem, st, di); break;
      case 4: s = launch_one<4, kSinIn, kSilu>(a, cfg, b0, grid, smem, st, di); break;
      default: s = launch_one<8, kSinIn, kSilu>(a, cfg, b0, grid, smem, st, di); break;
    }
    if (s) return s;
    if (int e = after_launch("temb_layer_kernel")) return e;
  }
  return JO_OK;
}

}  // namespace

// Shared by the entry points: checks, then the three layers with s1 / s2 at
// scratch and scratch + B * dim.
int timestep_mlp_run(void* vec, const float* t, int64_t batch, const void* w1, const void* b1,
                     int64_t freq_dim, int64_t dim, const void* w2, const void* b2, const void* w3,
                     const void* b3, int64_t proj_dim, __nv_bfloat16* scratch, float max_period,
                     cudaStream_t st, const DeviceInfo* di, const void* tables, void* mods, int64_t n_tables) {
  TembLayer l{};
  l.t = t;
  l.B = (int)batch;
  l.neg_log_period = (float)(-log((double)max_period));
  __nv_bfloat16* s1 = scratch;
  __nv_bfloat16* s2 = scratch + batch * dim;
  // layer 1: sinusoid -> linear_1 -> SiLU
  l.x = nullptr;
  l.w = reinterpret_cast<const __nv_bfloat16*>(w1);
  l.bias = reinterpret_cast<const __nv_bfloat16*>(b1);
  l.y = s1;
  l.K = (int)freq_dim;
  l.N = (int)dim;
  if (int s = launch_layer<true, true>(l, st, di)) return s;
  // layer 2: linear_2 -> SiLU (act_fn before time_proj)
  l.x = s1;
  l.w = reinterpret_cast<const __nv_bfloat16*>(w2);
  l.bias = reinterpret_cast<const __nv_bfloat16*>(b2);
  l.y = s2;
  l.K = (int)dim;
  l.N = (int)dim;
  if (JO_TEMB_PF_ROWS > 0) {  // time_proj's partition: one CTA per SM, 1 row per unit at dim >= 3072
    const int64_t r3 = std::max<int64_t>(1, 6144 / (dim * 2));
    const int64_t g3 = std::max<int64_t>(1, std::min<int64_t>(di->sm_count, cdiv(proj_dim, r3)));
    l.pf_w = reinterpret_cast<const __nv_bfloat16*>(w3);
    l.pf_per = cdiv(proj_dim, g3);
    l.pf_rows = JO_TEMB_PF_ROWS;
    l.pf_ctas = (int)g3;
    l.pf_row_bytes = (int)(dim * 2);
    l.pf_n = (int)proj_dim;
  }
  if (int s = launch_layer<false, true>(l, st, di)) return s;
  l.pf_w = nullptr;
  // layer 3: time_proj
  l.x = s2;
  l.w = reinterpret_cast<const __nv_bfloat16*>(w3);
  l.bias = reinterpret_cast<const __nv_bfloat16*>(b3);
  l.y = reinterpret_cast<__nv_bfloat16*>(vec);
  l.K = (int)dim;
  l.N = (int)proj_dim;
  l.tables = reinterpret_cast<const __nv_bfloat16*>(tables);
  l.mods = reinterpret_cast<__nv_bfloat16*>(mods);
  l.T = (int)n_tables;
  return launch_layer<false, false>(l, st, di);
}

int timestep_mlp_check(void* vec, const float* t, int64_t batch, const void* w1, int64_t freq_dim,
                       int64_t dim, const void* w2, const void* w3, int64_t proj_dim, float max_period) {
  const char* op = "timestep_mlp";
  if (batch < 0 || freq_dim < 2 || dim < 1 || proj_dim < 1) return fail(JO_ERR_SHAPE, "%s: bad sizes", op);
  if (freq_dim % 2 || freq_dim % 8 || dim % 8)
    return fail(JO_ERR_ALIGN, "%s: freq_dim and dim must be multiples of 8", op);
  if (freq_dim > kMaxK || dim > kMaxK)
    return fail(JO_ERR_SHAPE, "%s: freq_dim and dim must be <= %d", op, kMaxK);
  if (proj_dim > INT32_MAX || batch > INT32_MAX) return fail(JO_ERR_SHAPE, "%s: size too large", op);
  if (!vec || !t || !w1 || !w2 || !w3) return fail(JO_ERR_INVALID, "%s: null operand", op);
  if (!aligned16(w1) || !aligned16(w2) || !aligned16(w3))
    return fail(JO_ERR_ALIGN, "%s: weights must be 16-byte aligned", op);
  if (!(max_period > 0.f)) return fail(JO_ERR_INVALID, "%s: max_period must be > 0", op);
  return JO_OK;
}

}  // namespace jo

using namespace jo;

extern "C" {

int jo_timestep_mlp(void* vec, const float* t, int64_t batch, const void* w1, const void* b1,
                    int64_t freq_dim, int64_t dim, const void* w2, const void* b2, const void* w3,
                    const void* b3, int64_t proj_dim, void* scratch, int64_t scratch_bytes,
                    float max_period, void* stream) {
  const DeviceInfo* di;
  if (int s = device_info(&di)) return s;
  if (int s = timestep_mlp_check(vec, t, batch, w1, freq_dim, dim, w2, w3, proj_dim, max_period)) return s;
  if (batch == 0) return JO_OK;
  if (!scratch || !aligned16(scratch)) return fail(JO_ERR_ALIGN, "timestep_mlp: scratch must be 16-byte aligned");
  if (scratch_bytes < 4 * batch * dim)
    return fail(JO_ERR_SHAPE, "timestep_mlp: scratch needs %lld bytes, got %lld", (long long)(4 * batch * dim),
                (long long)scratch_bytes);
  return timestep_mlp_run(vec, t, batch, w1, b1, freq_dim, dim, w2, b2, w3, b3, proj_dim,
                          reinterpret_cast<__nv_bfloat16*>(scratch), max_period, (cudaStream_t)stream, di, nullptr,
                          nullptr, 0);
}

int jo_timestep_mlp_modulate(void* vec, void* mods, const void* tables, int64_t n_tables, const float* t,
                             int64_t batch, const void* w1, const void* b1, int64_t freq_dim, int64_t dim,
                             const void* w2, const void* b2, const void* w3, const void* b3, int64_t proj_dim,
                             void* scratch, int64_t scratch_bytes, float max_period, void* stream) {
  const char* op = "timestep_mlp_modulate";
  const DeviceInfo* di;
  if (int s = device_info(&di)) return s;
  if (int s = timestep_mlp_check(vec, t, batch, w1, freq_dim, dim, w2, w3, proj_dim, max_period)) return s;
  if (n_tables < 0 || n_tables > INT32_MAX) return fail(JO_ERR_SHAPE, "%s: bad table count", op);
  if (n_tables > 0 && (!tables || !mods)) return fail(JO_ERR_INVALID, "%s: null tables / mods", op);
  if (n_tables * batch * proj_dim > INT64_MAX / 2) return fail(JO_ERR_SHAPE, "%s: output too large", op);
  if (batch == 0) return JO_OK;
  if (!scratch || !aligned16(scratch)) return fail(JO_ERR_ALIGN, "%s: scratch must be 16-byte aligned", op);
  if (scratch_bytes < 4 * batch * dim)
    return fail(JO_ERR_SHAPE, "%s: scratch needs %lld bytes, got %lld", op, (long long)(4 * batch * dim),
                (long long)scratch_bytes);
  return timestep_mlp_run(vec, t, batch, w1, b1, freq_dim, dim, w2, b2, w3, b3, proj_dim,
                          reinterpret_cast<__nv_bfloat16*>(scratch), max_period, (cudaStream_t)stream, di, tables,
                          mods, n_tables);
}

// ---------------------------------------------------------------------------
// Allocation-free variant: the scratch is a file-scope device array of a fixed
// size, shared by every call on a device.
constexpr int64_t kStaticScratchElems = 2 * 16 * 4096;  // s1 + s2 for batch * dim <= 65536 (256 KB)
static __device__ __align__(256) __nv_bfloat16 g_temb_scratch[kStaticScratchElems];

int jo_timestep_mlp_noalloc(void* vec, const float* t, int64_t batch, const void* w1, const void* b1,
                            int64_t freq_dim, int64_t dim, const void* w2, const void* b2, const void* w3,
                            const void* b3, int64_t proj_dim, float max_period, void* stream) {
  const DeviceInfo* di;
  if (int s = device_info(&di)) return s;
  if (int s = timestep_mlp_check(vec, t, batch, w1, freq_dim, dim, w2, w3, proj_dim, max_period)) return s;
  if (batch == 0) return JO_OK;
  if (2 * batch * dim > kStaticScratchElems)
    return fail(JO_ERR_SHAPE, "timestep_mlp_noalloc: batch * dim = %lld exceeds the static scratch limit of %lld",
                (long long)(batch * dim), (long long)(kStaticScratchElems / 2));
  // the array's address on the current device: looked up on the first call on each
  // device (and again if the device's context is re-created), cached otherwise
  static SymbolCache cache;
  void* ptr = nullptr;
  if (int s = symbol_address(cache, g_temb_scratch, di->ordinal, (cudaStream_t)stream, &ptr, "timestep_mlp_noalloc"))
    return s;
  return timestep_mlp_run(vec, t, batch, w1, b1, freq_dim, dim, w2, b2, w3, b3, proj_dim,
                          reinterpret_cast<__nv_bfloat16*>(ptr), max_period, (cudaStream_t)stream, di, nullptr, nullptr, 0);
}

}  // extern "C"
