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
// one HBM stream: a warp owns one output row at a time, issues all of its 16-byte
// weight loads (up to 4096 elements) before the first use, and multiplies them
// against the batch's input rows staged once per CTA in shared memory; one warp
// shuffle reduction per batch row.  The two intermediates live in caller-owned
// scratch (4 * B * dim bytes) between the launches; the sinusoid is computed in
// the first layer's prologue.
#include <math.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace jo {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxK = 4096;            // input features per layer (16 x 256)
constexpr int kJ = kMaxK / 256;         // 16-byte weight vectors per lane per row

struct TembLayer {
  const __nv_bfloat16* x;  // [B, K] input rows (null for the sinusoid layer)
  const float* t;          // [B] timesteps (sinusoid layer)
  const __nv_bfloat16* w;  // [N, K] row-major
  const __nv_bfloat16* bias;  // [N] or null
  __nv_bfloat16* y;        // [B, N]
  int K, N, B;
  float neg_log_period;    // -ln(max_period) rounded to fp32
};

__device__ __forceinline__ float silu_exact(float v) { return v / (1.f + expf(-v)); }

// One layer for batch rows [b0, b0 + kB) (rows >= B are skipped).
template <int kB, bool kSinIn, bool kSilu>
__global__ void __launch_bounds__(kThreads) temb_layer_kernel(const TembLayer a, int b0) {
  extern __shared__ __align__(16) __nv_bfloat16 xs[];  // [kB, K]
  const int K = a.K;
  // ---- stage the batch's input rows
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

  const int lane = threadIdx.x & 31;
  const int warps = (int)(gridDim.x * kThreads / 32);
  for (int n = (int)(blockIdx.x * kThreads + threadIdx.x) / 32; n < a.N; n += warps) {
    const __nv_bfloat16* wr = a.w + (int64_t)n * K;
    uint4 w[kJ];
#pragma unroll
    for (int j = 0; j < kJ; ++j) {
      const int k = j * 256 + lane * 8;
      w[j] = k < K ? ld_stream(wr + k) : make_uint4(0, 0, 0, 0);
    }
    float acc[kB];
#pragma unroll
    for (int b = 0; b < kB; ++b) acc[b] = 0.f;
#pragma unroll
    for (int j = 0; j < kJ; ++j) {
      const int k = j * 256 + lane * 8;
      if (k >= K) continue;
      float wf[8];
      Elt<__nv_bfloat16>::unpack(w[j], wf);
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        float xf[8];
        Elt<__nv_bfloat16>::unpack(*reinterpret_cast<const uint4*>(xs + b * K + k), xf);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[b] = fmaf(wf[e], xf[e], acc[b]);
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
}

template <bool kSinIn, bool kSilu>
int launch_layer(const TembLayer& a, cudaStream_t st, const DeviceInfo* di) {
  for (int b0 = 0; b0 < a.B; b0 += 8) {
    const int nb = std::min(8, a.B - b0);
    const int kb = nb <= 1 ? 1 : (nb <= 2 ? 2 : (nb <= 4 ? 4 : 8));
    const size_t smem = (size_t)kb * a.K * 2;
    const int64_t need = cdiv((int64_t)a.N * 32, (int64_t)kThreads);  // one warp per output row
    auto go = [&](auto kern) -> int {
      // the staged input rows take up to 8 x 4096 bf16 = 64 KB of shared memory
      if (smem > 48 * 1024 &&
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return fail(JO_ERR_CUDA, "timestep_mlp: cannot reserve %zu bytes of shared memory", smem);
      // one wave: the resident CTAs walk the rows with a grid stride
      const int64_t cap = (int64_t)di->sm_count * std::max(1, occupancy((const void*)kern, kThreads, smem));
      kern<<<(unsigned)std::min(need, cap), kThreads, smem, st>>>(a, b0);
      return JO_OK;
    };
    int s = JO_OK;
    switch (kb) {
      case 1: s = go(temb_layer_kernel<1, kSinIn, kSilu>); break;
      case 2: s = go(temb_layer_kernel<2, kSinIn, kSilu>); break;
      case 4: s = go(temb_layer_kernel<4, kSinIn, kSilu>); break;
      default: s = go(temb_layer_kernel<8, kSinIn, kSilu>); break;
    }
    if (s) return s;
    if (int s = after_launch("temb_layer_kernel")) return s;
  }
  return JO_OK;
}

}  // namespace

// Shared by the entry points: checks, then the three layers with s1 / s2 at
// scratch and scratch + B * dim.
int timestep_mlp_run(void* vec, const float* t, int64_t batch, const void* w1, const void* b1,
                     int64_t freq_dim, int64_t dim, const void* w2, const void* b2, const void* w3,
                     const void* b3, int64_t proj_dim, __nv_bfloat16* scratch, float max_period,
                     cudaStream_t st, const DeviceInfo* di) {
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
  if (int s = launch_layer<false, true>(l, st, di)) return s;
  // layer 3: time_proj
  l.x = s2;
  l.w = reinterpret_cast<const __nv_bfloat16*>(w3);
  l.bias = reinterpret_cast<const __nv_bfloat16*>(b3);
  l.y = reinterpret_cast<__nv_bfloat16*>(vec);
  l.K = (int)dim;
  l.N = (int)proj_dim;
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
                          reinterpret_cast<__nv_bfloat16*>(scratch), max_period, (cudaStream_t)stream, di);
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
  // the array's address on the current device, looked up once per device
  static std::mutex mu;
  static void* addr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(JO_ERR_CUDA, "timestep_mlp_noalloc: no current device");
  void* ptr;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
      const cudaError_t e = cudaGetSymbolAddress(&addr[dev], g_temb_scratch);
      if (e != cudaSuccess) {
        addr[dev] = nullptr;
        return fail(JO_ERR_CUDA, "timestep_mlp_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      }
    }
    ptr = addr[dev];
  }
  return timestep_mlp_run(vec, t, batch, w1, b1, freq_dim, dim, w2, b2, w3, b3, proj_dim,
                          reinterpret_cast<__nv_bfloat16*>(ptr), max_period, (cudaStream_t)stream, di);
}

}  // extern "C"
