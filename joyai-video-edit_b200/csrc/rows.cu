// Row kernels: every op here reads whole rows of an [rows, cols] activation,
// optionally reduces over the row, and writes per-element results.
//
//   rmsnorm                          joyomni_ops/csrc/rmsnorm.cu:60-126
//   fused_norm_scale_shift           joyomni_ops/csrc/fused_norm_scale_shift.cu:226-403
//   gated residual (torch.addcmul)   deploy/xvideo/models/dit/sgl_fused_ops.py:302-305
//   gated residual + norm + modulate deploy/xvideo/models/dit/dit.py:525-534
//   per-token FP8 quant              deploy/xvideo/models/dit/fp8_linear.py:38-43
//   rmsnorm / norm+modulate -> FP8   (fusions of the above)
//
// Design (B200): the ops are HBM-bound, so each row is read from HBM exactly
// once, kept in registers across the reduction(s), and written once with
// 16-byte stores.  Rows of up to 512 vectors (4096 bf16) stream through a
// shared-memory ring filled by 1-D TMA bulk copies (one producer warp, eight
// consumer warps, one row per consumer at a time, reductions by warp shuffle):
// the loads in flight are held by the copy engine, not by registers, so each
// SM keeps ~192 KB of rows in flight while its warps compute.  Longer rows are
// owned by a CTA with direct 16-byte loads; shapes that break 16-byte
// alignment take a scalar block-per-row path.
#include "pipeline.cuh"

namespace jo {
namespace {

enum NormKind { kNoNorm = 0, kLayer = 1, kRms = 2 };
enum ProKind { kLoadX = 0, kResidGate = 1 };
enum EpiKind { kStoreY = 0, kQuantY = 1, kNoY = 2 };

struct RowArgs {
  void* out;
  int64_t out_stride;
  uint8_t* out_q;
  int64_t q_stride;
  float* out_s;
  void* out_h;
  int64_t h_stride;
  const void* x;
  int64_t x_stride;
  const void* res;
  int64_t res_stride;
  const void* gate;
  int64_t gate_stride;  // 0 => one gate row broadcast over all rows
  const void* gamma;
  const void* beta;
  const void* scale;
  const void* shift;
  int64_t mod_stride;  // 0 => one modulation row broadcast over all rows
  int64_t rows;
  int64_t cols;
  float eps;
};

// Reduction over the threads that own one row.
template <bool kWarp>
__device__ __forceinline__ float row_reduce_sum(float v, float* smem) {
  v = warp_sum(v);
  if constexpr (kWarp) {
    return v;
  } else {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();  // smem may still be read by a previous reduction
    if (l == 0) smem[w] = v;
    __syncthreads();
    return warp_sum(l < nw ? smem[l] : 0.f);
  }
}
template <bool kWarp>
__device__ __forceinline__ float row_reduce_max(float v, float* smem) {
  v = warp_max(v);
  if constexpr (kWarp) {
    return v;
  } else {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (l == 0) smem[w] = v;
    __syncthreads();
    return warp_max(l < nw ? smem[l] : 0.f);
  }
}

// Per-element norm + affine + modulation (fused_norm_scale_shift.cu:296-307,
// rmsnorm.cu:81): LayerNorm ((x-mean)*rstd*g + b)*(1+sc)+sh, RMS (x*rstd*g)*(1+sc)+sh.
template <int kNorm>
__device__ __forceinline__ float norm_elem(float x, float mean, float rstd, float g, float b,
                                           float sc, float sh, bool has_g, bool has_b,
                                           bool has_mod) {
  float n;
  if constexpr (kNorm == kLayer) {
    n = (x - mean) * rstd;
    if (has_g) n = n * g;
    if (has_b) n = n + b;
  } else if constexpr (kNorm == kRms) {
    n = x * rstd;
    if (has_g) n = n * g;
  } else {
    n = x;
  }
  if (has_mod) n = n * (1.f + sc) + sh;
  return n;
}

// ------------------------------------------------------------------ row math
// Everything after the row is in registers: (gated residual), reductions,
// per-element norm/modulation, store or FP8 quantisation.  `raw` holds x (or
// the residual in kResidGate mode, where `xv` holds x); vector idx = g + i*G.
// h = residual + x * gate for one vector, rounded to T (the tensor the model
// materialises), and written to out_h.
template <typename T>
__device__ __forceinline__ uint4 resid_vec(const RowArgs& a, int64_t row, int idx, const uint4& xv,
                                           const uint4& rv) {
  constexpr int V = Elt<T>::kVec;
  const T* gr = reinterpret_cast<const T*>(a.gate) + row * a.gate_stride;
  float fx[V], fr[V], fg[V], fh[V];
  Elt<T>::unpack(xv, fx);
  Elt<T>::unpack(rv, fr);
  Elt<T>::unpack(ld_bcast(gr + (int64_t)idx * V), fg);
#pragma unroll
  for (int j = 0; j < V; ++j) fh[j] = fr[j] + fx[j] * fg[j];
  const uint4 h = Elt<T>::pack(fh);
  st_global(reinterpret_cast<T*>(a.out_h) + row * a.h_stride + (int64_t)idx * V, h);
  return h;
}

// kHDone: the caller already formed h (kResidGate) into raw and stored it.
template <typename T, int kVPT, int kNorm, int kPro, int kEpi, bool kWarp, bool kHDone = false>
__device__ __forceinline__ void row_math(const RowArgs& a, int64_t row, uint4 (&raw)[kVPT],
                                         const uint4 (&xv)[kVPT], int g, int G, float* smem) {
  constexpr int V = Elt<T>::kVec;
  const int nvec = (int)(a.cols / V);
  if constexpr (kPro == kResidGate && !kHDone) {
#pragma unroll
    for (int i = 0; i < kVPT; ++i) {
      const int idx = g + i * G;
      if (idx < nvec) raw[i] = resid_vec<T>(a, row, idx, xv[i], raw[i]);
    }
  }
  if constexpr (kEpi == kNoY) return;

  float mean = 0.f, rstd = 1.f;
  if constexpr (kNorm == kLayer) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kVPT; ++i) {
      if (g + i * G < nvec) {
        float f[V];
        Elt<T>::unpack(raw[i], f);
#pragma unroll
        for (int j = 0; j < V; ++j) s += f[j];
      }
    }
    mean = __fdiv_rn(row_reduce_sum<kWarp>(s, smem), (float)a.cols);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < kVPT; ++i) {
      if (g + i * G < nvec) {
        float f[V];
        Elt<T>::unpack(raw[i], f);
#pragma unroll
        for (int j = 0; j < V; ++j) {
          const float d = f[j] - mean;
          q += d * d;
        }
      }
    }
    rstd = rsqrt_ieee(__fdiv_rn(row_reduce_sum<kWarp>(q, smem), (float)a.cols) + a.eps);
  } else if constexpr (kNorm == kRms) {
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < kVPT; ++i) {
      if (g + i * G < nvec) {
        float f[V];
        Elt<T>::unpack(raw[i], f);
#pragma unroll
        for (int j = 0; j < V; ++j) q += f[j] * f[j];
      }
    }
    rstd = rsqrt_ieee(__fdiv_rn(row_reduce_sum<kWarp>(q, smem), (float)a.cols) + a.eps);
  }

  const bool has_g = a.gamma != nullptr, has_b = a.beta != nullptr, has_mod = a.scale != nullptr;
  const T* gam = reinterpret_cast<const T*>(a.gamma);
  const T* bet = reinterpret_cast<const T*>(a.beta);
  const T* scr = has_mod ? reinterpret_cast<const T*>(a.scale) + row * a.mod_stride : nullptr;
  const T* shr = has_mod ? reinterpret_cast<const T*>(a.shift) + row * a.mod_stride : nullptr;
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kVPT; ++i) {
    const int idx = g + i * G;
    if (idx < nvec) {
      float f[V], fg[V], fb[V], fs[V], fh[V], y[V];
      Elt<T>::unpack(raw[i], f);
      if (has_g) Elt<T>::unpack(ld_bcast(gam + (int64_t)idx * V), fg);
      if (has_b) Elt<T>::unpack(ld_bcast(bet + (int64_t)idx * V), fb);
      if (has_mod) {
        Elt<T>::unpack(ld_bcast(scr + (int64_t)idx * V), fs);
        Elt<T>::unpack(ld_bcast(shr + (int64_t)idx * V), fh);
      }
#pragma unroll
      for (int j = 0; j < V; ++j)
        y[j] = norm_elem<kNorm>(f[j], mean, rstd, fg[j], fb[j], fs[j], fh[j], has_g, has_b, has_mod);
      if constexpr (kEpi == kStoreY) {
        T* orow = reinterpret_cast<T*>(a.out) + row * a.out_stride;
        st_global(orow + (int64_t)idx * V, Elt<T>::pack(y));
      } else {
        raw[i] = Elt<T>::pack(y);  // y rounded to T, as the unfused chain materialises it
        float r[V];
        Elt<T>::unpack(raw[i], r);
#pragma unroll
        for (int j = 0; j < V; ++j) amax = fmaxf(amax, fabsf(r[j]));
      }
    }
  }
  if constexpr (kEpi == kQuantY) {
    const float s = quant_scale(row_reduce_max<kWarp>(amax, smem));
    uint8_t* qrow = a.out_q + row * a.q_stride;
#pragma unroll
    for (int i = 0; i < kVPT; ++i) {
      const int idx = g + i * G;
      if (idx < nvec) {
        float r[V];
        Elt<T>::unpack(raw[i], r);
        if constexpr (V == 8) {
          uint2 o;
          o.x = (uint32_t)e4m3x2(quant_clamp(r[0], s), quant_clamp(r[1], s)) |
                ((uint32_t)e4m3x2(quant_clamp(r[2], s), quant_clamp(r[3], s)) << 16);
          o.y = (uint32_t)e4m3x2(quant_clamp(r[4], s), quant_clamp(r[5], s)) |
                ((uint32_t)e4m3x2(quant_clamp(r[6], s), quant_clamp(r[7], s)) << 16);
          *reinterpret_cast<uint2*>(qrow + (int64_t)idx * 8) = o;
        } else {
          uint32_t o = (uint32_t)e4m3x2(quant_clamp(r[0], s), quant_clamp(r[1], s)) |
                       ((uint32_t)e4m3x2(quant_clamp(r[2], s), quant_clamp(r[3], s)) << 16);
          *reinterpret_cast<uint32_t*>(qrow + (int64_t)idx * 4) = o;
        }
      }
    }
    if (g == 0) a.out_s[row] = s;
  }
}

// ------------------------------------------------------------------ staged path
// Rows of up to 512 vectors (4096 bf16).  One producer warp keeps a ring of
// rows in flight with 1-D bulk copies (TMA) into shared memory; kConsumers
// warps each take every kConsumers-th row of the CTA's contiguous chunk, read
// it into registers, release the slot at once, and compute + store.  The
// prefetch depth lives in shared memory, not in registers.  One CTA per SM.
constexpr int kConsumers = 12;
constexpr int kStagedThreads = (kConsumers + 1) * 32;

template <typename T, int kVPT, int kNorm, int kPro, int kEpi>
__global__ void __launch_bounds__(kStagedThreads, 1)
    row_staged_kernel(const RowArgs a, int slots, uint32_t slot_bytes, unsigned int* fault) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ float red[32];
  constexpr int V = Elt<T>::kVec;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t per = (a.rows + gridDim.x - 1) / gridDim.x;
  const int64_t r0 = (int64_t)blockIdx.x * per;
  const int64_t rend = r0 + per < a.rows ? r0 + per : a.rows;
  const int units = rend > r0 ? (int)(rend - r0) : 0;
  const int nvec = (int)(a.cols / V);
  const uint32_t row_bytes = (uint32_t)nvec * 16u;
  const uint32_t base = smem_u32(smem_raw);
  Ring ring{base + (uint32_t)(((2 * slots * 8) + 127) & ~127), base, slot_bytes, slots};
  if (threadIdx.x == 0) {
    for (int s = 0; s < slots; ++s) {
      mbar_init(ring.full(s), 1);
      mbar_init(ring.empty(s), 1);
    }
    mbar_init_fence();
  }
  __syncthreads();
  if (warp == kConsumers) {
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < units; ++i) {
        if (!mbar_wait(ring.empty(i), ring.parity(i) ^ 1u, fault)) break;
        const int64_t row = r0 + i;
        if constexpr (kPro == kLoadX) {
          mbar_expect_tx(ring.full(i), row_bytes);
          bulk_load(ring.slot(i), reinterpret_cast<const T*>(a.x) + row * a.x_stride, row_bytes, ring.full(i));
        } else {
          mbar_expect_tx(ring.full(i), 2 * row_bytes);
          bulk_load(ring.slot(i), reinterpret_cast<const T*>(a.x) + row * a.x_stride, row_bytes, ring.full(i));
          bulk_load(ring.slot(i) + row_bytes, reinterpret_cast<const T*>(a.res) + row * a.res_stride, row_bytes,
                    ring.full(i));
        }
        issued = i + 1;
      }
      // the copies of the last window must land before the CTA may exit
      for (int i = issued > slots ? issued - slots : 0; i < issued; ++i) mbar_wait(ring.full(i), ring.parity(i), fault);
    }
    return;
  }
  for (int i = warp; i < units; i += kConsumers) {
    if (!mbar_wait(ring.full(i), ring.parity(i), fault)) break;
    uint4 raw[kVPT];
    const uint32_t sl = ring.slot(i);
#pragma unroll
    for (int k = 0; k < kVPT; ++k) {
      const int idx = lane + 32 * k;
      if (idx < nvec) {
        if constexpr (kPro == kLoadX)
          raw[k] = lds128(sl + idx * 16);
        else  // form h = residual + x * gate straight from the slot
          raw[k] = resid_vec<T>(a, r0 + i, idx, lds128(sl + idx * 16), lds128(sl + row_bytes + idx * 16));
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(ring.empty(i));  // slot free: the row is in registers
    row_math<T, kVPT, kNorm, kPro, kEpi, true, true>(a, r0 + i, raw, raw, lane, 32, red);
  }
}

// ------------------------------------------------------------------ long rows
// One CTA per row, loads straight from global memory into registers.
template <typename T, int kVPT, int kNorm, int kPro, int kEpi>
__global__ void __launch_bounds__(kVPT <= 4 ? 1024 : (kVPT <= 8 ? 512 : 256))
    row_block_kernel(const RowArgs a) {
  constexpr int V = Elt<T>::kVec;
  __shared__ float smem[32];
  const int G = blockDim.x, g = threadIdx.x;
  const int64_t row = blockIdx.x;
  const int nvec = (int)(a.cols / V);
  uint4 raw[kVPT], xv[kVPT];
  const T* xr = reinterpret_cast<const T*>(a.x) + row * a.x_stride;
  const T* rr = reinterpret_cast<const T*>(a.res) + row * a.res_stride;
#pragma unroll
  for (int i = 0; i < kVPT; ++i) {
    const int idx = g + i * G;
    if (idx < nvec) {
      if constexpr (kPro == kLoadX) {
        raw[i] = ld_stream(xr + (int64_t)idx * V);
      } else {
        xv[i] = ld_stream(xr + (int64_t)idx * V);
        raw[i] = ld_stream(rr + (int64_t)idx * V);
      }
    }
  }
  row_math<T, kVPT, kNorm, kPro, kEpi, false>(a, row, raw, xv, g, G, smem);
}

// ------------------------------------------------------------------ scalar path
// Any alignment, any cols.  One CTA per row; the row is re-read from global
// memory for each pass (LayerNorm: 3 passes, quant: +1).
template <typename T>
__device__ __forceinline__ float ldf(const void* base, int64_t i) {
  return Elt<T>::to_f(reinterpret_cast<const T*>(base)[i]);
}

template <typename T, int kNorm, int kPro, int kEpi>
__global__ void __launch_bounds__(256) row_scalar_kernel(const RowArgs a) {
  __shared__ float smem[32];
  const int64_t row = blockIdx.x;
  const int g = threadIdx.x, G = blockDim.x, n = (int)a.cols;
  const T* src = reinterpret_cast<const T*>(a.x) + row * a.x_stride;
  if constexpr (kPro == kResidGate) {
    const T* xr = src;
    const T* rr = reinterpret_cast<const T*>(a.res) + row * a.res_stride;
    const T* gr = reinterpret_cast<const T*>(a.gate) + row * a.gate_stride;
    T* hr = reinterpret_cast<T*>(a.out_h) + row * a.h_stride;
    for (int c = g; c < n; c += G)
      hr[c] = Elt<T>::from_f(Elt<T>::to_f(rr[c]) + Elt<T>::to_f(xr[c]) * Elt<T>::to_f(gr[c]));
    src = hr;  // each thread re-reads only the elements it wrote itself
  }
  if constexpr (kEpi == kNoY) return;
  float mean = 0.f, rstd = 1.f;
  if constexpr (kNorm == kLayer) {
    float s = 0.f;
    for (int c = g; c < n; c += G) s += Elt<T>::to_f(src[c]);
    mean = __fdiv_rn(row_reduce_sum<false>(s, smem), (float)n);
    float q = 0.f;
    for (int c = g; c < n; c += G) {
      const float d = Elt<T>::to_f(src[c]) - mean;
      q += d * d;
    }
    rstd = rsqrt_ieee(__fdiv_rn(row_reduce_sum<false>(q, smem), (float)n) + a.eps);
  } else if constexpr (kNorm == kRms) {
    float q = 0.f;
    for (int c = g; c < n; c += G) {
      const float v = Elt<T>::to_f(src[c]);
      q += v * v;
    }
    rstd = rsqrt_ieee(__fdiv_rn(row_reduce_sum<false>(q, smem), (float)n) + a.eps);
  }
  const bool has_g = a.gamma != nullptr, has_b = a.beta != nullptr, has_mod = a.scale != nullptr;
  const T* scr = has_mod ? reinterpret_cast<const T*>(a.scale) + row * a.mod_stride : nullptr;
  const T* shr = has_mod ? reinterpret_cast<const T*>(a.shift) + row * a.mod_stride : nullptr;
  auto y_at = [&](int c) {
    return norm_elem<kNorm>(Elt<T>::to_f(src[c]), mean, rstd, has_g ? ldf<T>(a.gamma, c) : 1.f,
                            has_b ? ldf<T>(a.beta, c) : 0.f, has_mod ? Elt<T>::to_f(scr[c]) : 0.f,
                            has_mod ? Elt<T>::to_f(shr[c]) : 0.f, has_g, has_b, has_mod);
  };
  if constexpr (kEpi == kStoreY) {
    T* orow = reinterpret_cast<T*>(a.out) + row * a.out_stride;
    for (int c = g; c < n; c += G) orow[c] = Elt<T>::from_f(y_at(c));
  } else {
    float amax = 0.f;
    for (int c = g; c < n; c += G) amax = fmaxf(amax, fabsf(round_through<T>(y_at(c))));
    const float s = quant_scale(row_reduce_max<false>(amax, smem));
    uint8_t* qrow = a.out_q + row * a.q_stride;
    for (int c = g; c < n; c += G)
      qrow[c] = (uint8_t)(e4m3x2(quant_clamp(round_through<T>(y_at(c)), s), 0.f) & 0xff);
    if (g == 0) a.out_s[row] = s;
  }
}

// ------------------------------------------------------------------ dispatch
bool row_vec_ok(const RowArgs& a, int esize) {
  const int V = 16 / esize;
  if (a.cols % V) return false;
  const void* ptrs[] = {a.out, a.out_h, a.x, a.res, a.gate, a.gamma, a.beta, a.scale, a.shift};
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return false;
  const int64_t strides[] = {a.out_stride, a.h_stride, a.x_stride, a.res_stride, a.gate_stride,
                             a.mod_stride};
  for (int64_t s : strides)
    if ((s * esize) % 16) return false;
  if (a.out_q && (!aligned16(a.out_q) || (a.q_stride % 8))) return false;
  return true;
}

template <typename T, int kVPT, int kNorm, int kPro, int kEpi>
int launch_staged(const RowArgs& a, cudaStream_t st, const DeviceInfo* di) {
  auto kern = row_staged_kernel<T, kVPT, kNorm, kPro, kEpi>;
  const uint32_t row_bytes = (uint32_t)(a.cols * sizeof(T)) * (kPro == kResidGate ? 2u : 1u);
  const uint32_t slot_bytes = (row_bytes + 127u) & ~127u;
  // ~192 KB of ring per CTA (one CTA per SM).  The slot count is a multiple of
  // kConsumers so that every slot is only ever used by one consumer warp (unit
  // i -> warp i % kConsumers, slot i % slots): a warp then never waits on a
  // slot more than one phase ahead, which a parity wait could not tell apart.
  int slots = (int)((192u * 1024u) / slot_bytes) / kConsumers * kConsumers;
  if (slots < kConsumers) slots = kConsumers;
  if (slots > 4 * kConsumers) slots = 4 * kConsumers;
  const size_t smem = (size_t)slots * slot_bytes + ((2 * slots * 8 + 127) & ~127);
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024) != cudaSuccess)
      return fail(JO_ERR_CUDA, "row kernel: cannot reserve shared memory");
    attr = true;
  }
  const int occ = occupancy((const void*)kern, kStagedThreads, smem);
  int64_t grid = (int64_t)di->sm_count * occ;
  const int64_t min_rows_per_cta = 4;
  if (grid * min_rows_per_cta > a.rows) grid = cdiv(a.rows, min_rows_per_cta);
  if (grid < 1) grid = 1;
  kern<<<(unsigned)grid, kStagedThreads, smem, st>>>(a, slots, slot_bytes, di->fault);
  return after_launch("row_staged_kernel");
}

template <typename T, int kVPT, int kNorm, int kPro, int kEpi>
int launch_block(const RowArgs& a, int threads, cudaStream_t st) {
  row_block_kernel<T, kVPT, kNorm, kPro, kEpi><<<(unsigned)a.rows, threads, 0, st>>>(a);
  return after_launch("row_block_kernel");
}

template <typename T, int kNorm, int kPro, int kEpi>
int launch_rows_t(const RowArgs& a, cudaStream_t st) {
  constexpr int V = Elt<T>::kVec;
  if (a.rows == 0 || a.cols == 0) return JO_OK;
  const DeviceInfo* di;
  if (int s = device_info(&di)) return s;
  if (row_vec_ok(a, sizeof(T))) {
    const int nvec = (int)(a.cols / V);
    if (nvec <= 32 * 16) {
      const int per = (nvec + 31) / 32;
#define JO_STAGED(VPT) return launch_staged<T, VPT, kNorm, kPro, kEpi>(a, st, di)
      if (per <= 1) JO_STAGED(1);
      if (per <= 2) JO_STAGED(2);
      if (per <= 4) JO_STAGED(4);
      if (per <= 8) JO_STAGED(8);
      if (per <= 12) JO_STAGED(12);
      JO_STAGED(16);
#undef JO_STAGED
    }
    if (nvec <= 256 * 16) {
#define JO_BLOCK(VPT, MAXTH)                                                                   \
  do {                                                                                         \
    const int th = (int)(((nvec + VPT - 1) / VPT + 31) / 32 * 32);                             \
    if (th <= MAXTH) return launch_block<T, VPT, kNorm, kPro, kEpi>(a, th, st);                \
  } while (0)
      JO_BLOCK(4, 1024);
      JO_BLOCK(8, 512);
      JO_BLOCK(16, 256);
#undef JO_BLOCK
    }
  }
  row_scalar_kernel<T, kNorm, kPro, kEpi><<<(unsigned)a.rows, 256, 0, st>>>(a);
  return after_launch("row_scalar_kernel");
}

template <int kNorm, int kPro, int kEpi>
int launch_rows(int dtype, const RowArgs& a, cudaStream_t st, bool allow_f32) {
  switch (dtype) {
    case JO_BF16: return launch_rows_t<__nv_bfloat16, kNorm, kPro, kEpi>(a, st);
    case JO_F16: return launch_rows_t<__half, kNorm, kPro, kEpi>(a, st);
    case JO_F32:
      if (allow_f32) return launch_rows_t<float, kNorm, kPro, kEpi>(a, st);
      // The quantising epilogues accept 16-bit input only (per_token_quant_fp8.cu:168-175).
      return fail(JO_ERR_DTYPE, "float32 input is not supported by this op; use bf16 or fp16");
    default: return fail(JO_ERR_DTYPE, "unsupported dtype code %d", dtype);
  }
}

int check_common(const RowArgs& a, const char* op) {
  const DeviceInfo* di;
  if (int s = device_info(&di)) return s;
  if (a.rows < 0 || a.cols < 0) return fail(JO_ERR_SHAPE, "%s: negative size", op);
  if (a.cols > (int64_t)INT32_MAX / 2) return fail(JO_ERR_SHAPE, "%s: cols too large", op);
  if (a.rows > (int64_t)INT32_MAX) return fail(JO_ERR_SHAPE, "%s: rows too large", op);
  if (a.rows > 0 && a.cols > 0 && !a.x) return fail(JO_ERR_INVALID, "%s: x is null", op);
  return JO_OK;
}

int mod_setup(RowArgs& a, const void* scale, const void* shift, int64_t mod_rows,
              int64_t mod_row_stride, int64_t rows, const char* op) {
  if (!scale && !shift) {
    a.scale = a.shift = nullptr;
    a.mod_stride = 0;
    return JO_OK;
  }
  if (!scale || !shift) return fail(JO_ERR_INVALID, "%s: scale and shift must both be given", op);
  if (mod_rows != 1 && mod_rows != rows)
    return fail(JO_ERR_SHAPE, "%s: scale/shift rows must be 1 (broadcast) or %lld, got %lld", op,
                (long long)rows, (long long)mod_rows);
  a.scale = scale;
  a.shift = shift;
  a.mod_stride = (mod_rows == 1) ? 0 : mod_row_stride;
  return JO_OK;
}

int norm_code(int norm, const char* op) {
  if (norm == JO_NORM_LAYER) return kLayer;
  if (norm == JO_NORM_RMS) return kRms;
  return fail(JO_ERR_INVALID, "%s: norm must be 0 (layer) or 1 (rms), got %d", op, norm);
}

}  // namespace
}  // namespace jo

using namespace jo;

extern "C" {

int jo_rmsnorm(void* out, int64_t out_row_stride, const void* x, int64_t x_row_stride,
               const void* weight, int64_t rows, int64_t cols, int dtype, float eps,
               void* stream) {
  RowArgs a{};
  a.out = out;
  a.out_stride = out_row_stride;
  a.x = x;
  a.x_stride = x_row_stride;
  a.gamma = weight;
  a.rows = rows;
  a.cols = cols;
  a.eps = eps;
  if (int s = check_common(a, "rmsnorm")) return s;
  if (rows > 0 && cols > 0 && (!out || !weight))
    return fail(JO_ERR_INVALID, "rmsnorm: out and weight must be non-null");
  return launch_rows<kRms, kLoadX, kStoreY>(dtype, a, (cudaStream_t)stream, true);
}

int jo_norm_scale_shift(void* out, int64_t out_row_stride, const void* x, int64_t x_row_stride,
                        const void* gamma, const void* beta, const void* scale,
                        const void* shift, int64_t mod_rows, int64_t mod_row_stride,
                        int64_t rows, int64_t cols, int norm, int dtype, float eps,
                        void* stream) {
  RowArgs a{};
  a.out = out;
  a.out_stride = out_row_stride;
  a.x = x;
  a.x_stride = x_row_stride;
  a.gamma = gamma;
  a.beta = beta;
  a.rows = rows;
  a.cols = cols;
  a.eps = eps;
  if (int s = check_common(a, "norm_scale_shift")) return s;
  if (rows > 0 && cols > 0 && !out) return fail(JO_ERR_INVALID, "norm_scale_shift: out is null");
  if (!scale || !shift) return fail(JO_ERR_INVALID, "norm_scale_shift: scale/shift are required");
  if (int s = mod_setup(a, scale, shift, mod_rows, mod_row_stride, rows, "norm_scale_shift")) return s;
  const int nk = norm_code(norm, "norm_scale_shift");
  if (nk < 0) return nk;
  if (nk == kRms) a.beta = nullptr;  // beta is a LayerNorm-only operand
  cudaStream_t st = (cudaStream_t)stream;
  return nk == kLayer ? launch_rows<kLayer, kLoadX, kStoreY>(dtype, a, st, true)
                      : launch_rows<kRms, kLoadX, kStoreY>(dtype, a, st, true);
}

int jo_per_token_quant_fp8(void* out_q, int64_t q_row_stride, float* out_s, const void* x,
                           int64_t x_row_stride, int64_t rows, int64_t cols, int dtype,
                           void* stream) {
  RowArgs a{};
  a.out_q = (uint8_t*)out_q;
  a.q_stride = q_row_stride;
  a.out_s = out_s;
  a.x = x;
  a.x_stride = x_row_stride;
  a.rows = rows;
  a.cols = cols;
  if (int s = check_common(a, "per_token_quant_fp8")) return s;
  if (rows > 0 && (!out_q || !out_s))
    return fail(JO_ERR_INVALID, "per_token_quant_fp8: outputs must be non-null");
  return launch_rows<kNoNorm, kLoadX, kQuantY>(dtype, a, (cudaStream_t)stream, false);
}

int jo_rmsnorm_quant_fp8(void* out_q, int64_t q_row_stride, float* out_s, const void* x,
                         int64_t x_row_stride, const void* weight, int64_t rows, int64_t cols,
                         int dtype, float eps, void* stream) {
  RowArgs a{};
  a.out_q = (uint8_t*)out_q;
  a.q_stride = q_row_stride;
  a.out_s = out_s;
  a.x = x;
  a.x_stride = x_row_stride;
  a.gamma = weight;
  a.rows = rows;
  a.cols = cols;
  a.eps = eps;
  if (int s = check_common(a, "rmsnorm_quant_fp8")) return s;
  if (rows > 0 && (!out_q || !out_s || !weight))
    return fail(JO_ERR_INVALID, "rmsnorm_quant_fp8: outputs and weight must be non-null");
  return launch_rows<kRms, kLoadX, kQuantY>(dtype, a, (cudaStream_t)stream, false);
}

int jo_norm_scale_shift_quant_fp8(void* out_q, int64_t q_row_stride, float* out_s,
                                  const void* x, int64_t x_row_stride, const void* gamma,
                                  const void* beta, const void* scale, const void* shift,
                                  int64_t mod_rows, int64_t mod_row_stride, int64_t rows,
                                  int64_t cols, int norm, int dtype, float eps, void* stream) {
  RowArgs a{};
  a.out_q = (uint8_t*)out_q;
  a.q_stride = q_row_stride;
  a.out_s = out_s;
  a.x = x;
  a.x_stride = x_row_stride;
  a.gamma = gamma;
  a.beta = beta;
  a.rows = rows;
  a.cols = cols;
  a.eps = eps;
  if (int s = check_common(a, "norm_scale_shift_quant_fp8")) return s;
  if (rows > 0 && (!out_q || !out_s))
    return fail(JO_ERR_INVALID, "norm_scale_shift_quant_fp8: outputs must be non-null");
  if (int s = mod_setup(a, scale, shift, mod_rows, mod_row_stride, rows, "norm_scale_shift_quant_fp8"))
    return s;
  const int nk = norm_code(norm, "norm_scale_shift_quant_fp8");
  if (nk < 0) return nk;
  if (nk == kRms) a.beta = nullptr;
  cudaStream_t st = (cudaStream_t)stream;
  return nk == kLayer ? launch_rows<kLayer, kLoadX, kQuantY>(dtype, a, st, false)
                      : launch_rows<kRms, kLoadX, kQuantY>(dtype, a, st, false);
}

int jo_gated_residual(void* out, int64_t out_row_stride, const void* residual,
                      int64_t res_row_stride, const void* x, int64_t x_row_stride,
                      const void* gate, int64_t gate_rows, int64_t gate_row_stride,
                      int64_t rows, int64_t cols, int dtype, void* stream) {
  RowArgs a{};
  a.out_h = out;
  a.h_stride = out_row_stride;
  a.x = x;
  a.x_stride = x_row_stride;
  a.res = residual;
  a.res_stride = res_row_stride;
  a.gate = gate;
  a.rows = rows;
  a.cols = cols;
  if (int s = check_common(a, "gated_residual")) return s;
  if (rows > 0 && cols > 0 && (!out || !residual || !gate))
    return fail(JO_ERR_INVALID, "gated_residual: null operand");
  if (gate_rows != 1 && gate_rows != rows)
    return fail(JO_ERR_SHAPE, "gated_residual: gate rows must be 1 or %lld", (long long)rows);
  a.gate_stride = gate_rows == 1 ? 0 : gate_row_stride;
  return launch_rows<kNoNorm, kResidGate, kNoY>(dtype, a, (cudaStream_t)stream, true);
}

int jo_gated_residual_norm_scale_shift(
    void* out_h, int64_t h_row_stride, void* out, int64_t out_row_stride,
    const void* residual, int64_t res_row_stride, const void* x, int64_t x_row_stride,
    const void* gate, int64_t gate_rows, int64_t gate_row_stride, const void* gamma,
    const void* beta, const void* scale, const void* shift, int64_t mod_rows,
    int64_t mod_row_stride, int64_t rows, int64_t cols, int norm, int dtype, float eps,
    void* stream) {
  RowArgs a{};
  a.out_h = out_h;
  a.h_stride = h_row_stride;
  a.out = out;
  a.out_stride = out_row_stride;
  a.x = x;
  a.x_stride = x_row_stride;
  a.res = residual;
  a.res_stride = res_row_stride;
  a.gate = gate;
  a.gamma = gamma;
  a.beta = beta;
  a.rows = rows;
  a.cols = cols;
  a.eps = eps;
  const char* op = "gated_residual_norm_scale_shift";
  if (int s = check_common(a, op)) return s;
  if (rows > 0 && cols > 0 && (!out_h || !out || !residual || !gate))
    return fail(JO_ERR_INVALID, "%s: null operand", op);
  if (gate_rows != 1 && gate_rows != rows)
    return fail(JO_ERR_SHAPE, "%s: gate rows must be 1 or %lld", op, (long long)rows);
  a.gate_stride = gate_rows == 1 ? 0 : gate_row_stride;
  if (int s = mod_setup(a, scale, shift, mod_rows, mod_row_stride, rows, op)) return s;
  const int nk = norm_code(norm, op);
  if (nk < 0) return nk;
  if (nk == kRms) a.beta = nullptr;
  cudaStream_t st = (cudaStream_t)stream;
  return nk == kLayer ? launch_rows<kLayer, kResidGate, kStoreY>(dtype, a, st, true)
                      : launch_rows<kRms, kResidGate, kStoreY>(dtype, a, st, true);
}

}  // extern "C"
