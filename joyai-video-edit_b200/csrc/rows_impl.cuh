// Row-kernel implementation shared by the per-dtype translation units
// (rows_bf16.cu, rows_f16.cu, rows_f32.cu); the C entry points live in rows.cu.
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
// 16-byte stores.  Rows of up to 512 vectors (4096 bf16) stream through
// shared memory: every warp owns a few row slots that it refills itself with
// 1-D TMA bulk copies (the loads in flight are held by the copy engine, not by
// registers), reductions are warp shuffles / warp reduce instructions, and
// broadcast operands are cached per CTA as fp32.  Longer rows, or per-row
// modulation / gate operands, are owned by a CTA with direct 16-byte loads;
// shapes that break 16-byte alignment take a scalar block-per-row path.
#pragma once
#include "pipeline.cuh"
#include "quant.cuh"
#include "rows_decl.cuh"

namespace jo {
namespace rows {

// L2 hints of the staged path: 1 = row loads evict-first (each byte is read
// once), 2 = the output stores too.  Measured: +1.5 % on LN + modulate, -2 to -4 %
// on the quant and the short RMSNorm, so off.
#ifndef JO_ROW_HINT
#define JO_ROW_HINT 0
#endif
constexpr int kRowHint = JO_ROW_HINT;

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
  // |y| maximum: on the packed 16-bit values for bf16/fp16 (absmax16x2), as
  // floats for fp32
  constexpr bool k16 = V == 8;
  float amax = 0.f;
  uint32_t amax16 = 0;
  // no norm and no affine / modulation operand: y is the row itself (quant, GELU -> quant)
  const bool ident = kNorm == kNoNorm && !has_g && !has_b && !has_mod;
#pragma unroll
  for (int i = 0; i < kVPT; ++i) {
    const int idx = g + i * G;
    if constexpr (k16 && kEpi == kQuantY) {
      if (ident) {
        if (idx < nvec) {
          amax16 = absmax16x2<T>(absmax16x2<T>(amax16, raw[i].x), raw[i].y);
          amax16 = absmax16x2<T>(absmax16x2<T>(amax16, raw[i].z), raw[i].w);
        }
        continue;
      }
    }
    if (idx < nvec) {
      float f[V], fg[V], fb[V], fs[V], fh[V], y[V];
      Elt<T>::unpack(raw[i], f);
      // generic loads: these operands may live in shared memory (staged path)
      if (has_g) Elt<T>::unpack(*reinterpret_cast<const uint4*>(gam + (int64_t)idx * V), fg);
      if (has_b) Elt<T>::unpack(*reinterpret_cast<const uint4*>(bet + (int64_t)idx * V), fb);
      if (has_mod) {
        Elt<T>::unpack(*reinterpret_cast<const uint4*>(scr + (int64_t)idx * V), fs);
        Elt<T>::unpack(*reinterpret_cast<const uint4*>(shr + (int64_t)idx * V), fh);
      }
#pragma unroll
      for (int j = 0; j < V; ++j)
        y[j] = norm_elem<kNorm>(f[j], mean, rstd, fg[j], fb[j], fs[j], fh[j], has_g, has_b, has_mod);
      if constexpr (kEpi == kStoreY) {
        T* orow = reinterpret_cast<T*>(a.out) + row * a.out_stride;
        st_global(orow + (int64_t)idx * V, Elt<T>::pack(y));
      } else {
        raw[i] = Elt<T>::pack(y);  // y rounded to T, as the unfused chain materialises it
        if constexpr (k16) {
          amax16 = absmax16x2<T>(absmax16x2<T>(amax16, raw[i].x), raw[i].y);
          amax16 = absmax16x2<T>(absmax16x2<T>(amax16, raw[i].z), raw[i].w);
        } else {
          float r[V];
          Elt<T>::unpack(raw[i], r);
#pragma unroll
          for (int j = 0; j < V; ++j) amax = fmaxf(amax, fabsf(r[j]));
        }
      }
    }
  }
  if constexpr (kEpi == kQuantY) {
    if constexpr (k16) amax = bits16_to_f<T>(amax16_bits(amax16));
    const float s = quant_scale(row_reduce_max<kWarp>(amax, smem));
    uint8_t* qrow = a.out_q + row * a.q_stride;
    // 16-bit rows: the correctly rounded quotient from RN(1/s) (div2_ms) with the
    // signs of -0 restored on the bytes, as the staged path; fp32: IEEE division
    const float2 ns2 = f2(-s), rc2 = f2(__frcp_rn(s));
#pragma unroll
    for (int i = 0; i < kVPT; ++i) {
      const int idx = g + i * G;
      if (idx < nvec) {
        if constexpr (k16) {
          float2 p[4], q[4];
          to_pairs<T>(raw[i], p);
#pragma unroll
          for (int e = 0; e < 4; ++e) q[e] = div2_ms(p[e], ns2, rc2);
          uint2 o;
          o.x = ((uint32_t)e4m3x2(q[0].x, q[0].y) | ((uint32_t)e4m3x2(q[1].x, q[1].y) << 16)) |
                e4m3_signs(raw[i].x, raw[i].y);
          o.y = ((uint32_t)e4m3x2(q[2].x, q[2].y) | ((uint32_t)e4m3x2(q[3].x, q[3].y) << 16)) |
                e4m3_signs(raw[i].z, raw[i].w);
          *reinterpret_cast<uint2*>(qrow + (int64_t)idx * 8) = o;
        } else {
          float r[V];
          Elt<T>::unpack(raw[i], r);
          uint32_t o = (uint32_t)e4m3x2(quant_clamp(r[0], s), quant_clamp(r[1], s)) |
                       ((uint32_t)e4m3x2(quant_clamp(r[2], s), quant_clamp(r[3], s)) << 16);
          *reinterpret_cast<uint32_t*>(qrow + (int64_t)idx * 4) = o;
        }
      }
    }
    if (g == 0) a.out_s[row] = s;
  }
}

// Feature bits of a staged row op (compile-time, no per-element branches).
// Every feature is a broadcast row (one [cols] vector for all rows).
enum Feat { kFG = 1, kFB = 2, kFMod = 4, kFGate = 8 };
constexpr int kMaxG = 4;  // warps per row group, at most

// Broadcast operands live in shared memory as fp32 so the row math converts
// nothing for them: one set of 4*cols bytes per present operand, in the order
// gamma, beta, 1+scale, shift, gate.  Within a set, vector idx (V elements) is
// V/4 float4 at plane p: set + (p * nvec + idx) * 16, so the float4 reads of a
// warp (consecutive idx) are contiguous and free of bank conflicts.
template <int kF>
struct Sets {
  static constexpr int g = 0;
  static constexpr int b = g + ((kF & kFG) ? 1 : 0);
  static constexpr int c1 = b + ((kF & kFB) ? 1 : 0);
  static constexpr int sh = c1 + ((kF & kFMod) ? 1 : 0);
  static constexpr int gate = sh + ((kF & kFMod) ? 1 : 0);
  static constexpr int n = gate + ((kF & kFGate) ? 1 : 0);
};

template <int V>
__device__ __forceinline__ void ld_set(uint32_t set, int nvec, int idx, float2* p) {
#pragma unroll
  for (int pl = 0; pl < V / 4; ++pl) {
    const uint4 u = lds128(set + (uint32_t)(pl * nvec + idx) * 16u);
    p[2 * pl] = make_float2(__uint_as_float(u.x), __uint_as_float(u.y));
    p[2 * pl + 1] = make_float2(__uint_as_float(u.z), __uint_as_float(u.w));
  }
}

// Reductions over the warps of a row group: warp shuffle / warp reduce, then
// (G > 1) the G warp partials through shared memory and the group's named
// barrier, summed in warp order by every thread (identical results in all
// warps).  Each kind (0 sum, 1 variance sum, 2 amax) has its own partial slots;
// every row starts with a group barrier, so no slot is rewritten before all
// warps have read it.
struct GroupRed {
  float* part;  // this group's [3][kMaxG] partials
  int G, wg, lane, bar_id;
  __device__ __forceinline__ void sync() const {
    asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(G * 32) : "memory");
  }
  __device__ __forceinline__ float sum(float v, int kind) const {
    v = warp_sum(v);
    if (G == 1) return v;
    float* r = part + kind * kMaxG;
    if (lane == 0) r[wg] = v;
    sync();
    float s = r[0];
    for (int i = 1; i < G; ++i) s += r[i];
    return s;
  }
  __device__ __forceinline__ uint32_t umax(uint32_t v, int kind) const {
    v = __reduce_max_sync(0xffffffffu, v);
    if (G == 1) return v;
    uint32_t* r = reinterpret_cast<uint32_t*>(part) + kind * kMaxG;
    if (lane == 0) r[wg] = v;
    sync();
    uint32_t s = r[0];
    for (int i = 1; i < G; ++i) s = max(s, r[i]);
    return s;
  }
  // AND of `v` over the group (every warp of the group must call it)
  __device__ __forceinline__ bool all(bool v) const {
    if (G == 1) return __all_sync(0xffffffffu, v);
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(bar_id), "r"(G * 32)
        : "memory");
    return r != 0;
  }
};

// Row math of the staged path, f32x2 throughout.  Same operation order as
// row_math (LayerNorm ((x-mean)*rstd*g + b)*(1+sc)+sh, RMS (x*rstd*g)*(1+sc)+sh;
// two-pass mean/variance; quant on the T-rounded y).  The statistics use the
// reciprocal of the row length and the hardware rsqrt, as the reference kernel
// does (fused_norm_scale_shift.cu:136,157): both move rstd by a few fp32 ulps.
template <typename T, int kVPT, int kNorm, int kEpi, int kF>
__device__ __forceinline__ void row_math2(const RowArgs& a, int64_t row, uint4 (&raw)[kVPT], int lane,
                                          uint32_t cache, int nvec, float inv_n, const GroupRed& red,
                                          uint64_t pol) {
  const int GT = red.G * 32;  // threads of the row group; this thread's vectors: lane + GT * i
  constexpr int V = Elt<T>::kVec, P = V / 2;
  constexpr bool k16 = V == 8;
  constexpr bool kIdentity = kNorm == kNoNorm && (kF & (kFG | kFB | kFMod)) == 0;  // y == x
  using S = Sets<kF>;
  const uint32_t set_bytes = (uint32_t)nvec * (uint32_t)V * 4u;
  float mean = 0.f, rstd = 1.f;
  if constexpr (kNorm == kLayer) {
    float2 s0 = f2(0.f), s1 = f2(0.f);
#pragma unroll
    for (int i = 0; i < kVPT; ++i)
      if (lane + GT * i < nvec) {
        float2 p[P];
        to_pairs<T>(raw[i], p);
#pragma unroll
        for (int e = 0; e < P; e += 2) {
          s0 = __fadd2_rn(s0, p[e]);
          s1 = __fadd2_rn(s1, p[e + 1]);
        }
      }
    mean = red.sum((s0.x + s1.x) + (s0.y + s1.y), 0) * inv_n;
    const float2 nm = f2(-mean);
    float2 q0 = f2(0.f), q1 = f2(0.f);
#pragma unroll
    for (int i = 0; i < kVPT; ++i)
      if (lane + GT * i < nvec) {
        float2 p[P];
        to_pairs<T>(raw[i], p);
#pragma unroll
        for (int e = 0; e < P; e += 2) {
          const float2 d0 = __fadd2_rn(p[e], nm), d1 = __fadd2_rn(p[e + 1], nm);
          q0 = __ffma2_rn(d0, d0, q0);
          q1 = __ffma2_rn(d1, d1, q1);
        }
      }
    rstd = rsqrtf(fmaf(red.sum((q0.x + q1.x) + (q0.y + q1.y), 1), inv_n, a.eps));
  } else if constexpr (kNorm == kRms) {
    float2 q0 = f2(0.f), q1 = f2(0.f);
#pragma unroll
    for (int i = 0; i < kVPT; ++i)
      if (lane + GT * i < nvec) {
        float2 p[P];
        to_pairs<T>(raw[i], p);
#pragma unroll
        for (int e = 0; e < P; e += 2) {
          q0 = __ffma2_rn(p[e], p[e], q0);
          q1 = __ffma2_rn(p[e + 1], p[e + 1], q1);
        }
      }
    rstd = rsqrtf(fmaf(red.sum((q0.x + q1.x) + (q0.y + q1.y), 1), inv_n, a.eps));
  }
  const float2 nm2 = f2(-mean), r2 = f2(rstd);
  uint32_t amax16 = 0u;  // 16-bit types: packed |y| maximum
  float amaxf = 0.f;     // fp32 rows
#pragma unroll
  for (int i = 0; i < kVPT; ++i) {
    const int idx = lane + GT * i;
    if (idx >= nvec) continue;
    if constexpr (!kIdentity) {
      float2 y[P];
      to_pairs<T>(raw[i], y);
      if constexpr (kNorm == kLayer) {
#pragma unroll
        for (int e = 0; e < P; ++e) y[e] = __fmul2_rn(__fadd2_rn(y[e], nm2), r2);
      } else if constexpr (kNorm == kRms) {
#pragma unroll
        for (int e = 0; e < P; ++e) y[e] = __fmul2_rn(y[e], r2);
      }
      if constexpr ((kF & kFG) != 0) {
        float2 g[P];
        ld_set<V>(cache + S::g * set_bytes, nvec, idx, g);
#pragma unroll
        for (int e = 0; e < P; ++e) y[e] = __fmul2_rn(y[e], g[e]);
      }
      if constexpr ((kF & kFB) != 0) {
        float2 b[P];
        ld_set<V>(cache + S::b * set_bytes, nvec, idx, b);
#pragma unroll
        for (int e = 0; e < P; ++e) y[e] = __fadd2_rn(y[e], b[e]);
      }
      if constexpr ((kF & kFMod) != 0) {
        float2 c1[P], sh[P];
        ld_set<V>(cache + S::c1 * set_bytes, nvec, idx, c1);
        ld_set<V>(cache + S::sh * set_bytes, nvec, idx, sh);
#pragma unroll
        for (int e = 0; e < P; ++e) y[e] = __ffma2_rn(y[e], c1[e], sh[e]);
      }
      if constexpr (kEpi == kStoreY) {
        if constexpr (kRowHint > 1)
          st_global_hint(reinterpret_cast<T*>(a.out) + row * a.out_stride + (int64_t)idx * V, from_pairs<T>(y), pol);
        else
          st_global(reinterpret_cast<T*>(a.out) + row * a.out_stride + (int64_t)idx * V, from_pairs<T>(y));
        continue;
      } else {
        raw[i] = from_pairs<T>(y);  // y rounded to T, as the unfused chain materialises it
      }
    }
    if constexpr (kEpi == kQuantY) {
      if constexpr (k16) {
        amax16 = absmax16x2<T>(amax16, raw[i].x);
        amax16 = absmax16x2<T>(amax16, raw[i].y);
        amax16 = absmax16x2<T>(amax16, raw[i].z);
        amax16 = absmax16x2<T>(amax16, raw[i].w);
      } else {
        float f[V];
        Elt<T>::unpack(raw[i], f);
#pragma unroll
        for (int e = 0; e < V; ++e) amaxf = fmaxf(amaxf, fabsf(f[e]));
      }
    }
  }
  if constexpr (kEpi == kQuantY) {
    float amax;
    if constexpr (k16) {
      amax = bits16_to_f<T>(red.umax(amax16_bits(amax16), 2));
    } else {
      amax = __uint_as_float(red.umax(__float_as_uint(amaxf), 2));  // |y| >= 0: bits order as values
    }
    const float s = quant_scale(amax);
    const float2 s2 = f2(s), ns2 = f2(-s), rc2 = f2(__frcp_rn(s));
    uint8_t* qrow = a.out_q + row * a.q_stride;
#pragma unroll
    for (int i = 0; i < kVPT; ++i) {
      const int idx = lane + GT * i;
      if (idx >= nvec) continue;
      float2 p[P];
      to_pairs<T>(raw[i], p);
      if constexpr (k16) {
        // satfinite conversion saturates |q| > 448 to 448, as the reference clamp does
        float2 q[P];
#pragma unroll
        for (int e = 0; e < P; ++e) q[e] = div2_ms(p[e], ns2, rc2);
        const uint32_t w0 = ((uint32_t)e4m3x2(q[0].x, q[0].y) | ((uint32_t)e4m3x2(q[1].x, q[1].y) << 16)) |
                            e4m3_signs(raw[i].x, raw[i].y);
        const uint32_t w1 = ((uint32_t)e4m3x2(q[2].x, q[2].y) | ((uint32_t)e4m3x2(q[3].x, q[3].y) << 16)) |
                            e4m3_signs(raw[i].z, raw[i].w);
        if constexpr (kRowHint > 1)
          st_global_hint8(qrow + (int64_t)idx * 8, make_uint2(w0, w1), pol);
        else
          *reinterpret_cast<uint2*>(qrow + (int64_t)idx * 8) = make_uint2(w0, w1);
      } else {
        const float2 q0 = div2_markstein(p[0], s2, rc2), q1 = div2_markstein(p[1], s2, rc2);
        *reinterpret_cast<uint32_t*>(qrow + (int64_t)idx * 4) =
            (uint32_t)e4m3x2(q0.x, q0.y) | ((uint32_t)e4m3x2(q1.x, q1.y) << 16);
      }
    }
    if (lane == 0) a.out_s[row] = s;  // thread 0 of the group
  }
}

// ------------------------------------------------------------------ staged path
// Rows of up to 512 vectors (4096 bf16).  A row group of G warps (G = 1, 2, 4
// by row length, so each thread holds at most 4 vectors) owns `m` shared-
// memory slots and feeds itself: its leader thread keeps the group's next m
// rows in flight with 1-D TMA bulk copies; when a row lands the G warps pull it
// into registers, the leader refills the slot with the row m ahead, and the
// group computes + stores while those copies fly.  32 warps per SM hide the
// latency of the reductions.  Groups never wait on each other, and each slot
// has a single owner group whose warps all pass a group barrier before the
// refill, so no mbarrier is waited on more than one phase ahead.  Broadcast
// operands (gamma, beta, 1+scale, shift, gate) are staged once per CTA in
// shared memory as fp32 sets.
constexpr int kMaxWarps = 32;
// Bytes of row slots per SM the staged launcher aims for (see launch_staged_f).
// Measured on B200 (LN + modulate, quant, RMSNorm -> FP8 at [10800, 3072]):
// 96 KB beats 144 and 180 KB by 5-12 %; more bytes in flight per SM only slowed
// the stream down.
#ifndef JO_ROW_INFLIGHT_SM
#define JO_ROW_INFLIGHT_SM (96u * 1024u)
#endif
constexpr uint32_t kRowInflightSm = JO_ROW_INFLIGHT_SM;
// Groups with at most three rows in all keep every one of them in flight from
// the start (1), or refill one slot at a time like longer matrices (0).  Measured
// on RMSNorm [3600, 3072] (1-2 rows per group): 10.2 us with 1, 9.6 us with 0 --
// loads issued as slots free up interleave the reads with the writes.
#ifndef JO_ROW_SMALL_ALL
#define JO_ROW_SMALL_ALL 0
#endif
// Rows of more than 128 vectors split over two warps (half the vectors per
// thread, twice the warps per SM) for: 0 = residual rows only, 1 = also rows
// with a quantising epilogue, 2 = also every normalising op.  Measured at
// [10800, 3072]: RMSNorm -> FP8 22.5 us with 0, 26.5 us with 1 or 2 (the
// cross-warp reductions cost more than the extra warps hide).
#ifndef JO_ROW_G2
#define JO_ROW_G2 0
#endif
// Upper bound on the warps of a staged CTA (0: as many as the register budget allows).
#ifndef JO_ROW_WARPS_CAP
#define JO_ROW_WARPS_CAP 0
#endif
// Compile-time row length for 3072-wide 16-bit rows (1) or always the generic kernel (0).
#ifndef JO_ROW_SPEC
#define JO_ROW_SPEC 1
#endif
// threads per CTA by vectors per thread (register budget: 64 / 85 / 128 per thread);
// JO_ROW_T12 sets it for 9-12 vectors per thread (3072-wide bf16 rows)
#ifndef JO_ROW_T12
#define JO_ROW_T12 512
#endif
// GELU rows wider than 512 vectors (the MLP activation's 12288 bf16) through the
// staged kernel in 4-warp groups (1) or the block path (0).
#ifndef JO_ROW_WIDE
#define JO_ROW_WIDE 0
#endif
constexpr int staged_threads(int vpt) { return vpt <= 4 ? 1024 : (vpt <= 8 ? 768 : (vpt <= 12 ? JO_ROW_T12 : 512)); }

struct StagedCfg {
  int warps;            // warps per CTA (blockDim.x / 32), a multiple of G
  int G;                // warps per row group (1, 2 or 4)
  int m;                // slots per group
  uint32_t slot_bytes;  // >= one row (two for kResidGate)
  uint32_t red_off;     // byte offset of the groups' reduction partials
  uint32_t cache_off;   // byte offset of the broadcast-operand sets
  uint32_t data_off;    // byte offset of slot 0
};

// kNV > 0: the row length in vectors is known at compile time (the launcher takes
// it only when a.cols matches), so the bounds checks and shared-memory offsets of
// the row loops fold into constants; the row group size follows from it.
template <typename T, int kVPT, int kNorm, int kPro, int kEpi, int kF, int kNV = 0>
__global__ void __launch_bounds__(staged_threads(kVPT), 1)
    row_staged_kernel(RowArgs a, const StagedCfg cfg, unsigned int* fault) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  constexpr int V = Elt<T>::kVec, P = V / 2;
  using S = Sets<kF>;
  constexpr int kG = kNV > 0 ? (kNV + 32 * kVPT - 1) / (32 * kVPT) : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = kG > 0 ? kG : cfg.G, NG = cfg.warps / G, m = cfg.m;
  const int grp = warp / G, wg = warp % G;
  const int gl = wg * 32 + lane, GT = G * 32;  // thread within the group; group size
  const bool leader = gl == 0;
  const int64_t per = (a.rows + gridDim.x - 1) / gridDim.x;
  const int64_t r0 = (int64_t)blockIdx.x * per;
  const int64_t rend = r0 + per < a.rows ? r0 + per : a.rows;
  const int units = rend > r0 ? (int)(rend - r0) : 0;
  const int nvec = kNV > 0 ? kNV : (int)(a.cols / V);
  const uint32_t row_bytes = (uint32_t)nvec * 16u;
  const uint32_t base = smem_u32(smem_raw);
  const uint32_t cache = base + cfg.cache_off;
  const uint32_t set_bytes = (uint32_t)nvec * (uint32_t)V * 4u;
  const float inv_n = 1.0f / (float)a.cols;
  const GroupRed red{reinterpret_cast<float*>(smem_raw + cfg.red_off) + grp * 3 * kMaxG, G, wg, lane, 1 + grp};

  if (threadIdx.x < NG * m) mbar_init(base + 8u * threadIdx.x, 1);
  if (threadIdx.x == 0) mbar_init_fence();
  __syncthreads();
  pdl_wait();  // the previous kernel's outputs (our inputs) are complete from here on
  pdl_trigger();

  const uint32_t bar0 = base + 8u * (uint32_t)(grp * m);
  const uint32_t slot0 = base + cfg.data_off + (uint32_t)(grp * m) * cfg.slot_bytes;
  // unit k of this group is row r0 + grp + k * NG, in slot k % m, phase (k / m) & 1
  uint64_t pol = 0;
  if constexpr (kRowHint > 0) pol = policy_evict_first();
  auto load = [&](uint32_t dst, const void* src, uint32_t bar) {
    if constexpr (kRowHint > 0)
      bulk_load_hint(dst, src, row_bytes, bar, pol);
    else
      bulk_load(dst, src, row_bytes, bar);
  };
  auto issue = [&](int k) {
    const int i = grp + k * NG;
    if (i >= units) return;
    const int64_t row = r0 + i;
    const uint32_t bar = bar0 + 8u * (uint32_t)(k % m), dst = slot0 + (uint32_t)(k % m) * cfg.slot_bytes;
    if constexpr (kPro != kResidGate) {
      mbar_expect_tx(bar, row_bytes);
      load(dst, reinterpret_cast<const T*>(a.x) + row * a.x_stride, bar);
    } else {
      mbar_expect_tx(bar, 2 * row_bytes);
      load(dst, reinterpret_cast<const T*>(a.x) + row * a.x_stride, bar);
      load(dst + row_bytes, reinterpret_cast<const T*>(a.res) + row * a.res_stride, bar);
    }
  };
  if (leader)
    for (int k = 0; k < m; ++k) issue(k);
  // stage the broadcast operands once per CTA, converted to fp32 (scale as 1+scale),
  // while the first rows are in flight
  {
    const void* src[5] = {a.gamma, a.beta, a.scale, a.shift, a.gate};
    const int set_of[5] = {(kF & kFG) ? S::g : -1, (kF & kFB) ? S::b : -1, (kF & kFMod) ? S::c1 : -1,
                           (kF & kFMod) ? S::sh : -1, (kF & kFGate) ? S::gate : -1};
#pragma unroll
    for (int o = 0; o < 5; ++o) {
      if (set_of[o] < 0) continue;
      const uint4* s4 = reinterpret_cast<const uint4*>(src[o]);
      uint4* d4 = reinterpret_cast<uint4*>(smem_raw + cfg.cache_off + (size_t)set_of[o] * set_bytes);
      const float add = o == 2 ? 1.f : 0.f;
      for (int k = threadIdx.x; k < nvec; k += blockDim.x) {
        float f[V];
        Elt<T>::unpack(ld_bcast(s4 + k), f);
#pragma unroll
        for (int pl = 0; pl < V / 4; ++pl)
          d4[pl * nvec + k] = make_uint4(__float_as_uint(f[4 * pl] + add), __float_as_uint(f[4 * pl + 1] + add),
                                         __float_as_uint(f[4 * pl + 2] + add), __float_as_uint(f[4 * pl + 3] + add));
      }
    }
  }
  __syncthreads();
  int k = 0;
  for (; grp + k * NG < units; ++k) {
    const uint32_t bar = bar0 + 8u * (uint32_t)(k % m), sl = slot0 + (uint32_t)(k % m) * cfg.slot_bytes;
    // warp 0 of the group waits for the row; the others sleep at the group barrier
    bool ok = true;
    if (wg == 0) ok = mbar_wait(bar, (uint32_t)((k / m) & 1), fault);
    if (!red.all(ok)) break;  // uniform across the group
    const int64_t row = r0 + grp + k * NG;
    uint4 raw[kVPT];
    {
#pragma unroll
      for (int v = 0; v < kVPT; ++v) {
        const int idx = gl + GT * v;
        if (idx < nvec) {
          if constexpr (kPro == kLoadX) {
            raw[v] = lds128(sl + idx * 16);
          } else if constexpr (kPro == kGeluX) {
            raw[v] = gelu_vec<T>(lds128(sl + idx * 16));
          } else {  // h = residual + x * gate straight from the slot, rounded to T and stored
            float2 x[P], r[P], g[P];
            to_pairs<T>(lds128(sl + idx * 16), x);
            to_pairs<T>(lds128(sl + row_bytes + idx * 16), r);
            ld_set<V>(cache + S::gate * set_bytes, nvec, idx, g);
#pragma unroll
            for (int e = 0; e < P; ++e) x[e] = __ffma2_rn(x[e], g[e], r[e]);
            raw[v] = from_pairs<T>(x);
            if constexpr (kRowHint > 1)
              st_global_hint(reinterpret_cast<T*>(a.out_h) + row * a.h_stride + (int64_t)idx * V, raw[v], pol);
            else
              st_global(reinterpret_cast<T*>(a.out_h) + row * a.h_stride + (int64_t)idx * V, raw[v]);
          }
        }
      }
    }
    // every warp of the group has read the slot before the leader refills it
    if (G == 1)
      __syncwarp();
    else
      red.sync();
    if (leader) {
      // order the group's shared-memory reads before the copy engine overwrites the slot
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(k + m);
    }
    if constexpr (kEpi != kNoY) row_math2<T, kVPT, kNorm, kEpi, kF>(a, row, raw, gl, cache, nvec, inv_n, red, pol);
  }
  // error path only (a wait expired at unit k): the copies the leader issued
  // for units k .. k+m-1 must land before the CTA exits
  if (leader && grp + k * NG < units)
    for (int j = k; j < k + m && grp + j * NG < units; ++j)
      mbar_wait(bar0 + 8u * (uint32_t)(j % m), (uint32_t)((j / m) & 1), fault);
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
      } else if constexpr (kPro == kGeluX) {
        raw[i] = ld_stream(xr + (int64_t)idx * V);
      } else {
        xv[i] = ld_stream(xr + (int64_t)idx * V);
        raw[i] = ld_stream(rr + (int64_t)idx * V);
      }
    }
  }
  if constexpr (kPro == kGeluX) {
#pragma unroll
    for (int i = 0; i < kVPT; ++i)
      if (g + i * G < nvec) raw[i] = gelu_vec<T>(raw[i]);
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
  auto xval = [&](int c) {
    const float v = Elt<T>::to_f(src[c]);
    if constexpr (kPro == kGeluX) return round_through<T>(gelu_tanh_f(v));
    return v;
  };
  float mean = 0.f, rstd = 1.f;
  if constexpr (kNorm == kLayer) {
    float s = 0.f;
    for (int c = g; c < n; c += G) s += xval(c);
    mean = __fdiv_rn(row_reduce_sum<false>(s, smem), (float)n);
    float q = 0.f;
    for (int c = g; c < n; c += G) {
      const float d = xval(c) - mean;
      q += d * d;
    }
    rstd = rsqrt_ieee(__fdiv_rn(row_reduce_sum<false>(q, smem), (float)n) + a.eps);
  } else if constexpr (kNorm == kRms) {
    float q = 0.f;
    for (int c = g; c < n; c += G) {
      const float v = xval(c);
      q += v * v;
    }
    rstd = rsqrt_ieee(__fdiv_rn(row_reduce_sum<false>(q, smem), (float)n) + a.eps);
  }
  const bool has_g = a.gamma != nullptr, has_b = a.beta != nullptr, has_mod = a.scale != nullptr;
  const T* scr = has_mod ? reinterpret_cast<const T*>(a.scale) + row * a.mod_stride : nullptr;
  const T* shr = has_mod ? reinterpret_cast<const T*>(a.shift) + row * a.mod_stride : nullptr;
  auto y_at = [&](int c) {
    return norm_elem<kNorm>(xval(c), mean, rstd, has_g ? ldf<T>(a.gamma, c) : 1.f,
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
inline bool row_vec_ok(const RowArgs& a, int esize) {
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

// 3072-wide 16-bit rows (the model's hidden size, 384 vectors): one warp per row
// (12 vectors per thread) or four-warp groups of residual rows (3 per thread).
// Not for single-input LayerNorm + modulate: fully unrolled, it reaches the
// 128-register cap and spills (measured 25.6 us against 24.7 us unspecialised).
constexpr int kSpecNV = 384;
template <typename T, int kVPT, int kNorm, int kPro, int kF>
constexpr bool spec_ok() {
  return JO_ROW_SPEC && sizeof(T) == 2 && (kVPT == 12 || (kVPT == 3 && kPro == kResidGate)) &&
         !(kNorm == kLayer && kPro != kResidGate && (kF & kFMod) != 0);
}

template <typename T, int kVPT, int kNorm, int kPro, int kEpi, int kF>
int launch_staged_f(const RowArgs& a, cudaStream_t st, const DeviceInfo* di) {
  constexpr int V = Elt<T>::kVec;
  constexpr bool kSpec = spec_ok<T, kVPT, kNorm, kPro, kF>();
  const bool spec = kSpec && a.cols / V == kSpecNV;
  auto kern = spec ? row_staged_kernel<T, kVPT, kNorm, kPro, kEpi, kF, kSpec ? kSpecNV : 0>
                   : row_staged_kernel<T, kVPT, kNorm, kPro, kEpi, kF, 0>;
  constexpr uint32_t kBudget = 216u * 1024u;
  const int nvec = (int)(a.cols / V);
  const uint32_t row_bytes = (uint32_t)(a.cols * sizeof(T)) * (kPro == kResidGate ? 2u : 1u);
  StagedCfg cfg{};
  cfg.slot_bytes = (row_bytes + 127u) & ~127u;
  // one warp per row, except two-input rows (residual + x), whose row groups
  // of G warps hold at most kVPT vectors per thread; warps per CTA by the
  // register budget (30 for G = 2: named barriers 1..15 name the groups)
  cfg.G = nvec <= 32 * kVPT ? 1 : (nvec <= 64 * kVPT ? 2 : 4);
  if (cfg.G * 32 * kVPT < nvec) return fail(JO_ERR_SHAPE, "row kernel: row group too small");
  cfg.warps = staged_threads(kVPT) / 32;
  if (cfg.G == 2 && cfg.warps > 30) cfg.warps = 30;
  if (JO_ROW_WARPS_CAP > 0 && cfg.warps > JO_ROW_WARPS_CAP)
    cfg.warps = JO_ROW_WARPS_CAP >= cfg.G ? JO_ROW_WARPS_CAP / cfg.G * cfg.G : cfg.G;
  const uint32_t cache_bytes = (uint32_t)(Sets<kF>::n * 4 * a.cols + 127) & ~127u;
  if (cache_bytes + 2048u >= kBudget) return fail(JO_ERR_SHAPE, "row kernel: rows too large to stage");
  const uint32_t avail = kBudget - cache_bytes - 2048u;
  // Slots: a group refills a slot as soon as it has pulled the row out of it,
  // but while it computes, its landed rows wait and nothing else is in flight
  // for it; so the SM keeps kRowInflightSm bytes of slots (m per group, at most
  // 3), giving up a group (down to 3/4 of them) before it gives up a slot.
  const int ng_max = cfg.warps / cfg.G;
  int ng = ng_max;
  cfg.m = (int)((kRowInflightSm + (uint32_t)ng * cfg.slot_bytes - 1) / ((uint32_t)ng * cfg.slot_bytes));
  if (cfg.m < 1) cfg.m = 1;
  // a group with only 2-3 rows in all keeps all of them in flight from the start
  const int64_t group_rows = cdiv(cdiv(a.rows, (int64_t)di->sm_count), (int64_t)ng);
  if (JO_ROW_SMALL_ALL && group_rows <= 3 && cfg.m < group_rows) cfg.m = (int)group_rows;
  if (cfg.m > 3) cfg.m = 3;
  while ((uint32_t)(ng * cfg.m) * cfg.slot_bytes > avail) {
    if (cfg.m > 1 && 4 * (ng - 1) < 3 * ng_max)
      --cfg.m;
    else if (ng > 1)
      --ng;
    else
      break;
  }
  cfg.warps = ng * cfg.G;
  if ((uint32_t)ng * cfg.slot_bytes > avail) {  // fewer groups, one slot each
    ng = (int)(avail / cfg.slot_bytes);
    cfg.warps = ng * cfg.G;
  }
  ng = cfg.warps / cfg.G;
  if (ng < 1) return fail(JO_ERR_SHAPE, "row kernel: rows too large to stage");
  cfg.red_off = (uint32_t)((8 * ng * cfg.m + 15) & ~15);
  cfg.cache_off = (cfg.red_off + (uint32_t)(ng * 3 * kMaxG * 4) + 127u) & ~127u;
  cfg.data_off = cfg.cache_off + cache_bytes;
  const size_t smem = cfg.data_off + (size_t)ng * cfg.m * cfg.slot_bytes;
  static std::atomic<uint64_t> reserved[2];  // generic and specialised kernels
  if (int s = reserve_smem((const void*)kern, 220 * 1024, reserved[spec ? 1 : 0], di, "row kernel")) return s;
  // one CTA per SM whenever every SM gets a row: a short matrix (3600 rows: ~25
  // per SM) is spread over all SMs with each group's 1-3 rows in flight at once
  // (m above), rather than packed into fewer CTAs that leave SMs idle
  int64_t grid = a.rows < di->sm_count ? a.rows : di->sm_count;
  if (grid < 1) grid = 1;
  if (cudaError_t e = launch_pdl(kern, dim3((unsigned)grid), dim3(cfg.warps * 32), smem, st, a, cfg, di->fault))
    return launch_failed(e, "row kernel");
  return after_launch("row_staged_kernel");
}

// The staged path takes broadcast (one-row) modulation and gate operands only;
// per-row operands go to the block path.
inline bool staged_operands_ok(const RowArgs& a, int pro) {
  if (a.scale != nullptr && a.mod_stride != 0) return false;
  if (pro == kResidGate && a.gate_stride != 0) return false;
  return true;
}

template <typename T, int kVPT, int kNorm, int kPro, int kEpi>
int launch_staged(const RowArgs& a, cudaStream_t st, const DeviceInfo* di) {
  constexpr int kG = kPro == kResidGate ? kFGate : 0;
  const bool g = a.gamma != nullptr, b = a.beta != nullptr, mod = a.scale != nullptr;
  if constexpr (kNorm == kNoNorm) {
    return launch_staged_f<T, kVPT, kNorm, kPro, kEpi, kG>(a, st, di);
  } else if constexpr (kNorm == kRms) {  // beta is a LayerNorm-only operand
    if (mod) return g ? launch_staged_f<T, kVPT, kNorm, kPro, kEpi, kG | kFG | kFMod>(a, st, di)
                      : launch_staged_f<T, kVPT, kNorm, kPro, kEpi, kG | kFMod>(a, st, di);
    return g ? launch_staged_f<T, kVPT, kNorm, kPro, kEpi, kG | kFG>(a, st, di)
             : launch_staged_f<T, kVPT, kNorm, kPro, kEpi, kG>(a, st, di);
  } else {
    if (mod) {
      if (g && b) return launch_staged_f<T, kVPT, kNorm, kPro, kEpi, kG | kFG | kFB | kFMod>(a, st, di);
      if (g) return launch_staged_f<T, kVPT, kNorm, kPro, kEpi, kG | kFG | kFMod>(a, st, di);
      if (b) return launch_staged_f<T, kVPT, kNorm, kPro, kEpi, kG | kFB | kFMod>(a, st, di);
      return launch_staged_f<T, kVPT, kNorm, kPro, kEpi, kG | kFMod>(a, st, di);
    }
    if (g && b) return launch_staged_f<T, kVPT, kNorm, kPro, kEpi, kG | kFG | kFB>(a, st, di);
    if (g) return launch_staged_f<T, kVPT, kNorm, kPro, kEpi, kG | kFG>(a, st, di);
    if (b) return launch_staged_f<T, kVPT, kNorm, kPro, kEpi, kG | kFB>(a, st, di);
    return launch_staged_f<T, kVPT, kNorm, kPro, kEpi, kG>(a, st, di);
  }
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
    // staged rows: up to 512 vectors (4096 bf16); wider GELU rows (the MLP
    // activation's 12288 bf16) too when JO_ROW_WIDE is set, else the block path.
    const int max_staged = JO_ROW_WIDE && kPro == kGeluX ? 4 * 32 * 12 : 32 * 16;
    if (nvec <= max_staged && staged_operands_ok(a, kPro)) {
#define JO_STAGED(VPT) return launch_staged<T, VPT, kNorm, kPro, kEpi>(a, st, di)
      // vectors per thread: one warp per row, or (residual + x rows) the
      // smallest row group G in {1, 2, 4} with at most 4 vectors per thread
      const bool split = kPro == kResidGate || (JO_ROW_G2 >= 1 && kEpi == kQuantY && kNorm != kNoNorm) ||
                         (JO_ROW_G2 >= 2 && kNorm != kNoNorm);
      int G = !split || nvec <= 128 ? 1 : (kPro != kResidGate || nvec <= 256 ? 2 : 4);
      if (nvec > 32 * 16) G = 4;  // wide GELU rows: 12 vectors per thread
      const int vpt = (nvec + 32 * G - 1) / (32 * G);
      if (vpt <= 2) JO_STAGED(2);
      if (vpt <= 3) JO_STAGED(3);
      if (vpt <= 4) JO_STAGED(4);
      if (vpt <= 6) JO_STAGED(6);
      if (vpt <= 8) JO_STAGED(8);
      if (vpt <= 12) JO_STAGED(12);
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

}  // namespace rows
}  // namespace jo
