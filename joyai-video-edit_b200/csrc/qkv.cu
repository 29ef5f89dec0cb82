// Per-head q/k RMSNorm + interleaved RoPE, and the q/k/v packing around it.
//
//   jo_qkv_norm_rope_pack      qkv projection -> packed (head-major) q/k/v in one
//                              pass; replaces dit.py:408-429 + sgl_fused_ops.py:137-168
//   jo_qk_norm_rope_3d_paired  in place, joyomni_ops/csrc/fused_qknorm_rope_3d_kernel.cu:141-319
//   jo_joint_qkv_pack          joyomni_ops/csrc/fused_joint_qkv_pack.cu:81-164,237-342
//   jo_cached_kv_pack          joyomni_ops/csrc/fused_joint_qkv_pack.cu:166-220,344-415
//
// Design (B200): all four are HBM-bound streams of 2*D-byte head rows.  A head
// row is owned by D/8 consecutive lanes that each move one 16-byte vector, so
// one warp covers 512 contiguous bytes of the source and the per-head sum of
// squares is a 3-4 step xor-shuffle inside the lane group (no shared memory,
// no barrier).  Each thread keeps kUnroll head rows in flight (all loads are
// issued before the first use); grids are sized to the resident-CTA capacity
// of the 148 SMs and walk the rows with a grid-stride loop.  Destination
// rows are 2*D contiguous bytes, so every store fills whole 32-byte sectors.
#include "pipeline.cuh"

namespace jo {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

__device__ __forceinline__ void unpack_bf16x4(uint2 u, float* f) {
  f[0] = __uint_as_float(u.x << 16);
  f[1] = __uint_as_float(u.x & 0xffff0000u);
  f[2] = __uint_as_float(u.y << 16);
  f[3] = __uint_as_float(u.y & 0xffff0000u);
}

// Sum of squares of a head row distributed as 8 floats per lane over kTPH
// lanes.  Every lane of the warp must call this (full-mask shuffles), whether
// or not its row is valid or needs the norm.
template <int kTPH>
__device__ __forceinline__ float head_sumsq(const float* f) {
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
  return group_sum<kTPH>(ss);
}

// (x * rstd) * w with rstd = 1/sqrt(ss/D + eps): the association of the fp32
// reference (joyomni_ops/tests/test_parity_light.py:93-103).
__device__ __forceinline__ void head_scale(float* f, const float* w, float ss, float inv_d,
                                           float eps) {
  const float r = rsqrt_ieee(__fmul_rn(ss, inv_d) + eps);
#pragma unroll
  for (int e = 0; e < 8; ++e) f[e] = (f[e] * r) * w[e];
}

// Interleaved-pair rotation (x0, x1) -> (x0 c - x1 s, x0 s + x1 c).
__device__ __forceinline__ void rope4(float* f, const float* c, const float* s) {
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const float x0 = f[2 * m], x1 = f[2 * m + 1];
    f[2 * m] = x0 * c[m] - x1 * s[m];
    f[2 * m + 1] = x0 * s[m] + x1 * c[m];
  }
}

// ---------------------------------------------------------------------------
// Mode kPack: rows come from the qkv projection [tokens, 3*H*D] (K H D order);
//   row index i -> token t = i / (3H), column c = i % (3H), part p = c / H.
// Mode kInPlace: rows are q and k of [B, L*H, D], interleaved (q row r, k row r).
enum QkMode { kPack = 0, kInPlace = 1 };

struct QkArgs {
  // kPack
  const __nv_bfloat16* qkv;
  int64_t qkv_stride;
  __nv_bfloat16* out[3];
  int64_t os_h, os_t;
  // kInPlace
  __nv_bfloat16* q;
  __nv_bfloat16* k;
  int seq_len;
  // shared
  __nv_bfloat16* k_pre;  // optional
  const __nv_bfloat16* qw;
  const __nv_bfloat16* kw;
  const __nv_bfloat16* cos;  // [tokens, D/2]
  const __nv_bfloat16* sin;
  uint32_t heads;
  uint32_t total_rows;
  float eps;
};

template <int kD, int kMode, bool kPre, bool kRope>
__global__ void __launch_bounds__(kThreads) qk_norm_rope_kernel(const QkArgs a) {
  constexpr int kTPH = kD / 8;                  // lanes per head row
  constexpr int kRowsPerPass = kThreads / kTPH;  // head rows per CTA per unrolled slot
  const int j = threadIdx.x % kTPH;
  const uint32_t sub = threadIdx.x / kTPH;
  float wq[8], wk[8];
  {
    float t[8];
    Elt<__nv_bfloat16>::unpack(ld_bcast(a.qw + j * 8), t);
#pragma unroll
    for (int e = 0; e < 8; ++e) wq[e] = t[e];
    Elt<__nv_bfloat16>::unpack(ld_bcast(a.kw + j * 8), t);
#pragma unroll
    for (int e = 0; e < 8; ++e) wk[e] = t[e];
  }
  const float inv_d = 1.0f / (float)kD;  // exact for power-of-two D
  const uint32_t H = a.heads, H3 = 3 * a.heads;
  const uint32_t chunk = kRowsPerPass * kUnroll;
  for (uint32_t base = blockIdx.x * chunk; base < a.total_rows; base += gridDim.x * chunk) {
    uint4 v[kUnroll];
    uint2 cs[kUnroll], sn[kUnroll];
    uint32_t tok[kUnroll], part[kUnroll], head[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const uint32_t i = base + u * kRowsPerPass + sub;
      v[u] = make_uint4(0, 0, 0, 0);
      part[u] = 2;
      if (i < a.total_rows) {
        const __nv_bfloat16* src;
        if constexpr (kMode == kPack) {
          const uint32_t t = i / H3, c = i - t * H3;
          const uint32_t p = c / H;
          tok[u] = t;
          part[u] = p;
          head[u] = c - p * H;
          src = a.qkv + (int64_t)t * a.qkv_stride + (int64_t)c * kD + j * 8;
        } else {
          const uint32_t r = i >> 1;
          part[u] = i & 1;
          tok[u] = (r / H) % (uint32_t)a.seq_len;
          head[u] = r;  // row index within q / k
          src = (part[u] ? a.k : a.q) + (int64_t)r * kD + j * 8;
        }
        v[u] = ld_stream(src);
        if (kRope && part[u] < 2) {
          const int64_t co = (int64_t)tok[u] * (kD / 2) + j * 4;
          cs[u] = __ldg(reinterpret_cast<const uint2*>(a.cos + co));
          sn[u] = __ldg(reinterpret_cast<const uint2*>(a.sin + co));
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const uint32_t i = base + u * kRowsPerPass + sub;
      float f[8];
      Elt<__nv_bfloat16>::unpack(v[u], f);
      const float ss = head_sumsq<kTPH>(f);  // all lanes, before any divergence
      if (i >= a.total_rows) continue;       // whole lane group agrees (same i)
      const uint32_t p = part[u];
      if (p < 2 && !kRope) {
        // text rows: the model's RMSNorm rounds twice (see the staged kernel)
        const float r = rsqrt_ieee(__fmul_rn(ss, inv_d) + a.eps);
        const float* w = p == 0 ? wq : wk;
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = round_through<__nv_bfloat16>(f[e] * r) * w[e];
        int64_t dst_off;
        if constexpr (kMode == kPack)
          dst_off = (int64_t)head[u] * a.os_h + (int64_t)tok[u] * a.os_t + j * 8;
        else
          dst_off = (int64_t)head[u] * kD + j * 8;
        if constexpr (kPre) {
          if (p == 1) st_global(a.k_pre + dst_off, Elt<__nv_bfloat16>::pack(f));
        }
        __nv_bfloat16* dst;
        if constexpr (kMode == kPack)
          dst = a.out[p];
        else
          dst = p ? a.k : a.q;
        st_global(dst + dst_off, Elt<__nv_bfloat16>::pack(f));
      } else if (p < 2) {
        head_scale(f, p == 0 ? wq : wk, ss, inv_d, a.eps);
        int64_t dst_off;
        if constexpr (kMode == kPack)
          dst_off = (int64_t)head[u] * a.os_h + (int64_t)tok[u] * a.os_t + j * 8;
        else
          dst_off = (int64_t)head[u] * kD + j * 8;
        if constexpr (kPre) {
          if (p == 1) st_global(a.k_pre + dst_off, Elt<__nv_bfloat16>::pack(f));
        }
        float c[4], s[4];
        unpack_bf16x4(cs[u], c);
        unpack_bf16x4(sn[u], s);
        rope4(f, c, s);
        __nv_bfloat16* dst;
        if constexpr (kMode == kPack)
          dst = a.out[p];
        else
          dst = p ? a.k : a.q;
        st_global(dst + dst_off, Elt<__nv_bfloat16>::pack(f));
      } else {
        // v: pure copy (kPack only)
        st_global(a.out[2] + (int64_t)head[u] * a.os_h + (int64_t)tok[u] * a.os_t + j * 8, v[u]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Staged variant (B200 fast path).  Unit = all heads of one token for one of
// q/k/v (kPack: a contiguous H*D slice of the qkv row) or for q/k (kInPlace: a
// contiguous token row of q or k).  Each warp owns kQkSlots shared-memory
// slots and feeds itself with 1-D TMA bulk copies.
//   v units (kPack): never enter registers -- each head row goes from the slot
//     to its destination with one 2*D-byte bulk store (shared -> global).
//   q/k units: the warp pulls the unit into registers (D/8 lanes per head, 16
//     bytes per lane), refills the slot with its unit kQkSlots ahead, then
//     normalises + rotates with packed fp32 (f32x2) arithmetic and stores
//     2*D-byte rows.
// Rotation with the norm weight folded in, per pair (x0, x1) of a head row:
//   out = r * (x0 * (w0 c, w0 s) + x1 * (-w1 s, w1 c))
// where the four per-lane products depend only on the token (c, s) and the
// lane (w), so they are formed once per unit.  Vectors hold the even / odd
// elements of two adjacent pairs, so no operand needs a broadcast.  The head
// rsqrt uses the hardware approximation (rel. error ~2^-22, far below the bf16
// output ulp); the regrouped products move the fp32 result by a few fp32 ulps
// (at most one bf16 ulp after rounding).
#ifndef JO_QK_WARPS
#define JO_QK_WARPS 8
#endif
#ifndef JO_QK_SLOTS
#define JO_QK_SLOTS 1
#endif
#ifndef JO_QK_HINT
#define JO_QK_HINT 2
#endif
// config 1: 72.5 us with 16 warps, 71.6 with 12, 71.1 with 10, 69.5 with 8
constexpr int kQkWarps = JO_QK_WARPS;
constexpr int kQkSlots = JO_QK_SLOTS;  // 6 KB units in flight per warp (two, 15 warps: 4.5 % slower)
// L2 hints: 1 = the unit loads are evict-first (each byte is read once), 2 = the
// output stores too (measured at config 1: 74.7 us without, 73.4 with 1, 73.1 with 2)
constexpr int kQkHint = JO_QK_HINT;
constexpr uint32_t kQkBarBytes = (8u * kQkWarps * kQkSlots + 127u) & ~127u;
constexpr int kQkMaxIt = 16;  // head iterations held in registers (H <= 16 * 32/(D/8))

__device__ __forceinline__ float2 bf2f(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
// (lo(a), lo(b)) and (hi(a), hi(b)): even / odd elements of two bf16 pairs
__device__ __forceinline__ float2 bf_lo2(uint32_t a, uint32_t b) {
  return make_float2(__uint_as_float(a << 16), __uint_as_float(b << 16));
}
__device__ __forceinline__ float2 bf_hi2(uint32_t a, uint32_t b) {
  return make_float2(__uint_as_float(a & 0xffff0000u), __uint_as_float(b & 0xffff0000u));
}

template <int kD, int kMode, bool kPre, bool kRope>
__global__ void __launch_bounds__(kQkWarps * 32, 1)
    qk_staged_kernel(const QkArgs a, int tok_per_cta, uint32_t slot_bytes, unsigned int* fault) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  constexpr int kTPH = kD / 8;
  constexpr int kHPI = 32 / kTPH;  // heads per warp iteration
  constexpr int kParts = kMode == kPack ? 3 : 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = lane % kTPH, sub = lane / kTPH;
  const int H = (int)a.heads;
  const int NI = (H + kHPI - 1) / kHPI;
  const int64_t ntok = (int64_t)a.total_rows / ((int64_t)kParts * H);
  const int64_t t0 = (int64_t)blockIdx.x * tok_per_cta;
  const int64_t t1 = t0 + tok_per_cta < ntok ? t0 + tok_per_cta : ntok;
  const int units = t1 > t0 ? (int)(t1 - t0) * kParts : 0;
  const uint32_t unit_bytes = (uint32_t)H * kD * 2u;
  const uint32_t base = smem_u32(smem_raw);
  if (threadIdx.x < kQkWarps * kQkSlots) mbar_init(base + 8u * threadIdx.x, 1);
  if (threadIdx.x == 0) mbar_init_fence();
  __syncthreads();
  pdl_wait();  // the previous kernel's outputs (our inputs) are complete from here on
  pdl_trigger();
  const uint32_t bar0 = base + 8u * (uint32_t)(warp * kQkSlots);
  const uint32_t slot0 = base + kQkBarBytes + (uint32_t)(warp * kQkSlots) * slot_bytes;
  uint64_t pol = 0;
  if constexpr (kQkHint > 0) pol = policy_evict_first();
  auto unit_ptr = [&](int i, int64_t& tok, int& part) -> __nv_bfloat16* {
    tok = t0 + i / kParts;
    part = i % kParts;
    if constexpr (kMode == kPack)
      return const_cast<__nv_bfloat16*>(a.qkv) + tok * a.qkv_stride + (int64_t)part * H * kD;
    else
      return (part ? a.k : a.q) + tok * (int64_t)H * kD;
  };
  // unit kk of this warp is unit warp + kk * kQkWarps of the CTA, slot kk % kQkSlots
  auto issue = [&](int kk) {
    const int i = warp + kk * kQkWarps;
    if (i >= units) return;
    int64_t tok;
    int part;
    const __nv_bfloat16* src = unit_ptr(i, tok, part);
    const uint32_t bar = bar0 + 8u * (uint32_t)(kk % kQkSlots);
    mbar_expect_tx(bar, unit_bytes);
    if constexpr (kQkHint > 0)
      bulk_load_hint(slot0 + (uint32_t)(kk % kQkSlots) * slot_bytes, src, unit_bytes, bar, pol);
    else
      bulk_load(slot0 + (uint32_t)(kk % kQkSlots) * slot_bytes, src, unit_bytes, bar);
  };
  if (lane == 0)
    for (int kk = 0; kk < kQkSlots; ++kk) issue(kk);
  // norm weights of this lane's 4 pairs as (even, odd) vectors of pair groups 0 / 1
  float2 wq0[2], wq1[2], wk0[2], wk1[2];
  {
    const uint4 q4 = ld_bcast(a.qw + j * 8), k4 = ld_bcast(a.kw + j * 8);
    wq0[0] = bf_lo2(q4.x, q4.y), wq1[0] = bf_hi2(q4.x, q4.y);
    wq0[1] = bf_lo2(q4.z, q4.w), wq1[1] = bf_hi2(q4.z, q4.w);
    wk0[0] = bf_lo2(k4.x, k4.y), wk1[0] = bf_hi2(k4.x, k4.y);
    wk0[1] = bf_lo2(k4.z, k4.w), wk1[1] = bf_hi2(k4.z, k4.w);
  }
  const float inv_d = 1.0f / (float)kD;  // exact for power-of-two D
  int kk = 0;
  for (; warp + kk * kQkWarps < units; ++kk) {
    const int i = warp + kk * kQkWarps;
    int64_t tok;
    int part;
    __nv_bfloat16* unit_dst = unit_ptr(i, tok, part);  // kInPlace destination
    const uint32_t bar = bar0 + 8u * (uint32_t)(kk % kQkSlots);
    const uint32_t sl = slot0 + (uint32_t)(kk % kQkSlots) * slot_bytes;
    if constexpr (kMode == kPack) {
      if (part == 2) {
        if (!mbar_wait(bar, (uint32_t)((kk / kQkSlots) & 1), fault)) break;
        __nv_bfloat16* vdst = a.out[2] + tok * a.os_t;
        for (int h = lane; h < H; h += 32) {
          if constexpr (kQkHint > 1)
            bulk_store_hint(vdst + (int64_t)h * a.os_h, sl + (uint32_t)h * kD * 2u, kD * 2u, pol);
          else
            bulk_store(vdst + (int64_t)h * a.os_h, sl + (uint32_t)h * kD * 2u, kD * 2u);
        }
        bulk_commit();
        bulk_wait_read_all();
        __syncwarp();
        if (lane == 0) issue(kk + kQkSlots);
        continue;
      }
    }
    float2 w0[2], w1[2];  // selected by value: a pointer select would put the arrays on the stack
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      w0[g] = part == 0 ? wq0[g] : wk0[g];
      w1[g] = part == 0 ? wq1[g] : wk1[g];
    }
    // folded rotation operands of pair groups 0 / 1: A = W0*C, B = -W1*S, C' = W0*S, D' = W1*C
    float2 fa[2], fb[2], fc[2], fd[2];
    if constexpr (kRope) {
      const int64_t rt = kMode == kPack ? tok : tok % a.seq_len;
      const uint2 c2 = __ldg(reinterpret_cast<const uint2*>(a.cos + rt * (kD / 2) + j * 4));
      const uint2 s2 = __ldg(reinterpret_cast<const uint2*>(a.sin + rt * (kD / 2) + j * 4));
      const float2 c[2] = {bf2f(c2.x), bf2f(c2.y)}, s[2] = {bf2f(s2.x), bf2f(s2.y)};
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        fa[g] = __fmul2_rn(w0[g], c[g]);
        fb[g] = __fmul2_rn(make_float2(-w1[g].x, -w1[g].y), s[g]);
        fc[g] = __fmul2_rn(w0[g], s[g]);
        fd[g] = __fmul2_rn(w1[g], c[g]);
      }
    }
    if (!mbar_wait(bar, (uint32_t)((kk / kQkSlots) & 1), fault)) break;
    uint4 v[kQkMaxIt];
#pragma unroll
    for (int it = 0; it < kQkMaxIt; ++it) {
      const int h = it * kHPI + sub;
      v[it] = (it < NI && h < H) ? lds128(sl + (uint32_t)(h * kD + j * 8) * 2u) : make_uint4(0, 0, 0, 0);
    }
    __syncwarp();
    if (lane == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // reads before the refill
      issue(kk + kQkSlots);
    }
    // destination of head row sub (+ kHPI per iteration), this lane's 16 bytes
    __nv_bfloat16* dst;
    int64_t step;
    if constexpr (kMode == kPack) {
      dst = a.out[part] + tok * a.os_t + (int64_t)sub * a.os_h + j * 8;
      step = (int64_t)kHPI * a.os_h;
    } else {
      dst = unit_dst + sub * kD + j * 8;
      step = (int64_t)kHPI * kD;
    }
    __nv_bfloat16* pre = nullptr;  // pre-RoPE k, laid out as k
    if constexpr (kPre) {
      if (part == 1) pre = a.k_pre + (kMode == kPack ? dst - a.out[1] : dst - a.k);
    }
    // groups of 4 head iterations, phase-major, so the 4 shuffle + rsqrt
    // dependency chains of a group overlap
#pragma unroll
    for (int g0 = 0; g0 < kQkMaxIt; g0 += 4) {
      if (g0 >= NI) break;  // uniform across the warp
      float2 e[4][2], o[4][2];
      float ss[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 u = v[g0 + q];
        e[q][0] = bf_lo2(u.x, u.y), o[q][0] = bf_hi2(u.x, u.y);
        e[q][1] = bf_lo2(u.z, u.w), o[q][1] = bf_hi2(u.z, u.w);
        float2 acc = __fmul2_rn(e[q][0], e[q][0]);
        acc = __ffma2_rn(o[q][0], o[q][0], acc);
        acc = __ffma2_rn(e[q][1], e[q][1], acc);
        acc = __ffma2_rn(o[q][1], o[q][1], acc);
        ss[q] = acc.x + acc.y;
      }
#pragma unroll
      for (int off = kTPH / 2; off > 0; off >>= 1)  // every lane, before any divergence
#pragma unroll
        for (int q = 0; q < 4; ++q) ss[q] += __shfl_xor_sync(0xffffffffu, ss[q], off);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int it = g0 + q;
        if (it >= NI || it * kHPI + sub >= H) continue;
        const float r = rsqrtf(fmaf(ss[q], inv_d, a.eps));
        const float2 r2 = make_float2(r, r);
        __nv_bfloat16* d = dst + it * step;
        uint32_t o4[4];
        if constexpr (!kRope) {
          // text rows: the model's RMSNorm rounds twice, bf16(x * r) then bf16(. * w)
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            const uint32_t n0 = pack_bf16x2(__fmul_rn(e[q][g].x, r), __fmul_rn(o[q][g].x, r));
            const uint32_t n1 = pack_bf16x2(__fmul_rn(e[q][g].y, r), __fmul_rn(o[q][g].y, r));
            const float2 ye = __fmul2_rn(bf_lo2(n0, n1), w0[g]), yo = __fmul2_rn(bf_hi2(n0, n1), w1[g]);
            o4[2 * g] = pack_bf16x2(ye.x, yo.x);
            o4[2 * g + 1] = pack_bf16x2(ye.y, yo.y);
          }
          if constexpr (kPre) {
            if (part == 1) st_global(pre + it * step, make_uint4(o4[0], o4[1], o4[2], o4[3]));
          }
          if constexpr (kQkHint > 1)
            st_global_hint(d, make_uint4(o4[0], o4[1], o4[2], o4[3]), pol);
          else
            st_global(d, make_uint4(o4[0], o4[1], o4[2], o4[3]));
          continue;
        }
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          e[q][g] = __fmul2_rn(e[q][g], r2);
          o[q][g] = __fmul2_rn(o[q][g], r2);
        }
        if constexpr (kPre) {
          if (part == 1) {  // pre-RoPE k: (x * r) * w
            uint32_t p4[4];
#pragma unroll
            for (int g = 0; g < 2; ++g) {
              const float2 ye = __fmul2_rn(e[q][g], w0[g]), yo = __fmul2_rn(o[q][g], w1[g]);
              p4[2 * g] = pack_bf16x2(ye.x, yo.x);
              p4[2 * g + 1] = pack_bf16x2(ye.y, yo.y);
            }
            st_global(pre + it * step, make_uint4(p4[0], p4[1], p4[2], p4[3]));
          }
        }
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          const float2 y0 = __ffma2_rn(o[q][g], fb[g], __fmul2_rn(e[q][g], fa[g]));  // x0 w0 c - x1 w1 s
          const float2 y1 = __ffma2_rn(o[q][g], fd[g], __fmul2_rn(e[q][g], fc[g]));  // x0 w0 s + x1 w1 c
          o4[2 * g] = pack_bf16x2(y0.x, y1.x);
          o4[2 * g + 1] = pack_bf16x2(y0.y, y1.y);
        }
        if constexpr (kQkHint > 1)
          st_global_hint(d, make_uint4(o4[0], o4[1], o4[2], o4[3]), pol);
        else
          st_global(d, make_uint4(o4[0], o4[1], o4[2], o4[3]));
      }
    }
  }
  // error path only (a wait expired at unit kk): every copy issued, unit kk's
  // included, must have landed (or its wait expired too) before the CTA exits
  if (lane == 0 && warp + kk * kQkWarps < units)
    for (int jj = kk; jj < kk + kQkSlots && warp + jj * kQkWarps < units; ++jj)
      mbar_wait(bar0 + 8u * (uint32_t)(jj % kQkSlots), (uint32_t)((jj / kQkSlots) & 1), fault);
}

template <int kD, int kMode, bool kPre, bool kRope>
int launch_qk_staged(const QkArgs& a, cudaStream_t st, const DeviceInfo* di, bool& taken) {
  constexpr int kParts = kMode == kPack ? 3 : 2;
  constexpr int kHPI = 32 / (kD / 8);
  taken = false;
  const uint32_t unit_bytes = a.heads * kD * 2u;
  const uint32_t slot_bytes = (unit_bytes + 127u) & ~127u;
  if ((int64_t)a.heads > (int64_t)kQkMaxIt * kHPI) return JO_OK;  // too many heads to hold: direct path
  const size_t smem = kQkBarBytes + (size_t)kQkWarps * kQkSlots * slot_bytes;
  if (smem > 220 * 1024) return JO_OK;
  taken = true;
  auto kern = qk_staged_kernel<kD, kMode, kPre, kRope>;
  static std::atomic<uint64_t> reserved{0};
  if (int s = reserve_smem((const void*)kern, 220 * 1024, reserved, di, "qk kernel")) return s;
  const int64_t ntok = (int64_t)a.total_rows / ((int64_t)kParts * a.heads);
  int64_t per = cdiv(ntok, di->sm_count);
  if (per < 2) per = 2;
  const int64_t grid = cdiv(ntok, per);
  if (cudaError_t e = launch_pdl(kern, dim3((unsigned)grid), dim3(kQkWarps * 32), smem, st, a, (int)per, slot_bytes,
                                 di->fault))
    return launch_failed(e, "qk kernel");
  return after_launch("qk_staged_kernel");
}

template <int kD, int kMode, bool kPre, bool kRope>
int launch_qk(const QkArgs& a, cudaStream_t st, const DeviceInfo* di) {
  auto kern = qk_norm_rope_kernel<kD, kMode, kPre, kRope>;
  constexpr int chunk = (kThreads / (kD / 8)) * kUnroll;
  const int64_t need = cdiv(a.total_rows, chunk);
  static int occ = 0;  // resident CTAs per SM; identical on every B200
  if (!occ) occ = occupancy((const void*)kern, kThreads, 0);
  const int64_t cap = (int64_t)di->sm_count * occ;
  const int64_t grid = need < cap ? need : cap;
  if (grid <= 0) return JO_OK;
  kern<<<(unsigned)grid, kThreads, 0, st>>>(a);
  return after_launch("qk_norm_rope_kernel");
}

template <int kD, int kMode, bool kPre, bool kRope>
int run_qk(const QkArgs& a, cudaStream_t st, const DeviceInfo* di) {
  bool taken = false;
  const int s = launch_qk_staged<kD, kMode, kPre, kRope>(a, st, di, taken);
  if (taken) return s;
  return launch_qk<kD, kMode, kPre, kRope>(a, st, di);
}

template <int kD, int kMode>
int run_qk_flags(bool pre, bool rope, const QkArgs& a, cudaStream_t st, const DeviceInfo* di) {
  if (rope) return pre ? run_qk<kD, kMode, true, true>(a, st, di) : run_qk<kD, kMode, false, true>(a, st, di);
  return pre ? run_qk<kD, kMode, true, false>(a, st, di) : run_qk<kD, kMode, false, false>(a, st, di);
}

template <int kMode>
int dispatch_qk(int64_t head_dim, bool pre, const QkArgs& a, cudaStream_t st,
                const DeviceInfo* di) {
  const bool rope = a.cos != nullptr;
  switch (head_dim) {
    case 64: return run_qk_flags<64, kMode>(pre, rope, a, st, di);
    case 128: return run_qk_flags<128, kMode>(pre, rope, a, st, di);
    case 256: return run_qk_flags<256, kMode>(pre, rope, a, st, di);
    default: return fail(JO_ERR_SHAPE, "head_dim must be 64, 128 or 256, got %lld", (long long)head_dim);
  }
}

// ---------------------------------------------------------------------------
// Joint / cached packs (D = 128).  Row sources are strided [1, L, H, 128] views.
struct View {
  const __nv_bfloat16* p;
  int64_t sl, sh;
};

__device__ __forceinline__ const __nv_bfloat16* view_row(const View& v, uint32_t row, uint32_t heads) {
  const uint32_t t = row / heads, h = row - t * heads;
  return v.p + (int64_t)t * v.sl + (int64_t)h * v.sh;
}

template <bool kVec>
__device__ __forceinline__ uint4 load_row_chunk(const __nv_bfloat16* p) {
  if constexpr (kVec) {
    return ld_stream(p);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t lo = *reinterpret_cast<const unsigned short*>(p + 2 * e);
      const uint32_t hi = *reinterpret_cast<const unsigned short*>(p + 2 * e + 1);
      w[e] = lo | (hi << 16);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
}

struct JointArgs {
  View iq, ik, iv, tq, tk, tv, ck, cv;
  const __nv_bfloat16* qw;
  const __nv_bfloat16* kw;
  __nv_bfloat16* oq;
  __nv_bfloat16* ok;
  __nv_bfloat16* ov;
  uint32_t heads, img_rows, txt_rows, cache_rows, q_rows, kv_rows, total_rows;
  float eps;
};

// Text RMSNorm of fused_joint_qkv_pack.cu:59-79: bf16(x * rsqrt(mean(x^2)+eps))
// first, then bf16(normalized * w) -- two roundings, as the model's RMSNorm.
__device__ __forceinline__ void text_rmsnorm16(float* f, const float* w, float ss, float eps) {
  const float r = rsqrt_ieee(__fmul_rn(ss, 1.0f / 128.0f) + eps);
#pragma unroll
  for (int e = 0; e < 8; ++e) f[e] = round_through<__nv_bfloat16>(f[e] * r) * w[e];
}

template <bool kVec>
__global__ void __launch_bounds__(kThreads) joint_pack_kernel(const JointArgs a) {
  constexpr int kRowsPerPass = kThreads / 16;
  const int j = threadIdx.x % 16;
  const uint32_t sub = threadIdx.x / 16;
  float wq[8], wk[8];
  Elt<__nv_bfloat16>::unpack(ld_bcast(a.qw + j * 8), wq);
  Elt<__nv_bfloat16>::unpack(ld_bcast(a.kw + j * 8), wk);
  const uint32_t chunk = kRowsPerPass * kUnroll;
  for (uint32_t base = blockIdx.x * chunk; base < a.total_rows; base += gridDim.x * chunk) {
    uint4 v[kUnroll];
    __nv_bfloat16* dst[kUnroll];
    int norm[kUnroll];  // 0 none, 1 text q, 2 text k
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const uint32_t i = base + u * kRowsPerPass + sub;
      norm[u] = -1;
      v[u] = make_uint4(0, 0, 0, 0);
      if (i >= a.total_rows) continue;
      const __nv_bfloat16* src;
      if (i < a.q_rows) {
        dst[u] = a.oq + (int64_t)i * 128;
        if (i < a.img_rows) {
          src = view_row(a.iq, i, a.heads);
          norm[u] = 0;
        } else {
          src = view_row(a.tq, i - a.img_rows, a.heads);
          norm[u] = 1;
        }
      } else {
        const uint32_t r = i - a.q_rows;
        const bool isv = r >= a.kv_rows;
        const uint32_t kr = isv ? r - a.kv_rows : r;
        dst[u] = (isv ? a.ov : a.ok) + (int64_t)kr * 128;
        norm[u] = 0;
        if (kr < a.cache_rows) {
          src = view_row(isv ? a.cv : a.ck, kr, a.heads);
        } else if (kr - a.cache_rows < a.img_rows) {
          src = view_row(isv ? a.iv : a.ik, kr - a.cache_rows, a.heads);
        } else {
          src = view_row(isv ? a.tv : a.tk, kr - a.cache_rows - a.img_rows, a.heads);
          norm[u] = isv ? 0 : 2;
        }
      }
      v[u] = load_row_chunk<kVec>(src + j * 8);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      float f[8];
      Elt<__nv_bfloat16>::unpack(v[u], f);
      const float ss = head_sumsq<16>(f);  // all lanes, before any divergence
      if (norm[u] < 0) continue;
      if (norm[u] == 0) {
        st_global(dst[u] + j * 8, v[u]);
      } else {
        text_rmsnorm16(f, norm[u] == 1 ? wq : wk, ss, a.eps);
        st_global(dst[u] + j * 8, Elt<__nv_bfloat16>::pack(f));
      }
    }
  }
}

struct CachedArgs {
  View k0, v0, k1, v1;
  const float* cos;  // [len0+len1, 128]
  const float* sin;
  __nv_bfloat16* ok;
  __nv_bfloat16* ov;
  uint32_t heads, rows0, total_rows, all_rows;  // all_rows = 2 * total_rows
};

template <bool kVec>
__global__ void __launch_bounds__(kThreads) cached_pack_kernel(const CachedArgs a) {
  constexpr int kRowsPerPass = kThreads / 16;
  const int j = threadIdx.x % 16;
  const uint32_t sub = threadIdx.x / 16;
  const uint32_t chunk = kRowsPerPass * kUnroll;
  for (uint32_t base = blockIdx.x * chunk; base < a.all_rows; base += gridDim.x * chunk) {
    uint4 v[kUnroll];
    float4 c0[kUnroll], c1[kUnroll], s0[kUnroll], s1[kUnroll];
    bool isk[kUnroll], ok[kUnroll];
    uint32_t kr[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const uint32_t i = base + u * kRowsPerPass + sub;
      ok[u] = i < a.all_rows;
      if (!ok[u]) continue;
      const bool isv = i >= a.total_rows;
      const uint32_t r = isv ? i - a.total_rows : i;
      kr[u] = r;
      isk[u] = !isv;
      const bool second = r >= a.rows0;
      const View& vw = isv ? (second ? a.v1 : a.v0) : (second ? a.k1 : a.k0);
      v[u] = load_row_chunk<kVec>(view_row(vw, second ? r - a.rows0 : r, a.heads) + j * 8);
      if (!isv) {
        const int64_t fo = (int64_t)(r / a.heads) * 128 + j * 8;
        c0[u] = __ldg(reinterpret_cast<const float4*>(a.cos + fo));
        c1[u] = __ldg(reinterpret_cast<const float4*>(a.cos + fo + 4));
        s0[u] = __ldg(reinterpret_cast<const float4*>(a.sin + fo));
        s1[u] = __ldg(reinterpret_cast<const float4*>(a.sin + fo + 4));
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (!ok[u]) continue;
      if (!isk[u]) {
        st_global(a.ov + (int64_t)kr[u] * 128 + j * 8, v[u]);
      } else {
        float f[8];
        Elt<__nv_bfloat16>::unpack(v[u], f);
        // full-width fp32 tables: the pair (2m, 2m+1) uses entry 2m
        // (fused_joint_qkv_pack.cu:209-216)
        const float c[4] = {c0[u].x, c0[u].z, c1[u].x, c1[u].z};
        const float s[4] = {s0[u].x, s0[u].z, s1[u].x, s1[u].z};
        rope4(f, c, s);
        st_global(a.ok + (int64_t)kr[u] * 128 + j * 8, Elt<__nv_bfloat16>::pack(f));
      }
    }
  }
}

template <typename K, typename A>
int launch_grid(K kern, const A& a, uint32_t rows, cudaStream_t st, const DeviceInfo* di,
                const char* what) {
  constexpr int chunk = (kThreads / 16) * kUnroll;
  const int64_t need = cdiv(rows, chunk);
  const int64_t cap = (int64_t)di->sm_count * occupancy((const void*)kern, kThreads, 0);
  const int64_t grid = need < cap ? need : cap;
  if (grid <= 0) return JO_OK;
  kern<<<(unsigned)grid, kThreads, 0, st>>>(a);
  return after_launch(what);
}

bool view_aligned(const jo_view4& v) {
  return aligned16(v.ptr) && (v.stride_l % 8 == 0) && (v.stride_h % 8 == 0);
}
View to_view(const jo_view4& v) {
  return View{reinterpret_cast<const __nv_bfloat16*>(v.ptr), v.stride_l, v.stride_h};
}

}  // namespace
}  // namespace jo

using namespace jo;

extern "C" {

int jo_qkv_norm_rope_pack(void* out_q, void* out_k, void* out_v, void* k_pre_rope,
                          int64_t out_stride_h, int64_t out_stride_t, const void* qkv,
                          int64_t qkv_row_stride, int64_t tokens, int64_t heads,
                          int64_t head_dim, const void* q_weight, const void* k_weight,
                          const void* cos, const void* sin, float eps, void* stream) {
  const char* op = "qkv_norm_rope_pack";
  const DeviceInfo* di;
  if (int s = device_info(&di)) return s;
  if (tokens < 0 || heads <= 0) return fail(JO_ERR_SHAPE, "%s: bad tokens/heads", op);
  if (tokens == 0) return JO_OK;
  if (tokens * 3 * heads > (int64_t)INT32_MAX)
    return fail(JO_ERR_SHAPE, "%s: tokens*3*heads exceeds 2^31", op);
  if (!out_q || !out_k || !out_v || !qkv || !q_weight || !k_weight)
    return fail(JO_ERR_INVALID, "%s: null operand", op);
  if ((cos == nullptr) != (sin == nullptr))
    return fail(JO_ERR_INVALID, "%s: cos and sin must both be given (RoPE) or both be null (text rows)", op);
  if (qkv_row_stride < 3 * heads * head_dim) return fail(JO_ERR_SHAPE, "%s: qkv row stride too small", op);
  const void* ptrs[] = {out_q, out_k, out_v, qkv, q_weight, k_weight};
  for (const void* p : ptrs)
    if (!aligned16(p)) return fail(JO_ERR_ALIGN, "%s: operands must be 16-byte aligned", op);
  if (k_pre_rope && !aligned16(k_pre_rope)) return fail(JO_ERR_ALIGN, "%s: k_pre_rope alignment", op);
  if ((reinterpret_cast<uintptr_t>(cos) | reinterpret_cast<uintptr_t>(sin)) & 7)
    return fail(JO_ERR_ALIGN, "%s: cos/sin must be 8-byte aligned", op);
  if (qkv_row_stride % 8 || out_stride_h % 8 || out_stride_t % 8)
    return fail(JO_ERR_ALIGN, "%s: strides must be multiples of 8 elements", op);
  QkArgs a{};
  a.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv);
  a.qkv_stride = qkv_row_stride;
  a.out[0] = reinterpret_cast<__nv_bfloat16*>(out_q);
  a.out[1] = reinterpret_cast<__nv_bfloat16*>(out_k);
  a.out[2] = reinterpret_cast<__nv_bfloat16*>(out_v);
  a.os_h = out_stride_h;
  a.os_t = out_stride_t;
  a.k_pre = reinterpret_cast<__nv_bfloat16*>(k_pre_rope);
  a.qw = reinterpret_cast<const __nv_bfloat16*>(q_weight);
  a.kw = reinterpret_cast<const __nv_bfloat16*>(k_weight);
  a.cos = reinterpret_cast<const __nv_bfloat16*>(cos);
  a.sin = reinterpret_cast<const __nv_bfloat16*>(sin);
  a.heads = (uint32_t)heads;
  a.total_rows = (uint32_t)(tokens * 3 * heads);
  a.eps = eps;
  return dispatch_qk<kPack>(head_dim, k_pre_rope != nullptr, a, (cudaStream_t)stream, di);
}

int jo_qk_norm_rope_3d_paired(void* q, void* k, int64_t batch, int64_t seq_len,
                              int64_t num_heads, int64_t head_dim, float eps,
                              const void* q_weight, const void* k_weight, const void* cos,
                              const void* sin, void* k_pre_rope, void* stream) {
  const char* op = "qk_norm_rope_3d_paired";
  const DeviceInfo* di;
  if (int s = device_info(&di)) return s;
  if (batch < 0 || seq_len < 0 || num_heads <= 0) return fail(JO_ERR_SHAPE, "%s: bad sizes", op);
  const int64_t rows = batch * seq_len * num_heads;
  if (rows == 0) return JO_OK;
  if (2 * rows > (int64_t)INT32_MAX) return fail(JO_ERR_SHAPE, "%s: too many rows", op);
  if (!q || !k || !q_weight || !k_weight || !cos || !sin) return fail(JO_ERR_INVALID, "%s: null operand", op);
  const void* ptrs[] = {q, k, q_weight, k_weight};
  for (const void* p : ptrs)
    if (!aligned16(p)) return fail(JO_ERR_ALIGN, "%s: operands must be 16-byte aligned", op);
  if (k_pre_rope && !aligned16(k_pre_rope)) return fail(JO_ERR_ALIGN, "%s: k_pre_rope alignment", op);
  if ((reinterpret_cast<uintptr_t>(cos) | reinterpret_cast<uintptr_t>(sin)) & 7)
    return fail(JO_ERR_ALIGN, "%s: cos/sin must be 8-byte aligned", op);
  QkArgs a{};
  a.q = reinterpret_cast<__nv_bfloat16*>(q);
  a.k = reinterpret_cast<__nv_bfloat16*>(k);
  a.seq_len = (int)seq_len;
  a.k_pre = reinterpret_cast<__nv_bfloat16*>(k_pre_rope);
  a.qw = reinterpret_cast<const __nv_bfloat16*>(q_weight);
  a.kw = reinterpret_cast<const __nv_bfloat16*>(k_weight);
  a.cos = reinterpret_cast<const __nv_bfloat16*>(cos);
  a.sin = reinterpret_cast<const __nv_bfloat16*>(sin);
  a.heads = (uint32_t)num_heads;
  a.total_rows = (uint32_t)(2 * rows);
  a.eps = eps;
  return dispatch_qk<kInPlace>(head_dim, k_pre_rope != nullptr, a, (cudaStream_t)stream, di);
}

int jo_joint_qkv_pack(void* out_q, void* out_k, void* out_v, jo_view4 img_q, jo_view4 img_k,
                      jo_view4 img_v, jo_view4 txt_q, jo_view4 txt_k, jo_view4 txt_v,
                      jo_view4 cache_k, jo_view4 cache_v, const void* txt_q_weight,
                      const void* txt_k_weight, int64_t heads, float eps, void* stream) {
  const char* op = "joint_qkv_pack";
  const DeviceInfo* di;
  if (int s = device_info(&di)) return s;
  if (heads <= 0 || img_q.len <= 0 || txt_q.len <= 0)
    return fail(JO_ERR_SHAPE, "%s: image/text lengths and heads must be positive", op);
  if (img_k.len != img_q.len || img_v.len != img_q.len || txt_k.len != txt_q.len ||
      txt_v.len != txt_q.len)
    return fail(JO_ERR_SHAPE, "%s: Q/K/V lengths must match", op);
  const bool has_cache = cache_k.ptr != nullptr;
  if (has_cache != (cache_v.ptr != nullptr))
    return fail(JO_ERR_INVALID, "%s: cached_k and cached_v must both be present or absent", op);
  const int64_t cache_len = has_cache ? cache_k.len : 0;
  if (has_cache && cache_v.len != cache_len) return fail(JO_ERR_SHAPE, "%s: cache K/V lengths differ", op);
  if (!out_q || !out_k || !out_v || !img_q.ptr || !img_k.ptr || !img_v.ptr || !txt_q.ptr ||
      !txt_k.ptr || !txt_v.ptr || !txt_q_weight || !txt_k_weight)
    return fail(JO_ERR_INVALID, "%s: null operand", op);
  const int64_t q_rows = (img_q.len + txt_q.len) * heads;
  const int64_t kv_rows = (cache_len + img_q.len + txt_q.len) * heads;
  if (q_rows + 2 * kv_rows > (int64_t)INT32_MAX) return fail(JO_ERR_SHAPE, "%s: too many rows", op);
  if (!aligned16(out_q) || !aligned16(out_k) || !aligned16(out_v) || !aligned16(txt_q_weight) ||
      !aligned16(txt_k_weight))
    return fail(JO_ERR_ALIGN, "%s: outputs and weights must be 16-byte aligned", op);
  JointArgs a{};
  a.iq = to_view(img_q);
  a.ik = to_view(img_k);
  a.iv = to_view(img_v);
  a.tq = to_view(txt_q);
  a.tk = to_view(txt_k);
  a.tv = to_view(txt_v);
  a.ck = has_cache ? to_view(cache_k) : View{nullptr, 0, 0};
  a.cv = has_cache ? to_view(cache_v) : View{nullptr, 0, 0};
  a.qw = reinterpret_cast<const __nv_bfloat16*>(txt_q_weight);
  a.kw = reinterpret_cast<const __nv_bfloat16*>(txt_k_weight);
  a.oq = reinterpret_cast<__nv_bfloat16*>(out_q);
  a.ok = reinterpret_cast<__nv_bfloat16*>(out_k);
  a.ov = reinterpret_cast<__nv_bfloat16*>(out_v);
  a.heads = (uint32_t)heads;
  a.img_rows = (uint32_t)(img_q.len * heads);
  a.txt_rows = (uint32_t)(txt_q.len * heads);
  a.cache_rows = (uint32_t)(cache_len * heads);
  a.q_rows = (uint32_t)q_rows;
  a.kv_rows = (uint32_t)kv_rows;
  a.total_rows = (uint32_t)(q_rows + 2 * kv_rows);
  a.eps = eps;
  bool vec = view_aligned(img_q) && view_aligned(img_k) && view_aligned(img_v) &&
             view_aligned(txt_q) && view_aligned(txt_k) && view_aligned(txt_v);
  if (has_cache) vec = vec && view_aligned(cache_k) && view_aligned(cache_v);
  cudaStream_t st = (cudaStream_t)stream;
  return vec ? launch_grid(joint_pack_kernel<true>, a, a.total_rows, st, di, "joint_pack_kernel")
             : launch_grid(joint_pack_kernel<false>, a, a.total_rows, st, di, "joint_pack_kernel");
}

int jo_cached_kv_pack(void* out_key, void* out_value, jo_view4 key0, jo_view4 value0,
                      jo_view4 key1, jo_view4 value1, const float* cos, const float* sin,
                      int64_t heads, void* stream) {
  const char* op = "cached_kv_pack";
  const DeviceInfo* di;
  if (int s = device_info(&di)) return s;
  if (heads <= 0 || key0.len <= 0) return fail(JO_ERR_SHAPE, "%s: cache length and heads must be positive", op);
  // K only (value0.ptr == out_value == NULL): rotate the keys, copy no values
  const bool has_v = value0.ptr != nullptr;
  if (!has_v && (out_value != nullptr || value1.ptr != nullptr))
    return fail(JO_ERR_INVALID, "%s: without value0, out_value and value1 must be null too", op);
  if (has_v && value0.len != key0.len) return fail(JO_ERR_SHAPE, "%s: key0/value0 lengths must match", op);
  const bool two = key1.ptr != nullptr;
  if (has_v && two != (value1.ptr != nullptr))
    return fail(JO_ERR_INVALID, "%s: key1 and value1 must both be present or absent", op);
  if (two && (key1.len <= 0 || (has_v && value1.len != key1.len)))
    return fail(JO_ERR_SHAPE, "%s: key1/value1 lengths must match and be positive", op);
  if (!out_key || (has_v && !out_value) || !key0.ptr || !cos || !sin)
    return fail(JO_ERR_INVALID, "%s: null operand", op);
  const int64_t len1 = two ? key1.len : 0;
  const int64_t total = (key0.len + len1) * heads;
  if (2 * total > (int64_t)INT32_MAX) return fail(JO_ERR_SHAPE, "%s: too many rows", op);
  if (!aligned16(out_key) || (has_v && !aligned16(out_value)) || !aligned16(cos) || !aligned16(sin))
    return fail(JO_ERR_ALIGN, "%s: outputs and cos/sin must be 16-byte aligned", op);
  CachedArgs a{};
  a.k0 = to_view(key0);
  a.v0 = has_v ? to_view(value0) : View{nullptr, 0, 0};
  a.k1 = two ? to_view(key1) : View{nullptr, 0, 0};
  a.v1 = two && has_v ? to_view(value1) : View{nullptr, 0, 0};
  a.cos = cos;
  a.sin = sin;
  a.ok = reinterpret_cast<__nv_bfloat16*>(out_key);
  a.ov = reinterpret_cast<__nv_bfloat16*>(out_value);
  a.heads = (uint32_t)heads;
  a.rows0 = (uint32_t)(key0.len * heads);
  a.total_rows = (uint32_t)total;
  a.all_rows = (uint32_t)(has_v ? 2 * total : total);
  bool vec = view_aligned(key0) && (!has_v || view_aligned(value0));
  if (two) vec = vec && view_aligned(key1) && (!has_v || view_aligned(value1));
  cudaStream_t st = (cudaStream_t)stream;
  return vec ? launch_grid(cached_pack_kernel<true>, a, a.all_rows, st, di, "cached_pack_kernel")
             : launch_grid(cached_pack_kernel<false>, a, a.all_rows, st, di, "cached_pack_kernel");
}

}  // extern "C"
