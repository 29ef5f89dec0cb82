// Packed f32x2 helpers shared by the per-token FP8 quantisers (the row kernels'
// quant epilogue and the FP8 GEMM's GELU -> FP8 pass): a 16-byte vector as float
// pairs, the correctly rounded quotient x / s from RN(1/s), the signs of -0
// restored on packed e4m3 bytes, and a running |x| maximum over 16-bit floats.
#pragma once

#include "common.cuh"

namespace jo {

// ------------------------------------------------------------------ packed math
// A 16-byte vector of T as V/2 float pairs.
template <typename T>
__device__ __forceinline__ void to_pairs(const uint4& u, float2* p) {
  float f[Elt<T>::kVec];
  Elt<T>::unpack(u, f);
#pragma unroll
  for (int e = 0; e < Elt<T>::kVec / 2; ++e) p[e] = make_float2(f[2 * e], f[2 * e + 1]);
}
template <typename T>
__device__ __forceinline__ uint4 from_pairs(const float2* p) {
  float f[Elt<T>::kVec];
#pragma unroll
  for (int e = 0; e < Elt<T>::kVec / 2; ++e) {
    f[2 * e] = p[e].x;
    f[2 * e + 1] = p[e].y;
  }
  return Elt<T>::pack(f);
}
__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }

// Correctly rounded x / s from the correctly rounded reciprocal rc = RN(1/s):
// q0 = RN(x*rc), r = x - q0*s (exact with an FMA), q = RN(q0 + r*rc).
// Markstein, "Computation of elementary functions on the IBM RISC System/6000
// processor" (IBM J. Res. Dev. 34(1), 1990), Theorem 1; valid while nothing
// over- or underflows, which holds for |q| >= 2^-10, the only range where an
// e4m3 byte depends on the quotient.
// The quotient takes the sign of x (s > 0): copied back explicitly because the
// correction step turns x = -0 into (+0) + (-0) = +0.
__device__ __forceinline__ float2 div2_markstein(float2 x, float2 s, float2 rc) {
  const float2 q0 = __fmul2_rn(x, rc);
  const float2 r = __ffma2_rn(q0, make_float2(-s.x, -s.y), x);
  const float2 q = __ffma2_rn(r, rc, q0);
  return make_float2(copysignf(q.x, x.x), copysignf(q.y, x.y));
}
// The same quotient without the sign copy (ns = -s): for 16-bit inputs the
// sign of x = -0 is restored on the packed e4m3 bytes instead (e4m3_signs),
// one byte permute for four elements.
__device__ __forceinline__ float2 div2_ms(float2 x, float2 ns, float2 rc) {
  const float2 q0 = __fmul2_rn(x, rc);
  const float2 r = __ffma2_rn(q0, ns, x);
  return __ffma2_rn(r, rc, q0);
}
// Sign bits of the four 16-bit elements of words (w0, w1), at bit 7 of the
// byte each element's e4m3 code occupies.  OR-ing them in is exact: a nonzero
// quotient already carries its sign, a zero one gets the sign of x.
__device__ __forceinline__ uint32_t e4m3_signs(uint32_t w0, uint32_t w1) {
  return __byte_perm(w0, w1, 0x7531) & 0x80808080u;
}
// Running |x| maximum over packed 16-bit floats, one instruction per word:
// max.NaN.xorsign.abs gives max(|m|, |w|) per half with the XOR of the two
// signs in bit 15, so the magnitude bits hold the running maximum whatever
// sign the accumulator carries; a NaN operand makes the half NaN (as torch's
// amax).  Typed: a bf16 pattern read as fp16 could be mistaken for a NaN.
// amax16_bits reads the larger magnitude out of the two halves (bit patterns
// of non-negative values order as unsigned integers).
template <typename T>
__device__ __forceinline__ uint32_t absmax16x2(uint32_t m, uint32_t w);
template <>
__device__ __forceinline__ uint32_t absmax16x2<__nv_bfloat16>(uint32_t m, uint32_t w) {
  uint32_t r;
  asm("max.NaN.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(m), "r"(w));
  return r;
}
template <>
__device__ __forceinline__ uint32_t absmax16x2<__half>(uint32_t m, uint32_t w) {
  uint32_t r;
  asm("max.NaN.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(r) : "r"(m), "r"(w));
  return r;
}
template <>
__device__ __forceinline__ uint32_t absmax16x2<float>(uint32_t m, uint32_t) {
  return m;  // not used: fp32 rows keep a float maximum
}
__device__ __forceinline__ uint32_t amax16_bits(uint32_t m) {
  return max(m & 0x7fffu, (m >> 16) & 0x7fffu);
}
template <typename T>
__device__ __forceinline__ float bits16_to_f(uint32_t h);
template <>
__device__ __forceinline__ float bits16_to_f<__nv_bfloat16>(uint32_t h) {
  return __uint_as_float(h << 16);
}
template <>
__device__ __forceinline__ float bits16_to_f<__half>(uint32_t h) {
  return __half2float(__ushort_as_half((unsigned short)h));
}
template <>
__device__ __forceinline__ float bits16_to_f<float>(uint32_t) {
  return 0.f;
}

}  // namespace jo
