// Shared device/host helpers for the sm_100a joyomni kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "joyomni_b200.h"

namespace jo {

// ---------------------------------------------------------------- host side
// Records `fmt` as the thread's last error and returns `code`.
int fail(int code, const char* fmt, ...);
// Checks cudaGetLastError() after a launch; counts the launch.
int after_launch(const char* what);
// A launch call returned `e`: clear the runtime's pending error (so the next
// call does not report it) and return JO_ERR_CUDA with the reason.
int launch_failed(cudaError_t e, const char* what);
// Per-device facts, cached on first use.  Returns JO_OK or an error status.
struct DeviceInfo {
  int ordinal;  // CUDA device index (< 64)
  int sm_count;
  int major, minor;
  int max_smem_optin;
  unsigned int* fault;  // device address of this device's fault counter
};
int device_info(const DeviceInfo** out);
// Device address of a __device__ symbol (its host-side shadow `symbol`) on the
// current device `dev`, cached per device.  The cache is keyed by the device's
// context: a context created anew (after cudaDeviceReset, the module is loaded
// again and the symbol may move) is looked up again.  `stream` (may be null) is
// checked before a lookup: a lookup is refused while it is capturing, since the
// first lookup on a device may load the module.
struct SymbolCache {
  std::atomic<uint64_t> ctx[64];
  std::atomic<void*> addr[64];
};
int symbol_address(SymbolCache& cache, const void* symbol, int dev, cudaStream_t stream, void** out,
                   const char* what);
// Raises `kernel`'s dynamic shared-memory limit to `bytes` on the current device,
// once per device: the attribute is per device, so `done` (one per kernel, at
// the call site) records the devices already set (bit = device ordinal).
int reserve_smem(const void* kernel, int bytes, std::atomic<uint64_t>& done, const DeviceInfo* di,
                 const char* what);
// Asks for `kernel` to run with the whole shared-memory carveout (once per device, as
// reserve_smem): a kernel that shares SMs with a large-shared-memory successor then
// leaves no carveout change (which needs the SM to drain) in that successor's way.
int prefer_max_carveout(const void* kernel, std::atomic<uint64_t>& done, const DeviceInfo* di, const char* what);
// Resident CTAs per SM for `kernel` at `threads` threads and `smem` bytes.
int occupancy(const void* kernel, int threads, size_t smem);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Programmatic dependent launch: the kernel may be scheduled while the previous
// kernel of the stream is still finishing; it touches global memory only after
// pdl_wait() (which returns once that kernel has completed and its writes are
// visible) and lets its own successor be scheduled with pdl_trigger().  Kernels
// launched this way do nothing before pdl_wait() but set up shared memory,
// barriers and tensor memory.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...);
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------- device side
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Sum over aligned groups of G lanes (G a power of two <= 32).
template <int G>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// 16-byte global accesses.  Read-once data uses the non-coherent path without
// L1 allocation; broadcast operands use plain __ldg.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint4 ld_bcast(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ void st_global(void* p, const uint4& v) {
  *reinterpret_cast<uint4*>(p) = v;
}

// Element traits: 16-byte vectors of T, conversion to/from fp32.
template <typename T>
struct Elt;
template <>
struct Elt<float> {
  static constexpr int kVec = 4;
  __device__ __forceinline__ static float to_f(float v) { return v; }
  __device__ __forceinline__ static float from_f(float v) { return v; }
  __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
  }
};
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
struct Elt<__nv_bfloat16> {
  static constexpr int kVec = 8;
  __device__ __forceinline__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                      pack_bf16x2(f[6], f[7]));
  }
};
template <>
struct Elt<__half> {
  static constexpr int kVec = 8;
  __device__ __forceinline__ static float to_f(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half from_f(float v) { return __float2half_rn(v); }
  __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 t = __half22float2(h);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    return make_uint4(pack_f16x2(f[0], f[1]), pack_f16x2(f[2], f[3]), pack_f16x2(f[4], f[5]),
                      pack_f16x2(f[6], f[7]));
  }
};

// Round a float through T and back (the value a bf16/fp16 tensor would hold).
template <typename T>
__device__ __forceinline__ float round_through(float v) {
  return Elt<T>::to_f(Elt<T>::from_f(v));
}
template <>
__device__ __forceinline__ float round_through<float>(float v) {
  return v;
}

// e4m3 (float8_e4m3fn) conversion of two floats, round-to-nearest-even with
// saturation to +-448; `lo` lands in the low byte.
__device__ __forceinline__ uint16_t e4m3x2(float lo, float hi) {
  __nv_fp8x2_storage_t s = __nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3);
  return static_cast<uint16_t>(s);
}

// Per-token quantisation helpers, semantics of fp8_linear.py:38-43:
//   scale = max(amax, 1e-8) / 448 ; q = e4m3(clamp(x / scale, -448, 448)).
constexpr float kFp8Max = 448.0f;
__device__ __forceinline__ float quant_scale(float amax) {
  return __fdiv_rn(fmaxf(amax, 1e-8f), kFp8Max);
}
__device__ __forceinline__ float quant_clamp(float x, float scale) {
  float v = __fdiv_rn(x, scale);
  return fminf(fmaxf(v, -kFp8Max), kFp8Max);
}

// GELU, tanh approximation: x * sigmoid(2u), u = sqrt(2/pi) * (x + 0.044715 x^3);
// 0.5 * (1 + tanh(u)) == 1 / (1 + e^(-2u)) exactly.  Every step is spelled out
// (one rounding each) so that the scalar and the f32x2 forms below give the
// same bits:  t = fma(0.044715, x^3, x);  z = min(-2 sqrt(2/pi) t, 80);
// e = 2^(z log2(e)) with the hardware base-2 exponential (ex2.approx, relative
// error about 2^-22); y = x * rcp(1 + e) with the hardware reciprocal
// (rcp.approx, 1 ulp).  The cap keeps 1 + e <= 5.6e34, far from the flush-to-
// zero range of the reciprocal, so y keeps the sign of x (also for -0).
constexpr float kGeluC = 0.044715f;
constexpr float kGeluNegK = -1.5957691216057308f;  // -2 * sqrt(2/pi)
constexpr float kLog2E = 1.4426950408889634f;
__device__ __forceinline__ float ex2_approx(float v) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}
__device__ __forceinline__ float rcp_approx(float v) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}
__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float x3 = __fmul_rn(__fmul_rn(x, x), x);
  const float t = __fmaf_rn(kGeluC, x3, x);
  const float z = fminf(__fmul_rn(kGeluNegK, t), 80.f);
  const float e = ex2_approx(__fmul_rn(z, kLog2E));
  return __fmul_rn(x, rcp_approx(__fadd_rn(1.f, e)));
}
// Two elements at once: the same steps on the packed f32x2 pipe (half the
// issue slots of the scalar form); the exponential and reciprocal stay scalar.
__device__ __forceinline__ float2 gelu_tanh_f2(float2 x) {
  const float2 x3 = __fmul2_rn(__fmul2_rn(x, x), x);
  const float2 t = __ffma2_rn(make_float2(kGeluC, kGeluC), x3, x);
  float2 z = __fmul2_rn(make_float2(kGeluNegK, kGeluNegK), t);
  z = make_float2(fminf(z.x, 80.f), fminf(z.y, 80.f));
  z = __fmul2_rn(z, make_float2(kLog2E, kLog2E));
  const float2 d = __fadd2_rn(make_float2(1.f, 1.f), make_float2(ex2_approx(z.x), ex2_approx(z.y)));
  return __fmul2_rn(x, make_float2(rcp_approx(d.x), rcp_approx(d.y)));
}

// GELU-tanh of one 16-byte vector of T, rounded to T (the tensor the unfused
// chain materialises), two elements per step.
template <typename T>
__device__ __forceinline__ uint4 gelu_vec(const uint4& u) {
  float f[Elt<T>::kVec];
  Elt<T>::unpack(u, f);
#pragma unroll
  for (int e = 0; e < Elt<T>::kVec; e += 2) {
    const float2 g = gelu_tanh_f2(make_float2(f[e], f[e + 1]));
    f[e] = g.x;
    f[e + 1] = g.y;
  }
  return Elt<T>::pack(f);
}

// 1/sqrt(v) rounded as torch's CPU rsqrt (IEEE sqrt, then IEEE reciprocal).
__device__ __forceinline__ float rsqrt_ieee(float v) { return __fdiv_rn(1.0f, __fsqrt_rn(v)); }

}  // namespace jo

#define JO_CHECK_ARG(cond, code, ...)              \
  do {                                             \
    if (!(cond)) return ::jo::fail(code, __VA_ARGS__); \
  } while (0)
