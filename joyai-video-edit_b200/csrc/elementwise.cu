// Elementwise activations and the sinusoidal timestep projection.
//
//   jo_gelu_tanh           F.gelu(x, approximate="tanh")  (deploy/xvideo/models/dit/dit.py:87-89)
//   jo_silu_mul            silu(a) * b                    (SiLU-gated MLP; no reference kernel)
//   jo_timestep_embedding  diffusers Timesteps(256, flip_sin_to_cos=True, shift=0)
//                          (deploy/xvideo/models/dit/dit.py:574-575, 614)
//
// Design (B200): GELU and SiLU-mul are pure HBM streams; each thread moves
// kUnroll 16-byte vectors per grid-stride step with all loads issued first.
// The per-element math is kept short so the kernels stay memory-bound at
// ~8 TB/s: 0.5*(1+tanh(u)) is evaluated as the identical logistic 1/(1+e^(-2u)),
// one exp and one division, instead of a full tanh.
#include <math.h>

#include "common.cuh"

namespace jo {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

// gelu_tanh_f / gelu_vec (common.cuh): x * sigmoid(2u), the identical form of
// 0.5 * x * (1 + tanh(u)).

__device__ __forceinline__ float silu_f(float a) {
  const float e = __expf(fminf(-a, 80.f));
  return __fdividef(a, 1.f + e);
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
    gelu_vec_kernel(T* __restrict__ out, const T* __restrict__ x, int64_t nvec) {
  constexpr int V = Elt<T>::kVec;
  pdl_wait();  // launched with launch_pdl: inputs complete from here on
  pdl_trigger();
  const int64_t stride = (int64_t)gridDim.x * kThreads * kUnroll;
  for (int64_t base = (int64_t)blockIdx.x * kThreads * kUnroll + threadIdx.x; base < nvec;
       base += stride) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + (int64_t)u * kThreads;
      if (i < nvec) v[u] = ld_stream(x + i * V);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + (int64_t)u * kThreads;
      if (i < nvec) {
        st_global(out + i * V, gelu_vec<T>(v[u]));
      }
    }
  }
}

template <typename T>
__global__ void gelu_scalar_kernel(T* __restrict__ out, const T* __restrict__ x, int64_t begin,
                                   int64_t n) {
  for (int64_t i = begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = Elt<T>::from_f(gelu_tanh_f(Elt<T>::to_f(x[i])));
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
    silu_mul_vec_kernel(T* __restrict__ out, int64_t os, const T* __restrict__ a, int64_t as,
                        const T* __restrict__ b, int64_t bs, int64_t rows, int64_t vpr) {
  constexpr int V = Elt<T>::kVec;
  pdl_wait();  // launched with launch_pdl: inputs complete from here on
  pdl_trigger();
  const int64_t nvec = rows * vpr;
  const int64_t stride = (int64_t)gridDim.x * kThreads * kUnroll;
  for (int64_t base = (int64_t)blockIdx.x * kThreads * kUnroll + threadIdx.x; base < nvec;
       base += stride) {
    uint4 va[kUnroll], vb[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + (int64_t)u * kThreads;
      if (i < nvec) {
        const int64_t r = i / vpr, c = (i - r * vpr) * V;
        va[u] = ld_stream(a + r * as + c);
        vb[u] = ld_stream(b + r * bs + c);
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + (int64_t)u * kThreads;
      if (i < nvec) {
        const int64_t r = i / vpr, c = (i - r * vpr) * V;
        float fa[V], fb[V];
        Elt<T>::unpack(va[u], fa);
        Elt<T>::unpack(vb[u], fb);
#pragma unroll
        for (int e = 0; e < V; ++e) fa[e] = silu_f(fa[e]) * fb[e];
        st_global(out + r * os + c, Elt<T>::pack(fa));
      }
    }
  }
}

template <typename T>
__global__ void silu_mul_scalar_kernel(T* __restrict__ out, int64_t os, const T* __restrict__ a,
                                       int64_t as, const T* __restrict__ b, int64_t bs,
                                       int64_t rows, int64_t cols) {
  const int64_t n = rows * cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    out[r * os + c] =
        Elt<T>::from_f(silu_f(Elt<T>::to_f(a[r * as + c])) * Elt<T>::to_f(b[r * bs + c]));
  }
}

// One CTA per timestep; thread i owns frequency i of dim/2.
__global__ void timestep_kernel(float* __restrict__ out, const float* __restrict__ t, int dim,
                                int flip, float shift, float scale, float neg_log_period) {
  const int half = dim / 2;
  const int b = blockIdx.x;
  const float tb = t[b];
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    // exponent = (-ln(max_period) * i) / (half - shift), then exp, all fp32
    const float ex = __fdiv_rn(__fmul_rn(neg_log_period, (float)i), (float)half - shift);
    const float arg = __fmul_rn(scale, __fmul_rn(tb, expf(ex)));
    float s, c;
    sincosf(arg, &s, &c);
    float* o = out + (int64_t)b * dim;
    o[flip ? i : half + i] = c;
    o[flip ? half + i : i] = s;
  }
  if ((dim & 1) && threadIdx.x == 0) out[(int64_t)b * dim + dim - 1] = 0.f;
}

template <typename K>
int grid_for(K kern, int64_t work_items, const DeviceInfo* di) {
  const int64_t need = cdiv(work_items, (int64_t)kThreads * kUnroll);
  const int64_t cap = (int64_t)di->sm_count * occupancy((const void*)kern, kThreads, 0) * 4;
  return (int)(need < cap ? need : cap);
}

template <typename T>
int gelu_t(void* out, const void* x, int64_t n, cudaStream_t st, const DeviceInfo* di) {
  constexpr int V = Elt<T>::kVec;
  T* o = reinterpret_cast<T*>(out);
  const T* xi = reinterpret_cast<const T*>(x);
  int64_t done = 0;
  if (aligned16(out) && aligned16(x)) {
    const int64_t nvec = n / V;
    if (nvec > 0) {
      const int grid = grid_for(gelu_vec_kernel<T>, nvec, di);
      if (cudaError_t e = launch_pdl(gelu_vec_kernel<T>, dim3(grid), dim3(kThreads), 0, st, o, xi, nvec))
        return launch_failed(e, "gelu_tanh");
      if (int s = after_launch("gelu_vec_kernel")) return s;
    }
    done = nvec * V;
  }
  if (done < n) {
    const int64_t rest = n - done;
    const int grid = (int)std::min<int64_t>(cdiv(rest, kThreads), (int64_t)di->sm_count * 8);
    gelu_scalar_kernel<T><<<grid, kThreads, 0, st>>>(o, xi, done, n);
    return after_launch("gelu_scalar_kernel");
  }
  return JO_OK;
}

template <typename T>
int silu_mul_t(void* out, int64_t os, const void* a, int64_t as, const void* b, int64_t bs,
               int64_t rows, int64_t cols, cudaStream_t st, const DeviceInfo* di) {
  constexpr int V = Elt<T>::kVec;
  T* o = reinterpret_cast<T*>(out);
  const T* pa = reinterpret_cast<const T*>(a);
  const T* pb = reinterpret_cast<const T*>(b);
  const bool vec = aligned16(out) && aligned16(a) && aligned16(b) && cols % V == 0 &&
                   (os * (int64_t)sizeof(T)) % 16 == 0 && (as * (int64_t)sizeof(T)) % 16 == 0 &&
                   (bs * (int64_t)sizeof(T)) % 16 == 0;
  if (vec) {
    const int64_t vpr = cols / V;
    const int grid = grid_for(silu_mul_vec_kernel<T>, rows * vpr, di);
    if (cudaError_t e = launch_pdl(silu_mul_vec_kernel<T>, dim3(grid), dim3(kThreads), 0, st, o, os, pa, as, pb, bs,
                                   rows, vpr))
      return launch_failed(e, "silu_mul");
    return after_launch("silu_mul_vec_kernel");
  }
  const int grid = (int)std::min<int64_t>(cdiv(rows * cols, kThreads), (int64_t)di->sm_count * 8);
  silu_mul_scalar_kernel<T><<<grid, kThreads, 0, st>>>(o, os, pa, as, pb, bs, rows, cols);
  return after_launch("silu_mul_scalar_kernel");
}

}  // namespace
}  // namespace jo

using namespace jo;

extern "C" {

int jo_gelu_tanh(void* out, const void* x, int64_t n, int dtype, void* stream) {
  const DeviceInfo* di;
  if (int s = device_info(&di)) return s;
  if (n < 0) return fail(JO_ERR_SHAPE, "gelu_tanh: negative size");
  if (n == 0) return JO_OK;
  if (!out || !x) return fail(JO_ERR_INVALID, "gelu_tanh: null operand");
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case JO_BF16: return gelu_t<__nv_bfloat16>(out, x, n, st, di);
    case JO_F16: return gelu_t<__half>(out, x, n, st, di);
    case JO_F32: return gelu_t<float>(out, x, n, st, di);
    default: return fail(JO_ERR_DTYPE, "gelu_tanh: unsupported dtype %d", dtype);
  }
}

int jo_silu_mul(void* out, int64_t out_row_stride, const void* a, int64_t a_row_stride,
                const void* b, int64_t b_row_stride, int64_t rows, int64_t cols, int dtype,
                void* stream) {
  const DeviceInfo* di;
  if (int s = device_info(&di)) return s;
  if (rows < 0 || cols < 0) return fail(JO_ERR_SHAPE, "silu_mul: negative size");
  if (rows == 0 || cols == 0) return JO_OK;
  if (!out || !a || !b) return fail(JO_ERR_INVALID, "silu_mul: null operand");
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case JO_BF16:
      return silu_mul_t<__nv_bfloat16>(out, out_row_stride, a, a_row_stride, b, b_row_stride, rows, cols, st, di);
    case JO_F16:
      return silu_mul_t<__half>(out, out_row_stride, a, a_row_stride, b, b_row_stride, rows, cols, st, di);
    case JO_F32:
      return silu_mul_t<float>(out, out_row_stride, a, a_row_stride, b, b_row_stride, rows, cols, st, di);
    default: return fail(JO_ERR_DTYPE, "silu_mul: unsupported dtype %d", dtype);
  }
}

int jo_timestep_embedding(float* out, const float* t, int64_t batch, int64_t dim,
                          int flip_sin_to_cos, float downscale_freq_shift, float scale,
                          float max_period, void* stream) {
  const DeviceInfo* di;
  if (int s = device_info(&di)) return s;
  if (batch < 0 || dim < 2 || dim > 65536) return fail(JO_ERR_SHAPE, "timestep_embedding: bad sizes");
  if (batch == 0) return JO_OK;
  if (batch > (int64_t)INT32_MAX) return fail(JO_ERR_SHAPE, "timestep_embedding: batch too large");
  if (!out || !t) return fail(JO_ERR_INVALID, "timestep_embedding: null operand");
  if (!(max_period > 0.f)) return fail(JO_ERR_INVALID, "timestep_embedding: max_period must be > 0");
  // -math.log(max_period) is a Python double rounded to fp32 when it meets the
  // fp32 arange (diffusers get_timestep_embedding).
  const float neg_log = (float)(-log((double)max_period));
  const int threads = (int)std::min<int64_t>(256, ((dim / 2) + 31) / 32 * 32);
  timestep_kernel<<<(unsigned)batch, threads, 0, (cudaStream_t)stream>>>(
      out, t, (int)dim, flip_sin_to_cos, downscale_freq_shift, scale, neg_log);
  return after_launch("timestep_kernel");
}

}  // extern "C"
