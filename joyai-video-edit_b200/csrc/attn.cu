// Merge of two partial attention results computed over disjoint key sets.
//
// Softmax attention over keys K = A u B (disjoint) splits exactly: with the
// per-(query, head) log-sum-exp l_A, l_B of the scaled scores and the partial
// outputs o_A, o_B (each normalised over its own keys),
//
//   m = max(l_A, l_B),  w_A = exp(l_A - m),  w_B = exp(l_B - m)
//   o = (w_A o_A + w_B o_B) / (w_A + w_B),   l = m + log(w_A + w_B)
//
// This is what lets the sequence-parallel block attend over the replicated
// cache rows while the NCCL all-gather of the current chunk's K/V is still in
// flight (the reference attends over [cache | img | txt] in one call,
// deploy/xvideo/models/dit/dit.py:154-189, 498).
//
// Design (B200): an HBM-bound elementwise pass (read o_A, o_B, write o; the
// log-sum-exps are 1/64 of the bytes): one 16-byte vector per thread and
// step, grid-stride over (row, head, vector), the two weights formed per
// thread from broadcast loads of the two log-sum-exps.
#include "common.cuh"

namespace jo {
namespace {

constexpr int kThreads = 256;

struct MergeArgs {
  void* out;
  int64_t os_s, os_h;
  const void* oa;
  int64_t as_s, as_h;
  const void* ob;
  int64_t bs_s, bs_h;
  const float* la;
  int64_t la_h, la_s;
  const float* lb;
  int64_t lb_h, lb_s;
  int64_t rows, heads;
  int vecs;  // 16-byte vectors per head row
};

template <typename T>
__global__ void __launch_bounds__(kThreads) attn_merge_kernel(const MergeArgs a) {
  constexpr int V = Elt<T>::kVec;
  const int64_t n = a.rows * a.heads * a.vecs;
  pdl_wait();
  pdl_trigger();
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
    const int64_t sh = i / a.vecs;
    const int v = (int)(i - sh * a.vecs);
    const int64_t s = sh / a.heads, h = sh - s * a.heads;
    const float la = __ldg(a.la + h * a.la_h + s * a.la_s), lb = __ldg(a.lb + h * a.lb_h + s * a.lb_s);
    const float m = fmaxf(la, lb);
    float wa = 0.f, wb = 0.f;
    if (m != -INFINITY) {  // both key sets empty (-inf, -inf): the output is zero
      wa = expf(la - m);
      wb = expf(lb - m);
    }
    const float inv = m != -INFINITY ? 1.f / (wa + wb) : 0.f;
    wa *= inv;
    wb *= inv;
    float fa[V], fb[V];
    Elt<T>::unpack(ld_stream(reinterpret_cast<const T*>(a.oa) + s * a.as_s + h * a.as_h + v * V), fa);
    Elt<T>::unpack(ld_stream(reinterpret_cast<const T*>(a.ob) + s * a.bs_s + h * a.bs_h + v * V), fb);
#pragma unroll
    for (int e = 0; e < V; ++e) fa[e] = fmaf(wa, fa[e], wb * fb[e]);
    st_global(reinterpret_cast<T*>(a.out) + s * a.os_s + h * a.os_h + v * V, Elt<T>::pack(fa));
  }
}

}  // namespace
}  // namespace jo

using namespace jo;

extern "C" {

int jo_attn_merge(void* out, int64_t out_stride_s, int64_t out_stride_h, const void* o_a, int64_t a_stride_s,
                  int64_t a_stride_h, const float* lse_a, int64_t lse_a_stride_h, int64_t lse_a_stride_s,
                  const void* o_b, int64_t b_stride_s, int64_t b_stride_h, const float* lse_b,
                  int64_t lse_b_stride_h, int64_t lse_b_stride_s, int64_t rows, int64_t heads, int64_t head_dim,
                  int dtype, void* stream) {
  const char* op = "attn_merge";
  const DeviceInfo* di;
  if (int s = device_info(&di)) return s;
  if (rows < 0 || heads <= 0 || head_dim <= 0) return fail(JO_ERR_SHAPE, "%s: bad sizes", op);
  if (rows == 0) return JO_OK;
  if (dtype != JO_BF16 && dtype != JO_F16) return fail(JO_ERR_DTYPE, "%s: outputs must be bf16 or fp16", op);
  if (head_dim % 8) return fail(JO_ERR_SHAPE, "%s: head_dim must be a multiple of 8", op);
  if (!out || !o_a || !o_b || !lse_a || !lse_b) return fail(JO_ERR_INVALID, "%s: null operand", op);
  if (!aligned16(out) || !aligned16(o_a) || !aligned16(o_b))
    return fail(JO_ERR_ALIGN, "%s: outputs must be 16-byte aligned", op);
  const int64_t strides[] = {out_stride_s, out_stride_h, a_stride_s, a_stride_h, b_stride_s, b_stride_h};
  for (int64_t s : strides)
    if (s % 8) return fail(JO_ERR_ALIGN, "%s: row / head strides must be multiples of 8 elements", op);
  MergeArgs a{out, out_stride_s, out_stride_h, o_a, a_stride_s, a_stride_h, o_b, b_stride_s, b_stride_h,
              lse_a, lse_a_stride_h, lse_a_stride_s, lse_b, lse_b_stride_h, lse_b_stride_s, rows, heads,
              (int)(head_dim / 8)};
  const int64_t n = rows * heads * a.vecs;
  cudaStream_t st = (cudaStream_t)stream;
  auto launch = [&](auto kern) -> int {
    const int64_t cap = (int64_t)di->sm_count * occupancy((const void*)kern, kThreads, 0);
    const int64_t need = cdiv(n, kThreads);
    const int64_t grid = need < cap ? need : cap;
    if (cudaError_t e = launch_pdl(kern, dim3((unsigned)grid), dim3(kThreads), 0, st, a))
      return launch_failed(e, op);
    return after_launch("attn_merge_kernel");
  };
  return dtype == JO_BF16 ? launch(attn_merge_kernel<__nv_bfloat16>) : launch(attn_merge_kernel<__half>);
}

}  // extern "C"
