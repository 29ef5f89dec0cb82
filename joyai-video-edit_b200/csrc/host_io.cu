// Host-buffer entry points: the q/k/v pack from and to pinned host memory,
// pipelined by token chunks so that both directions of the host link and the
// kernel overlap.
//
//   h2d stream:   [in 0][in 1][in 2] ...
//   stream:             [pack 0][pack 1] ...
//   d2h stream:                 [out 0][out 1] ...
//
// The bytes that cross the host link are fixed by the op (the qkv rows in, q/k/v
// out), so a serial upload -> kernel -> download takes the sum of the two copy
// times; overlapping the directions brings a call close to the slower direction
// alone plus one chunk of each.  One cudaMemcpyAsync per chunk for the input
// rows and one (2-D for head-major outputs) per output tensor per chunk.
#include <vector>

#include "common.cuh"

namespace jo {
namespace {

struct EventSet {
  std::vector<cudaEvent_t> ev;
  ~EventSet() {
    for (cudaEvent_t e : ev) cudaEventDestroy(e);  // released once the event has completed
  }
  cudaError_t make(size_t n) {
    ev.reserve(n);
    for (size_t i = 0; i < n; ++i) {
      cudaEvent_t e;
      const cudaError_t r = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
      if (r != cudaSuccess) return r;
      ev.push_back(e);
    }
    return cudaSuccess;
  }
};

}  // namespace
}  // namespace jo

using namespace jo;

extern "C" {

int jo_qkv_norm_rope_pack_host(void* host_q, void* host_k, void* host_v, int64_t out_stride_h, int64_t out_stride_t,
                               const void* host_qkv, void* dev_q, void* dev_k, void* dev_v, void* dev_qkv,
                               int64_t tokens, int64_t heads, int64_t head_dim, const void* q_weight,
                               const void* k_weight, const void* cos, const void* sin, float eps,
                               int64_t chunk_tokens, void* stream, void* h2d_stream, void* d2h_stream) {
  const char* op = "qkv_norm_rope_pack_host";
  const DeviceInfo* di;
  if (int s = device_info(&di)) return s;
  if (tokens < 0 || heads <= 0 || head_dim <= 0 || chunk_tokens <= 0)
    return fail(JO_ERR_SHAPE, "%s: bad tokens/heads/head_dim/chunk_tokens", op);
  if (tokens == 0) return JO_OK;
  if (!host_q || !host_k || !host_v || !host_qkv || !dev_q || !dev_k || !dev_v || !dev_qkv)
    return fail(JO_ERR_INVALID, "%s: null buffer", op);
  if (!h2d_stream || !d2h_stream)
    return fail(JO_ERR_INVALID, "%s: the two copy streams must be given (cudaStream_t, not the legacy stream)", op);
  const int64_t row = 3 * heads * head_dim;  // qkv row, elements (rows are contiguous)
  const bool head_major = out_stride_t == head_dim && out_stride_h == tokens * head_dim;
  const bool token_major = out_stride_h == head_dim && out_stride_t == heads * head_dim;
  if (!head_major && !token_major)
    return fail(JO_ERR_SHAPE, "%s: outputs must be head-major [heads, tokens, D] or token-major [tokens, heads, D]",
                op);
  cudaStream_t st = (cudaStream_t)stream, in = (cudaStream_t)h2d_stream, out = (cudaStream_t)d2h_stream;
  const int64_t n_chunks = cdiv(tokens, chunk_tokens);
  EventSet evs;
  if (cudaError_t e = evs.make((size_t)(2 * n_chunks + 2)))
    return fail(JO_ERR_CUDA, "%s: cudaEventCreate: %s", op, cudaGetErrorString(e));
  cudaEvent_t* ev_in = evs.ev.data();               // chunk c uploaded
  cudaEvent_t* ev_out = ev_in + n_chunks;           // chunk c packed
  cudaEvent_t ev_start = ev_in[2 * n_chunks], ev_done = ev_in[2 * n_chunks + 1];
  auto cuda = [&](cudaError_t e, const char* what) -> int {
    if (e == cudaSuccess) return JO_OK;
    cudaGetLastError();
    return fail(JO_ERR_CUDA, "%s: %s: %s", op, what, cudaGetErrorString(e));
  };
  // the copy streams start after everything already queued on `stream` (the
  // previous call's readers of the staging buffers included)
  if (int s = cuda(cudaEventRecord(ev_start, st), "event record")) return s;
  if (int s = cuda(cudaStreamWaitEvent(in, ev_start, 0), "stream wait")) return s;
  if (int s = cuda(cudaStreamWaitEvent(out, ev_start, 0), "stream wait")) return s;
  const auto* hq = static_cast<const uint8_t*>(host_qkv);
  auto* dq = static_cast<uint8_t*>(dev_qkv);
  uint8_t* hosts[3] = {static_cast<uint8_t*>(host_q), static_cast<uint8_t*>(host_k), static_cast<uint8_t*>(host_v)};
  uint8_t* devs[3] = {static_cast<uint8_t*>(dev_q), static_cast<uint8_t*>(dev_k), static_cast<uint8_t*>(dev_v)};
  const auto* cs = static_cast<const uint8_t*>(cos);
  const auto* sn = static_cast<const uint8_t*>(sin);
  for (int64_t c = 0; c < n_chunks; ++c) {
    const int64_t t0 = c * chunk_tokens;
    const int64_t nc = (t0 + chunk_tokens < tokens ? chunk_tokens : tokens - t0);
    const size_t in_off = (size_t)(t0 * row) * 2, in_bytes = (size_t)(nc * row) * 2;
    if (int s = cuda(cudaMemcpyAsync(dq + in_off, hq + in_off, in_bytes, cudaMemcpyHostToDevice, in), "upload"))
      return s;
    if (int s = cuda(cudaEventRecord(ev_in[c], in), "event record")) return s;
    if (int s = cuda(cudaStreamWaitEvent(st, ev_in[c], 0), "stream wait")) return s;
    const size_t o_off = (size_t)(t0 * out_stride_t) * 2;
    const size_t r_off = (size_t)(t0 * (head_dim / 2)) * 2;
    if (int s = jo_qkv_norm_rope_pack(devs[0] + o_off, devs[1] + o_off, devs[2] + o_off, nullptr, out_stride_h,
                                      out_stride_t, dq + in_off, row, nc, heads, head_dim, q_weight, k_weight,
                                      cos ? cs + r_off : nullptr, sin ? sn + r_off : nullptr, eps, st))
      return s;
    if (int s = cuda(cudaEventRecord(ev_out[c], st), "event record")) return s;
    if (int s = cuda(cudaStreamWaitEvent(out, ev_out[c], 0), "stream wait")) return s;
    for (int p = 0; p < 3; ++p) {
      cudaError_t e;
      if (token_major)  // the chunk's rows are one contiguous run
        e = cudaMemcpyAsync(hosts[p] + o_off, devs[p] + o_off, (size_t)(nc * heads * head_dim) * 2,
                            cudaMemcpyDeviceToHost, out);
      else  // one run of nc*D elements per head, heads runs tokens*D apart
        e = cudaMemcpy2DAsync(hosts[p] + o_off, (size_t)out_stride_h * 2, devs[p] + o_off, (size_t)out_stride_h * 2,
                              (size_t)(nc * head_dim) * 2, (size_t)heads, cudaMemcpyDeviceToHost, out);
      if (int s = cuda(e, "download")) return s;
    }
  }
  // `stream` resumes once every download has finished: the caller synchronises
  // on `stream` alone, and later work on it may reuse the staging buffers
  if (int s = cuda(cudaEventRecord(ev_done, out), "event record")) return s;
  return cuda(cudaStreamWaitEvent(st, ev_done, 0), "stream wait");
}

}  // extern "C"
