// torch.ops.joyomni_ops.* registration over the C ABI (include/joyomni_b200.h).
//
// The seven reference schemas are kept verbatim (joyomni_ops/csrc/pybind.cpp:52-75)
// so deploy/xvideo's call sites and torch.compile graphs bind unchanged; the
// argument checks mirror the reference entry points so the same inputs raise
// the same RuntimeErrors.  Every op validates, allocates its outputs from the
// caching allocator, and calls one jo_* entry point on the current stream.
// A non-zero status becomes a RuntimeError carrying jo_last_error().
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/all.h>
#include <torch/library.h>

#include "joyomni_b200.h"

namespace {

#define JO_CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define JO_CHECK_CONTIGUOUS(x) TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")
#define JO_CHECK_DTYPE(x, dt) \
  TORCH_CHECK((x).scalar_type() == (dt), #x " dtype is ", (x).scalar_type(), ", expected ", (dt))
#define JO_CHECK_INPUT(x, dt) \
  JO_CHECK_CUDA(x);           \
  JO_CHECK_CONTIGUOUS(x);     \
  JO_CHECK_DTYPE(x, dt)

void jo_check(int status, const char* op) {
  // An unsupported device raises NotImplementedError, as the reference's GEMM does on an
  // architecture it has no kernel for (fp8_gemm.cu:1531); every other failure is a RuntimeError.
  TORCH_CHECK_NOT_IMPLEMENTED(status != JO_ERR_UNSUPPORTED, "joyomni_ops::", op, ": ", jo_last_error());
  TORCH_CHECK(status == JO_OK, "joyomni_ops::", op, " failed (", jo_status_name(status), "): ",
              jo_last_error());
}

int dt_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return JO_F32;
    case at::kHalf: return JO_F16;
    case at::kBFloat16: return JO_BF16;
    case at::kFloat8_e4m3fn: return JO_E4M3;
    default: TORCH_CHECK(false, "Unsupported dtype ", t);
  }
}

void* stream_of(const torch::Tensor& t) {
  return (void*)at::cuda::getCurrentCUDAStream(t.get_device()).stream();
}

const void* opt_ptr(const c10::optional<torch::Tensor>& t) {
  return (t.has_value() && t->defined()) ? t->data_ptr() : nullptr;
}

jo_view4 view4(const torch::Tensor& t) {
  return jo_view4{t.data_ptr(), t.size(1), t.stride(1), t.stride(2)};
}
jo_view4 no_view() { return jo_view4{nullptr, 0, 0, 0}; }

// Every tensor operand must be a CUDA tensor on the op's device (the device of
// `anchor`): a host pointer or another device's pointer handed to a kernel would
// fault the GPU instead of raising here.
void check_dev(const torch::Tensor& t, const torch::Tensor& anchor, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.device() == anchor.device(), name, " is on ", t.device(), " but the op runs on ", anchor.device());
}
void check_dev(const c10::optional<torch::Tensor>& t, const torch::Tensor& anchor, const char* name) {
  if (t.has_value() && t->defined()) check_dev(*t, anchor, name);
}

// ------------------------------------------------------------------ drop-in ops

// joyomni_ops/csrc/rmsnorm.cu:107-126
torch::Tensor rmsnorm(const torch::Tensor& x, const torch::Tensor& weight, double eps) {
  JO_CHECK_CUDA(x);
  JO_CHECK_CUDA(weight);
  check_dev(weight, x, "weight");
  TORCH_CHECK(x.dim() == 2, "x must be 2D [M, N]");
  TORCH_CHECK(x.stride(-1) == 1, "x last dim must be contiguous");
  TORCH_CHECK(weight.dim() == 1 && weight.numel() == x.size(1), "weight must be 1D [N]");
  TORCH_CHECK(x.dtype() == weight.dtype(), "x and weight dtype must match");
  TORCH_CHECK(weight.is_contiguous(), "weight must be contiguous");
  const c10::cuda::CUDAGuard guard(x.device());
  auto out = torch::empty({x.size(0), x.size(1)}, x.options());
  jo_check(jo_rmsnorm(out.data_ptr(), out.stride(0), x.data_ptr(), x.stride(0), weight.data_ptr(),
                      x.size(0), x.size(1), dt_code(x.scalar_type()), (float)eps, stream_of(x)),
           "rmsnorm");
  return out;
}

void check_mod(const torch::Tensor& x, const torch::Tensor& scale, const torch::Tensor& shift) {
  const int64_t M = x.size(0), N = x.size(1);
  check_dev(scale, x, "scale");
  check_dev(shift, x, "shift");
  TORCH_CHECK(scale.dim() == 2 && shift.dim() == 2, "scale/shift must be 2D [M, N] or [1, N]");
  TORCH_CHECK(scale.size(0) == shift.size(0), "scale/shift row counts must match");
  TORCH_CHECK(scale.size(0) == 1 || scale.size(0) == M,
              "scale/shift rows must be 1 (broadcast) or M (per-row modulation)");
  TORCH_CHECK(scale.size(1) == N && shift.size(1) == N, "scale/shift last dim must be N");
  TORCH_CHECK(scale.stride(-1) == 1 && shift.stride(-1) == 1, "scale/shift last dim must be contiguous");
  TORCH_CHECK(scale.size(0) == 1 || scale.stride(0) == shift.stride(0),
              "scale/shift must share a row stride");
  TORCH_CHECK(x.dtype() == scale.dtype() && x.dtype() == shift.dtype(), "x/scale/shift dtype must match");
}

void check_affine(const torch::Tensor& x, const c10::optional<torch::Tensor>& gamma,
                  const c10::optional<torch::Tensor>& beta) {
  const int64_t N = x.size(1);
  check_dev(gamma, x, "gamma");
  check_dev(beta, x, "beta");
  if (gamma.has_value() && gamma->defined()) {
    TORCH_CHECK(gamma->numel() == N, "gamma must be length N");
    TORCH_CHECK(gamma->is_contiguous() && gamma->dtype() == x.dtype(), "gamma must be contiguous with x's dtype");
  }
  if (beta.has_value() && beta->defined()) {
    TORCH_CHECK(beta->numel() == N, "beta must be length N");
    TORCH_CHECK(beta->is_contiguous() && beta->dtype() == x.dtype(), "beta must be contiguous with x's dtype");
  }
}

// joyomni_ops/csrc/fused_norm_scale_shift.cu:364-403
torch::Tensor fused_norm_scale_shift(const torch::Tensor& x, const c10::optional<torch::Tensor>& gamma_opt,
                                     const c10::optional<torch::Tensor>& beta_opt,
                                     const torch::Tensor& scale, const torch::Tensor& shift,
                                     int64_t norm_type, double eps) {
  JO_CHECK_CUDA(x);
  JO_CHECK_CUDA(scale);
  JO_CHECK_CUDA(shift);
  TORCH_CHECK(x.dim() == 2, "x must be 2D [M, N]");
  TORCH_CHECK(x.stride(-1) == 1, "x last dim must be contiguous");
  TORCH_CHECK((x.size(1) % 4) == 0, "N must be divisible by 4");
  check_mod(x, scale, shift);
  TORCH_CHECK(norm_type == 0 || norm_type == 1, "norm_type must be 0 (layer) or 1 (rms)");
  check_affine(x, gamma_opt, beta_opt);
  const c10::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty({x.size(0), x.size(1)}, x.options());
  jo_check(jo_norm_scale_shift(y.data_ptr(), y.stride(0), x.data_ptr(), x.stride(0), opt_ptr(gamma_opt),
                               opt_ptr(beta_opt), scale.data_ptr(), shift.data_ptr(), scale.size(0),
                               scale.stride(0), x.size(0), x.size(1), (int)norm_type,
                               dt_code(x.scalar_type()), (float)eps, stream_of(x)),
           "fused_norm_scale_shift");
  return y;
}

// joyomni_ops/csrc/fused_qknorm_rope_3d_kernel.cu:280-319
void fused_qk_norm_rope_3d_paired(torch::Tensor& q, torch::Tensor& k, int64_t seq_len, int64_t num_heads,
                                  double eps, torch::Tensor& q_weight, torch::Tensor& k_weight,
                                  torch::Tensor& cos, torch::Tensor& sin,
                                  const c10::optional<torch::Tensor>& k_pre_rope_opt) {
  TORCH_CHECK(q.dim() == 3, "q must be 3D [batch, seq_len*num_heads, head_dim]");
  TORCH_CHECK(k.dim() == 3, "k must be 3D [batch, seq_len*num_heads, head_dim]");
  TORCH_CHECK(q.sizes() == k.sizes(), "q and k must have the same shape");
  TORCH_CHECK(q_weight.dim() == 1 && k_weight.dim() == 1, "weights must be 1D [head_dim]");
  TORCH_CHECK(cos.dim() == 2 && sin.dim() == 2, "cos/sin must be 2D [seq_len, head_dim/2]");
  JO_CHECK_INPUT(q, torch::kBFloat16);
  JO_CHECK_INPUT(k, torch::kBFloat16);
  JO_CHECK_INPUT(q_weight, torch::kBFloat16);
  JO_CHECK_INPUT(k_weight, torch::kBFloat16);
  JO_CHECK_INPUT(cos, torch::kBFloat16);
  JO_CHECK_INPUT(sin, torch::kBFloat16);
  check_dev(k, q, "k");
  check_dev(q_weight, q, "q_weight");
  check_dev(k_weight, q, "k_weight");
  check_dev(cos, q, "cos");
  check_dev(sin, q, "sin");
  check_dev(k_pre_rope_opt, q, "k_pre_rope");
  const int64_t batch = q.size(0), head_dim = q.size(2);
  TORCH_CHECK(q.size(1) == seq_len * num_heads, "q.size(1) must equal seq_len*num_heads");
  TORCH_CHECK(q_weight.size(0) == head_dim && k_weight.size(0) == head_dim, "weight size must match head_dim");
  TORCH_CHECK(cos.size(0) == seq_len && cos.size(1) == head_dim / 2, "cos shape must be [seq_len, head_dim/2]");
  TORCH_CHECK(sin.size(0) == seq_len && sin.size(1) == head_dim / 2, "sin shape must be [seq_len, head_dim/2]");
  TORCH_CHECK(head_dim == 64 || head_dim == 128 || head_dim == 256,
              "Unsupported head_dim for fused_qk_norm_rope_3d_paired: ", head_dim);
  void* k_pre = nullptr;
  if (k_pre_rope_opt.has_value() && k_pre_rope_opt->defined()) {
    const auto& cache = k_pre_rope_opt.value();
    TORCH_CHECK(cache.sizes() == k.sizes(), "k_pre_rope must have the same shape as k");
    JO_CHECK_INPUT(cache, torch::kBFloat16);
    k_pre = cache.data_ptr();
  }
  const c10::cuda::CUDAGuard guard(q.device());
  jo_check(jo_qk_norm_rope_3d_paired(q.data_ptr(), k.data_ptr(), batch, seq_len, num_heads, head_dim,
                                     (float)eps, q_weight.data_ptr(), k_weight.data_ptr(), cos.data_ptr(),
                                     sin.data_ptr(), k_pre, stream_of(q)),
           "fused_qk_norm_rope_3d_paired");
}

void check_qkv_tensor(const torch::Tensor& t, const char* name, int64_t batch, int64_t heads,
                      int64_t head_dim) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == torch::kBFloat16, name, " must be bfloat16");
  TORCH_CHECK(t.dim() == 4, name, " must be [B,L,H,D]");
  TORCH_CHECK(t.size(0) == batch && t.size(2) == heads && t.size(3) == head_dim, name,
              " has incompatible shape ", t.sizes());
  TORCH_CHECK(t.stride(3) == 1, name, " last dimension must be contiguous");
}

// joyomni_ops/csrc/fused_joint_qkv_pack.cu:237-342
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> fused_joint_qkv_pack(
    const torch::Tensor& img_q, const torch::Tensor& img_k, const torch::Tensor& img_v,
    const torch::Tensor& txt_q, const torch::Tensor& txt_k, const torch::Tensor& txt_v,
    const c10::optional<torch::Tensor>& cached_k_opt, const c10::optional<torch::Tensor>& cached_v_opt,
    const torch::Tensor& txt_q_weight, const torch::Tensor& txt_k_weight, double eps) {
  TORCH_CHECK(img_q.dim() == 4, "img_q must be [B,L,H,D]");
  const int64_t batch = img_q.size(0), img_len = img_q.size(1), heads = img_q.size(2),
                head_dim = img_q.size(3);
  TORCH_CHECK(batch == 1, "fused_joint_qkv_pack fast path requires batch=1");
  TORCH_CHECK(head_dim == 128, "fused_joint_qkv_pack requires head_dim=128");
  TORCH_CHECK(img_len > 0 && heads > 0, "image length and heads must be positive");
  check_qkv_tensor(img_q, "img_q", batch, heads, head_dim);
  check_qkv_tensor(img_k, "img_k", batch, heads, head_dim);
  check_qkv_tensor(img_v, "img_v", batch, heads, head_dim);
  TORCH_CHECK(img_k.size(1) == img_len && img_v.size(1) == img_len, "image Q/K/V lengths must match");
  const int64_t txt_len = txt_q.size(1);
  check_qkv_tensor(txt_q, "txt_q", batch, heads, head_dim);
  check_qkv_tensor(txt_k, "txt_k", batch, heads, head_dim);
  check_qkv_tensor(txt_v, "txt_v", batch, heads, head_dim);
  TORCH_CHECK(txt_len > 0 && txt_k.size(1) == txt_len && txt_v.size(1) == txt_len,
              "text Q/K/V lengths must match and be positive");
  JO_CHECK_INPUT(txt_q_weight, torch::kBFloat16);
  JO_CHECK_INPUT(txt_k_weight, torch::kBFloat16);
  check_dev(img_k, img_q, "img_k");
  check_dev(img_v, img_q, "img_v");
  check_dev(txt_q, img_q, "txt_q");
  check_dev(txt_k, img_q, "txt_k");
  check_dev(txt_v, img_q, "txt_v");
  check_dev(cached_k_opt, img_q, "cached_k");
  check_dev(cached_v_opt, img_q, "cached_v");
  check_dev(txt_q_weight, img_q, "txt_q_weight");
  check_dev(txt_k_weight, img_q, "txt_k_weight");
  TORCH_CHECK(txt_q_weight.dim() == 1 && txt_q_weight.numel() == head_dim, "txt_q_weight must be [head_dim]");
  TORCH_CHECK(txt_k_weight.dim() == 1 && txt_k_weight.numel() == head_dim, "txt_k_weight must be [head_dim]");
  TORCH_CHECK(cached_k_opt.has_value() == cached_v_opt.has_value(),
              "cached_k and cached_v must either both be present or both be absent");
  int64_t cache_len = 0;
  jo_view4 ck = no_view(), cv = no_view();
  if (cached_k_opt.has_value()) {
    check_qkv_tensor(*cached_k_opt, "cached_k", batch, heads, head_dim);
    check_qkv_tensor(*cached_v_opt, "cached_v", batch, heads, head_dim);
    cache_len = cached_k_opt->size(1);
    TORCH_CHECK(cached_v_opt->size(1) == cache_len, "cached K/V lengths must match");
    if (cache_len > 0) {
      ck = view4(*cached_k_opt);
      cv = view4(*cached_v_opt);
    }
  }
  const c10::cuda::CUDAGuard guard(img_q.device());
  const auto options = img_q.options();
  auto out_q = torch::empty({batch, img_len + txt_len, heads, head_dim}, options);
  auto out_k = torch::empty({batch, cache_len + img_len + txt_len, heads, head_dim}, options);
  auto out_v = torch::empty_like(out_k);
  jo_check(jo_joint_qkv_pack(out_q.data_ptr(), out_k.data_ptr(), out_v.data_ptr(), view4(img_q), view4(img_k),
                             view4(img_v), view4(txt_q), view4(txt_k), view4(txt_v), ck, cv,
                             txt_q_weight.data_ptr(), txt_k_weight.data_ptr(), heads, (float)eps,
                             stream_of(img_q)),
           "fused_joint_qkv_pack");
  return std::make_tuple(out_q, out_k, out_v);
}

// joyomni_ops/csrc/fused_joint_qkv_pack.cu:344-415
std::tuple<torch::Tensor, torch::Tensor> fused_cached_kv_pack(const torch::Tensor& key0,
                                                              const torch::Tensor& value0,
                                                              const c10::optional<torch::Tensor>& key1_opt,
                                                              const c10::optional<torch::Tensor>& value1_opt,
                                                              const torch::Tensor& cos, const torch::Tensor& sin) {
  TORCH_CHECK(key0.dim() == 4, "key0 must be [B,L,H,D]");
  const int64_t batch = key0.size(0), len0 = key0.size(1), heads = key0.size(2), head_dim = key0.size(3);
  TORCH_CHECK(batch == 1, "fused_cached_kv_pack requires batch=1");
  TORCH_CHECK(head_dim == 128, "fused_cached_kv_pack requires head_dim=128");
  TORCH_CHECK(len0 > 0 && heads > 0, "cache length and heads must be positive");
  check_qkv_tensor(key0, "key0", batch, heads, head_dim);
  check_qkv_tensor(value0, "value0", batch, heads, head_dim);
  TORCH_CHECK(value0.size(1) == len0, "key0/value0 lengths must match");
  TORCH_CHECK(key1_opt.has_value() == value1_opt.has_value(),
              "key1 and value1 must either both be present or both be absent");
  int64_t len1 = 0;
  jo_view4 k1 = no_view(), v1 = no_view();
  if (key1_opt.has_value()) {
    check_qkv_tensor(*key1_opt, "key1", batch, heads, head_dim);
    check_qkv_tensor(*value1_opt, "value1", batch, heads, head_dim);
    len1 = key1_opt->size(1);
    TORCH_CHECK(len1 > 0 && value1_opt->size(1) == len1, "key1/value1 lengths must match and be positive");
    k1 = view4(*key1_opt);
    v1 = view4(*value1_opt);
  }
  JO_CHECK_INPUT(cos, torch::kFloat32);
  JO_CHECK_INPUT(sin, torch::kFloat32);
  check_dev(value0, key0, "value0");
  check_dev(key1_opt, key0, "key1");
  check_dev(value1_opt, key0, "value1");
  check_dev(cos, key0, "cos");
  check_dev(sin, key0, "sin");
  TORCH_CHECK(cos.sizes() == sin.sizes(), "cos/sin shapes must match");
  TORCH_CHECK(cos.numel() == (len0 + len1) * head_dim, "cos/sin must contain [total_cache_len, head_dim], got ",
              cos.sizes());
  const c10::cuda::CUDAGuard guard(key0.device());
  auto out_key = torch::empty({batch, len0 + len1, heads, head_dim}, key0.options());
  auto out_value = torch::empty_like(out_key);
  jo_check(jo_cached_kv_pack(out_key.data_ptr(), out_value.data_ptr(), view4(key0), view4(value0), k1, v1,
                             cos.data_ptr<float>(), sin.data_ptr<float>(), heads, stream_of(key0)),
           "fused_cached_kv_pack");
  return std::make_tuple(out_key, out_value);
}

// Rotation of pre-RoPE cached keys [L, H, 128] (any row / head strides) into a
// contiguous [L, H, 128] buffer with fp32 full-width tables [L, 128]: the keys of
// fused_cached_kv_pack (fused_joint_qkv_pack.cu:166-220) without the value copy.
void cached_k_rotate_into(const torch::Tensor& key, const torch::Tensor& cos, const torch::Tensor& sin,
                          torch::Tensor& out_key) {
  JO_CHECK_CUDA(key);
  check_dev(cos, key, "cos");
  check_dev(sin, key, "sin");
  check_dev(out_key, key, "out_key");
  TORCH_CHECK(key.dim() == 3 && key.size(2) == 128 && key.stride(2) == 1, "key must be [L, H, 128]");
  JO_CHECK_DTYPE(key, torch::kBFloat16);
  JO_CHECK_INPUT(out_key, torch::kBFloat16);
  TORCH_CHECK(out_key.sizes() == key.sizes(), "out_key must have key's shape");
  JO_CHECK_INPUT(cos, torch::kFloat32);
  JO_CHECK_INPUT(sin, torch::kFloat32);
  TORCH_CHECK(cos.numel() == key.size(0) * 128 && sin.sizes() == cos.sizes(), "cos/sin must be [L, 128]");
  const c10::cuda::CUDAGuard guard(key.device());
  jo_view4 k0{key.data_ptr(), key.size(0), key.stride(0), key.stride(1)};
  jo_check(jo_cached_kv_pack(out_key.data_ptr(), nullptr, k0, no_view(), no_view(), no_view(), cos.data_ptr<float>(),
                             sin.data_ptr<float>(), key.size(1), stream_of(key)),
           "cached_k_rotate_into");
}

// joyomni_ops/csrc/per_token_quant_fp8.cu:148-176
void sgl_per_token_quant_fp8(torch::Tensor input, torch::Tensor output_q, torch::Tensor output_s) {
  JO_CHECK_CUDA(input);
  JO_CHECK_CONTIGUOUS(input);
  JO_CHECK_CUDA(output_q);
  JO_CHECK_CUDA(output_s);
  check_dev(output_q, input, "output_q");
  check_dev(output_s, input, "output_s");
  TORCH_CHECK(input.dim() == 2, "input must be 2D [num_tokens, hidden_dim]");
  const int64_t num_tokens = input.size(0), hidden_dim = input.size(1);
  TORCH_CHECK(hidden_dim % 4 == 0, "hidden_dim must be divisible by 4, got ", hidden_dim);
  TORCH_CHECK(input.scalar_type() == torch::kBFloat16 || input.scalar_type() == torch::kHalf,
              "per_token_quant_fp8: input must be bf16 or fp16");
  JO_CHECK_CONTIGUOUS(output_q);
  JO_CHECK_DTYPE(output_q, torch::kFloat8_e4m3fn);
  TORCH_CHECK(output_q.numel() == input.numel(), "output_q must have the input's shape");
  JO_CHECK_CONTIGUOUS(output_s);
  JO_CHECK_DTYPE(output_s, torch::kFloat32);
  TORCH_CHECK(output_s.numel() == num_tokens, "output_s must hold one scale per token");
  const c10::cuda::CUDAGuard guard(input.device());
  jo_check(jo_per_token_quant_fp8(output_q.data_ptr(), hidden_dim, output_s.data_ptr<float>(), input.data_ptr(),
                                  hidden_dim, num_tokens, hidden_dim, dt_code(input.scalar_type()),
                                  stream_of(input)),
           "sgl_per_token_quant_fp8");
}

// joyomni_ops/csrc/fp8_gemm.cu:1450-1546
torch::Tensor fp8_scaled_mm(const torch::Tensor& mat_a, const torch::Tensor& mat_b, const torch::Tensor& scales_a,
                            const torch::Tensor& scales_b, const torch::ScalarType& out_dtype,
                            const c10::optional<torch::Tensor>& bias) {
  TORCH_CHECK(mat_a.is_cuda(), "mat_a must be a CUDA tensor");
  TORCH_CHECK(mat_b.is_cuda(), "mat_b must be a CUDA tensor");
  TORCH_CHECK(mat_a.dim() == 2, "mat_a must be a 2D tensor");
  TORCH_CHECK(mat_b.dim() == 2, "mat_b must be a 2D tensor");
  TORCH_CHECK(mat_a.stride(1) == 1, "mat_a must be a row major tensor");
  TORCH_CHECK(mat_b.stride(0) == 1, "mat_b must be a column major tensor");
  TORCH_CHECK(mat_a.size(1) == mat_b.size(0), "mat_a and mat_b shapes cannot be multiplied");
  TORCH_CHECK((mat_a.size(1) * mat_a.element_size()) % 16 == 0,
              "mat_a must be multiple of 16 bytes for memory alignment");
  TORCH_CHECK((mat_b.size(0) * mat_b.element_size()) % 16 == 0,
              "mat_b must be multiple of 16 bytes for memory alignment");
  TORCH_CHECK(mat_a.scalar_type() == torch::kFloat8_e4m3fn, "mat_a must be Float8_e4m3fn");
  TORCH_CHECK(mat_b.scalar_type() == torch::kFloat8_e4m3fn, "mat_b must be Float8_e4m3fn");
  TORCH_CHECK(out_dtype == torch::kHalf || out_dtype == torch::kBFloat16, "out_dtype must be Half or BFloat16");
  TORCH_CHECK(scales_a.numel() == mat_a.size(0), "size of scales_a is not matched");
  TORCH_CHECK(scales_b.numel() == mat_b.size(1), "size of scales_b is not matched");
  TORCH_CHECK(scales_a.is_contiguous(), "scales_a must be contiguous");
  TORCH_CHECK(scales_b.is_contiguous(), "scales_b msut be contiguous");
  TORCH_CHECK(scales_a.scalar_type() == torch::kFloat32, "scales_a must be Float32");
  TORCH_CHECK(scales_b.scalar_type() == torch::kFloat32, "scales_b must be Float32");
  check_dev(mat_b, mat_a, "mat_b");
  check_dev(scales_a, mat_a, "scales_a");
  check_dev(scales_b, mat_a, "scales_b");
  check_dev(bias, mat_a, "bias");
  if (bias) {
    TORCH_CHECK(bias->numel() == mat_b.size(1), "size of bias is not matched");
    TORCH_CHECK(bias->is_contiguous(), "bias must be contiguous");
    TORCH_CHECK(bias->dtype() == out_dtype, "bias dtype must match output dtype");
  }
  const c10::cuda::CUDAGuard guard(mat_a.device());
  torch::Tensor out = torch::empty({mat_a.size(0), mat_b.size(1)}, mat_a.options().dtype(out_dtype));
  TORCH_CHECK((out.size(1) * out.element_size()) % 16 == 0, "out must be multiple of 16 bytes for memory alignment");
  jo_check(jo_fp8_scaled_mm(out.data_ptr(), out.stride(0), mat_a.data_ptr(), mat_a.stride(0), mat_b.data_ptr(),
                            mat_b.stride(1), scales_a.data_ptr<float>(), scales_b.data_ptr<float>(),
                            bias ? bias->data_ptr() : nullptr, mat_a.size(0), mat_b.size(1), mat_a.size(1),
                            dt_code(out_dtype), stream_of(mat_a)),
           "fp8_scaled_mm");
  return out;
}

// ------------------------------------------------------------------ new fused ops
// Operand checks of the fused FP8 GEMMs (fp8_scaled_mm's contract, in fewer messages).
void check_fused_gemm_operands(const torch::Tensor& mat_a, const torch::Tensor& mat_b, const torch::Tensor& scales_a,
                               const torch::Tensor& scales_b, const torch::ScalarType& out_dtype,
                               const c10::optional<torch::Tensor>& bias) {
  TORCH_CHECK(mat_a.is_cuda() && mat_b.is_cuda(), "mat_a and mat_b must be CUDA tensors");
  TORCH_CHECK(mat_a.dim() == 2 && mat_b.dim() == 2, "mat_a and mat_b must be 2D tensors");
  TORCH_CHECK(mat_a.stride(1) == 1, "mat_a must be a row major tensor");
  TORCH_CHECK(mat_b.stride(0) == 1, "mat_b must be a column major tensor");
  TORCH_CHECK(mat_a.size(1) == mat_b.size(0), "mat_a and mat_b shapes cannot be multiplied");
  TORCH_CHECK(mat_a.scalar_type() == torch::kFloat8_e4m3fn && mat_b.scalar_type() == torch::kFloat8_e4m3fn,
              "mat_a and mat_b must be Float8_e4m3fn");
  TORCH_CHECK(out_dtype == torch::kHalf || out_dtype == torch::kBFloat16, "out_dtype must be Half or BFloat16");
  TORCH_CHECK(scales_a.numel() == mat_a.size(0) && scales_a.is_contiguous() &&
                  scales_a.scalar_type() == torch::kFloat32,
              "scales_a must be contiguous Float32 with one value per row of mat_a");
  TORCH_CHECK(scales_b.numel() == mat_b.size(1) && scales_b.is_contiguous() &&
                  scales_b.scalar_type() == torch::kFloat32,
              "scales_b must be contiguous Float32 with one value per column of mat_b");
  check_dev(mat_b, mat_a, "mat_b");
  check_dev(scales_a, mat_a, "scales_a");
  check_dev(scales_b, mat_a, "scales_b");
  check_dev(bias, mat_a, "bias");
  if (bias) {
    TORCH_CHECK(bias->numel() == mat_b.size(1) && bias->is_contiguous() && bias->dtype() == out_dtype,
                "bias must be contiguous [N] of the output dtype");
  }
}

// fp8_scaled_mm + torch.addcmul(residual, ., gate) in the GEMM epilogue (dit.py:536-538).
torch::Tensor fp8_scaled_mm_gated_residual(const torch::Tensor& mat_a, const torch::Tensor& mat_b,
                                           const torch::Tensor& scales_a, const torch::Tensor& scales_b,
                                           const torch::ScalarType& out_dtype, const c10::optional<torch::Tensor>& bias,
                                           const torch::Tensor& residual, const torch::Tensor& gate) {
  check_fused_gemm_operands(mat_a, mat_b, scales_a, scales_b, out_dtype, bias);
  check_dev(residual, mat_a, "residual");
  check_dev(gate, mat_a, "gate");
  const int64_t M = mat_a.size(0), N = mat_b.size(1);
  TORCH_CHECK(residual.is_cuda() && residual.dim() == 2 && residual.size(0) == M && residual.size(1) == N &&
                  residual.stride(1) == 1 && residual.scalar_type() == out_dtype,
              "residual must be [M, N] of the output dtype with contiguous rows");
  TORCH_CHECK(gate.is_cuda() && gate.numel() == N && gate.is_contiguous() && gate.scalar_type() == out_dtype,
              "gate must be contiguous [N] (or [1, N]) of the output dtype");
  const c10::cuda::CUDAGuard guard(mat_a.device());
  torch::Tensor out = torch::empty({M, N}, mat_a.options().dtype(out_dtype));
  jo_check(jo_fp8_scaled_mm_gated_residual(out.data_ptr(), out.stride(0), mat_a.data_ptr(), mat_a.stride(0),
                                           mat_b.data_ptr(), mat_b.stride(1), scales_a.data_ptr<float>(),
                                           scales_b.data_ptr<float>(), bias ? bias->data_ptr() : nullptr,
                                           residual.data_ptr(), residual.stride(0), gate.data_ptr(), M, N,
                                           mat_a.size(1), dt_code(out_dtype), stream_of(mat_a)),
           "fp8_scaled_mm_gated_residual");
  return out;
}

// fp8_scaled_mm -> GELU-tanh -> per-token FP8 (dit.py:508-513 with the next
// Fp8Linear's quantisation): (q [M, N] e4m3, s [M, 1] fp32); the GELU output is
// a workspace of out_dtype.
std::tuple<torch::Tensor, torch::Tensor> fp8_scaled_mm_gelu_quant(const torch::Tensor& mat_a,
                                                                  const torch::Tensor& mat_b,
                                                                  const torch::Tensor& scales_a,
                                                                  const torch::Tensor& scales_b,
                                                                  const torch::ScalarType& out_dtype,
                                                                  const c10::optional<torch::Tensor>& bias) {
  check_fused_gemm_operands(mat_a, mat_b, scales_a, scales_b, out_dtype, bias);
  const int64_t M = mat_a.size(0), N = mat_b.size(1);
  TORCH_CHECK(N > 0 || M == 0, "fp8_scaled_mm_gelu_quant: N must be positive");
  const c10::cuda::CUDAGuard guard(mat_a.device());
  torch::Tensor y = torch::empty({M, N}, mat_a.options().dtype(out_dtype));
  torch::Tensor amax = torch::empty({M}, mat_a.options().dtype(torch::kInt32));
  torch::Tensor q = torch::empty({M, N}, mat_a.options().dtype(torch::kFloat8_e4m3fn));
  torch::Tensor s = torch::empty({M, 1}, mat_a.options().dtype(torch::kFloat32));
  jo_check(jo_fp8_scaled_mm_gelu_quant(q.data_ptr(), q.stride(0), s.data_ptr<float>(), y.data_ptr(), y.stride(0),
                                       reinterpret_cast<uint32_t*>(amax.data_ptr<int32_t>()), mat_a.data_ptr(),
                                       mat_a.stride(0), mat_b.data_ptr(), mat_b.stride(1), scales_a.data_ptr<float>(),
                                       scales_b.data_ptr<float>(), bias ? bias->data_ptr() : nullptr, M, N,
                                       mat_a.size(1), dt_code(out_dtype), stream_of(mat_a)),
           "fp8_scaled_mm_gelu_quant");
  return {q, s};
}


torch::Tensor as_rows(const torch::Tensor& t, int64_t cols, const char* name) {
  TORCH_CHECK(t.size(-1) == cols, name, " last dim must be ", cols);
  TORCH_CHECK(t.stride(-1) == 1, name, " last dim must be contiguous");
  return t.reshape({-1, cols});
}

// gate given as [N], [1, N] or [M, N]
std::pair<int64_t, int64_t> gate_rows(const torch::Tensor& gate, int64_t M, int64_t N) {
  TORCH_CHECK(gate.size(-1) == N && gate.stride(-1) == 1, "gate last dim must be contiguous N");
  const int64_t gr = gate.numel() / N;
  TORCH_CHECK(gr == 1 || gr == M, "gate must hold 1 or M rows");
  if (gr == 1) return {1, 0};
  TORCH_CHECK(gate.dim() == 2, "a per-row gate must be 2D [M, N]");
  return {gr, gate.stride(0)};
}

// Shared checks of the qkv pack ops; returns (tokens, head_dim).
std::pair<int64_t, int64_t> check_qkv_pack(const torch::Tensor& qkv, int64_t num_heads, const torch::Tensor& q_weight,
                                           const torch::Tensor& k_weight, const c10::optional<torch::Tensor>& cos,
                                           const c10::optional<torch::Tensor>& sin) {
  JO_CHECK_CUDA(qkv);
  TORCH_CHECK(qkv.dim() == 2, "qkv must be 2D [tokens, 3*heads*head_dim]");
  TORCH_CHECK(qkv.stride(1) == 1, "qkv last dim must be contiguous");
  JO_CHECK_DTYPE(qkv, torch::kBFloat16);
  TORCH_CHECK(num_heads > 0 && qkv.size(1) % (3 * num_heads) == 0, "qkv width must be 3*num_heads*head_dim");
  const int64_t L = qkv.size(0), D = qkv.size(1) / (3 * num_heads);
  TORCH_CHECK(D == 64 || D == 128 || D == 256, "head_dim must be 64, 128 or 256, got ", D);
  JO_CHECK_INPUT(q_weight, torch::kBFloat16);
  JO_CHECK_INPUT(k_weight, torch::kBFloat16);
  check_dev(q_weight, qkv, "q_weight");
  check_dev(k_weight, qkv, "k_weight");
  check_dev(cos, qkv, "cos");
  check_dev(sin, qkv, "sin");
  TORCH_CHECK(q_weight.numel() == D && k_weight.numel() == D, "weight size must match head_dim");
  const bool hc = cos.has_value() && cos->defined(), hs = sin.has_value() && sin->defined();
  TORCH_CHECK(hc == hs, "cos and sin must both be given (RoPE) or both be None (text rows, no rotation)");
  if (hc) {
    JO_CHECK_INPUT(*cos, torch::kBFloat16);
    JO_CHECK_INPUT(*sin, torch::kBFloat16);
    TORCH_CHECK(cos->dim() == 2 && cos->size(0) == L && cos->size(1) == D / 2,
                "cos shape must be [tokens, head_dim/2]");
    TORCH_CHECK(sin->sizes() == cos->sizes(), "sin shape must match cos");
  }
  return {L, D};
}

std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> qkv_norm_rope_pack(
    const torch::Tensor& qkv, int64_t num_heads, const torch::Tensor& q_weight, const torch::Tensor& k_weight,
    const c10::optional<torch::Tensor>& cos, const c10::optional<torch::Tensor>& sin, double eps, bool head_major,
    const c10::optional<torch::Tensor>& k_pre_rope) {
  const auto [L, D] = check_qkv_pack(qkv, num_heads, q_weight, k_weight, cos, sin);
  const c10::cuda::CUDAGuard guard(qkv.device());
  auto shape = head_major ? std::vector<int64_t>{num_heads, L, D} : std::vector<int64_t>{L, num_heads, D};
  auto q = torch::empty(shape, qkv.options());
  auto k = torch::empty(shape, qkv.options());
  auto v = torch::empty(shape, qkv.options());
  void* pre = nullptr;
  if (k_pre_rope.has_value() && k_pre_rope->defined()) {
    JO_CHECK_INPUT(*k_pre_rope, torch::kBFloat16);
    check_dev(*k_pre_rope, qkv, "k_pre_rope");
    TORCH_CHECK(k_pre_rope->sizes() == k.sizes(), "k_pre_rope must have the output shape ", k.sizes());
    pre = k_pre_rope->data_ptr();
  }
  const int64_t sh = head_major ? L * D : D, st = head_major ? D : num_heads * D;
  jo_check(jo_qkv_norm_rope_pack(q.data_ptr(), k.data_ptr(), v.data_ptr(), pre, sh, st, qkv.data_ptr(), qkv.stride(0),
                                 L, num_heads, D, q_weight.data_ptr(), k_weight.data_ptr(), opt_ptr(cos),
                                 opt_ptr(sin), (float)eps, stream_of(qkv)),
           "qkv_norm_rope_pack");
  return std::make_tuple(q, k, v);
}

// Same op writing into caller-provided [tokens, heads, head_dim] views (any
// token/head strides, shared by q/k/v): e.g. slices of persistent Q and KV
// buffers, so no concatenation copy is needed before attention.
void qkv_norm_rope_pack_into(const torch::Tensor& qkv, int64_t num_heads, const torch::Tensor& q_weight,
                             const torch::Tensor& k_weight, const c10::optional<torch::Tensor>& cos,
                             const c10::optional<torch::Tensor>& sin, double eps, torch::Tensor& q_out,
                             torch::Tensor& k_out, torch::Tensor& v_out,
                             const c10::optional<torch::Tensor>& k_pre_out) {
  const auto [L, D] = check_qkv_pack(qkv, num_heads, q_weight, k_weight, cos, sin);
  void* pre = nullptr;
  if (k_pre_out.has_value() && k_pre_out->defined()) {
    const torch::Tensor& p = *k_pre_out;
    check_dev(p, qkv, "k_pre_out");
    JO_CHECK_DTYPE(p, torch::kBFloat16);
    TORCH_CHECK(p.dim() == 3 && p.size(0) == L && p.size(1) == num_heads && p.size(2) == D && p.stride(2) == 1 &&
                    p.stride(0) == q_out.stride(0) && p.stride(1) == q_out.stride(1),
                "k_pre_out must be a [tokens, heads, head_dim] view with the outputs' strides");
    pre = p.data_ptr();
  }
  for (const torch::Tensor* t : {&q_out, &k_out, &v_out}) {
    JO_CHECK_CUDA(*t);
    check_dev(*t, qkv, "q/k/v output");
    JO_CHECK_DTYPE(*t, torch::kBFloat16);
    TORCH_CHECK(t->dim() == 3 && t->size(0) == L && t->size(1) == num_heads && t->size(2) == D,
                "outputs must be [tokens, heads, head_dim] views, got ", t->sizes());
    TORCH_CHECK(t->stride(2) == 1 && t->stride(0) == q_out.stride(0) && t->stride(1) == q_out.stride(1),
                "q/k/v outputs must share token and head strides with a contiguous last dim");
  }
  const c10::cuda::CUDAGuard guard(qkv.device());
  jo_check(jo_qkv_norm_rope_pack(q_out.data_ptr(), k_out.data_ptr(), v_out.data_ptr(), pre, q_out.stride(1),
                                 q_out.stride(0), qkv.data_ptr(), qkv.stride(0), L, num_heads, D, q_weight.data_ptr(),
                                 k_weight.data_ptr(), opt_ptr(cos), opt_ptr(sin), (float)eps, stream_of(qkv)),
           "qkv_norm_rope_pack_into");
}

// qkv_norm_rope_pack from pinned host memory to pinned host memory: the upload of
// each token chunk, its pack and the download of its q/k/v overlap on three
// streams (the current stream and two from the pool).  Device staging buffers
// come from the caching allocator on the current stream; the call returns with
// every copy ordered before later work on the current stream.
void qkv_norm_rope_pack_host(const torch::Tensor& qkv_host, int64_t num_heads, const torch::Tensor& q_weight,
                             const torch::Tensor& k_weight, const c10::optional<torch::Tensor>& cos,
                             const c10::optional<torch::Tensor>& sin, double eps, bool head_major,
                             torch::Tensor& q_host, torch::Tensor& k_host, torch::Tensor& v_host,
                             int64_t chunk_tokens) {
  TORCH_CHECK(!qkv_host.is_cuda() && qkv_host.is_pinned(), "qkv_host must be a pinned host tensor");
  TORCH_CHECK(qkv_host.dim() == 2 && qkv_host.is_contiguous(), "qkv_host must be contiguous [tokens, 3*heads*head_dim]");
  JO_CHECK_DTYPE(qkv_host, torch::kBFloat16);
  TORCH_CHECK(num_heads > 0 && qkv_host.size(1) % (3 * num_heads) == 0, "qkv width must be 3*num_heads*head_dim");
  const int64_t L = qkv_host.size(0), D = qkv_host.size(1) / (3 * num_heads);
  JO_CHECK_INPUT(q_weight, torch::kBFloat16);
  JO_CHECK_INPUT(k_weight, torch::kBFloat16);
  check_dev(k_weight, q_weight, "k_weight");
  check_dev(cos, q_weight, "cos");
  check_dev(sin, q_weight, "sin");
  const bool hc = cos.has_value() && cos->defined(), hs = sin.has_value() && sin->defined();
  TORCH_CHECK(hc == hs, "cos and sin must both be given (RoPE) or both be None (text rows, no rotation)");
  if (hc) {
    JO_CHECK_INPUT(*cos, torch::kBFloat16);
    JO_CHECK_INPUT(*sin, torch::kBFloat16);
    TORCH_CHECK(cos->dim() == 2 && cos->size(0) == L && cos->size(1) == D / 2 && sin->sizes() == cos->sizes(),
                "cos/sin shape must be [tokens, head_dim/2]");
  }
  auto shape = head_major ? std::vector<int64_t>{num_heads, L, D} : std::vector<int64_t>{L, num_heads, D};
  for (const torch::Tensor* t : {&q_host, &k_host, &v_host}) {
    TORCH_CHECK(!t->is_cuda() && t->is_pinned() && t->is_contiguous(), "q/k/v_host must be contiguous pinned host tensors");
    JO_CHECK_DTYPE(*t, torch::kBFloat16);
    TORCH_CHECK(t->sizes() == shape, "q/k/v_host must be ", shape, ", got ", t->sizes());
  }
  TORCH_CHECK(chunk_tokens > 0, "chunk_tokens must be positive");
  const c10::cuda::CUDAGuard guard(q_weight.device());
  auto dev_qkv = torch::empty({L, qkv_host.size(1)}, q_weight.options());
  auto dq = torch::empty(shape, q_weight.options());
  auto dk = torch::empty(shape, q_weight.options());
  auto dv = torch::empty(shape, q_weight.options());
  auto in = c10::cuda::getStreamFromPool(false, q_weight.get_device());
  auto out = c10::cuda::getStreamFromPool(false, q_weight.get_device());
  const int64_t sh = head_major ? L * D : D, st = head_major ? D : num_heads * D;
  jo_check(jo_qkv_norm_rope_pack_host(q_host.data_ptr(), k_host.data_ptr(), v_host.data_ptr(), sh, st,
                                      qkv_host.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                                      dev_qkv.data_ptr(), L, num_heads, D, q_weight.data_ptr(), k_weight.data_ptr(),
                                      opt_ptr(cos), opt_ptr(sin), (float)eps, chunk_tokens, stream_of(q_weight),
                                      (void*)in.stream(), (void*)out.stream()),
           "qkv_norm_rope_pack_host");
}

// Partial attention outputs o_a / o_b [1, H, S, D] (any row / head strides, as
// SDPA returns them) with their log-sum-exps [1, H, S] -> merged [S, H, D].
torch::Tensor attn_merge(const torch::Tensor& o_a, const torch::Tensor& lse_a, const torch::Tensor& o_b,
                         const torch::Tensor& lse_b) {
  JO_CHECK_CUDA(o_a);
  check_dev(o_b, o_a, "o_b");
  check_dev(lse_a, o_a, "lse_a");
  check_dev(lse_b, o_a, "lse_b");
  TORCH_CHECK(o_a.dim() == 4 && o_a.size(0) == 1 && o_b.sizes() == o_a.sizes(), "o_a / o_b must be [1, H, S, D]");
  TORCH_CHECK(o_a.stride(3) == 1 && o_b.stride(3) == 1, "o_a / o_b last dim must be contiguous");
  TORCH_CHECK(o_a.scalar_type() == o_b.scalar_type(), "o_a / o_b dtypes must match");
  const int64_t H = o_a.size(1), S = o_a.size(2), D = o_a.size(3);
  for (const torch::Tensor* l : {&lse_a, &lse_b})
    TORCH_CHECK(l->dim() == 3 && l->size(0) == 1 && l->size(1) == H && l->size(2) == S &&
                    l->scalar_type() == torch::kFloat32,
                "lse must be fp32 [1, H, S]");
  const c10::cuda::CUDAGuard guard(o_a.device());
  auto out = torch::empty({S, H, D}, o_a.options());
  jo_check(jo_attn_merge(out.data_ptr(), H * D, D, o_a.data_ptr(), o_a.stride(2), o_a.stride(1),
                         lse_a.data_ptr<float>(), lse_a.stride(1), lse_a.stride(2), o_b.data_ptr(), o_b.stride(2),
                         o_b.stride(1), lse_b.data_ptr<float>(), lse_b.stride(1), lse_b.stride(2), S, H, D,
                         dt_code(o_a.scalar_type()), stream_of(o_a)),
           "attn_merge");
  return out;
}

std::tuple<torch::Tensor, torch::Tensor> gelu_quant_fp8(const torch::Tensor& x) {
  JO_CHECK_CUDA(x);
  TORCH_CHECK(x.dim() == 2 && x.stride(-1) == 1, "x must be 2D [M, N] with contiguous rows");
  const c10::cuda::CUDAGuard guard(x.device());
  auto q = torch::empty({x.size(0), x.size(1)}, x.options().dtype(torch::kFloat8_e4m3fn));
  auto s = torch::empty({x.size(0), 1}, x.options().dtype(torch::kFloat32));
  jo_check(jo_gelu_quant_fp8(q.data_ptr(), x.size(1), s.data_ptr<float>(), x.data_ptr(), x.stride(0), x.size(0),
                             x.size(1), dt_code(x.scalar_type()), stream_of(x)),
           "gelu_quant_fp8");
  return std::make_tuple(q, s);
}

std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> gated_residual_norm_scale_shift_quant_fp8(
    const torch::Tensor& residual, const torch::Tensor& x, const torch::Tensor& gate,
    const c10::optional<torch::Tensor>& gamma, const c10::optional<torch::Tensor>& beta, const torch::Tensor& scale,
    const torch::Tensor& shift, int64_t norm_type, double eps) {
  JO_CHECK_CUDA(residual);
  JO_CHECK_CUDA(x);
  check_dev(residual, x, "residual");
  check_dev(gate, x, "gate");
  TORCH_CHECK(residual.sizes() == x.sizes(), "residual and x must have the same shape");
  TORCH_CHECK(residual.dtype() == x.dtype() && x.dtype() == gate.dtype(), "dtypes must match");
  TORCH_CHECK(norm_type == 0 || norm_type == 1, "norm_type must be 0 (layer) or 1 (rms)");
  const int64_t N = x.size(-1);
  auto r2 = as_rows(residual.contiguous(), N, "residual");
  auto x2 = as_rows(x.contiguous(), N, "x");
  auto g = gate_rows(gate, x2.size(0), N);
  auto sc = scale.reshape({-1, N});
  auto sh = shift.reshape({-1, N});
  check_mod(x2, sc, sh);
  check_affine(x2, gamma, beta);
  const c10::cuda::CUDAGuard guard(x.device());
  auto h = torch::empty_like(r2);
  auto q = torch::empty({x2.size(0), N}, x.options().dtype(torch::kFloat8_e4m3fn));
  auto s = torch::empty({x2.size(0), 1}, x.options().dtype(torch::kFloat32));
  jo_check(jo_gated_residual_norm_scale_shift_quant_fp8(
               h.data_ptr(), N, q.data_ptr(), N, s.data_ptr<float>(), r2.data_ptr(), N, x2.data_ptr(), N,
               gate.data_ptr(), g.first, g.second, opt_ptr(gamma), opt_ptr(beta), sc.data_ptr(), sh.data_ptr(),
               sc.size(0), sc.stride(0), x2.size(0), N, (int)norm_type, dt_code(x.scalar_type()), (float)eps,
               stream_of(x)),
           "gated_residual_norm_scale_shift_quant_fp8");
  return std::make_tuple(h.view(residual.sizes()), q, s);
}

torch::Tensor gated_residual(const torch::Tensor& residual, const torch::Tensor& x, const torch::Tensor& gate) {
  JO_CHECK_CUDA(residual);
  JO_CHECK_CUDA(x);
  JO_CHECK_CUDA(gate);
  check_dev(residual, x, "residual");
  check_dev(gate, x, "gate");
  TORCH_CHECK(residual.sizes() == x.sizes(), "residual and x must have the same shape");
  TORCH_CHECK(residual.dtype() == x.dtype() && x.dtype() == gate.dtype(), "dtypes must match");
  const int64_t N = x.size(-1);
  auto r2 = as_rows(residual.contiguous(), N, "residual");
  auto x2 = as_rows(x.contiguous(), N, "x");
  auto g = gate_rows(gate, x2.size(0), N);
  const c10::cuda::CUDAGuard guard(x.device());
  auto out = torch::empty_like(r2);
  jo_check(jo_gated_residual(out.data_ptr(), N, r2.data_ptr(), N, x2.data_ptr(), N, gate.data_ptr(), g.first, g.second,
                             x2.size(0), N, dt_code(x.scalar_type()), stream_of(x)),
           "gated_residual");
  return out.view(residual.sizes());
}

std::tuple<torch::Tensor, torch::Tensor> gated_residual_norm_scale_shift(
    const torch::Tensor& residual, const torch::Tensor& x, const torch::Tensor& gate,
    const c10::optional<torch::Tensor>& gamma, const c10::optional<torch::Tensor>& beta, const torch::Tensor& scale,
    const torch::Tensor& shift, int64_t norm_type, double eps) {
  JO_CHECK_CUDA(residual);
  JO_CHECK_CUDA(x);
  check_dev(residual, x, "residual");
  check_dev(gate, x, "gate");
  TORCH_CHECK(residual.sizes() == x.sizes(), "residual and x must have the same shape");
  TORCH_CHECK(residual.dtype() == x.dtype() && x.dtype() == gate.dtype(), "dtypes must match");
  TORCH_CHECK(norm_type == 0 || norm_type == 1, "norm_type must be 0 (layer) or 1 (rms)");
  const int64_t N = x.size(-1);
  auto r2 = as_rows(residual.contiguous(), N, "residual");
  auto x2 = as_rows(x.contiguous(), N, "x");
  auto g = gate_rows(gate, x2.size(0), N);
  auto sc = scale.reshape({-1, N});
  auto sh = shift.reshape({-1, N});
  check_mod(x2, sc, sh);
  check_affine(x2, gamma, beta);
  const c10::cuda::CUDAGuard guard(x.device());
  auto h = torch::empty_like(r2);
  auto y = torch::empty_like(r2);
  jo_check(jo_gated_residual_norm_scale_shift(h.data_ptr(), N, y.data_ptr(), N, r2.data_ptr(), N, x2.data_ptr(), N,
                                              gate.data_ptr(), g.first, g.second, opt_ptr(gamma), opt_ptr(beta),
                                              sc.data_ptr(), sh.data_ptr(), sc.size(0), sc.stride(0), x2.size(0), N,
                                              (int)norm_type, dt_code(x.scalar_type()), (float)eps, stream_of(x)),
           "gated_residual_norm_scale_shift");
  return std::make_tuple(h.view(residual.sizes()), y.view(residual.sizes()));
}

torch::Tensor gelu_tanh(const torch::Tensor& x) {
  JO_CHECK_CUDA(x);
  auto xc = x.contiguous();
  const c10::cuda::CUDAGuard guard(x.device());
  auto out = torch::empty_like(xc);
  jo_check(jo_gelu_tanh(out.data_ptr(), xc.data_ptr(), xc.numel(), dt_code(x.scalar_type()), stream_of(x)),
           "gelu_tanh");
  return out;
}

torch::Tensor silu_mul(const torch::Tensor& a, const torch::Tensor& b) {
  JO_CHECK_CUDA(a);
  JO_CHECK_CUDA(b);
  check_dev(b, a, "b");
  TORCH_CHECK(a.sizes() == b.sizes() && a.dtype() == b.dtype(), "a and b must match in shape and dtype");
  const int64_t N = a.size(-1);
  auto a2 = as_rows(a, N, "a");
  auto b2 = as_rows(b, N, "b");
  TORCH_CHECK(a2.dim() == 2 && b2.dim() == 2, "a/b must be viewable as [rows, N]");
  const c10::cuda::CUDAGuard guard(a.device());
  auto out = torch::empty({a2.size(0), N}, a.options());
  jo_check(jo_silu_mul(out.data_ptr(), N, a2.data_ptr(), a2.stride(0), b2.data_ptr(), b2.stride(0), a2.size(0), N,
                       dt_code(a.scalar_type()), stream_of(a)),
           "silu_mul");
  return out.view(a.sizes());
}

torch::Tensor timestep_embedding(const torch::Tensor& t, int64_t dim, bool flip_sin_to_cos,
                                 double downscale_freq_shift, double scale, double max_period) {
  JO_CHECK_CUDA(t);
  TORCH_CHECK(t.dim() == 1, "timesteps must be 1D");
  auto tf = t.to(torch::kFloat32).contiguous();
  const c10::cuda::CUDAGuard guard(t.device());
  auto out = torch::empty({t.size(0), dim}, t.options().dtype(torch::kFloat32));
  jo_check(jo_timestep_embedding(out.data_ptr<float>(), tf.data_ptr<float>(), t.size(0), dim, flip_sin_to_cos ? 1 : 0,
                                 (float)downscale_freq_shift, (float)scale, (float)max_period, stream_of(t)),
           "timestep_embedding");
  return out;
}

// Returns (vec [B, proj_dim], s2 [B, dim]): s2 = silu(temb) is the time_proj input
// (the second intermediate, kept for callers that reuse it).
std::tuple<torch::Tensor, torch::Tensor> timestep_mlp(const torch::Tensor& t, const torch::Tensor& w1,
                                                      const c10::optional<torch::Tensor>& b1,
                                                      const torch::Tensor& w2,
                                                      const c10::optional<torch::Tensor>& b2,
                                                      const torch::Tensor& w3,
                                                      const c10::optional<torch::Tensor>& b3, double max_period) {
  JO_CHECK_CUDA(t);
  TORCH_CHECK(t.dim() == 1, "timesteps must be 1D");
  for (const torch::Tensor* w : {&w1, &w2, &w3})
    TORCH_CHECK(w->dim() == 2 && w->is_contiguous() && w->scalar_type() == torch::kBFloat16 &&
                    w->device() == t.device(),
                "weights must be contiguous bf16 [out, in] on the timesteps' device");
  const int64_t dim = w1.size(0), freq = w1.size(1), proj = w3.size(0);
  TORCH_CHECK(w2.size(0) == dim && w2.size(1) == dim && w3.size(1) == dim, "weight shapes do not chain");
  auto bias_ptr = [&](const c10::optional<torch::Tensor>& b, int64_t n) -> const void* {
    if (!b.has_value()) return nullptr;
    TORCH_CHECK(b->dim() == 1 && b->numel() == n && b->is_contiguous() && b->scalar_type() == torch::kBFloat16 &&
                    b->device() == t.device(),
                "bias must be contiguous bf16 [out] on the timesteps' device");
    return b->data_ptr();
  };
  const void* pb1 = bias_ptr(b1, dim);
  const void* pb2 = bias_ptr(b2, dim);
  const void* pb3 = bias_ptr(b3, proj);
  auto tf = t.to(torch::kFloat32).contiguous();
  const c10::cuda::CUDAGuard guard(t.device());
  const int64_t B = t.size(0);
  auto vec = torch::empty({B, proj}, w1.options());
  auto scratch = torch::empty({2, B, dim}, w1.options());  // s1, s2
  jo_check(jo_timestep_mlp(vec.data_ptr(), tf.data_ptr<float>(), B, w1.data_ptr(), pb1, freq, dim, w2.data_ptr(),
                           pb2, w3.data_ptr(), pb3, proj, scratch.data_ptr(), scratch.numel() * 2,
                           (float)max_period, stream_of(t)),
           "timestep_mlp");
  return std::make_tuple(vec, scratch[1]);
}

// timestep_mlp + every block's ModulateWan add in time_proj's epilogue:
// returns (vec [B, proj_dim], mods [T, B, proj_dim]) for tables [T, proj_dim].
std::tuple<torch::Tensor, torch::Tensor> timestep_mlp_modulate(const torch::Tensor& t, const torch::Tensor& w1,
                                                               const c10::optional<torch::Tensor>& b1,
                                                               const torch::Tensor& w2,
                                                               const c10::optional<torch::Tensor>& b2,
                                                               const torch::Tensor& w3,
                                                               const c10::optional<torch::Tensor>& b3,
                                                               const torch::Tensor& tables, double max_period) {
  JO_CHECK_CUDA(t);
  TORCH_CHECK(t.dim() == 1, "timesteps must be 1D");
  for (const torch::Tensor* w : {&w1, &w2, &w3})
    TORCH_CHECK(w->dim() == 2 && w->is_contiguous() && w->scalar_type() == torch::kBFloat16 &&
                    w->device() == t.device(),
                "weights must be contiguous bf16 [out, in] on the timesteps' device");
  const int64_t dim = w1.size(0), freq = w1.size(1), proj = w3.size(0);
  TORCH_CHECK(w2.size(0) == dim && w2.size(1) == dim && w3.size(1) == dim, "weight shapes do not chain");
  check_dev(tables, t, "tables");
  TORCH_CHECK(tables.is_contiguous() && tables.scalar_type() == torch::kBFloat16 && tables.numel() % proj == 0,
              "tables must be contiguous bf16 [T, proj_dim]");
  auto bias_ptr = [&](const c10::optional<torch::Tensor>& b, int64_t n) -> const void* {
    if (!b.has_value()) return nullptr;
    TORCH_CHECK(b->dim() == 1 && b->numel() == n && b->is_contiguous() && b->scalar_type() == torch::kBFloat16 &&
                    b->device() == t.device(),
                "bias must be contiguous bf16 [out] on the timesteps' device");
    return b->data_ptr();
  };
  const void* pb1 = bias_ptr(b1, dim);
  const void* pb2 = bias_ptr(b2, dim);
  const void* pb3 = bias_ptr(b3, proj);
  auto tf = t.to(torch::kFloat32).contiguous();
  const c10::cuda::CUDAGuard guard(t.device());
  const int64_t B = t.size(0), T = tables.numel() / proj;
  auto vec = torch::empty({B, proj}, w1.options());
  auto mods = torch::empty({T, B, proj}, w1.options());
  auto scratch = torch::empty({2, B, dim}, w1.options());
  jo_check(jo_timestep_mlp_modulate(vec.data_ptr(), mods.data_ptr(), tables.data_ptr(), T, tf.data_ptr<float>(), B,
                                    w1.data_ptr(), pb1, freq, dim, w2.data_ptr(), pb2, w3.data_ptr(), pb3, proj,
                                    scratch.data_ptr(), scratch.numel() * 2, (float)max_period, stream_of(t)),
           "timestep_mlp_modulate");
  return std::make_tuple(vec, mods);
}

std::tuple<torch::Tensor, torch::Tensor> rmsnorm_quant_fp8(const torch::Tensor& x, const torch::Tensor& weight,
                                                           double eps) {
  JO_CHECK_CUDA(x);
  TORCH_CHECK(x.dim() == 2 && x.stride(-1) == 1, "x must be 2D [M, N] with contiguous rows");
  check_dev(weight, x, "weight");
  TORCH_CHECK(weight.dim() == 1 && weight.numel() == x.size(1) && weight.dtype() == x.dtype() &&
                  weight.is_contiguous(),
              "weight must be contiguous [N] of x's dtype");
  const c10::cuda::CUDAGuard guard(x.device());
  auto q = torch::empty({x.size(0), x.size(1)}, x.options().dtype(torch::kFloat8_e4m3fn));
  auto s = torch::empty({x.size(0), 1}, x.options().dtype(torch::kFloat32));
  jo_check(jo_rmsnorm_quant_fp8(q.data_ptr(), x.size(1), s.data_ptr<float>(), x.data_ptr(), x.stride(0),
                                weight.data_ptr(), x.size(0), x.size(1), dt_code(x.scalar_type()), (float)eps,
                                stream_of(x)),
           "rmsnorm_quant_fp8");
  return std::make_tuple(q, s);
}

std::tuple<torch::Tensor, torch::Tensor> norm_scale_shift_quant_fp8(
    const torch::Tensor& x, const c10::optional<torch::Tensor>& gamma, const c10::optional<torch::Tensor>& beta,
    const torch::Tensor& scale, const torch::Tensor& shift, int64_t norm_type, double eps) {
  JO_CHECK_CUDA(x);
  TORCH_CHECK(x.dim() == 2 && x.stride(-1) == 1, "x must be 2D [M, N] with contiguous rows");
  check_mod(x, scale, shift);
  check_affine(x, gamma, beta);
  TORCH_CHECK(norm_type == 0 || norm_type == 1, "norm_type must be 0 (layer) or 1 (rms)");
  const c10::cuda::CUDAGuard guard(x.device());
  auto q = torch::empty({x.size(0), x.size(1)}, x.options().dtype(torch::kFloat8_e4m3fn));
  auto s = torch::empty({x.size(0), 1}, x.options().dtype(torch::kFloat32));
  jo_check(jo_norm_scale_shift_quant_fp8(q.data_ptr(), x.size(1), s.data_ptr<float>(), x.data_ptr(), x.stride(0),
                                         opt_ptr(gamma), opt_ptr(beta), scale.data_ptr(), shift.data_ptr(),
                                         scale.size(0), scale.stride(0), x.size(0), x.size(1), (int)norm_type,
                                         dt_code(x.scalar_type()), (float)eps, stream_of(x)),
           "norm_scale_shift_quant_fp8");
  return std::make_tuple(q, s);
}

}  // namespace

TORCH_LIBRARY(joyomni_ops, m) {
  // Reference schemas, verbatim (joyomni_ops/csrc/pybind.cpp:52-75).
  m.def(
      "fused_qk_norm_rope_3d_paired(Tensor! q, Tensor! k, int seq_len, int num_heads, float eps, "
      "Tensor q_weight, Tensor k_weight, Tensor cos, Tensor sin, Tensor? k_pre_rope) -> ()");
  m.def(
      "fused_joint_qkv_pack(Tensor img_q, Tensor img_k, Tensor img_v, "
      "Tensor txt_q, Tensor txt_k, Tensor txt_v, Tensor? cached_k, Tensor? cached_v, "
      "Tensor txt_q_weight, Tensor txt_k_weight, float eps) -> (Tensor, Tensor, Tensor)");
  m.def(
      "fused_cached_kv_pack(Tensor key0, Tensor value0, Tensor? key1, Tensor? value1, "
      "Tensor cos, Tensor sin) -> (Tensor, Tensor)");
  m.def(
      "fused_norm_scale_shift(Tensor x, Tensor? gamma_opt, Tensor? beta_opt, "
      "Tensor scale, Tensor shift, int norm_type, float eps) -> Tensor");
  m.def("rmsnorm(Tensor x, Tensor weight, float eps) -> Tensor");
  m.def("sgl_per_token_quant_fp8(Tensor input, Tensor! output_q, Tensor! output_s) -> ()");
  m.def(
      "fp8_scaled_mm(Tensor mat_a, Tensor mat_b, Tensor scales_a, Tensor scales_b, "
      "ScalarType out_dtype, Tensor? bias) -> Tensor");
  // New fused ops on the same path.
  m.def(
      "fp8_scaled_mm_gated_residual(Tensor mat_a, Tensor mat_b, Tensor scales_a, Tensor scales_b, "
      "ScalarType out_dtype, Tensor? bias, Tensor residual, Tensor gate) -> Tensor");
  m.def(
      "fp8_scaled_mm_gelu_quant(Tensor mat_a, Tensor mat_b, Tensor scales_a, Tensor scales_b, "
      "ScalarType out_dtype, Tensor? bias=None) -> (Tensor, Tensor)");
  m.def(
      "qkv_norm_rope_pack(Tensor qkv, int num_heads, Tensor q_weight, Tensor k_weight, Tensor? cos, "
      "Tensor? sin, float eps, bool head_major, Tensor(a!)? k_pre_rope) -> (Tensor, Tensor, Tensor)");
  m.def(
      "qkv_norm_rope_pack_into(Tensor qkv, int num_heads, Tensor q_weight, Tensor k_weight, Tensor? cos, "
      "Tensor? sin, float eps, Tensor(a!) q_out, Tensor(b!) k_out, Tensor(c!) v_out, Tensor(d!)? k_pre_out=None) "
      "-> ()");
  m.def(
      "qkv_norm_rope_pack_host(Tensor qkv_host, int num_heads, Tensor q_weight, Tensor k_weight, Tensor? cos, "
      "Tensor? sin, float eps, bool head_major, Tensor(a!) q_host, Tensor(b!) k_host, Tensor(c!) v_host, "
      "int chunk_tokens) -> ()");
  m.def("attn_merge(Tensor o_a, Tensor lse_a, Tensor o_b, Tensor lse_b) -> Tensor");
  m.def("cached_k_rotate_into(Tensor key, Tensor cos, Tensor sin, Tensor(a!) out_key) -> ()");
  m.def("gelu_quant_fp8(Tensor x) -> (Tensor, Tensor)");
  m.def(
      "gated_residual_norm_scale_shift_quant_fp8(Tensor residual, Tensor x, Tensor gate, Tensor? gamma, "
      "Tensor? beta, Tensor scale, Tensor shift, int norm_type, float eps) -> (Tensor, Tensor, Tensor)");
  m.def("gated_residual(Tensor residual, Tensor x, Tensor gate) -> Tensor");
  m.def(
      "gated_residual_norm_scale_shift(Tensor residual, Tensor x, Tensor gate, Tensor? gamma, "
      "Tensor? beta, Tensor scale, Tensor shift, int norm_type, float eps) -> (Tensor, Tensor)");
  m.def("gelu_tanh(Tensor x) -> Tensor");
  m.def("silu_mul(Tensor a, Tensor b) -> Tensor");
  m.def(
      "timestep_embedding(Tensor t, int dim, bool flip_sin_to_cos, float downscale_freq_shift, "
      "float scale, float max_period) -> Tensor");
  m.def(
      "timestep_mlp(Tensor t, Tensor w1, Tensor? b1, Tensor w2, Tensor? b2, Tensor w3, Tensor? b3, "
      "float max_period) -> (Tensor, Tensor)");
  m.def(
      "timestep_mlp_modulate(Tensor t, Tensor w1, Tensor? b1, Tensor w2, Tensor? b2, Tensor w3, Tensor? b3, "
      "Tensor tables, float max_period) -> (Tensor, Tensor)");
  m.def("rmsnorm_quant_fp8(Tensor x, Tensor weight, float eps) -> (Tensor, Tensor)");
  m.def(
      "norm_scale_shift_quant_fp8(Tensor x, Tensor? gamma, Tensor? beta, Tensor scale, Tensor shift, "
      "int norm_type, float eps) -> (Tensor, Tensor)");
}

TORCH_LIBRARY_IMPL(joyomni_ops, CUDA, m) {
  m.impl("fused_qk_norm_rope_3d_paired", &fused_qk_norm_rope_3d_paired);
  m.impl("fused_joint_qkv_pack", &fused_joint_qkv_pack);
  m.impl("fused_cached_kv_pack", &fused_cached_kv_pack);
  m.impl("fused_norm_scale_shift", &fused_norm_scale_shift);
  m.impl("rmsnorm", &rmsnorm);
  m.impl("sgl_per_token_quant_fp8", &sgl_per_token_quant_fp8);
  m.impl("fp8_scaled_mm", &fp8_scaled_mm);
  m.impl("fp8_scaled_mm_gated_residual", &fp8_scaled_mm_gated_residual);
  m.impl("fp8_scaled_mm_gelu_quant", &fp8_scaled_mm_gelu_quant);
  m.impl("qkv_norm_rope_pack", &qkv_norm_rope_pack);
  m.impl("qkv_norm_rope_pack_into", &qkv_norm_rope_pack_into);
  m.impl("qkv_norm_rope_pack_host", &qkv_norm_rope_pack_host);
  m.impl("attn_merge", &attn_merge);
  m.impl("cached_k_rotate_into", &cached_k_rotate_into);
  m.impl("gelu_quant_fp8", &gelu_quant_fp8);
  m.impl("gated_residual_norm_scale_shift_quant_fp8", &gated_residual_norm_scale_shift_quant_fp8);
  m.impl("gated_residual", &gated_residual);
  m.impl("gated_residual_norm_scale_shift", &gated_residual_norm_scale_shift);
  m.impl("gelu_tanh", &gelu_tanh);
  m.impl("silu_mul", &silu_mul);
  m.impl("timestep_embedding", &timestep_embedding);
  m.impl("timestep_mlp", &timestep_mlp);
  m.impl("timestep_mlp_modulate", &timestep_mlp_modulate);
  m.impl("rmsnorm_quant_fp8", &rmsnorm_quant_fp8);
  m.impl("norm_scale_shift_quant_fp8", &norm_scale_shift_quant_fp8);
}
