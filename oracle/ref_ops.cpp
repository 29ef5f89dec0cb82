// Test infrastructure only: registers the REFERENCE's own light CUDA kernels
// (compiled unmodified from joyomni_ops/csrc/{rmsnorm,fused_norm_scale_shift,
// fused_qknorm_rope_3d_kernel,fused_joint_qkv_pack,per_token_quant_fp8}.cu by
// oracle/build_ref.py) as torch.ops.joyomni_ref.*, so that they can be loaded
// in the same process as this repository's torch.ops.joyomni_ops.* and used as
// a checker and a GPU-side baseline.  Nothing in the product loads this file.
//
// The declarations restate the reference entry points' signatures
// (joyomni_ops/csrc/pybind.cpp:10-50) and the schemas are those of
// joyomni_ops/csrc/pybind.cpp:52-69; the FP8 GEMM is absent (it needs CUTLASS at
// a pinned tag that is not available to this build).
#include <torch/all.h>
#include <torch/library.h>

namespace joyomni_ops {

void fused_qk_norm_rope_3d_paired(torch::Tensor& q, torch::Tensor& k, int64_t seq_len, int64_t num_heads,
                                  double eps, torch::Tensor& q_weight, torch::Tensor& k_weight, torch::Tensor& cos,
                                  torch::Tensor& sin, const c10::optional<torch::Tensor>& k_pre_rope_opt);

std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> fused_joint_qkv_pack(
    const torch::Tensor& img_q, const torch::Tensor& img_k, const torch::Tensor& img_v, const torch::Tensor& txt_q,
    const torch::Tensor& txt_k, const torch::Tensor& txt_v, const c10::optional<torch::Tensor>& cached_k_opt,
    const c10::optional<torch::Tensor>& cached_v_opt, const torch::Tensor& txt_q_weight,
    const torch::Tensor& txt_k_weight, double eps);

std::tuple<torch::Tensor, torch::Tensor> fused_cached_kv_pack(const torch::Tensor& key0, const torch::Tensor& value0,
                                                              const c10::optional<torch::Tensor>& key1_opt,
                                                              const c10::optional<torch::Tensor>& value1_opt,
                                                              const torch::Tensor& cos, const torch::Tensor& sin);

torch::Tensor fused_norm_scale_shift(const torch::Tensor& x, const c10::optional<torch::Tensor>& gamma_opt,
                                     const c10::optional<torch::Tensor>& beta_opt, const torch::Tensor& scale,
                                     const torch::Tensor& shift, int64_t norm_type, double eps);

torch::Tensor rmsnorm(const torch::Tensor& x, const torch::Tensor& weight, double eps);

void sgl_per_token_quant_fp8(torch::Tensor input, torch::Tensor output_q, torch::Tensor output_s);

}  // namespace joyomni_ops

TORCH_LIBRARY(joyomni_ref, m) {
  m.def(
      "fused_qk_norm_rope_3d_paired(Tensor! q, Tensor! k, int seq_len, int num_heads, float eps, "
      "Tensor q_weight, Tensor k_weight, Tensor cos, Tensor sin, Tensor? k_pre_rope) -> ()");
  m.def(
      "fused_joint_qkv_pack(Tensor img_q, Tensor img_k, Tensor img_v, Tensor txt_q, Tensor txt_k, Tensor txt_v, "
      "Tensor? cached_k, Tensor? cached_v, Tensor txt_q_weight, Tensor txt_k_weight, float eps) "
      "-> (Tensor, Tensor, Tensor)");
  m.def(
      "fused_cached_kv_pack(Tensor key0, Tensor value0, Tensor? key1, Tensor? value1, Tensor cos, Tensor sin) "
      "-> (Tensor, Tensor)");
  m.def(
      "fused_norm_scale_shift(Tensor x, Tensor? gamma_opt, Tensor? beta_opt, Tensor scale, Tensor shift, "
      "int norm_type, float eps) -> Tensor");
  m.def("rmsnorm(Tensor x, Tensor weight, float eps) -> Tensor");
  m.def("sgl_per_token_quant_fp8(Tensor input, Tensor! output_q, Tensor! output_s) -> ()");
}

TORCH_LIBRARY_IMPL(joyomni_ref, CUDA, m) {
  m.impl("fused_qk_norm_rope_3d_paired", &joyomni_ops::fused_qk_norm_rope_3d_paired);
  m.impl("fused_joint_qkv_pack", &joyomni_ops::fused_joint_qkv_pack);
  m.impl("fused_cached_kv_pack", &joyomni_ops::fused_cached_kv_pack);
  m.impl("fused_norm_scale_shift", &joyomni_ops::fused_norm_scale_shift);
  m.impl("rmsnorm", &joyomni_ops::rmsnorm);
  m.impl("sgl_per_token_quant_fp8", &joyomni_ops::sgl_per_token_quant_fp8);
}
