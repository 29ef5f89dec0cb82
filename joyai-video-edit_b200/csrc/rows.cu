// C entry points of the row kernels (implementation: rows_impl.cuh, instantiated
// per dtype in rows_bf16.cu / rows_f16.cu / rows_f32.cu).
#include "rows_decl.cuh"

namespace jo {
namespace rows {

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
using namespace jo::rows;

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

int jo_gelu_quant_fp8(void* out_q, int64_t q_row_stride, float* out_s, const void* x, int64_t x_row_stride,
                      int64_t rows, int64_t cols, int dtype, void* stream) {
  RowArgs a{};
  a.out_q = (uint8_t*)out_q;
  a.q_stride = q_row_stride;
  a.out_s = out_s;
  a.x = x;
  a.x_stride = x_row_stride;
  a.rows = rows;
  a.cols = cols;
  if (int s = check_common(a, "gelu_quant_fp8")) return s;
  if (rows > 0 && (!out_q || !out_s)) return fail(JO_ERR_INVALID, "gelu_quant_fp8: outputs must be non-null");
  return launch_rows<kNoNorm, kGeluX, kQuantY>(dtype, a, (cudaStream_t)stream, false);
}

int jo_gated_residual_norm_scale_shift_quant_fp8(
    void* out_h, int64_t h_row_stride, void* out_q, int64_t q_row_stride, float* out_s, const void* residual,
    int64_t res_row_stride, const void* x, int64_t x_row_stride, const void* gate, int64_t gate_rows,
    int64_t gate_row_stride, const void* gamma, const void* beta, const void* scale, const void* shift,
    int64_t mod_rows, int64_t mod_row_stride, int64_t rows, int64_t cols, int norm, int dtype, float eps,
    void* stream) {
  RowArgs a{};
  a.out_h = out_h;
  a.h_stride = h_row_stride;
  a.out_q = (uint8_t*)out_q;
  a.q_stride = q_row_stride;
  a.out_s = out_s;
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
  const char* op = "gated_residual_norm_scale_shift_quant_fp8";
  if (int s = check_common(a, op)) return s;
  if (rows > 0 && cols > 0 && (!out_h || !out_q || !out_s || !residual || !gate))
    return fail(JO_ERR_INVALID, "%s: null operand", op);
  if (gate_rows != 1 && gate_rows != rows)
    return fail(JO_ERR_SHAPE, "%s: gate rows must be 1 or %lld", op, (long long)rows);
  a.gate_stride = gate_rows == 1 ? 0 : gate_row_stride;
  if (int s = mod_setup(a, scale, shift, mod_rows, mod_row_stride, rows, op)) return s;
  const int nk = norm_code(norm, op);
  if (nk < 0) return nk;
  if (nk == kRms) a.beta = nullptr;
  cudaStream_t st = (cudaStream_t)stream;
  return nk == kLayer ? launch_rows<kLayer, kResidGate, kQuantY>(dtype, a, st, false)
                      : launch_rows<kRms, kResidGate, kQuantY>(dtype, a, st, false);
}

}  // extern "C"
