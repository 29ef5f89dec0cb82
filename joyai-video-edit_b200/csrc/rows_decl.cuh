// Declarations shared by the row-kernel entry points (rows.cu) and their
// per-dtype implementations (rows_impl.cuh).
#pragma once
#include "common.cuh"

namespace jo {
namespace rows {

enum NormKind { kNoNorm = 0, kLayer = 1, kRms = 2 };
enum ProKind { kLoadX = 0, kResidGate = 1, kGeluX = 2 };  // kGeluX: x -> T(gelu_tanh(x))
enum EpiKind { kStoreY = 0, kQuantY = 1, kNoY = 2 };

struct RowArgs {
  void* out;
  int64_t out_stride;
  uint8_t* out_q;
  int64_t q_stride;
  float* out_s;
  void* out_h;
  int64_t h_stride;
  const void* x;
  int64_t x_stride;
  const void* res;
  int64_t res_stride;
  const void* gate;
  int64_t gate_stride;  // 0 => one gate row broadcast over all rows
  const void* gamma;
  const void* beta;
  const void* scale;
  const void* shift;
  int64_t mod_stride;  // 0 => one modulation row broadcast over all rows
  int64_t rows;
  int64_t cols;
  float eps;
};

// Launch the row op (kNorm, kPro, kEpi) for element type T; explicitly
// instantiated in rows_bf16.cu, rows_f16.cu and rows_f32.cu.
template <typename T, int kNorm, int kPro, int kEpi>
int launch_rows_t(const RowArgs& a, cudaStream_t st);

}  // namespace rows
}  // namespace jo
