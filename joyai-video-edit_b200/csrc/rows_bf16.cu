// Row kernels instantiated for __nv_bfloat16.
#include "rows_impl.cuh"

namespace jo {
namespace rows {
template int launch_rows_t<__nv_bfloat16, kRms, kLoadX, kStoreY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__nv_bfloat16, kLayer, kLoadX, kStoreY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__nv_bfloat16, kLayer, kResidGate, kStoreY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__nv_bfloat16, kRms, kResidGate, kStoreY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__nv_bfloat16, kNoNorm, kLoadX, kQuantY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__nv_bfloat16, kRms, kLoadX, kQuantY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__nv_bfloat16, kLayer, kLoadX, kQuantY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__nv_bfloat16, kNoNorm, kResidGate, kNoY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__nv_bfloat16, kNoNorm, kGeluX, kQuantY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__nv_bfloat16, kLayer, kResidGate, kQuantY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__nv_bfloat16, kRms, kResidGate, kQuantY>(const RowArgs&, cudaStream_t);
}  // namespace rows
}  // namespace jo
