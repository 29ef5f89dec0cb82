// Row kernels instantiated for __half.
#include "rows_impl.cuh"

namespace jo {
namespace rows {
template int launch_rows_t<__half, kRms, kLoadX, kStoreY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__half, kLayer, kLoadX, kStoreY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__half, kLayer, kResidGate, kStoreY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__half, kRms, kResidGate, kStoreY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__half, kNoNorm, kLoadX, kQuantY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__half, kRms, kLoadX, kQuantY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__half, kLayer, kLoadX, kQuantY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__half, kNoNorm, kResidGate, kNoY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__half, kNoNorm, kGeluX, kQuantY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__half, kLayer, kResidGate, kQuantY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<__half, kRms, kResidGate, kQuantY>(const RowArgs&, cudaStream_t);
}  // namespace rows
}  // namespace jo
