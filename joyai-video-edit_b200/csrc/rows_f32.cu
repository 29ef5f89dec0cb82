// Row kernels instantiated for float.
#include "rows_impl.cuh"

namespace jo {
namespace rows {
template int launch_rows_t<float, kRms, kLoadX, kStoreY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<float, kLayer, kLoadX, kStoreY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<float, kLayer, kResidGate, kStoreY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<float, kRms, kResidGate, kStoreY>(const RowArgs&, cudaStream_t);
template int launch_rows_t<float, kNoNorm, kResidGate, kNoY>(const RowArgs&, cudaStream_t);
}  // namespace rows
}  // namespace jo
