// Explicit instantiations of the persistent W8A16 GEMM (split across files to compile in parallel): planar sources.
#include "gemm_persist.cuh"
namespace vela {
template void launch_gemm_persist<64, 6, SRC_I8, EPI_PLAIN>(const GemmArgs&, cudaStream_t);
template void launch_gemm_persist<128, 6, SRC_I8, EPI_PLAIN>(const GemmArgs&, cudaStream_t);
template void launch_gemm_persist<160, 6, SRC_I8, EPI_PLAIN>(const GemmArgs&, cudaStream_t);
template void launch_gemm_persist<256, 5, SRC_I8, EPI_PLAIN>(const GemmArgs&, cudaStream_t);
template void launch_gemm_persist<128, 6, SRC_I8, EPI_GEGLU>(const GemmArgs&, cudaStream_t);
template void launch_gemm_persist<128, 6, SRC_I8, EPI_SPLIT3>(const GemmArgs&, cudaStream_t);
template void launch_gemm_persist<128, 6, SRC_I8, EPI_QKV>(const GemmArgs&, cudaStream_t);
}  // namespace vela
