// Explicit instantiations of the persistent W8A16 GEMM (split across files to compile in parallel): SRC_CONV32.
#include "gemm_persist.cuh"
namespace vela {
template void launch_gemm_persist<64, 4, SRC_CONV32, EPI_PLAIN>(const GemmArgs&, cudaStream_t);
template void launch_gemm_persist<128, 4, SRC_CONV32, EPI_PLAIN>(const GemmArgs&, cudaStream_t);
template void launch_gemm_persist<160, 4, SRC_CONV32, EPI_PLAIN>(const GemmArgs&, cudaStream_t);
}  // namespace vela
