// Explicit instantiations of the W8A16 GEMM (split across files to compile in parallel).
#include "gemm_kernel.cuh"
namespace vela {
template void launch_gemm<64, 6, SRC_X32, EPI_PLAIN>(const GemmArgs&, int, cudaStream_t);
template void launch_gemm<128, 4, SRC_X32, EPI_PLAIN>(const GemmArgs&, int, cudaStream_t);
template void launch_gemm<256, 4, SRC_X32, EPI_PLAIN>(const GemmArgs&, int, cudaStream_t);
}  // namespace vela
