// Explicit instantiations of the W8A16 GEMM (split across files to compile in parallel).
#include "gemm_kernel.cuh"
namespace vela {
template void launch_gemm<64, 3, SRC_CONV32, EPI_PLAIN>(const GemmArgs&, int, cudaStream_t);
template void launch_gemm<128, 3, SRC_CONV32, EPI_PLAIN>(const GemmArgs&, int, cudaStream_t);
template void launch_gemm<256, 3, SRC_CONV32, EPI_PLAIN>(const GemmArgs&, int, cudaStream_t);
}  // namespace vela
