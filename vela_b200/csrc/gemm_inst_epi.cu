// Explicit instantiations of the W8A16 GEMM with the GEGLU, split3 and q|k|v epilogues.
#include "gemm_kernel.cuh"
namespace vela {
template void launch_gemm<128, 4, SRC_I8, EPI_GEGLU>(const GemmArgs&, int, cudaStream_t);
template void launch_gemm<256, 4, SRC_I8, EPI_GEGLU>(const GemmArgs&, int, cudaStream_t);
template void launch_gemm<128, 4, SRC_I8, EPI_SPLIT3>(const GemmArgs&, int, cudaStream_t);
template void launch_gemm<128, 4, SRC_I8, EPI_QKV>(const GemmArgs&, int, cudaStream_t);
}  // namespace vela
