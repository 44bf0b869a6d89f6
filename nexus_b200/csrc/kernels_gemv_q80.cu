// kernels_gemv_q80.cu -- instantiation of the fused GEMV for GGUF type 8.
#include "kernels_gemv.cuh"

namespace nx {
template cudaError_t launch_gemv_fmt<8>(const GemvParams &p, cudaStream_t st);
}  // namespace nx
