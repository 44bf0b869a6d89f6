// kernels_gemv_q40.cu -- instantiation of the fused GEMV for GGUF type 2.
#include "kernels_gemv.cuh"

namespace nx {
template cudaError_t launch_gemv_fmt<2>(const GemvParams &p, cudaStream_t st);
}  // namespace nx
