// kernels_gemv_q2k.cu -- instantiation of the fused GEMV for GGUF type 10.
#include "kernels_gemv.cuh"

namespace nx {
template cudaError_t launch_gemv_fmt<10>(const GemvParams &p, cudaStream_t st);
}  // namespace nx
