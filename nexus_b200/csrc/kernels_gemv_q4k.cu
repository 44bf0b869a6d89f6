// kernels_gemv_q4k.cu -- instantiation of the fused GEMV for GGUF type 12.
#include "kernels_gemv.cuh"

namespace nx {
template cudaError_t launch_gemv_fmt<12>(const GemvParams &p, cudaStream_t st);
}  // namespace nx
