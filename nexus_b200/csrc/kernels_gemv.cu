// kernels_gemv.cu -- format dispatch of the dequant-fused GEMV
// (kernels_gemv.cuh); each block format is instantiated in its own
// translation unit (kernels_gemv_<fmt>.cu) so they compile in parallel.
#include "kernels.h"

namespace nx {
template <int FMT>
cudaError_t launch_gemv_fmt(const GemvParams &p, cudaStream_t st);

cudaError_t launch_gemv(const GemvParams &p, cudaStream_t st) {
    if (p.k % 256 != 0 || p.n <= 0) return cudaErrorInvalidValue;
    switch (p.fmt) {
    case 12: return launch_gemv_fmt<12>(p, st);
    case 8: return launch_gemv_fmt<8>(p, st);
    case 2: return launch_gemv_fmt<2>(p, st);
    case 10: return launch_gemv_fmt<10>(p, st);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace nx
