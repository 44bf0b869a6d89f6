// kernels_misc.cu -- kernels behind the generic KernelOp surface
// (src/backend/mod.rs:118-183): norms, softmax, element-wise ops, an f32
// matmul, RoPE and argmax.  These serve Backend::execute callers; the decode
// step uses the fused kernels in kernels_gemv.cu / kernels_attn.cu.
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace nx {

__device__ __forceinline__ float block_sum(float v, float *sh) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    float t = 0.0f;
    for (int w = 0; w < nw; w++) t += sh[w];
    return t;
}
__device__ __forceinline__ float block_max(float v, float *sh) {
    v = warp_max(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    float t = -INFINITY;
    for (int w = 0; w < nw; w++) t = fmaxf(t, sh[w]);
    return t;
}

// rms_norm, src/kernel/mod.rs:199-209 (one row per CTA)
__global__ void k_rms_norm(const float *x, const float *w, float *out, int n, float eps) {
    __shared__ float sh[32];
    const float *xr = x + (size_t)blockIdx.x * n;
    float *orow = out + (size_t)blockIdx.x * n;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss += xr[i] * xr[i];
    ss = block_sum(ss, sh);
    const float rstd = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) orow[i] = __fmul_rn(__fmul_rn(xr[i], rstd), w[i]);
}

// layer_norm, src/kernel/mod.rs:212-231
__global__ void k_layer_norm(const float *x, const float *w, const float *b, float *out, int n, float eps) {
    __shared__ float sh[32];
    const float *xr = x + (size_t)blockIdx.x * n;
    float *orow = out + (size_t)blockIdx.x * n;
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += xr[i];
    const float mean = block_sum(s, sh) / (float)n;
    float v = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) v += (xr[i] - mean) * (xr[i] - mean);
    const float var = block_sum(v, sh) / (float)n;
    const float rstd = 1.0f / sqrtf(var + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float nrm = (xr[i] - mean) * rstd;
        orow[i] = nrm * w[i] + (b ? b[i] : 0.0f);
    }
}

// softmax, src/kernel/mod.rs:234-255
__global__ void k_softmax(const float *x, float *out, int n) {
    __shared__ float sh[32];
    const float *xr = x + (size_t)blockIdx.x * n;
    float *orow = out + (size_t)blockIdx.x * n;
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, xr[i]);
    mx = block_max(mx, sh);
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += expf(xr[i] - mx);
    s = block_sum(s, sh);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float e = expf(xr[i] - mx);
        orow[i] = s > 0.0f ? e / s : e;
    }
}

__global__ void k_binary(int op, const float *a, const float *b, float *out, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = op == 0 ? a[i] + b[i] : a[i] * b[i];
}

// C[m,n] = A[m,k] @ B, B = [n,k] (transpose_b) or [k,n]; 16x16 smem tiles, f32
__global__ void k_matmul(const float *a, const float *b, float *c, int m, int n, int k, int tb) {
    __shared__ float As[16][17], Bs[16][17];
    const int row = blockIdx.y * 16 + threadIdx.y, col = blockIdx.x * 16 + threadIdx.x;
    float acc = 0.0f;
    for (int k0 = 0; k0 < k; k0 += 16) {
        const int ka = k0 + threadIdx.x, kb = k0 + threadIdx.y;
        As[threadIdx.y][threadIdx.x] = (row < m && ka < k) ? a[(size_t)row * k + ka] : 0.0f;
        float bv = 0.0f;
        if (col < n && kb < k) bv = tb ? b[(size_t)col * k + kb] : b[(size_t)kb * n + col];
        Bs[threadIdx.y][threadIdx.x] = bv;
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 16; i++) acc += As[threadIdx.y][i] * Bs[i][threadIdx.x];
        __syncthreads();
    }
    if (row < m && col < n) c[(size_t)row * n + col] = acc;
}

// rope_single over `heads` heads (src/kernel/mod.rs:258-271).  The angle uses
// the device powf/cosf/sinf; the decode path uses a host-computed table.
__global__ void k_rope(float *x, int heads, int head_dim, int position, float base) {
    const int half = head_dim / 2;
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < heads * half; idx += gridDim.x * blockDim.x) {
        const int h = idx / half, d = idx % half;
        const float inv_freq = (float)position / powf(base, 2.0f * (float)d / (float)head_dim);
        const float cs = cosf(inv_freq), sn = sinf(inv_freq);
        float *p = x + (size_t)h * head_dim;
        const float x0 = p[d], x1 = p[d + half];
        p[d] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
        p[d + half] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
    }
}

// greedy_token (src/engine/mod.rs:809-817) as a packed 64-bit atomic max
__global__ void k_argmax(const float *x, size_t n, unsigned long long *best) {
    unsigned long long key = 0ull;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float v = x[i];
        if (!isfinite(v)) continue;
        const unsigned long long k2 =
            ((unsigned long long)((unsigned)total_key(v) ^ 0x80000000u) << 32) | (unsigned)i;
        key = k2 > key ? k2 : key;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
    }
    if ((threadIdx.x & 31) == 0 && key) atomicMax(best, key);
}

cudaError_t launch_rms_norm(const float *x, const float *w, float *out, int rows, int n, float eps, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    k_rms_norm<<<rows, 256, 0, st>>>(x, w, out, n, eps);
    return cudaGetLastError();
}
cudaError_t launch_layer_norm(const float *x, const float *w, const float *b, float *out, int rows, int n,
                              float eps, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    k_layer_norm<<<rows, 256, 0, st>>>(x, w, b, out, n, eps);
    return cudaGetLastError();
}
cudaError_t launch_softmax(const float *x, float *out, int rows, int n, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    k_softmax<<<rows, 256, 0, st>>>(x, out, n);
    return cudaGetLastError();
}
cudaError_t launch_binary(int op, const float *a, const float *b, float *out, size_t n, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    size_t g = (n + 255) / 256;
    if (g > 148 * 16) g = 148 * 16;
    k_binary<<<(unsigned)g, 256, 0, st>>>(op, a, b, out, n);
    return cudaGetLastError();
}
cudaError_t launch_matmul_f32(const float *a, const float *b, float *c, int m, int n, int k, int transpose_b,
                              cudaStream_t st) {
    if (m <= 0 || n <= 0) return cudaSuccess;
    dim3 grid((n + 15) / 16, (m + 15) / 16), block(16, 16);
    k_matmul<<<grid, block, 0, st>>>(a, b, c, m, n, k, transpose_b);
    return cudaGetLastError();
}
cudaError_t launch_rope(float *x, int heads, int head_dim, int position, float base, cudaStream_t st) {
    const int total = heads * (head_dim / 2);
    if (total <= 0) return cudaSuccess;
    k_rope<<<(total + 255) / 256, 256, 0, st>>>(x, heads, head_dim, position, base);
    return cudaGetLastError();
}
cudaError_t launch_argmax(const float *x, size_t n, unsigned long long *best, cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(best, 0, sizeof(unsigned long long), st);
    if (e != cudaSuccess || n == 0) return e;
    size_t g = (n + 255) / 256;
    if (g > 148 * 8) g = 148 * 8;
    k_argmax<<<(unsigned)g, 256, 0, st>>>(x, n, best);
    return cudaGetLastError();
}

}  // namespace nx
