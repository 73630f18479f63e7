// On-device quality statistics of a quantized model, the numbers the
// reference prints after quantizing (code/run_any_model.py:89-110): per
// weight, MSE and cosine between the original weight and w_hat; for the
// model, MSE and cosine between baseline and quantized logits. One reduction
// serves both: for two arrays a, b of n bf16 or float32 values it returns
// sum (a - b)^2, sum a*b, sum a^2, sum b^2 in float64. Block partial sums go
// to a caller workspace and one block adds them in block order, so the result
// does not depend on scheduling (the same inputs give the same bits).
#include <cuda_runtime.h>

#include "cdq.h"

namespace {

constexpr int kThreads = 256;
constexpr int kMaxBlocks = 1024;

__device__ __forceinline__ double val(const void* p, int dt, int64_t i) {
    if (dt == 0) return (double)__uint_as_float((uint32_t) static_cast<const uint16_t*>(p)[i] << 16);
    return (double)static_cast<const float*>(p)[i];
}

__device__ __forceinline__ void block_sum4(double (&s)[4], double (*red)[kThreads / 32]) {
    for (int k = 0; k < 4; ++k)
        for (int o = 16; o; o >>= 1) s[k] += __shfl_xor_sync(0xFFFFFFFFu, s[k], o);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0)
        for (int k = 0; k < 4; ++k) red[k][w] = s[k];
    __syncthreads();
    if (threadIdx.x == 0)
        for (int k = 0; k < 4; ++k) {
            double t = 0.0;
            for (int j = 0; j < kThreads / 32; ++j) t += red[k][j];
            s[k] = t;
        }
}

__global__ void __launch_bounds__(kThreads) compare_partials(const void* a, const void* b, int dt, int64_t n,
                                                           double* __restrict__ part) {
    __shared__ double red[4][kThreads / 32];
    double s[4] = {0.0, 0.0, 0.0, 0.0};
    for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
        const double x = val(a, dt, i), y = val(b, dt, i), d = x - y;
        s[0] = fma(d, d, s[0]);
        s[1] = fma(x, y, s[1]);
        s[2] = fma(x, x, s[2]);
        s[3] = fma(y, y, s[3]);
    }
    block_sum4(s, red);
    if (threadIdx.x == 0)
        for (int k = 0; k < 4; ++k) part[4 * blockIdx.x + k] = s[k];
}

__global__ void __launch_bounds__(kThreads) compare_final(const double* __restrict__ part, int blocks,
                                                        double* __restrict__ out) {
    __shared__ double red[4][kThreads / 32];
    double s[4] = {0.0, 0.0, 0.0, 0.0};
    for (int i = threadIdx.x; i < blocks; i += kThreads)
        for (int k = 0; k < 4; ++k) s[k] += part[4 * i + k];
    block_sum4(s, red);
    if (threadIdx.x == 0)
        for (int k = 0; k < 4; ++k) out[k] = s[k];
}

}  // namespace

extern "C" cdq_status cdq_compare_stats(const void* a, const void* b, int64_t n, int32_t dtype, double* out,
                                        double* workspace, int64_t workspace_bytes, void* stream) {
    if (!a || !b || !out || !workspace || n < 1 || (dtype != 0 && dtype != 1)) return CDQ_ERR_ARG;
    if (workspace_bytes < (int64_t)kMaxBlocks * 4 * (int64_t)sizeof(double)) return CDQ_ERR_WORKSPACE;
    const int64_t want = (n + kThreads * 8 - 1) / (kThreads * 8);
    const int blocks = (int)(want < 1 ? 1 : (want > kMaxBlocks ? kMaxBlocks : want));
    compare_partials<<<blocks, kThreads, 0, (cudaStream_t)stream>>>(a, b, dtype, n, workspace);
    compare_final<<<1, kThreads, 0, (cudaStream_t)stream>>>(workspace, blocks, out);
    return cudaGetLastError() == cudaSuccess ? CDQ_OK : CDQ_ERR_CUDA;
}
