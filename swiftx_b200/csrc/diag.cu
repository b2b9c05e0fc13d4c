// Diagnostic entry point: evaluates the FMA-pipe 2^x (ex2x2_fma, common.cuh) that the
// backward's summary kernel uses for part of its decays, so its accuracy can be checked
// against a float64 reference on the device that runs it.
#include <algorithm>

#include "common.cuh"

namespace {

__global__ void exp2_fma_eval_kernel(const float* x, float* y, int64_t n) {
    for (int64_t i = 2 * (blockIdx.x * (int64_t)blockDim.x + threadIdx.x); i < n;
         i += 2 * (int64_t)gridDim.x * blockDim.x) {
        const float2 v = swx::f2(x[i], i + 1 < n ? x[i + 1] : 0.f);
        const float2 r = swx::ex2x2_fma(v);
        y[i] = r.x;
        if (i + 1 < n) y[i + 1] = r.y;
    }
}

}  // namespace

extern "C" int swx_exp2_fma_eval(const float* x, float* y, int64_t n, void* stream) {
    if (n < 0 || (n > 0 && (!x || !y))) return SWX_ERR_INVALID_ARG;
    if (n == 0) return SWX_OK;
    const int blocks = (int)std::min<int64_t>((n / 2 + 255) / 256 + 1, 148 * 8);
    exp2_fma_eval_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n);
    return cudaGetLastError() == cudaSuccess ? SWX_OK : SWX_ERR_CUDA;
}
