// Gradient of the SiftX per-token group weights when the pathway mix is fused into the
// scan's gate (models/sift_block.py:137-142: y * w[..., group_of], then * silu(z)):
//   d_group_w[b, t, g] = sum over channels d of group g of dout[b,t,d] * silu(z[b,t,d]) * y[b,t,d]
// with y the pre-gate output the forward saved.  One warp per (b, t) row: lane l takes
// channels l, l+32, ... and keeps one running sum per group (the channel's group compared
// with each of the SWX_MAX_GROUPS slots, so no register array is indexed at run time);
// then an xor butterfly per group.  The order of every sum is fixed: bit-reproducible.
// Reads 2 input-dtype values and one fp32 value per (b, t, d), writes b*L*ngroups floats.
#include <algorithm>

#include "common.cuh"
#include "scan_params.cuh"

namespace swx {

constexpr int PG_THREADS = 256;

template <typename Tin>
__global__ void __launch_bounds__(PG_THREADS) group_w_grad_kernel(const ScanDev p) {
    const int lane = threadIdx.x & 31;
    const int64_t rows = (int64_t)p.b * p.L;
    const int64_t nwarps = (int64_t)gridDim.x * (PG_THREADS / 32);
    for (int64_t r = blockIdx.x * (int64_t)(PG_THREADS / 32) + (threadIdx.x >> 5); r < rows; r += nwarps) {
        const int bi = (int)(r / p.L);
        const int64_t t = r - (int64_t)bi * p.L;
        const Tin* dout = static_cast<const Tin*>(p.dout) + bi * p.dout_sb + t * p.dout_sl;
        const Tin* z = static_cast<const Tin*>(p.z) + bi * p.z_sb + t * p.z_sl;
        const float* y = p.ypre + r * p.D;
        float acc[SWX_MAX_GROUPS];
#pragma unroll
        for (int k = 0; k < SWX_MAX_GROUPS; ++k) acc[k] = 0.f;
        for (int d = lane; d < p.D; d += 32) {
            const float v = Elem<Tin>::to_f(dout[d]) * silu_f(Elem<Tin>::to_f(z[d])) * y[d];
            const int g = p.gof[d];
#pragma unroll
            for (int k = 0; k < SWX_MAX_GROUPS; ++k) acc[k] += g == k ? v : 0.f;
        }
#pragma unroll
        for (int k = 0; k < SWX_MAX_GROUPS; ++k) {
            if (k >= p.ngroups) break;
            float v = acc[k];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) p.dgw[r * p.ngroups + k] = v;
        }
    }
}

cudaError_t launch_group_w_grad(const ScanDev& p, int in_dtype, cudaStream_t st) {
    const int64_t rows = (int64_t)p.b * p.L;
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, 148 * 8));
    if (in_dtype == SWX_DTYPE_BF16) group_w_grad_kernel<__nv_bfloat16><<<blocks, PG_THREADS, 0, st>>>(p);
    else group_w_grad_kernel<float><<<blocks, PG_THREADS, 0, st>>>(p);
    return cudaGetLastError();
}

}  // namespace swx
