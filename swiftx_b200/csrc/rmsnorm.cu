// RMSNorm of the LM around the mixer (models/sift_model.py:17-26, the pre-norm of every
// residual block and the final norm):  y = (x * rsqrt(mean(x^2) + eps)) * w,  in fp32.
// In the reference this is six elementwise / reduction launches forward and about ten
// backward per use; here it is one launch each way (plus a fixed-order sum of the weight
// gradient), which matters in a training step of many small launches.
//
// Forward: one warp per row held in registers; lanes stride the columns (coalesced
// 128-byte accesses), the sum of squares is a warp reduction; the per-row rsqrt is saved
// for the backward.
// Backward (x^ = x r, g = w dy):  dx = r (g - x^ mean(x^ g)),  dw = sum_rows dy x^.
// A fixed grid of warps walks the rows in a fixed assignment, accumulating dw per lane in
// registers; each CTA sums its warps' partials in warp order and a second kernel sums the
// CTAs' partials in CTA order (deterministic).
// Residual form (x_{i+1} = x_i + h_i feeding the next norm): the forward adds the residual
// input first and writes the sum; the backward adds the sum's other incoming gradient to
// dx and writes it a second time in the residual input's type -- the separate add, its
// backward and the gradient cast folded into the norm's two launches.
#include "common.cuh"

#include <algorithm>

namespace swx {

constexpr int NORM_WARPS = 8;                 // warps per CTA
constexpr int NORM_MAXC = 32;                 // columns per lane (the row in registers): d <= 1024
constexpr int NORM_BWD_CTAS = 148 * 2;                 // fixed backward grid
constexpr int NORM_BWD_WARPS = NORM_BWD_CTAS * NORM_WARPS;

struct NormDev {
    int rows, d;
    float eps;
    const void* x; const float* w; void* y; float* rstd;
    const void* dy; void* dx; float* dw_part; float* dw;
    const void* res; void* sum;        // residual form, forward: s = x + res -> sum
    const float* dsum; void* dres;     // residual form, backward: dx += dsum; dres = dx
    int res_bf16;                      // res / dres element type
};

__device__ __forceinline__ float load_res(const void* base, int64_t i, int bf16) {
    return bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]) : static_cast<const float*>(base)[i];
}

__device__ __forceinline__ void store_res(void* base, int64_t i, float v, int bf16) {
    if (bf16) static_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
    else static_cast<float*>(base)[i] = v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// The row stays in registers (NC columns per lane), so x (and the residual) are read once.
template <typename T, typename TY, int NC>
__global__ void __launch_bounds__(32 * NORM_WARPS) rmsnorm_fwd_kernel(const NormDev p) {
    const int row = blockIdx.x * NORM_WARPS + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= p.rows) return;
    const int64_t o = (int64_t)row * p.d;
    const T* x = static_cast<const T*>(p.x) + o;
    TY* y = static_cast<TY*>(p.y) + o;
    float v[NC];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        const int c = lane + 32 * k;
        v[k] = 0.f;
        if (c < p.d) {
            v[k] = Elem<T>::to_f(x[c]);
            // residual form: normalise s = x + res (rounded to T, as a stored sum would be)
            if (p.res) v[k] = Elem<T>::to_f(Elem<T>::from_f(v[k] + load_res(p.res, o + c, p.res_bf16)));
        }
        ss = fmaf(v[k], v[k], ss);
    }
    if (p.res) {
        T* sum = static_cast<T*>(p.sum) + o;
#pragma unroll
        for (int k = 0; k < NC; ++k) {
            const int c = lane + 32 * k;
            if (c < p.d) sum[c] = Elem<T>::from_f(v[k]);
        }
    }
    const float r = rsqrtf(warp_sum(ss) / p.d + p.eps);
    if (lane == 0 && p.rstd) p.rstd[row] = r;
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        const int c = lane + 32 * k;
        if (c < p.d) y[c] = Elem<TY>::from_f((v[k] * r) * p.w[c]);
    }
}

template <typename T, typename TY, int NC>
__global__ void __launch_bounds__(32 * NORM_WARPS) rmsnorm_bwd_kernel(const NormDev p) {
    const int gw = blockIdx.x * NORM_WARPS + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    float wv[NC], dwacc[NC];
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        const int c = lane + 32 * k;
        wv[k] = c < p.d ? p.w[c] : 0.f;
        dwacc[k] = 0.f;
    }
    for (int row = gw; row < p.rows; row += NORM_BWD_WARPS) {
        const T* x = static_cast<const T*>(p.x) + (int64_t)row * p.d;
        const TY* dy = static_cast<const TY*>(p.dy) + (int64_t)row * p.d;
        T* dx = static_cast<T*>(p.dx) + (int64_t)row * p.d;
        const float r = p.rstd[row];
        float xh[NC], g[NC], dyv[NC], dsv[NC];
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < NC; ++k) {
            const int c = lane + 32 * k;
            const bool ok = c < p.d;
            xh[k] = ok ? Elem<T>::to_f(x[c]) * r : 0.f;
            dyv[k] = ok ? Elem<TY>::to_f(dy[c]) : 0.f;
            dsv[k] = (ok && p.dsum) ? p.dsum[(int64_t)row * p.d + c] : 0.f;     // loaded with x, dy
            g[k] = wv[k] * dyv[k];
            s = fmaf(xh[k], g[k], s);
        }
        const float m = warp_sum(s) / p.d;
#pragma unroll
        for (int k = 0; k < NC; ++k) {
            const int c = lane + 32 * k;
            if (c < p.d) {
                float v = r * (g[k] - xh[k] * m);
                // an explicit add (never contracted into an FMA with the product above), so
                // dx is the separately rounded norm gradient plus dsum, as an unfused add gives
                if (p.dsum) v = __fadd_rn(v, dsv[k]);
                dx[c] = Elem<T>::from_f(v);
                if (p.dres) store_res(p.dres, (int64_t)row * p.d + c, v, p.res_bf16);
            }
            dwacc[k] = fmaf(dyv[k], xh[k], dwacc[k]);
        }
    }
    // the CTA's dw partial: its warps' partials summed in warp order
    __shared__ float red[NORM_WARPS][NC * 32];
    const int wi = threadIdx.x >> 5;
#pragma unroll
    for (int k = 0; k < NC; ++k) red[wi][lane + 32 * k] = dwacc[k];
    __syncthreads();
    for (int c = threadIdx.x; c < p.d; c += 32 * NORM_WARPS) {
        float t = 0.f;
#pragma unroll
        for (int i = 0; i < NORM_WARPS; ++i) t += red[i][c];
        p.dw_part[(int64_t)blockIdx.x * p.d + c] = t;
    }
}

// dw[c] = sum over the backward grid's CTAs of dw_part[cta][c], in a fixed order.
__global__ void __launch_bounds__(1024) rmsnorm_dw_kernel(const NormDev p) {
    __shared__ float part[32][33];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int c = blockIdx.x * 32 + lane;
    float s = 0.f;
    if (c < p.d) {
        // rows w, w + 32, ... in order; a fixed trip count so every load is issued up front
#pragma unroll
        for (int i = 0; i < (NORM_BWD_CTAS + 31) / 32; ++i) {
            const int r = w + 32 * i;
            if (r < NORM_BWD_CTAS) s += p.dw_part[(int64_t)r * p.d + c];
        }
    }
    part[w][lane] = s;
    __syncthreads();
    if (w == 0 && c < p.d) {
        float t = 0.f;
#pragma unroll 8
        for (int i = 0; i < 32; ++i) t += part[i][lane];
        p.dw[c] = t;
    }
}

template <typename T, typename TY>
static void launch_bwd(const NormDev& p, cudaStream_t st) {
    const int nc = (p.d + 31) / 32;
    const dim3 grid(NORM_BWD_CTAS);
    if (nc <= 8) rmsnorm_bwd_kernel<T, TY, 8><<<grid, 32 * NORM_WARPS, 0, st>>>(p);
    else if (nc <= 16) rmsnorm_bwd_kernel<T, TY, 16><<<grid, 32 * NORM_WARPS, 0, st>>>(p);
    else rmsnorm_bwd_kernel<T, TY, NORM_MAXC><<<grid, 32 * NORM_WARPS, 0, st>>>(p);
    rmsnorm_dw_kernel<<<(p.d + 31) / 32, 1024, 0, st>>>(p);
}

template <typename T, typename TY>
static void launch_fwd(const NormDev& p, unsigned grid, cudaStream_t st) {
    const int nc = (p.d + 31) / 32;
    if (nc <= 8) rmsnorm_fwd_kernel<T, TY, 8><<<grid, 32 * NORM_WARPS, 0, st>>>(p);
    else if (nc <= 16) rmsnorm_fwd_kernel<T, TY, 16><<<grid, 32 * NORM_WARPS, 0, st>>>(p);
    else rmsnorm_fwd_kernel<T, TY, NORM_MAXC><<<grid, 32 * NORM_WARPS, 0, st>>>(p);
}

template <typename T>
static void launch_fwd_x(const NormDev& p, int out_dtype, unsigned grid, cudaStream_t st) {
    if (out_dtype == SWX_DTYPE_F32) launch_fwd<T, float>(p, grid, st);
    else launch_fwd<T, __nv_bfloat16>(p, grid, st);
}

template <typename T>
static void launch_bwd_x(const NormDev& p, int out_dtype, cudaStream_t st) {
    if (out_dtype == SWX_DTYPE_F32) launch_bwd<T, float>(p, st);
    else launch_bwd<T, __nv_bfloat16>(p, st);
}

}  // namespace swx

namespace {
int norm_check(const swx_rmsnorm_args* a, bool bwd) {
    if (!a) return SWX_ERR_INVALID_ARG;
    if (a->rows < 0 || a->dim < 0) return SWX_ERR_INVALID_ARG;
    if (a->dtype != SWX_DTYPE_F32 && a->dtype != SWX_DTYPE_BF16) return SWX_ERR_UNSUPPORTED;
    if (a->out_dtype != SWX_DTYPE_F32 && a->out_dtype != SWX_DTYPE_BF16) return SWX_ERR_UNSUPPORTED;
    if (a->rows > INT32_MAX || a->dim > 32 * swx::NORM_MAXC) return SWX_ERR_UNSUPPORTED;
    const bool res_form = bwd ? a->dres != nullptr : a->residual != nullptr;
    if (res_form && a->res_dtype != SWX_DTYPE_F32 && a->res_dtype != SWX_DTYPE_BF16) return SWX_ERR_UNSUPPORTED;
    if (a->rows * a->dim == 0) return SWX_OK;
    if (!a->x || !a->weight) return SWX_ERR_INVALID_ARG;
    if (!bwd && !a->y) return SWX_ERR_INVALID_ARG;
    if (!bwd && a->residual && !a->sum) return SWX_ERR_INVALID_ARG;
    if (bwd && (!a->dy || !a->dx || !a->dweight || !a->rstd || !a->workspace)) return SWX_ERR_INVALID_ARG;
    return SWX_OK;
}

swx::NormDev norm_pack(const swx_rmsnorm_args* a) {
    swx::NormDev p{};
    p.rows = (int)a->rows; p.d = (int)a->dim; p.eps = a->eps;
    p.x = a->x; p.w = a->weight; p.y = a->y; p.rstd = a->rstd;
    p.dy = a->dy; p.dx = a->dx; p.dw_part = static_cast<float*>(a->workspace); p.dw = a->dweight;
    p.res = a->residual; p.sum = a->sum; p.dsum = a->dsum; p.dres = a->dres;
    p.res_bf16 = a->res_dtype == SWX_DTYPE_BF16 ? 1 : 0;
    return p;
}
}  // namespace

extern "C" {

int64_t swx_rmsnorm_args_size(void) { return (int64_t)sizeof(swx_rmsnorm_args); }

int64_t swx_rmsnorm_bwd_workspace_bytes(int64_t dim) { return (int64_t)swx::NORM_BWD_CTAS * dim * 4; }

int swx_rmsnorm_fwd(const swx_rmsnorm_args* a, void* stream) {
    const int s = norm_check(a, false);
    if (s != SWX_OK || a->rows * a->dim == 0) return s;
    const swx::NormDev p = norm_pack(a);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const unsigned grid = (unsigned)((p.rows + swx::NORM_WARPS - 1) / swx::NORM_WARPS);
    if (a->dtype == SWX_DTYPE_F32) swx::launch_fwd_x<float>(p, a->out_dtype, grid, st);
    else swx::launch_fwd_x<__nv_bfloat16>(p, a->out_dtype, grid, st);
    return cudaGetLastError() == cudaSuccess ? SWX_OK : SWX_ERR_CUDA;
}

int swx_rmsnorm_bwd(const swx_rmsnorm_args* a, void* stream) {
    const int s = norm_check(a, true);
    if (s != SWX_OK) return s;
    if (a->rows * a->dim == 0) {          // no row contributes: the weight gradient is zero
        if (a->dweight && a->dim > 0)
            return cudaMemsetAsync(a->dweight, 0, a->dim * 4, static_cast<cudaStream_t>(stream)) == cudaSuccess
                       ? SWX_OK : SWX_ERR_CUDA;
        return SWX_OK;
    }
    if (a->workspace_bytes < swx_rmsnorm_bwd_workspace_bytes(a->dim)) return SWX_ERR_INVALID_ARG;
    const swx::NormDev p = norm_pack(a);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (a->dtype == SWX_DTYPE_F32) swx::launch_bwd_x<float>(p, a->out_dtype, st);
    else swx::launch_bwd_x<__nv_bfloat16>(p, a->out_dtype, st);
    return cudaGetLastError() == cudaSuccess ? SWX_OK : SWX_ERR_CUDA;
}

}  // extern "C"
