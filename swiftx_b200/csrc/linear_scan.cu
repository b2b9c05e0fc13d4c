// Linear recurrence h_t = a_t * h_{t-1} + x_t along the sequence for sm_100a -- the
// reference's parallel_scan / sequential_scan (models/selective_scan.py:66-99) -- and its
// adjoint.  The reference materialises (b, L, D, N) tensors for this (537 MB each at
// b=8, L=2048, D=512, N=16), so the op is a pure HBM stream: read a and x, write h.
//
// Thread = one (batch row, element) chain, adjacent threads adjacent elements, so every
// step is one coalesced row access per warp; the loads of LS_U consecutive steps are
// issued before their (serially dependent) updates, so a thread keeps 2*LS_U loads in
// flight.  Each update is one fused multiply-add.
#include "common.cuh"

namespace swx {

struct LsDev {
    int b, L;
    int64_t W;
    const void* a; int64_t a_sb, a_sl;
    const void* x; int64_t x_sb, x_sl;
    void* h;
    const void* dh; int64_t dh_sb, dh_sl;
    void* da; void* dx;
};

constexpr int LS_NT = 128;
constexpr int LS_U = 16;

template <typename T>
__global__ void __launch_bounds__(LS_NT) linear_scan_fwd_kernel(const LsDev p) {
    const int64_t m = (int64_t)blockIdx.x * LS_NT + threadIdx.x;
    if (m >= p.W) return;
    const int bi = blockIdx.y;
    const T* __restrict__ a = static_cast<const T*>(p.a) + bi * p.a_sb + m;
    const T* __restrict__ x = static_cast<const T*>(p.x) + bi * p.x_sb + m;
    T* __restrict__ h = static_cast<T*>(p.h) + (int64_t)bi * p.L * p.W + m;
    T acc = T(0);
    int t = 0;
    for (; t + LS_U <= p.L; t += LS_U) {
        T av[LS_U], xv[LS_U];
#pragma unroll
        for (int u = 0; u < LS_U; ++u) {
            av[u] = a[(int64_t)(t + u) * p.a_sl];
            xv[u] = x[(int64_t)(t + u) * p.x_sl];
        }
#pragma unroll
        for (int u = 0; u < LS_U; ++u) {
            acc = fma(av[u], acc, xv[u]);
            h[(int64_t)(t + u) * p.W] = acc;
        }
    }
    for (; t < p.L; ++t) {
        acc = fma(a[(int64_t)t * p.a_sl], acc, x[(int64_t)t * p.x_sl]);
        h[(int64_t)t * p.W] = acc;
    }
}

// g_t = dh_t + a_{t+1} g_{t+1}, walked from the last step; dx_t = g_t, da_t = g_t h_{t-1}.
template <typename T>
__global__ void __launch_bounds__(LS_NT) linear_scan_bwd_kernel(const LsDev p) {
    const int64_t m = (int64_t)blockIdx.x * LS_NT + threadIdx.x;
    if (m >= p.W) return;
    const int bi = blockIdx.y;
    const T* __restrict__ a = static_cast<const T*>(p.a) + bi * p.a_sb + m;
    const T* __restrict__ dh = static_cast<const T*>(p.dh) + bi * p.dh_sb + m;
    const int64_t row = (int64_t)bi * p.L * p.W + m;
    const T* __restrict__ h = static_cast<const T*>(p.h) + row;
    T* __restrict__ da = static_cast<T*>(p.da) + row;
    T* __restrict__ dx = static_cast<T*>(p.dx) + row;
    T g = T(0), an = T(0);                 // an = a_{t+1} (0 past the end)
    int t = p.L - 1;
    for (; t - LS_U + 1 >= 0; t -= LS_U) {
        T dv[LS_U], av[LS_U], hp[LS_U];
#pragma unroll
        for (int u = 0; u < LS_U; ++u) {
            const int s = t - u;
            dv[u] = dh[(int64_t)s * p.dh_sl];
            av[u] = a[(int64_t)s * p.a_sl];
            hp[u] = s > 0 ? h[(int64_t)(s - 1) * p.W] : T(0);
        }
#pragma unroll
        for (int u = 0; u < LS_U; ++u) {
            const int s = t - u;
            g = fma(an, g, dv[u]);
            dx[(int64_t)s * p.W] = g;
            da[(int64_t)s * p.W] = g * hp[u];
            an = av[u];
        }
    }
    for (; t >= 0; --t) {
        g = fma(an, g, dh[(int64_t)t * p.dh_sl]);
        dx[(int64_t)t * p.W] = g;
        da[(int64_t)t * p.W] = g * (t > 0 ? h[(int64_t)(t - 1) * p.W] : T(0));
        an = a[(int64_t)t * p.a_sl];
    }
}

}  // namespace swx

namespace {
int ls_check(const swx_linear_scan_args* s, bool bwd) {
    if (!s) return SWX_ERR_INVALID_ARG;
    if (s->batch < 0 || s->seqlen < 0 || s->width < 0) return SWX_ERR_INVALID_ARG;
    if (s->dtype != SWX_DTYPE_F32 && s->dtype != SWX_DTYPE_F64) return SWX_ERR_UNSUPPORTED;
    if (s->batch > 65535 || s->seqlen > INT32_MAX) return SWX_ERR_UNSUPPORTED;
    if (s->batch * s->seqlen * s->width == 0) return SWX_OK;
    if (!s->a || !s->h) return SWX_ERR_INVALID_ARG;
    if (!bwd && !s->x) return SWX_ERR_INVALID_ARG;
    if (bwd && (!s->dh || !s->da || !s->dx)) return SWX_ERR_INVALID_ARG;
    return SWX_OK;
}

swx::LsDev ls_pack(const swx_linear_scan_args* s) {
    swx::LsDev p{};
    p.b = (int)s->batch; p.L = (int)s->seqlen; p.W = s->width;
    p.a = s->a; p.a_sb = s->a_sb; p.a_sl = s->a_sl;
    p.x = s->x; p.x_sb = s->x_sb; p.x_sl = s->x_sl;
    p.h = s->h;
    p.dh = s->dh; p.dh_sb = s->dh_sb; p.dh_sl = s->dh_sl;
    p.da = s->da; p.dx = s->dx;
    return p;
}
}  // namespace

extern "C" {

int64_t swx_linear_scan_args_size(void) { return (int64_t)sizeof(swx_linear_scan_args); }

int swx_linear_scan_fwd(const swx_linear_scan_args* s, void* stream) {
    const int st = ls_check(s, false);
    if (st != SWX_OK || s->batch * s->seqlen * s->width == 0) return st;
    const swx::LsDev p = ls_pack(s);
    const dim3 grid((unsigned)((p.W + swx::LS_NT - 1) / swx::LS_NT), p.b);
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    if (s->dtype == SWX_DTYPE_F32) swx::linear_scan_fwd_kernel<float><<<grid, swx::LS_NT, 0, cs>>>(p);
    else swx::linear_scan_fwd_kernel<double><<<grid, swx::LS_NT, 0, cs>>>(p);
    return cudaGetLastError() == cudaSuccess ? SWX_OK : SWX_ERR_CUDA;
}

int swx_linear_scan_bwd(const swx_linear_scan_args* s, void* stream) {
    const int st = ls_check(s, true);
    if (st != SWX_OK || s->batch * s->seqlen * s->width == 0) return st;
    const swx::LsDev p = ls_pack(s);
    const dim3 grid((unsigned)((p.W + swx::LS_NT - 1) / swx::LS_NT), p.b);
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    if (s->dtype == SWX_DTYPE_F32) swx::linear_scan_bwd_kernel<float><<<grid, swx::LS_NT, 0, cs>>>(p);
    else swx::linear_scan_bwd_kernel<double><<<grid, swx::LS_NT, 0, cs>>>(p);
    return cudaGetLastError() == cudaSuccess ? SWX_OK : SWX_ERR_CUDA;
}

}  // extern "C"
