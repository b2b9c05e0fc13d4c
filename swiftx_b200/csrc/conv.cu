// Causal depthwise conv1d (+ SiLU) forward / backward for sm_100a.
//
// out[b,t,d] = silu(bias[d] + sum_{k<K} w[d,k] * x[b, t-(K-1)+k, d]),  x[s<0] = 0
// (nn.Conv1d(D, D, K, groups=D, padding=K-1) keeping the first L outputs, then SiLU:
// models/sift_block.py:62-65,117-118).
//
// The op is HBM-bound (K=4 multiply-adds per element), so the layout is chosen for
// coalescing: a thread owns one channel and a tile of consecutive steps, a warp covers
// 32 adjacent channels (128 contiguous bytes per step for fp32), and the K-1 step halo is
// kept in registers as a sliding window.  x may be the strided x half of the in_proj
// output (row stride 2D); no copy is made.
//
// Backward recomputes the pre-activation from x, so nothing but the inputs is saved.
// dw and dbias are per-(batch row, step tile) partials summed in fixed order by a
// second kernel (deterministic, no float atomics).
#include "common.cuh"

namespace swx {

constexpr int CONV_MAXK = 6;
constexpr int CONV_TT = 16;       // steps per thread (short tiles: more threads in flight)
constexpr int CONV_NT = 128;      // threads (channels) per CTA

struct ConvDev {
    int b, L, D, K, silu;
    const void* x; int64_t x_sb, x_sl;
    const float* w; const float* bias;
    void* out;
    const void* dout; int64_t do_sb, do_sl;
    void* dx; float* dw; float* dbias;
    int64_t dx_sb, dx_sl;   // element strides of dx (dense: L*D, D)
    float* ws;        // (b, ntiles, D, K+1) partials of dw | dbias
    int ntiles;
};

template <typename T, int K>
__global__ void __launch_bounds__(CONV_NT) conv_fwd_kernel(const ConvDev p) {
    const int d = blockIdx.x * CONV_NT + threadIdx.x;
    const int t0 = blockIdx.y * CONV_TT;
    const int bi = blockIdx.z;
    if (d >= p.D) return;
    const T* x = static_cast<const T*>(p.x) + bi * p.x_sb + d;
    T* out = static_cast<T*>(p.out) + (int64_t)bi * p.L * p.D + d;
    float w[K], win[K];
#pragma unroll
    for (int k = 0; k < K; ++k) w[k] = p.w[(int64_t)d * K + k];
    const float bias = p.bias ? p.bias[d] : 0.f;
    // window slot k holds x[t-(K-1)+k]; prime it with the K-1 steps before the tile
#pragma unroll
    for (int k = 0; k < K - 1; ++k) {
        const int s = t0 - (K - 1) + k;
        win[k] = s >= 0 ? Elem<T>::to_f(x[(int64_t)s * p.x_sl]) : 0.f;
    }
    const int tend = min(t0 + CONV_TT, p.L);
    for (int t = t0; t < tend; ++t) {
        win[K - 1] = Elem<T>::to_f(x[(int64_t)t * p.x_sl]);
        float acc = bias;
#pragma unroll
        for (int k = 0; k < K; ++k) acc = fmaf(w[k], win[k], acc);
        out[(int64_t)t * p.D] = Elem<T>::from_f(p.silu ? silu_f(acc) : acc);
#pragma unroll
        for (int k = 0; k < K - 1; ++k) win[k] = win[k + 1];
    }
}

template <typename T, int K>
__global__ void __launch_bounds__(CONV_NT) conv_bwd_kernel(const ConvDev p) {
    const int d = blockIdx.x * CONV_NT + threadIdx.x;
    const int tile = blockIdx.y;
    const int t0 = tile * CONV_TT;
    const int bi = blockIdx.z;
    if (d >= p.D) return;
    const T* x = static_cast<const T*>(p.x) + bi * p.x_sb + d;
    const T* dout = static_cast<const T*>(p.dout) + bi * p.do_sb + d;
    T* dx = static_cast<T*>(p.dx) + (int64_t)bi * p.dx_sb + d;
    float w[K];
#pragma unroll
    for (int k = 0; k < K; ++k) w[k] = p.w[(int64_t)d * K + k];
    const float bias = p.bias ? p.bias[d] : 0.f;

    // xw[k] = x[s-(K-1)+k] for the current step s; gq[k] = dL/dpre at step s-(K-1)+k
    float xw[K], gq[K], dwacc[K];
    float dbacc = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) { dwacc[k] = 0.f; gq[k] = 0.f; }
#pragma unroll
    for (int k = 0; k < K - 1; ++k) {
        const int s = t0 - (K - 1) + k;
        xw[k] = s >= 0 ? Elem<T>::to_f(x[(int64_t)s * p.x_sl]) : 0.f;
    }
    // dx[t] = sum_k w[k] * gp(t + K-1-k): walk s over the tile plus a K-1 step halo
    const int tend = min(t0 + CONV_TT, p.L);
    const int send = min(tend + K - 1, p.L);
    for (int s = t0; s < send; ++s) {
        xw[K - 1] = Elem<T>::to_f(x[(int64_t)s * p.x_sl]);
        float acc = bias;
#pragma unroll
        for (int k = 0; k < K; ++k) acc = fmaf(w[k], xw[k], acc);
        float g = Elem<T>::to_f(dout[(int64_t)s * p.do_sl]);
        if (p.silu) {
            const float sg = sigmoid_f(acc);
            g *= sg * fmaf(acc, 1.f - sg, 1.f);
        }
        if (s < tend) {                 // dw, dbias partials of the steps this tile owns
            dbacc += g;
#pragma unroll
            for (int k = 0; k < K; ++k) dwacc[k] = fmaf(g, xw[k], dwacc[k]);
        }
#pragma unroll
        for (int k = 0; k < K - 1; ++k) gq[k] = gq[k + 1];
        gq[K - 1] = g;                  // gq holds gp(s-K+1 .. s)
        const int t = s - (K - 1);
        if (t >= t0) {
            float a = 0.f;
#pragma unroll
            for (int k = 0; k < K; ++k) a = fmaf(w[k], gq[K - 1 - k], a);
            dx[(int64_t)t * p.dx_sl] = Elem<T>::from_f(a);
        }
#pragma unroll
        for (int k = 0; k < K - 1; ++k) xw[k] = xw[k + 1];
    }
    // steps whose window reaches past the end of the sequence see gp = 0 there
    for (int t = send - (K - 1); t < tend; ++t) {
#pragma unroll
        for (int k = 0; k < K - 1; ++k) gq[k] = gq[k + 1];
        gq[K - 1] = 0.f;
        if (t >= t0) {
            float a = 0.f;
#pragma unroll
            for (int k = 0; k < K; ++k) a = fmaf(w[k], gq[K - 1 - k], a);
            dx[(int64_t)t * p.dx_sl] = Elem<T>::from_f(a);
        }
    }
    float* ws = p.ws + (((int64_t)bi * p.ntiles + tile) * p.D + d) * (K + 1);
#pragma unroll
    for (int k = 0; k < K; ++k) ws[k] = dwacc[k];
    ws[K] = dbacc;
}

// ---------------------------------------------------------------- 4-channel forward
// Four adjacent channels per thread: 8-byte (bf16) or 16-byte (fp32) loads and stores, so
// a warp moves 128 channels of a row per access; adjacent threads take adjacent channel
// groups of the same (row, tile), and a complete tile's 16 rows are loaded before the
// math.  Used when D and the row strides are multiples of 4 and the pointers are aligned;
// per channel the arithmetic is conv_fwd_kernel's, in the same order (identical results).
// (The backward stays one channel per thread: its per-step loads sit on a dependency
// chain and need the 4x larger thread count to hide their latency.)
constexpr int CV = 4;

template <typename T> struct Vec4;
template <> struct Vec4<float> {
    static __device__ __forceinline__ void load(const float* __restrict__ q, float (&v)[CV]) {
        const float4 a = *reinterpret_cast<const float4*>(q);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    }
    static __device__ __forceinline__ void store(float* __restrict__ q, const float (&v)[CV]) {
        *reinterpret_cast<float4*>(q) = make_float4(v[0], v[1], v[2], v[3]);
    }
};
template <> struct Vec4<__nv_bfloat16> {
    static __device__ __forceinline__ void load(const __nv_bfloat16* __restrict__ q, float (&v)[CV]) {
        const uint2 a = *reinterpret_cast<const uint2*>(q);
        const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a.x));
        const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a.y));
        v[0] = lo.x; v[1] = lo.y; v[2] = hi.x; v[3] = hi.y;
    }
    static __device__ __forceinline__ void store(__nv_bfloat16* __restrict__ q, const float (&v)[CV]) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(v[0], v[1]), hi = __floats2bfloat162_rn(v[2], v[3]);
        uint2 a;
        a.x = *reinterpret_cast<uint32_t*>(&lo);
        a.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(q) = a;
    }
};

// (row, tile, channel group) of this thread; false past the end of the grid
__device__ __forceinline__ bool conv_vec_coords(const ConvDev& p, int& bi, int& tile, int& d) {
    const int Dv = p.D / CV;
    const int64_t gid = (int64_t)blockIdx.x * CONV_NT + threadIdx.x;
    if (gid >= (int64_t)p.b * p.ntiles * Dv) return false;
    d = (int)(gid % Dv) * CV;
    const int64_t rest = gid / Dv;
    tile = (int)(rest % p.ntiles);
    bi = (int)(rest / p.ntiles);
    return true;
}

template <typename T, int K>
__global__ void __launch_bounds__(CONV_NT) conv_fwd_vec_kernel(const ConvDev p) {
    int bi, tile, d;
    if (!conv_vec_coords(p, bi, tile, d)) return;
    const int t0 = tile * CONV_TT;
    const T* __restrict__ x = static_cast<const T*>(p.x) + bi * p.x_sb + d;
    T* __restrict__ out = static_cast<T*>(p.out) + (int64_t)bi * p.L * p.D + d;
    float w[CV][K], bias[CV], win[CV][K];
#pragma unroll
    for (int c = 0; c < CV; ++c) {
#pragma unroll
        for (int k = 0; k < K; ++k) w[c][k] = p.w[(int64_t)(d + c) * K + k];
        bias[c] = p.bias ? p.bias[d + c] : 0.f;
    }
#pragma unroll
    for (int k = 0; k < K - 1; ++k) {
        const int s = t0 - (K - 1) + k;
        float v[CV] = {0.f, 0.f, 0.f, 0.f};
        if (s >= 0) Vec4<T>::load(x + (int64_t)s * p.x_sl, v);
#pragma unroll
        for (int c = 0; c < CV; ++c) win[c][k] = v[c];
    }
    auto step = [&](int t, const float (&v)[CV]) {
        float o[CV];
#pragma unroll
        for (int c = 0; c < CV; ++c) {
            win[c][K - 1] = v[c];
            float acc = bias[c];
#pragma unroll
            for (int k = 0; k < K; ++k) acc = fmaf(w[c][k], win[c][k], acc);
            o[c] = p.silu ? silu_f(acc) : acc;
#pragma unroll
            for (int k = 0; k < K - 1; ++k) win[c][k] = win[c][k + 1];
        }
        Vec4<T>::store(out + (int64_t)t * p.D, o);
    };
    if (t0 + CONV_TT <= p.L) {
        float v[CONV_TT][CV];
#pragma unroll
        for (int tt = 0; tt < CONV_TT; ++tt) Vec4<T>::load(x + (int64_t)(t0 + tt) * p.x_sl, v[tt]);
#pragma unroll
        for (int tt = 0; tt < CONV_TT; ++tt) step(t0 + tt, v[tt]);
    } else {
        for (int t = t0; t < p.L; ++t) {
            float v[CV];
            Vec4<T>::load(x + (int64_t)t * p.x_sl, v);
            step(t, v);
        }
    }
}

// Fixed-order column sums of the (row, tile) partials ws[(bi * ntiles + tl)][d][k]:
// one block per 32 consecutive (d, k) columns; warp w adds rows w, w+32, ... (lanes read
// 32 adjacent columns of a row: one 128-byte load), then the 32 warp sums of a column are
// added in warp order.
constexpr int FIN_WARPS = 32;
__global__ void __launch_bounds__(32 * FIN_WARPS) conv_bwd_finalize_kernel(const ConvDev p) {
    __shared__ float part[FIN_WARPS][33];
    const int K1 = p.K + 1;
    const int W = p.D * K1;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int col = blockIdx.x * 32 + lane;
    const int rows = p.b * p.ntiles;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    if (col < W) {
        int r = w;
        for (; r + 3 * FIN_WARPS < rows; r += 4 * FIN_WARPS) {
            a0 += p.ws[(int64_t)r * W + col];
            a1 += p.ws[(int64_t)(r + FIN_WARPS) * W + col];
            a2 += p.ws[(int64_t)(r + 2 * FIN_WARPS) * W + col];
            a3 += p.ws[(int64_t)(r + 3 * FIN_WARPS) * W + col];
        }
        for (; r < rows; r += FIN_WARPS) a0 += p.ws[(int64_t)r * W + col];
    }
    part[w][lane] = (a0 + a1) + (a2 + a3);
    __syncthreads();
    if (w == 0 && col < W) {
        float s = 0.f;
#pragma unroll 8
        for (int i = 0; i < FIN_WARPS; ++i) s += part[i][lane];
        const int d = col / K1, k = col % K1;
        if (k < p.K) p.dw[(int64_t)d * p.K + k] = s;
        else if (p.dbias) p.dbias[d] = s;
    }
}

// The 4-channel forward needs every row of x and out to start on a 4-element boundary of
// an aligned pointer (8 bytes for bf16, 16 for fp32).
static bool conv_vec_ok(const ConvDev& p, int es) {
    auto al = [es](const void* q) { return (reinterpret_cast<uintptr_t>(q) % (CV * es)) == 0; };
    return p.D % CV == 0 && p.x_sb % CV == 0 && p.x_sl % CV == 0 && al(p.x) && al(p.out);
}

template <typename T, int K>
static void launch_k(const ConvDev& p, dim3 grid, cudaStream_t st, bool bwd) {
    if (!bwd && conv_vec_ok(p, sizeof(T))) {
        const int64_t n = (int64_t)p.b * p.ntiles * (p.D / CV);
        conv_fwd_vec_kernel<T, K><<<(unsigned)((n + CONV_NT - 1) / CONV_NT), CONV_NT, 0, st>>>(p);
        return;
    }
    if (bwd) conv_bwd_kernel<T, K><<<grid, CONV_NT, 0, st>>>(p);
    else conv_fwd_kernel<T, K><<<grid, CONV_NT, 0, st>>>(p);
}

template <typename T>
static void dispatch_k(const ConvDev& p, dim3 grid, cudaStream_t st, bool bwd) {
    switch (p.K) {
        case 1: launch_k<T, 1>(p, grid, st, bwd); break;
        case 2: launch_k<T, 2>(p, grid, st, bwd); break;
        case 3: launch_k<T, 3>(p, grid, st, bwd); break;
        case 4: launch_k<T, 4>(p, grid, st, bwd); break;
        case 5: launch_k<T, 5>(p, grid, st, bwd); break;
        default: launch_k<T, 6>(p, grid, st, bwd); break;
    }
}

}  // namespace swx

// ----------------------------------------------------------------- C ABI
namespace {
int conv_es(int dt) { return dt == SWX_DTYPE_F32 ? 4 : (dt == SWX_DTYPE_BF16 ? 2 : 0); }

int conv_check(const swx_conv_args* a) {
    if (!a) return SWX_ERR_INVALID_ARG;
    if (a->batch < 0 || a->seqlen < 0 || a->dim < 0) return SWX_ERR_INVALID_ARG;
    if (a->width < 1 || a->width > swx::CONV_MAXK) return SWX_ERR_UNSUPPORTED;
    if (conv_es(a->dtype) == 0) return SWX_ERR_UNSUPPORTED;
    // batch rows and time tiles index the grid's z and y dimensions (at most 65535 each)
    if (a->batch > 65535 || (a->seqlen + swx::CONV_TT - 1) / swx::CONV_TT > 65535 || a->dim > INT32_MAX)
        return SWX_ERR_UNSUPPORTED;
    if (a->batch * a->seqlen * a->dim == 0) return SWX_OK;
    if (!a->x || !a->weight) return SWX_ERR_INVALID_ARG;
    return SWX_OK;
}

swx::ConvDev conv_pack(const swx_conv_args* a) {
    swx::ConvDev p{};
    p.b = (int)a->batch; p.L = (int)a->seqlen; p.D = (int)a->dim; p.K = (int)a->width;
    p.silu = a->silu ? 1 : 0;
    p.x = a->x; p.x_sb = a->x_sb; p.x_sl = a->x_sl;
    p.w = a->weight; p.bias = a->bias;
    p.out = a->out;
    p.dout = a->dout; p.do_sb = a->dout_sb; p.do_sl = a->dout_sl;
    p.dx = a->dx; p.dw = a->dweight; p.dbias = a->dbias;
    p.dx_sl = a->dx_sl ? a->dx_sl : a->dim;
    p.dx_sb = a->dx_sb ? a->dx_sb : a->seqlen * p.dx_sl;
    p.ntiles = (int)((a->seqlen + swx::CONV_TT - 1) / swx::CONV_TT);
    return p;
}
}  // namespace

extern "C" {

int64_t swx_conv1d_bwd_workspace_bytes(int64_t batch, int64_t seqlen, int64_t dim, int64_t width) {
    const int64_t ntiles = (seqlen + swx::CONV_TT - 1) / swx::CONV_TT;
    return batch * ntiles * dim * (width + 1) * 4;
}

int swx_conv1d_fwd(const swx_conv_args* a, void* stream) {
    int s = conv_check(a);
    if (s != SWX_OK || a->batch * a->seqlen * a->dim == 0) return s;
    if (!a->out) return SWX_ERR_INVALID_ARG;
    swx::ConvDev p = conv_pack(a);
    dim3 grid((p.D + swx::CONV_NT - 1) / swx::CONV_NT, p.ntiles, p.b);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (a->dtype == SWX_DTYPE_F32) swx::dispatch_k<float>(p, grid, st, false);
    else swx::dispatch_k<__nv_bfloat16>(p, grid, st, false);
    return cudaGetLastError() == cudaSuccess ? SWX_OK : SWX_ERR_CUDA;
}

int swx_conv1d_bwd(const swx_conv_args* a, void* stream) {
    int s = conv_check(a);
    if (s != SWX_OK) return s;
    if (a->batch * a->seqlen * a->dim == 0) {
        // no step contributes: the weight and bias gradients are zero
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        cudaError_t e = cudaSuccess;
        if (a->dweight && a->dim * a->width > 0) e = cudaMemsetAsync(a->dweight, 0, a->dim * a->width * 4, st);
        if (e == cudaSuccess && a->dbias && a->dim > 0) e = cudaMemsetAsync(a->dbias, 0, a->dim * 4, st);
        return e == cudaSuccess ? SWX_OK : SWX_ERR_CUDA;
    }
    if (!a->dout || !a->dx || !a->dweight || !a->workspace) return SWX_ERR_INVALID_ARG;
    if ((a->dx_sb != 0) != (a->dx_sl != 0)) return SWX_ERR_INVALID_ARG;
    if (a->dx_sl && (a->dx_sl < a->dim || a->dx_sb < a->seqlen * a->dx_sl)) return SWX_ERR_INVALID_ARG;
    if (a->workspace_bytes < swx_conv1d_bwd_workspace_bytes(a->batch, a->seqlen, a->dim, a->width))
        return SWX_ERR_INVALID_ARG;
    swx::ConvDev p = conv_pack(a);
    p.ws = static_cast<float*>(a->workspace);
    dim3 grid((p.D + swx::CONV_NT - 1) / swx::CONV_NT, p.ntiles, p.b);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (a->dtype == SWX_DTYPE_F32) swx::dispatch_k<float>(p, grid, st, true);
    else swx::dispatch_k<__nv_bfloat16>(p, grid, st, true);
    if (cudaGetLastError() != cudaSuccess) return SWX_ERR_CUDA;
    const int n = p.D * (p.K + 1);
    swx::conv_bwd_finalize_kernel<<<(n + 31) / 32, 32 * swx::FIN_WARPS, 0, st>>>(p);
    return cudaGetLastError() == cudaSuccess ? SWX_OK : SWX_ERR_CUDA;
}

}  // extern "C"
