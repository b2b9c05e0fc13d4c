// Single-token recurrent step (generation) for sm_100a, following SiftBlock.step
// (models/sift_block.py:153-175):
//   conv_state <- roll left, append x ;  xc = silu(<conv_state, w> + conv_bias)
//   delta = softplus(delta_raw + delta_bias) ;  h <- exp(delta*A) * h + delta * B * xc
//   y = <h, C> + Dskip * xc ;  out = y * silu(z)
// The state is updated in place.  In the model, x_proj / dt_proj (small GEMVs on cuBLAS)
// sit between the conv and the state update, so the step can run as two launches
// (SWX_DECODE_CONV, then SWX_DECODE_SSM); with delta/B/C given it is one fused launch.
//
// HBM-bound: per (row, channel) the state (N floats) is read and written once, the conv
// window once, and the per-token vectors once.  Four adjacent lanes own the 16 states of
// a channel (one 16-byte load/store each, fully coalesced across the warp); the readout
// is reduced over the 4 lanes with two xor-shuffles.
#include "common.cuh"

namespace swx {

struct DecDev {
    int b, D, N, K, softplus, mode;
    const float* x; int64_t x_sb;
    const float* z; int64_t z_sb;
    const float* dl; int64_t dl_sb;
    const float* B; int64_t B_sb;
    const float* C; int64_t C_sb;
    const float* cw; const float* cb;
    const float* A; const float* Dskip; const float* dbias;
    float* conv_state; float* ssm_state; float* xc_out; float* out;
};

constexpr int DEC_NT = 256;

template <int K, bool HAS_Z>
__global__ void __launch_bounds__(DEC_NT) decode_kernel(const DecDev p) {
    const int64_t gid = (int64_t)blockIdx.x * DEC_NT + threadIdx.x;
    const int j = (int)(gid & 3);
    const int64_t total = (int64_t)p.b * p.D;
    const int64_t bd = gid >> 2;
    const bool valid = bd < total;
    const int64_t bdc = valid ? bd : 0;
    const int bi = (int)(bdc / p.D), d = (int)(bdc % p.D);

    float xc;
    if (p.mode & SWX_DECODE_CONV) {
        const float xin = p.x[bi * p.x_sb + d];
        float win[K];
        const float* cs = p.conv_state + bdc * K;
#pragma unroll
        for (int k = 0; k < K - 1; ++k) win[k] = cs[k + 1];
        win[K - 1] = xin;
        float acc = p.cb ? p.cb[d] : 0.f;
#pragma unroll
        for (int k = 0; k < K; ++k) acc = fmaf(win[k], p.cw[(int64_t)d * K + k], acc);
        xc = silu_f(acc);
        if (valid && j == 0) {
            float* csw = p.conv_state + bdc * K;
#pragma unroll
            for (int k = 0; k < K; ++k) csw[k] = win[k];
            if (p.xc_out) p.xc_out[bdc] = xc;
        }
    } else {
        xc = p.x[bi * p.x_sb + d];
    }
    if (!(p.mode & SWX_DECODE_SSM)) return;

    const float raw = p.dl[bi * p.dl_sb + d] + (p.dbias ? p.dbias[d] : 0.f);
    float dte = raw;
    if (p.softplus) {
        float2 sp, dsp;
        softplus2(bc2(raw), sp, dsp);
        dte = sp.x;
    }
    const float dxc = dte * xc;
    float* hp = p.ssm_state + bdc * p.N;
    float y = 0.f;
    if (p.N == NS) {
        const float4 h4 = *reinterpret_cast<const float4*>(hp + 4 * j);
        const float4 a4 = *reinterpret_cast<const float4*>(p.A + (int64_t)d * NS + 4 * j);
        const float4 b4 = *reinterpret_cast<const float4*>(p.B + bi * p.B_sb + 4 * j);
        const float4 c4 = *reinterpret_cast<const float4*>(p.C + bi * p.C_sb + 4 * j);
        const float2 dt = bc2(dte * LOG2E), dx = bc2(dxc);
        float2 h01 = fma2(ex2x2(mul2(dt, f2(a4.x, a4.y))), f2(h4.x, h4.y), mul2(dx, f2(b4.x, b4.y)));
        float2 h23 = fma2(ex2x2(mul2(dt, f2(a4.z, a4.w))), f2(h4.z, h4.w), mul2(dx, f2(b4.z, b4.w)));
        float2 yy = mul2(h01, f2(c4.x, c4.y));
        yy = fma2(h23, f2(c4.z, c4.w), yy);
        y = yy.x + yy.y;
        if (valid) *reinterpret_cast<float4*>(hp + 4 * j) = make_float4(h01.x, h01.y, h23.x, h23.y);
    } else {
        for (int i = 0; i < 4; ++i) {
            const int n = 4 * j + i;
            if (n < p.N) {
                const float h = fmaf(ex2(dte * p.A[(int64_t)d * p.N + n] * LOG2E), hp[n], dxc * p.B[bi * p.B_sb + n]);
                y = fmaf(h, p.C[bi * p.C_sb + n], y);
                if (valid) hp[n] = h;
            }
        }
    }
    y += __shfl_xor_sync(0xffffffffu, y, 1);
    y += __shfl_xor_sync(0xffffffffu, y, 2);
    if (valid && j == 0) {
        y = fmaf(p.Dskip ? p.Dskip[d] : 0.f, xc, y);
        if (HAS_Z) y *= silu_f(p.z[bi * p.z_sb + d]);
        p.out[bdc] = y;
    }
}

template <int K>
static void launch_dec(const DecDev& p, cudaStream_t st) {
    const int64_t threads = (int64_t)p.b * p.D * 4;
    const int blocks = (int)((threads + DEC_NT - 1) / DEC_NT);
    if (p.z) decode_kernel<K, true><<<blocks, DEC_NT, 0, st>>>(p);
    else decode_kernel<K, false><<<blocks, DEC_NT, 0, st>>>(p);
}

}  // namespace swx

extern "C" int swx_decode_step(const swx_decode_args* a, void* stream) {
    if (!a) return SWX_ERR_INVALID_ARG;
    if (a->batch < 0 || a->dim < 0) return SWX_ERR_INVALID_ARG;
    if (a->mode < 1 || a->mode > 3) return SWX_ERR_INVALID_ARG;
    if ((a->mode & SWX_DECODE_CONV) && (a->width < 1 || a->width > 6)) return SWX_ERR_UNSUPPORTED;
    if ((a->mode & SWX_DECODE_SSM) && (a->dstate < 1 || a->dstate > swx::NS)) return SWX_ERR_UNSUPPORTED;
    if (a->batch * a->dim == 0) return SWX_OK;
    if (a->batch * a->dim * 4 > (int64_t)INT32_MAX * 256) return SWX_ERR_UNSUPPORTED;
    if (!a->x) return SWX_ERR_INVALID_ARG;
    if ((a->mode & SWX_DECODE_CONV) && (!a->conv_weight || !a->conv_state)) return SWX_ERR_INVALID_ARG;
    if ((a->mode & SWX_DECODE_SSM) && (!a->delta || !a->B || !a->C || !a->A || !a->ssm_state || !a->out))
        return SWX_ERR_INVALID_ARG;
    if ((a->mode & SWX_DECODE_SSM) && a->dstate == swx::NS &&
        (((uintptr_t)a->ssm_state | (uintptr_t)a->A | (uintptr_t)a->B | (uintptr_t)a->C) & 15u ||
         (a->B_sb % 4) || (a->C_sb % 4)))
        return SWX_ERR_INVALID_ARG;
    swx::DecDev p{};
    p.b = (int)a->batch; p.D = (int)a->dim; p.N = (int)a->dstate; p.K = (int)a->width;
    p.softplus = a->delta_softplus ? 1 : 0; p.mode = a->mode;
    p.x = a->x; p.x_sb = a->x_sb; p.z = a->z; p.z_sb = a->z_sb;
    p.dl = a->delta; p.dl_sb = a->delta_sb; p.B = a->B; p.B_sb = a->B_sb; p.C = a->C; p.C_sb = a->C_sb;
    p.cw = a->conv_weight; p.cb = a->conv_bias; p.A = a->A; p.Dskip = a->Dskip; p.dbias = a->delta_bias;
    p.conv_state = a->conv_state; p.ssm_state = a->ssm_state; p.xc_out = a->xc_out; p.out = a->out;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch ((a->mode & SWX_DECODE_CONV) ? p.K : 4) {
        case 1: swx::launch_dec<1>(p, st); break;
        case 2: swx::launch_dec<2>(p, st); break;
        case 3: swx::launch_dec<3>(p, st); break;
        case 4: swx::launch_dec<4>(p, st); break;
        case 5: swx::launch_dec<5>(p, st); break;
        default: swx::launch_dec<6>(p, st); break;
    }
    return cudaGetLastError() == cudaSuccess ? SWX_OK : SWX_ERR_CUDA;
}
