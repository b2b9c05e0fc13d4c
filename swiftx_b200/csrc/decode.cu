// Single-token recurrent step (generation) for sm_100a, following SiftBlock.step
// (models/sift_block.py:153-175):
//   conv_state <- roll left, append x ;  xc = silu(<conv_state, w> + conv_bias)
//   delta = softplus(delta_raw + delta_bias) ;  h <- exp(delta*A) * h + delta * B * xc
//   y = <h, C> + Dskip * xc ;  out = y * silu(z)
// The state is updated in place.  In the model, x_proj / dt_proj sit between the conv and
// the state update, so the step can run as two launches (SWX_DECODE_CONV, then
// SWX_DECODE_SSM) around the caller's GEMMs; with delta/B/C given it is one fused launch.
// dt_proj can be folded into the state update (dt_in / dt_weight), and
// swx_decode_layer_step folds both projections: the conv kernel writes each 64-channel
// block's partial x_proj products, the state update sums them in block order.
//
// HBM-bound: per (row, channel) the state (N floats) is read and written once, the conv
// window once, and the per-token vectors once.  Four adjacent lanes own the 16 states of
// a channel (one 16-byte load/store each, fully coalesced across the warp); the readout
// is reduced over the 4 lanes with two xor-shuffles.
#include "common.cuh"
#include "launch_util.cuh"

#include <algorithm>

namespace swx {

struct DecDev {
    int b, D, N, K, softplus, mode;
    int a_log;                       // A holds log(-A): the kernels use -expf(A[i])
    const float* x; int64_t x_sb;
    const float* z; int64_t z_sb;
    const float* dl; int64_t dl_sb;
    const float* B; int64_t B_sb;
    const float* C; int64_t C_sb;
    const float* cw; const float* cb;
    const float* A; const float* Dskip; const float* dbias;
    float* conv_state; float* ssm_state; float* xc_out; float* out;
    const float* gw; int64_t gw_sb;    // SiftX pathway mix: (b, ngroups) weights, or nullptr
    const int* gof;                    // (D,) group of each channel
    const float* dti; int64_t dti_sb;  // dt_proj folded in: (b, R) low-rank dt rows, or nullptr
    const float* dtw;                  // (D, R) dt_proj weight
    int R;
    // x_proj folded in too (the layer path): (J, D) weight, J = R + 2N; the conv kernel
    // writes each 64-channel block's partial products (nblk, b, J) and the conv output
    // (b, D) to the workspace, the state-update kernel sums the partials in block order
    const float* xw; int J;
    float* xpart; float* xcbuf;
};

// Lane j's share of <dt_weight[d, :], v> (the float4 groups j, j+4, ...); the four lanes of
// a channel add their shares with two xor shuffles, so all four hold the same sum.
__device__ __forceinline__ float dt_dot_part(const float* __restrict__ w, const float* v, int R, int j) {
    float acc = 0.f;
    for (int r4 = j; 4 * r4 < R; r4 += 4) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(w) + r4);
        const float4 b = *reinterpret_cast<const float4*>(v + 4 * r4);
        acc = fmaf(a.x, b.x, acc);
        acc = fmaf(a.y, b.y, acc);
        acc = fmaf(a.z, b.z, acc);
        acc = fmaf(a.w, b.w, acc);
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    return acc;
}

// Pathway weight of channel d's group for batch row r (1 without the mix).
__device__ __forceinline__ float dec_group_weight(const DecDev& p, int64_t r, int d) {
    return p.gw ? p.gw[r * p.gw_sb + p.gof[d]] : 1.f;
}

// Four consecutive entries of A from offset i (16-byte aligned), formed as -expf(A_log)
// when the caller passed log(-A) -- expf is the function torch.exp evaluates for fp32.
__device__ __forceinline__ float4 load_A4(const DecDev& p, int64_t i) {
    float4 a = *reinterpret_cast<const float4*>(p.A + i);
    if (p.a_log) a = make_float4(-expf(a.x), -expf(a.y), -expf(a.z), -expf(a.w));
    return a;
}

constexpr int DEC_NT = 256;          // 64 channels x 4 state groups per CTA
constexpr int DEC_CH = DEC_NT / 4;
constexpr int DEC_RB = 4;            // batch rows per thread (independent chains in flight)

// Thread (channel d, state group j) handles DEC_RB batch rows of that channel: all of
// their loads are issued before any math, and the per-channel parameters (A, conv
// weights, biases) are loaded once and reused across the rows.
// DTP: delta from the folded dt_proj (DecDev::dti / dtw) instead of a delta row.
template <int K, bool HAS_Z, bool DTP = false>
__global__ void __launch_bounds__(DEC_NT) decode_kernel(const DecDev p) {
    const int j = threadIdx.x & 3;
    const int d = blockIdx.x * DEC_CH + (threadIdx.x >> 2);
    const int b0 = blockIdx.y * DEC_RB;
    const bool dvalid = d < p.D;
    const int dc = dvalid ? d : 0;
    const bool conv = p.mode & SWX_DECODE_CONV, ssm = p.mode & SWX_DECODE_SSM;
    const bool full = (p.N == NS);

    float cw[K];
    float cb = 0.f;
    if (conv) {
#pragma unroll
        for (int k = 0; k < K; ++k) cw[k] = p.cw[(int64_t)dc * K + k];
        cb = p.cb ? p.cb[dc] : 0.f;
    }
    float4 A4 = make_float4(0.f, 0.f, 0.f, 0.f);
    float dsk = 0.f, dbi = 0.f;
    if (ssm) {
        if (full) A4 = load_A4(p, (int64_t)dc * NS + 4 * j);
        dsk = p.Dskip ? p.Dskip[dc] : 0.f;
        dbi = p.dbias ? p.dbias[dc] : 0.f;
    }

    // ---- loads for all rows
    float xin[DEC_RB], zv[DEC_RB], gwv[DEC_RB], raw[DEC_RB], win[DEC_RB][K];
    float4 h4[DEC_RB], b4[DEC_RB], c4[DEC_RB];
    bool valid[DEC_RB];
#pragma unroll
    for (int r = 0; r < DEC_RB; ++r) {
        const int bi = b0 + r;
        valid[r] = dvalid && bi < p.b;
        const int bc = valid[r] ? bi : 0;
        const int64_t bd = (int64_t)bc * p.D + dc;
        xin[r] = p.x[bc * p.x_sb + dc];
        gwv[r] = 1.f;
        if (conv) {
            const float* cs = p.conv_state + bd * K;
            if (K == 4) {
                const float4 w = *reinterpret_cast<const float4*>(cs);
                win[r][0] = w.y; win[r][1 % K] = w.z; win[r][2 % K] = w.w;
            } else {
#pragma unroll
                for (int k = 0; k < K - 1; ++k) win[r][k] = cs[k + 1];
            }
        }
        if (ssm) {
            raw[r] = (DTP ? dt_dot_part(p.dtw + (int64_t)dc * p.R, p.dti + bc * p.dti_sb, p.R, j)
                          : p.dl[bc * p.dl_sb + dc]) + dbi;
            zv[r] = HAS_Z ? p.z[bc * p.z_sb + dc] : 0.f;
            gwv[r] = HAS_Z ? dec_group_weight(p, bc, dc) : 1.f;
            if (full) {
                h4[r] = *reinterpret_cast<const float4*>(p.ssm_state + bd * NS + 4 * j);
                b4[r] = *reinterpret_cast<const float4*>(p.B + bc * p.B_sb + 4 * j);
                c4[r] = *reinterpret_cast<const float4*>(p.C + bc * p.C_sb + 4 * j);
            }
        }
    }

    // ---- math and stores
#pragma unroll
    for (int r = 0; r < DEC_RB; ++r) {
        const int bc = valid[r] ? b0 + r : 0;
        const int64_t bd = (int64_t)bc * p.D + dc;
        float xc = xin[r];
        if (conv) {
            win[r][K - 1] = xin[r];
            float acc = cb;
#pragma unroll
            for (int k = 0; k < K; ++k) acc = fmaf(win[r][k], cw[k], acc);
            xc = silu_f(acc);
            if (valid[r] && j == 0) {
                float* csw = p.conv_state + bd * K;
                if (K == 4) {
                    *reinterpret_cast<float4*>(csw) = make_float4(win[r][0], win[r][1 % K], win[r][2 % K], win[r][3 % K]);
                } else {
#pragma unroll
                    for (int k = 0; k < K; ++k) csw[k] = win[r][k];
                }
                if (p.xc_out) p.xc_out[bd] = xc;
            }
        }
        if (!ssm) continue;
        float dte = raw[r];
        if (p.softplus) {
            float2 sp, dsp;
            softplus2(bc2(raw[r]), sp, dsp);
            dte = sp.x;
        }
        const float dxc = dte * xc;
        float y = 0.f;
        if (full) {
            const float2 dt = bc2(dte * LOG2E), dx = bc2(dxc);
            const float2 h01 = fma2(ex2x2(mul2(dt, f2(A4.x, A4.y))), f2(h4[r].x, h4[r].y), mul2(dx, f2(b4[r].x, b4[r].y)));
            const float2 h23 = fma2(ex2x2(mul2(dt, f2(A4.z, A4.w))), f2(h4[r].z, h4[r].w), mul2(dx, f2(b4[r].z, b4[r].w)));
            float2 yy = mul2(h01, f2(c4[r].x, c4[r].y));
            yy = fma2(h23, f2(c4[r].z, c4[r].w), yy);
            y = yy.x + yy.y;
            if (valid[r]) *reinterpret_cast<float4*>(p.ssm_state + bd * NS + 4 * j) = make_float4(h01.x, h01.y, h23.x, h23.y);
        } else {
            float* hp = p.ssm_state + bd * p.N;
            for (int i = 0; i < 4; ++i) {
                const int n = 4 * j + i;
                if (n < p.N) {
                    const float an = p.a_log ? -expf(p.A[(int64_t)dc * p.N + n]) : p.A[(int64_t)dc * p.N + n];
                    const float h = fmaf(ex2(dte * an * LOG2E), hp[n], dxc * p.B[bc * p.B_sb + n]);
                    y = fmaf(h, p.C[bc * p.C_sb + n], y);
                    if (valid[r]) hp[n] = h;
                }
            }
        }
        y += __shfl_xor_sync(0xffffffffu, y, 1);
        y += __shfl_xor_sync(0xffffffffu, y, 2);
        if (valid[r] && j == 0) {
            y = fmaf(dsk, xc, y);
            if (HAS_Z) y *= silu_f(zv[r]) * gwv[r];
            p.out[bd] = y;
        }
    }
}

// ---------------------------------------------------------------- streaming variant
// For the common shape (width 4, d_state 16, D a multiple of 64, 16-byte aligned rows)
// the step is a pure stream: per (row, channel) 64 B of state in and out, the conv
// window in and out, a few per-token scalars.  A launch of one short-lived CTA per tile
// leaves the memory pipe idle between waves, so here each CTA stays resident, owns one
// 64-channel block (its per-channel parameters are loaded once) and walks a strided
// subset of the batch rows, with the inputs of the next DP_STAGES-1 rows in flight in a
// cp.async ring while it computes the current one.  Outputs go straight to global memory.
constexpr int DP_CH = 64;                 // channels per tile
constexpr int DP_NT = 4 * DP_CH;          // thread = (channel, 4-state group)
constexpr int DP_STAGES = 4;

struct __align__(16) DecTile {
    float4 ss[DP_CH][4];                  // SSM state, 64 channels x 16
    float4 cs[DP_CH];                     // conv window, 64 channels x 4 taps
    float x[DP_CH], z[DP_CH], dr[DP_CH];  // token input (or xc), gate, delta before bias
    float4 B[4], C[4];
};

// Folded dt_proj: a CTA computes delta for all of its rows before its walk (so the dot
// products stay off the walk's per-row path) into a (rows, 64) block of shared memory;
// the launcher keeps a CTA's rows at or below this count.
constexpr int DTP_MAX_ROWS = 32;

// Row stride (floats) of the CTA's dt_proj weight block in shared memory: at least R and
// 16 more than a multiple of 32, so that the float4 loads of one quarter-warp (two
// channels x four lanes, lane j at float offset 4j + 16i of its channel's row) hit 32
// different banks.
__host__ __device__ constexpr int dtw_stride(int R) { return R + ((16 - R % 32) + 32) % 32; }

// Lane j's share of <W row, v> from shared memory, then the sum over the channel's four
// lanes (same order as dt_dot_part: float4 groups j, j+4, ...; two xor shuffles).
__device__ __forceinline__ float dt_dot_smem(const float* w, const float* v, int R, int j) {
    float acc = 0.f;
#pragma unroll 4
    for (int r4 = j; 4 * r4 < R; r4 += 4) {
        const float4 a = *reinterpret_cast<const float4*>(w + 4 * r4);
        const float4 b = *reinterpret_cast<const float4*>(v + 4 * r4);   // global or shared
        acc = fmaf(a.x, b.x, acc);
        acc = fmaf(a.y, b.y, acc);
        acc = fmaf(a.z, b.z, acc);
        acc = fmaf(a.w, b.w, acc);
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    return acc;
}

// XP (with DTP): x_proj folded in as well; the CTA's rows' (DTP_MAX_ROWS, J) x_proj
// outputs follow the delta block in shared memory, summed from the conv kernel's
// per-block partials, and B, C come from there.
template <bool CONV, bool HAS_Z, bool DTP, bool XP = false>
__device__ __forceinline__ void decode_stream_body(const DecDev& p, int row_groups) {
    __shared__ DecTile S[DP_STAGES];
    // DTP: the CTA's (64, dtw_stride(R)) dt_proj block, then its rows' (DTP_MAX_ROWS, 64) delta
    extern __shared__ __align__(16) float sW[];
    const int tid = threadIdx.x;
    const int j = tid & 3, ch = tid >> 2;
    const int nblk = p.D / DP_CH;
    const int cb = blockIdx.x % nblk, rg = blockIdx.x / nblk;
    const int d0 = cb * DP_CH, d = d0 + ch;

    // per-channel parameters, once per CTA
    const float4 A4 = load_A4(p, (int64_t)d * NS + 4 * j);
    float4 cw = make_float4(0.f, 0.f, 0.f, 0.f);
    float cbias = 0.f;
    if (CONV) {
        cw = *reinterpret_cast<const float4*>(p.cw + (int64_t)d * 4);
        cbias = p.cb ? p.cb[d] : 0.f;
    }
    const float dsk = p.Dskip ? p.Dskip[d] : 0.f;
    const float dbi = p.dbias ? p.dbias[d] : 0.f;
    const float2 A01 = f2(A4.x, A4.y), A23 = f2(A4.z, A4.w);
    const int ws = DTP ? dtw_stride(p.R) : 0;
    if (DTP) {                            // the weight block, once per CTA
        const int q4 = p.R / 4;
        for (int i = tid; i < DP_CH * q4; i += DP_NT) {
            const int c = i / q4, q = i - c * q4;
            *reinterpret_cast<float4*>(sW + c * ws + 4 * q) =
                __ldg(reinterpret_cast<const float4*>(p.dtw + (int64_t)(d0 + c) * p.R) + q);
        }
        __syncthreads();
    }

    // tile copies: every thread one 16-byte piece of the state; threads 0..63 the conv
    // window, 64..111 x / z / delta, 112..119 B and C
    auto issue = [&](int r, int slot) {
        DecTile& T = S[slot];
        cp_async16(&T.ss[0][0] + tid, p.ssm_state + ((int64_t)r * p.D + d0) * NS + 4 * tid, 16);
        if (tid < 64) {
            if (CONV) cp_async16(&T.cs[tid], p.conv_state + ((int64_t)r * p.D + d0 + tid) * 4, 16);
        } else if (tid < 80) {
            cp_async16(&T.x[4 * (tid - 64)], p.x + r * p.x_sb + d0 + 4 * (tid - 64), 16);
        } else if (tid < 96) {
            if (HAS_Z) cp_async16(&T.z[4 * (tid - 80)], p.z + r * p.z_sb + d0 + 4 * (tid - 80), 16);
        } else if (tid < 112) {
            if (!DTP) cp_async16(&T.dr[4 * (tid - 96)], p.dl + r * p.dl_sb + d0 + 4 * (tid - 96), 16);
        } else if (tid < 116) {
            if (!XP) cp_async16(&T.B[tid - 112], p.B + r * p.B_sb + 4 * (tid - 112), 16);
        } else if (tid < 120) {
            if (!XP) cp_async16(&T.C[tid - 116], p.C + r * p.C_sb + 4 * (tid - 116), 16);
        }
    };

#pragma unroll
    for (int k = 0; k < DP_STAGES - 1; ++k) {
        const int r = rg + k * row_groups;
        if (r < p.b) issue(r, k);
        cp_async_commit();
    }
    float* sDr = sW + DP_CH * ws;
    float* sX = sDr + DTP_MAX_ROWS * DP_CH;
    if (XP) {                             // x_proj outputs of this CTA's rows: partials in block order
        for (int k = 0; rg + k * row_groups < p.b; ++k) {
            const int r = rg + k * row_groups;
            for (int o = tid; o < p.J; o += DP_NT) {
                float acc = 0.f;
                for (int q = 0; q < nblk; ++q) acc += p.xpart[((int64_t)q * p.b + r) * p.J + o];
                sX[k * p.J + o] = acc;
            }
        }
        __syncthreads();
    }
    if (DTP) {                            // delta of every row of this CTA, while the ring fills
        for (int k = 0; rg + k * row_groups < p.b; ++k) {
            const float* v = XP ? sX + k * p.J : p.dti + (int64_t)(rg + k * row_groups) * p.dti_sb;
            const float dv = dt_dot_smem(sW + ch * ws, v, p.R, j);
            if (j == 0) sDr[k * DP_CH + ch] = dv;
        }
    }
    for (int k = 0;; ++k) {
        const int r = rg + k * row_groups;
        if (r >= p.b) break;
        const int rn = rg + (k + DP_STAGES - 1) * row_groups;
        if (rn < p.b) issue(rn, (k + DP_STAGES - 1) % DP_STAGES);   // slot read at k-1
        cp_async_commit();
        cp_async_wait<DP_STAGES - 1>();
        __syncthreads();

        const DecTile& T = S[k % DP_STAGES];
        const int64_t bd = (int64_t)r * p.D + d;
        float xc = T.x[ch];
        float4 win = make_float4(0.f, 0.f, 0.f, 0.f);
        if (CONV) {
            const float4 w = T.cs[ch];
            win = make_float4(w.y, w.z, w.w, xc);
            float acc = cbias;
            acc = fmaf(win.x, cw.x, acc);
            acc = fmaf(win.y, cw.y, acc);
            acc = fmaf(win.z, cw.z, acc);
            acc = fmaf(win.w, cw.w, acc);
            xc = silu_f(acc);
        }
        const float raw = (DTP ? sDr[k * DP_CH + ch] : T.dr[ch]) + dbi;
        float dte = raw;
        if (p.softplus) {
            float2 sp, dsp;
            softplus2(bc2(raw), sp, dsp);
            dte = sp.x;
        }
        const float4 h4 = T.ss[ch][j];
        const float4 b4 = XP ? *reinterpret_cast<const float4*>(sX + k * p.J + p.R + 4 * j) : T.B[j];
        const float4 c4 = XP ? *reinterpret_cast<const float4*>(sX + k * p.J + p.R + NS + 4 * j) : T.C[j];
        // same operation order as decode_kernel, so both give identical bits
        const float2 dt = bc2(dte * LOG2E), dx = bc2(dte * xc);
        const float2 h01 = fma2(ex2x2(mul2(dt, A01)), f2(h4.x, h4.y), mul2(dx, f2(b4.x, b4.y)));
        const float2 h23 = fma2(ex2x2(mul2(dt, A23)), f2(h4.z, h4.w), mul2(dx, f2(b4.z, b4.w)));
        float2 yy = mul2(h01, f2(c4.x, c4.y));
        yy = fma2(h23, f2(c4.z, c4.w), yy);
        float y = yy.x + yy.y;
        y += __shfl_xor_sync(0xffffffffu, y, 1);
        y += __shfl_xor_sync(0xffffffffu, y, 2);
        *reinterpret_cast<float4*>(p.ssm_state + bd * NS + 4 * j) = make_float4(h01.x, h01.y, h23.x, h23.y);
        if (j == 0) {
            if (CONV) {
                *reinterpret_cast<float4*>(p.conv_state + bd * 4) = win;
                if (p.xc_out) p.xc_out[bd] = xc;
            }
            y = fmaf(dsk, xc, y);
            if (HAS_Z) y *= silu_f(T.z[ch]) * dec_group_weight(p, r, d);
            p.out[bd] = y;
        }
        __syncthreads();                  // slot k % DP_STAGES is refilled at k+1
    }
    cp_async_wait<0>();
}

template <bool CONV, bool HAS_Z>
__global__ void __launch_bounds__(DP_NT) decode_stream_kernel(const DecDev p, int row_groups) {
    decode_stream_body<CONV, HAS_Z, false>(p, row_groups);
}

// The folded-dt_proj variant: at most 64 registers, so that four CTAs share an SM as the
// plain kernel's do.
template <bool HAS_Z>
__global__ void __launch_bounds__(DP_NT, 4) decode_stream_dtp_kernel(const DecDev p, int row_groups) {
    decode_stream_body<false, HAS_Z, true>(p, row_groups);
}

// x_proj and dt_proj folded in: the state-update half of the layer path.
template <bool HAS_Z>
__global__ void __launch_bounds__(DP_NT, 3) decode_stream_xp_kernel(const DecDev p, int row_groups) {
    decode_stream_body<false, HAS_Z, true, true>(p, row_groups);
}

// The conv half of the layer path (width 4, D a multiple of 64): CTA = 64 channels of
// one row.  It rolls the conv window, writes xc = silu(conv + bias) to the workspace and
// the block's partial x_proj products  sum_{d in block} W[o, d] xc[d]  for every output
// o < J (the state-update kernel adds the blocks in order).
__global__ void __launch_bounds__(DP_NT) decode_conv_xproj_kernel(const DecDev p) {
    __shared__ __align__(16) float xs[DP_CH];
    const int tid = threadIdx.x;
    const int cb = blockIdx.x, r = blockIdx.y;
    const int d0 = cb * DP_CH;
    if (tid < DP_CH) {
        const int d = d0 + tid;
        const int64_t bd = (int64_t)r * p.D + d;
        const float4 w = *reinterpret_cast<const float4*>(p.conv_state + bd * 4);
        const float4 cw = *reinterpret_cast<const float4*>(p.cw + (int64_t)d * 4);
        const float4 win = make_float4(w.y, w.z, w.w, p.x[r * p.x_sb + d]);
        float acc = p.cb ? p.cb[d] : 0.f;          // same order as the streaming kernel's conv
        acc = fmaf(win.x, cw.x, acc);
        acc = fmaf(win.y, cw.y, acc);
        acc = fmaf(win.z, cw.z, acc);
        acc = fmaf(win.w, cw.w, acc);
        const float xc = silu_f(acc);
        *reinterpret_cast<float4*>(p.conv_state + bd * 4) = win;
        p.xcbuf[bd] = xc;
        xs[tid] = xc;
    }
    __syncthreads();
    for (int o = tid; o < p.J; o += DP_NT) {
        const float4* wr = reinterpret_cast<const float4*>(p.xw + (int64_t)o * p.D + d0);
        float acc = 0.f;
#pragma unroll 4
        for (int c4 = 0; c4 < DP_CH / 4; ++c4) {
            const float4 a = __ldg(wr + c4);
            acc = fmaf(a.x, xs[4 * c4], acc);
            acc = fmaf(a.y, xs[4 * c4 + 1], acc);
            acc = fmaf(a.z, xs[4 * c4 + 2], acc);
            acc = fmaf(a.w, xs[4 * c4 + 3], acc);
        }
        p.xpart[((int64_t)cb * p.b + r) * p.J + o] = acc;
    }
}

// The streaming variant applies when every tile is full and every row is 16-byte aligned.
static bool stream_ok(const DecDev& p) {
    auto al = [](const void* q) { return q == nullptr || (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    const bool conv = p.mode & SWX_DECODE_CONV;
    if (!(p.mode & SWX_DECODE_SSM) || p.N != NS || (conv && p.K != 4) || p.D % DP_CH != 0) return false;
    if (!al(p.x) || !al(p.z) || !al(p.dl) || !al(p.B) || !al(p.C) || !al(p.A) || !al(p.ssm_state)) return false;
    if (conv && (!al(p.conv_state) || !al(p.cw))) return false;
    if (p.x_sb % 4 || p.dl_sb % 4 || p.B_sb % 4 || p.C_sb % 4 || (p.z && p.z_sb % 4)) return false;
    return true;
}

template <bool CONV, bool HAS_Z, bool DTP = false>
static cudaError_t launch_stream_t(const DecDev& p, cudaStream_t st) {
    auto k = DTP ? decode_stream_dtp_kernel<HAS_Z> : decode_stream_kernel<CONV, HAS_Z>;
    // dynamic shared memory: the weight block and the rows' delta (opted in up to the
    // largest a call can pass)
    const int used = DTP ? DP_CH * (dtw_stride(p.R) + DTP_MAX_ROWS) * 4 : 0;
    cudaError_t e = DTP ? allow_smem(k, DP_CH * (dtw_stride(SWX_DECODE_MAX_DT_RANK) + DTP_MAX_ROWS) * 4)
                        : cudaSuccess;
    if (e != cudaSuccess) return e;
    int sms = 0, per_sm = 0;
    e = sm_fit(k, DP_NT, 0, &sms, &per_sm);
    if (e != cudaSuccess) return e;
    if (DTP) {                           // CTAs per SM at this call's weight-block size
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, DP_NT, used);
        if (e != cudaSuccess) return e;
    }
    const int nblk = p.D / DP_CH;
    const int slots = std::max(1, sms * per_sm);
    int row_groups = std::max(1, std::min(p.b, slots / nblk));
    if (DTP) row_groups = std::max(row_groups, (p.b + DTP_MAX_ROWS - 1) / DTP_MAX_ROWS);   // rows per CTA <= 32
    k<<<nblk * row_groups, DP_NT, used, st>>>(p, row_groups);
    return cudaGetLastError();
}

static cudaError_t launch_stream(const DecDev& p, cudaStream_t st) {
    const bool conv = p.mode & SWX_DECODE_CONV;
    if (p.dti) return p.z ? launch_stream_t<false, true, true>(p, st) : launch_stream_t<false, false, true>(p, st);
    if (conv) return p.z ? launch_stream_t<true, true>(p, st) : launch_stream_t<true, false>(p, st);
    return p.z ? launch_stream_t<false, true>(p, st) : launch_stream_t<false, false>(p, st);
}

// The layer path: the conv + partial x_proj kernel, then the state update with x_proj
// and dt_proj folded in, reading the conv output from the workspace.
static cudaError_t launch_layer(const DecDev& p0, cudaStream_t st) {
    const int nblk = p0.D / DP_CH;
    decode_conv_xproj_kernel<<<dim3(nblk, p0.b), DP_NT, 0, st>>>(p0);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    DecDev p = p0;
    p.x = p0.xcbuf; p.x_sb = p0.D; p.mode = SWX_DECODE_SSM;
    auto k = p.z ? decode_stream_xp_kernel<true> : decode_stream_xp_kernel<false>;
    const int used = (DP_CH * (dtw_stride(p.R) + DTP_MAX_ROWS) + DTP_MAX_ROWS * p.J) * 4;
    const int most = (DP_CH * (dtw_stride(SWX_DECODE_MAX_DT_RANK) + DTP_MAX_ROWS) +
                      DTP_MAX_ROWS * (SWX_DECODE_MAX_DT_RANK + 2 * NS)) * 4;
    if ((e = allow_smem(k, most)) != cudaSuccess) return e;
    int sms = 0, per_sm = 0;
    if ((e = sm_fit(k, DP_NT, 0, &sms, &per_sm)) != cudaSuccess) return e;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, DP_NT, used)) != cudaSuccess) return e;
    const int slots = std::max(1, sms * per_sm);
    int row_groups = std::max(1, std::min(p.b, slots / nblk));
    row_groups = std::max(row_groups, (p.b + DTP_MAX_ROWS - 1) / DTP_MAX_ROWS);   // rows per CTA <= 32
    k<<<nblk * row_groups, DP_NT, used, st>>>(p, row_groups);
    return cudaGetLastError();
}

int64_t layer_workspace_floats(int64_t b, int64_t D, int64_t J) {
    return (D / DP_CH) * b * J + b * D;
}

template <int K>
static void launch_dec(const DecDev& p, cudaStream_t st) {
    dim3 grid((p.D + DEC_CH - 1) / DEC_CH, (p.b + DEC_RB - 1) / DEC_RB);
    if (p.dti) {
        if (p.z) decode_kernel<K, true, true><<<grid, DEC_NT, 0, st>>>(p);
        else decode_kernel<K, false, true><<<grid, DEC_NT, 0, st>>>(p);
    } else if (p.z) {
        decode_kernel<K, true><<<grid, DEC_NT, 0, st>>>(p);
    } else {
        decode_kernel<K, false><<<grid, DEC_NT, 0, st>>>(p);
    }
}

}  // namespace swx

extern "C" int swx_decode_step(const swx_decode_args* a, void* stream) {
    if (!a) return SWX_ERR_INVALID_ARG;
    if (a->batch < 0 || a->dim < 0) return SWX_ERR_INVALID_ARG;
    if (a->mode < 1 || a->mode > 3) return SWX_ERR_INVALID_ARG;
    if (a->flags & ~SWX_DECODE_A_LOG) return SWX_ERR_INVALID_ARG;
    if ((a->mode & SWX_DECODE_CONV) && (a->width < 1 || a->width > 6)) return SWX_ERR_UNSUPPORTED;
    if ((a->mode & SWX_DECODE_SSM) && (a->dstate < 1 || a->dstate > swx::NS)) return SWX_ERR_UNSUPPORTED;
    if (a->batch * a->dim == 0) return SWX_OK;
    if (a->dim > (int64_t)INT32_MAX || (a->batch + 3) / 4 > 65535) return SWX_ERR_UNSUPPORTED;
    if (!a->x) return SWX_ERR_INVALID_ARG;
    if ((a->mode & SWX_DECODE_CONV) && (!a->conv_weight || !a->conv_state)) return SWX_ERR_INVALID_ARG;
    if (a->dt_in) {
        // dt_proj folded in: SSM-only steps (the conv's output feeds x_proj first)
        if (a->mode != SWX_DECODE_SSM) return SWX_ERR_UNSUPPORTED;
        if (a->delta || !a->dt_weight || a->dt_rank < 4 || a->dt_rank % 4 || a->dt_rank > SWX_DECODE_MAX_DT_RANK)
            return SWX_ERR_INVALID_ARG;
        if ((((uintptr_t)a->dt_in | (uintptr_t)a->dt_weight) & 15u) || a->dt_in_sb < 0 || a->dt_in_sb % 4)
            return SWX_ERR_INVALID_ARG;
    } else if ((a->mode & SWX_DECODE_SSM) && !a->delta) {
        return SWX_ERR_INVALID_ARG;
    }
    if ((a->mode & SWX_DECODE_SSM) && (!a->B || !a->C || !a->A || !a->ssm_state || !a->out))
        return SWX_ERR_INVALID_ARG;
    if ((a->mode & SWX_DECODE_SSM) && a->dstate == swx::NS &&
        (((uintptr_t)a->ssm_state | (uintptr_t)a->A | (uintptr_t)a->B | (uintptr_t)a->C) & 15u ||
         (a->B_sb % 4) || (a->C_sb % 4)))
        return SWX_ERR_INVALID_ARG;
    if ((a->mode & SWX_DECODE_CONV) && a->width == 4 && ((uintptr_t)a->conv_state & 15u))
        return SWX_ERR_INVALID_ARG;
    swx::DecDev p{};
    p.b = (int)a->batch; p.D = (int)a->dim; p.N = (int)a->dstate; p.K = (int)a->width;
    p.softplus = a->delta_softplus ? 1 : 0; p.mode = a->mode;
    p.a_log = (a->flags & SWX_DECODE_A_LOG) ? 1 : 0;
    p.x = a->x; p.x_sb = a->x_sb; p.z = a->z; p.z_sb = a->z_sb;
    p.dl = a->delta; p.dl_sb = a->delta_sb; p.B = a->B; p.B_sb = a->B_sb; p.C = a->C; p.C_sb = a->C_sb;
    p.cw = a->conv_weight; p.cb = a->conv_bias; p.A = a->A; p.Dskip = a->Dskip; p.dbias = a->delta_bias;
    p.conv_state = a->conv_state; p.ssm_state = a->ssm_state; p.xc_out = a->xc_out; p.out = a->out;
    if (a->dt_in) {
        p.dti = a->dt_in; p.dti_sb = a->dt_in_sb; p.dtw = a->dt_weight; p.R = a->dt_rank;
    }
    if (a->group_w) {
        if (!a->z || !(a->mode & SWX_DECODE_SSM)) return SWX_ERR_UNSUPPORTED;
        if (!a->group_of || a->group_w_sb < 0 || a->ngroups < 1 || a->ngroups > SWX_MAX_GROUPS)
            return SWX_ERR_INVALID_ARG;
        p.gw = a->group_w; p.gw_sb = a->group_w_sb; p.gof = a->group_of;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (swx::stream_ok(p)) return swx::launch_stream(p, st) == cudaSuccess ? SWX_OK : SWX_ERR_CUDA;
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

extern "C" int64_t swx_decode_layer_workspace_bytes(int64_t batch, int64_t dim, int64_t xproj_rows) {
    if (batch < 0 || dim < 0 || xproj_rows < 0 || dim > (int64_t)INT32_MAX || xproj_rows > 4096) return -1;
    return swx::layer_workspace_floats(batch, dim, xproj_rows) * 4;
}

extern "C" int swx_decode_layer_step(const swx_decode_args* a, void* stream) {
    if (!a) return SWX_ERR_INVALID_ARG;
    if (a->batch < 0 || a->dim < 0 || a->flags & ~SWX_DECODE_A_LOG) return SWX_ERR_INVALID_ARG;
    if (a->mode != (SWX_DECODE_CONV | SWX_DECODE_SSM) || a->dstate != swx::NS || a->width != 4 ||
        a->dim % swx::DP_CH != 0 || a->group_w)
        return SWX_ERR_UNSUPPORTED;
    if (a->batch * a->dim == 0) return SWX_OK;
    if (a->dim > (int64_t)INT32_MAX || a->batch > 65535) return SWX_ERR_UNSUPPORTED;
    if (a->delta || a->B || a->C || a->dt_in) return SWX_ERR_INVALID_ARG;
    if (!a->x || !a->conv_weight || !a->conv_state || !a->A || !a->ssm_state || !a->out || !a->dt_weight ||
        !a->xproj_weight || !a->workspace)
        return SWX_ERR_INVALID_ARG;
    if (a->dt_rank < 4 || a->dt_rank % 4 || a->dt_rank > SWX_DECODE_MAX_DT_RANK ||
        a->xproj_rows != a->dt_rank + 2 * a->dstate)
        return SWX_ERR_INVALID_ARG;
    auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    if (!al(a->x) || (a->z && !al(a->z)) || !al(a->conv_state) || !al(a->conv_weight) || !al(a->A) ||
        !al(a->ssm_state) || !al(a->dt_weight) || !al(a->xproj_weight) || !al(a->workspace) ||
        a->x_sb % 4 || (a->z && a->z_sb % 4) || a->x_sb < 0 || a->z_sb < 0)
        return SWX_ERR_INVALID_ARG;
    const int64_t need = swx_decode_layer_workspace_bytes(a->batch, a->dim, a->xproj_rows);
    if (need < 0 || a->workspace_bytes < need) return SWX_ERR_INVALID_ARG;
    swx::DecDev p{};
    p.b = (int)a->batch; p.D = (int)a->dim; p.N = (int)a->dstate; p.K = 4;
    p.softplus = a->delta_softplus ? 1 : 0; p.mode = a->mode;
    p.a_log = (a->flags & SWX_DECODE_A_LOG) ? 1 : 0;
    p.x = a->x; p.x_sb = a->x_sb; p.z = a->z; p.z_sb = a->z_sb;
    p.cw = a->conv_weight; p.cb = a->conv_bias; p.A = a->A; p.Dskip = a->Dskip; p.dbias = a->delta_bias;
    p.conv_state = a->conv_state; p.ssm_state = a->ssm_state; p.out = a->out;
    p.dtw = a->dt_weight; p.R = a->dt_rank;
    p.xw = a->xproj_weight; p.J = a->xproj_rows;
    p.xpart = static_cast<float*>(a->workspace);
    p.xcbuf = p.xpart + (int64_t)(a->dim / swx::DP_CH) * a->batch * a->xproj_rows;
    // the conv output's rows must stay 16-byte aligned for the state update's tile copies
    if (reinterpret_cast<uintptr_t>(p.xcbuf) & 15u) return SWX_ERR_INVALID_ARG;
    return swx::launch_layer(p, static_cast<cudaStream_t>(stream)) == cudaSuccess ? SWX_OK : SWX_ERR_CUDA;
}
