// Initial-state correction of a scanned chunk, for the sequence-parallel scan.
//
// The scan is linear in its initial state: scanned from h_in instead of 0, every state
// gains  P_t h_in  with P_t = prod_{s<=t} exp(delta_s A) = exp(A S_t),  S_t = sum_{s<=t}
// delta_s  (per channel; one decay per state), so the output gains
//     corr_t = sum_n C_t[n] exp(A[n] S_t) h_in[n],   out_t += gate_t * corr_t
// (gate_t = silu(z_t), times the pathway group weight when the mix is fused, the gate
// being a factor of the pre-gate output).  Unlike a
// rescan, no step depends on the previous one except through the running sum S_t, so the
// work is split over (channel, 256-step block) threads:
//   1. scan_correct_sums_kernel: sum of delta_eff over each block, then
//      scan_correct_prefix_kernel: each block's starting S, the earlier blocks' sums;
//   2. scan_correct_kernel: from its block's starting S, per step S += delta_eff and the
//      16 decays exp2(A log2e S) against
//      C_t h_in.  The kernel is bound by instruction issue, so the decays stay on the MUFU
//      unit (moving a share to the FMA-pipe exp2 was measured slower: 1.78 ms with none,
//      2.07 with half, 2.70 with all at b=4, L=32768, D=2048, bf16; with 2, 4 or 6 of the
//      16 decays 1.78, 1.83 and 1.93 against 1.80 ms in a later run).  Skipping the state
//      groups whose decays have underflowed in every lane (S only grows under softplus)
//      was measured too: with one warp-uniform dispatch per 8 steps over copies of the
//      step body for 4..0 live groups, 1.75 against 1.79 ms at L=32768 but 0.71 against
//      0.59 ms at L=8192, where few decays underflow and the copies miss the instruction
//      cache; not kept.
#include <algorithm>

#include "common.cuh"
#include "launch_util.cuh"
#include "scan_params.cuh"

namespace swx {

constexpr int CR_THREADS = 128;      // channels per CTA
constexpr int CR_BLK = 256;          // steps per thread
constexpr int CR_CROWS = 64;         // C rows staged in shared memory at a time

__device__ __forceinline__ float load_A_cr(const ScanDev& p, int64_t i) {
    const float a = p.A[i];
    return p.a_log ? -expf(a) : a;
}

template <typename Tin>
__global__ void __launch_bounds__(CR_THREADS) scan_correct_sums_kernel(const ScanDev p, float* bsum, int nblk) {
    const int d = blockIdx.x * CR_THREADS + threadIdx.x;
    const int bi = blockIdx.y, k = blockIdx.z;
    if (d >= p.D) return;
    const Tin* dl = static_cast<const Tin*>(p.dl) + bi * p.dl_sb + d;
    const float bias = p.dbias ? p.dbias[d] : 0.f;
    const int t0 = k * CR_BLK, t1 = min(p.L, t0 + CR_BLK);
    float s = 0.f;
#pragma unroll 8
    for (int t = t0; t < t1; ++t) {
        const float raw = Elem<Tin>::to_f(dl[(int64_t)t * p.dl_sl]) + bias;
        s += p.softplus ? softplus_f(raw) : raw;
    }
    bsum[((int64_t)bi * nblk + k) * p.D + d] = s;
}

// In place, per (row, channel): each block's sum of delta_eff becomes the sum over the
// blocks before it (an exclusive prefix in block order).
__global__ void scan_correct_prefix_kernel(float* bsum, int64_t rows_d, int D, int nblk) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;       // row * D + channel
    if (i >= rows_d) return;
    float* bs = bsum + (i / D) * (int64_t)nblk * D + i % D;
    float s = 0.f;
    for (int q = 0; q < nblk; ++q) {
        const float v = bs[(int64_t)q * D];
        bs[(int64_t)q * D] = s;
        s += v;
    }
}

// FIX: the correction of a split forward -- besides the output, the 16-step state
// checkpoints (each gains exp(A S) h_in at its step) and the pre-gate output (gains the
// un-gated term) are corrected too, when the forward wrote them.
template <typename Tin, typename Tout, bool HAS_Z, bool GW = false, bool FIX = false>
__global__ void __launch_bounds__(CR_THREADS) scan_correct_kernel(const ScanDev p, const float* bsum, int nblk) {
    __shared__ __align__(16) float Cs[CR_CROWS][NS];
    const int tid = threadIdx.x;
    const int d = blockIdx.x * CR_THREADS + tid;
    const int bi = blockIdx.y, k = blockIdx.z;
    if (p.skip_first_seg && bi % p.seg_g == 0) return;      // a first segment: h_in = 0
    const bool ok = d < p.D;
    const int dc = ok ? d : p.D - 1;
    const int t0 = k * CR_BLK, t1 = min(p.L, t0 + CR_BLK);
    // S at the block's start: the earlier blocks' sums, added in block order by
    // scan_correct_prefix_kernel
    float S = bsum[((int64_t)bi * nblk + k) * p.D + dc];
    float2 A2[NS / 2], H[NS / 2];
    const float* h_in = p.h0 + ((int64_t)bi * p.D + dc) * p.N;
#pragma unroll
    for (int i = 0; i < NS / 2; ++i) {
        const int n0 = 2 * i, n1 = 2 * i + 1;
        A2[i] = f2(n0 < p.N ? load_A_cr(p, (int64_t)dc * p.N + n0) * LOG2E : 0.f,
                   n1 < p.N ? load_A_cr(p, (int64_t)dc * p.N + n1) * LOG2E : 0.f);
        H[i] = f2(n0 < p.N ? h_in[n0] : 0.f, n1 < p.N ? h_in[n1] : 0.f);
    }
    const Tin* dl = static_cast<const Tin*>(p.dl) + bi * p.dl_sb + dc;
    const Tin* zp = HAS_Z ? static_cast<const Tin*>(p.z) + bi * p.z_sb + dc : nullptr;
    const Tin* gC = static_cast<const Tin*>(p.C) + bi * p.C_sb;
    Tout* out = static_cast<Tout*>(p.out) + (int64_t)bi * p.L * p.D + dc;
    float* yp = (FIX && p.ypre) ? p.ypre + (int64_t)bi * p.L * p.D + dc : nullptr;
    float* ckb = (FIX && p.ck) ? p.ck + ((int64_t)bi * p.nck * p.D + dc) * NS : nullptr;
    const float bias = p.dbias ? p.dbias[dc] : 0.f;
    const int grp = GW ? p.gof[dc] : 0;        // pathway group of the channel (mix fused into the gate)
    for (int tb = t0; tb < t1; tb += CR_CROWS) {
        const int nr = min(CR_CROWS, t1 - tb);
        __syncthreads();
        for (int i = tid; i < nr * NS; i += CR_THREADS) {
            const int row = i / NS, n = i % NS;
            Cs[row][n] = n < p.N ? Elem<Tin>::to_f(gC[(int64_t)(tb + row) * p.C_sl + n]) : 0.f;
        }
        __syncthreads();
        if (!ok) continue;
        // eight steps at a time: their delta, z and output loads are issued before the
        // arithmetic (the running sum S is the only dependence between steps)
        for (int r0 = 0; r0 < nr; r0 += 8) {
            float raw[8], zz[8], oo[8], yy[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const bool v = r0 + i < nr;
                const int64_t t = tb + r0 + (v ? i : 0);
                raw[i] = Elem<Tin>::to_f(dl[t * p.dl_sl]) + bias;
                zz[i] = HAS_Z ? Elem<Tin>::to_f(zp[t * p.z_sl]) : 0.f;
                oo[i] = Elem<Tout>::to_f(out[t * p.D]);
                yy[i] = (FIX && yp) ? yp[t * p.D] : 0.f;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (r0 + i >= nr) break;
                if (FIX && ckb && i == 0 && (r0 & 8) == 0) {
                    // checkpoint of the 16-step chunk starting here: the state before this
                    // step, i.e. with S still the sum through the previous step
                    const float2 sp = bc2(S);
                    float4* cq = reinterpret_cast<float4*>(ckb + (((int64_t)(tb + r0) >> 4) * p.D) * NS);
#pragma unroll
                    for (int v = 0; v < NS / 4; ++v) {
                        const float2 q0 = mul2(ex2x2(mul2(sp, A2[2 * v])), H[2 * v]);
                        const float2 q1 = mul2(ex2x2(mul2(sp, A2[2 * v + 1])), H[2 * v + 1]);
                        float4 c = cq[v];
                        c.x += q0.x; c.y += q0.y; c.z += q1.x; c.w += q1.y;
                        cq[v] = c;
                    }
                }
                S += p.softplus ? softplus_f(raw[i]) : raw[i];
                const float2 s2 = bc2(S);
                const float4* cr = reinterpret_cast<const float4*>(&Cs[r0 + i][0]);
                // two accumulators halve the dependent chain of the 16-term sum
                float2 acc0 = bc2(0.f), acc1 = bc2(0.f);
#pragma unroll
                for (int v = 0; v < NS / 4; ++v) {
                    const float4 c4 = cr[v];
                    const float2 p0 = ex2x2(mul2(s2, A2[2 * v])), p1 = ex2x2(mul2(s2, A2[2 * v + 1]));
                    acc0 = fma2(mul2(p0, H[2 * v]), f2(c4.x, c4.y), acc0);
                    acc1 = fma2(mul2(p1, H[2 * v + 1]), f2(c4.z, c4.w), acc1);
                }
                const float2 acc = add2(acc0, acc1);
                float corr = acc.x + acc.y;
                if (FIX) yy[i] += corr;                  // the pre-gate output gains the bare term
                if (HAS_Z) corr *= silu_f(zz[i]);
                if (GW) corr *= p.gw[(int64_t)bi * p.gw_sb + (int64_t)(tb + r0 + i) * p.gw_sl + grp];
                oo[i] += corr;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (r0 + i < nr) {
                    out[(int64_t)(tb + r0 + i) * p.D] = Elem<Tout>::from_f(oo[i]);
                    if (FIX && yp) yp[(int64_t)(tb + r0 + i) * p.D] = yy[i];
                }
        }
    }
}

template <typename Tin, typename Tout, bool FIX>
static void launch_correct_k(const ScanDev& p, float* ws, int nblk, bool has_z, dim3 grid, cudaStream_t st) {
    if (has_z && p.gw) scan_correct_kernel<Tin, Tout, true, true, FIX><<<grid, CR_THREADS, 0, st>>>(p, ws, nblk);
    else if (has_z) scan_correct_kernel<Tin, Tout, true, false, FIX><<<grid, CR_THREADS, 0, st>>>(p, ws, nblk);
    else scan_correct_kernel<Tin, Tout, false, false, FIX><<<grid, CR_THREADS, 0, st>>>(p, ws, nblk);
}

template <typename Tin, typename Tout>
static cudaError_t launch_correct_t(const ScanDev& p, float* ws, bool has_z, bool fix, cudaStream_t st) {
    const int nblk = (p.L + CR_BLK - 1) / CR_BLK;
    dim3 grid((p.D + CR_THREADS - 1) / CR_THREADS, p.b, nblk);
    scan_correct_sums_kernel<Tin><<<grid, CR_THREADS, 0, st>>>(p, ws, nblk);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int64_t rows_d = (int64_t)p.b * p.D;
    scan_correct_prefix_kernel<<<(unsigned)((rows_d + 255) / 256), 256, 0, st>>>(ws, rows_d, p.D, nblk);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if (fix) launch_correct_k<Tin, Tout, true>(p, ws, nblk, has_z, grid, st);
    else launch_correct_k<Tin, Tout, false>(p, ws, nblk, has_z, grid, st);
    return cudaGetLastError();
}

int64_t scan_correct_workspace_floats(int64_t b, int64_t L, int64_t D) {
    return b * ((L + CR_BLK - 1) / CR_BLK) * D;
}

cudaError_t launch_scan_correct(const ScanDev& p, int in_dtype, int out_dtype, bool has_z, float* ws,
                                cudaStream_t st, bool fix) {
    const bool bf_in = in_dtype == SWX_DTYPE_BF16, bf_out = out_dtype == SWX_DTYPE_BF16;
    if (!bf_in && !bf_out) return launch_correct_t<float, float>(p, ws, has_z, fix, st);
    if (!bf_in && bf_out) return launch_correct_t<float, __nv_bfloat16>(p, ws, has_z, fix, st);
    if (bf_in && !bf_out) return launch_correct_t<__nv_bfloat16, float>(p, ws, has_z, fix, st);
    return launch_correct_t<__nv_bfloat16, __nv_bfloat16>(p, ws, has_z, fix, st);
}

// Initial states of the segments of a split forward: thread = (row, channel, state);
// h_in of segment 0 is the row's initial state (or 0), then h_in[s+1] =
// exp(A dsum[s]) h_in[s] + h_end[s] in segment order; the row's final state and the sum
// of its segments' delta sums go to the caller's h_last / delta_sum.  h_end, dsum, h_in:
// (b * G, D, N), (b * G, D), (b * G, D, N).
__global__ void seg_combine_kernel(const ScanDev p, int G, const float* h_end, const float* dsum, float* h_in,
                                   float* h_last, float* dsum_out) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t total = (int64_t)p.b * p.D * p.N;
    if (i >= total) return;
    const int n = (int)(i % p.N);
    const int64_t bd = i / p.N;
    const int d = (int)(bd % p.D), b = (int)(bd / p.D);
    const float a = p.a_log ? -expf(p.A[(int64_t)d * p.N + n]) : p.A[(int64_t)d * p.N + n];
    float h = p.h0 ? p.h0[i] : 0.f;
    float ds = 0.f;
    for (int s = 0; s < G; ++s) {
        const int64_t rs = (int64_t)b * G + s;                 // the segment's row in the split view
        const int64_t o = (rs * p.D + d) * p.N + n;
        const float sd = dsum[rs * p.D + d];
        h_in[o] = h;
        h = expf(a * sd) * h + h_end[o];
        ds += sd;
    }
    if (h_last) h_last[i] = h;
    if (dsum_out && n == 0) dsum_out[bd] = ds;
}

cudaError_t launch_seg_combine(const ScanDev& p, int G, const float* h_end, const float* dsum, float* h_in,
                               float* h_last, float* dsum_out, cudaStream_t st) {
    const int64_t total = (int64_t)p.b * p.D * p.N;
    const int blocks = (int)((total + 255) / 256);
    seg_combine_kernel<<<blocks, 256, 0, st>>>(p, G, h_end, dsum, h_in, h_last, dsum_out);
    return cudaGetLastError();
}

}  // namespace swx
