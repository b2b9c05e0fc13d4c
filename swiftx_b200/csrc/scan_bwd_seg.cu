// Selective-scan backward for sm_100a, time-segmented.
//
// The reverse recurrence g_t = a_{t+1} g_{t+1} + dy_t C_t (models/selective_scan.py:146-148,
// :225-238) is linear in the carry that enters a stretch of time from its future, so the
// sequence is cut into segments that are walked in parallel:
//
//   1. summary (scan_bwd_summary_kernel): every sub-segment of sub_len steps after the
//      first segment is walked backwards from a zero carry; it leaves its local outgoing
//      carry Q = a_t0 g_t0 and the sum of its delta_eff (its decay is exp(A * sum)).
//   2. main (scan_bwd_seg_kernel): each CTA owns 64 channels of one row for one segment.
//      Its prologue chains the carries of the later sub-segments from the end of the
//      sequence, c <- Q + exp(A * S) c, to the value that enters its segment; then it
//      walks its 16-step checkpoint chunks last to first, starting from that carry.
//   3. finalize: fixed-order sums of the partials (dB, dC over channel blocks; dA, dD,
//      d(delta_bias) over segments and rows).
//
// Main kernel layout: a warp covers 16 channels x 16 states; lane (q, j) = (lane >> 2,
// lane & 3) owns channels 2q, 2q+1 of its warp and states 4j..4j+3 -- 8 state chains, so
// each B_t / C_t load from shared memory serves two channels and each per-channel scalar
// serves four states.  Per chunk the CTA
//   A. derives the per-(step, channel) scalars once (softplus(delta + bias) and its
//      derivative, delta*u, dy = dout*silu(z), the gate-gradient factor);
//   B. per warp: recomputes the chunk's states from the forward's checkpoint in two
//      8-step halves, keeping each half's states and decays in registers, and runs the
//      reverse recurrence over them.  The sum over the warp's 16 channels of the dB / dC
//      contributions and the sum over the 16 states of the du / d delta terms are
//      reduce-scatters through warp shuffles (no shared-memory hand-off);
//   C. finishes the per-(step, channel) gradients (du, d delta_raw, dz) with coalesced
//      stores and sums the four warps' dB / dC values into the CTA's partial row.
// Every sum is taken in a fixed order: the gradients are bit-reproducible (no atomics,
// unlike models/triton_scan.py:101-102,108-109).
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "launch_util.cuh"
#include "scan_params.cuh"
#include "tma_util.cuh"

namespace swx {

// TMA descriptors of the main kernel's inputs: (channel, step, row) tiles of 64 x 16 x 1
// for u, delta, z, dout and the saved pre-gate output, 16 x 16 x 1 for B and C.  `ok`:
// every descriptor was encoded (16-byte-aligned bases and strides); otherwise the kernel
// stages with per-thread cp.async.
struct SegMaps {
    CUtensorMap u, dl, z, dout, yp, B, C;
    int ok;
};

constexpr int SG_WARPS = 4;
constexpr int SG_CH = 16 * SG_WARPS;      // channels per CTA
constexpr int SG_THREADS = 32 * SG_WARPS;
constexpr int SG_HALF = TCK / 2;          // steps whose states / decays live in registers
constexpr int SG_RING = 2;                // raw staging slots
constexpr int SUM_THREADS = 128;          // summary kernel: one channel per thread
constexpr uint32_t SG_WAIT_POLLS = 1u << 24;   // mbarrier polls before a tile wait gives up

__device__ __forceinline__ float load_A_sg(const ScanDev& p, int64_t i) {
    const float a = p.A[i];
    return p.a_log ? -expf(a) : a;
}

// Four consecutive staged elements as fp32.
__device__ __forceinline__ float4 ld4s(const float* q) { return *reinterpret_cast<const float4*>(q); }
__device__ __forceinline__ float4 ld4s(const __nv_bfloat16* q) {
    const uint2 v = *reinterpret_cast<const uint2*>(q);
    return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u),
                       __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xffff0000u));
}

// Two adjacent outputs (8-byte fp32 / 4-byte bf16 store; the address is aligned to it).
__device__ __forceinline__ void store2(float* q, float2 v) { *reinterpret_cast<float2*>(q) = v; }
__device__ __forceinline__ void store2(__nv_bfloat16* q, float2 v) {
    *reinterpret_cast<__nv_bfloat162*>(q) = __floats2bfloat162_rn(v.x, v.y);
}

// ===================================================================== 1. summaries
// Thread = one channel of one row, all 16 states; walks its sub-segment backwards from a
// zero carry.  The sub-segment's C rows (the same for every thread of the CTA) are staged
// in shared memory once; the CTA's delta / dout / z rows arrive in 16-step blocks through
// a two-slot pipeline, one block ahead of the arithmetic: TMA tile copies issued by one
// thread (per-thread cp.async when a tensor is not 16-byte aligned).  The decays of the
// first SUM_FMA_PAIRS state pairs are computed on the FMA pipe (ex2x2_fma), the others on
// the MUFU unit, which this kernel otherwise saturates.
constexpr int SUM_MAXLEN = 128;           // longest sub-segment (sub_len <= 128)
constexpr int SUM_BLK = 16;               // steps per staged block
constexpr int SUM_FMA_PAIRS = 2;          // of the 8 state pairs

template <typename Tin>
struct SumSmem {
    float C[SUM_MAXLEN][NS];
    Tin dl[2][SUM_BLK][SUM_THREADS];
    Tin dout[2][SUM_BLK][SUM_THREADS];
    Tin z[2][SUM_BLK][SUM_THREADS];
    uint64_t mbar[2];                     // completion of each slot's TMA copies
};

// TMA descriptors of the summary kernel: (channel, step, row) tiles of 128 x 16 x 1 for
// delta, dout and z.  ok = 0: per-thread cp.async staging.
struct SumMaps {
    CUtensorMap dl, dout, z;
    int ok;
};

// GW (with HAS_Z): the forward applied the SiftX pathway mix before the gate, so the
// gate's input gradient carries the channel's group weight.
template <typename Tin, bool HAS_Z, bool GW = false>
__global__ void __launch_bounds__(SUM_THREADS)
    scan_bwd_summary_kernel(const ScanDev p, const __grid_constant__ SumMaps tm) {
    extern __shared__ __align__(128) unsigned char smem_raw[];   // TMA destinations: 128-byte aligned
    SumSmem<Tin>& S = *reinterpret_cast<SumSmem<Tin>*>(smem_raw);
    const int tid = threadIdx.x;
    const bool fast = tm.ok != 0;
    if (fast) {
        if (tid == 0) {
            mbar_init(&S.mbar[0], 1);
            mbar_init(&S.mbar[1], 1);
            mbar_fence_init();
        }
        __syncthreads();
    }
    const int nxb = (p.D + SUM_THREADS - 1) / SUM_THREADS;
    const int64_t blk = blockIdx.x;                      // (sub-segment, row, channel block)
    const int d0 = (int)(blk % nxb) * SUM_THREADS;
    const int d = d0 + tid;
    const int bi = (int)((blk / nxb) % p.b);
    const int ss = p.first_sub + (int)(blk / ((int64_t)nxb * p.b));
    const int nd = min(SUM_THREADS, p.D - d0);
    const bool ok = d < p.D;
    const int dc = ok ? d : p.D - 1;
    const int t0 = ss * p.sub_len, t1 = min(p.L, t0 + p.sub_len), nt = t1 - t0;
    const int nblk = (nt + SUM_BLK - 1) / SUM_BLK;
    const Tin* gdl = static_cast<const Tin*>(p.dl) + bi * p.dl_sb + d0;
    const Tin* gdo = static_cast<const Tin*>(p.dout) + bi * p.dout_sb + d0;
    const Tin* gz = HAS_Z ? static_cast<const Tin*>(p.z) + bi * p.z_sb + d0 : nullptr;
    const Tin* gC = static_cast<const Tin*>(p.C) + bi * p.C_sb;

    // block k of the walk covers steps [hi - SUM_BLK, hi), hi = t1 - k * SUM_BLK, clipped at t0
    // (the TMA tile always starts at hi - SUM_BLK >= 0: the rows before t0 are loaded, not used)
    bool stop = false;                                   // a tile wait gave up (all threads alike)
    constexpr uint32_t TILE_S = SUM_BLK * SUM_THREADS * sizeof(Tin);
    auto issue = [&](int k) {
        if (fast) {
            if (k < nblk && tid == 0 && !stop) {
                const int r = k & 1;
                fence_proxy_async_smem();                // the slot's last readers are past a barrier
                mbar_arrive_expect_tx(&S.mbar[r], (HAS_Z ? 3 : 2) * TILE_S);
                const int y = t1 - k * SUM_BLK - SUM_BLK;
                tma_load_3d(&S.dl[r][0][0], &tm.dl, d0, y, bi, &S.mbar[r]);
                tma_load_3d(&S.dout[r][0][0], &tm.dout, d0, y, bi, &S.mbar[r]);
                if (HAS_Z) tma_load_3d(&S.z[r][0][0], &tm.z, d0, y, bi, &S.mbar[r]);
            }
            return;
        }
        if (k < nblk) {
            const int hi = t1 - k * SUM_BLK, lo = max(t0, hi - SUM_BLK), rv = hi - lo, r = k & 1;
            stage_tile<Tin, SUM_THREADS>(&S.dl[r][0][0], gdl + (int64_t)lo * p.dl_sl, p.dl_sl, SUM_BLK, rv, nd,
                                         p.vec_dl, tid, SUM_THREADS);
            stage_tile<Tin, SUM_THREADS>(&S.dout[r][0][0], gdo + (int64_t)lo * p.dout_sl, p.dout_sl, SUM_BLK, rv,
                                         nd, p.vec_dout, tid, SUM_THREADS);
            if (HAS_Z)
                stage_tile<Tin, SUM_THREADS>(&S.z[r][0][0], gz + (int64_t)lo * p.z_sl, p.z_sl, SUM_BLK, rv, nd,
                                             p.vec_z, tid, SUM_THREADS);
        }
        cp_async_commit();
    };
    issue(0);
    for (int i = tid; i < nt * NS; i += SUM_THREADS) {
        const int row = i / NS, n = i % NS;
        S.C[row][n] = n < p.N ? Elem<Tin>::to_f(gC[(int64_t)(t0 + row) * p.C_sl + n]) : 0.f;
    }
    const float bias = p.dbias ? p.dbias[dc] : 0.f;
    const int grp = GW ? p.gof[dc] : 0;                  // pathway group of the channel
    float2 A2[NS / 2], g[NS / 2], an[NS / 2];
#pragma unroll
    for (int i = 0; i < NS / 2; ++i) {
        const float a0 = 2 * i < p.N ? load_A_sg(p, (int64_t)dc * p.N + 2 * i) * LOG2E : 0.f;
        const float a1 = 2 * i + 1 < p.N ? load_A_sg(p, (int64_t)dc * p.N + 2 * i + 1) * LOG2E : 0.f;
        A2[i] = f2(a0, a1);
        g[i] = an[i] = f2(0.f, 0.f);
    }
    float ssum = 0.f;
    for (int k = 0; k < nblk; ++k) {
        issue(k + 1);
        if (fast) {
            // bounded wait; one that gives up is recorded and stops further copies (the pass
            // then runs on what is in shared memory: incomplete results, intact context)
            bool ok = stop || mbar_wait_bounded(&S.mbar[k & 1], (k >> 1) & 1, SG_WAIT_POLLS);
            if (__syncthreads_or(!ok)) {
                if (!stop && tid == 0 && p.err) *p.err = SWX_ERR_TIMEOUT;
                stop = true;
            }
        } else {
            cp_async_wait<1>();
            __syncthreads();
        }
        const int hi = t1 - k * SUM_BLK, r = k & 1;
        const int base = fast ? hi - SUM_BLK : max(t0, hi - SUM_BLK);   // step of staged row 0
#pragma unroll 4
        for (int i = SUM_BLK - 1; i >= 0; --i) {
            const int t = hi - SUM_BLK + i;
            if (t < t0) break;
            const int row = t - base;
            const float raw = Elem<Tin>::to_f(S.dl[r][row][tid]) + bias;
            const float dov = Elem<Tin>::to_f(S.dout[r][row][tid]);
            const float dte = p.softplus ? softplus_f(raw) : raw;
            ssum += dte;
            float dy = HAS_Z ? dov * silu_f(Elem<Tin>::to_f(S.z[r][row][tid])) : dov;
            if (GW) dy *= p.gw[(int64_t)bi * p.gw_sb + (int64_t)t * p.gw_sl + grp];
            const float4* cr = reinterpret_cast<const float4*>(&S.C[t - t0][0]);
            const float2 dt2 = bc2(dte), dy2 = bc2(dy);
#pragma unroll
            for (int v = 0; v < NS / 4; ++v) {
                const float4 c4 = cr[v];
                g[2 * v] = fma2(an[2 * v], g[2 * v], mul2(dy2, f2(c4.x, c4.y)));
                g[2 * v + 1] = fma2(an[2 * v + 1], g[2 * v + 1], mul2(dy2, f2(c4.z, c4.w)));
                const float2 x0 = mul2(dt2, A2[2 * v]), x1 = mul2(dt2, A2[2 * v + 1]);
                an[2 * v] = 2 * v < SUM_FMA_PAIRS ? ex2x2_fma(x0) : ex2x2(x0);
                an[2 * v + 1] = 2 * v + 1 < SUM_FMA_PAIRS ? ex2x2_fma(x1) : ex2x2(x1);
            }
        }
        __syncthreads();                                  // slot r is refilled two blocks on
    }
    if (!fast) {
        cp_async_wait<0>();
    } else if (stop && tid == 0) {
        // the copies that may still be landing: the last block issued into each slot
        for (int k = max(0, nblk - 2); k < nblk; ++k) mbar_wait_bounded(&S.mbar[k & 1], (k >> 1) & 1, SG_WAIT_POLLS);
    }
    if (ok) {
        float* q = p.ws_q + (((int64_t)ss * p.b + bi) * p.D + d) * NS;
#pragma unroll
        for (int k = 0; k < NS / 4; ++k) {
            const float2 lo = mul2(an[2 * k], g[2 * k]), hi = mul2(an[2 * k + 1], g[2 * k + 1]);
            *reinterpret_cast<float4*>(q + 4 * k) = make_float4(lo.x, lo.y, hi.x, hi.y);
        }
        p.ws_s[((int64_t)ss * p.b + bi) * p.D + d] = ssum;
    }
}

// ===================================================================== 2. main kernel
template <typename Tin, bool YV>
struct SegSmem {
    Tin u[SG_RING][TCK][SG_CH];
    Tin dl[SG_RING][TCK][SG_CH];
    Tin z[SG_RING][TCK][SG_CH];
    Tin dout[SG_RING][TCK][SG_CH];
    float yp[SG_RING][TCK][SG_CH];         // pre-gate output saved by the forward (YPRE)
    Tin B[SG_RING][TCK][NS];
    Tin C[SG_RING][TCK][NS];
    float4 dd2[TCK][SG_CH / 2];            // (delta_eff, delta_eff * u) of a channel pair
    float2 dy2[TCK][SG_CH / 2];            // dy of a channel pair
    // (softplus', dz factor) of the even / odd channel of each pair.  In phase A the lanes
    // alternate even / odd channels: rows 40 float2 (16 banks) apart put a half-warp's even
    // and odd stores on disjoint banks; phase C reads consecutive pairs of one row
    float2 ee[TCK][2][SG_CH / 2 + 8];
    // per (state-group half jh, pair): (sum gB, sum g a h_prev A) of one channel of the pair
    // over that half's 8 states (channel jh after phase B's exchange), summed over the two
    // halves in phase C.  Rows padded to 36 float2: in phase B each half-warp stores 4 pairs
    // into each of the 4 rows of a step, and rows 36 float2 apart start 8 banks apart, so
    // the 16 stores cover 32 distinct banks; phase C reads consecutive pairs of one row
    float2 nsp[TCK][2][2][SG_CH / 2 + 4];
    // the same for the readout (without YPRE), one float each: rows 40 floats (8 banks) apart
    float ypv[YV ? TCK : 1][2][2][SG_CH / 2 + 8];
    float bcw[SG_WARPS][TCK][32];          // per-warp dB | dC sums over its 16 channels
    float red[4][SG_THREADS];
    uint64_t mbar[SG_RING];                // completion of each staging slot's TMA copies
};

// The states of one 8-step half: the chunk's states after each step and each step's
// decays, for the lane's 2 channels x 4 states as four float2 (c0 s01, c0 s23, c1 s01,
// c1 s23).
struct Half {
    float2 h[SG_HALF][4];
    float2 a[SG_HALF][4];
};

__device__ __forceinline__ void step_fwd(const float4 dd, const float4 b, const float2 (&A2)[4], float2 (&h)[4],
                                         float2 (&a)[4]) {
    const float2 dt0 = bc2(dd.x), du0 = bc2(dd.y), dt1 = bc2(dd.z), du1 = bc2(dd.w);
    const float2 b01 = f2(b.x, b.y), b23 = f2(b.z, b.w);
    a[0] = ex2x2(mul2(dt0, A2[0]));
    a[1] = ex2x2(mul2(dt0, A2[1]));
    a[2] = ex2x2(mul2(dt1, A2[2]));
    a[3] = ex2x2(mul2(dt1, A2[3]));
    h[0] = fma2(a[0], h[0], mul2(du0, b01));
    h[1] = fma2(a[1], h[1], mul2(du0, b23));
    h[2] = fma2(a[2], h[2], mul2(du1, b01));
    h[3] = fma2(a[3], h[3], mul2(du1, b23));
}

// One step of lane-wise reduce-scatter: lanes whose `bit` is clear keep the lower half of
// x (plus their partner's lower half), the others the upper half.
template <int K>
__device__ __forceinline__ void rs_round(float (&x)[2 * K], float (&y)[K], int lane, int bit) {
    const bool up = (lane & bit) != 0;
#pragma unroll
    for (int i = 0; i < K; ++i) {
        const float keep = up ? x[K + i] : x[i];
        const float send = up ? x[i] : x[K + i];
        y[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
    }
}

// Per-warp recurrence state of phase B.
struct LaneState {
    float2 A2[4], An[4];       // A * log2(e) and A for the lane's 2 channels x 4 states
    float2 g[4], an[4], dA[4]; // adjoint, decay of the later step, dA partial
};

// One half (HN = 8 steps, or fewer in a partial chunk when !FULL) of the reverse walk:
// recompute the half's states from `hstart`, then the reverse recurrence over them.
template <bool FULL, bool YV, typename Tin>
__device__ __forceinline__ void half_pass(SegSmem<Tin, YV>& S, int r, int tlo, int nh, int pair, int j, int lane,
                                          int warp, int slot, LaneState& L, const float2 (&hstart)[4]) {
    Half H;
    float2 h[4] = {hstart[0], hstart[1], hstart[2], hstart[3]};
#pragma unroll
    for (int t = 0; t < SG_HALF; ++t) {
        if (FULL || t < nh) {
            step_fwd(S.dd2[tlo + t][pair], ld4s(&S.B[r][tlo + t][4 * j]), L.A2, h, H.a[t]);
        } else {
            H.a[t][0] = H.a[t][1] = H.a[t][2] = H.a[t][3] = bc2(1.f);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) H.h[t][i] = h[i];
    }
#pragma unroll
    for (int t = SG_HALF - 1; t >= 0; --t) {
        if (!FULL && t >= nh) continue;
        const int tt = tlo + t;
        const float4 dd = S.dd2[tt][pair];
        const float2 dyv = S.dy2[tt][pair];
        const float4 b = ld4s(&S.B[r][tt][4 * j]);
        const float4 cc = ld4s(&S.C[r][tt][4 * j]);
        const float2 dy0 = bc2(dyv.x), dy1 = bc2(dyv.y);
        const float2 c01 = f2(cc.x, cc.y), c23 = f2(cc.z, cc.w);
        const float2 b01 = f2(b.x, b.y), b23 = f2(b.z, b.w);
        L.g[0] = fma2(L.an[0], L.g[0], mul2(dy0, c01));
        L.g[1] = fma2(L.an[1], L.g[1], mul2(dy0, c23));
        L.g[2] = fma2(L.an[2], L.g[2], mul2(dy1, c01));
        L.g[3] = fma2(L.an[3], L.g[3], mul2(dy1, c23));
        float2 w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 hp = t > 0 ? H.h[t > 0 ? t - 1 : 0][i] : hstart[i];
            w[i] = mul2(mul2(L.g[i], H.a[t][i]), hp);
        }
        const float2 dt0 = bc2(dd.x), dt1 = bc2(dd.z), du0 = bc2(dd.y), du1 = bc2(dd.w);
        L.dA[0] = fma2(w[0], dt0, L.dA[0]);
        L.dA[1] = fma2(w[1], dt0, L.dA[1]);
        L.dA[2] = fma2(w[2], dt1, L.dA[2]);
        L.dA[3] = fma2(w[3], dt1, L.dA[3]);
        const float2 sd0 = fma2(w[1], L.An[1], mul2(w[0], L.An[0]));
        const float2 sd1 = fma2(w[3], L.An[3], mul2(w[2], L.An[2]));
        const float2 sg0 = fma2(L.g[1], b23, mul2(L.g[0], b01));
        const float2 sg1 = fma2(L.g[3], b23, mul2(L.g[2], b01));
        // per-lane partial sums over its 4 states; one exchange with the lane of the other
        // state-group half (lane bit 1) leaves lane (q, j) with channel j >> 1 of its pair
        // summed over 8 states, and phase C adds the two halves
        {
            float z4[4] = {sg0.x + sg0.y, sd0.x + sd0.y, sg1.x + sg1.y, sd1.x + sd1.y};
            float z2[2];
            rs_round<2>(z4, z2, lane, 2);
            S.nsp[tt][j & 1][j >> 1][pair] = f2(z2[0], z2[1]);
        }
        if (YV) {
            const float2 y0 = fma2(H.h[t][1], c23, mul2(H.h[t][0], c01));
            const float2 y1 = fma2(H.h[t][3], c23, mul2(H.h[t][2], c01));
            float y2[2] = {y0.x + y0.y, y1.x + y1.y};
            float y1v[1];
            rs_round<1>(y2, y1v, lane, 2);
            S.ypv[tt][j & 1][j >> 1][pair] = y1v[0];
        }
        // dB_n = sum over the lane's two channels of g * delta*u; dC_n of dy * h; then the
        // sum over the warp's 8 channel pairs (lane bits 4, 3, 2): lane (q, j) ends with
        // value q of its state group
        const float2 db01 = fma2(L.g[2], du1, mul2(L.g[0], du0));
        const float2 db23 = fma2(L.g[3], du1, mul2(L.g[1], du0));
        const float2 dc01 = fma2(H.h[t][2], dy1, mul2(H.h[t][0], dy0));
        const float2 dc23 = fma2(H.h[t][3], dy1, mul2(H.h[t][1], dy0));
        float x8[8] = {db01.x, db01.y, db23.x, db23.y, dc01.x, dc01.y, dc23.x, dc23.y};
        float x4[4], x2[2], x1[1];
        rs_round<4>(x8, x4, lane, 16);
        rs_round<2>(x4, x2, lane, 8);
        rs_round<1>(x2, x1, lane, 4);
        S.bcw[warp][tt][slot] = x1[0];
#pragma unroll
        for (int i = 0; i < 4; ++i) L.an[i] = H.a[t][i];
    }
}

// Phase B for one checkpoint chunk: the first half's end state, then the second half and
// the first half walked in reverse.
template <bool FULL, bool YV, typename Tin>
__device__ __forceinline__ void chunk_pass(SegSmem<Tin, YV>& S, int r, int nt, int pair, int j, int lane, int warp,
                                           int slot, LaneState& L, const float2 (&hck)[4]) {
    float2 hmid[4] = {hck[0], hck[1], hck[2], hck[3]};
    if (FULL || nt > SG_HALF) {
#pragma unroll
        for (int t = 0; t < SG_HALF; ++t) {
            float2 a[4];
            step_fwd(S.dd2[t][pair], ld4s(&S.B[r][t][4 * j]), L.A2, hmid, a);
        }
    }
    // the second half, then the first (one copy of the code: the halves do not overlap)
#pragma unroll 1
    for (int half = 1; half >= 0; --half) {
        const int tlo = half * SG_HALF;
        const int nh = FULL ? SG_HALF : min(SG_HALF, nt - tlo);
        if (nh <= 0) continue;
        const float2 hs[4] = {half ? hmid[0] : hck[0], half ? hmid[1] : hck[1], half ? hmid[2] : hck[2],
                              half ? hmid[3] : hck[3]};
        half_pass<FULL, YV>(S, r, tlo, nh, pair, j, lane, warp, slot, L, hs);
    }
}

// DZS (with HAS_Z): dz has its own strides (the z half of a (b, L, 2D) gradient); without
// it dz is dense like du and dd and shares their offsets.
template <typename Tin, bool HAS_Z, bool YPRE, bool GW = false, bool DZS = false>
__global__ void __launch_bounds__(SG_THREADS, 2) scan_bwd_seg_kernel(const ScanDev p, const __grid_constant__ SegMaps tm) {
    constexpr bool YV = HAS_Z && !YPRE;
    extern __shared__ __align__(128) unsigned char smem_raw[];   // TMA destinations: 128-byte aligned
    SegSmem<Tin, YV>& S = *reinterpret_cast<SegSmem<Tin, YV>*>(smem_raw);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cblk = blockIdx.x, bi = blockIdx.y, seg = blockIdx.z;
    const int d0 = cblk * SG_CH;
    const int nd = min(SG_CH, p.D - d0);
    const int ts = seg * p.seg_len, te = min(p.L, ts + p.seg_len);
    const int ck0 = ts / TCK, nk = (te - ts + TCK - 1) / TCK;   // chunks of this segment

    const Tin* gu = static_cast<const Tin*>(p.u) + bi * p.u_sb + d0;
    const Tin* gdl = static_cast<const Tin*>(p.dl) + bi * p.dl_sb + d0;
    const Tin* gz = HAS_Z ? static_cast<const Tin*>(p.z) + bi * p.z_sb + d0 : nullptr;
    const Tin* gdo = static_cast<const Tin*>(p.dout) + bi * p.dout_sb + d0;
    const Tin* gB = static_cast<const Tin*>(p.B) + bi * p.B_sb;
    const Tin* gC = static_cast<const Tin*>(p.C) + bi * p.C_sb;
    const float* gyp = YPRE ? p.ypre + (int64_t)bi * p.L * p.D + d0 : nullptr;

    // staging.  When the inputs' bases and strides are 16-byte aligned (the common case),
    // one thread loads each input's whole 16-step tile with one TMA copy per tensor, all
    // completing on the slot's mbarrier (steps past L and channels past D read zeros);
    // otherwise every thread stages with 16-byte cp.async (stage_tile).
    const bool fast = tm.ok != 0;
    constexpr uint32_t TILE = TCK * SG_CH * sizeof(Tin), TILE_Y = TCK * SG_CH * 4, TILE_BC = TCK * NS * sizeof(Tin);
    if (fast) {
        if (tid == 0) {
            mbar_init(&S.mbar[0], 1);
            mbar_init(&S.mbar[1], 1);
            mbar_fence_init();
        }
        __syncthreads();
    }
    auto issue = [&](int k) {
        if (k < nk) {
            const int c = ck0 + nk - 1 - k, t0 = c * TCK, rv = min(TCK, p.L - t0), r = k & 1;
            if (fast) {
                if (tid == 0) {
                    fence_proxy_async_smem();            // the slot's last readers are past a barrier
                    const uint32_t bytes = (HAS_Z ? 4 : 3) * TILE + (YPRE ? TILE_Y : 0) + 2 * TILE_BC;
                    mbar_arrive_expect_tx(&S.mbar[r], bytes);
                    tma_load_3d(&S.u[r][0][0], &tm.u, d0, t0, bi, &S.mbar[r]);
                    tma_load_3d(&S.dl[r][0][0], &tm.dl, d0, t0, bi, &S.mbar[r]);
                    if (HAS_Z) tma_load_3d(&S.z[r][0][0], &tm.z, d0, t0, bi, &S.mbar[r]);
                    tma_load_3d(&S.dout[r][0][0], &tm.dout, d0, t0, bi, &S.mbar[r]);
                    if (YPRE) tma_load_3d(&S.yp[r][0][0], &tm.yp, d0, t0, bi, &S.mbar[r]);
                    tma_load_3d(&S.B[r][0][0], &tm.B, 0, t0, bi, &S.mbar[r]);
                    tma_load_3d(&S.C[r][0][0], &tm.C, 0, t0, bi, &S.mbar[r]);
                }
            } else {
                stage_tile<Tin, SG_CH>(&S.u[r][0][0], gu + t0 * p.u_sl, p.u_sl, TCK, rv, nd, p.vec_u, tid, SG_THREADS);
                stage_tile<Tin, SG_CH>(&S.dl[r][0][0], gdl + t0 * p.dl_sl, p.dl_sl, TCK, rv, nd, p.vec_dl, tid,
                                       SG_THREADS);
                if (HAS_Z)
                    stage_tile<Tin, SG_CH>(&S.z[r][0][0], gz + t0 * p.z_sl, p.z_sl, TCK, rv, nd, p.vec_z, tid,
                                           SG_THREADS);
                stage_tile<Tin, SG_CH>(&S.dout[r][0][0], gdo + t0 * p.dout_sl, p.dout_sl, TCK, rv, nd, p.vec_dout,
                                       tid, SG_THREADS);
                if (YPRE)
                    stage_tile<float, SG_CH>(&S.yp[r][0][0], gyp + (int64_t)t0 * p.D, p.D, TCK, rv, nd, p.vec_yp,
                                             tid, SG_THREADS);
                stage_tile<Tin, NS>(&S.B[r][0][0], gB + t0 * p.B_sl, p.B_sl, TCK, rv, p.N, p.vec_B, tid, SG_THREADS);
                stage_tile<Tin, NS>(&S.C[r][0][0], gC + t0 * p.C_sl, p.C_sl, TCK, rv, p.N, p.vec_C, tid, SG_THREADS);
            }
        }
        if (!fast) cp_async_commit();
    };
    // Wait for chunk k's inputs; false (every thread alike) if a bounded wait gave up.
    auto arrived = [&](int k) -> bool {
        bool ok = true;
        if (fast) ok = mbar_wait_bounded(&S.mbar[k & 1], (k >> 1) & 1, SG_WAIT_POLLS);
        else cp_async_wait<1>();
        const bool bad = __syncthreads_or(!ok);
        if (bad && tid == 0) {
            if (p.err) *p.err = SWX_ERR_TIMEOUT;
            // the copies still in flight (chunk k's and, if issued, chunk k+1's) write into
            // this CTA's shared memory: give each a second bounded wait before leaving
            mbar_wait_bounded(&S.mbar[k & 1], (k >> 1) & 1, SG_WAIT_POLLS);
            if (k + 1 < nk) mbar_wait_bounded(&S.mbar[(k + 1) & 1], ((k + 1) >> 1) & 1, SG_WAIT_POLLS);
        }
        return !bad;
    };

    // ---- per-thread roles
    // phase A: channel ech of the CTA, steps eh, eh + 2, ..., eh + 14
    const int ech = tid & (SG_CH - 1), eh = tid >> 6;
    const bool evalid = ech < nd;
    const float ebias = (p.dbias && evalid) ? p.dbias[d0 + ech] : 0.f;
    const int egroup = (GW && evalid) ? p.gof[d0 + ech] : 0;       // pathway group of the channel
    // phase C: channel pair cp (channels 2cp, 2cp + 1), steps ch4, ch4 + 4, ch4 + 8, ch4 + 12
    const int cpair = tid & 31, ch4 = tid >> 5;
    const bool cv0 = 2 * cpair < nd, cv1 = 2 * cpair + 1 < nd;
    const float2 cD = f2((p.Dskip && cv0) ? p.Dskip[d0 + 2 * cpair] : 0.f,
                         (p.Dskip && cv1) ? p.Dskip[d0 + 2 * cpair + 1] : 0.f);
    // phase B: lane (q, j) of warp `warp`
    const int q = lane >> 2, j = lane & 3;
    const int pair = 8 * warp + q;                       // channel pair within the CTA
    const int ca = d0 + 2 * pair;                        // its first channel
    const bool va = 2 * pair < nd, vb = 2 * pair + 1 < nd;
    LaneState Ls;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const bool v = c ? vb : va;
        float av[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int n = 4 * j + i;
            av[i] = (v && n < p.N) ? load_A_sg(p, (int64_t)(ca + c) * p.N + n) : 0.f;
        }
        Ls.An[2 * c] = f2(av[0], av[1]);
        Ls.An[2 * c + 1] = f2(av[2], av[3]);
        Ls.A2[2 * c] = mul2(Ls.An[2 * c], bc2(LOG2E));
        Ls.A2[2 * c + 1] = mul2(Ls.An[2 * c + 1], bc2(LOG2E));
        // the carry entering this segment from the later ones (zero for the last segment),
        // chained from the end of the sequence over the later sub-segments' summaries:
        // c <- Q_ss + exp(A * S_ss) * c.  g starts as that carry and the first step's
        // "a_{t+1}" is 1
        float2 c01 = bc2(0.f), c23 = bc2(0.f);
        if (v) {
            const int lo = (seg + 1) * (p.seg_len / p.sub_len);
#pragma unroll 4
            for (int ss = p.nsub - 1; ss >= lo; --ss) {
                const int64_t o = ((int64_t)ss * p.b + bi) * p.D + ca + c;
                const float2 sv = bc2(p.ws_s[o]);
                const float4 qv = *reinterpret_cast<const float4*>(p.ws_q + o * NS + 4 * j);
                c01 = fma2(ex2x2(mul2(Ls.A2[2 * c], sv)), c01, f2(qv.x, qv.y));
                c23 = fma2(ex2x2(mul2(Ls.A2[2 * c + 1], sv)), c23, f2(qv.z, qv.w));
            }
        }
        Ls.g[2 * c] = c01;
        Ls.g[2 * c + 1] = c23;
        Ls.an[2 * c] = Ls.an[2 * c + 1] = bc2(1.f);
        Ls.dA[2 * c] = Ls.dA[2 * c + 1] = bc2(0.f);
    }
    float2 accD = bc2(0.f), accB = bc2(0.f);
    // dB (q < 4) / dC (q >= 4) column of the value the lane ends up holding
    const int slot = q < 4 ? 4 * j + q : NS + 4 * j + (q - 4);

    issue(0);
    for (int k = 0; k < nk; ++k) {
        const int c = ck0 + nk - 1 - k, t0 = c * TCK, nt = min(TCK, p.L - t0), r = k & 1;
        issue(k + 1);
        if (!arrived(k)) return;                         // inputs never arrived: leave, flagged

        // ---------------------------------------------------------------- A: derive
#pragma unroll
        for (int m = 0; m < TCK / 2; m += 2) {
            const int ta = eh + 2 * m, tb = ta + 2;      // two steps of channel ech
            const float2 uv = f2(Elem<Tin>::to_f(S.u[r][ta][ech]), Elem<Tin>::to_f(S.u[r][tb][ech]));
            const float2 raw = add2(f2(Elem<Tin>::to_f(S.dl[r][ta][ech]), Elem<Tin>::to_f(S.dl[r][tb][ech])),
                                    bc2(ebias));
            float2 dov = f2(Elem<Tin>::to_f(S.dout[r][ta][ech]), Elem<Tin>::to_f(S.dout[r][tb][ech]));
            if (GW)                                      // the pathway mix scales the gate's input
                dov = mul2(dov, f2(ta < nt ? group_weight(p, bi, t0 + ta, egroup) : 0.f,
                                   tb < nt ? group_weight(p, bi, t0 + tb, egroup) : 0.f));
            float2 dte = raw, dsp = bc2(1.f);
            if (p.softplus) softplus2(raw, dte, dsp);
            float2 dy = dov, qz = bc2(0.f);
            if (HAS_Z) {
                const float2 zv = f2(Elem<Tin>::to_f(S.z[r][ta][ech]), Elem<Tin>::to_f(S.z[r][tb][ech]));
                const float2 sg = sigmoid2(zv);
                dy = mul2(dov, mul2(zv, sg));
                // d silu / dz = sg * (1 + z * (1 - sg))
                qz = mul2(mul2(dov, sg), fma2(zv, add2(bc2(1.f), mul2(sg, bc2(-1.f))), bc2(1.f)));
            }
            if (!evalid) dte = dy = bc2(0.f);            // padding channels stay inert
            const float2 du = mul2(dte, uv);
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
                const int t = h2 ? tb : ta;
                const float dt_ = h2 ? dte.y : dte.x, du_ = h2 ? du.y : du.x, dy_ = h2 ? dy.y : dy.x;
                float2* d2 = reinterpret_cast<float2*>(&S.dd2[t][ech >> 1]) + (ech & 1);
                *d2 = f2(dt_, du_);
                reinterpret_cast<float*>(&S.dy2[t][ech >> 1])[ech & 1] = dy_;
                S.ee[t][ech & 1][ech >> 1] = f2(h2 ? dsp.y : dsp.x, h2 ? qz.y : qz.x);
            }
        }
        __syncthreads();

        // ---------------------------------------------------------------- B: recurrence
        {
            float2 hck[4];
            if (va || vb) {
                const float* ckp = p.ck + (((int64_t)bi * p.nck + c) * p.D + ca) * NS + 4 * j;
                const float4 x0 = va ? *reinterpret_cast<const float4*>(ckp) : make_float4(0.f, 0.f, 0.f, 0.f);
                const float4 x1 = vb ? *reinterpret_cast<const float4*>(ckp + NS) : make_float4(0.f, 0.f, 0.f, 0.f);
                hck[0] = f2(x0.x, x0.y); hck[1] = f2(x0.z, x0.w);
                hck[2] = f2(x1.x, x1.y); hck[3] = f2(x1.z, x1.w);
            } else {
                hck[0] = hck[1] = hck[2] = hck[3] = bc2(0.f);
            }
            if (nt == TCK) chunk_pass<true, YV>(S, r, nt, pair, j, lane, warp, slot, Ls, hck);
            else chunk_pass<false, YV>(S, r, nt, pair, j, lane, warp, slot, Ls, hck);
        }
        __syncthreads();

        // ---------------------------------------------------------------- C: epilogue
        {
            const int64_t orow = (int64_t)bi * p.L * p.D + d0 + 2 * cpair;
            Tin* gdu = static_cast<Tin*>(p.du) + orow;
            Tin* gddl = static_cast<Tin*>(p.ddl) + orow;
            Tin* gdz = HAS_Z ? static_cast<Tin*>(p.dz) + (DZS ? (int64_t)bi * p.dz_sb + d0 + 2 * cpair : orow)
                             : nullptr;
            const bool pair_out = cv1 && (p.D % 2 == 0);   // both channels, 2-element aligned rows
            // strided dz: paired stores only where its strides and base keep every pair aligned
            const bool pair_dz = pair_out && (!DZS || (((p.dz_sb | p.dz_sl) & 1) == 0 &&
                                 (reinterpret_cast<uintptr_t>(p.dz) % (2 * sizeof(Tin))) == 0));
#pragma unroll
            for (int m = 0; m < TCK / 4; ++m) {
                const int t = ch4 + 4 * m;
                if (t < nt && cv0) {
                    // the two state-group halves' partial sums of this pair's two channels
                    const float2 a0 = S.nsp[t][0][0][cpair], a1 = S.nsp[t][1][0][cpair];   // channel 0
                    const float2 b0 = S.nsp[t][0][1][cpair], b1 = S.nsp[t][1][1][cpair];   // channel 1
                    const float2 sgB = f2(a0.x + a1.x, b0.x + b1.x), sdA = f2(a0.y + a1.y, b0.y + b1.y);
                    const float2 e0 = S.ee[t][0][cpair], e1 = S.ee[t][1][cpair];           // (sp', q)
                    const float4 dd = S.dd2[t][cpair];
                    const float2 dyy = S.dy2[t][cpair];
                    const float2 uu = f2(Elem<Tin>::to_f(S.u[r][t][2 * cpair]), Elem<Tin>::to_f(S.u[r][t][2 * cpair + 1]));
                    const float2 dsp = f2(e0.x, e1.x), qq = f2(e0.y, e1.y);
                    const float2 du = fma2(f2(dd.x, dd.z), sgB, mul2(cD, dyy));
                    const float2 draw = mul2(fma2(uu, sgB, sdA), dsp);
                    float2 dz = bc2(0.f);
                    if (HAS_Z) {
                        float2 y;
                        if (YPRE) {
                            y = *reinterpret_cast<const float2*>(&S.yp[r][t][2 * cpair]);
                        } else {
                            y = fma2(cD, uu, f2(S.ypv[YV ? t : 0][0][0][cpair] + S.ypv[YV ? t : 0][1][0][cpair],
                                                S.ypv[YV ? t : 0][0][1][cpair] + S.ypv[YV ? t : 0][1][1][cpair]));
                        }
                        dz = mul2(qq, y);
                    }
                    const int64_t o = (int64_t)(t0 + t) * p.D;
                    if (pair_out) {
                        store2(gdu + o, du);
                        store2(gddl + o, draw);
                        if (HAS_Z && !DZS) store2(gdz + o, dz);
                    } else {
                        gdu[o] = Elem<Tin>::from_f(du.x);
                        gddl[o] = Elem<Tin>::from_f(draw.x);
                        if (HAS_Z && !DZS) gdz[o] = Elem<Tin>::from_f(dz.x);
                        if (cv1) {
                            gdu[o + 1] = Elem<Tin>::from_f(du.y);
                            gddl[o + 1] = Elem<Tin>::from_f(draw.y);
                            if (HAS_Z && !DZS) gdz[o + 1] = Elem<Tin>::from_f(dz.y);
                        }
                    }
                    if (HAS_Z && DZS) {
                        const int64_t oz = (int64_t)(t0 + t) * p.dz_sl;
                        if (pair_dz) {
                            store2(gdz + oz, dz);
                        } else {
                            gdz[oz] = Elem<Tin>::from_f(dz.x);
                            if (cv1) gdz[oz + 1] = Elem<Tin>::from_f(dz.y);
                        }
                    }
                    accD = fma2(dyy, uu, accD);
                    accB = add2(accB, draw);
                }
            }
            // the CTA's dB | dC partial row: the four warps' sums in warp order
            float* wbc = p.ws_bc + ((int64_t)cblk * p.b + bi) * p.L * 2 * NS;
#pragma unroll
            for (int m = 0; m < TCK * 32 / SG_THREADS; ++m) {
                const int t = (tid >> 5) + m * (SG_THREADS / 32), s2 = tid & 31;
                if (t < nt) {
                    const float v = ((S.bcw[0][t][s2] + S.bcw[1][t][s2]) + S.bcw[2][t][s2]) + S.bcw[3][t][s2];
                    wbc[(int64_t)(t0 + t) * 2 * NS + s2] = v;
                }
            }
        }
        __syncthreads();
    }
    cp_async_wait<0>();

    // ---- per-segment partials: dA per (channel, state), dD / d(delta_bias) per channel
    const int64_t prow = (int64_t)seg * p.b + bi;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        if (c ? vb : va) {
            *reinterpret_cast<float4*>(p.ws_a + (prow * p.D + ca + c) * NS + 4 * j) =
                make_float4(Ls.dA[2 * c].x, Ls.dA[2 * c].y, Ls.dA[2 * c + 1].x, Ls.dA[2 * c + 1].y);
            if (p.dh0 && seg == 0) {
                const float hv[4] = {Ls.an[2 * c].x * Ls.g[2 * c].x, Ls.an[2 * c].y * Ls.g[2 * c].y,
                                     Ls.an[2 * c + 1].x * Ls.g[2 * c + 1].x, Ls.an[2 * c + 1].y * Ls.g[2 * c + 1].y};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int n = 4 * j + i;
                    if (n < p.N) p.dh0[((int64_t)bi * p.D + ca + c) * p.N + n] = hv[i];
                }
            }
        }
    }
    // each channel pair's sums from the four threads that handled its steps, in order
    S.red[0][tid] = accD.x;
    S.red[1][tid] = accD.y;
    S.red[2][tid] = accB.x;
    S.red[3][tid] = accB.y;
    __syncthreads();
    if (tid < SG_CH && tid < nd) {
        const int pr = tid >> 1, hi = tid & 1;
        float sD = 0.f, sB = 0.f;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            sD += S.red[hi][pr + 32 * m];
            sB += S.red[2 + hi][pr + 32 * m];
        }
        p.ws_d[prow * p.D + d0 + tid] = sD;
        p.ws_bias[prow * p.D + d0 + tid] = sB;
    }
}

// ===================================================================== 3. finalize
template <typename Tin>
__global__ void scan_bwd_seg_finalize_kernel(const ScanDev p) {
    const int64_t nrow = (int64_t)p.b * p.L;
    const int64_t nbc = nrow * 2 * NS;
    const int64_t total = nbc + (int64_t)p.D * p.N + p.D;
    const int64_t slab = nrow * 2 * NS;
    const int nparts = p.nseg * p.b;                           // (segment, row) partials
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        if (i < nbc) {
            const int col = (int)(i & (2 * NS - 1));
            const int kind = col >= NS, n = col & (NS - 1);
            if (n >= p.N) continue;
            const float* src = p.ws_bc + i;
            float s = 0.f;
#pragma unroll 8
            for (int k = 0; k < p.nblk64; ++k) s += src[(int64_t)k * slab];
            Tin* dst = static_cast<Tin*>(kind ? p.dC : p.dB);
            dst[(i >> 5) * p.N + n] = Elem<Tin>::from_f(s);
        } else if (i < nbc + (int64_t)p.D * p.N) {
            const int64_t r = i - nbc;
            const int dd = (int)(r / p.N), n = (int)(r % p.N);
            float s = 0.f;
            for (int k = 0; k < nparts; ++k) s += p.ws_a[((int64_t)k * p.D + dd) * NS + n];
            p.dA[r] = p.a_log ? s * load_A_sg(p, r) : s;        // d/dA_log = dA * A
        } else {
            const int dd = (int)(i - nbc - (int64_t)p.D * p.N);
            float sD = 0.f, sB = 0.f;
            for (int k = 0; k < nparts; ++k) {
                sD += p.ws_d[(int64_t)k * p.D + dd];
                sB += p.ws_bias[(int64_t)k * p.D + dd];
            }
            if (p.dD) p.dD[dd] = sD;
            if (p.ddbias) p.ddbias[dd] = sB;
        }
    }
}

// ===================================================================== launchers
template <typename Tin, bool HAS_Z>
static SegMaps seg_maps(const ScanDev& p) {
    SegMaps m{};
    const int es = sizeof(Tin);
    bool ok = encode_3d(&m.u, p.u, es, p.D, p.L, p.b, p.u_sl, p.u_sb, SG_CH, TCK) &&
              encode_3d(&m.dl, p.dl, es, p.D, p.L, p.b, p.dl_sl, p.dl_sb, SG_CH, TCK) &&
              encode_3d(&m.dout, p.dout, es, p.D, p.L, p.b, p.dout_sl, p.dout_sb, SG_CH, TCK) &&
              encode_3d(&m.B, p.B, es, p.N, p.L, p.b, p.B_sl, p.B_sb, NS, TCK) &&
              encode_3d(&m.C, p.C, es, p.N, p.L, p.b, p.C_sl, p.C_sb, NS, TCK);
    if (ok && HAS_Z) ok = encode_3d(&m.z, p.z, es, p.D, p.L, p.b, p.z_sl, p.z_sb, SG_CH, TCK);
    if (ok && HAS_Z && p.ypre) ok = encode_3d(&m.yp, p.ypre, 4, p.D, p.L, p.b, p.D, (int64_t)p.L * p.D, SG_CH, TCK);
    m.ok = ok ? 1 : 0;
    return m;
}

template <typename Tin, bool HAS_Z>
static cudaError_t launch_seg_t(const ScanDev& p0, cudaStream_t st) {
    cudaError_t e;
    ScanDev p = p0;
    p.err = wait_status_address();               // where a timed-out tile wait is recorded
    if (p.nseg > 1) {
        const int64_t nsum = p.nsub - p.first_sub;
        const int64_t gs = (int64_t)((p.D + SUM_THREADS - 1) / SUM_THREADS) * p.b * nsum;
        if (gs > INT32_MAX) return cudaErrorInvalidConfiguration;
        auto ks = scan_bwd_summary_kernel<Tin, HAS_Z>;
        if constexpr (HAS_Z) {
            if (p.gw) ks = scan_bwd_summary_kernel<Tin, true, true>;
        }
        const int ssm = sizeof(SumSmem<Tin>);
        if ((e = allow_smem(ks, ssm)) != cudaSuccess) return e;
        SumMaps sm{};
        const int es = sizeof(Tin);
        bool ok = encode_3d(&sm.dl, p.dl, es, p.D, p.L, p.b, p.dl_sl, p.dl_sb, SUM_THREADS, SUM_BLK) &&
                  encode_3d(&sm.dout, p.dout, es, p.D, p.L, p.b, p.dout_sl, p.dout_sb, SUM_THREADS, SUM_BLK);
        if (ok && HAS_Z) ok = encode_3d(&sm.z, p.z, es, p.D, p.L, p.b, p.z_sl, p.z_sb, SUM_THREADS, SUM_BLK);
        sm.ok = ok ? 1 : 0;
        ks<<<(unsigned)gs, SUM_THREADS, ssm, st>>>(p, sm);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    const bool ypre = HAS_Z && p.ypre;
    auto k = ypre ? scan_bwd_seg_kernel<Tin, HAS_Z, true> : scan_bwd_seg_kernel<Tin, HAS_Z, false>;
    if constexpr (HAS_Z) {
        const bool dzs = p.dz_sl != p.D || p.dz_sb != (int64_t)p.L * p.D;    // strided dz
        if (p.gw && dzs)
            k = ypre ? scan_bwd_seg_kernel<Tin, true, true, true, true> : scan_bwd_seg_kernel<Tin, true, false, true, true>;
        else if (p.gw)
            k = ypre ? scan_bwd_seg_kernel<Tin, true, true, true> : scan_bwd_seg_kernel<Tin, true, false, true>;
        else if (dzs)
            k = ypre ? scan_bwd_seg_kernel<Tin, true, true, false, true> : scan_bwd_seg_kernel<Tin, true, false, false, true>;
    }
    const int smem = ypre ? sizeof(SegSmem<Tin, false>) : sizeof(SegSmem<Tin, HAS_Z>);
    if ((e = allow_smem(k, smem)) != cudaSuccess) return e;
    dim3 grid(p.nblk64, p.b, p.nseg);
    k<<<grid, SG_THREADS, smem, st>>>(p, seg_maps<Tin, HAS_Z>(p));
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const int64_t total = 2LL * NS * p.b * p.L + (int64_t)p.D * p.N + p.D;
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 8);
    scan_bwd_seg_finalize_kernel<Tin><<<blocks, 256, 0, st>>>(p);
    return cudaGetLastError();
}

template <typename Tin, bool HAS_Z>
static cudaError_t seg_ctas_per_sm_t(const ScanDev& p, int* ctas) {
    const bool ypre = HAS_Z && p.ypre;
    auto k = ypre ? scan_bwd_seg_kernel<Tin, HAS_Z, true> : scan_bwd_seg_kernel<Tin, HAS_Z, false>;
    const int smem = ypre ? sizeof(SegSmem<Tin, false>) : sizeof(SegSmem<Tin, HAS_Z>);
    cudaError_t e = allow_smem(k, smem);
    if (e != cudaSuccess) return e;
    int sms = 0;
    return sm_fit(k, SG_THREADS, smem, &sms, ctas);
}

cudaError_t scan_bwd_seg_ctas_per_sm(const ScanDev& p, int in_dtype, bool has_z, int* ctas) {
    if (in_dtype == SWX_DTYPE_F32)
        return has_z ? seg_ctas_per_sm_t<float, true>(p, ctas) : seg_ctas_per_sm_t<float, false>(p, ctas);
    return has_z ? seg_ctas_per_sm_t<__nv_bfloat16, true>(p, ctas) : seg_ctas_per_sm_t<__nv_bfloat16, false>(p, ctas);
}

cudaError_t launch_scan_bwd_seg(const ScanDev& p, int in_dtype, bool has_z, cudaStream_t st) {
    if (in_dtype == SWX_DTYPE_F32)
        return has_z ? launch_seg_t<float, true>(p, st) : launch_seg_t<float, false>(p, st);
    return has_z ? launch_seg_t<__nv_bfloat16, true>(p, st) : launch_seg_t<__nv_bfloat16, false>(p, st);
}

}  // namespace swx
