// Selective-scan backward over whole rows, for bf16 grids that fill the GPU.
//
// One CTA owns 32 channels of one batch row for the whole sequence (walked last chunk to
// first), warp-specialised: 4 recurrence warps (thread = one channel x 4 of its 16
// states) and 4 helper warps (staging, per-(t, channel) scalars, epilogues), handing
// 4-step tiles over through shared memory and named barriers; built for two CTAs per SM
// (at most 128 registers a thread).  When a bf16 problem has at least one such CTA per
// SM (batch rows x 32-channel blocks >= SM count) this runs instead of the time-segmented
// backward (scan_bwd_seg.cu), which it beats there (the Sift LM block: 16 rows x 512
// channels x 512 steps, ~130 us against ~167 us); the segmented kernel covers everything
// else.  Per 16-step chunk the recurrence warps reload the checkpoint, recompute the
// states into registers and run g_t = a_{t+1} g_{t+1} + dy_t C_t (models/selective_scan.py
// :146-148); every reduction is a fixed-order sum (no float atomics).  Tiles arrive by TMA
// (one helper thread, completion on the ring slot's mbarrier, bounded waits), or by
// per-thread cp.async when a tensor is not 16-byte aligned.
#include <algorithm>

#include "common.cuh"
#include "launch_util.cuh"
#include "scan_params.cuh"
#include "tma_util.cuh"

namespace swx {
namespace rowk {

constexpr int SCH = 32;               // channels per CTA
constexpr int NSCAN = 128;            // recurrence threads
constexpr int NAUX = 128;             // helper threads
constexpr int NTH = NSCAN + NAUX;
constexpr int HT = TCK / 2;
constexpr int RING = 4;               // raw staging slots

enum : int { BAR_AUX = 1, BAR_D0 = 2, BAR_X0 = 4, BAR_E0 = 6 };
constexpr uint32_t ROW_WAIT_POLLS = 1u << 24;   // mbarrier polls before a tile wait gives up

// TMA descriptors: (channel, step, row) tiles of 32 x 16 x 1 for u, delta, z, dout and the
// saved pre-gate output, 16 x 16 x 1 for B and C.  ok = 0: per-thread cp.async staging.
struct RowMaps {
    CUtensorMap u, dl, z, dout, yp, B, C;
    int ok;
};

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ld4(const __nv_bfloat16* p) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u),
                       __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xffff0000u));
}

__device__ __forceinline__ float load_A(const ScanDev& p, int64_t i) {
    const float a = p.A[i];
    return p.a_log ? -expf(a) : a;
}

// =============================================================== backward
template <typename Tin, int HTQ>
struct BwdSmem {
    Tin u[RING][TCK][SCH];
    Tin dl[RING][TCK][SCH];
    Tin z[RING][TCK][SCH];
    Tin dout[RING][TCK][SCH];
    Tin B[RING][TCK][NS];
    Tin C[RING][TCK][NS];
    float2 dd[2][TCK][SCH];            // (delta_eff, delta_eff * u)
    float dy[2][TCK][SCH];             // dy = dout * silu(z) (or dout)
    float4 ee[2][TCK][SCH];            // (u, d delta_eff / d delta_raw, dout * silu'(z), dy)
    float yp[RING][TCK][SCH];          // pre-gate output saved by the forward (YPRE)
    float bc[2][HTQ][SCH][2 * NS];     // per-channel dB | dC contributions of a hand-off tile; the
                                       // two 16-wide halves swap on odd channels (conflict-free stores)
    float2 nsd[2][HTQ][SCH][4];        // per state group: (sum g*B, sum g*a*h_prev*A)
    float nyp[2][HTQ][SCH][4];         // per state group: sum h*C (gate without YPRE)
    float red[2][NAUX];
    uint64_t mbar[RING];               // completion of each ring slot's TMA copies
    int stop;                          // a tile wait gave up: no further copies, no further waits
};

// Recompute the 16 states of a chunk from its checkpoint (and, without a saved pre-gate
// output, the partial readouts); bv receives each step's decays (AREG) or its B.  FULL
// chunks are branch-free so the scheduler can overlap the steps' loads and exponentials
// with the state chain.
template <bool FULL, bool YV, bool AREG, typename Tin>
__device__ __forceinline__ void bwd_recompute(const float2 (*__restrict__ dd)[SCH], const Tin (*__restrict__ Bs)[NS],
                                              const Tin (*__restrict__ Cs)[NS], int nt, int ch, int j,
                                              float2 A01, float2 A23, float2 hck01, float2 hck23,
                                              float2 (&hs01)[TCK], float2 (&hs23)[TCK], float4 (&bv)[TCK],
                                              float (&yv)[TCK]) {
    float2 h01 = hck01, h23 = hck23;
#pragma unroll
    for (int t = 0; t < TCK; ++t) {
        if (FULL || t < nt) {
            const float2 dv = dd[t][ch];
            const float4 b = ld4(&Bs[t][4 * j]);
            const float2 dt = bc2(dv.x), du = bc2(dv.y);
            const float2 a01 = ex2x2(mul2(dt, A01)), a23 = ex2x2(mul2(dt, A23));
            bv[t] = AREG ? make_float4(a01.x, a01.y, a23.x, a23.y) : b;
            h01 = fma2(a01, h01, mul2(du, f2(b.x, b.y)));
            h23 = fma2(a23, h23, mul2(du, f2(b.z, b.w)));
            hs01[t] = h01;
            hs23[t] = h23;
            if (YV) {
                const float4 cc = ld4(&Cs[t][4 * j]);
                float2 y = mul2(h01, f2(cc.x, cc.y));
                y = fma2(h23, f2(cc.z, cc.w), y);
                yv[t] = y.x + y.y;
            } else {
                yv[t] = 0.f;
            }
        } else {
            hs01[t] = hs23[t] = f2(0.f, 0.f);
            bv[t] = make_float4(0.f, 0.f, 0.f, 0.f);
            yv[t] = 0.f;
        }
    }
}

// One hand-off tile (HTQ steps, processed last to first) of the reverse recurrence.  The
// states come from the chunk's registers.  AREG (one CTA per SM): the recompute pass
// left each step's decays in bv, so this pass needs no exponential, and B comes from
// shared memory.  Otherwise bv holds B (or, NOBV, the two-CTAs-per-SM variant at most
// 128 registers a thread, B comes from shared memory too) and the decays are
// recomputed here (one exp per element).  Both give the same bits.
template <bool FULL, bool YV, int HTQ, bool NOBV, bool AREG, typename Tin>
__device__ __forceinline__ void bwd_half(const float2 (*__restrict__ dd)[SCH], const float (*__restrict__ dyv)[SCH],
                                         const Tin (*__restrict__ Bs)[NS], const Tin (*__restrict__ Cs)[NS],
                                         float (*__restrict__ bc)[SCH][2 * NS], float2 (*__restrict__ nsd)[SCH][4],
                                         float (*__restrict__ nyp)[SCH][4],
                                         int tlo, int nt, int ch, int j, float2 A01, float2 A23,
                                         const float4 (&bv)[TCK], const float2 (&hs01)[TCK], const float2 (&hs23)[TCK],
                                         const float (&yv)[TCK], float2 hck01, float2 hck23,
                                         float2 An01, float2 An23, float2& g01, float2& g23,
                                         float2& an01, float2& an23, float2& dA01, float2& dA23) {
    const int colB = (ch & 1) * NS + 4 * j;           // swizzled dB / dC columns
    const int colC = ((ch & 1) ^ 1) * NS + 4 * j;
    constexpr bool BSM = NOBV || AREG;                // B from shared memory
    // the next (earlier) step's shared-memory inputs are loaded before this step's stores
    float2 dn = dd[tlo + HTQ - 1][ch];
    float dyn = dyv[tlo + HTQ - 1][ch];
    float4 cn = ld4(&Cs[tlo + HTQ - 1][4 * j]);
    float4 bn = BSM ? ld4(&Bs[tlo + HTQ - 1][4 * j]) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int tt = HTQ - 1; tt >= 0; --tt) {
        const int t = tlo + tt;
        const float2 d = dn;
        const float2 dy = bc2(dyn);
        const float4 c = cn;
        const float4 b = BSM ? bn : bv[t];
        if (tt > 0) {
            dn = dd[t - 1][ch];
            dyn = dyv[t - 1][ch];
            cn = ld4(&Cs[t - 1][4 * j]);
            if (BSM) bn = ld4(&Bs[t - 1][4 * j]);
        }
        if (FULL || t < nt) {
            const float2 dte = bc2(d.x);
            float2 a01, a23;
            if (AREG) {
                a01 = f2(bv[t].x, bv[t].y);
                a23 = f2(bv[t].z, bv[t].w);
            } else {
                a01 = ex2x2(mul2(dte, A01));
                a23 = ex2x2(mul2(dte, A23));
            }
            g01 = fma2(an01, g01, mul2(dy, f2(c.x, c.y)));
            g23 = fma2(an23, g23, mul2(dy, f2(c.z, c.w)));
            const float2 du = bc2(d.y);
            const float2 db01 = mul2(g01, du), db23 = mul2(g23, du);
            const float2 dc01 = mul2(dy, hs01[t]), dc23 = mul2(dy, hs23[t]);
            *reinterpret_cast<float4*>(&bc[tt][ch][colB]) = make_float4(db01.x, db01.y, db23.x, db23.y);
            *reinterpret_cast<float4*>(&bc[tt][ch][colC]) = make_float4(dc01.x, dc01.y, dc23.x, dc23.y);
            float2 sg = mul2(g01, f2(b.x, b.y));
            sg = fma2(g23, f2(b.z, b.w), sg);
            const float2 hp01 = (t > 0) ? hs01[t > 0 ? t - 1 : 0] : hck01;
            const float2 hp23 = (t > 0) ? hs23[t > 0 ? t - 1 : 0] : hck23;
            const float2 w01 = mul2(mul2(g01, a01), hp01);
            const float2 w23 = mul2(mul2(g23, a23), hp23);
            dA01 = fma2(w01, dte, dA01);
            dA23 = fma2(w23, dte, dA23);
            float2 sd = mul2(w01, An01);
            sd = fma2(w23, An23, sd);
            nsd[tt][ch][j] = f2(sg.x + sg.y, sd.x + sd.y);
            if (YV) nyp[tt][ch][j] = yv[t];
            an01 = a01;
            an23 = a23;
        }
    }
}

// YPRE: the forward saved the pre-gate output, so the gate gradient reads it instead
// of recomputing the readout (which would need C in the recompute pass).
//
// LOWREG: the variant for grids larger than the SM count, built for two CTAs per SM (at
// most 128 registers a thread, about 100 KB of shared memory with bf16 inputs): B is
// reloaded from shared memory in the reverse pass instead of kept in registers, and the
// per-step results are handed to the helper warps in 4-step tiles instead of 8.
// GW (with HAS_Z): the forward applied the SiftX pathway mix before the gate.
// DZS (with HAS_Z): dz has its own strides (the z half of a (b, L, 2D) gradient).
template <typename Tin, bool HAS_Z, bool YPRE, bool LOWREG, bool GW = false, bool DZS = false>
__global__ void __launch_bounds__(NTH, LOWREG ? 2 : 1) scan_bwd_kernel(const ScanDev p, const __grid_constant__ RowMaps tm) {
    constexpr bool YV = HAS_Z && !YPRE;
    constexpr int HTQ = LOWREG ? 4 : HT;       // steps per hand-off tile
    constexpr int NQ = TCK / HTQ;              // hand-off tiles per chunk
    constexpr bool AREG = !LOWREG;             // decays kept in registers (see bwd_half)
    extern __shared__ __align__(128) unsigned char smem_raw[];   // TMA destinations: 128-byte aligned
    BwdSmem<Tin, HTQ>& S = *reinterpret_cast<BwdSmem<Tin, HTQ>*>(smem_raw);

    const int tid = threadIdx.x;
    const int bi = blockIdx.y;
    const int d0 = blockIdx.x * SCH;
    const int nd = min(SCH, p.D - d0);
    const int nck = p.nck;
    const bool fast = tm.ok != 0;
    if (fast) {
        if (tid == 0) {
#pragma unroll
            for (int r = 0; r < RING; ++r) mbar_init(&S.mbar[r], 1);
            mbar_fence_init();
            S.stop = 0;
        }
        __syncthreads();
    }

    if (tid < NSCAN) {
        // ------------------------------------------------ recurrence warps
        const int ch = tid >> 2, j = tid & 3;
        const int d = d0 + ch;
        const bool dvalid = ch < nd;
        float av[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int n = 4 * j + i;
            av[i] = (dvalid && n < p.N) ? load_A(p, (int64_t)d * p.N + n) : 0.f;
        }
        const float2 An01 = f2(av[0], av[1]), An23 = f2(av[2], av[3]);
        const float2 A01 = mul2(An01, bc2(LOG2E)), A23 = mul2(An23, bc2(LOG2E));
        float2 g01 = f2(0.f, 0.f), g23 = g01, an01 = g01, an23 = g01, dA01 = g01, dA23 = g01;

        for (int k = 0; k < nck; ++k) {
            const int c = nck - 1 - k, s = k & 1, r = k % RING, t0 = c * TCK, nt = min(TCK, p.L - t0);
            bar_sync(BAR_D0 + s, NTH);
            // the helpers waited for this chunk before deriving it; the wait here orders the
            // bulk copies' writes of B / C before this thread's reads (it returns at once)
            if (fast && !*reinterpret_cast<volatile int*>(&S.stop))
                mbar_wait_bounded(&S.mbar[r], (k / RING) & 1, ROW_WAIT_POLLS);
            float2 hck01 = f2(0.f, 0.f), hck23 = hck01;
            if (dvalid) {
                const float4 v = *reinterpret_cast<const float4*>(
                    p.ck + (((int64_t)bi * nck + c) * p.D + d) * NS + 4 * j);
                hck01 = f2(v.x, v.y);
                hck23 = f2(v.z, v.w);
            }
            // recompute the chunk's states (B kept in registers for the reverse pass)
            float2 hs01[TCK], hs23[TCK];
            float4 bv[TCK];
            float yv[TCK];
            if (nt == TCK)
                bwd_recompute<true, YV, AREG>(S.dd[s], S.B[r], S.C[r], nt, ch, j, A01, A23, hck01, hck23, hs01, hs23, bv, yv);
            else
                bwd_recompute<false, YV, AREG>(S.dd[s], S.B[r], S.C[r], nt, ch, j, A01, A23, hck01, hck23, hs01, hs23, bv, yv);
            // reverse recurrence: hand-off tiles from the last steps down, alternating slots
#pragma unroll
            for (int hh = 0; hh < NQ; ++hh) {
                const int slot = hh & 1, tlo = (NQ - 1 - hh) * HTQ;
                bar_sync(BAR_E0 + slot, NTH);
                if (nt == TCK)
                    bwd_half<true, YV, HTQ, LOWREG, AREG>(S.dd[s], S.dy[s], S.B[r], S.C[r], S.bc[slot], S.nsd[slot],
                                                    S.nyp[slot], tlo, nt, ch, j, A01, A23, bv, hs01, hs23, yv, hck01,
                                                    hck23, An01, An23, g01, g23, an01, an23, dA01, dA23);
                else
                    bwd_half<false, YV, HTQ, LOWREG, AREG>(S.dd[s], S.dy[s], S.B[r], S.C[r], S.bc[slot], S.nsd[slot],
                                                     S.nyp[slot], tlo, nt, ch, j, A01, A23, bv, hs01, hs23, yv, hck01,
                                                     hck23, An01, An23, g01, g23, an01, an23, dA01, dA23);
                bar_arrive(BAR_X0 + slot, NTH);
            }
        }
        if (dvalid) {
            *reinterpret_cast<float4*>(p.ws_a + ((int64_t)bi * p.D + d) * NS + 4 * j) =
                make_float4(dA01.x, dA01.y, dA23.x, dA23.y);
            if (p.dh0) {
                const float hv[4] = {an01.x * g01.x, an01.y * g01.y, an23.x * g23.x, an23.y * g23.y};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int n = 4 * j + i;
                    if (n < p.N) p.dh0[((int64_t)bi * p.D + d) * p.N + n] = hv[i];
                }
            }
        }
    } else {
        // ------------------------------------------------ helper warps
        const int at = tid - NSCAN;
        const int ech = at & (SCH - 1);
        const bool evalid = ech < nd;
        const float eD = (p.Dskip && evalid) ? p.Dskip[d0 + ech] : 0.f;
        const float ebias = (p.dbias && evalid) ? p.dbias[d0 + ech] : 0.f;
        const int egroup = (GW && evalid) ? p.gof[d0 + ech] : 0;       // pathway group of the channel
        const Tin* gu = static_cast<const Tin*>(p.u) + bi * p.u_sb + d0;
        const Tin* gdl = static_cast<const Tin*>(p.dl) + bi * p.dl_sb + d0;
        const Tin* gz = HAS_Z ? static_cast<const Tin*>(p.z) + bi * p.z_sb + d0 : nullptr;
        const Tin* gdo = static_cast<const Tin*>(p.dout) + bi * p.dout_sb + d0;
        const Tin* gB = static_cast<const Tin*>(p.B) + bi * p.B_sb;
        const Tin* gC = static_cast<const Tin*>(p.C) + bi * p.C_sb;
        const int64_t orow = (int64_t)bi * p.L * p.D + d0;
        Tin* gdu = static_cast<Tin*>(p.du) + orow;
        Tin* gddl = static_cast<Tin*>(p.ddl) + orow;
        Tin* gdz = HAS_Z ? static_cast<Tin*>(p.dz) + (DZS ? (int64_t)bi * p.dz_sb + d0 : orow) : nullptr;
        float* wbc = p.ws_bc + ((int64_t)blockIdx.x * p.b + bi) * p.L * 2 * NS;
        const float* gyp = YPRE ? p.ypre + (int64_t)bi * p.L * p.D + d0 : nullptr;
        float accD = 0.f, accB = 0.f;

        // staging.  TMA: helper thread 0 issues one tile copy per tensor for chunk k into ring
        // slot k % RING, all completing on the slot's mbarrier; after a wait that gave up it
        // issues nothing more (copies still in flight are waited for at the end)
        int issued = 0;
        volatile int* stop = &S.stop;
        constexpr uint32_t TILE = TCK * SCH * sizeof(Tin), TILE_Y = TCK * SCH * 4, TILE_BC = TCK * NS * sizeof(Tin);
        auto issue = [&](int k) {
            if (fast) {
                if (k < nck && at == 0 && !*stop) {
                    const int t0 = (nck - 1 - k) * TCK, r = k % RING;
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
                    issued = k + 1;
                }
                return;
            }
            if (k < nck) {
                const int c = nck - 1 - k, t0 = c * TCK, rv = min(TCK, p.L - t0), r = k % RING;
                stage_tile<Tin, SCH>(&S.u[r][0][0], gu + t0 * p.u_sl, p.u_sl, TCK, rv, nd, p.vec_u, at, NAUX);
                stage_tile<Tin, SCH>(&S.dl[r][0][0], gdl + t0 * p.dl_sl, p.dl_sl, TCK, rv, nd, p.vec_dl, at, NAUX);
                if (HAS_Z)
                    stage_tile<Tin, SCH>(&S.z[r][0][0], gz + t0 * p.z_sl, p.z_sl, TCK, rv, nd, p.vec_z, at, NAUX);
                stage_tile<Tin, SCH>(&S.dout[r][0][0], gdo + t0 * p.dout_sl, p.dout_sl, TCK, rv, nd, p.vec_dout, at, NAUX);
                if (YPRE)
                    stage_tile<float, SCH>(&S.yp[r][0][0], gyp + (int64_t)t0 * p.D, p.D, TCK, rv, nd, p.vec_yp, at, NAUX);
                stage_tile<Tin, NS>(&S.B[r][0][0], gB + t0 * p.B_sl, p.B_sl, TCK, rv, p.N, p.vec_B, at, NAUX);
                stage_tile<Tin, NS>(&S.C[r][0][0], gC + t0 * p.C_sl, p.C_sl, TCK, rv, p.N, p.vec_C, at, NAUX);
            }
            cp_async_commit();
        };
        // Wait for chunk k's copies; a wait that gives up is recorded in the status word and
        // stops further copies and waits (the kernel runs to its end on what is in shared
        // memory: incomplete results, intact barrier protocol and context).
        auto tile_wait = [&](int k) {
            if (*stop) return;
            if (!mbar_wait_bounded(&S.mbar[k % RING], (k / RING) & 1, ROW_WAIT_POLLS)) {
                *stop = 1;
                if (p.err) *p.err = SWX_ERR_TIMEOUT;
            }
        };
        const float2 bias2 = bc2(ebias);
        auto derive = [&](int k) {
            const int r = k % RING, s = k & 1;
            const int t0 = (nck - 1 - k) * TCK, nt = min(TCK, p.L - t0);
#pragma unroll
            for (int m = 0; m < TCK * SCH / (2 * NAUX); ++m) {
                const int t = 2 * (at / SCH + m * (NAUX / SCH));
                const float2 raw = add2(f2(Elem<Tin>::to_f(S.dl[r][t][ech]), Elem<Tin>::to_f(S.dl[r][t + 1][ech])), bias2);
                const float2 uv = f2(Elem<Tin>::to_f(S.u[r][t][ech]), Elem<Tin>::to_f(S.u[r][t + 1][ech]));
                float2 dov = f2(Elem<Tin>::to_f(S.dout[r][t][ech]), Elem<Tin>::to_f(S.dout[r][t + 1][ech]));
                if (GW)                                // the pathway mix scales the gate's input
                    dov = mul2(dov, f2(t < nt ? group_weight(p, bi, t0 + t, egroup) : 0.f,
                                       t + 1 < nt ? group_weight(p, bi, t0 + t + 1, egroup) : 0.f));
                float2 dte = raw, dsp = bc2(1.f);
                if (p.softplus) softplus2(raw, dte, dsp);
                float2 dy = dov, q = bc2(0.f);
                if (HAS_Z) {
                    const float2 zv = f2(Elem<Tin>::to_f(S.z[r][t][ech]), Elem<Tin>::to_f(S.z[r][t + 1][ech]));
                    const float2 sg = sigmoid2(zv);
                    dy = mul2(dov, mul2(zv, sg));
                    // d silu / dz = sg * (1 + z * (1 - sg))
                    q = mul2(mul2(dov, sg), fma2(zv, add2(bc2(1.f), mul2(sg, bc2(-1.f))), bc2(1.f)));
                }
                const float2 du = mul2(dte, uv);
                S.dd[s][t][ech] = f2(dte.x, du.x);
                S.dd[s][t + 1][ech] = f2(dte.y, du.y);
                S.dy[s][t][ech] = dy.x;
                S.dy[s][t + 1][ech] = dy.y;
                S.ee[s][t][ech] = make_float4(uv.x, dsp.x, q.x, dy.x);
                S.ee[s][t + 1][ech] = make_float4(uv.y, dsp.y, q.y, dy.y);
            }
        };
        auto epilogue = [&](int k, int hh) {
            const int c = nck - 1 - k, s = k & 1, t0 = c * TCK, nt = min(TCK, p.L - t0);
            const int tlo = (NQ - 1 - hh) * HTQ, slot = hh & 1;
            if (evalid) {
#pragma unroll
                for (int m = 0; m < HTQ * SCH / NAUX; ++m) {
                    const int tt = at / SCH + m * (NAUX / SCH);
                    const int t = tlo + tt;
                    if (t < nt) {
                        // rotate the state-group order per lane quad: conflict-free 8-byte loads
                        const int rot = (ech >> 2) & 3;
                        const float2 n0 = S.nsd[slot][tt][ech][(rot + 0) & 3];
                        const float2 n1 = S.nsd[slot][tt][ech][(rot + 1) & 3];
                        const float2 n2 = S.nsd[slot][tt][ech][(rot + 2) & 3];
                        const float2 n3 = S.nsd[slot][tt][ech][(rot + 3) & 3];
                        const float sgb = (n0.x + n1.x) + (n2.x + n3.x);
                        const float sda = (n0.y + n1.y) + (n2.y + n3.y);
                        const float dte = S.dd[s][t][ech].x;
                        const float4 e = S.ee[s][t][ech];          // (u, dsoftplus, q, dy)
                        const float du = fmaf(dte, sgb, eD * e.w);
                        const float draw = fmaf(e.x, sgb, sda) * e.y;
                        const int64_t o = (int64_t)(t0 + t) * p.D + ech;
                        gdu[o] = Elem<Tin>::from_f(du);
                        gddl[o] = Elem<Tin>::from_f(draw);
                        if (HAS_Z) {
                            float y;
                            if (YPRE) {
                                y = S.yp[k % RING][t][ech];
                            } else {
                                const float4 q4 = *reinterpret_cast<const float4*>(&S.nyp[slot][tt][ech][0]);
                                y = fmaf(eD, e.x, (q4.x + q4.y) + (q4.z + q4.w));
                            }
                            gdz[DZS ? (int64_t)(t0 + t) * p.dz_sl + ech : o] = Elem<Tin>::from_f(e.z * y);
                        }
                        accD = fmaf(e.w, e.x, accD);
                        accB += draw;
                    }
                }
            }
            // CTA partial of dB | dC: fixed-order sum over the 32 channels.  8-step tiles: one
            // thread per (step, column pair); 4-step tiles: two, each summing 16 channels,
            // joined by one shuffle.
            if (HTQ == 8) {
                const int o2 = at & 15, tt = at >> 4, t = tlo + tt;
                if (t < nt) {
                    float2 s0 = f2(0.f, 0.f), s1 = s0, s2 = s0, s3 = s0;
                    const int col0 = 2 * o2, col1 = (2 * o2) ^ NS;   // even / odd channel columns
#pragma unroll
                    for (int cc = 0; cc < SCH; cc += 4) {
                        s0 = add2(s0, *reinterpret_cast<const float2*>(&S.bc[slot][tt][cc + 0][col0]));
                        s1 = add2(s1, *reinterpret_cast<const float2*>(&S.bc[slot][tt][cc + 1][col1]));
                        s2 = add2(s2, *reinterpret_cast<const float2*>(&S.bc[slot][tt][cc + 2][col0]));
                        s3 = add2(s3, *reinterpret_cast<const float2*>(&S.bc[slot][tt][cc + 3][col1]));
                    }
                    *reinterpret_cast<float2*>(wbc + (int64_t)(t0 + t) * 2 * NS + 2 * o2) =
                        add2(add2(s0, s1), add2(s2, s3));
                }
            } else {
                // lanes 0-15 sum channels 0-15 and lanes 16-31 channels 16-31 of the same 16
                // column pairs, so each half-warp reads one contiguous 128-byte row
                const int half = (at >> 4) & 1, o2 = at & 15, tt = (at >> 5) & (HTQ - 1), t = tlo + tt;
                float2 s0 = f2(0.f, 0.f), s1 = s0, s2 = s0, s3 = s0;
                const int col0 = 2 * o2, col1 = (2 * o2) ^ NS;
#pragma unroll
                for (int cc = 16 * half; cc < 16 * half + 16; cc += 4) {
                    s0 = add2(s0, *reinterpret_cast<const float2*>(&S.bc[slot][tt][cc + 0][col0]));
                    s1 = add2(s1, *reinterpret_cast<const float2*>(&S.bc[slot][tt][cc + 1][col1]));
                    s2 = add2(s2, *reinterpret_cast<const float2*>(&S.bc[slot][tt][cc + 2][col0]));
                    s3 = add2(s3, *reinterpret_cast<const float2*>(&S.bc[slot][tt][cc + 3][col1]));
                }
                float2 sum = add2(add2(s0, s1), add2(s2, s3));
                const float2 other = f2(__shfl_xor_sync(0xffffffffu, sum.x, 16),
                                        __shfl_xor_sync(0xffffffffu, sum.y, 16));
                sum = half ? add2(other, sum) : add2(sum, other);
                if (half == 0 && t < nt)
                    *reinterpret_cast<float2*>(wbc + (int64_t)(t0 + t) * 2 * NS + 2 * o2) = sum;
            }
        };

        issue(0);
        issue(1);
        issue(2);
        if (fast) tile_wait(0);
        else cp_async_wait<2>();
        bar_sync(BAR_AUX, NAUX);
        derive(0);
        bar_arrive(BAR_D0, NTH);
        bar_arrive(BAR_E0, NTH);          // both hand-off slots start empty
        bar_arrive(BAR_E0 + 1, NTH);
        for (int k = 0; k < nck; ++k) {
            if (k + 1 < nck) {
                if (fast) tile_wait(k + 1);
                else cp_async_wait<1>();
                bar_sync(BAR_AUX, NAUX);
                derive(k + 1);
                bar_arrive(BAR_D0 + ((k + 1) & 1), NTH);
            }
#pragma unroll
            for (int hh = 0; hh < NQ; ++hh) {
                bar_sync(BAR_X0 + (hh & 1), NTH);
                epilogue(k, hh);
                // the slot is free again for the tile two hand-offs later, if there is one
                if (k * NQ + hh + 2 < NQ * nck) bar_arrive(BAR_E0 + (hh & 1), NTH);
            }
            bar_sync(BAR_AUX, NAUX);      // raw slot (k-1) % RING no longer read
            issue(k + 3);
        }
        if (!fast) {
            cp_async_wait<0>();
        } else if (at == 0 && *stop) {
            // copies that may still be landing in this CTA's shared memory: the last chunk
            // issued into each slot, each given a second bounded wait before the CTA exits
            for (int k = max(0, issued - RING); k < issued; ++k)
                mbar_wait_bounded(&S.mbar[k % RING], (k / RING) & 1, ROW_WAIT_POLLS);
        }
        S.red[0][at] = accD;
        S.red[1][at] = accB;
        bar_sync(BAR_AUX, NAUX);
        if (at < SCH && at < nd) {
            float sD = 0.f, sB = 0.f;
#pragma unroll
            for (int m = 0; m < NAUX / SCH; ++m) { sD += S.red[0][at + m * SCH]; sB += S.red[1][at + m * SCH]; }
            p.ws_d[(int64_t)bi * p.D + d0 + at] = sD;
            p.ws_bias[(int64_t)bi * p.D + d0 + at] = sB;
        }
    }
}

// Second pass: fixed-order sums of the partials.  The dB | dC partials are read as whole
// 32-float rows (one (row, step) of one CTA's channel block: both halves together), so
// consecutive threads read consecutive words; the per-block sum runs in block order.
template <typename Tin>
__global__ void scan_bwd_finalize_kernel(const ScanDev p) {
    const int64_t nrow = (int64_t)p.b * p.L;                 // (bi, t) rows
    const int64_t nbc = nrow * 2 * NS;                         // dB | dC words
    const int64_t total = nbc + (int64_t)p.D * p.N + p.D;
    const int64_t slab = nrow * 2 * NS;                        // one channel block's partials
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        if (i < nbc) {
            const int col = (int)(i & (2 * NS - 1));
            const int kind = col >= NS, n = col & (NS - 1);
            if (n >= p.N) continue;
            const int64_t bl = i >> 5;                         // bi * L + t
            const float* src = p.ws_bc + i;
            float s = 0.f;
#pragma unroll 16
            for (int k = 0; k < p.nblk; ++k) s += src[(int64_t)k * slab];   // loads in flight, adds in order
            Tin* dst = static_cast<Tin*>(kind ? p.dC : p.dB);
            dst[bl * p.N + n] = Elem<Tin>::from_f(s);
        } else if (i < nbc + (int64_t)p.D * p.N) {
            const int64_t r = i - nbc;
            const int dd = r / p.N, n = r % p.N;
            float s = 0.f;
            for (int bi = 0; bi < p.b; ++bi) s += p.ws_a[((int64_t)bi * p.D + dd) * NS + n];
            p.dA[r] = p.a_log ? s * load_A(p, r) : s;       // d/dA_log = dA * A
        } else {
            const int dd = i - nbc - (int64_t)p.D * p.N;
            float sD = 0.f, sB = 0.f;
            for (int bi = 0; bi < p.b; ++bi) {
                sD += p.ws_d[(int64_t)bi * p.D + dd];
                sB += p.ws_bias[(int64_t)bi * p.D + dd];
            }
            if (p.dD) p.dD[dd] = sD;
            if (p.ddbias) p.ddbias[dd] = sB;
        }
    }
}


template <typename Tin, bool HAS_Z>
static cudaError_t fits_t(const ScanDev& p, int* per_sm, int* sms) {
    const bool ypre = HAS_Z && p.ypre;
    auto k = ypre ? scan_bwd_kernel<Tin, HAS_Z, true, true> : scan_bwd_kernel<Tin, HAS_Z, false, true>;
    const int smem = sizeof(BwdSmem<Tin, 4>);
    cudaError_t e = allow_smem(k, smem);
    if (e != cudaSuccess) return e;
    return sm_fit(k, NTH, smem, sms, per_sm);
}

template <typename Tin, bool HAS_Z>
static RowMaps row_maps(const ScanDev& p) {
    RowMaps m{};
    const int es = sizeof(Tin);
    bool ok = encode_3d(&m.u, p.u, es, p.D, p.L, p.b, p.u_sl, p.u_sb, SCH, TCK) &&
              encode_3d(&m.dl, p.dl, es, p.D, p.L, p.b, p.dl_sl, p.dl_sb, SCH, TCK) &&
              encode_3d(&m.dout, p.dout, es, p.D, p.L, p.b, p.dout_sl, p.dout_sb, SCH, TCK) &&
              encode_3d(&m.B, p.B, es, p.N, p.L, p.b, p.B_sl, p.B_sb, NS, TCK) &&
              encode_3d(&m.C, p.C, es, p.N, p.L, p.b, p.C_sl, p.C_sb, NS, TCK);
    if (ok && HAS_Z) ok = encode_3d(&m.z, p.z, es, p.D, p.L, p.b, p.z_sl, p.z_sb, SCH, TCK);
    if (ok && HAS_Z && p.ypre) ok = encode_3d(&m.yp, p.ypre, 4, p.D, p.L, p.b, p.D, (int64_t)p.L * p.D, SCH, TCK);
    m.ok = ok ? 1 : 0;
    return m;
}

template <typename Tin, bool HAS_Z>
static cudaError_t launch_t(const ScanDev& p0, cudaStream_t st) {
    ScanDev p = p0;
    p.err = wait_status_address();               // where a timed-out tile wait is recorded
    const bool ypre = HAS_Z && p.ypre;
    auto k = ypre ? scan_bwd_kernel<Tin, HAS_Z, true, true> : scan_bwd_kernel<Tin, HAS_Z, false, true>;
    if constexpr (HAS_Z) {
        const bool dzs = p.dz_sl != p.D || p.dz_sb != (int64_t)p.L * p.D;    // strided dz
        if (p.gw && dzs)
            k = ypre ? scan_bwd_kernel<Tin, true, true, true, true, true> : scan_bwd_kernel<Tin, true, false, true, true, true>;
        else if (p.gw)
            k = ypre ? scan_bwd_kernel<Tin, true, true, true, true> : scan_bwd_kernel<Tin, true, false, true, true>;
        else if (dzs)
            k = ypre ? scan_bwd_kernel<Tin, true, true, true, false, true> : scan_bwd_kernel<Tin, true, false, true, false, true>;
    }
    const int smem = sizeof(BwdSmem<Tin, 4>);
    cudaError_t e = allow_smem(k, smem);
    if (e != cudaSuccess) return e;
    dim3 grid((p.D + SCH - 1) / SCH, p.b);
    k<<<grid, NTH, smem, st>>>(p, row_maps<Tin, HAS_Z>(p));
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const int64_t total = 2LL * NS * p.b * p.L + (int64_t)p.D * p.N + p.D;
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 8);
    scan_bwd_finalize_kernel<Tin><<<blocks, 256, 0, st>>>(p);
    return cudaGetLastError();
}

}  // namespace rowk

// Whether swx_scan_bwd takes the row kernel for these arguments on the current device:
// bf16 inputs, two CTAs of it fit on an SM, and the grid has at least one CTA per SM.
cudaError_t scan_bwd_rows_applicable(const ScanDev& p, int in_dtype, bool has_z, bool* yes) {
    *yes = false;
    if (in_dtype != SWX_DTYPE_BF16) return cudaSuccess;
    int per_sm = 0, sms = 0;
    const cudaError_t e = has_z ? rowk::fits_t<__nv_bfloat16, true>(p, &per_sm, &sms)
                                : rowk::fits_t<__nv_bfloat16, false>(p, &per_sm, &sms);
    if (e != cudaSuccess) return e;
    const long long ctas = (long long)((p.D + rowk::SCH - 1) / rowk::SCH) * p.b;
    *yes = per_sm >= 2 && ctas >= sms;
    return cudaSuccess;
}

cudaError_t launch_scan_bwd_rows(const ScanDev& p, bool has_z, cudaStream_t st) {
    return has_z ? rowk::launch_t<__nv_bfloat16, true>(p, st) : rowk::launch_t<__nv_bfloat16, false>(p, st);
}

}  // namespace swx
