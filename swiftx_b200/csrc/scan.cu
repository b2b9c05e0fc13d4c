// Selective scan forward kernel for sm_100a.
//
// Work decomposition: one CTA owns 32 channels of one batch row for the whole sequence.
// A state chain h[d, n] is a first-order recurrence in time, so time is walked
// sequentially and the parallelism is b * D * N chains.  The CTA is warp-specialised:
//
//   * 4 recurrence warps: thread (channel, state group) owns 4 of the 16 states of
//     one channel in fp32 registers (4 adjacent lanes hold a channel, a warp covers
//     8 channels).  Per step: a = 2^(delta_eff * A*log2e) on the MUFU unit, then
//     h = a*h + delta_eff*u*B with packed f32x2 FMAs.  They read only pre-computed
//     per-(t, channel) scalars and the channel-shared B_t / C_t from shared memory.
//   * 4 or 8 helper warps: stage raw tiles of u, delta, z, B, C into a 4-slot ring (three
//     tiles ahead) -- one thread issues a TMA tile copy per tensor (cp.async.bulk.tensor,
//     completion on the slot's mbarrier; per-thread 16-byte cp.async when a tensor's base
//     or strides are not 16-byte aligned) --, compute the per-(t, channel) scalars once
//     per channel (softplus(delta + bias), delta*u), and run the epilogue (readout sum,
//     D skip, SiLU(z) gate, coalesced stores).
//
// The two groups hand tiles over through double-buffered shared memory guarded by
// named barriers (producer bar.arrive, consumer bar.sync), so the recurrence never
// waits for the per-channel work of the neighbouring tiles.  The state before every
// 16-step chunk is checkpointed for the backward (scan_bwd_seg.cu).
#include <mutex>
#include <vector>

#include "common.cuh"
#include "scan_params.cuh"
#include "launch_util.cuh"
#include "tma_util.cuh"

namespace swx {

constexpr int SCH = 32;               // channels per CTA
constexpr int NSCAN = 128;            // recurrence threads
constexpr int NAUX = 128;             // helper threads
constexpr int NTH = NSCAN + NAUX;
constexpr int FNAUX_MAX = 256;        // helper threads of the forward: 128 or 256 (see launch_fwd_t)
constexpr int FT = 32;                // forward tile (steps)
constexpr int RING = 4;               // raw staging slots

enum : int { BAR_AUX = 1, BAR_D0 = 2, BAR_X0 = 4 };
constexpr uint32_t FWD_WAIT_POLLS = 1u << 24;   // mbarrier polls before a tile wait gives up

// TMA descriptors of the forward's inputs: (channel, step, row) tiles of 32 x 32 x 1 for u,
// delta, z and 16 x 32 x 1 for B and C.  ok = 0: some tensor is not 16-byte aligned; the
// helpers stage with per-thread cp.async.
struct FwdMaps {
    CUtensorMap u, dl, z, B, C;
    int ok;
};

// Four consecutive staged elements as fp32 (one 16-byte load for fp32, 8-byte for bf16).
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ld4(const __nv_bfloat16* p) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u),
                       __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xffff0000u));
}

// A[d, n] (flat index i of the (D, N) array), formed as -expf(A_log) when the caller
// passed log(-A) -- expf is the function torch.exp evaluates for fp32 on CUDA.
__device__ __forceinline__ float load_A(const ScanDev& p, int64_t i) {
    const float a = p.A[i];
    return p.a_log ? -expf(a) : a;
}

// =============================================================== forward
template <typename Tin>
struct FwdSmem {
    Tin u[RING][FT][SCH];
    Tin dl[RING][FT][SCH];
    Tin z[RING][FT][SCH];
    Tin B[RING][FT][NS];
    Tin C[RING][FT][NS];
    float2 dd[2][FT][SCH];        // (delta_eff, delta_eff * u)
    float yp[2][FT][SCH][4];      // partial readouts of the 4 state groups
    float red[FNAUX_MAX];          // per-thread sums of delta_eff
    uint64_t mbar[RING];           // completion of each ring slot's TMA copies
    int stop;                      // a tile wait gave up: no further copies, no further waits
};

template <bool FULL, bool WR, typename Tin>
__device__ __forceinline__ void fwd_tile(const float2 (*__restrict__ dd)[SCH], const Tin (*__restrict__ Bs)[NS],
                                         const Tin (*__restrict__ Cs)[NS], float (*__restrict__ yp)[SCH][4],
                                         int nt, int ch, int j, float2 A01, float2 A23, float2& h01, float2& h23,
                                         float* __restrict__ ckp, int64_t ck_stride) {
#pragma unroll
    for (int g = 0; g < FT / 8; ++g) {
        float yv[8];
        // the 8 steps' decays and inputs first (they do not depend on the state), then
        // the chain: the MUFU work of the group is issued back to back (3.5 % faster on
        // bf16 grids of two CTAs per SM, unchanged at one; same arithmetic, same bits)
        float2 av[8][2], ub[8][2];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int t = 8 * g + q;
            if (FULL || t < nt) {
                const float2 d = dd[t][ch];
                const float4 b = ld4(&Bs[t][4 * j]);
                const float2 dt = bc2(d.x), du = bc2(d.y);
                av[q][0] = ex2x2(mul2(dt, A01));
                av[q][1] = ex2x2(mul2(dt, A23));
                ub[q][0] = mul2(du, f2(b.x, b.y));
                ub[q][1] = mul2(du, f2(b.z, b.w));
            }
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int t = 8 * g + q;
            if (FULL || t < nt) {
                if ((t % TCK) == 0 && ckp)
                    *reinterpret_cast<float4*>(ckp + (t / TCK) * ck_stride) = make_float4(h01.x, h01.y, h23.x, h23.y);
                h01 = fma2(av[q][0], h01, ub[q][0]);
                h23 = fma2(av[q][1], h23, ub[q][1]);
                if (WR) {
                    const float4 c = ld4(&Cs[t][4 * j]);
                    float2 y = mul2(h01, f2(c.x, c.y));
                    y = fma2(h23, f2(c.z, c.w), y);
                    yv[q] = y.x + y.y;
                }
            }
        }
        if (WR) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int t = 8 * g + q;
                if (FULL || t < nt) yp[t][ch][j] = yv[q];
            }
        }
    }
}

// WR: write the output (pass 1 of the sequence-parallel scan needs only the final state
// and the per-channel sum of delta_eff, so it skips C, z, the readout and the stores).
// NA: helper threads (128 = one helper warp per sub-partition, 256 = two).  The 128-helper
// variant is built for two CTAs per SM (at most 128 registers a thread): the output-writing
// kernels need ~100 anyway, and the sequence-parallel pass 1 (no output) then fits two CTAs
// per SM at the cost of a few spilled bytes.
// GW: the SiftX pathway mix is applied before the gate (only with HAS_Z and WR).
template <typename Tin, typename Tout, bool HAS_Z, bool WR, int NA, bool GW = false>
__global__ void __launch_bounds__(NSCAN + NA, NA == 128 ? 2 : 1)
    scan_fwd_kernel(const ScanDev p, const __grid_constant__ FwdMaps tm) {
    constexpr int FNAUX = NA, FNTH = NSCAN + NA;
    extern __shared__ __align__(128) unsigned char smem_raw[];   // TMA destinations: 128-byte aligned
    FwdSmem<Tin>& S = *reinterpret_cast<FwdSmem<Tin>*>(smem_raw);

    const int tid = threadIdx.x;
    const int bi = blockIdx.y;
    const int d0 = blockIdx.x * SCH;
    const int nd = min(SCH, p.D - d0);
    const int nchunk = (p.L + FT - 1) / FT;
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
        float av[4], hv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int n = 4 * j + i;
            const bool ok = dvalid && n < p.N;
            av[i] = ok ? load_A(p, (int64_t)d * p.N + n) * LOG2E : 0.f;
            hv[i] = (ok && p.h0) ? p.h0[((int64_t)bi * p.D + d) * p.N + n] : 0.f;
        }
        const float2 A01 = f2(av[0], av[1]), A23 = f2(av[2], av[3]);
        float2 h01 = f2(hv[0], hv[1]), h23 = f2(hv[2], hv[3]);
        const int64_t ck_stride = (int64_t)p.D * NS;
        for (int c = 0; c < nchunk; ++c) {
            const int s = c & 1, t0 = c * FT, nt = min(FT, p.L - t0);
            bar_sync(BAR_D0 + s, FNTH);
            float* ckp = (p.ck && dvalid)
                             ? p.ck + (((int64_t)bi * p.nck + t0 / TCK) * p.D + d) * NS + 4 * j
                             : nullptr;
            const int r = c % RING;
            // the helpers waited for this tile before deriving it; the wait here orders the
            // bulk copies' writes of B / C before this thread's reads (it returns at once)
            if (fast && !*reinterpret_cast<volatile int*>(&S.stop))
                mbar_wait_bounded(&S.mbar[r], (c / RING) & 1, FWD_WAIT_POLLS);
            if (nt == FT)
                fwd_tile<true, WR>(S.dd[s], S.B[r], S.C[r], S.yp[s], nt, ch, j, A01, A23, h01, h23, ckp, ck_stride);
            else
                fwd_tile<false, WR>(S.dd[s], S.B[r], S.C[r], S.yp[s], nt, ch, j, A01, A23, h01, h23, ckp, ck_stride);
            bar_arrive(BAR_X0 + s, FNTH);
        }
        if (p.h_last && dvalid) {
            hv[0] = h01.x; hv[1] = h01.y; hv[2] = h23.x; hv[3] = h23.y;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int n = 4 * j + i;
                if (n < p.N) p.h_last[((int64_t)bi * p.D + d) * p.N + n] = hv[i];
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
        const Tin* gB = static_cast<const Tin*>(p.B) + bi * p.B_sb;
        const Tin* gC = static_cast<const Tin*>(p.C) + bi * p.C_sb;
        Tout* gout = static_cast<Tout*>(p.out) + (int64_t)bi * p.L * p.D + d0;

        // staging.  TMA: helper thread 0 issues one tile copy per tensor for tile c into
        // ring slot c % RING, all completing on the slot's mbarrier; after a wait that gave
        // up it issues nothing more (the copies still in flight are waited for at the end)
        int issued = 0;
        volatile int* stop = &S.stop;
        constexpr uint32_t TILE = FT * SCH * sizeof(Tin), TILE_BC = FT * NS * sizeof(Tin);
        auto issue = [&](int c) {
            if (fast) {
                if (c < nchunk && at == 0 && !*stop) {
                    const int t0 = c * FT, r = c % RING;
                    fence_proxy_async_smem();            // the slot's last readers are past a barrier
                    const uint32_t bytes = (HAS_Z && WR ? 3 : 2) * TILE + (WR ? 2 : 1) * TILE_BC;
                    mbar_arrive_expect_tx(&S.mbar[r], bytes);
                    tma_load_3d(&S.u[r][0][0], &tm.u, d0, t0, bi, &S.mbar[r]);
                    tma_load_3d(&S.dl[r][0][0], &tm.dl, d0, t0, bi, &S.mbar[r]);
                    if (HAS_Z && WR) tma_load_3d(&S.z[r][0][0], &tm.z, d0, t0, bi, &S.mbar[r]);
                    tma_load_3d(&S.B[r][0][0], &tm.B, 0, t0, bi, &S.mbar[r]);
                    if (WR) tma_load_3d(&S.C[r][0][0], &tm.C, 0, t0, bi, &S.mbar[r]);
                    issued = c + 1;
                }
                return;
            }
            if (c < nchunk) {
                const int t0 = c * FT, rv = min(FT, p.L - t0), r = c % RING;
                stage_tile<Tin, SCH>(&S.u[r][0][0], gu + t0 * p.u_sl, p.u_sl, FT, rv, nd, p.vec_u, at, FNAUX);
                stage_tile<Tin, SCH>(&S.dl[r][0][0], gdl + t0 * p.dl_sl, p.dl_sl, FT, rv, nd, p.vec_dl, at, FNAUX);
                if (HAS_Z && WR)
                    stage_tile<Tin, SCH>(&S.z[r][0][0], gz + t0 * p.z_sl, p.z_sl, FT, rv, nd, p.vec_z, at, FNAUX);
                stage_tile<Tin, NS>(&S.B[r][0][0], gB + t0 * p.B_sl, p.B_sl, FT, rv, p.N, p.vec_B, at, FNAUX);
                if (WR)
                    stage_tile<Tin, NS>(&S.C[r][0][0], gC + t0 * p.C_sl, p.C_sl, FT, rv, p.N, p.vec_C, at, FNAUX);
            }
            cp_async_commit();
        };
        // Wait for tile k's copies.  A wait that gives up is recorded in the status word and
        // stops further copies and waits; the kernel then runs to its end on what is in
        // shared memory (its results are incomplete, the barrier protocol and the context
        // stay intact).
        auto tile_wait = [&](int k) {
            if (*stop) return;
            if (!mbar_wait_bounded(&S.mbar[k % RING], (k / RING) & 1, FWD_WAIT_POLLS)) {
                *stop = 1;
                if (p.err) *p.err = SWX_ERR_TIMEOUT;
            }
        };
        // per-(t, channel) work: each thread takes pairs of steps (t, t+1) of channel `ech`
        const float2 bias2 = bc2(ebias), D2 = bc2(eD);
        float dsum = 0.f;
        auto derive = [&](int c) {
            const int r = c % RING, s = c & 1, nt = min(FT, p.L - c * FT);
#pragma unroll
            for (int m = 0; m < FT * SCH / (2 * FNAUX); ++m) {
                const int t = 2 * (at / SCH + m * (FNAUX / SCH));
                const float2 raw = add2(f2(Elem<Tin>::to_f(S.dl[r][t][ech]), Elem<Tin>::to_f(S.dl[r][t + 1][ech])), bias2);
                float2 dte = raw, dsp;
                if (p.softplus) softplus2(raw, dte, dsp);
                const float2 du = mul2(dte, f2(Elem<Tin>::to_f(S.u[r][t][ech]), Elem<Tin>::to_f(S.u[r][t + 1][ech])));
                S.dd[s][t][ech] = f2(dte.x, du.x);
                S.dd[s][t + 1][ech] = f2(dte.y, du.y);
                if (t < nt) dsum += dte.x;
                if (t + 1 < nt) dsum += dte.y;
            }
        };
        auto epilogue = [&](int c) {
            if (!WR) return;
            const int r = c % RING, s = c & 1, t0 = c * FT, nt = min(FT, p.L - t0);
#pragma unroll
            for (int m = 0; m < FT * SCH / (2 * FNAUX); ++m) {
                const int t = 2 * (at / SCH + m * (FNAUX / SCH));
                const float4 q0 = *reinterpret_cast<const float4*>(&S.yp[s][t][ech][0]);
                const float4 q1 = *reinterpret_cast<const float4*>(&S.yp[s][t + 1][ech][0]);
                float2 y = f2((q0.x + q0.y) + (q0.z + q0.w), (q1.x + q1.y) + (q1.z + q1.w));
                y = fma2(D2, f2(Elem<Tin>::to_f(S.u[r][t][ech]), Elem<Tin>::to_f(S.u[r][t + 1][ech])), y);
                if (HAS_Z) {
                    if (p.ypre && evalid) {            // pre-gate output, saved for the backward
                        float* q = p.ypre + (int64_t)bi * p.L * p.D + (int64_t)(t0 + t) * p.D + d0 + ech;
                        if (t < nt) q[0] = y.x;
                        if (t + 1 < nt) q[p.D] = y.y;
                    }
                    if (GW)                            // SiftX pathway mix, before the gate
                        y = mul2(y, f2(t < nt ? group_weight(p, bi, t0 + t, egroup) : 0.f,
                                       t + 1 < nt ? group_weight(p, bi, t0 + t + 1, egroup) : 0.f));
                    const float2 zz = f2(Elem<Tin>::to_f(S.z[r][t][ech]), Elem<Tin>::to_f(S.z[r][t + 1][ech]));
                    y = mul2(y, mul2(zz, sigmoid2(zz)));
                }
                if (evalid) {
                    Tout* o = gout + (int64_t)(t0 + t) * p.D + ech;
                    if (t < nt) o[0] = Elem<Tout>::from_f(y.x);
                    if (t + 1 < nt) o[p.D] = Elem<Tout>::from_f(y.y);
                }
            }
        };

        issue(0);
        issue(1);
        issue(2);
        if (fast) tile_wait(0);
        else cp_async_wait<2>();
        bar_sync(BAR_AUX, FNAUX);
        derive(0);
        bar_arrive(BAR_D0, FNTH);
        for (int c = 0; c < nchunk; ++c) {
            if (c >= 1) {
                bar_sync(BAR_X0 + ((c - 1) & 1), FNTH);
                epilogue(c - 1);
            }
            if (c + 1 < nchunk) {
                if (fast) tile_wait(c + 1);
                else cp_async_wait<1>();
                bar_sync(BAR_AUX, FNAUX);
                derive(c + 1);
                bar_arrive(BAR_D0 + ((c + 1) & 1), FNTH);
            }
            bar_sync(BAR_AUX, FNAUX);      // raw slot (c-1) % RING no longer read
            issue(c + 3);
        }
        bar_sync(BAR_X0 + ((nchunk - 1) & 1), FNTH);
        epilogue(nchunk - 1);
        if (!fast) {
            cp_async_wait<0>();
        } else if (at == 0 && *stop) {
            // copies that may still be landing in this CTA's shared memory: the last tile
            // issued into each slot, each given a second bounded wait before the CTA exits
            for (int k = max(0, issued - RING); k < issued; ++k)
                mbar_wait_bounded(&S.mbar[k % RING], (k / RING) & 1, FWD_WAIT_POLLS);
        }
        if (p.dsum) {                      // sum over the 4 thread groups of a channel
            S.red[at] = dsum;
            bar_sync(BAR_AUX, FNAUX);
            if (at < SCH && evalid) {
                float sum = 0.f;
#pragma unroll
                for (int m = 0; m < FNAUX / SCH; ++m) sum += S.red[at + m * SCH];
                p.dsum[(int64_t)bi * p.D + d0 + at] = sum;
            }
        }
    }
}

// =============================================================== launchers
// Helper-warp count of the forward.  A CTA is paced by its helper warps, so two per SM
// sub-partition (256 helper threads) is faster when each SM holds one CTA.  When the grid
// has more CTAs than SMs and the 128-helper CTA fits twice on an SM (bf16 inputs: 95
// registers, 81 KB of shared memory), two co-resident CTAs -- two recurrence warps per
// sub-partition, one wave instead of two -- are faster.
template <typename Tin, bool HAS_Z>
static FwdMaps fwd_maps(const ScanDev& p) {
    FwdMaps m{};
    const int es = sizeof(Tin);
    bool ok = encode_3d(&m.u, p.u, es, p.D, p.L, p.b, p.u_sl, p.u_sb, SCH, FT) &&
              encode_3d(&m.dl, p.dl, es, p.D, p.L, p.b, p.dl_sl, p.dl_sb, SCH, FT) &&
              encode_3d(&m.B, p.B, es, p.N, p.L, p.b, p.B_sl, p.B_sb, NS, FT);
    if (ok && p.out) ok = encode_3d(&m.C, p.C, es, p.N, p.L, p.b, p.C_sl, p.C_sb, NS, FT);
    if (ok && HAS_Z && p.out) ok = encode_3d(&m.z, p.z, es, p.D, p.L, p.b, p.z_sl, p.z_sb, SCH, FT);
    m.ok = ok ? 1 : 0;
    return m;
}

template <typename Tin, typename Tout, bool HAS_Z>
static cudaError_t launch_fwd_t(const ScanDev& p0, cudaStream_t st) {
    ScanDev p = p0;
    p.err = wait_status_address();               // where a timed-out tile wait is recorded
    const FwdMaps maps = fwd_maps<Tin, HAS_Z>(p);
    auto k2 = p.out ? scan_fwd_kernel<Tin, Tout, HAS_Z, true, 256> : scan_fwd_kernel<Tin, Tout, HAS_Z, false, 256>;
    auto k1 = p.out ? scan_fwd_kernel<Tin, Tout, HAS_Z, true, 128> : scan_fwd_kernel<Tin, Tout, HAS_Z, false, 128>;
    if constexpr (HAS_Z) {
        if (p.gw && p.out) {
            k2 = scan_fwd_kernel<Tin, Tout, true, true, 256, true>;
            k1 = scan_fwd_kernel<Tin, Tout, true, true, 128, true>;
        }
    }
    const int smem = sizeof(FwdSmem<Tin>);
    dim3 grid((p.D + SCH - 1) / SCH, p.b);
    const long long nblocks = (long long)grid.x * grid.y;
    cudaError_t e = allow_smem(k1, smem);
    if (e != cudaSuccess) return e;
    int sms = 0, per_sm = 0;
    e = sm_fit(k1, NSCAN + 128, smem, &sms, &per_sm);
    if (e != cudaSuccess) return e;
    if (nblocks > sms && per_sm >= 2) {
        k1<<<grid, NSCAN + 128, smem, st>>>(p, maps);
    } else {
        e = allow_smem(k2, smem);
        if (e != cudaSuccess) return e;
        k2<<<grid, NSCAN + 256, smem, st>>>(p, maps);
    }
    return cudaGetLastError();
}

cudaError_t launch_scan_fwd(const ScanDev& p, int in_dtype, int out_dtype, bool has_z, cudaStream_t st) {
    if (in_dtype == SWX_DTYPE_F32) {
        if (out_dtype == SWX_DTYPE_F32)
            return has_z ? launch_fwd_t<float, float, true>(p, st) : launch_fwd_t<float, float, false>(p, st);
        return has_z ? launch_fwd_t<float, __nv_bfloat16, true>(p, st)
                     : launch_fwd_t<float, __nv_bfloat16, false>(p, st);
    }
    if (out_dtype == SWX_DTYPE_F32)
        return has_z ? launch_fwd_t<__nv_bfloat16, float, true>(p, st)
                     : launch_fwd_t<__nv_bfloat16, float, false>(p, st);
    return has_z ? launch_fwd_t<__nv_bfloat16, __nv_bfloat16, true>(p, st)
                 : launch_fwd_t<__nv_bfloat16, __nv_bfloat16, false>(p, st);
}

}  // namespace swx
