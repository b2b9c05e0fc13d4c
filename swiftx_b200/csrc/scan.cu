// Selective scan forward / backward kernels for sm_100a.
//
// Work decomposition (both directions): one CTA owns 32 channels of one batch
// row for the whole sequence; each thread owns one channel and 4 of its 16
// states, so the N=16 state of a channel lives in the fp32 registers of 4
// adjacent lanes and a warp covers 8 channels.  Time is walked sequentially
// (a state chain is a first-order recurrence); the channel-shared B_t / C_t and
// the per-channel u, delta, z, dout tiles are staged in shared memory by
// double-buffered 16-byte cp.async, one chunk ahead of the math.
//
// Per staged chunk the CTA runs three phases separated by __syncthreads:
//   A  per (t, channel) scalars, computed once per channel instead of once per
//      state: delta_eff = softplus(delta + bias), delta_eff*u, the gate.
//   B  the recurrence: a = 2^(delta_eff * A*log2e) on the MUFU unit, h = a*h + delta_eff*u*B.
//   C  per (t, channel) epilogue: sum of the 4 lanes' partial readouts, D-skip,
//      SiLU(z) gate, coalesced store.
//
// Backward: chunks of 16 steps are walked last to first.  Each chunk restarts
// from the state checkpoint the forward stored, recomputes the 16 states and
// decays into registers (one exp per element), then runs the reverse
// recurrence g_t = a_{t+1} g_{t+1} + dy_t C_t (models/selective_scan.py:146-148,
// :225-238).  Channel reductions (dB, dC) and state reductions (du, ddelta)
// go through shared memory in fixed order; cross-CTA and cross-batch sums are
// written as partials and summed by a second kernel in fixed order, so every
// gradient is bit-reproducible (no float atomics, unlike
// models/triton_scan.py:101-102,108-109).
#include "common.cuh"
#include "scan_params.cuh"

namespace swx {

constexpr int SCH = 32;   // channels per CTA
constexpr int SNT = 128;  // threads per CTA
constexpr int FTS = 64;   // staged steps per forward chunk (multiple of TCK)

// =============================================================== forward
template <typename Tin>
struct FwdSmem {
    Tin u[2][FTS][SCH];
    Tin dl[2][FTS][SCH];
    Tin z[2][FTS][SCH];
    Tin B[2][FTS][NS];
    Tin C[2][FTS][NS];
    float dlt[FTS][SCH];        // delta_eff
    float dlu[FTS][SCH];        // delta_eff * u
    float Bf[FTS][NS];
    float Cf[FTS][NS];
    float yp[FTS][SCH][4];      // partial readouts of the 4 state groups
};

template <typename Tin, typename Tout, bool HAS_Z>
__global__ void __launch_bounds__(SNT, 1) scan_fwd_kernel(const ScanDev p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    FwdSmem<Tin>& S = *reinterpret_cast<FwdSmem<Tin>*>(smem_raw);

    const int tid = threadIdx.x;
    const int bi = blockIdx.y;
    const int d0 = blockIdx.x * SCH;
    const int nd = min(SCH, p.D - d0);
    // recurrence role
    const int ch = tid >> 2, j = tid & 3;
    const int d = d0 + ch;
    const bool dvalid = ch < nd;
    // per-(t, channel) role
    const int ech = tid & (SCH - 1);
    const bool evalid = ech < nd;
    const float eD = (p.Dskip && evalid) ? p.Dskip[d0 + ech] : 0.f;
    const float ebias = (p.dbias && evalid) ? p.dbias[d0 + ech] : 0.f;

    float A2[4], h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int n = 4 * j + i;
        const bool ok = dvalid && n < p.N;
        A2[i] = ok ? p.A[(int64_t)d * p.N + n] * LOG2E : 0.f;
        h[i] = (ok && p.h0) ? p.h0[((int64_t)bi * p.D + d) * p.N + n] : 0.f;
    }

    const Tin* gu = static_cast<const Tin*>(p.u) + bi * p.u_sb + d0;
    const Tin* gdl = static_cast<const Tin*>(p.dl) + bi * p.dl_sb + d0;
    const Tin* gz = HAS_Z ? static_cast<const Tin*>(p.z) + bi * p.z_sb + d0 : nullptr;
    const Tin* gB = static_cast<const Tin*>(p.B) + bi * p.B_sb;
    const Tin* gC = static_cast<const Tin*>(p.C) + bi * p.C_sb;
    Tout* gout = static_cast<Tout*>(p.out) + (int64_t)bi * p.L * p.D + d0;

    const int nchunks = (p.L + FTS - 1) / FTS;
    auto issue = [&](int c) {
        const int t0 = c * FTS, rv = min(FTS, p.L - t0), buf = c & 1;
        stage_tile<Tin, SCH>(&S.u[buf][0][0], gu + t0 * p.u_sl, p.u_sl, FTS, rv, nd, p.vec_u, tid, SNT);
        stage_tile<Tin, SCH>(&S.dl[buf][0][0], gdl + t0 * p.dl_sl, p.dl_sl, FTS, rv, nd, p.vec_dl, tid, SNT);
        if (HAS_Z)
            stage_tile<Tin, SCH>(&S.z[buf][0][0], gz + t0 * p.z_sl, p.z_sl, FTS, rv, nd, p.vec_z, tid, SNT);
        stage_tile<Tin, NS>(&S.B[buf][0][0], gB + t0 * p.B_sl, p.B_sl, FTS, rv, p.N, p.vec_B, tid, SNT);
        stage_tile<Tin, NS>(&S.C[buf][0][0], gC + t0 * p.C_sl, p.C_sl, FTS, rv, p.N, p.vec_C, tid, SNT);
        cp_async_commit();
    };

    issue(0);
    for (int c = 0; c < nchunks; ++c) {
        if (c + 1 < nchunks) issue(c + 1); else cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const int buf = c & 1, t0 = c * FTS, nt = min(FTS, p.L - t0);

        // ---- phase A: per (t, channel) scalars
        for (int i = tid; i < FTS * SCH; i += SNT) {
            const int t = i / SCH, cc = i % SCH;
            const float raw = Elem<Tin>::to_f(S.dl[buf][t][cc]) + ebias;
            const float dte = p.softplus ? softplus_f(raw) : raw;
            S.dlt[t][cc] = dte;
            S.dlu[t][cc] = dte * Elem<Tin>::to_f(S.u[buf][t][cc]);
        }
        for (int i = tid; i < FTS * NS; i += SNT) {
            (&S.Bf[0][0])[i] = Elem<Tin>::to_f((&S.B[buf][0][0])[i]);
            (&S.Cf[0][0])[i] = Elem<Tin>::to_f((&S.C[buf][0][0])[i]);
        }
        __syncthreads();

        // ---- phase B: recurrence
        float* ckp = (p.ck && dvalid) ? p.ck + (((int64_t)bi * p.nck + t0 / TCK) * p.D + d) * NS + 4 * j
                                      : nullptr;
        for (int t = 0; t < nt; ++t) {
            if ((t & (TCK - 1)) == 0 && ckp) {
                *reinterpret_cast<float4*>(ckp) = make_float4(h[0], h[1], h[2], h[3]);
                ckp += (int64_t)p.D * NS;
            }
            const float dte = S.dlt[t][ch], dtu = S.dlu[t][ch];
            const float4 b4 = *reinterpret_cast<const float4*>(&S.Bf[t][4 * j]);
            const float4 c4 = *reinterpret_cast<const float4*>(&S.Cf[t][4 * j]);
            h[0] = fmaf(ex2(dte * A2[0]), h[0], dtu * b4.x);
            h[1] = fmaf(ex2(dte * A2[1]), h[1], dtu * b4.y);
            h[2] = fmaf(ex2(dte * A2[2]), h[2], dtu * b4.z);
            h[3] = fmaf(ex2(dte * A2[3]), h[3], dtu * b4.w);
            float y = h[0] * c4.x;
            y = fmaf(h[1], c4.y, y);
            y = fmaf(h[2], c4.z, y);
            y = fmaf(h[3], c4.w, y);
            S.yp[t][ch][j] = y;
        }
        __syncthreads();

        // ---- phase C: readout reduction, D-skip, gate, store
        if (evalid) {
            for (int t = tid / SCH; t < nt; t += SNT / SCH) {
                const float4 q = *reinterpret_cast<const float4*>(&S.yp[t][ech][0]);
                float y = (q.x + q.y) + (q.z + q.w);
                y = fmaf(eD, Elem<Tin>::to_f(S.u[buf][t][ech]), y);
                if (HAS_Z) y *= silu_f(Elem<Tin>::to_f(S.z[buf][t][ech]));
                gout[(int64_t)(t0 + t) * p.D + ech] = Elem<Tout>::from_f(y);
            }
        }
        __syncthreads();
    }

    if (p.h_last && dvalid) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int n = 4 * j + i;
            if (n < p.N) p.h_last[((int64_t)bi * p.D + d) * p.N + n] = h[i];
        }
    }
}

// =============================================================== backward
template <typename Tin>
struct BwdSmem {
    Tin u[2][TCK][SCH];
    Tin dl[2][TCK][SCH];
    Tin z[2][TCK][SCH];
    Tin dout[2][TCK][SCH];
    Tin B[2][TCK][NS];
    Tin C[2][TCK][NS];
    float dlt[TCK][SCH];
    float dlu[TCK][SCH];
    float dy[TCK][SCH];
    float Bf[TCK][NS];
    float Cf[TCK][NS];
    float nred[3][TCK][SCH][4];      // sum_n g*B, sum_n g*a*h_prev*A, sum_n h*C  (per state group)
    float bc[2][TCK][SCH][NS];       // dB, dC contributions per channel
    float red[2][SNT];               // per-thread dD / dbias accumulators
};

template <typename Tin, bool HAS_Z>
__global__ void __launch_bounds__(SNT, 1) scan_bwd_kernel(const ScanDev p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    BwdSmem<Tin>& S = *reinterpret_cast<BwdSmem<Tin>*>(smem_raw);

    const int tid = threadIdx.x;
    const int bi = blockIdx.y;
    const int d0 = blockIdx.x * SCH;
    const int nd = min(SCH, p.D - d0);
    const int ch = tid >> 2, j = tid & 3;
    const int d = d0 + ch;
    const bool dvalid = ch < nd;
    const int ech = tid & (SCH - 1);
    const bool evalid = ech < nd;
    const float eD = (p.Dskip && evalid) ? p.Dskip[d0 + ech] : 0.f;
    const float ebias = (p.dbias && evalid) ? p.dbias[d0 + ech] : 0.f;

    float A2[4], An[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int n = 4 * j + i;
        An[i] = (dvalid && n < p.N) ? p.A[(int64_t)d * p.N + n] : 0.f;
        A2[i] = An[i] * LOG2E;
    }

    const Tin* gu = static_cast<const Tin*>(p.u) + bi * p.u_sb + d0;
    const Tin* gdl = static_cast<const Tin*>(p.dl) + bi * p.dl_sb + d0;
    const Tin* gz = HAS_Z ? static_cast<const Tin*>(p.z) + bi * p.z_sb + d0 : nullptr;
    const Tin* gdo = static_cast<const Tin*>(p.dout) + bi * p.dout_sb + d0;
    const Tin* gB = static_cast<const Tin*>(p.B) + bi * p.B_sb;
    const Tin* gC = static_cast<const Tin*>(p.C) + bi * p.C_sb;
    const int64_t orow = (int64_t)bi * p.L * p.D + d0;      // dense (b, L, D) outputs
    Tin* gdu = static_cast<Tin*>(p.du) + orow;
    Tin* gddl = static_cast<Tin*>(p.ddl) + orow;
    Tin* gdz = HAS_Z ? static_cast<Tin*>(p.dz) + orow : nullptr;
    float* wbc = p.ws_bc + ((int64_t)blockIdx.x * p.b + bi) * p.L * 2 * NS;

    auto issue = [&](int c) {
        const int t0 = c * TCK, rv = min(TCK, p.L - t0), buf = c & 1;
        stage_tile<Tin, SCH>(&S.u[buf][0][0], gu + t0 * p.u_sl, p.u_sl, TCK, rv, nd, p.vec_u, tid, SNT);
        stage_tile<Tin, SCH>(&S.dl[buf][0][0], gdl + t0 * p.dl_sl, p.dl_sl, TCK, rv, nd, p.vec_dl, tid, SNT);
        if (HAS_Z)
            stage_tile<Tin, SCH>(&S.z[buf][0][0], gz + t0 * p.z_sl, p.z_sl, TCK, rv, nd, p.vec_z, tid, SNT);
        stage_tile<Tin, SCH>(&S.dout[buf][0][0], gdo + t0 * p.dout_sl, p.dout_sl, TCK, rv, nd, p.vec_dout, tid, SNT);
        stage_tile<Tin, NS>(&S.B[buf][0][0], gB + t0 * p.B_sl, p.B_sl, TCK, rv, p.N, p.vec_B, tid, SNT);
        stage_tile<Tin, NS>(&S.C[buf][0][0], gC + t0 * p.C_sl, p.C_sl, TCK, rv, p.N, p.vec_C, tid, SNT);
        cp_async_commit();
    };

    float g[4] = {0.f, 0.f, 0.f, 0.f};      // dL/dh_t carried backwards in time
    float an[4] = {0.f, 0.f, 0.f, 0.f};     // a_{t+1}; zero after the last step
    float dAacc[4] = {0.f, 0.f, 0.f, 0.f};
    float accD = 0.f, accB = 0.f;

    issue(p.nck - 1);
    for (int c = p.nck - 1; c >= 0; --c) {
        if (c > 0) issue(c - 1); else cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const int buf = c & 1, t0 = c * TCK, nt = min(TCK, p.L - t0);

        // ---- phase A
        for (int i = tid; i < TCK * SCH; i += SNT) {
            const int t = i / SCH, cc = i % SCH;
            const float raw = Elem<Tin>::to_f(S.dl[buf][t][cc]) + ebias;
            const float dte = p.softplus ? softplus_f(raw) : raw;
            S.dlt[t][cc] = dte;
            S.dlu[t][cc] = dte * Elem<Tin>::to_f(S.u[buf][t][cc]);
            float dyv = Elem<Tin>::to_f(S.dout[buf][t][cc]);
            if (HAS_Z) dyv *= silu_f(Elem<Tin>::to_f(S.z[buf][t][cc]));
            S.dy[t][cc] = dyv;
        }
        for (int i = tid; i < TCK * NS; i += SNT) {
            (&S.Bf[0][0])[i] = Elem<Tin>::to_f((&S.B[buf][0][0])[i]);
            (&S.Cf[0][0])[i] = Elem<Tin>::to_f((&S.C[buf][0][0])[i]);
        }
        __syncthreads();

        // ---- phase B1: recompute the chunk's decays and states from its checkpoint
        float hck[4] = {0.f, 0.f, 0.f, 0.f};
        if (dvalid) {
            const float4 v = *reinterpret_cast<const float4*>(
                p.ck + (((int64_t)bi * p.nck + c) * p.D + d) * NS + 4 * j);
            hck[0] = v.x; hck[1] = v.y; hck[2] = v.z; hck[3] = v.w;
        }
        float a[TCK][4], hs[TCK][4];
        {
            float h0 = hck[0], h1 = hck[1], h2 = hck[2], h3 = hck[3];
#pragma unroll
            for (int t = 0; t < TCK; ++t) {
                if (t < nt) {
                    const float dte = S.dlt[t][ch], dtu = S.dlu[t][ch];
                    const float4 b4 = *reinterpret_cast<const float4*>(&S.Bf[t][4 * j]);
                    a[t][0] = ex2(dte * A2[0]);
                    a[t][1] = ex2(dte * A2[1]);
                    a[t][2] = ex2(dte * A2[2]);
                    a[t][3] = ex2(dte * A2[3]);
                    h0 = fmaf(a[t][0], h0, dtu * b4.x);
                    h1 = fmaf(a[t][1], h1, dtu * b4.y);
                    h2 = fmaf(a[t][2], h2, dtu * b4.z);
                    h3 = fmaf(a[t][3], h3, dtu * b4.w);
                    hs[t][0] = h0; hs[t][1] = h1; hs[t][2] = h2; hs[t][3] = h3;
                    if (HAS_Z) {
                        const float4 c4 = *reinterpret_cast<const float4*>(&S.Cf[t][4 * j]);
                        float y = h0 * c4.x;
                        y = fmaf(h1, c4.y, y);
                        y = fmaf(h2, c4.z, y);
                        y = fmaf(h3, c4.w, y);
                        S.nred[2][t][ch][j] = y;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) { a[t][i] = 0.f; hs[t][i] = 0.f; }
                }
            }
        }

        // ---- phase B2: reverse recurrence through the chunk
#pragma unroll
        for (int t = TCK - 1; t >= 0; --t) {
            if (t < nt) {
                const float dte = S.dlt[t][ch], dtu = S.dlu[t][ch], dyv = S.dy[t][ch];
                const float4 b4 = *reinterpret_cast<const float4*>(&S.Bf[t][4 * j]);
                const float4 c4 = *reinterpret_cast<const float4*>(&S.Cf[t][4 * j]);
                const float bb[4] = {b4.x, b4.y, b4.z, b4.w};
                const float cv[4] = {c4.x, c4.y, c4.z, c4.w};
                float sgb = 0.f, sda = 0.f;
                float gB4[4], gC4[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    g[i] = fmaf(an[i], g[i], dyv * cv[i]);
                    gC4[i] = dyv * hs[t][i];
                    gB4[i] = g[i] * dtu;
                    sgb = fmaf(g[i], bb[i], sgb);
                    const float hp = (t > 0) ? hs[t > 0 ? t - 1 : 0][i] : hck[i];
                    const float w = g[i] * a[t][i] * hp;
                    dAacc[i] = fmaf(w, dte, dAacc[i]);
                    sda = fmaf(w, An[i], sda);
                    an[i] = a[t][i];
                }
                *reinterpret_cast<float4*>(&S.bc[0][t][ch][4 * j]) = make_float4(gB4[0], gB4[1], gB4[2], gB4[3]);
                *reinterpret_cast<float4*>(&S.bc[1][t][ch][4 * j]) = make_float4(gC4[0], gC4[1], gC4[2], gC4[3]);
                S.nred[0][t][ch][j] = sgb;
                S.nred[1][t][ch][j] = sda;
            }
        }
        __syncthreads();

        // ---- phase C: per (t, channel) gradients
        if (evalid) {
            for (int t = tid / SCH; t < nt; t += SNT / SCH) {
                const float4 q0 = *reinterpret_cast<const float4*>(&S.nred[0][t][ech][0]);
                const float4 q1 = *reinterpret_cast<const float4*>(&S.nred[1][t][ech][0]);
                const float sgb = (q0.x + q0.y) + (q0.z + q0.w);
                const float sda = (q1.x + q1.y) + (q1.z + q1.w);
                const float uv = Elem<Tin>::to_f(S.u[buf][t][ech]);
                const float dte = S.dlt[t][ech], dyv = S.dy[t][ech];
                const float du = fmaf(dte, sgb, eD * dyv);
                const float ddte = fmaf(uv, sgb, sda);
                const float raw = Elem<Tin>::to_f(S.dl[buf][t][ech]) + ebias;
                const float draw = p.softplus ? (raw > 20.f ? ddte : ddte * sigmoid_f(raw)) : ddte;
                const int64_t o = (int64_t)(t0 + t) * p.D + ech;
                gdu[o] = Elem<Tin>::from_f(du);
                gddl[o] = Elem<Tin>::from_f(draw);
                if (HAS_Z) {
                    const float4 q2 = *reinterpret_cast<const float4*>(&S.nred[2][t][ech][0]);
                    const float y = fmaf(eD, uv, (q2.x + q2.y) + (q2.z + q2.w));
                    const float zv = Elem<Tin>::to_f(S.z[buf][t][ech]);
                    const float sg = sigmoid_f(zv);
                    const float dsilu = sg * fmaf(zv, 1.f - sg, 1.f);
                    gdz[o] = Elem<Tin>::from_f(Elem<Tin>::to_f(S.dout[buf][t][ech]) * y * dsilu);
                }
                accD = fmaf(dyv, uv, accD);
                accB += draw;
            }
        }
        // CTA partial of dB / dC for this chunk: fixed-order sum over the 32 channels
        for (int i = tid; i < 2 * TCK * NS; i += SNT) {
            const int kind = i / (TCK * NS), t = (i / NS) % TCK, n = i % NS;
            if (t < nt) {
                float s = 0.f;
#pragma unroll 8
                for (int cc = 0; cc < SCH; ++cc) s += S.bc[kind][t][cc][n];
                wbc[((int64_t)(t0 + t) * 2 + kind) * NS + n] = s;
            }
        }
        __syncthreads();
    }

    // per-(b, d, n) and per-(b, d) partials; summed over b by the finalize kernel
    if (dvalid) {
        *reinterpret_cast<float4*>(p.ws_a + ((int64_t)bi * p.D + d) * NS + 4 * j) =
            make_float4(dAacc[0], dAacc[1], dAacc[2], dAacc[3]);
        if (p.dh0) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int n = 4 * j + i;
                if (n < p.N) p.dh0[((int64_t)bi * p.D + d) * p.N + n] = an[i] * g[i];
            }
        }
    }
    S.red[0][tid] = accD;
    S.red[1][tid] = accB;
    __syncthreads();
    if (tid < SCH && tid < nd) {
        float sD = 0.f, sB = 0.f;
#pragma unroll
        for (int k = 0; k < SNT / SCH; ++k) { sD += S.red[0][tid + k * SCH]; sB += S.red[1][tid + k * SCH]; }
        p.ws_d[(int64_t)bi * p.D + d0 + tid] = sD;
        p.ws_bias[(int64_t)bi * p.D + d0 + tid] = sB;
    }
}

// Second pass: fixed-order sums of the partials.
template <typename Tin>
__global__ void scan_bwd_finalize_kernel(const ScanDev p) {
    const int64_t nbc = (int64_t)p.b * p.L * p.N;
    const int64_t total = 2 * nbc + (int64_t)p.D * p.N + p.D;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        if (i < 2 * nbc) {
            const int kind = i >= nbc;
            const int64_t r = kind ? i - nbc : i;
            const int n = r % p.N;
            const int64_t bl = r / p.N;               // bi * L + t
            const int bi = bl / p.L;
            const int64_t t = bl % p.L;
            float s = 0.f;
            for (int k = 0; k < p.nblk; ++k)
                s += p.ws_bc[(((int64_t)k * p.b + bi) * p.L + t) * 2 * NS + kind * NS + n];
            Tin* dst = static_cast<Tin*>(kind ? p.dC : p.dB);
            dst[r] = Elem<Tin>::from_f(s);
        } else if (i < 2 * nbc + (int64_t)p.D * p.N) {
            const int64_t r = i - 2 * nbc;
            const int dd = r / p.N, n = r % p.N;
            float s = 0.f;
            for (int bi = 0; bi < p.b; ++bi) s += p.ws_a[((int64_t)bi * p.D + dd) * NS + n];
            p.dA[r] = s;
        } else {
            const int dd = i - 2 * nbc - (int64_t)p.D * p.N;
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

// =============================================================== launchers
template <typename Tin, typename Tout, bool HAS_Z>
static cudaError_t launch_fwd_t(const ScanDev& p, cudaStream_t st) {
    auto k = scan_fwd_kernel<Tin, Tout, HAS_Z>;
    const int smem = sizeof(FwdSmem<Tin>);
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    dim3 grid((p.D + SCH - 1) / SCH, p.b);
    k<<<grid, SNT, smem, st>>>(p);
    return cudaGetLastError();
}

template <typename Tin, bool HAS_Z>
static cudaError_t launch_bwd_t(const ScanDev& p, cudaStream_t st) {
    auto k = scan_bwd_kernel<Tin, HAS_Z>;
    const int smem = sizeof(BwdSmem<Tin>);
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    dim3 grid((p.D + SCH - 1) / SCH, p.b);
    k<<<grid, SNT, smem, st>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int64_t total = 2LL * p.b * p.L * p.N + (int64_t)p.D * p.N + p.D;
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 8);
    scan_bwd_finalize_kernel<Tin><<<blocks, 256, 0, st>>>(p);
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

cudaError_t launch_scan_bwd(const ScanDev& p, int in_dtype, bool has_z, cudaStream_t st) {
    if (in_dtype == SWX_DTYPE_F32)
        return has_z ? launch_bwd_t<float, true>(p, st) : launch_bwd_t<float, false>(p, st);
    return has_z ? launch_bwd_t<__nv_bfloat16, true>(p, st) : launch_bwd_t<__nv_bfloat16, false>(p, st);
}

}  // namespace swx
