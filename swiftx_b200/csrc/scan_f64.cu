// float64 selective scan, forward and backward.
//
// The path for float64 inputs: the reference runs its scan in the input dtype (h is
// built with u.dtype, models/selective_scan.py:52) and its tests check float64 gradients
// with torch.autograd.gradcheck (tests/test_selective_scan.py:53-55, 89-93), which needs
// float64 arithmetic end to end.  Throughput is not the aim here: one thread walks one
// channel of one batch row through the whole sequence with its N states in registers.
//
// With in_dtype == SWX_DTYPE_F64 every floating-point pointer of the argument block holds
// float64 values (A, Dskip, delta_bias, h0, h_last, checkpoints, delta_sum, out_pre, dA,
// dD, ddelta_bias, dh0 included); the checkpoint buffer holds
// swx_scan_checkpoint_floats() float64 values.
//
// Backward: 16-step chunks walked last to first, states and decays of a chunk recomputed
// from the forward's checkpoint (models/selective_scan.py:211-243), the reverse recurrence
// g_t = a_{t+1} g_{t+1} + dy_t C_t, and fixed-order reductions: dB / dC summed over the 32
// channels of a warp by a butterfly of shuffles, then over channel blocks and dA / dD /
// d(delta_bias) over batch rows by a second kernel -- no atomics, deterministic.
#include "common.cuh"
#include "scan_params.cuh"

namespace swx {
namespace {

constexpr int F64_CH = 32;   // channels per CTA (one warp)

__device__ __forceinline__ double softplus_d(double x) { return x > 20.0 ? x : log1p(exp(x)); }
__device__ __forceinline__ double sigmoid_d(double x) { return 1.0 / (1.0 + exp(-x)); }

__device__ __forceinline__ double load_A_d(const ScanDev& p, int64_t i) {
    const double a = reinterpret_cast<const double*>(p.A)[i];
    return p.a_log ? -exp(a) : a;
}

__global__ void scan_fwd_f64_kernel(const ScanDev p) {
    const int d = blockIdx.x * F64_CH + threadIdx.x;
    const int bi = blockIdx.y;
    if (d >= p.D) return;
    const double* u = static_cast<const double*>(p.u) + bi * p.u_sb + d;
    const double* dl = static_cast<const double*>(p.dl) + bi * p.dl_sb + d;
    const double* z = p.z ? static_cast<const double*>(p.z) + bi * p.z_sb + d : nullptr;
    const double* Bm = static_cast<const double*>(p.B) + bi * p.B_sb;
    const double* Cm = static_cast<const double*>(p.C) + bi * p.C_sb;
    const double* h0 = reinterpret_cast<const double*>(p.h0);
    const double bias = p.dbias ? reinterpret_cast<const double*>(p.dbias)[d] : 0.0;
    const double Dv = p.Dskip ? reinterpret_cast<const double*>(p.Dskip)[d] : 0.0;
    double* ck = reinterpret_cast<double*>(p.ck);
    double* ypre = reinterpret_cast<double*>(p.ypre);
    double* out = static_cast<double*>(p.out);
    double A[NS], h[NS];
#pragma unroll
    for (int n = 0; n < NS; ++n) {
        A[n] = n < p.N ? load_A_d(p, (int64_t)d * p.N + n) : 0.0;
        h[n] = (n < p.N && h0) ? h0[((int64_t)bi * p.D + d) * p.N + n] : 0.0;
    }
    double dsum = 0.0;
    for (int t = 0; t < p.L; ++t) {
        if (ck && (t % TCK) == 0) {
            double* c = ck + (((int64_t)bi * p.nck + t / TCK) * p.D + d) * NS;
#pragma unroll
            for (int n = 0; n < NS; ++n) c[n] = h[n];
        }
        const double raw = dl[(int64_t)t * p.dl_sl] + bias;
        const double dt = p.softplus ? softplus_d(raw) : raw;
        dsum += dt;
        const double uu = u[(int64_t)t * p.u_sl];
        const double du = dt * uu;
        double y = 0.0;
#pragma unroll
        for (int n = 0; n < NS; ++n) {
            if (n < p.N) {
                const double a = exp(dt * A[n]);
                h[n] = a * h[n] + du * Bm[(int64_t)t * p.B_sl + n];
                y += Cm[(int64_t)t * p.C_sl + n] * h[n];
            }
        }
        y += Dv * uu;
        const int64_t o = ((int64_t)bi * p.L + t) * p.D + d;
        if (ypre) ypre[o] = y;
        if (z) {
            const double zz = z[(int64_t)t * p.z_sl];
            y *= zz * sigmoid_d(zz);
        }
        if (out) out[o] = y;
    }
    if (p.h_last) {
        double* hl = reinterpret_cast<double*>(p.h_last) + ((int64_t)bi * p.D + d) * p.N;
        for (int n = 0; n < p.N; ++n) hl[n] = h[n];
    }
    if (p.dsum) reinterpret_cast<double*>(p.dsum)[(int64_t)bi * p.D + d] = dsum;
}

__global__ void __launch_bounds__(F64_CH) scan_bwd_f64_kernel(const ScanDev p) {
    const int lane = threadIdx.x;
    const int d = blockIdx.x * F64_CH + lane;
    const int bi = blockIdx.y;
    const bool ok = d < p.D;          // lanes past D take part in the shuffles with zeros
    const int dc = ok ? d : 0;
    const double* u = static_cast<const double*>(p.u) + bi * p.u_sb + dc;
    const double* dl = static_cast<const double*>(p.dl) + bi * p.dl_sb + dc;
    const double* z = p.z ? static_cast<const double*>(p.z) + bi * p.z_sb + dc : nullptr;
    const double* dout = static_cast<const double*>(p.dout) + bi * p.dout_sb + dc;
    const double* Bm = static_cast<const double*>(p.B) + bi * p.B_sb;
    const double* Cm = static_cast<const double*>(p.C) + bi * p.C_sb;
    const double* ck = reinterpret_cast<const double*>(p.ck);
    const double bias = p.dbias ? reinterpret_cast<const double*>(p.dbias)[dc] : 0.0;
    const double Dv = p.Dskip ? reinterpret_cast<const double*>(p.Dskip)[dc] : 0.0;
    double* gdu = static_cast<double*>(p.du);
    double* gddl = static_cast<double*>(p.ddl);
    double* gdz = static_cast<double*>(p.dz);
    double* wbc = reinterpret_cast<double*>(p.ws_bc) + ((int64_t)blockIdx.x * p.b + bi) * p.L * 2 * NS;
    double A[NS], g[NS], an[NS], dA[NS];
#pragma unroll
    for (int n = 0; n < NS; ++n) {
        A[n] = (ok && n < p.N) ? load_A_d(p, (int64_t)d * p.N + n) : 0.0;
        g[n] = an[n] = dA[n] = 0.0;
    }
    double accD = 0.0, accB = 0.0;
    for (int c = p.nck - 1; c >= 0; --c) {
        const int t0 = c * TCK, nt = min(TCK, p.L - t0);
        double hck[NS], hs[TCK][NS], as[TCK][NS];
#pragma unroll
        for (int n = 0; n < NS; ++n) hck[n] = ok ? ck[(((int64_t)bi * p.nck + c) * p.D + d) * NS + n] : 0.0;
        {
            double h[NS];
#pragma unroll
            for (int n = 0; n < NS; ++n) h[n] = hck[n];
            for (int tt = 0; tt < nt; ++tt) {
                const int64_t t = t0 + tt;
                const double raw = ok ? dl[t * p.dl_sl] + bias : 0.0;
                const double dt = p.softplus ? softplus_d(raw) : raw;
                const double du = dt * (ok ? u[t * p.u_sl] : 0.0);
#pragma unroll
                for (int n = 0; n < NS; ++n) {
                    const double a = n < p.N ? exp(dt * A[n]) : 0.0;
                    h[n] = n < p.N ? a * h[n] + du * Bm[t * p.B_sl + n] : 0.0;
                    as[tt][n] = a;
                    hs[tt][n] = h[n];
                }
            }
        }
        for (int tt = nt - 1; tt >= 0; --tt) {
            const int64_t t = t0 + tt;
            const double raw = ok ? dl[t * p.dl_sl] + bias : 0.0;
            const double dt = p.softplus ? softplus_d(raw) : raw;
            const double dsp = p.softplus ? (raw > 20.0 ? 1.0 : sigmoid_d(raw)) : 1.0;
            const double uu = ok ? u[t * p.u_sl] : 0.0;
            const double dov = ok ? dout[t * p.dout_sl] : 0.0;
            double dy = dov, sz = 0.0, zz = 0.0;
            if (z) {
                zz = ok ? z[t * p.z_sl] : 0.0;
                sz = sigmoid_d(zz);
                dy = dov * zz * sz;
            }
            double sgB = 0.0, sdA = 0.0, yv = 0.0;
            double dbc[2 * NS];
#pragma unroll
            for (int n = 0; n < NS; ++n) {
                if (n < p.N) {
                    const double Bv = Bm[t * p.B_sl + n], Cv = Cm[t * p.C_sl + n];
                    g[n] = an[n] * g[n] + Cv * dy;
                    const double hp = tt > 0 ? hs[tt - 1][n] : hck[n];
                    const double w = g[n] * as[tt][n] * hp;
                    dA[n] += w * dt;
                    sdA += w * A[n];
                    sgB += g[n] * Bv;
                    yv += Cv * hs[tt][n];
                    dbc[n] = g[n] * dt * uu;
                    dbc[NS + n] = dy * hs[tt][n];
                    an[n] = as[tt][n];
                } else {
                    dbc[n] = dbc[NS + n] = 0.0;
                }
            }
            const double gdelta = uu * sgB + sdA;
            const double graw = gdelta * dsp;
            if (ok) {
                const int64_t o = ((int64_t)bi * p.L + t) * p.D + d;
                gdu[o] = dt * sgB + Dv * dy;
                gddl[o] = graw;
                if (z) gdz[o] = dov * (yv + Dv * uu) * sz * (1.0 + zz * (1.0 - sz));
                accD += dy * uu;
                accB += graw;
            }
            // dB | dC: sum over the warp's channels (butterfly, the same order on every run)
#pragma unroll
            for (int k = 0; k < 2 * NS; ++k) {
                double v = dbc[k];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
                dbc[k] = v;
            }
            if (lane == 0) {
#pragma unroll
                for (int k = 0; k < 2 * NS; ++k) wbc[t * 2 * NS + k] = dbc[k];
            }
        }
    }
    if (ok) {
        double* wa = reinterpret_cast<double*>(p.ws_a) + ((int64_t)bi * p.D + d) * NS;
#pragma unroll
        for (int n = 0; n < NS; ++n) wa[n] = dA[n];
        reinterpret_cast<double*>(p.ws_d)[(int64_t)bi * p.D + d] = accD;
        reinterpret_cast<double*>(p.ws_bias)[(int64_t)bi * p.D + d] = accB;
        if (p.dh0) {
            double* dh = reinterpret_cast<double*>(p.dh0) + ((int64_t)bi * p.D + d) * p.N;
            for (int n = 0; n < p.N; ++n) dh[n] = an[n] * g[n];
        }
    }
}

// Fixed-order sums of the partials: dB / dC over channel blocks, dA / dD / d(delta_bias)
// over batch rows.
__global__ void scan_bwd_f64_finalize_kernel(const ScanDev p) {
    const int64_t nrow = (int64_t)p.b * p.L;
    const int64_t nbc = nrow * 2 * NS;
    const int64_t total = nbc + (int64_t)p.D * p.N + p.D;
    const int64_t slab = nrow * 2 * NS;
    const double* wbc = reinterpret_cast<const double*>(p.ws_bc);
    const double* wa = reinterpret_cast<const double*>(p.ws_a);
    const double* wd = reinterpret_cast<const double*>(p.ws_d);
    const double* wb = reinterpret_cast<const double*>(p.ws_bias);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        if (i < nbc) {
            const int col = (int)(i % (2 * NS));
            const int kind = col >= NS, n = col % NS;
            if (n >= p.N) continue;
            double s = 0.0;
            for (int k = 0; k < p.nblk; ++k) s += wbc[i + (int64_t)k * slab];
            double* dst = static_cast<double*>(kind ? p.dC : p.dB);
            dst[(i / (2 * NS)) * p.N + n] = s;
        } else if (i < nbc + (int64_t)p.D * p.N) {
            const int64_t r = i - nbc;
            const int dd = (int)(r / p.N), n = (int)(r % p.N);
            double s = 0.0;
            for (int bi = 0; bi < p.b; ++bi) s += wa[((int64_t)bi * p.D + dd) * NS + n];
            reinterpret_cast<double*>(p.dA)[r] = p.a_log ? s * load_A_d(p, r) : s;
        } else {
            const int dd = (int)(i - nbc - (int64_t)p.D * p.N);
            double sD = 0.0, sB = 0.0;
            for (int bi = 0; bi < p.b; ++bi) {
                sD += wd[(int64_t)bi * p.D + dd];
                sB += wb[(int64_t)bi * p.D + dd];
            }
            if (p.dD) reinterpret_cast<double*>(p.dD)[dd] = sD;
            if (p.ddbias) reinterpret_cast<double*>(p.ddbias)[dd] = sB;
        }
    }
}

}  // namespace

cudaError_t launch_scan_fwd_f64(const ScanDev& p, cudaStream_t st) {
    dim3 grid((p.D + F64_CH - 1) / F64_CH, p.b);
    scan_fwd_f64_kernel<<<grid, F64_CH, 0, st>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_scan_bwd_f64(const ScanDev& p, cudaStream_t st) {
    dim3 grid((p.D + F64_CH - 1) / F64_CH, p.b);
    scan_bwd_f64_kernel<<<grid, F64_CH, 0, st>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int64_t total = 2LL * NS * p.b * p.L + (int64_t)p.D * p.N + p.D;
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 8);
    scan_bwd_f64_finalize_kernel<<<blocks, 256, 0, st>>>(p);
    return cudaGetLastError();
}

}  // namespace swx
