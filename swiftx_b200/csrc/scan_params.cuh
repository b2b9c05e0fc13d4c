// Device-side parameter block shared by the scan kernels and their launchers.
#pragma once

#include <stdint.h>

namespace swx {

struct ScanDev {
    int b, L, D, N;
    int nck;                 // number of 16-step checkpoint slabs = ceil(L / 16)
    int softplus;
    int a_log;               // A holds log(-A): the kernels use -expf(A[i]); dA is d/d log(-A)
    // inputs (element strides; channel / state stride is 1)
    const void* u;  int64_t u_sb, u_sl;
    const void* dl; int64_t dl_sb, dl_sl;
    const void* z;  int64_t z_sb, z_sl;
    const void* B;  int64_t B_sb, B_sl;
    const void* C;  int64_t C_sb, C_sl;
    const float* A;
    const float* Dskip;
    const float* dbias;
    const float* h0;
    // 16-byte cp.async is legal for these tiles
    bool vec_u, vec_dl, vec_z, vec_B, vec_C, vec_dout, vec_yp;
    // forward outputs
    void* out;
    float* h_last;
    float* ck;               // (b, nck, D, 16)
    float* dsum;             // (b, D) sum over t of delta_eff, optional
    float* ypre;             // (b, L, D) fp32 pre-gate output: forward writes, backward reads
    // backward
    const void* dout; int64_t dout_sb, dout_sl;
    void* du; void* ddl; void* dz; void* dB; void* dC;
    int64_t dz_sb, dz_sl;    // element strides of dz (dense: L*D, D)
    float* dA; float* dD; float* ddbias; float* dh0;
    float* ws_bc;            // (nblk, b, L, 2, 16) per-CTA dB/dC partials
    float* ws_a;             // (b, D, 16)
    float* ws_d;             // (b, D)
    float* ws_bias;          // (b, D)
    int nblk;                // CTAs along D
    // time-segmented backward (scan_bwd_seg.cu): the sequence is cut into nseg segments
    // of seg_len steps (a multiple of 16, the last one may be shorter), walked in
    // parallel; the reverse carry entering each segment is chained from per-sub-segment
    // summaries (sub_len steps, dividing seg_len)
    int seg_len, nseg, sub_len, nsub, first_sub;
    int nblk64;              // 64-channel blocks along D
    float* ws_q;             // (nsub, b, D, 16) local carry a_t0 * g_t0 of each sub-segment
    float* ws_s;             // (nsub, b, D) sum of delta_eff over each sub-segment
    int* err;                // optional: set to SWX_ERR_TIMEOUT when a bounded wait gave up
    // SiftX pathway mix fused into the gate: out = y * gw[b, t, gof[d]] * silu(z)
    const float* gw; int64_t gw_sb, gw_sl;   // (b, L, ngroups) fp32, or nullptr
    const int* gof;                            // (D,) group of each channel
    int ngroups;
    float* dgw;                                // (b, L, ngroups) backward output, optional
    // the correction of a split forward (rows = segments of seg_g consecutive segments per
    // batch row): the first segment of each row needs none when the row starts from zero
    int seg_g, skip_first_seg;
};

// Weight of channel d's group at step t of row bi (the row's base and the channel's group
// resolved by the caller): 1 without the mix.
__device__ __forceinline__ float group_weight(const ScanDev& p, int bi, int64_t t, int g) {
    return p.gw ? p.gw[(int64_t)bi * p.gw_sb + t * p.gw_sl + g] : 1.f;
}

}  // namespace swx
