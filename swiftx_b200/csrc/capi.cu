// extern "C" entry points: argument checks, parameter packing, launches.
#include <algorithm>
#include <cstdint>

#include "common.cuh"
#include "scan_params.cuh"

namespace swx {
cudaError_t launch_scan_fwd(const ScanDev& p, int in_dtype, int out_dtype, bool has_z, cudaStream_t st);
cudaError_t scan_bwd_seg_ctas_per_sm(const ScanDev& p, int in_dtype, bool has_z, int* ctas);
cudaError_t launch_scan_fwd_f64(const ScanDev& p, cudaStream_t st);
cudaError_t launch_scan_bwd_f64(const ScanDev& p, cudaStream_t st);
cudaError_t launch_scan_bwd_seg(const ScanDev& p, int in_dtype, bool has_z, cudaStream_t st);
cudaError_t launch_scan_bwd_rows(const ScanDev& p, bool has_z, cudaStream_t st);
cudaError_t launch_group_w_grad(const ScanDev& p, int in_dtype, cudaStream_t st);
cudaError_t scan_bwd_rows_applicable(const ScanDev& p, int in_dtype, bool has_z, bool* yes);
cudaError_t launch_scan_correct(const ScanDev& p, int in_dtype, int out_dtype, bool has_z, float* ws,
                                cudaStream_t st, bool fix);
cudaError_t launch_seg_combine(const ScanDev& p, int G, const float* h_end, const float* dsum, float* h_in,
                               float* h_last, float* dsum_out, cudaStream_t st);
int64_t scan_correct_workspace_floats(int64_t b, int64_t L, int64_t D);
}  // namespace swx

namespace {

int elem_size(int dt) {
    return dt == SWX_DTYPE_F32 ? 4 : (dt == SWX_DTYPE_BF16 ? 2 : (dt == SWX_DTYPE_F64 ? 8 : 0));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 16-byte cp.async is legal for every row start of a (b, L, W) tile.
bool vec_ok(const void* p, int64_t sb, int64_t sl, int es) {
    return p && aligned16(p) && ((sb * es) % 16 == 0) && ((sl * es) % 16 == 0);
}

constexpr int64_t kAlign = 256;
int64_t round_up(int64_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// Segments of the time-segmented backward, a function of (L, D) and of the batch below
// 8 rows: results do not depend on the device, and the rows of batches of 8 rows or more
// get bit-identical gradients whether they are passed together or in smaller batches of
// 8 or more.  Sized for about two 64-channel CTAs per SM of a 148-SM B200, with segments
// of at least 128 steps; the reverse carries are summarised over sub-segments of up to
// 128 steps that divide a segment.
struct SegPlan {
    int64_t seg_len, nseg, sub_len, nsub, first_sub, nblk64;
};

SegPlan seg_plan(int64_t L, int64_t D, int64_t b) {
    SegPlan s{};
    const int64_t nck = (L + 15) / 16;
    s.nblk64 = (D + 63) / 64;
    // rows x blocks x G ~ 2 x 148 CTAs, counting at most 8 rows: batches of 8 rows or more
    // share one plan (and give bit-identical rows however they are split), smaller ones
    // cut their rows into more segments to fill the GPU
    const int64_t rows = std::min<int64_t>(8, std::max<int64_t>(1, b));
    int64_t G = std::max<int64_t>(1, 296 / (rows * std::max<int64_t>(1, s.nblk64)));
    G = std::min<int64_t>(G, std::max<int64_t>(1, nck / 8));
    const int64_t per = std::max<int64_t>(1, (nck + G - 1) / G);   // checkpoint chunks per segment
    s.nseg = std::max<int64_t>(1, (nck + per - 1) / per);
    s.seg_len = 16 * per;
    s.sub_len = s.seg_len % 128 == 0 ? 128 : s.seg_len % 64 == 0 ? 64 : s.seg_len % 32 == 0 ? 32 : 16;
    // very long sequences: fewer, longer summaries (at most 128 steps each, staged whole)
    while ((L + s.sub_len - 1) / s.sub_len > 8192 && s.sub_len < 128 && s.seg_len % (2 * s.sub_len) == 0)
        s.sub_len *= 2;
    s.nsub = (L + s.sub_len - 1) / s.sub_len;
    s.first_sub = s.seg_len / s.sub_len;
    return s;
}

struct WsLayout {
    int64_t bc, a, d, bias, q, s, total;
};

// es: bytes of one partial sum (4 for fp32 / bf16 inputs, 8 for float64 inputs).
// fp32 / bf16 inputs: one layout serves both backward kernels -- dB|dC partials per
// channel block (32-channel blocks of the row kernel, which need the most), dA / dD /
// d(delta_bias) partials per (segment, row) (per row for the row kernel), and the
// segmented kernel's sub-segment summaries.  float64 inputs: partials per 32-channel
// block and per row.
WsLayout ws_layout(int64_t b, int64_t L, int64_t D, int64_t es = 4) {
    WsLayout w{};
    const int64_t nblk32 = (D + 31) / 32;
    if (es == 8) {
        w.bc = 0;
        w.a = w.bc + round_up(nblk32 * b * L * 2 * swx::NS * es);
        w.d = w.a + round_up(b * D * swx::NS * es);
        w.bias = w.d + round_up(b * D * es);
        w.q = w.s = w.bias + round_up(b * D * es);
        w.total = w.q;
        return w;
    }
    const SegPlan sp = seg_plan(L, D, b);
    w.bc = 0;
    w.a = w.bc + round_up(nblk32 * b * L * 2 * swx::NS * 4);
    w.d = w.a + round_up(sp.nseg * b * D * swx::NS * 4);
    w.bias = w.d + round_up(sp.nseg * b * D * 4);
    w.q = w.bias + round_up(sp.nseg * b * D * 4);
    w.s = w.q + round_up(sp.nsub * b * D * swx::NS * 4);
    w.total = w.s + round_up(sp.nsub * b * D * 4);
    return w;
}

// b * L * D elements at most (2^40, far beyond any device's memory): every size product
// the launchers and workspace layouts form stays well inside int64.
constexpr int64_t kMaxElems = int64_t(1) << 40;

bool sizes_ok(int64_t b, int64_t L, int64_t D) {
    if (b < 0 || L < 0 || D < 0) return false;
    if (L != 0 && b > kMaxElems / L) return false;
    const int64_t bl = b * L;
    return D == 0 || bl <= kMaxElems / D;
}

int check_common(const swx_scan_args* a) {
    if (!a) return SWX_ERR_INVALID_ARG;
    if (!sizes_ok(a->batch, a->seqlen, a->dim)) return SWX_ERR_INVALID_ARG;
    if (a->dstate < 1 || a->dstate > swx::NS) return SWX_ERR_UNSUPPORTED;
    // batch rows index the grid's y dimension (at most 65535)
    if (a->batch > 65535 || a->seqlen > INT32_MAX || a->dim > INT32_MAX) return SWX_ERR_UNSUPPORTED;
    if (elem_size(a->in_dtype) == 0) return SWX_ERR_UNSUPPORTED;
    if (a->flags & ~(SWX_SCAN_A_LOG | SWX_SCAN_SPLIT_FWD)) return SWX_ERR_INVALID_ARG;
    if (a->group_w || a->d_group_w) {
        // the pathway mix: with the gate, fp32 / bf16 only, a bounded number of groups
        if (a->in_dtype == SWX_DTYPE_F64 || !a->z) return SWX_ERR_UNSUPPORTED;
        if (a->ngroups < 1 || a->ngroups > SWX_MAX_GROUPS) return SWX_ERR_UNSUPPORTED;
        if (!a->group_w || !a->group_of) return SWX_ERR_INVALID_ARG;
        if (a->group_w_sb < 0 || a->group_w_sl < 0) return SWX_ERR_INVALID_ARG;
    }
    if (a->batch * a->seqlen * a->dim == 0) return SWX_OK;
    if (!a->u || !a->delta || !a->B || !a->C || !a->A) return SWX_ERR_INVALID_ARG;
    return SWX_OK;
}

swx::ScanDev pack(const swx_scan_args* a) {
    swx::ScanDev p{};
    const int es = elem_size(a->in_dtype);
    p.b = (int)a->batch; p.L = (int)a->seqlen; p.D = (int)a->dim; p.N = (int)a->dstate;
    p.nck = (int)((a->seqlen + swx::TCK - 1) / swx::TCK);
    p.softplus = a->delta_softplus ? 1 : 0;
    p.a_log = (a->flags & SWX_SCAN_A_LOG) ? 1 : 0;
    p.u = a->u; p.u_sb = a->u_sb; p.u_sl = a->u_sl;
    p.dl = a->delta; p.dl_sb = a->delta_sb; p.dl_sl = a->delta_sl;
    p.z = a->z; p.z_sb = a->z_sb; p.z_sl = a->z_sl;
    p.B = a->B; p.B_sb = a->B_sb; p.B_sl = a->B_sl;
    p.C = a->C; p.C_sb = a->C_sb; p.C_sl = a->C_sl;
    p.A = a->A; p.Dskip = a->Dskip; p.dbias = a->delta_bias; p.h0 = a->h0;
    p.vec_u = vec_ok(a->u, a->u_sb, a->u_sl, es);
    p.vec_dl = vec_ok(a->delta, a->delta_sb, a->delta_sl, es);
    p.vec_z = vec_ok(a->z, a->z_sb, a->z_sl, es);
    p.vec_B = vec_ok(a->B, a->B_sb, a->B_sl, es);
    p.vec_C = vec_ok(a->C, a->C_sb, a->C_sl, es);
    p.vec_dout = vec_ok(a->dout, a->dout_sb, a->dout_sl, es);
    p.out = a->out; p.h_last = a->h_last; p.ck = a->checkpoints; p.dsum = a->delta_sum;
    p.ypre = a->z ? a->out_pre : nullptr;
    p.vec_yp = vec_ok(a->out_pre, a->seqlen * a->dim, a->dim, 4);
    p.dout = a->dout; p.dout_sb = a->dout_sb; p.dout_sl = a->dout_sl;
    p.du = a->du; p.ddl = a->ddelta; p.dz = a->dz; p.dB = a->dB; p.dC = a->dC;
    p.dz_sl = a->dz_sl ? a->dz_sl : a->dim;
    p.dz_sb = a->dz_sb ? a->dz_sb : a->seqlen * p.dz_sl;
    p.dA = a->dA; p.dD = a->dD; p.ddbias = a->ddelta_bias; p.dh0 = a->dh0;
    p.nblk = (int)((a->dim + 31) / 32);
    if (a->group_w) {
        p.gw = a->group_w; p.gw_sb = a->group_w_sb; p.gw_sl = a->group_w_sl;
        p.gof = a->group_of; p.ngroups = a->ngroups; p.dgw = a->d_group_w;
    }
    return p;
}

int from_cuda(cudaError_t e) { return e == cudaSuccess ? SWX_OK : SWX_ERR_CUDA; }

// An empty sequence (L = 0) still has per-row and per-channel results: the final state is
// the initial one (or zero), the sum of delta_eff is zero, and the gradients of the
// parameters and of h0 are zero (nothing depends on them).  Written with async copies /
// fills on the stream; nothing else is touched.
int empty_scan_fwd(const swx_scan_args* a, cudaStream_t st) {
    const int64_t es = a->in_dtype == SWX_DTYPE_F64 ? 8 : 4;
    const int64_t bdn = a->batch * a->dim * a->dstate, bd = a->batch * a->dim;
    cudaError_t e = cudaSuccess;
    if (a->h_last && bdn > 0)
        e = a->h0 ? cudaMemcpyAsync(a->h_last, a->h0, bdn * es, cudaMemcpyDeviceToDevice, st)
                  : cudaMemsetAsync(a->h_last, 0, bdn * es, st);
    if (e == cudaSuccess && a->delta_sum && bd > 0) e = cudaMemsetAsync(a->delta_sum, 0, bd * es, st);
    return from_cuda(e);
}

int empty_scan_bwd(const swx_scan_args* a, cudaStream_t st) {
    const int64_t es = a->in_dtype == SWX_DTYPE_F64 ? 8 : 4;
    const int64_t D = a->dim, N = a->dstate;
    cudaError_t e = cudaSuccess;
    if (a->dA && D * N > 0) e = cudaMemsetAsync(a->dA, 0, D * N * es, st);
    if (e == cudaSuccess && a->dD && D > 0) e = cudaMemsetAsync(a->dD, 0, D * es, st);
    if (e == cudaSuccess && a->ddelta_bias && D > 0) e = cudaMemsetAsync(a->ddelta_bias, 0, D * es, st);
    if (e == cudaSuccess && a->dh0 && a->batch * D * N > 0) e = cudaMemsetAsync(a->dh0, 0, a->batch * D * N * es, st);
    return from_cuda(e);
}

// ---- split forward (SWX_SCAN_SPLIT_FWD): each row's sequence cut into G segments that
// the forward scans as G independent rows of a (b * G, L / G, D) view of the same
// buffers (the checkpoint, output and pre-gate layouts of the view are the full rows'),
// then a prefix combine of the segments' end states and the correction of every later
// segment.
int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (!cached[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
        cached[dev] = n;
    }
    return cached[dev];
}

// Segments per row: the largest of 8, 4, 2 with (rows x 32-channel blocks x G) at most two
// CTAs per SM, segments of at least 2048 steps and a multiple of 16; 1 (no split) when the
// whole-row grid already holds an SM each or the rows are not laid out seqlen row
// strides apart.
int fwd_split_segments(const swx_scan_args* a) {
    if (!(a->flags & SWX_SCAN_SPLIT_FWD) || a->in_dtype == SWX_DTYPE_F64 || !a->out) return 1;
    const int64_t L = a->seqlen;
    auto rows_ok = [&](const void* ptr, int64_t sb, int64_t sl) { return !ptr || sb == L * sl; };
    if (!rows_ok(a->u, a->u_sb, a->u_sl) || !rows_ok(a->delta, a->delta_sb, a->delta_sl) ||
        !rows_ok(a->z, a->z_sb, a->z_sl) || !rows_ok(a->B, a->B_sb, a->B_sl) || !rows_ok(a->C, a->C_sb, a->C_sl) ||
        (a->group_w && a->group_w_sb != L * a->group_w_sl))
        return 1;
    const int sms = sm_count();
    const int64_t base = a->batch * ((a->dim + 31) / 32);
    if (sms <= 0 || base > sms) return 1;
    for (int G = 8; G >= 2; G /= 2)
        if (base * G <= 2LL * sms && L % (16LL * G) == 0 && L / G >= 2048 && a->batch * G <= 65535) return G;
    return 1;
}

struct FwdWs {
    int64_t h_end, dsum, h_in, corr, total;
};

FwdWs fwd_ws_layout(const swx_scan_args* a, int G) {
    FwdWs w{};
    const int64_t bg = a->batch * G, D = a->dim, N = a->dstate;
    w.h_end = 0;
    w.dsum = round_up(bg * D * N * 4);
    w.h_in = w.dsum + round_up(bg * D * 4);
    w.corr = w.h_in + round_up(bg * D * N * 4);
    w.total = w.corr + round_up(swx::scan_correct_workspace_floats(bg, a->seqlen / G, D) * 4);
    return w;
}

cudaError_t split_forward(const swx_scan_args* a, int G, const FwdWs& w, cudaStream_t st) {
    char* ws = static_cast<char*>(a->workspace);
    float* h_end = reinterpret_cast<float*>(ws + w.h_end);
    float* dsum = reinterpret_cast<float*>(ws + w.dsum);
    float* h_in = reinterpret_cast<float*>(ws + w.h_in);
    float* corr = reinterpret_cast<float*>(ws + w.corr);
    const int64_t Ls = a->seqlen / G;
    // the (b * G, Ls, D) view: segment s of row r is view row r * G + s
    swx_scan_args v = *a;
    v.batch = a->batch * G;
    v.seqlen = Ls;
    v.u_sb = Ls * a->u_sl; v.delta_sb = Ls * a->delta_sl; v.z_sb = Ls * a->z_sl;
    v.B_sb = Ls * a->B_sl; v.C_sb = Ls * a->C_sl; v.group_w_sb = Ls * a->group_w_sl;
    v.h0 = nullptr;                      // every segment from a zero state
    v.h_last = h_end;
    v.delta_sum = dsum;
    const bool has_z = a->z != nullptr;
    cudaError_t e = swx::launch_scan_fwd(pack(&v), a->in_dtype, a->out_dtype, has_z, st);
    if (e != cudaSuccess) return e;
    // each segment's true initial state; the rows' final states and delta sums
    e = swx::launch_seg_combine(pack(a), G, h_end, dsum, h_in, a->h_last, a->delta_sum, st);
    if (e != cudaSuccess) return e;
    // out, checkpoints and the pre-gate output of every segment gain its initial state's term
    swx_scan_args c = v;
    c.h0 = h_in;
    c.h_last = nullptr;
    c.delta_sum = nullptr;
    swx::ScanDev pc = pack(&c);
    pc.seg_g = G;
    pc.skip_first_seg = a->h0 ? 0 : 1;
    return swx::launch_scan_correct(pc, a->in_dtype, a->out_dtype, has_z, corr, st, true);
}

}  // namespace

namespace swx {
// Argument checks shared by every scan entry point (see check_common).
int scan_check_args(const swx_scan_args* a) { return check_common(a); }
}  // namespace swx

extern "C" {

int swx_abi_version(void) { return SWX_ABI_VERSION; }

int64_t swx_scan_args_size(void) { return (int64_t)sizeof(swx_scan_args); }
int64_t swx_conv_args_size(void) { return (int64_t)sizeof(swx_conv_args); }
int64_t swx_decode_args_size(void) { return (int64_t)sizeof(swx_decode_args); }

const char* swx_status_string(int status) {
    switch (status) {
        case SWX_OK: return "ok";
        case SWX_ERR_INVALID_ARG: return "invalid argument (shape, stride, size or missing pointer)";
        case SWX_ERR_UNSUPPORTED: return "unsupported dtype or layout";
        case SWX_ERR_CUDA: return "CUDA launch or runtime error";
        case SWX_ERR_TIMEOUT: return "a bounded device-side wait timed out";
        default: return "unknown status";
    }
}

int64_t swx_scan_checkpoint_floats(int64_t batch, int64_t seqlen, int64_t dim) {
    if (!sizes_ok(batch, seqlen, dim)) return -1;
    return batch * ((seqlen + swx::TCK - 1) / swx::TCK) * dim * swx::NS;
}

int64_t swx_scan_bwd_workspace_bytes(int64_t batch, int64_t seqlen, int64_t dim) {
    if (!sizes_ok(batch, seqlen, dim)) return -1;
    return ws_layout(batch, seqlen, dim).total;
}

int64_t swx_scan_bwd_workspace_bytes_f64(int64_t batch, int64_t seqlen, int64_t dim) {
    if (!sizes_ok(batch, seqlen, dim)) return -1;
    return ws_layout(batch, seqlen, dim, 8).total;
}

int swx_scan_fwd(const swx_scan_args* a, void* stream) {
    int s = check_common(a);
    if (s != SWX_OK) return s;
    if (a->batch * a->seqlen * a->dim == 0) return empty_scan_fwd(a, static_cast<cudaStream_t>(stream));
    if (elem_size(a->out_dtype) == 0) return SWX_ERR_UNSUPPORTED;
    if (!a->out && !a->h_last && !a->delta_sum && !a->checkpoints) return SWX_OK;   // nothing requested
    if (a->checkpoints && !aligned16(a->checkpoints)) return SWX_ERR_INVALID_ARG;
    swx::ScanDev p = pack(a);
    if (a->in_dtype == SWX_DTYPE_F64) {
        if (a->out_dtype != SWX_DTYPE_F64) return SWX_ERR_UNSUPPORTED;
        return from_cuda(swx::launch_scan_fwd_f64(p, static_cast<cudaStream_t>(stream)));
    }
    if (a->out_dtype == SWX_DTYPE_F64) return SWX_ERR_UNSUPPORTED;
    const int G = fwd_split_segments(a);
    if (G > 1) {
        const FwdWs w = fwd_ws_layout(a, G);
        if (!a->workspace || !aligned16(a->workspace) || a->workspace_bytes < w.total) return SWX_ERR_INVALID_ARG;
        return from_cuda(split_forward(a, G, w, static_cast<cudaStream_t>(stream)));
    }
    return from_cuda(swx::launch_scan_fwd(p, a->in_dtype, a->out_dtype, a->z != nullptr,
                                          static_cast<cudaStream_t>(stream)));
}

int64_t swx_scan_fwd_workspace_bytes(const swx_scan_args* a) {
    if (check_common(a) != SWX_OK) return -1;
    const int G = fwd_split_segments(a);
    return G > 1 ? fwd_ws_layout(a, G).total : 0;
}

int swx_scan_bwd(const swx_scan_args* a, void* stream) {
    int s = check_common(a);
    if (s != SWX_OK) return s;
    if (a->batch * a->seqlen * a->dim == 0) return empty_scan_bwd(a, static_cast<cudaStream_t>(stream));
    if (!a->dout || !a->du || !a->ddelta || !a->dB || !a->dC || !a->dA || !a->checkpoints)
        return SWX_ERR_INVALID_ARG;
    if (a->z && !a->dz) return SWX_ERR_INVALID_ARG;
    if ((a->dz_sb != 0) != (a->dz_sl != 0)) return SWX_ERR_INVALID_ARG;
    if (a->dz_sl) {                                  // strided dz (e.g. the z half of d(xz))
        if (a->in_dtype == SWX_DTYPE_F64) return SWX_ERR_UNSUPPORTED;
        if (a->dz_sl < a->dim || a->dz_sb < a->seqlen * a->dz_sl) return SWX_ERR_INVALID_ARG;
    }
    if (a->d_group_w && !a->out_pre) return SWX_ERR_INVALID_ARG;     // the weights' gradient reads y
    if (!aligned16(a->checkpoints) || !a->workspace || !aligned16(a->workspace)) return SWX_ERR_INVALID_ARG;
    const bool f64 = a->in_dtype == SWX_DTYPE_F64;
    const WsLayout w = ws_layout(a->batch, a->seqlen, a->dim, f64 ? 8 : 4);
    if (a->workspace_bytes < w.total) return SWX_ERR_INVALID_ARG;
    swx::ScanDev p = pack(a);
    char* ws = static_cast<char*>(a->workspace);
    p.ws_bc = reinterpret_cast<float*>(ws + w.bc);
    p.ws_a = reinterpret_cast<float*>(ws + w.a);
    p.ws_d = reinterpret_cast<float*>(ws + w.d);
    p.ws_bias = reinterpret_cast<float*>(ws + w.bias);
    if (f64) return from_cuda(swx::launch_scan_bwd_f64(p, static_cast<cudaStream_t>(stream)));
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    bool rows = false;
    if (swx::scan_bwd_rows_applicable(p, a->in_dtype, a->z != nullptr, &rows) != cudaSuccess) return SWX_ERR_CUDA;
    cudaError_t e;
    if (rows) {
        e = swx::launch_scan_bwd_rows(p, a->z != nullptr, st);
    } else {
        const SegPlan sp = seg_plan(a->seqlen, a->dim, a->batch);
        p.seg_len = (int)sp.seg_len; p.nseg = (int)sp.nseg; p.sub_len = (int)sp.sub_len;
        p.nsub = (int)sp.nsub; p.first_sub = (int)sp.first_sub; p.nblk64 = (int)sp.nblk64;
        p.ws_q = reinterpret_cast<float*>(ws + w.q);
        p.ws_s = reinterpret_cast<float*>(ws + w.s);
        e = swx::launch_scan_bwd_seg(p, a->in_dtype, a->z != nullptr, st);
    }
    if (e == cudaSuccess && p.dgw) e = swx::launch_group_w_grad(p, a->in_dtype, st);
    return from_cuda(e);
}

int64_t swx_scan_correct_workspace_bytes(int64_t batch, int64_t seqlen, int64_t dim) {
    if (!sizes_ok(batch, seqlen, dim)) return -1;
    return round_up(swx::scan_correct_workspace_floats(batch, seqlen, dim) * 4);
}

int swx_scan_correct(const swx_scan_args* a, void* stream) {
    int s = check_common(a);
    if (s != SWX_OK) return s;
    if (a->batch * a->seqlen * a->dim == 0) return SWX_OK;
    if (a->in_dtype == SWX_DTYPE_F64 || elem_size(a->out_dtype) == 0 || a->out_dtype == SWX_DTYPE_F64)
        return SWX_ERR_UNSUPPORTED;
    if (!a->out || !a->h0 || !a->workspace) return SWX_ERR_INVALID_ARG;
    if ((a->seqlen + 255) / 256 > 65535) return SWX_ERR_UNSUPPORTED;
    if (a->workspace_bytes < swx_scan_correct_workspace_bytes(a->batch, a->seqlen, a->dim)) return SWX_ERR_INVALID_ARG;
    swx::ScanDev p = pack(a);
    return from_cuda(swx::launch_scan_correct(p, a->in_dtype, a->out_dtype, a->z != nullptr,
                                              static_cast<float*>(a->workspace), static_cast<cudaStream_t>(stream),
                                              false));
}

int swx_scan_bwd_ctas_per_sm(const swx_scan_args* a) {
    int s = check_common(a);
    if (s != SWX_OK) return -s;
    if (a->in_dtype == SWX_DTYPE_F64) return 1;
    const swx::ScanDev p = pack(a);
    bool rows = false;
    if (swx::scan_bwd_rows_applicable(p, a->in_dtype, a->z != nullptr, &rows) != cudaSuccess) return -SWX_ERR_CUDA;
    if (rows) return 2;
    int ctas = 1;
    if (swx::scan_bwd_seg_ctas_per_sm(p, a->in_dtype, a->z != nullptr, &ctas) != cudaSuccess) return -SWX_ERR_CUDA;
    return ctas;
}

int swx_scan_bwd_segments(const swx_scan_args* a) {
    int s = check_common(a);
    if (s != SWX_OK) return -s;
    if (a->in_dtype == SWX_DTYPE_F64) return 0;
    const swx::ScanDev p = pack(a);
    bool rows = false;
    if (swx::scan_bwd_rows_applicable(p, a->in_dtype, a->z != nullptr, &rows) != cudaSuccess) return -SWX_ERR_CUDA;
    return rows ? 0 : (int)seg_plan(a->seqlen, a->dim, a->batch).nseg;
}

}  // extern "C"
