/*
 * swiftx_b200 -- C ABI of the B200 selective-scan hot path.
 *
 * Plain C: device pointers, element strides and sizes; no framework types.
 * Every entry point returns an int status (SWX_OK on success) and launches its
 * kernels on the given cudaStream_t (passed as void*; NULL = legacy default
 * stream).  Nothing here allocates device memory: outputs, checkpoints and
 * workspaces are provided by the caller (the Python host layer allocates them
 * with torch on the current stream).  Apart from swx_scan_bwd_static_scratch
 * (below), the library holds no global state and takes no locks; concurrent
 * calls on different streams are independent.
 *
 * Shapes follow the reference API (models/selective_scan.py:36-43):
 *   u, delta, z, out, dout, du, ddelta, dz : (b, L, D)   innermost stride 1
 *   B, C, dB, dC                           : (b, L, N)   innermost stride 1
 *   A, dA : (D, N) dense;  Dskip, delta_bias, dD, ddelta_bias : (D,)
 *   h0, h_last, dh0 : (b, D, N) dense fp32
 * Strides are in elements.  N <= 16, b <= 65535.
 */
#ifndef SWIFTX_B200_H
#define SWIFTX_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SWX_ABI_VERSION 13

/* status codes */
#define SWX_OK 0
#define SWX_ERR_INVALID_ARG 1   /* bad shape, size, stride or missing pointer */
#define SWX_ERR_UNSUPPORTED 2   /* dtype / layout the library does not handle */
#define SWX_ERR_CUDA 3          /* a CUDA launch or runtime call failed */
#define SWX_ERR_TIMEOUT 4       /* a bounded device-side wait gave up */

/* element types */
#define SWX_DTYPE_F32 0
#define SWX_DTYPE_BF16 1
#define SWX_DTYPE_F64 2   /* float64: the scan (in_dtype = out_dtype = F64) and the linear scan */

/* swx_scan_args.flags: A holds log(-A) -- the model's A_log parameter, A = -exp(A_log)
   (models/sift_block.py:121 forms A that way before every scan call).  The kernels form A
   themselves and the backward's dA receives the gradient with respect to A_log. */
#define SWX_SCAN_A_LOG 1
/* swx_scan_args.flags, forward only: the forward may cut each row's sequence into
   segments scanned in parallel when the batch is too small to fill the GPU (the chunk
   scans from a zero state, a prefix combine of their end states, then the initial-state
   correction of every later segment's output, checkpoints and pre-gate output).  It then
   uses args->workspace, which must hold swx_scan_fwd_workspace_bytes(args) bytes. */
#define SWX_SCAN_SPLIT_FWD 2

/* Arguments of the scan entry points (forward and backward share one struct). */
typedef struct swx_scan_args {
    int64_t batch, seqlen, dim, dstate;
    int32_t in_dtype;        /* u, delta, z, B, C, dout and the (b,L,*) gradients */
    int32_t out_dtype;       /* out; SWX_DTYPE_F64 exactly when in_dtype is.  With float64
                                inputs every floating-point pointer below (A, Dskip,
                                delta_bias, h0, h_last, checkpoints, delta_sum, out_pre,
                                dA, dD, ddelta_bias, dh0) holds float64 values, and the
                                checkpoint buffer holds swx_scan_checkpoint_floats()
                                float64 values; float64 is the correctness path of the
                                reference's float64 gradchecks, not a fast path */
    int32_t delta_softplus;  /* delta_eff = softplus(delta + delta_bias) when nonzero */
    int32_t flags;           /* SWX_SCAN_* bits below; other bits must be zero */
    /* inputs */
    const void* u;     int64_t u_sb, u_sl;
    const void* delta; int64_t delta_sb, delta_sl;
    const void* z;     int64_t z_sb, z_sl;      /* optional SiLU gate */
    const void* B;     int64_t B_sb, B_sl;
    const void* C;     int64_t C_sb, C_sl;
    const float* A;            /* (D, N); log(-A) with SWX_SCAN_A_LOG */
    const float* Dskip;        /* optional */
    const float* delta_bias;   /* optional */
    const float* h0;           /* optional initial state */
    /* forward outputs */
    void* out;                 /* (b, L, D) dense; NULL = compute only h_last / delta_sum /
                                  checkpoints (skips C, z, the readout and the stores) */
    float* h_last;             /* optional final state */
    float* checkpoints;        /* optional in forward (required for backward):
                                  swx_scan_checkpoint_floats() fp32 values */
    /* backward inputs / outputs */
    const void* dout;  int64_t dout_sb, dout_sl;
    void* du; void* ddelta; void* dz;   /* (b, L, D) dense, in_dtype; dz only with z */
    void* dB; void* dC;                 /* (b, L, N) dense, in_dtype */
    float* dA;                          /* (D, N); d/dA_log with SWX_SCAN_A_LOG */
    float* dD;                          /* optional (with Dskip) */
    float* ddelta_bias;                 /* optional (with delta_bias) */
    float* dh0;                         /* optional (with h0) */
    void* workspace; int64_t workspace_bytes;  /* >= swx_scan_bwd_workspace_bytes() */
    /* forward, optional: (b, D) fp32 sum over t of delta_eff, i.e. log of the chunk's
       decay per state is A * delta_sum (used to chain sequence-parallel chunks) */
    float* delta_sum;
    /* optional, with z: (b, L, D) dense fp32 pre-gate output y.  The forward writes it
       when non-NULL; the backward then reads it for the gate gradient instead of
       recomputing the readout (Mamba's save-vs-recompute trade for the gate). */
    float* out_pre;
    /* optional, with z: the SiftX pathway mix (models/sift_block.py:137-142) fused into the
       gate.  group_w: (b, L, ngroups) fp32 per-token group weights (group stride 1; the
       block's softmax(pathway(x)) * ngroups); group_of: (D,) int32 group of each channel,
       in [0, ngroups) (device memory, not checked: the caller guarantees the range);
       1 <= ngroups <= SWX_MAX_GROUPS.  The forward writes
       out_t = y_t * group_w[t, group_of[d]] * silu(z_t) (out_pre stays y_t).  The
       backward reads dout through the same factor and, when d_group_w is non-NULL
       (requires out_pre), writes d_group_w[b, t, g] = sum over the channels of group g of
       dout * silu(z) * y: (b, L, ngroups) dense fp32, fixed summation order.  Not for
       float64 inputs. */
    const float* group_w; int64_t group_w_sb, group_w_sl;
    const int32_t* group_of;
    int32_t ngroups;
    float* d_group_w;
    /* optional element strides (batch, row) of dz; 0, 0 = dense (L*D, D).  Lets the
       backward write the gate gradient straight into the z half of the in_proj output's
       gradient (row stride 2D).  dz_sl >= dim, dz_sb >= seqlen * dz_sl; fp32 / bf16 only. */
    int64_t dz_sb, dz_sl;
} swx_scan_args;

#define SWX_MAX_GROUPS 8

int swx_abi_version(void);
const char* swx_status_string(int status);
/* sizeof(swx_scan_args), so a binding can check its mirror of the struct. */
int64_t swx_scan_args_size(void);
/* sizeof(swx_conv_args) and sizeof(swx_decode_args), for the same check. */
int64_t swx_conv_args_size(void);
int64_t swx_decode_args_size(void);

/* Number of fp32 values of the forward's state checkpoints (one (D, 16) slab per
 * 16 time steps per batch row); -1 for a negative size or batch*seqlen*dim > 2^40. */
int64_t swx_scan_checkpoint_floats(int64_t batch, int64_t seqlen, int64_t dim);
/* Bytes of scratch the backward needs for its deterministic cross-CTA reductions; -1 for
 * a negative size or batch*seqlen*dim > 2^40 (the scan entry points reject those too). */
int64_t swx_scan_bwd_workspace_bytes(int64_t batch, int64_t seqlen, int64_t dim);
/* The same for float64 inputs (in_dtype SWX_DTYPE_F64), whose partial sums are float64. */
int64_t swx_scan_bwd_workspace_bytes_f64(int64_t batch, int64_t seqlen, int64_t dim);

/* Forward selective scan:
 *   delta_eff = softplus(delta + delta_bias) | delta + delta_bias | delta
 *   h_t = exp(delta_eff_t * A) * h_{t-1} + delta_eff_t * u_t * B_t     (h_{-1} = h0 or 0)
 *   y_t = <C_t, h_t> + Dskip * u_t ;  out_t = y_t * silu(z_t)  (or y_t without z)
 * Replaces selective_scan_fast / selective_scan_ref forward
 * (models/selective_scan.py:34-60, :112-125, :246-265) and TritonScanFn.forward
 * (models/triton_scan.py:118-135); the gate and softplus fold in the block glue of
 * models/sift_block.py:108,134.  An empty problem (batch * seqlen * dim = 0) launches no
 * kernel; with seqlen = 0 the forward sets h_last to h0 (or zeros) and delta_sum to zeros,
 * and the backward sets dA, dD, ddelta_bias and dh0 to zeros (async on the stream). */
int swx_scan_fwd(const swx_scan_args* args, void* stream);
/* Workspace bytes the forward uses with SWX_SCAN_SPLIT_FWD for these arguments on the
 * current device: 0 when it would not split (float64, no output, rows whose batch stride
 * is not seqlen row strides, a grid that already fills the GPU, or sequences shorter than
 * 4096 steps or not a multiple of 16 times the segment count); -1 for bad arguments. */
int64_t swx_scan_fwd_workspace_bytes(const swx_scan_args* args);

/* Backward of swx_scan_fwd; needs the checkpoints the forward wrote with the same
 * inputs.  Replaces _SelectiveScanFn.backward / _FusedScanFn.backward
 * (models/selective_scan.py:127-167, :209-243) and TritonScanFn.backward
 * (models/triton_scan.py:137-155).  Reductions (dA, dB, dC, dD, ddelta_bias) are
 * deterministic: fixed-order sums, no float atomics. */
int swx_scan_bwd(const swx_scan_args* args, void* stream);

/* Initial-state correction of a chunk scanned from a zero state, for a sequence split
 * across ranks or streams: the scan is linear in its initial state, so
 *   out_t += silu(z_t) * sum_n C_t[n] * exp(A[d, n] * S_t) * h_in[n],  S_t = sum_{s<=t} delta_eff_s
 * (without z the factor silu(z_t) is 1) turns the output of swx_scan_fwd with h0 = NULL
 * into the output it would have had with h0 = h_in.  Arguments as swx_scan_fwd: delta,
 * delta_bias, delta_softplus, z, C, A (SWX_SCAN_A_LOG allowed) and dims; args->h0 is
 * h_in (b, D, N) fp32 (required); args->out (b, L, D) dense in out_dtype is updated in
 * place; u, B, Dskip are not read (u and B must still be given, as for swx_scan_fwd).
 * workspace: >= swx_scan_correct_workspace_bytes().  No reference counterpart: the
 * reference has no sequence parallelism; this is the correction pass of the sequence-
 * parallel design (each rank scans its chunk from zero, then corrects). */
int swx_scan_correct(const swx_scan_args* args, void* stream);
int64_t swx_scan_correct_workspace_bytes(int64_t batch, int64_t seqlen, int64_t dim);

/* swx_scan_bwd runs one of two kernels.  The time-segmented one (the default) cuts the
 * sequence into segments walked in parallel, with the reverse carries between them from
 * sub-segment summaries; its segment plan is a function of (seqlen, dim) alone, so the
 * rows of a batch get the same bits whatever the batch.  bf16 problems whose grid of
 * 32-channel x row CTAs fills every SM at two CTAs per SM run a kernel that walks whole
 * rows instead (faster there).  Both reduce in fixed order (deterministic). */

/* How many CTAs of its main kernel swx_scan_bwd keeps on one SM of the current device for
 * these arguments (2 on a B200); a negative status on error.  Launches nothing. */
int swx_scan_bwd_ctas_per_sm(const swx_scan_args* args);

/* Number of time segments swx_scan_bwd walks in parallel for these arguments on the
 * current device; 0 when it runs the whole-row kernel (and for float64 inputs); a
 * negative status on error.  Launches nothing. */
int swx_scan_bwd_segments(const swx_scan_args* args);

/* Capacity of the static scratch used by swx_scan_bwd_static_scratch: 8 MiB, enough
 * for swx_scan_bwd_workspace_bytes(batch, seqlen, dim) of roughly batch*seqlen*dim up
 * to 2M (e.g. 2 x 1024 x 1024). */
#define SWX_STATIC_SCRATCH_BYTES (8u << 20)

/* swx_scan_bwd for callers that cannot allocate device memory (a process that has
 * reserved all of its device memory up front and forbids later cudaMalloc, or a
 * binding that receives ready-made buffers and has no allocator of its own).  It has
 * no counterpart in the reference.  The caller still passes every input and output
 * (including the forward's checkpoints); args->workspace is ignored and the scratch
 * comes from a fixed array in the library's device memory, which every GPU that loads
 * the library holds until the process exits.  Returns SWX_ERR_INVALID_ARG (without
 * launching) when swx_scan_bwd_workspace_bytes() exceeds SWX_STATIC_SCRATCH_BYTES.
 * Arguments are checked as swx_scan_bwd checks them, before any size arithmetic.
 * The first call in each (device, CUDA context) pair looks the array's address up
 * (cudaGetSymbolAddress, with that device current) and caches it under the pair; make
 * that first call before any stream capture.  After cudaDeviceReset, or under another
 * driver context, the library's module is loaded anew and the next call repeats the
 * lookup for the new context (again: outside stream capture).  All
 * calls on a device share the one array: calls that overlap on the GPU (other streams,
 * other host threads) race and must be serialised by the caller.  Every scratch byte
 * that is read is first written by the same call, so nothing needs clearing between
 * calls.  Calls no cudaMalloc / cudaFree. */
int swx_scan_bwd_static_scratch(const swx_scan_args* args, void* stream);

/* ------------------------------------------------------------------ conv1d */
/* Causal depthwise conv1d (+ SiLU).  x: (b, L, D) with element strides (x_sb, x_sl) and
 * unit channel stride (e.g. the x half of the in_proj output, row stride 2D);
 * weight (D, width) dense fp32 (= nn.Conv1d weight (D, 1, width)); bias (D,) optional;
 * out, dout-sized gradients (b, L, D) dense, same dtype as x.  width <= 6,
 * b <= 65535, L <= 65535 * 16. */
typedef struct swx_conv_args {
    int64_t batch, seqlen, dim, width;
    int32_t dtype;           /* SWX_DTYPE_F32 | SWX_DTYPE_BF16 for x, out, dout, dx */
    int32_t silu;            /* apply SiLU after the conv */
    const void* x; int64_t x_sb, x_sl;
    const float* weight;
    const float* bias;
    void* out;
    const void* dout; int64_t dout_sb, dout_sl;
    void* dx;
    float* dweight;          /* (D, width) */
    float* dbias;            /* (D,) optional */
    void* workspace; int64_t workspace_bytes;  /* >= swx_conv1d_bwd_workspace_bytes() */
    /* optional element strides (batch, row) of dx; 0, 0 = dense (L*D, D): the backward can
       write into the x half of the in_proj output's gradient (row stride 2D).
       dx_sl >= dim, dx_sb >= seqlen * dx_sl. */
    int64_t dx_sb, dx_sl;
} swx_conv_args;

/* out = silu(conv(x) + bias), the conv segment of SiftBlock.forward
 * (models/sift_block.py:62-65, 117-118: nn.Conv1d(padding=width-1) keeping the first
 * L outputs, then F.silu). */
int swx_conv1d_fwd(const swx_conv_args* args, void* stream);
/* Backward of swx_conv1d_fwd (recomputes the pre-activation); dweight / dbias are
 * fixed-order sums (deterministic). */
int swx_conv1d_bwd(const swx_conv_args* args, void* stream);
int64_t swx_conv1d_bwd_workspace_bytes(int64_t batch, int64_t seqlen, int64_t dim, int64_t width);

/* ------------------------------------------------------------------ decode step */
#define SWX_DECODE_CONV 1   /* roll the conv window, append x, xc = silu(conv + bias) */
#define SWX_DECODE_SSM 2    /* h = exp(delta*A)*h + delta*B*xc ; out = (<h,C> + D*xc)*silu(z) */
/* swx_decode_args.flags: A holds log(-A), the block's A_log parameter (SiftBlock.step forms
   A = -exp(A_log) before every token, models/sift_block.py:168); the kernel forms A itself */
#define SWX_DECODE_A_LOG 1

/* One token of recurrent generation, fp32.  Row strides are in elements; the channel
 * (and state) stride is 1.  States are updated in place. */
typedef struct swx_decode_args {
    int64_t batch, dim, dstate, width;
    int32_t delta_softplus;
    int32_t mode;                     /* SWX_DECODE_CONV, SWX_DECODE_SSM, or both */
    const float* x; int64_t x_sb;     /* (b, D): token input (CONV) or xc (SSM only) */
    const float* z; int64_t z_sb;     /* (b, D) optional gate */
    const float* delta; int64_t delta_sb;  /* (b, D) delta before softplus */
    const float* B; int64_t B_sb;     /* (b, N) */
    const float* C; int64_t C_sb;     /* (b, N) */
    const float* conv_weight;         /* (D, width) */
    const float* conv_bias;           /* (D,) optional */
    const float* A;                   /* (D, N); log(-A) with SWX_DECODE_A_LOG */
    const float* Dskip;               /* (D,) optional */
    const float* delta_bias;          /* (D,) optional */
    float* conv_state;                /* (b, D, width) in/out */
    float* ssm_state;                 /* (b, D, N) in/out */
    float* xc_out;                    /* (b, D) optional: the post-conv activation */
    float* out;                       /* (b, D) */
    int32_t flags;                    /* SWX_DECODE_A_LOG; other bits must be zero */
    int32_t reserved;
    /* optional, with z: the SiftX pathway mix before the gate (models/sift_block.py:
       137-142, 172-173), out = y * group_w[b, group_of[d]] * silu(z).  group_w (b, ngroups)
       fp32 with group stride 1; group_of (D,) int32 in [0, ngroups) (not checked: the
       caller guarantees the range); 1 <= ngroups <= SWX_MAX_GROUPS. */
    const float* group_w; int64_t group_w_sb;
    const int32_t* group_of;
    int32_t ngroups;
    int32_t reserved2;
    /* optional (SSM mode): dt_proj folded into the step (models/sift_block.py:167,106-108).
       With dt_in set, delta[b, d] = sum_r dt_weight[d, r] * dt_in[b, r] replaces the delta
       row (then delta must be NULL; delta_bias and softplus apply as before).  dt_in
       (b, dt_rank) fp32, unit element stride, row stride dt_in_sb (a multiple of 4);
       dt_weight (D, dt_rank) dense fp32; both 16-byte aligned; dt_rank a multiple of 4,
       at most SWX_DECODE_MAX_DT_RANK.  The sum runs in a fixed order. */
    const float* dt_in; int64_t dt_in_sb;
    const float* dt_weight;
    int32_t dt_rank;
    int32_t reserved3;
    /* swx_decode_layer_step only: x_proj (xproj_rows = dt_rank + 2 * dstate, D) dense fp32,
       16-byte aligned, and a scratch workspace of swx_decode_layer_workspace_bytes(). */
    const float* xproj_weight;
    int32_t xproj_rows;
    int32_t reserved4;
    void* workspace; int64_t workspace_bytes;
} swx_decode_args;

#define SWX_DECODE_MAX_DT_RANK 256

/* Replaces SiftBlock.step's conv-window roll, conv dot + bias + SiLU and in-place
 * state update / readout / gate (models/sift_block.py:153-175). */
int swx_decode_step(const swx_decode_args* args, void* stream);

/* The whole recurrent step of one block between in_proj and out_proj, with both of its
 * projections folded in (models/sift_block.py:160-175): conv window roll + conv + SiLU,
 * x_proj (xproj_weight) split into dt | B | C, delta = softplus(dt_weight @ dt +
 * delta_bias), the state update, readout, D skip and SiLU(z) gate.  Two launches: the conv
 * with each 64-channel block's partial x_proj products, then the state update, which
 * sums the partials in block order.  Arguments as swx_decode_step with mode =
 * SWX_DECODE_CONV | SWX_DECODE_SSM, delta / B / C / dt_in NULL, dt_weight and dt_rank
 * set, xproj_weight, xproj_rows = dt_rank + 2 * dstate, workspace; dstate 16, width 4,
 * dim a multiple of 64, 16-byte aligned rows (x_sb, z_sb multiples of 4); no pathway
 * mix (its weights need the conv output first).  Returns SWX_ERR_UNSUPPORTED for other
 * shapes, which the caller then runs as swx_decode_step around its own projections. */
int swx_decode_layer_step(const swx_decode_args* args, void* stream);
/* Scratch bytes of swx_decode_layer_step: the partial x_proj products and the conv
 * output; -1 for negative sizes. */
int64_t swx_decode_layer_workspace_bytes(int64_t batch, int64_t dim, int64_t xproj_rows);

/* Linear recurrence along the sequence, for every (batch row, element) chain:
 *   h_t = a_t * h_{t-1} + x_t,  h_{-1} = 0
 * a, x: (batch, seqlen, width) with unit element stride and any row / batch stride
 * (width = the product of the trailing dims); h: dense (batch, seqlen, width).
 * Replaces parallel_scan / sequential_scan (models/selective_scan.py:66-99), which
 * compute the same recurrence by a Hillis-Steele scan and by a loop. */
typedef struct swx_linear_scan_args {
    int64_t batch, seqlen, width;
    int32_t dtype;                    /* SWX_DTYPE_F32 or SWX_DTYPE_F64 */
    int32_t reserved;
    const void* a; int64_t a_sb, a_sl;
    const void* x; int64_t x_sb, x_sl;
    void* h;                          /* forward output; backward input (the forward's h) */
    const void* dh; int64_t dh_sb, dh_sl;   /* backward: gradient of h */
    void* da;                         /* backward outputs, dense (batch, seqlen, width) */
    void* dx;
} swx_linear_scan_args;

int64_t swx_linear_scan_args_size(void);
int swx_linear_scan_fwd(const swx_linear_scan_args* args, void* stream);
/* Adjoint of swx_linear_scan_fwd: g_t = dh_t + a_{t+1} g_{t+1} (g_{seqlen} = 0),
 * dx_t = g_t, da_t = g_t * h_{t-1} (h_{-1} = 0).  Reads the forward's h. */
int swx_linear_scan_bwd(const swx_linear_scan_args* args, void* stream);

/* RMSNorm of the language model around the mixer (models/sift_model.py:17-26):
 *   y = (x * rsqrt(mean(x^2) + eps)) * weight  over the last dim, computed in fp32.
 * x, dx: dense (rows, dim) in dtype; y, dy: dense (rows, dim) in out_dtype (fp32 or
 * bf16: a bf16 y is the fp32 result rounded once, as a cast after the norm would give);
 * weight, dweight: (dim,) fp32;
 * rstd: (rows,) fp32, written by the forward when given and read by the backward.
 * dim <= 1024.  The weight gradient is a fixed-order sum (deterministic).
 *
 * Residual form (the pre-norm residual stream, x_{i+1} = x_i + mixer_i(...), fused with
 * the next norm; models/sift_model.py:58):
 *   forward, residual given: s = x + residual (fp32 arithmetic, residual in res_dtype) is
 *     written to sum (dtype) and y = norm(s);
 *   backward: pass the saved s as x; dsum (rows, dim) fp32, optional, is the gradient of s
 *     from its other consumers and is added to dx; dres, optional, receives dx again in
 *     res_dtype (the gradient of the residual input).
 * With fp32 x both directions give bit-identical values to the separate add, norm,
 * gradient sum and cast (with bf16 x the gradient sum is rounded once instead of twice). */
typedef struct swx_rmsnorm_args {
    int64_t rows, dim;
    float eps;
    int32_t dtype;                    /* x, dx, sum: SWX_DTYPE_F32 or SWX_DTYPE_BF16 */
    int32_t out_dtype;                /* y, dy: SWX_DTYPE_F32 or SWX_DTYPE_BF16 */
    int32_t res_dtype;                /* residual, dres: SWX_DTYPE_F32 or SWX_DTYPE_BF16 */
    const void* x;
    const float* weight;
    void* y;
    float* rstd;
    const void* dy;                   /* backward */
    void* dx;
    float* dweight;
    void* workspace; int64_t workspace_bytes;
    const void* residual;             /* forward, residual form */
    void* sum;
    const float* dsum;                /* backward, residual form */
    void* dres;
} swx_rmsnorm_args;

int64_t swx_rmsnorm_args_size(void);
int64_t swx_rmsnorm_bwd_workspace_bytes(int64_t dim);
int swx_rmsnorm_fwd(const swx_rmsnorm_args* args, void* stream);
int swx_rmsnorm_bwd(const swx_rmsnorm_args* args, void* stream);

/* Weight gradient of the LM's token embedding (nn.Embedding, models/sift_model.py;
 * torch's embedding_dense_backward is what it replaces):
 *   dweight[v, :] = sum over tokens i with idx[i] == v of dy[i, :]
 * idx: (ntok,) int64; dy: dense (ntok, dim) fp32; dweight: dense (vocab, dim) fp32,
 * overwritten.  vocab <= 1024.  Tokens are summed in a fixed order (token slices, then
 * slices in order), so the result is deterministic for a given shape.  An id outside
 * [0, vocab) is skipped and, when status is given, sets *status = 1 (device int). */
typedef struct swx_embedding_args {
    int64_t ntok, vocab, dim;
    const int64_t* idx;
    const float* dy;
    float* dweight;
    int32_t* status;                  /* optional */
    void* workspace; int64_t workspace_bytes;
} swx_embedding_args;

int64_t swx_embedding_args_size(void);
int64_t swx_embedding_bwd_workspace_bytes(int64_t ntok, int64_t vocab, int64_t dim);
int swx_embedding_bwd(const swx_embedding_args* args, void* stream);

/* Diagnostic: y[i] = 2^x[i] computed by the FMA-pipe exponential the scan backward uses
 * for part of its decays (a degree-5 minimax polynomial after rounding x to an integer
 * part; x clamped to [-125, 127]), so its accuracy can be checked on the device.  x, y:
 * device fp32 arrays of n values.  Not part of any reference interface. */
int swx_exp2_fma_eval(const float* x, float* y, int64_t n, void* stream);

/* Status of the library's bounded device-side waits on the current device.  The scan
 * kernels (forward, both backward paths) wait for their TMA tiles with an iteration
 * limit (about a second); if a wait runs out, the kernel records SWX_ERR_TIMEOUT, leaves its outputs
 * incomplete and returns, and the context stays usable.  This call synchronises the
 * device and returns SWX_OK, or SWX_ERR_TIMEOUT once for every run of timeouts (it
 * clears the status), or SWX_ERR_CUDA. */
int swx_device_wait_status(void);

/* Diagnostic: one thread waits `polls` tries for an mbarrier phase that never
 * completes and records the timeout exactly as the backward does, so that the status
 * path above can be exercised without any real failure. */
int swx_diag_wait_timeout(uint32_t polls, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SWIFTX_B200_H */
