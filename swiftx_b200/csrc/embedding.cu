// Gradient of the LM's token embedding (nn.Embedding in models/sift_model.py), the
// scatter dW[v] = sum over tokens i with idx_i = v of dy_i, for small vocabularies.
// torch sorts the token ids and reduces segments; with a vocabulary of a few hundred
// rows the whole (vocab x 32 columns) block of partial sums fits in shared memory, so:
//   pass 1: CTA = one warp = (32-column block, slice of tokens); lane = column; the warp
//           loads EMB_BATCH tokens' rows at a time (all in flight) and adds them, in
//           token order, into its shared (vocab x 32) block, written out as the slice's
//           partial;
//   pass 2: the slices' partials are added in slice order.
// Every sum runs in a fixed order, so the result is deterministic for a given shape.
#include "common.cuh"
#include "launch_util.cuh"

#include <algorithm>

namespace swx {

constexpr int EMB_MAXV = 1024;        // vocabulary rows held in shared memory (128 KB)
constexpr int EMB_BATCH = 16;         // token rows in flight per warp
constexpr int EMB_MIN_TOK = 128;      // fewest tokens per slice

struct EmbDev {
    int64_t ntok, vocab, d;
    const int64_t* idx;
    const float* dy;
    float* part;                      // (nslice, vocab, d)
    float* dw;                        // (vocab, d)
    int64_t tok;                      // tokens per slice
    int nslice;
    int* bad;                         // optional: set when a token id is out of range
};

// Tokens per slice: enough slices for about six one-warp CTAs per SM, at least
// EMB_MIN_TOK tokens each, a multiple of EMB_BATCH.
static int64_t emb_tokens_per_slice(int64_t ntok, int64_t dim) {
    const int64_t ncb = (dim + 31) / 32;
    int64_t t = (ntok * ncb + 148 * 6 - 1) / (148 * 6);
    t = (t + EMB_BATCH - 1) / EMB_BATCH * EMB_BATCH;
    return std::max<int64_t>(t, EMB_MIN_TOK);
}

__global__ void __launch_bounds__(32) embedding_bwd_part_kernel(const EmbDev p) {
    extern __shared__ float acc[];    // [vocab][32]
    const int lane = threadIdx.x;
    const int64_t c0 = (int64_t)blockIdx.x * 32;
    const int64_t slice = blockIdx.y;
    for (int64_t v = 0; v < p.vocab; ++v) acc[v * 32 + lane] = 0.f;
    __syncwarp();
    const int64_t i0 = slice * p.tok, i1 = min(i0 + p.tok, p.ntok);
    const bool col_ok = c0 + lane < p.d;
    const float* dy = p.dy + c0 + lane;
    bool bad = false;
    for (int64_t b0 = i0; b0 < i1; b0 += EMB_BATCH) {
        const int n = (int)min((int64_t)EMB_BATCH, i1 - b0);
        const int64_t mine = lane < n ? p.idx[b0 + lane] : 0;
        float val[EMB_BATCH];
#pragma unroll
        for (int j = 0; j < EMB_BATCH; ++j) val[j] = (j < n && col_ok) ? dy[(b0 + j) * p.d] : 0.f;
#pragma unroll
        for (int j = 0; j < EMB_BATCH; ++j) {
            const int64_t v = __shfl_sync(0xffffffffu, mine, j);
            if (j < n) {
                if (v >= 0 && v < p.vocab) acc[v * 32 + lane] += val[j];
                else bad = true;
            }
        }
    }
    if (bad && lane == 0 && p.bad) *p.bad = 1;
    __syncwarp();
    if (col_ok) {
        float* out = p.part + slice * p.vocab * p.d + c0 + lane;
        for (int64_t v = 0; v < p.vocab; ++v) out[v * p.d] = acc[v * 32 + lane];
    }
}

__global__ void __launch_bounds__(256) embedding_bwd_sum_kernel(const EmbDev p) {
    const int64_t n = p.vocab * p.d;
    for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < n; q += (int64_t)gridDim.x * blockDim.x) {
        const float* src = p.part + q;
        float s = 0.f;
#pragma unroll 8
        for (int k = 0; k < p.nslice; ++k) s += src[(int64_t)k * n];
        p.dw[q] = s;
    }
}

}  // namespace swx

extern "C" {

int64_t swx_embedding_args_size(void) { return (int64_t)sizeof(swx_embedding_args); }

int64_t swx_embedding_bwd_workspace_bytes(int64_t ntok, int64_t vocab, int64_t dim) {
    if (ntok < 0 || vocab < 0 || dim < 0) return -SWX_ERR_INVALID_ARG;
    if (ntok == 0) return 0;
    const int64_t tok = swx::emb_tokens_per_slice(ntok, dim);
    return (ntok + tok - 1) / tok * vocab * dim * 4;
}

int swx_embedding_bwd(const swx_embedding_args* a, void* stream) {
    if (!a || a->ntok < 0 || a->vocab < 0 || a->dim < 0) return SWX_ERR_INVALID_ARG;
    if (a->vocab > swx::EMB_MAXV) return SWX_ERR_UNSUPPORTED;
    if (a->vocab * a->dim == 0) return SWX_OK;
    if (!a->dweight || (a->ntok > 0 && (!a->idx || !a->dy || !a->workspace))) return SWX_ERR_INVALID_ARG;
    if (a->workspace_bytes < swx_embedding_bwd_workspace_bytes(a->ntok, a->vocab, a->dim))
        return SWX_ERR_INVALID_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (a->ntok == 0) {
        cudaMemsetAsync(a->dweight, 0, (size_t)(a->vocab * a->dim) * 4, st);
        return cudaGetLastError() == cudaSuccess ? SWX_OK : SWX_ERR_CUDA;
    }
    swx::EmbDev p{};
    p.ntok = a->ntok; p.vocab = a->vocab; p.d = a->dim;
    p.idx = a->idx; p.dy = a->dy; p.dw = a->dweight; p.bad = a->status;
    p.tok = swx::emb_tokens_per_slice(a->ntok, a->dim);
    const int64_t nslice = (a->ntok + p.tok - 1) / p.tok;
    if (nslice > 65535) return SWX_ERR_UNSUPPORTED;
    p.nslice = (int)nslice;
    p.part = static_cast<float*>(a->workspace);
    const int smem = (int)(a->vocab * 32 * 4);
    if (swx::allow_smem(swx::embedding_bwd_part_kernel, swx::EMB_MAXV * 32 * 4) != cudaSuccess) return SWX_ERR_CUDA;
    const dim3 grid((unsigned)((a->dim + 31) / 32), (unsigned)nslice);
    swx::embedding_bwd_part_kernel<<<grid, 32, smem, st>>>(p);
    const int64_t n = a->vocab * a->dim;
    swx::embedding_bwd_sum_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 148 * 8), 256, 0, st>>>(p);
    return cudaGetLastError() == cudaSuccess ? SWX_OK : SWX_ERR_CUDA;
}

}  // extern "C"
