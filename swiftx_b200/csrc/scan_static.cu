// Selective-scan backward for callers that cannot allocate device memory.
//
// swx_scan_bwd needs a scratch workspace for its deterministic cross-CTA reductions and
// expects the caller to allocate it.  Some callers cannot: a serving process that
// reserves all of its device memory at start-up and forbids any later cudaMalloc (to
// keep its footprint fixed and avoid fragmentation), or a host binding (cgo, JNI, a
// plugin ABI) that receives ready-made tensors from a framework and has no allocator of
// its own to obtain an extra buffer from.  swx_scan_bwd_static_scratch serves them: its
// scratch is a fixed-size array in the library's own device memory, so the call
// allocates nothing.
#include "common.cuh"

namespace swx {
int scan_check_args(const swx_scan_args* a);
int device_symbol_address(const void* sym, void** out);
}  // namespace swx

namespace {

// The scratch array.  Every GPU on which the library's device code is loaded holds one
// copy of SWX_STATIC_SCRATCH_BYTES until the process exits.
static __device__ __align__(256) unsigned char g_static_scratch[SWX_STATIC_SCRATCH_BYTES];

}  // namespace

extern "C" int swx_scan_bwd_static_scratch(const swx_scan_args* a, void* stream) {
    // the same argument checks as swx_scan_bwd, before any size arithmetic
    const int chk = swx::scan_check_args(a);
    if (chk != SWX_OK) return chk;
    const int64_t need = a->in_dtype == SWX_DTYPE_F64
                             ? swx_scan_bwd_workspace_bytes_f64(a->batch, a->seqlen, a->dim)
                             : swx_scan_bwd_workspace_bytes(a->batch, a->seqlen, a->dim);
    if (need < 0 || need > (int64_t)SWX_STATIC_SCRATCH_BYTES) return SWX_ERR_INVALID_ARG;   // too large
    void* scratch = nullptr;
    const int s = swx::device_symbol_address(&g_static_scratch, &scratch);
    if (s != SWX_OK) return s;
    swx_scan_args b = *a;
    b.workspace = scratch;
    b.workspace_bytes = (int64_t)SWX_STATIC_SCRATCH_BYTES;
    return swx_scan_bwd(&b, stream);
}
