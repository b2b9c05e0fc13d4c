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
#include <mutex>

#include "common.cuh"

namespace {

// The scratch array.  Every GPU on which the library's device code is loaded holds one
// copy of SWX_STATIC_SCRATCH_BYTES until the process exits.
static __device__ __align__(256) unsigned char g_static_scratch[SWX_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 128;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_static_scratch on the current device.  In host code the array's
// name is only a host-side stand-in, so the address is looked up with
// cudaGetSymbolAddress once per device (with that device current) and cached.
int scratch_address(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return SWX_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p) return SWX_ERR_CUDA;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return SWX_OK;
}

}  // namespace

extern "C" int swx_scan_bwd_static_scratch(const swx_scan_args* a, void* stream) {
    if (!a) return SWX_ERR_INVALID_ARG;
    if (a->batch < 0 || a->seqlen < 0 || a->dim < 0) return SWX_ERR_INVALID_ARG;
    const int64_t need = swx_scan_bwd_workspace_bytes(a->batch, a->seqlen, a->dim);
    if (need > (int64_t)SWX_STATIC_SCRATCH_BYTES) return SWX_ERR_INVALID_ARG;   // too large
    void* scratch = nullptr;
    const int s = scratch_address(&scratch);
    if (s != SWX_OK) return s;
    swx_scan_args b = *a;
    b.workspace = scratch;
    b.workspace_bytes = (int64_t)SWX_STATIC_SCRATCH_BYTES;
    return swx_scan_bwd(&b, stream);
}
