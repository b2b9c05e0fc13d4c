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
#include <cuda.h>

#include <mutex>
#include <vector>

#include "common.cuh"

namespace swx {
int scan_check_args(const swx_scan_args* a);
}  // namespace swx

namespace {

// The scratch array.  Every GPU on which the library's device code is loaded holds one
// copy of SWX_STATIC_SCRATCH_BYTES until the process exits.
static __device__ __align__(256) unsigned char g_static_scratch[SWX_STATIC_SCRATCH_BYTES];

// cuCtxGetCurrent, resolved through the runtime so that the library needs no link to
// the driver library.
using CtxGetCurrentFn = CUresult (*)(CUcontext*);

CtxGetCurrentFn ctx_get_current() {
    static CtxGetCurrentFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<CtxGetCurrentFn>(nullptr);
        return reinterpret_cast<CtxGetCurrentFn>(p);
    }();
    return fn;
}

struct Entry {
    int dev;
    CUcontext ctx;
    void* ptr;
};
std::mutex g_mu;
std::vector<Entry> g_seen;

// Device address of g_static_scratch in the current context.  In host code the array's
// name is only a host-side stand-in, so the address is looked up with
// cudaGetSymbolAddress (with the device current) the first time a (device, context) pair
// is seen, and cached under that pair: after cudaDeviceReset, or when a binding makes its
// own driver context current, the module is loaded again, possibly at another address,
// and the new context gets its own lookup.
int scratch_address(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return SWX_ERR_CUDA;
    const CtxGetCurrentFn get = ctx_get_current();
    if (!get) return SWX_ERR_CUDA;
    CUcontext ctx = nullptr;
    if (get(&ctx) != CUDA_SUCCESS) return SWX_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_mu);
    if (ctx) {
        for (const Entry& e : g_seen)
            if (e.dev == dev && e.ctx == ctx) {
                *out = e.ptr;
                return SWX_OK;
            }
    }
    // first call in this context (or no context current yet on this thread: the lookup
    // makes the runtime's context current, and the pair is cached under it)
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p) return SWX_ERR_CUDA;
    if (!ctx && (get(&ctx) != CUDA_SUCCESS || !ctx)) return SWX_ERR_CUDA;
    g_seen.push_back({dev, ctx, p});
    *out = p;
    return SWX_OK;
}

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
    const int s = scratch_address(&scratch);
    if (s != SWX_OK) return s;
    swx_scan_args b = *a;
    b.workspace = scratch;
    b.workspace_bytes = (int64_t)SWX_STATIC_SCRATCH_BYTES;
    return swx_scan_bwd(&b, stream);
}
