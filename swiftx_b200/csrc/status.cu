// The status word of the library's bounded device-side waits, and the lookup of device
// addresses of the library's __device__ variables.
//
// A kernel that waits for its own asynchronous copies (the TMA tiles of the scan forward,
// the backward's summary and main kernels and the whole-row backward) gives every wait an
// iteration limit.  When a wait runs out the kernel records SWX_ERR_TIMEOUT in
// g_wait_status and returns, leaving its results incomplete but the context usable;
// swx_device_wait_status() reads (and clears) the word on the host.
#include <cuda.h>

#include <mutex>
#include <vector>

#include "common.cuh"
#include "launch_util.cuh"

namespace {

static __device__ int g_wait_status;

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
    const void* sym;
    void* ptr;
};
std::mutex g_mu;
std::vector<Entry> g_seen;

// One thread waits, with `polls` tries, for the first phase of an mbarrier on which
// nothing ever arrives, and records the timeout as the segmented backward does.
__global__ void wait_timeout_kernel(uint32_t polls, int* status) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    swx::mbar_init(&bar, 1);
    swx::mbar_fence_init();
    if (!swx::mbar_wait_bounded(&bar, 0, polls) && status) *status = SWX_ERR_TIMEOUT;
}

}  // namespace

namespace swx {

// Device address of a __device__ variable of this library in the current context.  In
// host code the variable's name is only a host-side stand-in, so the address is looked
// up with cudaGetSymbolAddress (with the device current) the first time a (device,
// context, variable) triple is seen, and cached under it: after cudaDeviceReset, or when
// a binding makes its own driver context current, the module is loaded again, possibly at
// another address, and the new context gets its own lookup.
int device_symbol_address(const void* sym, void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return SWX_ERR_CUDA;
    const CtxGetCurrentFn get = ctx_get_current();
    if (!get) return SWX_ERR_CUDA;
    CUcontext ctx = nullptr;
    if (get(&ctx) != CUDA_SUCCESS) return SWX_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_mu);
    if (ctx) {
        for (const Entry& e : g_seen)
            if (e.dev == dev && e.ctx == ctx && e.sym == sym) {
                *out = e.ptr;
                return SWX_OK;
            }
    }
    // first call in this context (or no context current yet on this thread: the lookup
    // makes the runtime's context current, and the triple is cached under it)
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, sym) != cudaSuccess || !p) return SWX_ERR_CUDA;
    if (!ctx && (get(&ctx) != CUDA_SUCCESS || !ctx)) return SWX_ERR_CUDA;
    g_seen.push_back({dev, ctx, sym, p});
    *out = p;
    return SWX_OK;
}

int* wait_status_address() {
    void* p = nullptr;
    return device_symbol_address(&g_wait_status, &p) == SWX_OK ? static_cast<int*>(p) : nullptr;
}

}  // namespace swx

extern "C" int swx_device_wait_status(void) {
    if (cudaDeviceSynchronize() != cudaSuccess) return SWX_ERR_CUDA;
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_wait_status, sizeof(int)) != cudaSuccess) return SWX_ERR_CUDA;
    if (v != 0) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_wait_status, &zero, sizeof(int)) != cudaSuccess) return SWX_ERR_CUDA;
    }
    return v == 0 ? SWX_OK : v;
}

extern "C" int swx_diag_wait_timeout(uint32_t polls, void* stream) {
    int* status = swx::wait_status_address();
    if (!status) return SWX_ERR_CUDA;
    wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(polls, status);
    return cudaGetLastError() == cudaSuccess ? SWX_OK : SWX_ERR_CUDA;
}
