// Host-side launch helpers shared by the kernel files: one-time opt-in to large
// dynamic shared memory and a cached occupancy query, both keyed by (device, kernel) so
// launches inside CUDA-graph capture make no configuration calls after the first.
#pragma once
#include <cuda_runtime.h>

#include <mutex>
#include <vector>

namespace swx {

// status.cu: device address of one of the library's __device__ variables in the current
// context (cached per device, context and variable), and the address of the status word
// that kernels with bounded waits set to SWX_ERR_TIMEOUT (nullptr if the lookup failed).
int device_symbol_address(const void* sym, void** out);
int* wait_status_address();

// Opt a kernel into more than 48 KB of dynamic shared memory.  Done once per kernel
// and device (cached), so later launches -- e.g. inside CUDA-graph capture -- make no
// runtime configuration calls.
template <typename K>
inline cudaError_t allow_smem(K kernel, int bytes) {
    struct Entry { int dev; const void* fn; };
    static std::mutex mu;
    static std::vector<Entry> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const void* fn = reinterpret_cast<const void*>(kernel);
    std::lock_guard<std::mutex> lock(mu);
    for (const Entry& x : done)
        if (x.dev == dev && x.fn == fn) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done.push_back({dev, fn});
    return e;
}

// SM count of the current device and how many CTAs of `kernel` fit on one SM at the given
// block and shared-memory size; queried once per (device, kernel), then cached.
template <typename K>
inline cudaError_t sm_fit(K kernel, int threads, int smem, int* sms, int* per_sm) {
    struct Entry { int dev; const void* fn; int sms, per_sm; };
    static std::mutex mu;
    static std::vector<Entry> seen;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const void* fn = reinterpret_cast<const void*>(kernel);
    std::lock_guard<std::mutex> lock(mu);
    for (const Entry& x : seen)
        if (x.dev == dev && x.fn == fn) { *sms = x.sms; *per_sm = x.per_sm; return cudaSuccess; }
    e = cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, kernel, threads, smem);
    if (e == cudaSuccess) seen.push_back({dev, fn, *sms, *per_sm});
    return e;
}

}  // namespace swx
