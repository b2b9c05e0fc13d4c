// Host-side encoding of the TMA tensor maps that the scan kernels stage their tiles with.
// Each map describes a (inner, L, b) tensor of this GPU's memory with element strides
// (1, row, batch) and a box of (box_inner, box_rows, 1); the kernels load it with
// cp.async.bulk.tensor.3d (common.cuh tma_load_3d, never with cluster multicast).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace swx {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled, resolved through the runtime (no link to the driver library).
inline EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) !=
                cudaSuccess || q != cudaDriverEntryPointSuccess)
            return static_cast<EncodeTiledFn>(nullptr);
        return reinterpret_cast<EncodeTiledFn>(f);
    }();
    return fn;
}

// False when the tensor cannot be described (base or strides not 16-byte aligned, no
// driver entry point): the caller then stages with per-thread cp.async.  es: element
// bytes, 4 (fp32) or 2 (bf16).  Coordinates past the extents read zeros.
inline bool encode_3d(CUtensorMap* m, const void* base, int es, int64_t inner, int64_t L, int64_t b, int64_t row,
                      int64_t batch, uint32_t box_inner, uint32_t box_rows) {
    const EncodeTiledFn f = encode_tiled();
    if (!f || !base || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
    const int64_t rs = row * es, bs = (b > 1 ? batch : row * L) * es;
    if (rs % 16 || bs % 16 || rs <= 0 || bs <= 0 || rs >= (int64_t(1) << 40) || bs >= (int64_t(1) << 40)) return false;
    cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)L, (cuuint64_t)b};
    cuuint64_t strides[2] = {(cuuint64_t)rs, (cuuint64_t)bs};
    cuuint32_t box[3] = {box_inner, box_rows, 1};
    cuuint32_t unit[3] = {1, 1, 1};
    return f(m, es == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
             const_cast<void*>(base), dims, strides, box, unit, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

}  // namespace swx
