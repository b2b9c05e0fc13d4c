// Shared device helpers for the sm_100a selective-scan kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "swiftx_b200.h"

namespace swx {

constexpr int NS = 16;        // padded state count (N <= 16)
constexpr int TCK = 16;       // checkpoint interval of the forward / chunk of the backward
constexpr float LOG2E = 1.4426950408889634f;

// ---------------------------------------------------------------- element types
template <typename T> struct Elem;
template <> struct Elem<float> {
    static __device__ __forceinline__ float to_f(float v) { return v; }
    static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Elem<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

// ---------------------------------------------------------------- math
// 2^x on the MUFU unit (PTX ex2.approx, flush-to-zero).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float lg2(float x) {
    float y;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rcp(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// softplus with torch's threshold (beta=1, threshold=20).  For e = exp(x) < 1/8,
// log1p(e) is its alternating Taylor series to e^8 (relative truncation error
// below e^8/9 / e < 6e-8), because lg2.approx has an absolute error near 1 that
// would be a large relative error of a small result; otherwise log2(1+e)*ln2.
__device__ __forceinline__ float softplus_f(float x) {
    float e = ex2(x * LOG2E);
    float p = -0.125f;
    p = fmaf(p, e, 0.14285715f);
    p = fmaf(p, e, -0.16666667f);
    p = fmaf(p, e, 0.2f);
    p = fmaf(p, e, -0.25f);
    p = fmaf(p, e, 0.33333334f);
    p = fmaf(p, e, -0.5f);
    p = fmaf(p, e, 1.f);
    float series = p * e;
    float logv = lg2(1.f + e) * 0.69314718055994531f;
    float r = e < 0.125f ? series : logv;
    return x > 20.f ? x : r;
}
__device__ __forceinline__ float sigmoid_f(float x) { return rcp(1.f + ex2(-x * LOG2E)); }
__device__ __forceinline__ float silu_f(float x) { return x * sigmoid_f(x); }

// ---------------------------------------------------------------- packed fp32 (sm_100 f32x2)
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 bc2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 ex2x2(float2 x) { return make_float2(ex2(x.x), ex2(x.y)); }

__device__ __forceinline__ float2 rcp2(float2 x) { return make_float2(rcp(x.x), rcp(x.y)); }

// 2^x of two values on the FMA pipe instead of the MUFU unit (which runs at 16 results per
// clock per SM, an eighth of the FMA pipe): x = j + r with j = rint(x) from the
// round-to-integer constant 1.5 * 2^23 and |r| <= 1/2, then a degree-5 polynomial for
// 2^r on [-1/2, 1/2] -- the minimax fit of the relative error by a Remez exchange
// (fit_exp2_poly.py; 7.5e-8 for the float64 fit, about 2e-7 as evaluated in fp32, the
// order of ex2.approx) -- and 2^j added to the exponent field.
// Below -125 the result is 0, as ex2.approx.ftz flushes results under 2^-126; x is
// clamped at 127 above (finite where ex2.approx overflows).
__device__ __forceinline__ float2 ex2x2_fma(float2 x) {
    const bool z0 = x.x < -125.f, z1 = x.y < -125.f;
    x.x = fminf(fmaxf(x.x, -125.f), 127.f);
    x.y = fminf(fmaxf(x.y, -125.f), 127.f);
    const float2 t = add2(x, bc2(12582912.f));          // 1.5 * 2^23 + rint(x)
    const float2 j = add2(t, bc2(-12582912.f));         // rint(x), exact
    const float2 r = fma2(j, bc2(-1.f), x);              // x - j, exact
    float2 q = bc2(1.3276472454890609e-3f);
    q = fma2(q, r, bc2(9.675540961325169e-3f));
    q = fma2(q, r, bc2(5.550713092088699e-2f));
    q = fma2(q, r, bc2(2.4022120237350464e-1f));
    q = fma2(q, r, bc2(6.931469440460205e-1f));
    q = fma2(q, r, bc2(1.0000001192092896f));
    // low mantissa bits of t hold j: (bits(t) << 23) = j << 23 (mod 2^32)
    const float2 y = make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                                 __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
    return make_float2(z0 ? 0.f : y.x, z1 ? 0.f : y.y);
}

// softplus of two values (torch threshold 20) and its derivative sigmoid(x), sharing
// e = exp(x).  For e < 1/16, log1p(e) is its alternating Taylor series through e^6
// (relative truncation error below e^6/7 < 3e-9) because lg2.approx has an absolute
// error near 1 that would be a large relative error of a small result; otherwise
// log2(1 + e) * ln2.  sigmoid(x) = e / (1 + e).
__device__ __forceinline__ void softplus2(float2 x, float2& sp, float2& dsp) {
    const float2 e = ex2x2(mul2(x, bc2(LOG2E)));
    float2 p = bc2(-0.16666667f);
    p = fma2(p, e, bc2(0.2f));
    p = fma2(p, e, bc2(-0.25f));
    p = fma2(p, e, bc2(0.33333334f));
    p = fma2(p, e, bc2(-0.5f));
    p = fma2(p, e, bc2(1.f));
    const float2 ser = mul2(p, e);
    const float2 ope = add2(bc2(1.f), e);
    const float2 lg = mul2(make_float2(lg2(ope.x), lg2(ope.y)), bc2(0.69314718055994531f));
    const float2 sg = mul2(e, rcp2(ope));
    sp.x = x.x > 20.f ? x.x : (e.x < 0.0625f ? ser.x : lg.x);
    sp.y = x.y > 20.f ? x.y : (e.y < 0.0625f ? ser.y : lg.y);
    dsp.x = x.x > 20.f ? 1.f : sg.x;
    dsp.y = x.y > 20.f ? 1.f : sg.y;
}
__device__ __forceinline__ float2 sigmoid2(float2 x) {
    return rcp2(add2(bc2(1.f), ex2x2(mul2(x, bc2(-LOG2E)))));
}

// ---------------------------------------------------------------- named barriers
// Producer/consumer hand-off between warp groups: the producer arrives (no wait),
// the consumer syncs; `n` counts all participating threads of both groups.
__device__ __forceinline__ void bar_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;\n" :: "r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void bar_arrive(int id, int n) {
    asm volatile("bar.arrive %0, %1;\n" :: "r"(id), "r"(n) : "memory");
}

// ---------------------------------------------------------------- async copies
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// 16-byte cp.async; bytes < 16 zero-fills the tail (bytes = 0 zero-fills all 16).
__device__ __forceinline__ void cp_async16(void* sdst, const void* gsrc, int bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n"
                 :: "r"(smem_u32(sdst)), "l"(gsrc), "r"(bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" :: "n"(N)); }

// ---------------------------------------------------------------- bulk copies (TMA engine)
// One-thread bulk global -> shared copies that complete on an mbarrier: the issuing thread
// announces the bytes it expects (arrive.expect_tx), the copies count them down, and the
// phase completes when all have landed.  Waits are bounded: a phase that does not complete
// within `limit` polls (a byte count that does not match the copies) is reported instead
// of spinning forever.
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    uint64_t state;
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 %0, [%1], %2;"
                 : "=l"(state) : "r"(smem_u32(bar)), "r"(bytes) : "memory");
    (void)state;
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile("{\n\t.reg .pred P;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
                 "selp.b32 %0, 1, 0, P;\n\t}"
                 : "=r"(done) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return done != 0;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
// Order this thread's view of shared memory (after a barrier that followed other threads'
// ordinary loads) before the bulk copies it issues next into the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// A 3-D tile of the tensor described by `map` (a __grid_constant__ kernel parameter),
// starting at element coordinates (x, y, z), into this CTA's shared memory; completes on
// `bar`.  x times the element size must be a multiple of 16 bytes; coordinates past the
// tensor's extent read zeros.  No multicast: the tile lands in this CTA only.
__device__ __forceinline__ void tma_load_3d(void* sdst, const void* map, int x, int y, int z, uint64_t* bar) {
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
                 "[%0], [%1, {%2, %3, %4}], [%5];"
                 :: "r"(smem_u32(sdst)), "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)) : "memory");
}

// Copy a [rows x W] tile (row r at g + r*row_stride, columns [0, w_valid)) into
// dense shared memory s[rows][W], zero-filling invalid rows and columns.
// vec: every row start is 16-byte aligned, so 16-byte cp.async is used;
// otherwise scalar loads (for odd shapes and strides).
template <typename T, int W>
__device__ __forceinline__ void stage_tile(T* s, const T* g, int64_t row_stride, int rows,
                                           int rows_valid, int w_valid, bool vec, int tid,
                                           int nthreads) {
    if (vec) {
        constexpr int EPS = 16 / sizeof(T);          // elements per 16-byte segment
        constexpr int SEGS = W / EPS;
        for (int i = tid; i < rows * SEGS; i += nthreads) {
            int r = i / SEGS, sg = i % SEGS;
            int c0 = sg * EPS;
            int valid = (r < rows_valid) ? min(EPS, max(0, w_valid - c0)) : 0;
            const T* src = valid > 0 ? g + (int64_t)r * row_stride + c0 : g;
            cp_async16(s + r * W + c0, src, valid * (int)sizeof(T));
        }
    } else {
        for (int i = tid; i < rows * W; i += nthreads) {
            int r = i / W, c = i % W;
            T v = T(0.f);
            if (r < rows_valid && c < w_valid) v = g[(int64_t)r * row_stride + c];
            s[i] = v;
        }
    }
}

}  // namespace swx
