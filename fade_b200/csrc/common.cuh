// Shared helpers for the sm_100a kernels of libfade_sm100.so.
//
// Numerics note: the library is compiled WITHOUT --use_fast_math.  The
// quantisers reproduce the reference's per-op rounding (torch computes a
// half/bfloat16 op in fp32 and rounds the result once), so every such op is
// written as an explicit fp32 op with _rn intrinsics followed by a rounding
// to the storage type.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/fade_b200.h"

namespace fade {

// ---------------------------------------------------------------------------
// Host-side status plumbing
// ---------------------------------------------------------------------------
void set_last_cuda_error(int e);

#define FADE_CHECK_ARG(cond)                  \
    do {                                      \
        if (!(cond)) return FADE_ERR_INVALID_ARG; \
    } while (0)

#define FADE_LAUNCH_CHECK()                          \
    do {                                             \
        cudaError_t _e = cudaGetLastError();         \
        if (_e != cudaSuccess) {                     \
            ::fade::set_last_cuda_error((int)_e);    \
            return FADE_ERR_CUDA;                    \
        }                                            \
    } while (0)

#define FADE_CUDA_TRY(call)                          \
    do {                                             \
        cudaError_t _e = (call);                     \
        if (_e != cudaSuccess) {                     \
            ::fade::set_last_cuda_error((int)_e);    \
            return FADE_ERR_CUDA;                    \
        }                                            \
    } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// Element types
// ---------------------------------------------------------------------------
template <int DT> struct Elem;
template <> struct Elem<FADE_F16> {
    using T = __half;
    __device__ __forceinline__ static float to_f(T x) { return __half2float(x); }
    __device__ __forceinline__ static T from_f(float x) { return __float2half_rn(x); }
    // Round an fp32 value to the nearest representable half, returned as fp32.
    __device__ __forceinline__ static float rnd(float x) { return __half2float(__float2half_rn(x)); }
    // torch's clamp(min=1e-8) evaluated in this dtype.
    __device__ __forceinline__ static float eps() { return __half2float(__float2half_rn(1e-8f)); }
};
template <> struct Elem<FADE_BF16> {
    using T = __nv_bfloat16;
    __device__ __forceinline__ static float to_f(T x) { return __bfloat162float(x); }
    __device__ __forceinline__ static T from_f(float x) { return __float2bfloat16_rn(x); }
    __device__ __forceinline__ static float rnd(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
    __device__ __forceinline__ static float eps() { return __bfloat162float(__float2bfloat16_rn(1e-8f)); }
};
template <> struct Elem<FADE_F32> {
    using T = float;
    __device__ __forceinline__ static float to_f(T x) { return x; }
    __device__ __forceinline__ static T from_f(float x) { return x; }
    __device__ __forceinline__ static float rnd(float x) { return x; }
    __device__ __forceinline__ static float eps() { return 1e-8f; }
};

// torch's float -> int8 conversion of a value already clamped to the code
// range; NaN (0 * inf when a channel is all zero in fp16) converts to 0, the
// value torch produces on CPU for that case.
__device__ __forceinline__ int code_from_float(float v) {
    return (v != v) ? 0 : (int)v;
}

// q = clamp(rint(x), lo, hi) with NaN -> 0; rintf rounds half to even like
// torch.round.
// round half to even, clamp to [lo, hi]; NaN -> 0 (torch.clamp keeps NaN and
// NaN -> int8 gives 0).  cvt.rni.s32.f32 rounds to nearest even, saturates
// out-of-range values and turns NaN into 0, so the integer clamp after it
// equals rint + clamp in fp32 + conversion.
__device__ __forceinline__ int quant_code(float x, float lo, float hi) {
    int i;
    asm("cvt.rni.s32.f32 %0, %1;" : "=r"(i) : "f"(x));
    return min(max(i, (int)lo), (int)hi);
}

// The reference's `qmax / absmax` is torch's __rtruediv__, i.e.
// reciprocal(absmax) rounded to the dtype, times qmax, rounded again.
template <int DT>
__device__ __forceinline__ float inv_scale(float absmax, float qmax) {
    float r = Elem<DT>::rnd(__frcp_rn(absmax));
    return Elem<DT>::rnd(__fmul_rn(r, qmax));
}

// ---------------------------------------------------------------------------
// Small PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t lop3_and_xor(uint32_t a, uint32_t mask, uint32_t k) {
    // (a & mask) ^ k
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(d) : "r"(a), "r"(mask), "r"(k));
    return d;
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void griddep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace fade
