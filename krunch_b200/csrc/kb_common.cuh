// Shared helpers for the krunch_b200 kernels: status plumbing, the library's
// fixed-order exp, and the range-coder constants.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/krunch_b200.h"

namespace kb {

// Thread-local CUDA error slot behind kb_last_cuda_error().
void set_cuda_error(cudaError_t e);

// Map the last launch error to a status; records the CUDA code.
inline int launch_status() {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_cuda_error(e);
        return KB_ERR_CUDA;
    }
    return KB_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// Range coder constants (32-bit state, E1/E2/E3 renormalisation):
// krunch_ac/cpu_reference.py:28-32, krunch_ac/cuda/range_coder.cuh:7-12.
// ---------------------------------------------------------------------------
constexpr uint32_t RC_HALF = 1u << 31;
constexpr uint32_t RC_QTR = 1u << 30;
constexpr uint32_t RC_THREE_QTR = RC_HALF + RC_QTR;

// ---------------------------------------------------------------------------
// kb_expf: the library's own exp, written with explicitly rounded operations
// (no contraction, no approximate hardware units) so that a plain C
// restatement reproduces it bit for bit.
//
// Method: Cody-Waite range reduction x = n*ln2 + r with ln2 split into a
// 12-bit head (exact n*head for |n| < 2^12) and a tail; e^r by its degree-6
// Taylor polynomial in Horner form (|r| <= 0.35, truncation < 1.5e-7
// relative); scaling by 2^n through the exponent field.  Inputs below -86
// return 0 (keeps every result a normal number, so flush-to-zero settings
// cannot change bits); NaN returns 0.  Inputs must be <= 88.
// ---------------------------------------------------------------------------
__host__ __device__ inline float kb_bits_to_float(uint32_t u) {
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    float f;
    __builtin_memcpy(&f, &u, 4);
    return f;
#endif
}

__device__ __forceinline__ float kb_expf(float x) {
    if (!(x >= -86.0f)) return 0.0f;
    const float LOG2E = kb_bits_to_float(0x3fb8aa3bu);   // 1/ln2 rounded to fp32
    const float LN2_HI = kb_bits_to_float(0x3f317000u);  // ln2 with 12 low bits cleared
    const float LN2_LO = kb_bits_to_float(0x3805fdf4u);  // ln2 - LN2_HI rounded
    const float n = rintf(__fmul_rn(x, LOG2E));
    float r = __fmaf_rn(-n, LN2_HI, x);
    r = __fmaf_rn(-n, LN2_LO, r);
    float p = 1.0f / 720.0f;
    p = __fmaf_rn(p, r, 1.0f / 120.0f);
    p = __fmaf_rn(p, r, 1.0f / 24.0f);
    p = __fmaf_rn(p, r, 1.0f / 6.0f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const uint32_t e = (uint32_t)((int)n + 127) << 23;
    return __fmul_rn(p, __uint_as_float(e));
}

__device__ __forceinline__ float h2f(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ uint16_t f2h(float f) {
    return __half_as_ushort(__float2half_rn(f));
}

}  // namespace kb
