// Shared helpers for the krunch_b200 kernels: status plumbing, the library's
// fixed-order exp, and the range-coder constants.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cuda_bf16.h>
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

// Runs f (a cudaError_t-returning setter, e.g. a kernel's shared-memory
// attribute) once per device of the process; idempotent if two host threads
// race on the first call.
template <class F>
inline cudaError_t once_per_device(std::atomic<unsigned long long>& done, F&& f) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    const unsigned long long bit = 1ull << (dev & 63);
    if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
    const cudaError_t e = f();
    if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

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
// Method: e^x = 2^y with y = x * log2(e) (one rounding); y = n + f with
// n = rint(y) (ties to even), |f| <= 1/2; 2^f by the degree-5 Taylor polynomial of
// e^(f ln 2) in Horner form (truncation < 2.6e-6 relative); 2^n added to the
// exponent field.  Relative error below 7e-6 over the domain.  Inputs below
// -86 return 0 (so every result is a normal number and flush-to-zero
// settings cannot change bits); NaN returns 0.  Inputs must be <= 88.
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

// kb_expf without the range check, for -86 <= x <= 88.
__device__ __forceinline__ float kb_expf_core(float x) {
    const float LOG2E = kb_bits_to_float(0x3fb8aa3bu);  // 1/ln2 rounded to fp32
    const float y = __fmul_rn(x, LOG2E);
    // n = rint(y) (half to even) without the conversion pipe: adding
    // 1.5 * 2^23 rounds y to an integer in the low mantissa bits (|y| < 2^22)
    const float MAGIC = 12582912.0f;
    const float t = __fadd_rn(y, MAGIC);
    const float n = __fsub_rn(t, MAGIC);
    const float f = __fsub_rn(y, n);
    float p = kb_bits_to_float(0x3aaec3ffu);             // ln2^5/5!
    p = __fmaf_rn(p, f, kb_bits_to_float(0x3c1d955bu));  // ln2^4/4!
    p = __fmaf_rn(p, f, kb_bits_to_float(0x3d635847u));  // ln2^3/3!
    p = __fmaf_rn(p, f, kb_bits_to_float(0x3e75fdf0u));  // ln2^2/2!
    p = __fmaf_rn(p, f, kb_bits_to_float(0x3f317218u));  // ln2
    p = __fmaf_rn(p, f, 1.0f);
    // bits(t) = 0x4B400000 + n; shifted left by 23 the constant part leaves
    // 32 bits, so this adds n to p's exponent field
    return __uint_as_float(__float_as_uint(p) + (__float_as_uint(t) << 23));
}

__device__ __forceinline__ float kb_expf(float x) {
    if (!(x >= -86.0f)) return 0.0f;
    return kb_expf_core(x);
}

__device__ __forceinline__ float h2f(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ uint16_t f2h(float f) {
    return __half_as_ushort(__float2half_rn(f));
}
__device__ __forceinline__ uint16_t f2bf(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

}  // namespace kb
