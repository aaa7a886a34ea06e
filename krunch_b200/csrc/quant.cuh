// Symmetric int8 quantisation used by the w8a8 model (KB_I8).
//   activations, per row:  amax = max |a| over the row's fp16 values,
//                          q = clamp(rint(a * (127 / amax)), -127, 127),
//                          dequantisation factor amax / 127 (fp32);
//   weights, per output channel n: s_n = fp16(amax_n / 127),
//                          q = clamp(rint(w / s_n), -127, 127).
// An all-zero row quantises to zeros with factor 0.  rint rounds half to
// even; every step is an explicitly rounded IEEE operation, so the packed
// encoder, the stepped decoder and the C oracle quantise identically.
#pragma once
#include "kb_common.cuh"

namespace kb {

__device__ __forceinline__ float q_inv(float amax) {
    return amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
}
__device__ __forceinline__ float q_factor(float amax) { return __fdiv_rn(amax, 127.0f); }
__device__ __forceinline__ int q8(float a, float inv) {
    const float r = rintf(__fmul_rn(a, inv));
    return (int)fminf(fmaxf(r, -127.0f), 127.0f);
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}
// four int8 values packed little-endian into a 32-bit word
__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
    return (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) | ((uint32_t)(c & 0xff) << 16) |
           ((uint32_t)(d & 0xff) << 24);
}

}  // namespace kb
