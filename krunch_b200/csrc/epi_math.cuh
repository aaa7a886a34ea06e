// Scalar arithmetic of the GEMM epilogues, shared by the tcgen05 GEMM
// (gemm_tc.cu) and the fused decode step (step_fused.cu), so that both
// produce the same bits.
#pragma once
#include "kb_common.cuh"

namespace kb {

// w8a8 dequantisation of an exact int32 accumulator
__device__ __forceinline__ float epi_dequant(int acc, float sa, float sw) {
    return __fmul_rn(__fmul_rn(__int2float_rn(acc), sa), sw);
}
__device__ __forceinline__ float epi_sigmoid(float y) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, __expf(-y)));
}
__device__ __forceinline__ float epi_relu_sq(float y) {
    y = fmaxf(y, 0.0f);
    return __fmul_rn(y, y);
}
// resid + g * y with one rounding (g = 1 for the plain residual)
__device__ __forceinline__ float epi_gate_resid(float g, float y, float resid) {
    return __fmaf_rn(g, y, resid);
}

}  // namespace kb
