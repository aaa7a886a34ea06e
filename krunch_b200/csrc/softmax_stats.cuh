// Softmax pieces shared by the head GEMM epilogue (gemm_tc.cu) and the CDF
// kernels (cdf.cu).
//
// A logits row x (fp16 values) is cut into 32-column subtiles.  For subtile u
// with columns [32u, min(32u+32, V)):
//   m_u  = max x_i
//   e_i  = fp16(kb_expf(x_i - m_u))                  (stored by the head GEMM)
//   s_u  = sum_i e_i, left to right in fp32
// The row normaliser (M, S) merges the (m_u, s_u): thread t of 512 merges
// u = t, t+512, ... in order, each warp combines in a xor butterfly, then the
// 16 warp results (padded to 32 with the neutral (-inf, 0)) combine in the
// same butterfly.  merge() keeps the larger max and adds the other sum scaled
// by e^(m_small - m_large) (ties add the sums); it is symmetric, so every
// lane ends with the same bits.  Then, with scale = T - V,
//   gs_u = (kb_expf(m_u - M) * (1/S)) * scale,   q_i = e_i * gs_u,
//   c_i  = floor(q_i) + 1,   argmax = smallest i with the largest q_i.
// All arithmetic is explicitly rounded and exp is kb_expf, so a plain C
// restatement reproduces every value bit for bit.
#pragma once
#include "kb_common.cuh"

namespace kb {

constexpr int SUBTILE = 32;  // columns per softmax partial (one TMEM load)
static_assert(SUBTILE == 32, "the CDF argmax search takes one warp ballot per subtile");

struct MS {
    float m, s;
};

__device__ __forceinline__ MS ms_merge(MS a, MS b) {
    if (a.m >= b.m) return MS{a.m, __fadd_rn(a.s, __fmul_rn(b.s, kb_expf(__fsub_rn(b.m, a.m))))};
    return MS{b.m, __fadd_rn(b.s, __fmul_rn(a.s, kb_expf(__fsub_rn(a.m, b.m))))};
}

__device__ __forceinline__ MS ms_shfl_xor(MS v, int off) {
    return MS{__shfl_xor_sync(0xffffffffu, v.m, off), __shfl_xor_sync(0xffffffffu, v.s, off)};
}

// e_i of a logit relative to its subtile max, as stored (fp16 bits).
__device__ __forceinline__ float exp_rel_core(float x, float m) {
    return kb_expf(__fsub_rn(x, m));
}
__device__ __forceinline__ uint16_t exp_rel_f16(float x, float m) {
    return f2h(exp_rel_core(x, m));
}
// Two consecutive numerators packed as stored (element j in the low half),
// and their fp16 values as floats for the running sum.
__device__ __forceinline__ uint32_t exp_rel_pair(float x0, float x1, float m, float& e0,
                                                 float& e1) {
    const __half2 h = __floats2half2_rn(exp_rel_core(x0, m), exp_rel_core(x1, m));
    const float2 f = __half22float2(h);
    e0 = f.x;
    e1 = f.y;
    return *reinterpret_cast<const uint32_t*>(&h);
}

}  // namespace kb
