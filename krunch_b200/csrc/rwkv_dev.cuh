// Row-local and recurrent device functions of the RWKV-4 layer, shared by
// the per-op kernels (rwkv_ops.cu) and the fused decode step
// (step_fused.cu): both compile the same arithmetic, which is what makes the
// stepped decoder reproduce the packed encoder bit for bit.
#pragma once
#include "kb_common.cuh"
#include "quant.cuh"

namespace kb {

constexpr float LN_EPS = 1e-5f;  // F.layer_norm default (rwkv4_step_ref.py:57)
constexpr int LN_WARPS = 8;      // warps (rows) per block

// One warp per row: lane l owns the EPL = C/32 elements
//   vector layout (EPL % 8 == 0): 8-element chunks j*32 + l, j < EPL/8
//   scalar layout (otherwise):    elements j*32 + l,       j < EPL
// Sums run over the lane's elements in j order, then a xor butterfly — a
// fixed order, so a row's LayerNorm is the same in every launch shape.
template <int EPL>
struct RowIdx {
    static constexpr bool VEC = (EPL % 8) == 0;
    __device__ __forceinline__ static int col(int lane, int e) {
        return VEC ? (((e >> 3) * 32 + lane) << 3) + (e & 7) : e * 32 + lane;
    }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

template <int EPL>
__device__ __forceinline__ void load_vec_f32(const float* __restrict__ p, int lane, float (&v)[EPL]) {
    if (RowIdx<EPL>::VEC) {
#pragma unroll
        for (int j = 0; j < EPL / 8; ++j) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(p) + (j * 32 + lane) * 2);
            const float4 b = __ldg(reinterpret_cast<const float4*>(p) + (j * 32 + lane) * 2 + 1);
            v[j * 8 + 0] = a.x; v[j * 8 + 1] = a.y; v[j * 8 + 2] = a.z; v[j * 8 + 3] = a.w;
            v[j * 8 + 4] = b.x; v[j * 8 + 5] = b.y; v[j * 8 + 6] = b.z; v[j * 8 + 7] = b.w;
        }
    } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) v[e] = __ldg(p + e * 32 + lane);
    }
}

// NC = false for data written earlier in the same launch (the fused step):
// the read-only path is only valid for data constant during the kernel.
template <int EPL, bool NC = true>
__device__ __forceinline__ void load_row(const uint16_t* __restrict__ x, int lane, float (&v)[EPL]) {
    if (RowIdx<EPL>::VEC) {
#pragma unroll
        for (int j = 0; j < EPL / 8; ++j) {
            const uint4* src = reinterpret_cast<const uint4*>(x) + j * 32 + lane;
            const uint4 q = NC ? __ldg(src) : *src;
            const __half2* h = reinterpret_cast<const __half2*>(&q);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = __half22float2(h[k]);
                v[j * 8 + 2 * k] = f.x;
                v[j * 8 + 2 * k + 1] = f.y;
            }
        }
    } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) v[e] = h2f(x[e * 32 + lane]);
    }
}

// LayerNorm of one row (values in v), result rounded to fp16 precision (the
// reference keeps xx in the fp16 activation dtype, rwkv4_step_ref.py:57-61).
template <int EPL>
__device__ __forceinline__ void ln_warp(const float (&v)[EPL], int C, int lane,
                                        const float* __restrict__ w, const float* __restrict__ b,
                                        float (&out)[EPL]) {
    float s = 0.0f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) s = __fadd_rn(s, v[e]);
    const float mean = __fdiv_rn(warp_sum(s), (float)C);
    float q = 0.0f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
        const float d = __fsub_rn(v[e], mean);
        q = __fmaf_rn(d, d, q);
    }
    const float rstd = __frsqrt_rn(__fadd_rn(__fdiv_rn(warp_sum(q), (float)C), LN_EPS));
    float wv[EPL], bv[EPL];
    load_vec_f32<EPL>(w, lane, wv);
    load_vec_f32<EPL>(b, lane, bv);
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
        const float y = __fmaf_rn(__fmul_rn(__fsub_rn(v[e], mean), rstd), wv[e], bv[e]);
        out[e] = __half2float(__float2half_rn(y));
    }
}

// bf16 rows (the GEMM operands of a KB_BF16 model), same layout as fp16
template <int EPL>
__device__ __forceinline__ void store_row_bf16(uint16_t* __restrict__ dst, int lane, const float (&v)[EPL]) {
    if (RowIdx<EPL>::VEC) {
#pragma unroll
        for (int j = 0; j < EPL / 8; ++j) {
            uint4 q;
            __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&q);
#pragma unroll
            for (int k = 0; k < 4; ++k) h[k] = __floats2bfloat162_rn(v[j * 8 + 2 * k], v[j * 8 + 2 * k + 1]);
            reinterpret_cast<uint4*>(dst)[j * 32 + lane] = q;
        }
    } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) dst[e * 32 + lane] = f2bf(v[e]);
    }
}

template <int EPL>
__device__ __forceinline__ void store_row_f16(uint16_t* __restrict__ dst, int lane, const float (&v)[EPL]) {
    if (RowIdx<EPL>::VEC) {
#pragma unroll
        for (int j = 0; j < EPL / 8; ++j) {
            uint4 q;
            __half2* h = reinterpret_cast<__half2*>(&q);
#pragma unroll
            for (int k = 0; k < 4; ++k) h[k] = __floats2half2_rn(v[j * 8 + 2 * k], v[j * 8 + 2 * k + 1]);
            reinterpret_cast<uint4*>(dst)[j * 32 + lane] = q;
        }
    } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) dst[e * 32 + lane] = f2h(v[e]);
    }
}

// Row quantised to int8 (quant.cuh) from the fp16 rounding of v; lane 0
// writes the row's dequantisation factor to *qs.
template <int EPL>
__device__ __forceinline__ void store_row_q(int8_t* __restrict__ dst, float* qs, int lane,
                                            const float (&v)[EPL]) {
    float a[EPL], m = 0.0f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
        a[e] = __half2float(__float2half_rn(v[e]));
        m = fmaxf(m, fabsf(a[e]));
    }
    const float amax = warp_max(m);
    const float inv = q_inv(amax);
    if (RowIdx<EPL>::VEC) {
#pragma unroll
        for (int j = 0; j < EPL / 8; ++j) {
            const float* c = a + 8 * j;
            reinterpret_cast<uint2*>(dst)[j * 32 + lane] =
                make_uint2(pack4(q8(c[0], inv), q8(c[1], inv), q8(c[2], inv), q8(c[3], inv)),
                           pack4(q8(c[4], inv), q8(c[5], inv), q8(c[6], inv), q8(c[7], inv)));
        }
    } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) dst[e * 32 + lane] = (int8_t)q8(a[e], inv);
    }
    if (lane == 0) *qs = q_factor(amax);
}

// WKV-4 recurrence, one thread per (stream, channel), sequential over T.
// KB_WKV_STEP_REF  (rwkv4_step_ref.py:76-94, batched_rwkv4.py:141-155):
//   ww = pp + u; p = max(ww, k); e1 = e^(ww-p); e2 = e^(k-p)
// KB_WKV_PRODUCTION (krunch_ac/cuda/wkv_kernel.cu:57-72):
//   ww = u + k; p = max(pp, ww); e1 = e^(pp-p); e2 = e^(ww-p)
// then y = (e1*aa + e2*v) / (e1*bb + e2) and, in both,
//   ww2 = pp - decay; p2 = max(ww2, k); aa = e^(ww2-p2)*aa + e^(k-p2)*v;
//   bb = e^(ww2-p2)*bb + e^(k-p2); pp = p2.
// Output ry = r * y in fp16 (the (r * y) @ Ow operand, rwkv4_step_ref.py:96).
// Loads are issued WKV_BLK time steps at a time; every operation is an
// explicit intrinsic, so the blocked loop and the one-step tail (the stepped
// decoder, T = 1) compute identical bits.
constexpr int WKV_BLK = 16;

// e^(a - p) and e^(b - p) for p = max(a, b) with one exponential: one of the
// two differences is exactly zero and e^0 = 1 exactly, so the pair equals
// the two-exponential form bit for bit whenever a, b are finite (the
// recurrence's operands always are).  Halves the SFU work of a step.
__device__ __forceinline__ void exp_pair(float a, float b, float p, float& ea, float& eb) {
    const float da = __fsub_rn(a, p), db = __fsub_rn(b, p);
    const bool a_max = da == 0.0f;
    const float e = __expf(a_max ? db : da);
    ea = a_max ? 1.0f : e;
    eb = a_max ? e : 1.0f;
}

template <int CONV>
__device__ __forceinline__ float wkv_step(float& aa, float& bb, float& pp, float kt, float vt,
                                          float u, float dec) {
    float e1, e2;
    if (CONV == KB_WKV_STEP_REF) {
        const float ww = __fadd_rn(pp, u);
        exp_pair(ww, kt, fmaxf(ww, kt), e1, e2);
    } else {
        const float ww = __fadd_rn(u, kt);
        exp_pair(pp, ww, fmaxf(pp, ww), e1, e2);
    }
    const float y = __fdividef(__fmaf_rn(e1, aa, __fmul_rn(e2, vt)), __fmaf_rn(e1, bb, e2));
    const float ww2 = __fsub_rn(pp, dec);
    float f1, f2;
    exp_pair(ww2, kt, fmaxf(ww2, kt), f1, f2);
    aa = __fmaf_rn(f1, aa, __fmul_rn(f2, vt));
    bb = __fmaf_rn(f1, bb, f2);
    pp = fmaxf(ww2, kt);
    return y;
}

}  // namespace kb
