// RWKV-4 row-local and recurrent kernels: embedding gather, LayerNorm fused
// with the token-shift mix, the WKV recurrence, decay preparation, state init.
//
// Row-local maths is fixed by the row alone (one warp per row, fixed
// reduction tree), and the token-shift input of the first row of a window is
// the carried state, so a window of T rows produces exactly the bits of T
// single-row steps.  That is what lets the stepped decoder reproduce the
// packed encoder's logits bit for bit.
#include <atomic>

#include "kb_common.cuh"
#include "quant.cuh"
#include "rwkv_dev.cuh"
#include "rwkv_ops.cuh"
#include "tc_common.cuh"

#ifndef KB_LN_TILE
#define KB_LN_TILE 1  // tiled LN + mix kernel (bulk-copied row tiles) for fp16 / bf16 outputs
#endif

namespace kb {

// LN + token-shift mix, one warp per strip of `rpw` consecutive rows:
//   prev(t) = state_in[b] for t == 0, else LN(x[t-1]) (carried from the
//             previous row of the strip, recomputed for the strip's first)
//   mix_j   = xx * m_j + prev * (1 - m_j)   (rwkv4_step_ref.py:59-61)
// Row index = b*T + t.  Every LN is the same function of its row alone, so
// the strip length changes no bits.  The stream's last row writes its xx to
// state_out[b]; xx_out (optional) receives xx.
template <int NMIX, int EPL>
__global__ void __launch_bounds__(LN_WARPS * 32) k_ln_mix(const uint16_t* __restrict__ x, int B,
                                                          int T, int C,
                                                          const float* __restrict__ lw,
                                                          const float* __restrict__ lb, MixArgs ma,
                                                          const float* __restrict__ state_in,
                                                          float* __restrict__ state_out,
                                                          uint16_t* __restrict__ xx_out, int rpw) {
    const int lane = threadIdx.x & 31;
    const int64_t rows = (int64_t)B * T;
    const int64_t r0 = ((int64_t)blockIdx.x * LN_WARPS + (threadIdx.x >> 5)) * rpw;
    float prev[EPL], cur[EPL];
    for (int j = 0; j < rpw; ++j) {
        const int64_t row = r0 + j;
        if (row >= rows) return;
        const int b = (int)(row / T);
        const int t = (int)(row - (int64_t)b * T);
        float v[EPL];
        load_row<EPL>(x + row * C, lane, v);
        if (NMIX > 0) {
            if (t == 0) {
#pragma unroll
                for (int e = 0; e < EPL; ++e)
                    prev[e] = state_in ? state_in[(int64_t)b * C + RowIdx<EPL>::col(lane, e)] : 0.0f;
            } else if (j == 0) {
                float pv[EPL];
                load_row<EPL>(x + (row - 1) * C, lane, pv);
                ln_warp<EPL>(pv, C, lane, lw, lb, prev);
            } else {
#pragma unroll
                for (int e = 0; e < EPL; ++e) prev[e] = cur[e];
            }
        }
        ln_warp<EPL>(v, C, lane, lw, lb, cur);
        if (xx_out) {
            if (ma.bf16) store_row_bf16<EPL>(xx_out + row * C, lane, cur);
            else store_row_f16<EPL>(xx_out + row * C, lane, cur);
        }
        if (NMIX == 0 && ma.q[0]) store_row_q<EPL>(ma.q[0] + row * C, ma.qs[0] + row, lane, cur);
#pragma unroll
        for (int m = 0; m < NMIX; ++m) {
            float mk[EPL];
            load_vec_f32<EPL>(ma.mix[m], lane, mk);
#pragma unroll
            for (int e = 0; e < EPL; ++e)
                mk[e] = __fmaf_rn(cur[e], mk[e], __fmul_rn(prev[e], __fsub_rn(1.0f, mk[e])));
            if (ma.q[m])
                store_row_q<EPL>(ma.q[m] + row * C, ma.qs[m] + row, lane, mk);
            else if (ma.bf16)
                store_row_bf16<EPL>(ma.out[m] + row * C, lane, mk);
            else
                store_row_f16<EPL>(ma.out[m] + row * C, lane, mk);
        }
        if (t == T - 1 && state_out) {
#pragma unroll
            for (int e = 0; e < EPL; ++e)
                state_out[(int64_t)b * C + RowIdx<EPL>::col(lane, e)] = cur[e];
        }
    }
}

// Packed form of k_ln_mix for vector rows (C % 256 == 0) with fp16 / bf16
// outputs: a row lives in registers as fp16 pairs — the input is fp16 and
// every LN output is rounded to fp16, so packing loses nothing — which halves
// the registers per row, so more warps keep loads in flight, and the next row
// of a strip is loaded while the current one is computed.  The operations
// and their order are those of ln_warp and k_ln_mix, so the bits are too.
__device__ __forceinline__ float2 h2f2(uint32_t u) {
    return __half22float2(*reinterpret_cast<const __half2*>(&u));
}
__device__ __forceinline__ uint32_t f2h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t f2bf2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// ln_warp on a packed row; out = the fp16-rounded LN values, packed
template <int EPL>
__device__ __forceinline__ void ln_warp_h2(const uint32_t (&v)[EPL / 2], int C, int lane,
                                           const float* __restrict__ w,
                                           const float* __restrict__ b, uint32_t (&out)[EPL / 2]) {
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < EPL / 2; ++i) {
        const float2 f = h2f2(v[i]);
        s = __fadd_rn(__fadd_rn(s, f.x), f.y);
    }
    const float mean = __fdiv_rn(warp_sum(s), (float)C);
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < EPL / 2; ++i) {
        const float2 f = h2f2(v[i]);
        const float d0 = __fsub_rn(f.x, mean), d1 = __fsub_rn(f.y, mean);
        q = __fmaf_rn(d0, d0, q);
        q = __fmaf_rn(d1, d1, q);
    }
    const float rstd = __frsqrt_rn(__fadd_rn(__fdiv_rn(warp_sum(q), (float)C), LN_EPS));
#pragma unroll
    for (int j = 0; j < EPL / 8; ++j) {
        const float4* w4 = reinterpret_cast<const float4*>(w) + (j * 32 + lane) * 2;
        const float4* b4 = reinterpret_cast<const float4*>(b) + (j * 32 + lane) * 2;
        const float4 wa = __ldg(w4), wb = __ldg(w4 + 1), ba = __ldg(b4), bb = __ldg(b4 + 1);
        const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        const float bv[8] = {ba.x, ba.y, ba.z, ba.w, bb.x, bb.y, bb.z, bb.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 f = h2f2(v[4 * j + k]);
            const float y0 = __fmaf_rn(__fmul_rn(__fsub_rn(f.x, mean), rstd), wv[2 * k], bv[2 * k]);
            const float y1 =
                __fmaf_rn(__fmul_rn(__fsub_rn(f.y, mean), rstd), wv[2 * k + 1], bv[2 * k + 1]);
            out[4 * j + k] = f2h2(y0, y1);
        }
    }
}

// Two rows of one warp at a time: the same operations on rows A and B,
// interleaved, so every parameter load (LN weight and bias) serves both.
template <int EPL>
__device__ __forceinline__ void ln_warp_h2x2(const uint32_t (&va)[EPL / 2],
                                             const uint32_t (&vb)[EPL / 2], int C, int lane,
                                             const float* __restrict__ w,
                                             const float* __restrict__ b, uint32_t (&oa)[EPL / 2],
                                             uint32_t (&ob)[EPL / 2]) {
    float sa = 0.0f, sb = 0.0f;
#pragma unroll
    for (int i = 0; i < EPL / 2; ++i) {
        const float2 fa = h2f2(va[i]), fb = h2f2(vb[i]);
        sa = __fadd_rn(__fadd_rn(sa, fa.x), fa.y);
        sb = __fadd_rn(__fadd_rn(sb, fb.x), fb.y);
    }
    const float ma = __fdiv_rn(warp_sum(sa), (float)C), mb = __fdiv_rn(warp_sum(sb), (float)C);
    float qa = 0.0f, qb = 0.0f;
#pragma unroll
    for (int i = 0; i < EPL / 2; ++i) {
        const float2 fa = h2f2(va[i]), fb = h2f2(vb[i]);
        const float a0 = __fsub_rn(fa.x, ma), a1 = __fsub_rn(fa.y, ma);
        const float b0 = __fsub_rn(fb.x, mb), b1 = __fsub_rn(fb.y, mb);
        qa = __fmaf_rn(a1, a1, __fmaf_rn(a0, a0, qa));
        qb = __fmaf_rn(b1, b1, __fmaf_rn(b0, b0, qb));
    }
    const float ra = __frsqrt_rn(__fadd_rn(__fdiv_rn(warp_sum(qa), (float)C), LN_EPS));
    const float rb = __frsqrt_rn(__fadd_rn(__fdiv_rn(warp_sum(qb), (float)C), LN_EPS));
#pragma unroll
    for (int j = 0; j < EPL / 8; ++j) {
        const float4* w4 = reinterpret_cast<const float4*>(w) + (j * 32 + lane) * 2;
        const float4* b4 = reinterpret_cast<const float4*>(b) + (j * 32 + lane) * 2;
        const float4 w0 = __ldg(w4), w1 = __ldg(w4 + 1), b0 = __ldg(b4), b1 = __ldg(b4 + 1);
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 fa = h2f2(va[4 * j + k]), fb = h2f2(vb[4 * j + k]);
            oa[4 * j + k] =
                f2h2(__fmaf_rn(__fmul_rn(__fsub_rn(fa.x, ma), ra), wv[2 * k], bv[2 * k]),
                     __fmaf_rn(__fmul_rn(__fsub_rn(fa.y, ma), ra), wv[2 * k + 1], bv[2 * k + 1]));
            ob[4 * j + k] =
                f2h2(__fmaf_rn(__fmul_rn(__fsub_rn(fb.x, mb), rb), wv[2 * k], bv[2 * k]),
                     __fmaf_rn(__fmul_rn(__fsub_rn(fb.y, mb), rb), wv[2 * k + 1], bv[2 * k + 1]));
        }
    }
}

// The same LN + mix for wide rows (C >= 1536, C % 256 == 0), without
// holding the row in registers: each warp stages its row in shared memory
// (fp16, as stored) and sums the statistics chunk by chunk in the lane order
// of ln_warp, so the bits are those of k_ln_mix.  The LN outputs of a strip's
// previous row are kept in shared memory for the token shift.  Quantised
// outputs take one more pass for the row maximum.
constexpr int LNS_MAX_C = 2048;
constexpr int LNS_WARPS = 4;  // 2 x 4 KB of row staging per warp
#ifndef LNS_MIN_EPL
#define LNS_MIN_EPL 48
#endif

__device__ __forceinline__ void unpack_chunk8(const uint4& q, float (&v)[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&q);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(h[k]);
        v[2 * k] = f.x;
        v[2 * k + 1] = f.y;
    }
}
__device__ __forceinline__ uint4 pack_chunk8(const float (&v)[8]) {
    uint4 o;
    __half2* h = reinterpret_cast<__half2*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) h[k] = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
    return o;
}
__device__ __forceinline__ uint4 pack_chunk8_bf(const float (&v)[8]) {
    uint4 o;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) h[k] = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
    return o;
}
__device__ __forceinline__ void load8f(const float* __restrict__ p, float (&v)[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// statistics of a row held as fp16 chunks (chunk j of lane at index j*32+lane)
__device__ __forceinline__ void ln_stats_chunks(const uint4* rowc, int C, int lane, float& mean,
                                                float& rstd) {
    const int nch = C / 256;
    float s = 0.0f;
    for (int j = 0; j < nch; ++j) {
        float v[8];
        unpack_chunk8(rowc[j * 32 + lane], v);
#pragma unroll
        for (int k = 0; k < 8; ++k) s = __fadd_rn(s, v[k]);
    }
    mean = __fdiv_rn(warp_sum(s), (float)C);
    float q = 0.0f;
    for (int j = 0; j < nch; ++j) {
        float v[8];
        unpack_chunk8(rowc[j * 32 + lane], v);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float d = __fsub_rn(v[k], mean);
            q = __fmaf_rn(d, d, q);
        }
    }
    rstd = __frsqrt_rn(__fadd_rn(__fdiv_rn(warp_sum(q), (float)C), LN_EPS));
}

__device__ __forceinline__ void ln_chunk8(const float (&v)[8], float mean, float rstd,
                                          const float (&w)[8], const float (&b)[8], float (&o)[8]) {
#pragma unroll
    for (int k = 0; k < 8; ++k)
        o[k] = __half2float(__float2half_rn(__fmaf_rn(__fmul_rn(__fsub_rn(v[k], mean), rstd), w[k], b[k])));
}

template <int NMIX>
__global__ void __launch_bounds__(LNS_WARPS * 32) k_ln_mix_stream(
    const uint16_t* __restrict__ x, int B, int T, int C, const float* __restrict__ lw,
    const float* __restrict__ lb, MixArgs ma, const float* __restrict__ state_in,
    float* __restrict__ state_out, uint16_t* __restrict__ xx_out, int rpw) {
    __shared__ uint4 s_row[LNS_WARPS][LNS_MAX_C / 8];   // this row, fp16
    __shared__ uint4 s_prev[LNS_WARPS][LNS_MAX_C / 8];  // LN of the previous row, fp16
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint4* rowc = s_row[warp];
    uint4* prevc = s_prev[warp];
    const int64_t rows = (int64_t)B * T;
    const int64_t r0 = ((int64_t)blockIdx.x * LNS_WARPS + warp) * rpw;
    const int nch = C / 256;
    const bool quant = ma.q[0] != nullptr;
    for (int jr = 0; jr < rpw; ++jr) {
        const int64_t row = r0 + jr;
        if (row >= rows) return;
        const int b = (int)(row / T);
        const int t = (int)(row - (int64_t)b * T);
        float mean, rstd;
        if (NMIX > 0 && t != 0 && jr == 0) {  // LN of the previous row into s_prev
            for (int j = 0; j < nch; ++j)
                rowc[j * 32 + lane] =
                    *reinterpret_cast<const uint4*>(x + (row - 1) * C + (j * 32 + lane) * 8);
            __syncwarp();
            ln_stats_chunks(rowc, C, lane, mean, rstd);
            for (int j = 0; j < nch; ++j) {
                const int c0 = (j * 32 + lane) * 8;
                float v[8], w[8], bb[8], o[8];
                unpack_chunk8(rowc[j * 32 + lane], v);
                load8f(lw + c0, w);
                load8f(lb + c0, bb);
                ln_chunk8(v, mean, rstd, w, bb, o);
                prevc[j * 32 + lane] = pack_chunk8(o);
            }
            __syncwarp();
        }
        for (int j = 0; j < nch; ++j)
            rowc[j * 32 + lane] = *reinterpret_cast<const uint4*>(x + row * C + (j * 32 + lane) * 8);
        __syncwarp();
        ln_stats_chunks(rowc, C, lane, mean, rstd);
        // chunk j of cur (LN) and of the mixes
        auto outputs = [&](int j, float (&cur)[8], float (&mk)[3][8]) {
            const int c0 = (j * 32 + lane) * 8;
            float v[8], w[8], bb[8];
            unpack_chunk8(rowc[j * 32 + lane], v);
            load8f(lw + c0, w);
            load8f(lb + c0, bb);
            ln_chunk8(v, mean, rstd, w, bb, cur);
            if (NMIX == 0) return;
            float prev[8];
            if (t == 0) {
                if (state_in) load8f(state_in + (int64_t)b * C + c0, prev);
                else
#pragma unroll
                    for (int k = 0; k < 8; ++k) prev[k] = 0.0f;
            } else {
                unpack_chunk8(prevc[j * 32 + lane], prev);
            }
#pragma unroll
            for (int m = 0; m < NMIX; ++m) {
                float mm[8];
                load8f(ma.mix[m] + c0, mm);
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    mk[m][k] = __half2float(__float2half_rn(
                        __fmaf_rn(cur[k], mm[k], __fmul_rn(prev[k], __fsub_rn(1.0f, mm[k])))));
            }
        };
        float inv[3] = {0.0f, 0.0f, 0.0f}, amax[3] = {0.0f, 0.0f, 0.0f};
        if (quant) {
            for (int j = 0; j < nch; ++j) {
                float cur[8], mk[3][8];
                outputs(j, cur, mk);
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    if (NMIX == 0) amax[0] = fmaxf(amax[0], fabsf(cur[k]));
#pragma unroll
                    for (int m = 0; m < NMIX; ++m) amax[m] = fmaxf(amax[m], fabsf(mk[m][k]));
                }
            }
#pragma unroll
            for (int m = 0; m < (NMIX > 0 ? NMIX : 1); ++m) {
                amax[m] = warp_max(amax[m]);
                inv[m] = q_inv(amax[m]);
            }
        }
        for (int j = 0; j < nch; ++j) {
            float cur[8], mk[3][8];
            outputs(j, cur, mk);
            const int c0 = (j * 32 + lane) * 8;
            if (xx_out)
                *reinterpret_cast<uint4*>(xx_out + row * C + c0) =
                    ma.bf16 ? pack_chunk8_bf(cur) : pack_chunk8(cur);
            if (NMIX == 0 && quant)
                *reinterpret_cast<uint2*>(ma.q[0] + row * C + c0) =
                    make_uint2(pack4(q8(cur[0], inv[0]), q8(cur[1], inv[0]), q8(cur[2], inv[0]), q8(cur[3], inv[0])),
                               pack4(q8(cur[4], inv[0]), q8(cur[5], inv[0]), q8(cur[6], inv[0]), q8(cur[7], inv[0])));
#pragma unroll
            for (int m = 0; m < NMIX; ++m) {
                if (quant) {
                    const float* a = mk[m];
                    *reinterpret_cast<uint2*>(ma.q[m] + row * C + c0) = make_uint2(
                        pack4(q8(a[0], inv[m]), q8(a[1], inv[m]), q8(a[2], inv[m]), q8(a[3], inv[m])),
                        pack4(q8(a[4], inv[m]), q8(a[5], inv[m]), q8(a[6], inv[m]), q8(a[7], inv[m])));
                } else {
                    *reinterpret_cast<uint4*>(ma.out[m] + row * C + c0) =
                        ma.bf16 ? pack_chunk8_bf(mk[m]) : pack_chunk8(mk[m]);
                }
            }
            if (t == T - 1 && state_out) {
                float4* so = reinterpret_cast<float4*>(state_out + (int64_t)b * C + c0);
                so[0] = make_float4(cur[0], cur[1], cur[2], cur[3]);
                so[1] = make_float4(cur[4], cur[5], cur[6], cur[7]);
            }
            if (NMIX > 0) prevc[j * 32 + lane] = pack_chunk8(cur);  // for the next row
        }
        if (quant && lane == 0) {
            if (NMIX == 0) ma.qs[0][row] = q_factor(amax[0]);
#pragma unroll
            for (int m = 0; m < NMIX; ++m) ma.qs[m][row] = q_factor(amax[m]);
        }
        __syncwarp();
    }
}

template <int CONV, bool BF>
__global__ void __launch_bounds__(128, 4) k_wkv(int B, int T, int C, const float* __restrict__ k,
                                                const float* __restrict__ v,
                                                const uint16_t* __restrict__ r,
                                                const float* __restrict__ decay,
                                                const float* __restrict__ first, float* aa_s,
                                                float* bb_s, float* pp_s,
                                                uint16_t* __restrict__ ry) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= B * C) return;
    const int b = idx / C, c = idx - b * C;
    const float dec = decay[c];
    const float u = first[c];
    float aa = aa_s[idx], bb = bb_s[idx], pp = pp_s[idx];
    const int64_t base = (int64_t)b * T * C + c;
    const float* kp = k + base;
    const float* vp = v + base;
    const uint16_t* rp = r + base;
    uint16_t* op = ry + base;
    // blocks of WKV_BLK steps; the next block's loads are in flight while
    // the current block is computed
    const int nblk = T / WKV_BLK;
    float kb[WKV_BLK], vb[WKV_BLK];
    uint16_t rb[WKV_BLK];
    if (nblk > 0) {
#pragma unroll
        for (int j = 0; j < WKV_BLK; ++j) {
            kb[j] = __ldg(kp + (int64_t)j * C);
            vb[j] = __ldg(vp + (int64_t)j * C);
            rb[j] = __ldg(rp + (int64_t)j * C);
        }
    }
    for (int ib = 0; ib < nblk; ++ib) {
        float kn[WKV_BLK], vn[WKV_BLK];
        uint16_t rn[WKV_BLK];
        const int64_t nx = (int64_t)WKV_BLK * C;
        if (ib + 1 < nblk) {
#pragma unroll
            for (int j = 0; j < WKV_BLK; ++j) {
                kn[j] = __ldg(kp + nx + (int64_t)j * C);
                vn[j] = __ldg(vp + nx + (int64_t)j * C);
                rn[j] = __ldg(rp + nx + (int64_t)j * C);
            }
        }
#pragma unroll
        for (int j = 0; j < WKV_BLK; ++j) {
            const float y = wkv_step<CONV>(aa, bb, pp, kb[j], vb[j], u, dec);
            const float o = __fmul_rn(h2f(rb[j]), y);
            op[(int64_t)j * C] = BF ? f2bf(o) : f2h(o);
        }
#pragma unroll
        for (int j = 0; j < WKV_BLK; ++j) {
            kb[j] = kn[j];
            vb[j] = vn[j];
            rb[j] = rn[j];
        }
        kp += nx;
        vp += nx;
        rp += nx;
        op += nx;
    }
    int t0 = nblk * WKV_BLK;
    for (; t0 < T; ++t0) {
        const float y = wkv_step<CONV>(aa, bb, pp, __ldg(kp), __ldg(vp), u, dec);
        const float o = __fmul_rn(h2f(__ldg(rp)), y);
        *op = BF ? f2bf(o) : f2h(o);
        kp += C;
        vp += C;
        rp += C;
        op += C;
    }
    aa_s[idx] = aa;
    bb_s[idx] = bb;
    pp_s[idx] = pp;
}

__global__ void k_embed(const int32_t* __restrict__ tok, int64_t rows, int V, int C,
                        const uint16_t* __restrict__ emb, uint16_t* __restrict__ x) {
    // one 16-byte vector (8 halves) per thread; C % 8 == 0
    const int vpr = C >> 3;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * vpr) return;
    const int64_t row = i / vpr;
    const int j = (int)(i - row * vpr);
    int t = tok[row];
    t = t < 0 ? 0 : (t >= V ? V - 1 : t);
    reinterpret_cast<uint4*>(x)[row * vpr + j] =
        __ldg(reinterpret_cast<const uint4*>(emb) + (int64_t)t * vpr + j);
}

__global__ void k_decay(const float* __restrict__ td, float* __restrict__ out, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = kb_expf(fminf(td[i], 80.0f));
}

// state fp32 [L][5][B][C]: slot 3 (pp) = -1e30, everything else 0
// (rwkv4_step_ref.py:33-37).
__global__ void k_state_init(float* st, int L, int B, int C) {
    const int64_t n = (int64_t)L * 5 * B * C;
    const int64_t per = (int64_t)B * C;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int slot = (int)((i / per) % 5);
        st[i] = (slot == 3) ? -1e30f : 0.0f;
    }
}

// ----------------------------------------------------------------------------
// host launchers (used by forward.cu)
// ----------------------------------------------------------------------------
int launch_embed(const int32_t* tok, int64_t rows, int V, int C, const uint16_t* emb, uint16_t* x,
                 cudaStream_t st) {
    const int64_t n = rows * (C / 8);
    if (n == 0) return KB_OK;
    k_embed<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(tok, rows, V, C, emb, x);
    return launch_status();
}

// Row-wise int8 quantisation of fp16 [R, K] (K % 8 == 0), one warp per row:
// the (r*y) and relu(k)^2 operands of the w8a8 model.
__global__ void __launch_bounds__(256) k_quant_rows(const uint16_t* __restrict__ x, int R, int K,
                                                    int8_t* __restrict__ q,
                                                    float* __restrict__ qs) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= R) return;
    const uint4* src = reinterpret_cast<const uint4*>(x + row * K);
    const int n8 = K / 8;
    float m = 0.0f;
    for (int i = lane; i < n8; i += 32) {
        const uint4 u = __ldg(src + i);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 f = __half22float2(h[k]);
            m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
    }
    const float amax = warp_max(m);
    const float inv = q_inv(amax);
    uint2* dst = reinterpret_cast<uint2*>(q + row * K);
    for (int i = lane; i < n8; i += 32) {
        const uint4 u = __ldg(src + i);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
        float f[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 t = __half22float2(h[k]);
            f[2 * k] = t.x;
            f[2 * k + 1] = t.y;
        }
        dst[i] = make_uint2(pack4(q8(f[0], inv), q8(f[1], inv), q8(f[2], inv), q8(f[3], inv)),
                            pack4(q8(f[4], inv), q8(f[5], inv), q8(f[6], inv), q8(f[7], inv)));
    }
    if (lane == 0) qs[row] = q_factor(amax);
}

// Per-output-channel weight quantisation of fp16 [N, K], one warp per row:
// s = fp16(amax / 127), q = clamp(rint(w / s), -127, 127).
__global__ void __launch_bounds__(256) k_quant_weight(const uint16_t* __restrict__ w, int N, int K,
                                                      int8_t* __restrict__ q,
                                                      uint16_t* __restrict__ scale) {
    const int lane = threadIdx.x & 31;
    const int64_t n = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (n >= N) return;
    const uint16_t* src = w + n * K;
    float m = 0.0f;
    for (int i = lane; i < K; i += 32) m = fmaxf(m, fabsf(h2f(src[i])));
    const float amax = warp_max(m);
    const uint16_t sh = f2h(__fdiv_rn(amax, 127.0f));
    const float s = h2f(sh);
    for (int i = lane; i < K; i += 32) {
        const float r = s > 0.0f ? rintf(__fdiv_rn(h2f(src[i]), s)) : 0.0f;
        q[n * K + i] = (int8_t)fminf(fmaxf(r, -127.0f), 127.0f);
    }
    if (lane == 0) scale[n] = sh;
}

int launch_quant_rows(const uint16_t* x, int R, int K, int8_t* q, float* scale, cudaStream_t st) {
    if (R == 0) return KB_OK;
    if (K % 8) return KB_ERR_SHAPE;
    k_quant_rows<<<(R + 7) / 8, 256, 0, st>>>(x, R, K, q, scale);
    return launch_status();
}

// ---------------------------------------------------------------------------
// LayerNorm + token-shift mix over tiles of consecutive rows (fp16 / bf16
// outputs, C = 32 EPL <= 1024).  A tile's rows are contiguous in memory, so
// one 1-D bulk copy brings them (and the row before the tile) into shared
// memory; a persistent CTA (as many per SM as registers and shared memory
// allow, the grid sized by the occupancy query) walks a contiguous run of
// tiles and double-buffers them on an mbarrier, so the next tile streams in
// while this one is computed.  Phase 1: each warp takes row pairs and
// computes their LayerNorm exactly as ln_warp_h2x2 does (same lane order and
// butterfly), writing the fp16 result back in place.  The row before a tile
// (the token-shift input of its first row) is the previous tile's last row,
// whose LayerNorm the CTA keeps from that tile; only a run's first tile
// normalises it again.  Phase 2: the mixes, one 16-byte chunk per thread at
// a time, coalesced across the CTA.
// ---------------------------------------------------------------------------
#ifndef KB_LNT_RT
#define KB_LNT_RT 16
#endif
#ifndef KB_LNT_CAP
#define KB_LNT_CAP 8
#endif
constexpr int LNT_WARPS = 8;
__device__ int g_ln_error = 0;

template <int EPL>
struct LnTile {
    static constexpr int C = 32 * EPL;
    static constexpr int RT = EPL <= 24 ? KB_LNT_RT : KB_LNT_RT / 2;  // rows per tile
    static constexpr uint32_t ROW = (uint32_t)C * 2;     // bytes per fp16 row
    static constexpr uint32_t BUF = (RT + 1) * ROW;      // slot 0: the row before
    // two buffers + the carried row + barriers + align
    static constexpr size_t SMEM = 2 * BUF + ROW + 64 + 128;
    // resident CTAs per SM the register budget is sized for
    static constexpr int MINB = EPL <= 24 ? 3 : 2;
};

template <int NMIX, int EPL>
__global__ void __launch_bounds__(LNT_WARPS * 32, LnTile<EPL>::MINB)
    k_ln_mix_tile(const uint16_t* __restrict__ x, int B, int T, const float* __restrict__ lw,
                  const float* __restrict__ lb, MixArgs ma, const float* __restrict__ state_in,
                  float* __restrict__ state_out, uint16_t* __restrict__ xx_out) {
    using L = LnTile<EPL>;
    constexpr int C = L::C, RT = L::RT, H = EPL / 2, CH = C / 8;
    extern __shared__ unsigned char lnt_raw[];
    unsigned char* smem = lnt_raw + ((128u - (tc::smem_addr(lnt_raw) & 127u)) & 127u);
    unsigned char* carry = smem + 2 * L::BUF;  // LN of the last row of this CTA's previous tile
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * L::BUF + L::ROW);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t rows = (int64_t)B * T;
    const int64_t tiles = (rows + RT - 1) / RT;
    // a contiguous run of tiles per CTA: the row before a tile is the last
    // row of the tile before it, already normalised by this CTA
    const int64_t t_begin = (int64_t)blockIdx.x * tiles / gridDim.x;
    const int64_t t_end = (int64_t)(blockIdx.x + 1) * tiles / gridDim.x;
    if (t_begin >= t_end) return;
    // rows [r0 - 1, r0 + n) of tile `tile` into buffer `bi` (slot 0 = r0 - 1)
    auto issue = [&](int64_t tile, int bi) {
        const int64_t r0 = tile * RT;
        const int64_t n = rows - r0 < RT ? rows - r0 : RT;
        const int64_t first = r0 > 0 ? r0 - 1 : 0;
        const uint32_t bytes = (uint32_t)((r0 + n - first) * L::ROW);
        unsigned char* dst = smem + bi * L::BUF + (r0 > 0 ? 0 : L::ROW);
        tc::mbar_expect_tx(&full[bi], bytes);
        tc::bulk_load(dst, x + first * C, bytes, &full[bi]);
    };
    if (threadIdx.x == 0) {
        tc::mbar_init(&full[0], 1);
        tc::mbar_init(&full[1], 1);
        tc::fence_barrier_init();
        issue(t_begin, 0);
    }
    __syncthreads();
    int it = 0;
    bool carried = false;  // `carry` holds the LN of row r0 - 1 of this tile
    for (int64_t tile = t_begin; tile < t_end; ++tile, ++it) {
        const int bi = it & 1;
        if (threadIdx.x == 0 && tile + 1 < t_end) {
            tc::fence_proxy_async_smem();  // this buffer's generic accesses (two tiles ago)
            issue(tile + 1, bi ^ 1);
        }
        if (!tc::mbar_wait(&full[bi], (uint32_t)(it >> 1) & 1u)) {
            // bounded wait expired: report, let the other buffer's copy (if
            // any) land, and leave
            if (threadIdx.x == 0) {
                atomicExch(&g_ln_error, 1);
                if (tile + 1 < t_end) tc::mbar_wait(&full[bi ^ 1], (uint32_t)((it + 1) >> 1) & 1u);
            }
            return;
        }
        unsigned char* buf = smem + bi * L::BUF;
        const int64_t r0 = tile * RT;
        const int n = (int)(rows - r0 < RT ? rows - r0 : RT);
        const bool need_prev = NMIX > 0 && r0 > 0 && (r0 % T) != 0;
        // ---- phase 1: LayerNorm of each row, in place -----------------------
        for (int pr = warp; pr < (n + 1) / 2; pr += LNT_WARPS) {
            uint32_t* ra = reinterpret_cast<uint32_t*>(buf + (1 + 2 * pr) * L::ROW);
            uint32_t* rb = reinterpret_cast<uint32_t*>(buf + (2 + 2 * pr) * L::ROW);
            const bool hasb = 2 * pr + 1 < n;
            uint32_t va[H], vb[H], oa[H], ob[H];
#pragma unroll
            for (int j = 0; j < EPL / 8; ++j) {
                const uint4 qa = reinterpret_cast<const uint4*>(ra)[j * 32 + lane];
                va[4 * j] = qa.x; va[4 * j + 1] = qa.y; va[4 * j + 2] = qa.z; va[4 * j + 3] = qa.w;
                uint4 qb = make_uint4(0u, 0u, 0u, 0u);
                if (hasb) qb = reinterpret_cast<const uint4*>(rb)[j * 32 + lane];
                vb[4 * j] = qb.x; vb[4 * j + 1] = qb.y; vb[4 * j + 2] = qb.z; vb[4 * j + 3] = qb.w;
            }
            ln_warp_h2x2<EPL>(va, vb, C, lane, lw, lb, oa, ob);
#pragma unroll
            for (int j = 0; j < EPL / 8; ++j) {
                reinterpret_cast<uint4*>(ra)[j * 32 + lane] =
                    make_uint4(oa[4 * j], oa[4 * j + 1], oa[4 * j + 2], oa[4 * j + 3]);
                if (hasb)
                    reinterpret_cast<uint4*>(rb)[j * 32 + lane] =
                        make_uint4(ob[4 * j], ob[4 * j + 1], ob[4 * j + 2], ob[4 * j + 3]);
            }
        }
        if (need_prev && carried) {
            // slot 0 <- the carried row (bulk copy landed: plain writes now)
            for (int c = threadIdx.x; c < CH; c += LNT_WARPS * 32)
                reinterpret_cast<uint4*>(buf)[c] = reinterpret_cast<const uint4*>(carry)[c];
        } else if (need_prev && warp == (((n + 1) / 2) % LNT_WARPS)) {  // the least loaded warp
            uint32_t* rp = reinterpret_cast<uint32_t*>(buf);
            uint32_t vp[H], op[H];
#pragma unroll
            for (int j = 0; j < EPL / 8; ++j) {
                const uint4 q = reinterpret_cast<const uint4*>(rp)[j * 32 + lane];
                vp[4 * j] = q.x; vp[4 * j + 1] = q.y; vp[4 * j + 2] = q.z; vp[4 * j + 3] = q.w;
            }
            ln_warp_h2<EPL>(vp, C, lane, lw, lb, op);
#pragma unroll
            for (int j = 0; j < EPL / 8; ++j)
                reinterpret_cast<uint4*>(rp)[j * 32 + lane] =
                    make_uint4(op[4 * j], op[4 * j + 1], op[4 * j + 2], op[4 * j + 3]);
        }
        __syncthreads();
        // ---- phase 2: token-shift mixes, xx / state outputs --------------------
        const int b0 = (int)(r0 / T), t0 = (int)(r0 - (int64_t)b0 * T);
        if (n == RT && tile + 1 < t_end)  // the next tile's row before it
            for (int c = threadIdx.x; c < CH; c += LNT_WARPS * 32)
                reinterpret_cast<uint4*>(carry)[c] = reinterpret_cast<const uint4*>(buf + RT * L::ROW)[c];
        carried = n == RT && tile + 1 < t_end;
        for (int q = threadIdx.x; q < n * CH; q += LNT_WARPS * 32) {
            const int r = q / CH, ch = q - r * CH;
            const int64_t g = r0 + r;
            int b = b0, t = t0 + r;
            if (t >= T) {
                b += t / T;
                t %= T;
            }
            const uint4 cq = reinterpret_cast<const uint4*>(buf + (1 + r) * L::ROW)[ch];
            const uint32_t cu[4] = {cq.x, cq.y, cq.z, cq.w};
            if (NMIX > 0) {
                float pf[8];
                if (t == 0) {
                    if (state_in) {
                        const float4* p4 = reinterpret_cast<const float4*>(state_in + (int64_t)b * C) + 2 * ch;
                        const float4 a = p4[0], c = p4[1];
                        pf[0] = a.x; pf[1] = a.y; pf[2] = a.z; pf[3] = a.w;
                        pf[4] = c.x; pf[5] = c.y; pf[6] = c.z; pf[7] = c.w;
                    } else {
#pragma unroll
                        for (int k = 0; k < 8; ++k) pf[k] = 0.0f;
                    }
                } else {
                    const uint4 pq = reinterpret_cast<const uint4*>(buf + r * L::ROW)[ch];
                    const uint32_t pu[4] = {pq.x, pq.y, pq.z, pq.w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float2 f = h2f2(pu[k]);
                        pf[2 * k] = f.x;
                        pf[2 * k + 1] = f.y;
                    }
                }
#pragma unroll
                for (int m = 0; m < NMIX; ++m) {
                    const float4* m4 = reinterpret_cast<const float4*>(ma.mix[m]) + 2 * ch;
                    const float4 m0 = __ldg(m4), m1 = __ldg(m4 + 1);
                    const float mk[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
                    uint32_t o[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float2 f = h2f2(cu[k]);
                        const float k0 = mk[2 * k], k1 = mk[2 * k + 1];
                        const float a0 = __fmaf_rn(f.x, k0, __fmul_rn(pf[2 * k], __fsub_rn(1.0f, k0)));
                        const float a1 = __fmaf_rn(f.y, k1, __fmul_rn(pf[2 * k + 1], __fsub_rn(1.0f, k1)));
                        o[k] = ma.bf16 ? f2bf2(a0, a1) : f2h2(a0, a1);
                    }
                    reinterpret_cast<uint4*>(ma.out[m] + g * C)[ch] = make_uint4(o[0], o[1], o[2], o[3]);
                }
            }
            if (xx_out) {
                uint4 o;
                if (ma.bf16) {
                    const float2 a = h2f2(cu[0]), c = h2f2(cu[1]), d = h2f2(cu[2]), e = h2f2(cu[3]);
                    o = make_uint4(f2bf2(a.x, a.y), f2bf2(c.x, c.y), f2bf2(d.x, d.y), f2bf2(e.x, e.y));
                } else {
                    o = cq;
                }
                reinterpret_cast<uint4*>(xx_out + g * C)[ch] = o;
            }
            if (state_out && t == T - 1) {
                float4* s4 = reinterpret_cast<float4*>(state_out + (int64_t)b * C) + 2 * ch;
                const float2 a = h2f2(cu[0]), c = h2f2(cu[1]), d = h2f2(cu[2]), e = h2f2(cu[3]);
                s4[0] = make_float4(a.x, a.y, c.x, c.y);
                s4[1] = make_float4(d.x, d.y, e.x, e.y);
            }
        }
        __syncthreads();  // the buffer is refilled two tiles on
    }
}

template <int NMIX, int EPL>
int launch_ln_tile(int B, int T, cudaStream_t st, const uint16_t* x, const float* lw,
                   const float* lb, const MixArgs& ma, const float* state_in, float* state_out,
                   uint16_t* xx_out) {
    using L = LnTile<EPL>;
    static std::atomic<unsigned long long> done{0};
    const cudaError_t e = once_per_device(done, [] {
        return cudaFuncSetAttribute(k_ln_mix_tile<NMIX, EPL>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::SMEM);
    });
    if (e != cudaSuccess) {
        set_cuda_error(e);
        return KB_ERR_CUDA;
    }
    const int64_t tiles = ((int64_t)B * T + L::RT - 1) / L::RT;
    int sms = 0, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // resident CTAs per SM (registers and shared memory), measured once
    static std::atomic<int> occ[64];
    int per_sm = dev >= 0 && dev < 64 ? occ[dev].load() : 0;
    if (per_sm <= 0) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_ln_mix_tile<NMIX, EPL>,
                                                          LNT_WARPS * 32, L::SMEM) != cudaSuccess ||
            per_sm <= 0) {
            cudaGetLastError();
            per_sm = 1;
        }
        if (dev >= 0 && dev < 64) occ[dev].store(per_sm);
    }
    const int64_t cap = (int64_t)(sms > 0 ? sms : 148) * (per_sm < KB_LNT_CAP ? per_sm : KB_LNT_CAP);
    const int grid = (int)(tiles < cap ? tiles : cap);
    k_ln_mix_tile<NMIX, EPL><<<grid, LNT_WARPS * 32, L::SMEM, st>>>(x, B, T, lw, lb, ma, state_in,
                                                                   state_out, xx_out);
    return KB_OK;
}

template <int NMIX>
static int ln_mix_epl(int epl, int blocks, int rpw, cudaStream_t st, const uint16_t* x, int B, int T, int C,
                      const float* lw, const float* lb, const MixArgs& ma, const float* state_in,
                      float* state_out, uint16_t* xx_out) {
#define KB_LN_CASE(E)                                                                           \
    case E:                                                                                     \
        k_ln_mix<NMIX, E><<<blocks, LN_WARPS * 32, 0, st>>>(x, B, T, C, lw, lb, ma, state_in,   \
                                                            state_out, xx_out, rpw);            \
        return KB_OK;
    switch (epl) {
        KB_LN_CASE(4) KB_LN_CASE(8) KB_LN_CASE(16) KB_LN_CASE(24) KB_LN_CASE(32) KB_LN_CASE(48)
        KB_LN_CASE(64)
        default:
            return KB_ERR_SHAPE;
    }
#undef KB_LN_CASE
}

int launch_ln_mix(int nmix, const uint16_t* x, int B, int T, int C, const float* lw,
                  const float* lb, const MixArgs& ma, const float* state_in, float* state_out,
                  uint16_t* xx_out, cudaStream_t st) {
    if (C % 32) return KB_ERR_SHAPE;
    const int epl = C / 32;
    const int64_t rows = (int64_t)B * T;
    // strips of 4 rows once there are enough rows to fill the GPU many times
    const int rpw = rows >= (int64_t)148 * LN_WARPS * 64 ? 4 : 1;
    const int blocks = (int)((rows + LN_WARPS * rpw - 1) / (LN_WARPS * rpw));
    int rc;
    if (epl >= LNS_MIN_EPL && C % 256 == 0 && C <= LNS_MAX_C) {  // staged variant
        const int sb = (int)((rows + LNS_WARPS * rpw - 1) / (LNS_WARPS * rpw));
        switch (nmix) {
            case 0: k_ln_mix_stream<0><<<sb, LNS_WARPS * 32, 0, st>>>(x, B, T, C, lw, lb, ma, state_in, state_out, xx_out, rpw); break;
            case 2: k_ln_mix_stream<2><<<sb, LNS_WARPS * 32, 0, st>>>(x, B, T, C, lw, lb, ma, state_in, state_out, xx_out, rpw); break;
            case 3: k_ln_mix_stream<3><<<sb, LNS_WARPS * 32, 0, st>>>(x, B, T, C, lw, lb, ma, state_in, state_out, xx_out, rpw); break;
            default: return KB_ERR_ARG;
        }
        return launch_status();
    }
    const bool quant = ma.q[0] || ma.q[1] || ma.q[2];
    if (KB_LN_TILE && !quant && epl % 8 == 0 && epl <= 32) {
#define KB_LNT_CASE(N, E)                                                                       \
    case E:                                                                                     \
        rc = launch_ln_tile<N, E>(B, T, st, x, lw, lb, ma, state_in, state_out, xx_out);        \
        break;
#define KB_LNT_NMIX(N)                                                                          \
    case N:                                                                                     \
        switch (epl) {                                                                          \
            KB_LNT_CASE(N, 8) KB_LNT_CASE(N, 16) KB_LNT_CASE(N, 24) KB_LNT_CASE(N, 32)          \
            default: return KB_ERR_SHAPE;                                                       \
        }                                                                                       \
        break;
        switch (nmix) {
            KB_LNT_NMIX(0) KB_LNT_NMIX(2) KB_LNT_NMIX(3)
            default: return KB_ERR_ARG;
        }
#undef KB_LNT_NMIX
#undef KB_LNT_CASE
        if (rc != KB_OK) return rc;
        return launch_status();
    }
    switch (nmix) {
        case 0: rc = ln_mix_epl<0>(epl, blocks, rpw, st, x, B, T, C, lw, lb, ma, state_in, state_out, xx_out); break;
        case 2: rc = ln_mix_epl<2>(epl, blocks, rpw, st, x, B, T, C, lw, lb, ma, state_in, state_out, xx_out); break;
        case 3: rc = ln_mix_epl<3>(epl, blocks, rpw, st, x, B, T, C, lw, lb, ma, state_in, state_out, xx_out); break;
        default: return KB_ERR_ARG;
    }
    if (rc != KB_OK) return rc;
    return launch_status();
}

int launch_wkv(int conv, int B, int T, int C, const float* k, const float* v, const uint16_t* r,
               const float* decay, const float* first, float* aa, float* bb, float* pp,
               uint16_t* ry, cudaStream_t st, bool ry_bf16) {
    const int n = B * C;
    const int grid = (n + 127) / 128;
#define KB_WKV(CV, BFV) \
    k_wkv<CV, BFV><<<grid, 128, 0, st>>>(B, T, C, k, v, r, decay, first, aa, bb, pp, ry)
    if (conv == KB_WKV_STEP_REF) {
        if (ry_bf16) KB_WKV(KB_WKV_STEP_REF, true);
        else KB_WKV(KB_WKV_STEP_REF, false);
    } else {
        if (ry_bf16) KB_WKV(KB_WKV_PRODUCTION, true);
        else KB_WKV(KB_WKV_PRODUCTION, false);
    }
#undef KB_WKV
    return launch_status();
}

int read_ln_error(int reset) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_ln_error, sizeof(int)) != cudaSuccess) return -1;
    if (reset && v) {
        const int z = 0;
        cudaMemcpyToSymbol(g_ln_error, &z, sizeof(int));
    }
    return v;
}

int launch_state_init(float* st, int L, int B, int C, cudaStream_t s) {
    const int64_t n = (int64_t)L * 5 * B * C;
    if (n == 0) return KB_OK;
    const int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
    k_state_init<<<grid, 256, 0, s>>>(st, L, B, C);
    return launch_status();
}

}  // namespace kb

extern "C" int kb_quantize_weight(const uint16_t* w, int N, int K, int8_t* q, uint16_t* scale,
                                  void* stream) {
    if (!w || !q || !scale || N <= 0 || K <= 0) return KB_ERR_ARG;
    kb::k_quant_weight<<<(N + 7) / 8, 256, 0, kb::as_stream(stream)>>>(w, N, K, q, scale);
    return kb::launch_status();
}

extern "C" int kb_quantize_rows(const uint16_t* x, int R, int K, int8_t* q, float* scale,
                                void* stream) {
    if (!x || !q || !scale || R < 0 || K <= 0) return KB_ERR_ARG;
    if (!kb::aligned16(x) || ((uintptr_t)q & 7u)) return KB_ERR_ALIGN;
    return kb::launch_quant_rows(x, R, K, q, scale, kb::as_stream(stream));
}

extern "C" int kb_prepare_decay(const float* td, float* out, int n, void* stream) {
    if (!td || !out || n < 0) return KB_ERR_ARG;
    if (n == 0) return KB_OK;
    kb::k_decay<<<(n + 255) / 256, 256, 0, kb::as_stream(stream)>>>(td, out, n);
    return kb::launch_status();
}
