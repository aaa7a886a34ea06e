// RWKV-4 row-local and recurrent kernels: embedding gather, LayerNorm fused
// with the token-shift mix, the WKV recurrence, decay preparation, state init.
//
// Row-local maths is fixed by the row alone (fixed block size, fixed
// reduction tree), and the token-shift input of the first row of a window is
// the carried state, so a window of T rows produces exactly the bits of T
// single-row steps.  That is what lets the stepped decoder reproduce the
// packed encoder's logits bit for bit.
#include "kb_common.cuh"
#include "rwkv_ops.cuh"

namespace kb {

constexpr int LN_NT = 256;          // fixed: part of the reduction order
constexpr float LN_EPS = 1e-5f;     // F.layer_norm default (rwkv4_step_ref.py:57)

__device__ __forceinline__ float ln_block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    if (lane == 0) red[w] = v;
    __syncthreads();
    float x = (lane < LN_NT / 32) ? red[lane] : 0.0f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) x = __fadd_rn(x, __shfl_xor_sync(0xffffffffu, x, off));
    __syncthreads();
    return x;
}

// LayerNorm of one row into registers, rounded to fp16 precision (the
// reference keeps xx in the fp16 activation dtype, rwkv4_step_ref.py:57-61).
template <int LN_EPT>
__device__ __forceinline__ void ln_row(const uint16_t* __restrict__ x, int C,
                                       const float* __restrict__ w, const float* __restrict__ b,
                                       float* red, float (&out)[LN_EPT]) {
    const int tid = threadIdx.x;
    float v[LN_EPT];
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < LN_EPT; ++j) {
        const int c = j * LN_NT + tid;
        v[j] = (c < C) ? h2f(x[c]) : 0.0f;
        s = __fadd_rn(s, v[j]);
    }
    const float mean = __fdiv_rn(ln_block_sum(s, red), (float)C);
    float q = 0.0f;
#pragma unroll
    for (int j = 0; j < LN_EPT; ++j) {
        const int c = j * LN_NT + tid;
        const float d = (c < C) ? __fsub_rn(v[j], mean) : 0.0f;
        q = __fmaf_rn(d, d, q);
    }
    const float var = __fdiv_rn(ln_block_sum(q, red), (float)C);
    const float rstd = __frsqrt_rn(__fadd_rn(var, LN_EPS));
#pragma unroll
    for (int j = 0; j < LN_EPT; ++j) {
        const int c = j * LN_NT + tid;
        if (c < C) {
            const float y = __fmaf_rn(__fmul_rn(__fsub_rn(v[j], mean), rstd), w[c], b[c]);
            out[j] = __half2float(__float2half_rn(y));
        } else {
            out[j] = 0.0f;
        }
    }
}

// LN + token-shift mix over a run of rows of one stream.
//   grid = (ceil(T / rows_per_cta), B); row index = b*T + t.
//   prev(t0) = state_in[b] if t0 == 0 else LN(x[t0-1]) (recomputed).
//   mix_j = xx * m_j + prev * (1 - m_j)   (rwkv4_step_ref.py:59-61)
// The last row's xx goes to state_out[b].  xx_out (optional) receives xx.
template <int NMIX, int LN_EPT>
__global__ void __launch_bounds__(LN_NT) k_ln_mix(const uint16_t* __restrict__ x, int T, int C,
                                                  int rows_per_cta, const float* __restrict__ lw,
                                                  const float* __restrict__ lb, MixArgs ma,
                                                  const float* __restrict__ state_in,
                                                  float* __restrict__ state_out,
                                                  uint16_t* __restrict__ xx_out) {
    __shared__ float red[LN_NT / 32];
    const int b = blockIdx.y;
    const int t0 = blockIdx.x * rows_per_cta;
    if (t0 >= T) return;
    const int t1 = min(t0 + rows_per_cta, T);
    const int tid = threadIdx.x;
    const int64_t row0 = (int64_t)b * T;

    float prev[LN_EPT], cur[LN_EPT];
    if (NMIX == 0) {
#pragma unroll
        for (int j = 0; j < LN_EPT; ++j) prev[j] = 0.0f;
    } else if (t0 == 0) {
#pragma unroll
        for (int j = 0; j < LN_EPT; ++j) {
            const int c = j * LN_NT + tid;
            prev[j] = (c < C && state_in) ? state_in[(int64_t)b * C + c] : 0.0f;
        }
    } else {
        ln_row(x + (row0 + t0 - 1) * C, C, lw, lb, red, prev);
    }
    float mk[NMIX > 0 ? NMIX : 1][LN_EPT];
#pragma unroll
    for (int m = 0; m < NMIX; ++m)
#pragma unroll
        for (int j = 0; j < LN_EPT; ++j) {
            const int c = j * LN_NT + tid;
            mk[m][j] = (c < C) ? ma.mix[m][c] : 0.0f;
        }

    for (int t = t0; t < t1; ++t) {
        const int64_t row = row0 + t;
        ln_row(x + row * C, C, lw, lb, red, cur);
#pragma unroll
        for (int j = 0; j < LN_EPT; ++j) {
            const int c = j * LN_NT + tid;
            if (c < C) {
                if (xx_out) xx_out[row * C + c] = f2h(cur[j]);
#pragma unroll
                for (int m = 0; m < NMIX; ++m) {
                    const float one_m = __fsub_rn(1.0f, mk[m][j]);
                    const float y = __fmaf_rn(cur[j], mk[m][j], __fmul_rn(prev[j], one_m));
                    ma.out[m][row * C + c] = f2h(y);
                }
            }
            prev[j] = cur[j];
        }
        if (t == T - 1 && state_out) {
#pragma unroll
            for (int j = 0; j < LN_EPT; ++j) {
                const int c = j * LN_NT + tid;
                if (c < C) state_out[(int64_t)b * C + c] = cur[j];
            }
        }
    }
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
template <int CONV>
__global__ void __launch_bounds__(128) k_wkv(int B, int T, int C, const float* __restrict__ k,
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
#pragma unroll 4
    for (int t = 0; t < T; ++t) {
        const int64_t o = base + (int64_t)t * C;
        const float kt = k[o];
        const float vt = v[o];
        const float rt = h2f(r[o]);
        float e1, e2;
        if (CONV == KB_WKV_STEP_REF) {
            const float ww = __fadd_rn(pp, u);
            const float p = fmaxf(ww, kt);
            e1 = __expf(__fsub_rn(ww, p));
            e2 = __expf(__fsub_rn(kt, p));
        } else {
            const float ww = __fadd_rn(u, kt);
            const float p = fmaxf(pp, ww);
            e1 = __expf(__fsub_rn(pp, p));
            e2 = __expf(__fsub_rn(ww, p));
        }
        const float num = __fmaf_rn(e1, aa, __fmul_rn(e2, vt));
        const float den = __fmaf_rn(e1, bb, e2);
        const float y = __fdiv_rn(num, den);
        ry[o] = f2h(__fmul_rn(rt, y));
        const float ww2 = __fsub_rn(pp, dec);
        const float p2 = fmaxf(ww2, kt);
        const float f1 = __expf(__fsub_rn(ww2, p2));
        const float f2 = __expf(__fsub_rn(kt, p2));
        aa = __fmaf_rn(f1, aa, __fmul_rn(f2, vt));
        bb = __fmaf_rn(f1, bb, f2);
        pp = p2;
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

template <int NMIX>
static void ln_mix_ept(int ept, dim3 grid, cudaStream_t st, const uint16_t* x, int T, int C,
                       int rpc, const float* lw, const float* lb, const MixArgs& ma,
                       const float* state_in, float* state_out, uint16_t* xx_out) {
#define KB_LN_CASE(E)                                                                         \
    case E:                                                                                   \
        k_ln_mix<NMIX, E><<<grid, LN_NT, 0, st>>>(x, T, C, rpc, lw, lb, ma, state_in,        \
                                                   state_out, xx_out);                        \
        break;
    switch (ept) {
        KB_LN_CASE(1) KB_LN_CASE(2) KB_LN_CASE(3) KB_LN_CASE(4) KB_LN_CASE(8) KB_LN_CASE(16)
    }
#undef KB_LN_CASE
}

int launch_ln_mix(int nmix, const uint16_t* x, int B, int T, int C, const float* lw,
                  const float* lb, const MixArgs& ma, const float* state_in, float* state_out,
                  uint16_t* xx_out, cudaStream_t st) {
    const int need = (C + LN_NT - 1) / LN_NT;
    const int ept = need <= 4 ? need : (need <= 8 ? 8 : 16);
    if (need > 16) return KB_ERR_SHAPE;
    const int rpc = T >= 64 ? 16 : (T >= 8 ? 4 : 1);
    dim3 grid((T + rpc - 1) / rpc, B);
    switch (nmix) {
        case 0: ln_mix_ept<0>(ept, grid, st, x, T, C, rpc, lw, lb, ma, state_in, state_out, xx_out); break;
        case 2: ln_mix_ept<2>(ept, grid, st, x, T, C, rpc, lw, lb, ma, state_in, state_out, xx_out); break;
        case 3: ln_mix_ept<3>(ept, grid, st, x, T, C, rpc, lw, lb, ma, state_in, state_out, xx_out); break;
        default: return KB_ERR_ARG;
    }
    return launch_status();
}

int launch_wkv(int conv, int B, int T, int C, const float* k, const float* v, const uint16_t* r,
               const float* decay, const float* first, float* aa, float* bb, float* pp,
               uint16_t* ry, cudaStream_t st) {
    const int n = B * C;
    const int grid = (n + 127) / 128;
    if (conv == KB_WKV_STEP_REF)
        k_wkv<KB_WKV_STEP_REF><<<grid, 128, 0, st>>>(B, T, C, k, v, r, decay, first, aa, bb, pp, ry);
    else
        k_wkv<KB_WKV_PRODUCTION><<<grid, 128, 0, st>>>(B, T, C, k, v, r, decay, first, aa, bb, pp, ry);
    return launch_status();
}

int launch_state_init(float* st, int L, int B, int C, cudaStream_t s) {
    const int64_t n = (int64_t)L * 5 * B * C;
    if (n == 0) return KB_OK;
    const int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
    k_state_init<<<grid, 256, 0, s>>>(st, L, B, C);
    return launch_status();
}

}  // namespace kb

extern "C" int kb_prepare_decay(const float* td, float* out, int n, void* stream) {
    if (!td || !out || n < 0) return KB_ERR_ARG;
    if (n == 0) return KB_OK;
    kb::k_decay<<<(n + 255) / 256, 256, 0, kb::as_stream(stream)>>>(td, out, n);
    return kb::launch_status();
}
