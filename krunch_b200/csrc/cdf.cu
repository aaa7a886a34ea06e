// logits -> softmax -> integer CDF, one CTA per row.
//
// Spec (krunch_ac/cdf.py:22-74, krunch_ac/cuda/det_softmax_cdf.cu:62-185):
//   p_i    = softmax(logits)_i
//   c_i    = floor(p_i * (T - V)) + 1           (MIN_PROB = 1)
//   c_amax += T - sum(c)                         (argmax of p, smallest index on ties)
//   cdf    = [0, cumsum(c)]
//
// The softmax follows softmax_stats.cuh: per 32-column subtile u a max m_u
// and fp16 numerators e_i = e^(x_i - m_u); the only floating-point reduction,
// the normaliser (M, S), merges the subtile partials in a fixed order.  With
// gs_u = (e^(m_u - M) / S) * (T - V) a count is c_i = floor(e_i * gs_u) + 1,
// and the argmax of q_i = e_i * gs_u (smallest index on ties) is the first
// e_i == 1 in the first subtile with the largest gs_u: every subtile's max has
// e = 1 exactly, and q_i < gs_u whenever e_i < 1 (the largest fp16 below 1 is
// 1 - 2^-11), so no per-element comparison is needed.  The head GEMM hands
// over e_i and the partials; given raw logits the kernel derives both.
// Everything is explicitly rounded or integer, so a row's CDF is
// bit-identical for any number of rows, any launch and any GPU, and the C
// restatement in oracle/ reproduces it bit for bit.
//
// Element pass: warp w of 16 owns the contiguous range [w*Lw, (w+1)*Lw)
// (Lw a multiple of 256); per step each lane takes 8 consecutive values with
// one 16-byte load.  Ranges are in index order, which gives the decoder its
// prefix sums.
//
// Modes: COUNTS / CDF write [rows, V+1] int32 (reference contract);
// LOHI writes only the (cdf[s], cdf[s+1]) pair of the row's symbol (the
// compress hot path — the [rows, V+1] CDF is never materialised);
// DECODE runs the range-decoder step for stream `row` in the same CTA.
// The probability-input variant (kb_cdf_from_probs) keeps a per-thread
// segmented sum (k_cdf_probs).
#include <float.h>
#include <limits.h>

#include <atomic>

#include "coder.cuh"
#include "profile.cuh"
#include "softmax_stats.cuh"

namespace kb {

constexpr int CDF_NT = 512;
constexpr int CDF_NW = CDF_NT / 32;
// 256-element steps per warp range: V <= CDF_NW * 256 * CT_STEPS
constexpr int CT_STEPS = 16;
constexpr int MODE_COUNTS = KB_CDF_COUNTS;
constexpr int MODE_CDF = KB_CDF_CDF;
constexpr int MODE_LOHI = KB_CDF_LOHI;
constexpr int MODE_DECODE = 3;
constexpr int MAX_SUB = 65536 / SUBTILE;

struct CdfRed {
    float f[CDF_NW];
    int i[CDF_NW];
    float v[CDF_NW];
    int i2[CDF_NW];
};

// Fixed-tree float sum: butterfly in each warp, then the same butterfly over
// the CDF_NW warp partials (zero padded to 32).
__device__ __forceinline__ float block_sum_f(float v, CdfRed& r) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    if (lane == 0) r.f[w] = v;
    __syncthreads();
    float x = (lane < CDF_NW) ? r.f[lane] : 0.0f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) x = __fadd_rn(x, __shfl_xor_sync(0xffffffffu, x, off));
    __syncthreads();
    return x;
}

__device__ __forceinline__ int block_sum_i(int v, CdfRed& r) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (lane == 0) r.i[w] = v;
    __syncthreads();
    int x = (lane < CDF_NW) ? r.i[lane] : 0;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
    __syncthreads();
    return x;
}

// Two integer sums in one reduction (integer addition: any order, same value).
__device__ __forceinline__ void block_sum_i2(int& a, int& b, CdfRed& r) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, off);
        b += __shfl_xor_sync(0xffffffffu, b, off);
    }
    if (lane == 0) {
        r.i[w] = a;
        r.i2[w] = b;
    }
    __syncthreads();
    int x = (lane < CDF_NW) ? r.i[lane] : 0, y = (lane < CDF_NW) ? r.i2[lane] : 0;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        x += __shfl_xor_sync(0xffffffffu, x, off);
        y += __shfl_xor_sync(0xffffffffu, y, off);
    }
    __syncthreads();
    a = x;
    b = y;
}

// (value desc, index asc) total order: the largest value, smallest index on ties.
__device__ __forceinline__ void am_merge(float& v, int& i, float ov, int oi) {
    if (ov > v || (ov == v && oi < i)) {
        v = ov;
        i = oi;
    }
}

__device__ __forceinline__ int block_argmax(float v, int i, CdfRed& r) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, off);
        const int oi = __shfl_xor_sync(0xffffffffu, i, off);
        am_merge(v, i, ov, oi);
    }
    if (lane == 0) {
        r.v[w] = v;
        r.i2[w] = i;
    }
    __syncthreads();
    float x = (lane < CDF_NW) ? r.v[lane] : -INFINITY;
    int xi = (lane < CDF_NW) ? r.i2[lane] : INT_MAX;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, x, off);
        const int oi = __shfl_xor_sync(0xffffffffu, xi, off);
        am_merge(x, xi, ov, oi);
    }
    __syncthreads();
    return xi;
}

// ---------------------------------------------------------------------------
// probabilities -> CDF (kb_cdf_from_probs): thread t sums its segment
// [t*L, min((t+1)*L, V)) left to right, partials meet in the fixed butterfly;
// p_i = x_i / S, c_i = floor(p_i * (T - V)) + 1, argmax over p_i.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(CDF_NT) k_cdf_probs(const float* __restrict__ probs, int V,
                                                      int bits, int32_t* __restrict__ out) {
    __shared__ CdfRed red;
    __shared__ int s_wsum[CDF_NT];
    const int row = blockIdx.x, tid = threadIdx.x;
    const int L = (V + CDF_NT - 1) / CDF_NT;
    const int a = min(tid * L, V), e = min(a + L, V);
    const int T = 1 << bits;
    const float scale = (float)(T - V);
    const float* x = probs + (int64_t)row * V;
    float st = 0.0f;
    for (int i = a; i < e; ++i) st = __fadd_rn(st, x[i]);
    const float S = fmaxf(block_sum_f(st, red), 1e-30f);
    int cs = 0;
    float bp = -INFINITY;
    int bi = INT_MAX;
    for (int i = a; i < e; ++i) {
        const float p = __fdiv_rn(x[i], S);
        cs += (int)floorf(__fmul_rn(p, scale)) + 1;
        if (p > bp) {
            bp = p;
            bi = i;
        }
    }
    const int amax = block_argmax(bp, bi, red);
    const int deficit = T - block_sum_i(cs, red);
    s_wsum[tid] = cs + ((amax >= a && amax < e) ? deficit : 0);
    __syncthreads();
    if (tid == 0) {  // exclusive prefix over threads (integers, exact)
        int run = 0;
        for (int t = 0; t < CDF_NT; ++t) {
            const int v = s_wsum[t];
            s_wsum[t] = run;
            run += v;
        }
    }
    __syncthreads();
    int run = s_wsum[tid];
    int32_t* o = out + (int64_t)row * (V + 1);
    if (tid == 0) o[0] = 0;
    for (int i = a; i < e; ++i) {
        run += (int)floorf(__fmul_rn(__fdiv_rn(x[i], S), scale)) + 1 + (i == amax ? deficit : 0);
        o[i + 1] = run;
    }
}

// ---------------------------------------------------------------------------
// logits -> CDF / (lo, hi) / decode step
// ---------------------------------------------------------------------------
struct RowShared {
    float2 wpart[CDF_NW];
    float M, inv;
    int amax;
    int csym;
};

// Normaliser (M, 1/S), per-subtile factors gs[u] and the argmax of one row.
// part(u) -> float2 (m_u, s_u); is_one(i) -> true iff e_i == 1.0.
template <class Part, class IsOne>
__device__ __forceinline__ void row_setup(Part part, IsOne is_one, int nsub, float scale,
                                          float* gs, RowShared& rs, CdfRed& red) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    MS acc{-INFINITY, 0.0f};
    for (int u = tid; u < nsub; u += CDF_NT) {
        const float2 p = part(u);
        acc = ms_merge(acc, MS{p.x, p.y});
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc = ms_merge(acc, ms_shfl_xor(acc, off));
    if (lane == 0) rs.wpart[warp] = make_float2(acc.m, acc.s);
    __syncthreads();
    if (warp == 0) {
        MS w{-INFINITY, 0.0f};
        if (lane < CDF_NW) w = MS{rs.wpart[lane].x, rs.wpart[lane].y};
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) w = ms_merge(w, ms_shfl_xor(w, off));
        if (lane == 0) {
            rs.M = w.m;
            rs.inv = __frcp_rn(w.s);
        }
    }
    __syncthreads();
    const float M = rs.M, inv = rs.inv;
    float best = -INFINITY;
    int bu = INT_MAX;
    for (int u = tid; u < nsub; u += CDF_NT) {
        const float g = __fmul_rn(__fmul_rn(kb_expf(__fsub_rn(part(u).x, M)), inv), scale);
        gs[u] = g;
        if (g > best) {
            best = g;
            bu = u;
        }
    }
    const int ustar = block_argmax(best, bu, red);  // contains __syncthreads
    if (warp == 0) {
        const int a = ustar * SUBTILE;  // SUBTILE == 32: one lane per column
        const unsigned b0 = __ballot_sync(0xffffffffu, is_one(a + lane));
        if (lane == 0) rs.amax = a + __ffs(b0) - 1;
    }
    __syncthreads();
}

// Counts of the 8 consecutive elements i0..i0+7 (< lim).
__device__ __forceinline__ int counts8(const float (&e)[8], float g, int i0, int lim, int (&c)[8]) {
    int sum = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        c[k] = (i0 + k < lim) ? (int)floorf(__fmul_rn(e[k], g)) + 1 : 0;
        sum += c[k];
    }
    return sum;
}

// Counts of 8 consecutive in-range elements: floor via the round-down
// conversion (the same value as (int)floorf for these magnitudes).
// SMALL (T - V < 2^23): floor(q) as the low bits of q + 2^23 rounded down,
// which is exact for 0 <= q < 2^23 and stays in the full-rate FP/INT pipes.
template <bool SMALL>
__device__ __forceinline__ int counts8_full(const float (&e)[8], float g, int (&c)[8]) {
    int sum = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float q = __fmul_rn(e[k], g);
        c[k] = (SMALL ? (__float_as_int(__fadd_rd(q, 8388608.0f)) - 0x4B000000)
                      : __float2int_rd(q)) + 1;
        sum += c[k];
    }
    return sum;
}

__device__ __forceinline__ void unpack8(const uint4& q, float (&e)[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&q);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(h[k]);
        e[2 * k] = f.x;
        e[2 * k + 1] = f.y;
    }
}

// Element source: numerators stored (global or shared), 16-byte loads.
struct NumSrc {
    const uint16_t* x;
    int V;
    __device__ __forceinline__ void load8(int i0, int lim, float (&e)[8]) const {
        if (((reinterpret_cast<uintptr_t>(x + i0)) & 15u) == 0 && i0 + 8 <= lim) {
            unpack8(*reinterpret_cast<const uint4*>(x + i0), e);
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) e[k] = (i0 + k < lim) ? h2f(x[i0 + k]) : 0.0f;
        }
    }
    // i0 + 8 <= V and x + i0 16-byte aligned (row starts 16-byte aligned)
    __device__ __forceinline__ void load8_full(int i0, float (&e)[8]) const {
        unpack8(*reinterpret_cast<const uint4*>(x + i0), e);
    }
    __device__ __forceinline__ bool is_one(int i) const {
        return i < V && x[i] == (uint16_t)0x3C00u;
    }
};

// Element source: raw logits; numerators computed against the subtile max.
struct RawSrc {
    const uint16_t* x;
    const float2* part;
    int V;
    __device__ __forceinline__ void load8(int i0, int lim, float (&e)[8]) const {
        const float m = part[i0 / SUBTILE].x;
#pragma unroll
        for (int k = 0; k < 8; ++k)
            e[k] = (i0 + k < lim) ? h2f(exp_rel_f16(h2f(x[i0 + k]), m)) : 0.0f;
    }
    __device__ __forceinline__ void load8_full(int i0, float (&e)[8]) const { load8(i0, i0 + 8, e); }
    __device__ __forceinline__ bool is_one(int i) const {
        return i < V && exp_rel_f16(h2f(x[i]), part[i / SUBTILE].x) == (uint16_t)0x3C00u;
    }
};

// Subtile partials of a raw logits row into smem (softmax_stats.cuh spec).
__device__ __forceinline__ void raw_partials(const uint16_t* x, int V, int nsub, float2* out) {
    for (int u = threadIdx.x; u < nsub; u += CDF_NT) {
        const int a = u * SUBTILE, e = min(a + SUBTILE, V);
        float m = -INFINITY;
        for (int i = a; i < e; ++i) m = fmaxf(m, h2f(x[i]));
        float sum = 0.0f;
        for (int i = a; i < e; ++i) sum = __fadd_rn(sum, h2f(exp_rel_f16(h2f(x[i]), m)));
        out[u] = make_float2(m, sum);
    }
    __syncthreads();
}

// Counts of the 8 elements from i0 (deficit added at the argmax), their sum.
template <class Src>
__device__ __forceinline__ int chunk_counts(const Src& src, const float* gs, int i0, int we,
                                            int amax, int deficit, bool small, int (&c)[8]) {
    int ls = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) c[k] = 0;
    if (i0 < we) {
        float e[8];
        if (gs[i0 / SUBTILE] < 1.0f) {  // cold subtile: every count is 1 (see cdf_row_body)
#pragma unroll
            for (int k = 0; k < 8; ++k) c[k] = i0 + k < we ? 1 : 0;
            ls = min(8, we - i0);
        } else if (i0 + 8 <= we && (reinterpret_cast<uintptr_t>(src.x) & 15u) == 0) {
            src.load8_full(i0, e);
            ls = small ? counts8_full<true>(e, gs[i0 / SUBTILE], c)
                       : counts8_full<false>(e, gs[i0 / SUBTILE], c);
        } else {
            src.load8(i0, we, e);
            ls = counts8(e, gs[i0 / SUBTILE], i0, we, c);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if (i0 + k == amax) c[k] += deficit;
        if (amax >= i0 && amax < i0 + 8) ls += deficit;
    }
    return ls;
}

// Walk the warp's range in 256-element steps: per step each lane's 8 counts
// (deficit added at the argmax) and their warp-inclusive prefix.  f(i0, c,
// ls, excl_in_warp_step, step_total) is called for every step; returning
// true stops the walk.
template <class Src, class F>
__device__ __forceinline__ void walk_counts(const Src& src, const float* gs, int wa, int we,
                                            int amax, int deficit, bool small, F f) {
    const int lane = threadIdx.x & 31;
    for (int base = wa; base < we; base += 256) {
        const int i0 = base + lane * 8;
        int c[8];
        const int ls = chunk_counts(src, gs, i0, we, amax, deficit, small, c);
        int inc = ls;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, inc, off);
            if (lane >= off) inc += y;
        }
        const int total = __shfl_sync(0xffffffffu, inc, 31);
        if (f(i0, c, ls, inc - ls, total)) break;
    }
}

template <int MODE, class Src>
__device__ void cdf_row_body(const Src& src, int V, int bits, const float* gs, RowShared& rs,
                             CdfRed& red, int row, int sym, void* out, const uint8_t* in,
                             int64_t in_bytes, const int64_t* in_offs, uint32_t* states,
                             int32_t* counters, int32_t* out_syms, int32_t* history,
                             int64_t hist_stride) {
    __shared__ int s_wsum[CDF_NW], s_wexcl[CDF_NW], s_owner, s_sym;
    __shared__ uint32_t s_target, s_lo, s_hi;
    // DECODE: count total of every 256-element step of each warp's range
    // (deficit excluded), step k of warp w at s_ct[w][k]
    __shared__ int s_ct[MODE == MODE_DECODE ? CDF_NW * CT_STEPS : 1];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int T = 1 << bits;
    const int Lw = ((V + CDF_NW * 256 - 1) / (CDF_NW * 256)) * 256;
    const int wa = min(warp * Lw, V), we = min(wa + Lw, V);
    const int amax = rs.amax;
    if (MODE == MODE_DECODE && tid == 0) s_target = decode_target(states + 4 * (int64_t)row, bits);

    // ---- element pass: totals (and the prefix below the symbol) ----------
    const bool aligned_row = (reinterpret_cast<uintptr_t>(src.x) & 15u) == 0;
    const bool small = (T - V) < (1 << 23);
    int cs = 0, below = 0;
    for (int base = wa, ks = 0; base < we; base += 256, ++ks) {
        const int i0 = base + lane * 8;
        const int cs0 = cs;
        do {  // one chunk; `continue` leaves it
        if (i0 >= we) continue;
        if (gs[i0 / SUBTILE] < 1.0f) {
            // cold subtile: e_i <= 1 (numerators are relative to the
            // subtile's max), so q_i = fl(e_i * gs_u) <= gs_u < 1 and every
            // count is floor(q_i) + 1 = 1 -- the numerators are not read
            const int n = min(8, we - i0);
            cs += n;
            if (MODE == MODE_LOHI) {
                if (i0 + n <= sym) {
                    below += n;
                } else if (i0 <= sym) {
                    below += sym - i0;
                    rs.csym = 1;
                }
            }
            continue;
        }
        float e[8];
        int c[8];
        int step;
        const bool full = i0 + 8 <= we && aligned_row;
        if (full && small && (MODE != MODE_LOHI || i0 + 8 <= sym || i0 > sym)) {
            // common case: only the chunk's total is needed.  floor(q) for
            // 0 <= q < 2^23 is the bit pattern of q + 2^23 (rounded down)
            // minus that of 2^23; the patterns add up in wrapping integer
            // arithmetic and the 8 offsets come off once
            src.load8_full(i0, e);
            const float g = gs[i0 / SUBTILE];
            uint32_t f = 8u - 8u * 0x4B000000u;
#pragma unroll
            for (int k = 0; k < 8; ++k) f += __float_as_uint(__fadd_rd(__fmul_rn(e[k], g), 8388608.0f));
            step = (int)f;
            cs += step;
            if (MODE == MODE_LOHI && i0 + 8 <= sym) below += step;
            continue;
        }
        if (full) {
            src.load8_full(i0, e);
            step = small ? counts8_full<true>(e, gs[i0 / SUBTILE], c)
                         : counts8_full<false>(e, gs[i0 / SUBTILE], c);
        } else {
            src.load8(i0, we, e);
            step = counts8(e, gs[i0 / SUBTILE], i0, we, c);
        }
        cs += step;
        if (MODE == MODE_LOHI) {
            if (i0 + 8 <= sym) {
                below += step;
            } else if (i0 <= sym) {
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    if (i0 + k < sym) below += c[k];
                    if (i0 + k == sym) rs.csym = c[k];
                }
            }
        }
        } while (0);
        if (MODE == MODE_DECODE) {
            // this step's count total over the warp, for the owner search
            int v = cs - cs0;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if (lane == 0) s_ct[warp * CT_STEPS + ks] = v;
        }
    }
    if (MODE == MODE_LOHI) {
        int tot = cs, below_all = below;
        block_sum_i2(tot, below_all, red);
        const int deficit = T - tot;
        if (tid == 0) {
            const uint32_t lo = (uint32_t)(below_all + (amax < sym ? deficit : 0));
            const uint32_t hi = lo + (uint32_t)(rs.csym + (amax == sym ? deficit : 0));
            reinterpret_cast<uint2*>(out)[row] = make_uint2(lo, hi);
        }
        return;
    }
    const int deficit = T - block_sum_i(cs, red);

    // ---- per-warp totals (deficit on the argmax's warp), exclusive scan ----
    int ws = cs;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ws += __shfl_xor_sync(0xffffffffu, ws, off);
    if (lane == 0) s_wsum[warp] = ws + ((amax >= wa && amax < we) ? deficit : 0);
    __syncthreads();
    if (tid == 0) {
        int run = 0;
        for (int w = 0; w < CDF_NW; ++w) {
            s_wexcl[w] = run;
            run += s_wsum[w];
        }
    }
    __syncthreads();

    if (MODE == MODE_COUNTS || MODE == MODE_CDF) {
        int32_t* o = reinterpret_cast<int32_t*>(out) + (int64_t)row * (V + 1);
        if (tid == 0) o[0] = 0;
        int run = s_wexcl[warp];
        walk_counts(src, gs, wa, we, amax, deficit, small,
                    [&](int i0, const int (&c)[8], int, int excl, int total) {
                        if (i0 < we) {
                            int r = run + excl;
#pragma unroll
                            for (int k = 0; k < 8; ++k) {
                                if (i0 + k < we) {
                                    r += c[k];
                                    o[i0 + k + 1] = (MODE == MODE_COUNTS) ? c[k] : r;
                                }
                            }
                        }
                        run += total;
                        return false;
                    });
        return;
    }

    // ---- DECODE: owner warp, then the step and lane holding the target -----
    const uint32_t target = s_target;
    if (tid < CDF_NW && s_wsum[tid] > 0 && (uint32_t)s_wexcl[tid] <= target &&
        target < (uint32_t)(s_wexcl[tid] + s_wsum[tid]))
        s_owner = tid;
    __syncthreads();
    if (warp == s_owner) {
        // the step totals recorded by the element pass locate the 256-element
        // step holding the target; only that step's counts are recomputed
        int run = s_wexcl[warp], base = wa;
        for (int ks = 0; base < we; base += 256, ++ks) {
            const int tot = s_ct[warp * CT_STEPS + ks] +
                            ((amax >= base && amax < min(base + 256, we)) ? deficit : 0);
            if (target < (uint32_t)(run + tot)) break;
            run += tot;
        }
        if (base < we) {
            const int i0 = base + lane * 8;
            int c[8];
            const int ls = chunk_counts(src, gs, i0, we, amax, deficit, small, c);
            int inc = ls;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, inc, off);
                if (lane >= off) inc += y;
            }
            int r = run + inc - ls;
            if (ls > 0 && (uint32_t)r <= target && target < (uint32_t)(r + ls)) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (c[j] > 0 && target < (uint32_t)(r + c[j])) {
                        s_sym = i0 + j;
                        s_lo = (uint32_t)r;
                        s_hi = (uint32_t)(r + c[j]);
                        break;
                    }
                    r += c[j];
                }
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        int64_t off, lim;
        stream_window(in_bytes, in_offs, row, off, lim);
        decode_apply(states + 4 * (int64_t)row, in + off, lim, s_lo, s_hi, bits);
        out_syms[row] = s_sym;
        if (counters) {
            const int pos = counters[2 * row];
            if (history) history[(int64_t)row * hist_stride + pos] = s_sym;
            counters[2 * row] = pos + 1;
        } else if (history) {
            history[(int64_t)row * hist_stride] = s_sym;
        }
    }
}

// One CTA per row; numerators + partials from global (stats != NULL) or raw
// logits (stats == NULL).
template <int MODE>
__global__ void __launch_bounds__(CDF_NT) k_cdf(const uint16_t* __restrict__ logits, int64_t stride,
                                                int V, int bits, const float2* __restrict__ stats,
                                                int64_t stats_stride,
                                                const int32_t* __restrict__ symbols, void* out,
                                                const uint8_t* in, int64_t in_bytes,
                                                const int64_t* __restrict__ in_offs,
                                                uint32_t* states, int32_t* counters,
                                                int32_t* out_syms, int32_t* history,
                                                int64_t hist_stride) {
    __shared__ float2 s_part[MAX_SUB];
    __shared__ float s_gs[MAX_SUB];
    __shared__ RowShared rs;
    __shared__ CdfRed red;
    const int row = blockIdx.x;
    if (MODE == MODE_DECODE && counters && counters[2 * row] >= counters[2 * row + 1]) {
        if (threadIdx.x == 0) out_syms[row] = 0;
        return;
    }
    const uint16_t* x = logits + (int64_t)row * stride;
    const int nsub = (V + SUBTILE - 1) / SUBTILE;
    const float scale = (float)((1 << bits) - V);

    int sym = 0;
    if (MODE == MODE_LOHI) {
        sym = symbols[row];
        sym = sym < 0 ? 0 : (sym >= V ? V - 1 : sym);
    }
    if (stats) {
        const float2* p = stats + (int64_t)row * stats_stride;
        const NumSrc src{x, V};
        row_setup([&](int u) { return p[u]; }, [&](int i) { return src.is_one(i); }, nsub, scale,
                  s_gs, rs, red);
        cdf_row_body<MODE>(src, V, bits, s_gs, rs, red, row, sym, out, in, in_bytes, in_offs,
                           states, counters, out_syms, history, hist_stride);
    } else {
        raw_partials(x, V, nsub, s_part);
        const RawSrc src{x, s_part, V};
        row_setup([&](int u) { return s_part[u]; }, [&](int i) { return src.is_one(i); }, nsub,
                  scale, s_gs, rs, red);
        cdf_row_body<MODE>(src, V, bits, s_gs, rs, red, row, sym, out, in, in_bytes, in_offs,
                           states, counters, out_syms, history, hist_stride);
    }
}

// ---------------------------------------------------------------------------
// (lo, hi) of the row's symbol with one warp per row (the compress hot path:
// numerators and partials from the head GEMM, 16-byte aligned rows).  Same
// numbers as k_cdf<MODE_LOHI>, computed without a CTA barrier so that the
// SM holds 48-64 rows at once and one row's reduction latency hides behind
// the others' loads:
// * the normaliser follows the 512-virtual-thread order of row_setup:
//   virtual thread 32j + lane folds u = 32j + lane + 512k in order, each
//   virtual warp j reduces by the xor butterfly, and the 16 warp partials
//   (identity-padded to 32 lanes) meet in the same butterfly;
// * lane l takes whole subtiles u = l + 32k (64 contiguous bytes, four
//   16-byte loads), with gs_u computed once per subtile;
// * the argmax is the (gs_u desc, u asc) maximum, then the first e == 1 in it.
// ---------------------------------------------------------------------------
#ifndef KB_CDF_WARP
#define KB_CDF_WARP 1
#endif
constexpr int CW_WARPS = 8;
#ifndef KB_CDFW_NJ
#define KB_CDFW_NJ 8  // virtual warps whose partials are folded together
#endif
#ifndef KB_CDFW_RU
#define KB_CDFW_RU 4  // rounds of hot-subtile loads in flight
#endif

__global__ void __launch_bounds__(CW_WARPS * 32)
    k_cdf_lohi_warp(const uint16_t* __restrict__ logits, int64_t stride, int V, int bits,
                    const float2* __restrict__ stats, int64_t stats_stride,
                    const int32_t* __restrict__ symbols, uint2* __restrict__ out, int rows) {
    extern __shared__ float cw_m[];  // per warp: the subtile maxima m_u of its row
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * CW_WARPS + (threadIdx.x >> 5);
    if (row >= rows) return;
    const uint16_t* x = logits + (int64_t)row * stride;
    const float2* p = stats + (int64_t)row * stats_stride;
    const int nsub = (V + SUBTILE - 1) / SUBTILE;
    float* ms = cw_m + (threadIdx.x >> 5) * nsub;
    const int T = 1 << bits;
    const float scale = (float)(T - V);
    const bool small = (T - V) < (1 << 23);
    int sym = symbols[row];
    sym = sym < 0 ? 0 : (sym >= V ? V - 1 : sym);

    // ---- normaliser (M, 1/S) ---------------------------------------------
    // virtual warps in batches of NJ: the loads of a batch are issued
    // together and its butterflies interleave
    MS w{-INFINITY, 0.0f};
    constexpr int NJ = KB_CDFW_NJ;  // a power of two, at most 16
    for (int j0 = 0; j0 < CDF_NW; j0 += NJ) {
        MS acc[NJ];
#pragma unroll
        for (int j = 0; j < NJ; ++j) acc[j] = MS{-INFINITY, 0.0f};
        for (int u0 = 32 * j0 + lane; u0 < nsub; u0 += CDF_NT) {
            float2 q[NJ];
#pragma unroll
            for (int j = 0; j < NJ; ++j)
                q[j] = u0 + 32 * j < nsub ? p[u0 + 32 * j] : make_float2(0.0f, 0.0f);
#pragma unroll
            for (int j = 0; j < NJ; ++j)
                if (u0 + 32 * j < nsub) {
                    acc[j] = ms_merge(acc[j], MS{q[j].x, q[j].y});
                    ms[u0 + 32 * j] = q[j].x;
                }
        }
        // The xor butterflies of the NJ virtual warps by recursive halving:
        // at offset `off` a lane keeps the half of its values selected by
        // lane bit `off` and merges it with the partner's copy of that half.
        // The partner shares every bit used so far, so it holds the same
        // partials the plain butterfly would, and ms_merge is symmetric: the
        // results are the butterflies' bits.  Lanes 32/NJ*j.. hold warp j0+j.
        constexpr int LV = NJ >= 16 ? 4 : NJ >= 8 ? 3 : NJ >= 4 ? 2 : NJ >= 2 ? 1 : 0;
#pragma unroll
        for (int lv = 0; lv < LV; ++lv) {
            const int h = (NJ >> lv) / 2, off = 16 >> lv;
            const bool up = (lane & off) != 0;
#pragma unroll
            for (int i = 0; i < h; ++i) {
                const MS keep = up ? acc[h + i] : acc[i];
                const MS give = up ? acc[i] : acc[h + i];
                acc[i] = ms_merge(keep, ms_shfl_xor(give, off));
            }
        }
#pragma unroll
        for (int off = 16 >> LV; off > 0; off >>= 1)
            acc[0] = ms_merge(acc[0], ms_shfl_xor(acc[0], off));
        const MS wj = MS{__shfl_sync(0xffffffffu, acc[0].m, (32 / NJ) * ((lane - j0) & (NJ - 1))),
                         __shfl_sync(0xffffffffu, acc[0].s, (32 / NJ) * ((lane - j0) & (NJ - 1)))};
        if (lane >= j0 && lane < j0 + NJ) w = wj;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) w = ms_merge(w, ms_shfl_xor(w, off));
    const float M = w.m, inv = __frcp_rn(w.s);

    // ---- counts -------------------------------------------------------------
    // Pass 1, step k: lane l owns subtile u = 32k + l and its factor gs_u.  A
    // cold subtile (gs_u < 1: e_i <= 1, so q_i = fl(e_i * gs_u) <= gs_u < 1)
    // has every count 1 and its numerators are not read; a hot one is
    // appended to a list kept in the already-consumed front of ms[].
    // Pass 2 counts the hot subtiles with the whole warp: lanes 4q..4q+3
    // take 8 elements each of list entry 8r + q, RU rounds of loads in flight.
    const unsigned lt = (1u << lane) - 1u;
    int* hot_u = reinterpret_cast<int*>(ms);
    const int usym = sym / SUBTILE;
    float best = -INFINITY, gsym = 0.0f;
    int bu = INT_MAX, cs = 0, below = 0, nhot = 0;
    for (int k0 = 0; k0 < nsub; k0 += 32) {
        const int u = k0 + lane;
        const bool valid = u < nsub;
        const int i0 = u * SUBTILE;
        const int n = valid ? min(SUBTILE, V - i0) : 0;
        const float g =
            valid ? __fmul_rn(__fmul_rn(kb_expf(__fsub_rn(ms[u], M)), inv), scale) : 0.0f;
        if (valid && g > best) {
            best = g;
            bu = u;
        }
        if (u == usym) gsym = g;
        const bool hot = valid && g >= 1.0f && n == SUBTILE;
        int csub = 0;
        if (valid && !hot) {
            if (g < 1.0f) {
                csub = n;
            } else {  // the row's last, partial subtile
                for (int j = 0; j < n; ++j) csub += (int)floorf(__fmul_rn(h2f(x[i0 + j]), g)) + 1;
            }
        }
        cs += csub;
        if (u < usym) below += csub;
        const unsigned hm = __ballot_sync(0xffffffffu, hot);
        if (hot) hot_u[nhot + __popc(hm & lt)] = u;  // index <= u: already read
        nhot += __popc(hm);
    }
    __syncwarp();
    constexpr int RU = KB_CDFW_RU;
    const int q = lane >> 2;
    for (int j0 = 0; j0 < nhot; j0 += 8 * RU) {
        uint4 v[RU];
        int uu[RU];
#pragma unroll
        for (int r = 0; r < RU; ++r) {
            const int j = j0 + 8 * r + q;
            uu[r] = j < nhot ? hot_u[j] : -1;
            v[r] = uu[r] >= 0 ? *reinterpret_cast<const uint4*>(x + (int64_t)uu[r] * SUBTILE +
                                                                 8 * (lane & 3))
                              : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int r = 0; r < RU; ++r) {
            int part = 0;
            if (uu[r] >= 0) {
                const float g =
                    __fmul_rn(__fmul_rn(kb_expf(__fsub_rn(p[uu[r]].x, M)), inv), scale);
                float e[8];
                int c[8];
                unpack8(v[r], e);
                part = small ? counts8_full<true>(e, g, c) : counts8_full<false>(e, g, c);
            }
            part += __shfl_xor_sync(0xffffffffu, part, 1);
            part += __shfl_xor_sync(0xffffffffu, part, 2);
            if ((lane & 3) == 0 && uu[r] >= 0) {
                cs += part;
                if (uu[r] < usym) below += part;
            }
        }
    }
    // the symbol's own subtile, one element per lane
    int csym;
    {
        const float g = __shfl_sync(0xffffffffu, gsym, usym & 31);
        const int i = usym * SUBTILE + lane;
        int c = 0;
        if (i < V) c = g < 1.0f ? 1 : (int)floorf(__fmul_rn(h2f(x[i]), g)) + 1;
        csym = __shfl_sync(0xffffffffu, c, sym & 31);
        below += i < sym ? c : 0;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        cs += __shfl_xor_sync(0xffffffffu, cs, off);
        below += __shfl_xor_sync(0xffffffffu, below, off);
        am_merge(best, bu, __shfl_xor_sync(0xffffffffu, best, off),
                 __shfl_xor_sync(0xffffffffu, bu, off));
    }
    const int a = bu * SUBTILE;
    const unsigned b0 = __ballot_sync(0xffffffffu, a + lane < V && x[a + lane] == (uint16_t)0x3C00u);
    const int amax = a + __ffs(b0) - 1;
    if (lane == 0) {
        const int deficit = T - cs;
        const uint32_t lo = (uint32_t)(below + (amax < sym ? deficit : 0));
        const uint32_t hi = lo + (uint32_t)(csym + (amax == sym ? deficit : 0));
        out[row] = make_uint2(lo, hi);
    }
}

static int launch_cdf_lohi_warp(int rows, const uint16_t* logits, int64_t stride, int V, int bits,
                                const float* stats, int64_t stats_stride, const int32_t* symbols,
                                void* out, cudaStream_t st) {
    ProfScope ps(PH_CDF, st, (double)rows * ((double)V * 2 + 16.0));
    const int grid = (rows + CW_WARPS - 1) / CW_WARPS;
    const size_t smem = (size_t)CW_WARPS * ((V + SUBTILE - 1) / SUBTILE) * sizeof(float);
    static std::atomic<unsigned long long> done{0};
    const cudaError_t e = once_per_device(done, [] {
        return cudaFuncSetAttribute(k_cdf_lohi_warp, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)(CW_WARPS * MAX_SUB * sizeof(float)));
    });
    if (e != cudaSuccess) {
        set_cuda_error(e);
        return KB_ERR_CUDA;
    }
    k_cdf_lohi_warp<<<grid, CW_WARPS * 32, smem, st>>>(logits, stride, V, bits,
                                                     reinterpret_cast<const float2*>(stats),
                                                     stats_stride, symbols,
                                                     reinterpret_cast<uint2*>(out), rows);
    return launch_status();
}

struct CdfArgs {
    const uint16_t* logits;
    int64_t stride;
    int V, bits;
    const float* stats;
    int64_t stats_stride;
    const int32_t* symbols;
    void* out;
    const uint8_t* in;
    int64_t in_bytes;
    const int64_t* in_offs;
    uint32_t* states;
    int32_t* counters;
    int32_t* out_syms;
    int32_t* history;
    int64_t hist_stride;
};

template <int MODE>
static int launch_cdf(int rows, const CdfArgs& a, cudaStream_t st) {
    ProfScope ps(MODE == MODE_DECODE ? PH_DECODE : PH_CDF, st,
                 (double)rows * ((double)a.V * 2 + 16.0));
    k_cdf<MODE><<<rows, CDF_NT, 0, st>>>(a.logits, a.stride, a.V, a.bits,
                                         reinterpret_cast<const float2*>(a.stats), a.stats_stride,
                                         a.symbols, a.out, a.in, a.in_bytes, a.in_offs, a.states,
                                         a.counters, a.out_syms, a.history, a.hist_stride);
    return launch_status();
}

}  // namespace kb

using namespace kb;

static inline bool cdf_args_ok(int V, int bits) {
    // V < T so that T - V >= 1; V <= 65536 bounds the subtile partials per row.
    return bits >= 2 && bits <= 30 && V >= 1 && V <= 65536 && V < (1 << bits);
}

static inline bool stats_ok(const float* stats, int64_t stats_stride, int V) {
    // stats_stride >= number of 32-column subtiles, float2-aligned
    return !stats || (stats_stride >= (V + SUBTILE - 1) / SUBTILE &&
                      (reinterpret_cast<uintptr_t>(stats) & 7u) == 0);
}

extern "C" int kb_cdf_rows(const uint16_t* logits, int64_t row_stride, int rows, int V, int bits,
                           int mode, const float* logit_stats, int64_t stats_stride,
                           const int32_t* symbols, void* out, void* stream) {
    if (!logits || !out || rows < 0 || !cdf_args_ok(V, bits) || row_stride < V ||
        !stats_ok(logit_stats, stats_stride, V))
        return KB_ERR_ARG;
    if (rows == 0) return KB_OK;
    cudaStream_t st = as_stream(stream);
    CdfArgs a{logits, row_stride, V, bits, logit_stats, stats_stride, symbols, out,
              nullptr, 0, nullptr, nullptr, nullptr, nullptr, nullptr, 0};
    switch (mode) {
        case KB_CDF_COUNTS: return launch_cdf<MODE_COUNTS>(rows, a, st);
        case KB_CDF_CDF: return launch_cdf<MODE_CDF>(rows, a, st);
        case KB_CDF_LOHI: {
            if (!symbols) return KB_ERR_ARG;
            if ((reinterpret_cast<uintptr_t>(out) & 7u) != 0) return KB_ERR_ALIGN;
            if (KB_CDF_WARP && logit_stats && aligned16(logits) && row_stride % 8 == 0)
                return launch_cdf_lohi_warp(rows, logits, row_stride, V, bits, logit_stats,
                                            stats_stride, symbols, out, st);
            return launch_cdf<MODE_LOHI>(rows, a, st);
        }
        default:
            return KB_ERR_ARG;
    }
}

extern "C" int kb_cdf_from_probs(const float* probs, int rows, int V, int bits, int32_t* out,
                                 void* stream) {
    if (!probs || !out || rows < 0 || !cdf_args_ok(V, bits)) return KB_ERR_ARG;
    if (rows == 0) return KB_OK;
    cudaStream_t st = as_stream(stream);
    ProfScope ps(PH_CDF, st, (double)rows * ((double)V * 4 + 16.0));
    k_cdf_probs<<<rows, CDF_NT, 0, st>>>(probs, V, bits, out);
    return launch_status();
}

extern "C" int kb_decode_logits_step(const uint16_t* logits, int64_t row_stride, int B, int V,
                                     int bits, const float* logit_stats, int64_t stats_stride,
                                     const uint8_t* in, int64_t in_bytes, const int64_t* in_offs,
                                     uint32_t* states, int32_t* counters, int32_t* out_syms,
                                     int32_t* history, int64_t hist_stride, void* stream) {
    if (!logits || !in || !states || !out_syms || B < 0 || !cdf_args_ok(V, bits) ||
        row_stride < V || hist_stride < 0 || !stats_ok(logit_stats, stats_stride, V))
        return KB_ERR_ARG;
    if (B > 1 && !in_offs) return KB_ERR_ARG;
    if (B == 0) return KB_OK;
    CdfArgs a{logits, row_stride, V, bits, logit_stats, stats_stride, nullptr, nullptr,
              in, in_bytes, in_offs, states, counters, out_syms, history, hist_stride};
    return launch_cdf<MODE_DECODE>(B, a, as_stream(stream));
}
