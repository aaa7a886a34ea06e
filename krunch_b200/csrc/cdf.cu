// Fused logits -> softmax -> integer CDF, one CTA per row.
//
// Spec (krunch_ac/cdf.py:22-74, krunch_ac/cuda/det_softmax_cdf.cu:62-185):
//   p_i    = softmax(logits)_i
//   c_i    = floor(p_i * (T - V)) + 1           (MIN_PROB = 1)
//   c_amax += T - sum(c)                         (argmax of p, smallest index on ties)
//   cdf    = [0, cumsum(c)]
//
// Every float operation of a row happens in an order fixed by V alone:
// thread t of the CDF_NT-thread block owns the contiguous segment
// [t*L, min((t+1)*L, V)) with L = ceil(V / CDF_NT), sums it sequentially,
// and the per-thread partials meet in a fixed xor-butterfly (warp) then a
// fixed butterfly over the warp partials.  exp is kb_expf (kb_common.cuh).
// Integer sums are exact, so their order is free.  A row's CDF is therefore
// bit-identical whatever the number of rows, the launch, or the GPU, and
// the C restatement in oracle/ reproduces it bit for bit.
//
// Modes: COUNTS / CDF write [rows, V+1] int32 (reference contract);
// LOHI writes only the (cdf[s], cdf[s+1]) pair of the row's symbol (the
// compress hot path — the [rows, V+1] CDF is never materialised);
// DECODE runs the range-decoder step for stream `row` in the same CTA.
#include <float.h>
#include <limits.h>

#include "coder.cuh"
#include "profile.cuh"

namespace kb {

constexpr int CDF_NT = 512;
constexpr int CDF_NW = CDF_NT / 32;
constexpr int MODE_COUNTS = KB_CDF_COUNTS;
constexpr int MODE_CDF = KB_CDF_CDF;
constexpr int MODE_LOHI = KB_CDF_LOHI;
constexpr int MODE_DECODE = 3;

struct CdfRed {
    float f[CDF_NW];
    int i[CDF_NW];
    float v[CDF_NW];
    int i2[CDF_NW];
};

__device__ __forceinline__ float block_max_f(float v, CdfRed& r) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    if (lane == 0) r.f[w] = v;
    __syncthreads();
    float x = (lane < CDF_NW) ? r.f[lane] : -INFINITY;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, off));
    __syncthreads();
    return x;
}

// Fixed-tree float sum: butterfly in each warp, then the same butterfly over
// the CDF_NW warp partials (zero padded to 32).  IEEE addition commutes, so
// every lane of a butterfly holds the same value.
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

// Exclusive prefix sum over threads (integer, exact).
__device__ __forceinline__ int block_excl_scan_i(int v, CdfRed& r) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int inc = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += y;
    }
    if (lane == 31) r.i[w] = inc;
    __syncthreads();
    if (w == 0) {
        int t = (lane < CDF_NW) ? r.i[lane] : 0;
        int tinc = t;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, tinc, off);
            if (lane >= off) tinc += y;
        }
        if (lane < CDF_NW) r.i2[lane] = tinc - t;
    }
    __syncthreads();
    const int res = r.i2[w] + inc - v;
    __syncthreads();
    return res;
}

// Copy one fp16 row into shared memory with the widest aligned loads.
__device__ __forceinline__ void load_row_f16(const uint16_t* __restrict__ x, uint16_t* sx, int V) {
    const int tid = threadIdx.x;
    if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
        const int nv = V >> 3;
        const uint4* xv = reinterpret_cast<const uint4*>(x);
        uint4* sv = reinterpret_cast<uint4*>(sx);
#pragma unroll 4
        for (int i = tid; i < nv; i += CDF_NT) sv[i] = __ldg(xv + i);
        for (int i = (nv << 3) + tid; i < V; i += CDF_NT) sx[i] = x[i];
    } else if ((reinterpret_cast<uintptr_t>(x) & 3u) == 0) {
        const int nv = V >> 1;
        const uint32_t* xv = reinterpret_cast<const uint32_t*>(x);
        uint32_t* sv = reinterpret_cast<uint32_t*>(sx);
#pragma unroll 4
        for (int i = tid; i < nv; i += CDF_NT) sv[i] = __ldg(xv + i);
        for (int i = (nv << 1) + tid; i < V; i += CDF_NT) sx[i] = x[i];
    } else {
        for (int i = tid; i < V; i += CDF_NT) sx[i] = x[i];
    }
}

// Row source: probability p_i of element i after the normalisation pass.
struct LogitsRow {
    const uint16_t* sx;  // shared memory copy of the row
    float m, inv;
    __device__ __forceinline__ float p(int i) const {
        return __fmul_rn(kb_expf(__fsub_rn(h2f(sx[i]), m)), inv);
    }
};
struct ProbsRow {
    const float* x;  // global row
    float s;
    __device__ __forceinline__ float p(int i) const { return __fdiv_rn(x[i], s); }
};

template <int MODE, bool FROM_PROBS>
__global__ void __launch_bounds__(CDF_NT) k_cdf(const void* __restrict__ src, int64_t stride,
                                                int V, int bits,
                                                const int32_t* __restrict__ symbols, void* out,
                                                const uint8_t* in, int64_t in_bytes,
                                                const int64_t* __restrict__ in_offs,
                                                uint32_t* states, int32_t* counters,
                                                int32_t* out_syms, int32_t* history,
                                                int64_t hist_stride) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ CdfRed red;
    __shared__ int s_csym, s_owner, s_owner_base, s_sym;
    __shared__ uint32_t s_target, s_lo, s_hi;

    const int row = blockIdx.x;
    const int tid = threadIdx.x;
    if (MODE == MODE_DECODE && counters && counters[2 * row] >= counters[2 * row + 1]) {
        if (tid == 0) out_syms[row] = 0;
        return;
    }
    const int L = (V + CDF_NT - 1) / CDF_NT;
    const int a = min(tid * L, V);
    const int e = min(a + L, V);
    const int T = 1 << bits;
    const float scale = (float)(T - V);

    int sym = 0;
    if (MODE == MODE_LOHI) {
        sym = symbols[row];
        sym = sym < 0 ? 0 : (sym >= V ? V - 1 : sym);
    }
    if (MODE == MODE_DECODE && tid == 0) s_target = decode_target(states + 4 * (int64_t)row, bits);

    // ---- normalisation pass ------------------------------------------------
    LogitsRow lr;
    ProbsRow pr;
    if (!FROM_PROBS) {
        uint16_t* sx = reinterpret_cast<uint16_t*>(smem_raw);
        load_row_f16(reinterpret_cast<const uint16_t*>(src) + (int64_t)row * stride, sx, V);
        __syncthreads();
        float mt = -INFINITY;
        for (int i = a; i < e; ++i) mt = fmaxf(mt, h2f(sx[i]));
        const float m = block_max_f(mt, red);
        float st = 0.0f;
        for (int i = a; i < e; ++i) st = __fadd_rn(st, kb_expf(__fsub_rn(h2f(sx[i]), m)));
        const float S = block_sum_f(st, red);
        lr.sx = sx;
        lr.m = m;
        lr.inv = __frcp_rn(S);
    } else {
        const float* x = reinterpret_cast<const float*>(src) + (int64_t)row * stride;
        float st = 0.0f;
        for (int i = a; i < e; ++i) st = __fadd_rn(st, x[i]);
        const float S = block_sum_f(st, red);
        pr.x = x;
        pr.s = fmaxf(S, 1e-30f);
    }
    auto prob = [&](int i) -> float { return FROM_PROBS ? pr.p(i) : lr.p(i); };
    auto count = [&](float p) -> int { return (int)floorf(__fmul_rn(p, scale)) + 1; };

    // ---- counts, argmax, totals ------------------------------------------
    int cs = 0, below = 0;
    float bp = -INFINITY;
    int bi = INT_MAX;
    for (int i = a; i < e; ++i) {
        const float p = prob(i);
        const int c = count(p);
        cs += c;
        if (p > bp) {  // ascending scan: strict '>' keeps the smallest index
            bp = p;
            bi = i;
        }
        if (MODE == MODE_LOHI) {
            if (i < sym) below += c;
            if (i == sym) s_csym = c;
        }
    }
    const int amax = block_argmax(bp, bi, red);
    const int total = block_sum_i(cs, red);
    const int deficit = T - total;

    if (MODE == MODE_LOHI) {
        const int below_all = block_sum_i(below, red);
        if (tid == 0) {
            const uint32_t lo = (uint32_t)(below_all + (amax < sym ? deficit : 0));
            const uint32_t hi = lo + (uint32_t)(s_csym + (amax == sym ? deficit : 0));
            reinterpret_cast<uint2*>(out)[row] = make_uint2(lo, hi);
        }
        return;
    }

    // ---- per-segment prefix (deficit folded into the argmax segment) --------
    const int segd = cs + ((amax >= a && amax < e) ? deficit : 0);
    const int excl = block_excl_scan_i(segd, red);

    if (MODE == MODE_COUNTS || MODE == MODE_CDF) {
        int32_t* o = reinterpret_cast<int32_t*>(out) + (int64_t)row * (V + 1);
        if (tid == 0) o[0] = 0;
        int run = excl;
        for (int i = a; i < e; ++i) {
            const int c = count(prob(i)) + (i == amax ? deficit : 0);
            run += c;
            o[i + 1] = (MODE == MODE_COUNTS) ? c : run;
        }
        return;
    }

    // ---- DECODE: locate target, then narrow the range ----------------------
    const uint32_t target = s_target;
    if (segd > 0 && (uint32_t)excl <= target && target < (uint32_t)(excl + segd)) {
        s_owner = tid;
        s_owner_base = excl;
    }
    __syncthreads();
    if (tid < 32) {
        const int lane = tid;
        const int oa = min(s_owner * L, V), oe = min(oa + L, V);
        const int q = (oe - oa + 31) / 32;
        const int la = min(oa + lane * q, oe), le = min(la + q, oe);
        int ls = 0;
        for (int i = la; i < le; ++i) ls += count(prob(i)) + (i == amax ? deficit : 0);
        int inc = ls;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, inc, off);
            if (lane >= off) inc += y;
        }
        const int base = s_owner_base + inc - ls;
        if (ls > 0 && (uint32_t)base <= target && target < (uint32_t)(base + ls)) {
            int run = base;
            for (int i = la; i < le; ++i) {
                const int c = count(prob(i)) + (i == amax ? deficit : 0);
                if (target < (uint32_t)(run + c)) {
                    s_sym = i;
                    s_lo = (uint32_t)run;
                    s_hi = (uint32_t)(run + c);
                    break;
                }
                run += c;
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

template <int MODE, bool FROM_PROBS>
static int launch_cdf(int rows, int V, const void* src, int64_t stride, int bits,
                      const int32_t* symbols, void* out, const uint8_t* in, int64_t in_bytes,
                      const int64_t* in_offs, uint32_t* states, int32_t* counters,
                      int32_t* out_syms, int32_t* history, int64_t hist_stride, cudaStream_t st) {
    const size_t smem = FROM_PROBS ? 0 : (size_t)((V * 2 + 15) / 16) * 16;
    static int configured = 0;  // per template instance
    if (!FROM_PROBS && smem > 48 * 1024 && !configured) {
        cudaError_t e = cudaFuncSetAttribute(k_cdf<MODE, FROM_PROBS>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)(66 * 1024 * 2));
        if (e != cudaSuccess) {
            set_cuda_error(e);
            return KB_ERR_CUDA;
        }
        configured = 1;
    }
    ProfScope ps(MODE == MODE_DECODE ? PH_DECODE : PH_CDF, st,
                 (double)rows * ((double)V * (FROM_PROBS ? 4 : 2) + 16.0));
    k_cdf<MODE, FROM_PROBS><<<rows, CDF_NT, smem, st>>>(src, stride, V, bits, symbols, out, in,
                                                         in_bytes, in_offs, states, counters,
                                                         out_syms, history, hist_stride);
    return launch_status();
}

}  // namespace kb

using namespace kb;

static inline bool cdf_args_ok(int V, int bits) {
    // V < T so that T - V >= 1; V <= 65536 bounds the shared-memory row copy.
    return bits >= 2 && bits <= 30 && V >= 1 && V <= 65536 && V < (1 << bits);
}

extern "C" int kb_cdf_rows(const uint16_t* logits, int64_t row_stride, int rows, int V, int bits,
                           int mode, const int32_t* symbols, void* out, void* stream) {
    if (!logits || !out || rows < 0 || !cdf_args_ok(V, bits) || row_stride < V) return KB_ERR_ARG;
    if (rows == 0) return KB_OK;
    cudaStream_t st = as_stream(stream);
    switch (mode) {
        case KB_CDF_COUNTS:
            return launch_cdf<MODE_COUNTS, false>(rows, V, logits, row_stride, bits, nullptr, out,
                                                  nullptr, 0, nullptr, nullptr, nullptr, nullptr,
                                                  nullptr, 0, st);
        case KB_CDF_CDF:
            return launch_cdf<MODE_CDF, false>(rows, V, logits, row_stride, bits, nullptr, out,
                                               nullptr, 0, nullptr, nullptr, nullptr, nullptr, nullptr, 0, st);
        case KB_CDF_LOHI:
            if (!symbols) return KB_ERR_ARG;
            if ((reinterpret_cast<uintptr_t>(out) & 7u) != 0) return KB_ERR_ALIGN;
            return launch_cdf<MODE_LOHI, false>(rows, V, logits, row_stride, bits, symbols, out,
                                                nullptr, 0, nullptr, nullptr, nullptr, nullptr,
                                                nullptr, 0, st);
        default:
            return KB_ERR_ARG;
    }
}

extern "C" int kb_cdf_from_probs(const float* probs, int rows, int V, int bits, int32_t* out,
                                 void* stream) {
    if (!probs || !out || rows < 0 || !cdf_args_ok(V, bits)) return KB_ERR_ARG;
    if (rows == 0) return KB_OK;
    return launch_cdf<MODE_CDF, true>(rows, V, probs, V, bits, nullptr, out, nullptr, 0, nullptr,
                                      nullptr, nullptr, nullptr, nullptr, 0, as_stream(stream));
}

extern "C" int kb_decode_logits_step(const uint16_t* logits, int64_t row_stride, int B, int V,
                                     int bits, const uint8_t* in, int64_t in_bytes,
                                     const int64_t* in_offs, uint32_t* states, int32_t* counters,
                                     int32_t* out_syms, int32_t* history, int64_t hist_stride,
                                     void* stream) {
    if (!logits || !in || !states || !out_syms || B < 0 || !cdf_args_ok(V, bits) ||
        row_stride < V || hist_stride < 0)
        return KB_ERR_ARG;
    if (B > 1 && !in_offs) return KB_ERR_ARG;
    if (B == 0) return KB_OK;
    return launch_cdf<MODE_DECODE, false>(B, V, logits, row_stride, bits, nullptr, nullptr, in,
                                          in_bytes, in_offs, states, counters, out_syms, history,
                                          hist_stride, as_stream(stream));
}
