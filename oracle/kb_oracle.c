/*
 * CPU oracle for the krunch_b200 coder and CDF kernels.  TEST INFRASTRUCTURE
 * ONLY: tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
 * arm use it as the checker.  The product path never loads it.
 *
 * Contents
 *  1. The 32-bit E1/E2/E3 range coder, a plain-C restatement of
 *     krunch_ac/cpu_reference.py (encode 91-147, RangeDecoder 161-211,
 *     _bsearch 225-234, bit packing 38-83).  Pinned against bitstreams the
 *     reference itself produced (tests/golden/).
 *  2. The probability -> integer CDF rule of krunch_ac/cdf.py:22-74
 *     (count = floor(p*(T-V))+1, deficit to the argmax, smallest index on
 *     ties), evaluated in the fixed order the GPU kernels use so that the
 *     result is bit-identical to them.
 *     From logits (fp16 row x, V valid columns), per 32-column subtile u
 *     [32u, min(32u+32, V)): m_u = max x_i; e_i = fp16(e^(x_i - m_u)); s_u =
 *     sum of e_i left to right.  The normaliser (M, S) merges the (m_u, s_u):
 *     virtual thread t of 512 merges u = t, t+512, ... in order; each warp of
 *     32 threads combines in a xor butterfly (16..1); the 16 warp results,
 *     padded to 32 with the neutral (-inf, 0), combine in the same butterfly.
 *     merge keeps the larger max and adds the other sum scaled by
 *     e^(m_small - m_large) (ties: plain sum), which is symmetric, so every
 *     butterfly lane gets the same value.  Then with scale = T - V,
 *       gs_u = (e^(m_u - M) * (1/S)) * scale,   q_i = e_i * gs_u,
 *       c_i  = floor(q_i) + 1,   argmax = smallest i with the largest q_i.
 *     exp is oc_expf below (the same algorithm as the kernels' kb_expf).
 *     The head GEMM's epilogue produces e_i and (m_u, s_u) as it computes the
 *     logits; the CDF kernels derive them when given raw logits.
 *     From probabilities the row sum uses NT = 512 virtual threads, thread t
 *     summing [t*L, min((t+1)*L, V)), L = ceil(V/NT), left to right, then a
 *     xor butterfly over 32 lanes and the same over the 16 warp results;
 *     p_i = x_i / S, c_i = floor(p_i * (T-V)) + 1, argmax over p_i.
 *     numpy's pairwise sum (cdf.py) can differ from these orders in a last
 *     bit, hence by +-1 in rare counts; tests compare against cdf.py with
 *     that allowance and against this file bit for bit.
 *
 * Build: gcc -O2 -fPIC -shared -ffp-contract=off -fno-fast-math (see build.py)
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OC_NT 512
#define OC_NW (OC_NT / 32)

/* ------------------------------------------------------------------------- */
/* float helpers                                                             */
/* ------------------------------------------------------------------------- */
static float bits_f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

float oc_half_to_float(uint16_t h) {
    const uint32_t s = (uint32_t)(h >> 15) << 31;
    const uint32_t e = (h >> 10) & 0x1f;
    const uint32_t m = h & 0x3ff;
    if (e == 0) {
        /* zero or subnormal: m * 2^-24, exact in fp32 */
        float v = (float)m * bits_f(0x33800000u);
        return s ? -v : v;
    }
    if (e == 31) return bits_f(s | 0x7f800000u | (m << 13));
    return bits_f(s | ((e + 112) << 23) | (m << 13));
}

/* fp32 -> fp16 bits, round to nearest even (IEEE). */
uint16_t oc_float_to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const int exp = (int)((x >> 23) & 0xff);
    uint32_t mant = x & 0x7fffffu;
    if (exp == 255) return (uint16_t)(sign | 0x7c00u | (mant ? 0x200u : 0u));
    const int e = exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (exp == 0) return (uint16_t)sign;
        const int shift = 126 - exp; /* bits dropped from the 24-bit significand */
        if (shift > 24) return (uint16_t)sign;
        mant |= 0x800000u;
        uint32_t h = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) ++h;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

/* e^x = 2^(x*log2e): n = rint(y), f = y - n, degree-5 Taylor polynomial of
 * 2^f, n added to the exponent field.  Same algorithm and constants as the
 * kernel-side kb_expf; every operation is a single IEEE rounding. */
float oc_expf(float x) {
    if (!(x >= -86.0f)) return 0.0f;
    const float y = x * bits_f(0x3fb8aa3bu);
    const float n = rintf(y);
    const float f = y - n;
    float p = bits_f(0x3aaec3ffu);
    p = fmaf(p, f, bits_f(0x3c1d955bu));
    p = fmaf(p, f, bits_f(0x3d635847u));
    p = fmaf(p, f, bits_f(0x3e75fdf0u));
    p = fmaf(p, f, bits_f(0x3f317218u));
    p = fmaf(p, f, 1.0f);
    uint32_t u;
    memcpy(&u, &p, 4);
    u += (uint32_t)((int32_t)n * (1 << 23));
    return bits_f(u);
}

static float butterfly32(float* v) {
    float t[32];
    for (int off = 16; off > 0; off >>= 1) {
        for (int i = 0; i < 32; ++i) t[i] = v[i] + v[i ^ off];
        memcpy(v, t, sizeof(t));
    }
    return v[0];
}

/* Block sum of OC_NT partials in the kernel's tree order. */
static float tree_sum(const float* part) {
    float ws[32], v[32];
    for (int w = 0; w < OC_NW; ++w) {
        memcpy(v, part + 32 * w, sizeof(v));
        ws[w] = butterfly32(v);
    }
    for (int i = OC_NW; i < 32; ++i) ws[i] = 0.0f;
    return butterfly32(ws);
}

/* ------------------------------------------------------------------------- */
/* CDF                                                                       */
/* ------------------------------------------------------------------------- */
typedef struct {
    float m, s;
} ms_t;

static ms_t ms_merge(ms_t a, ms_t b) {
    ms_t r;
    if (a.m >= b.m) {
        r.m = a.m;
        r.s = a.s + b.s * oc_expf(b.m - a.m);
    } else {
        r.m = b.m;
        r.s = b.s + a.s * oc_expf(a.m - b.m);
    }
    return r;
}

#define OC_SUB 32

/* Subtile numerators e_i (fp16 bits, 0 past V) and partials (m_u, s_u) of a
 * row of V fp16 logits: e16 has ceil(V/32)*32 entries, ms 2*ceil(V/32). */
void oc_softmax_parts(const uint16_t* logits, int V, uint16_t* e16, float* ms) {
    const int nsub = (V + OC_SUB - 1) / OC_SUB;
    for (int u = 0; u < nsub; ++u) {
        const int a = u * OC_SUB, e = a + OC_SUB < V ? a + OC_SUB : V;
        float m = -INFINITY, s = 0.0f;
        for (int i = a; i < e; ++i) {
            const float x = oc_half_to_float(logits[i]);
            if (x > m) m = x;
        }
        for (int i = a; i < a + OC_SUB; ++i) {
            if (i < e) {
                e16[i] = oc_float_to_half(oc_expf(oc_half_to_float(logits[i]) - m));
                s = s + oc_half_to_float(e16[i]);
            } else {
                e16[i] = 0;
            }
        }
        ms[2 * u] = m;
        ms[2 * u + 1] = s;
    }
}

/* Row normaliser (M, S) from the subtile partials, in the kernels' order. */
static ms_t row_normaliser(const float* ms, int nsub) {
    ms_t th[OC_NT];
    ms_t w[32], t[32];
    for (int i = 0; i < OC_NT; ++i) {
        ms_t acc = {-INFINITY, 0.0f};
        for (int u = i; u < nsub; u += OC_NT) {
            ms_t p = {ms[2 * u], ms[2 * u + 1]};
            acc = ms_merge(acc, p);
        }
        th[i] = acc;
    }
    for (int k = 0; k < OC_NW; ++k) {
        ms_t* v = th + 32 * k;
        for (int off = 16; off > 0; off >>= 1) {
            for (int i = 0; i < 32; ++i) t[i] = ms_merge(v[i], v[i ^ off]);
            memcpy(v, t, sizeof(t));
        }
        w[k] = v[0];
    }
    for (int k = OC_NW; k < 32; ++k) {
        w[k].m = -INFINITY;
        w[k].s = 0.0f;
    }
    for (int off = 16; off > 0; off >>= 1) {
        for (int i = 0; i < 32; ++i) t[i] = ms_merge(w[i], w[i ^ off]);
        memcpy(w, t, sizeof(t));
    }
    return w[0];
}

/* source: 0 = fp16 logits (softmax), 1 = fp32 probabilities. */
static void cdf_row(const void* src, int kind, int V, int bits, int32_t* out) {
    const int64_t T = (int64_t)1 << bits;
    const float scale = (float)(T - V);
    float* q = (float*)malloc(sizeof(float) * (size_t)V);  /* q_i (logits) or p_i (probs) */
    int64_t total = 0;
    int amax = -1;
    float best = -INFINITY;

    if (kind == 0) {
        const uint16_t* x = (const uint16_t*)src;
        const int nsub = (V + OC_SUB - 1) / OC_SUB;
        float* ms = (float*)malloc(sizeof(float) * 2 * (size_t)nsub);
        uint16_t* e16 = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)nsub * OC_SUB);
        oc_softmax_parts(x, V, e16, ms);
        const ms_t n = row_normaliser(ms, nsub);
        const float inv = 1.0f / n.s;
        for (int u = 0; u < nsub; ++u) {
            const float gs = (oc_expf(ms[2 * u] - n.m) * inv) * scale;
            const int a = u * OC_SUB, e = a + OC_SUB < V ? a + OC_SUB : V;
            for (int i = a; i < e; ++i) q[i] = oc_half_to_float(e16[i]) * gs;
        }
        free(ms);
        free(e16);
        for (int i = 0; i < V; ++i) {
            const int c = (int)floorf(q[i]) + 1;
            out[i + 1] = c;
            total += c;
            if (q[i] > best) { best = q[i]; amax = i; }
        }
    } else {
        const float* x = (const float*)src;
        const int L = (V + OC_NT - 1) / OC_NT;
        float part[OC_NT];
        for (int t = 0; t < OC_NT; ++t) {
            int a = t * L < V ? t * L : V, e = a + L < V ? a + L : V;
            float s = 0.0f;
            for (int i = a; i < e; ++i) s = s + x[i];
            part[t] = s;
        }
        float S = tree_sum(part);
        if (S < 1e-30f) S = 1e-30f;
        for (int i = 0; i < V; ++i) {
            const float p = x[i] / S;
            const int c = (int)floorf(p * scale) + 1;
            out[i + 1] = c;
            total += c;
            if (p > best) { best = p; amax = i; }
        }
    }
    out[amax + 1] += (int32_t)(T - total);
    out[0] = 0;
    for (int i = 1; i <= V; ++i) out[i] += out[i - 1];
    free(q);
}

void oc_cdf_from_logits(const uint16_t* logits, int64_t stride, int rows, int V, int bits,
                        int32_t* out) {
    for (int r = 0; r < rows; ++r)
        cdf_row(logits + (int64_t)r * stride, 0, V, bits, out + (int64_t)r * (V + 1));
}

void oc_cdf_from_probs(const float* probs, int rows, int V, int bits, int32_t* out) {
    for (int r = 0; r < rows; ++r)
        cdf_row(probs + (int64_t)r * V, 1, V, bits, out + (int64_t)r * (V + 1));
}

/* (cdf[s], cdf[s+1]) of each row's symbol, from logits, without keeping the
 * CDF: out uint32 [rows, 2]. */
void oc_lohi_from_logits(const uint16_t* logits, int64_t stride, int rows, int V, int bits,
                         const int32_t* syms, uint32_t* out) {
    int32_t* row = (int32_t*)malloc(sizeof(int32_t) * (size_t)(V + 1));
    for (int r = 0; r < rows; ++r) {
        cdf_row(logits + (int64_t)r * stride, 0, V, bits, row);
        int s = syms[r];
        s = s < 0 ? 0 : (s >= V ? V - 1 : s);
        out[2 * r] = (uint32_t)row[s];
        out[2 * r + 1] = (uint32_t)row[s + 1];
    }
    free(row);
}

/* ------------------------------------------------------------------------- */
/* range coder                                                               */
/* ------------------------------------------------------------------------- */
#define HALF 0x80000000u
#define QTR 0x40000000u
#define THREE_QTR 0xC0000000u

typedef struct {
    uint8_t* buf;
    int64_t cap, nbits;
    int overflow;
} bw_t;

static void bw_put(bw_t* w, unsigned bit) {
    const int64_t byte = w->nbits >> 3;
    if (byte >= w->cap) {
        w->overflow = 1;
    } else if (bit & 1u) {
        w->buf[byte] |= (uint8_t)(0x80u >> (w->nbits & 7));
    }
    w->nbits++;
}

static void bw_emit(bw_t* w, unsigned bit, uint64_t pending) {
    bw_put(w, bit);
    for (uint64_t i = 0; i < pending; ++i) bw_put(w, bit ^ 1u);
}

/* Encode n symbols given their (lo, hi) intervals; returns the byte length
 * (ceil(bits/8)) or -1 if `cap` bytes were not enough.  `out` is zeroed here. */
int64_t oc_encode_lohi(const uint32_t* lohi, int64_t n, int bits, uint8_t* out, int64_t cap) {
    bw_t w = {out, cap, 0, 0};
    memset(out, 0, (size_t)cap);
    uint32_t low = 0, high = 0xFFFFFFFFu;
    uint64_t pending = 0;
    for (int64_t i = 0; i < n; ++i) {
        const uint64_t rng = (uint64_t)(high - low) + 1u;
        high = low + (uint32_t)((rng * lohi[2 * i + 1]) >> bits) - 1u;
        low = low + (uint32_t)((rng * lohi[2 * i]) >> bits);
        for (;;) {
            if (high < HALF) {
                bw_emit(&w, 0, pending); pending = 0;
                low <<= 1; high = (high << 1) | 1u;
            } else if (low >= HALF) {
                bw_emit(&w, 1, pending); pending = 0;
                low = (low - HALF) << 1; high = ((high - HALF) << 1) | 1u;
            } else if (low >= QTR && high < THREE_QTR) {
                pending++;
                low = (low - QTR) << 1; high = ((high - QTR) << 1) | 1u;
            } else {
                break;
            }
        }
    }
    pending++;
    bw_emit(&w, low < QTR ? 0u : 1u, pending);
    if (w.overflow) return -1;
    return (w.nbits + 7) >> 3;
}

int64_t oc_encode_cdf(const uint32_t* cdf, int64_t stride, const int32_t* syms, int64_t n,
                      int bits, uint8_t* out, int64_t cap) {
    uint32_t* lohi = (uint32_t*)malloc(sizeof(uint32_t) * 2 * (size_t)(n > 0 ? n : 1));
    for (int64_t i = 0; i < n; ++i) {
        lohi[2 * i] = cdf[i * stride + syms[i]];
        lohi[2 * i + 1] = cdf[i * stride + syms[i] + 1];
    }
    const int64_t r = oc_encode_lohi(lohi, n, bits, out, cap);
    free(lohi);
    return r;
}

typedef struct {
    const uint8_t* data;
    int64_t len;
    uint64_t pos; /* next bit to read */
    uint32_t low, high, value;
} oc_dec;

static unsigned br_get(oc_dec* d) {
    const int64_t byte = (int64_t)(d->pos >> 3);
    const unsigned sh = 7u - (unsigned)(d->pos & 7u);
    d->pos++;
    if (byte >= d->len) return 0u; /* zero bits past EOF */
    return (d->data[byte] >> sh) & 1u;
}

void oc_dec_init(oc_dec* d, const uint8_t* data, int64_t len) {
    d->data = data; d->len = len; d->pos = 0;
    d->low = 0; d->high = 0xFFFFFFFFu; d->value = 0;
    for (int i = 0; i < 32; ++i) d->value = (d->value << 1) | br_get(d);
}

int oc_dec_symbol(oc_dec* d, const uint32_t* cdf, int V, int bits) {
    const uint64_t rng = (uint64_t)(d->high - d->low) + 1u;
    const uint64_t off = (uint64_t)(d->value - d->low) + 1u;
    const uint64_t target = ((off << bits) - 1u) / rng;
    int lo = 0, hi = V;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if ((uint64_t)cdf[mid + 1] <= target) lo = mid + 1; else hi = mid;
    }
    const int sym = lo;
    d->high = d->low + (uint32_t)((rng * cdf[sym + 1]) >> bits) - 1u;
    d->low = d->low + (uint32_t)((rng * cdf[sym]) >> bits);
    for (;;) {
        if (d->high < HALF) {
        } else if (d->low >= HALF) {
            d->low -= HALF; d->high -= HALF; d->value -= HALF;
        } else if (d->low >= QTR && d->high < THREE_QTR) {
            d->low -= QTR; d->high -= QTR; d->value -= QTR;
        } else {
            break;
        }
        d->low <<= 1;
        d->high = (d->high << 1) | 1u;
        d->value = (d->value << 1) | br_get(d);
    }
    return sym;
}

void oc_decode_cdf(const uint8_t* in, int64_t len, const uint32_t* cdf, int64_t stride,
                   int64_t n, int V, int bits, int32_t* out) {
    oc_dec d;
    oc_dec_init(&d, in, len);
    for (int64_t i = 0; i < n; ++i) out[i] = oc_dec_symbol(&d, cdf + i * stride, V, bits);
}

int oc_dec_size(void) { return (int)sizeof(oc_dec); }
