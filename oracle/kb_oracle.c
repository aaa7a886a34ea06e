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
 *     ties), evaluated in the fixed order the GPU kernel uses so that the
 *     result is bit-identical to it:
 *       - NT = 512 virtual threads, thread t owns [t*L, min((t+1)*L, V)),
 *         L = ceil(V/NT), and sums its segment left to right;
 *       - partials meet in a xor butterfly over 32 lanes (offsets 16..1),
 *         then the same butterfly over the 16 warp results (zero padded);
 *       - exp is oc_expf below (the same algorithm as the kernel's kb_expf).
 *     The numpy reference (cdf.py) sums in numpy's pairwise order, so it can
 *     differ from this in the last bit of a sum and hence by +-1 in rare
 *     counts; tests compare against it with that allowance and against this
 *     file bit for bit.
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

/* Cody-Waite reduction with a 12-bit ln2 head; degree-6 Taylor polynomial;
 * 2^n through the exponent field.  Same algorithm and constants as the
 * kernel-side kb_expf; every operation is a single IEEE rounding. */
float oc_expf(float x) {
    if (!(x >= -86.0f)) return 0.0f;
    const float LOG2E = bits_f(0x3fb8aa3bu);
    const float LN2_HI = bits_f(0x3f317000u);
    const float LN2_LO = bits_f(0x3805fdf4u);
    const float n = rintf(x * LOG2E);
    float r = fmaf(-n, LN2_HI, x);
    r = fmaf(-n, LN2_LO, r);
    float p = 1.0f / 720.0f;
    p = fmaf(p, r, 1.0f / 120.0f);
    p = fmaf(p, r, 1.0f / 24.0f);
    p = fmaf(p, r, 1.0f / 6.0f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    return p * bits_f((uint32_t)((int)n + 127) << 23);
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
/* p_i source: 0 = fp16 logits (softmax), 1 = fp32 probabilities. */
static void cdf_row(const void* src, int kind, int V, int bits, int32_t* out) {
    const int L = (V + OC_NT - 1) / OC_NT;
    const int64_t T = (int64_t)1 << bits;
    const float scale = (float)(T - V);
    float* vals = (float*)malloc(sizeof(float) * (size_t)V);
    float part[OC_NT];
    float m = -INFINITY, inv = 0.0f, S = 0.0f;

    if (kind == 0) {
        const uint16_t* x = (const uint16_t*)src;
        for (int i = 0; i < V; ++i) {
            vals[i] = oc_half_to_float(x[i]);
            if (vals[i] > m) m = vals[i];
        }
        for (int t = 0; t < OC_NT; ++t) {
            int a = t * L < V ? t * L : V, e = a + L < V ? a + L : V;
            float s = 0.0f;
            for (int i = a; i < e; ++i) s = s + oc_expf(vals[i] - m);
            part[t] = s;
        }
        S = tree_sum(part);
        inv = 1.0f / S;
    } else {
        const float* x = (const float*)src;
        for (int t = 0; t < OC_NT; ++t) {
            int a = t * L < V ? t * L : V, e = a + L < V ? a + L : V;
            float s = 0.0f;
            for (int i = a; i < e; ++i) s = s + x[i];
            part[t] = s;
        }
        S = tree_sum(part);
        if (S < 1e-30f) S = 1e-30f;
        memcpy(vals, x, sizeof(float) * (size_t)V);
    }

    int64_t total = 0;
    int amax = -1;
    float bp = -INFINITY;
    for (int i = 0; i < V; ++i) {
        const float p = kind == 0 ? oc_expf(vals[i] - m) * inv : vals[i] / S;
        const int c = (int)floorf(p * scale) + 1;
        out[i + 1] = c;
        total += c;
        if (p > bp) { bp = p; amax = i; }
    }
    out[amax + 1] += (int32_t)(T - total);
    out[0] = 0;
    for (int i = 1; i <= V; ++i) out[i] += out[i - 1];
    free(vals);
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
