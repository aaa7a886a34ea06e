// Device-side range coder primitives shared by coder.cu and cdf.cu.
//
// Arithmetic follows the 32-bit E1/E2/E3 range coder of
// krunch_ac/cpu_reference.py:91-147 (encode) and 161-211 (decode) exactly:
//   rng  = high - low + 1
//   high = low + (rng * cdf_hi >> bits) - 1
//   low  = low + (rng * cdf_lo >> bits)
// followed by renormalisation; bits are packed MSB-first.
#pragma once
#include "kb_common.cuh"

namespace kb {

// ----------------------------------------------------------------------------
// Bit I/O
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t low_mask(int n) { return n >= 32 ? 0xFFFFFFFFu : ((1u << n) - 1u); }

struct BitWriter {
    uint8_t* base;       // stream base
    int64_t limit;       // bytes writable from base (<= 0: nothing writable)
    uint32_t bit_offset; // absolute bit position inside the stream
    int64_t byte_pos;    // first byte not yet stored
    uint64_t acc;        // pending bits, right-aligned
    int nb;              // number of pending bits (< 8 between calls)

    __device__ void open(uint8_t* b, int64_t lim, uint32_t off) {
        base = b;
        limit = lim;
        bit_offset = off;
        byte_pos = off >> 3;
        nb = (int)(off & 7u);
        acc = (nb && byte_pos < limit) ? (uint64_t)(base[byte_pos] >> (8 - nb)) : 0u;
    }
    // Append the low n (<= 32) bits of v, most significant first.
    __device__ __forceinline__ void put(uint32_t v, int n) {
        acc = (acc << n) | (uint64_t)(v & low_mask(n));
        nb += n;
        bit_offset += (uint32_t)n;
        while (nb >= 8) {
            nb -= 8;
            if (byte_pos < limit) base[byte_pos] = (uint8_t)(acc >> nb);
            ++byte_pos;
        }
    }
    // `bit` followed by `pending` copies of its complement
    // (cpu_reference._emit, cpu_reference.py:150-154).
    __device__ __forceinline__ void emit(uint32_t bit, uint32_t pending) {
        put(bit, 1);
        const uint32_t fill = bit ? 0u : 0xFFFFFFFFu;
        while (pending >= 32) {
            put(fill, 32);
            pending -= 32;
        }
        if (pending) put(fill, (int)pending);
    }
    // Store the trailing partial byte, zero-padded on the right.
    __device__ void close() {
        if (nb && byte_pos < limit) base[byte_pos] = (uint8_t)(acc << (8 - nb));
    }
};

struct BitReader {
    const uint8_t* base;
    int64_t limit;
    uint32_t bit_offset;

    __device__ __forceinline__ uint32_t byte_at(int64_t i) const {
        return i < limit ? (uint32_t)base[i] : 0u;  // past the buffer: zero bits
    }
    // Next n (1..32) bits, most significant first.
    __device__ __forceinline__ uint32_t get(int n) {
        const int64_t b = bit_offset >> 3;
        const int sh = (int)(bit_offset & 7u);
        uint64_t w = ((uint64_t)byte_at(b) << 32) | (byte_at(b + 1) << 24) | (byte_at(b + 2) << 16) |
                     (byte_at(b + 3) << 8) | byte_at(b + 4);
        bit_offset += (uint32_t)n;
        return (uint32_t)((w << sh) >> (40 - n)) & low_mask(n);
    }
};

// ----------------------------------------------------------------------------
// Encoder / decoder steps.  Renormalisation moves whole runs at once: the n
// leading bits on which low and high agree are the n E1/E2 steps of the
// reference loop, and the following run of straddling bits (low = 01..1,
// high = 10..0) is its E3 steps; no E1/E2 step can follow an E3 step, so one
// pass of each reproduces the reference's loop exactly.
// ----------------------------------------------------------------------------
struct Enc {
    uint32_t low, high, pending;
};

__device__ __forceinline__ void enc_symbol(Enc& s, BitWriter& w, uint32_t lo, uint32_t hi,
                                           int bits) {
    const uint64_t rng = (uint64_t)(s.high - s.low) + 1ull;
    s.high = s.low + (uint32_t)((rng * (uint64_t)hi) >> bits) - 1u;
    s.low = s.low + (uint32_t)((rng * (uint64_t)lo) >> bits);
    const int n = __clz(s.low ^ s.high);  // E1/E2 steps (high > low, so n < 32)
    if (n > 0) {
        const uint32_t top = s.low >> (32 - n);
        w.emit(top >> (n - 1), s.pending);
        if (n > 1) w.put(top, n - 1);
        s.pending = 0;
        s.low <<= n;
        s.high = (s.high << n) | low_mask(n);
    }
    if (s.low >= RC_QTR && s.high < RC_THREE_QTR) {  // E3 steps
        const int k = min(__clz(~(s.low << 1)), __clz(s.high << 1));
        s.pending += (uint32_t)k;
        s.low = (s.low << k) & 0x7FFFFFFFu;
        s.high = (s.high << k) | 0x80000000u | low_mask(k);
    }
}

struct Dec {
    uint32_t low, high, value;
};

// target = ((value - low + 1) * T - 1) // rng  (cpu_reference.py:190-191)
__device__ __forceinline__ uint32_t dec_target(const Dec& s, int bits) {
    const uint64_t rng = (uint64_t)(s.high - s.low) + 1ull;
    const uint64_t off = (uint64_t)(s.value - s.low) + 1ull;
    return (uint32_t)(((off << bits) - 1ull) / rng);
}

__device__ __forceinline__ void dec_narrow(Dec& s, BitReader& r, uint32_t lo, uint32_t hi,
                                           int bits) {
    const uint64_t rng = (uint64_t)(s.high - s.low) + 1ull;
    s.high = s.low + (uint32_t)((rng * (uint64_t)hi) >> bits) - 1u;
    s.low = s.low + (uint32_t)((rng * (uint64_t)lo) >> bits);
    const int n = __clz(s.low ^ s.high);
    if (n > 0) {
        s.low <<= n;
        s.high = (s.high << n) | low_mask(n);
        s.value = (s.value << n) | r.get(n);
    }
    if (s.low >= RC_QTR && s.high < RC_THREE_QTR) {
        // k E3 steps: x -> ((x - QTR) << 1) | bit, i.e. ((x << k) ^ HALF) | next bits
        const int k = min(__clz(~(s.low << 1)), __clz(s.high << 1));
        s.low = (s.low << k) & 0x7FFFFFFFu;
        s.high = (s.high << k) | 0x80000000u | low_mask(k);
        s.value = ((s.value << k) ^ 0x80000000u) | r.get(k);
    }
}

// Largest sym in [0, V) with cdf[sym] <= target (cpu_reference._bsearch).
__device__ __forceinline__ int cdf_search(const int32_t* cdf, int V, uint32_t target) {
    int lo = 0, hi = V;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if ((uint32_t)cdf[mid + 1] <= target)
            lo = mid + 1;
        else
            hi = mid;
    }
    return lo;
}

// Used by the fused CDF+decode kernel (cdf.cu).
__device__ __forceinline__ void decode_apply(uint32_t* st, const uint8_t* base, int64_t limit, uint32_t lo,
                             uint32_t hi, int bits) {
    Dec s{st[0], st[1], st[2]};
    BitReader r{base, limit, st[3]};
    dec_narrow(s, r, lo, hi, bits);
    st[0] = s.low;
    st[1] = s.high;
    st[2] = s.value;
    st[3] = r.bit_offset;
}
__device__ __forceinline__ uint32_t decode_target(const uint32_t* st, int bits) {
    Dec s{st[0], st[1], st[2]};
    return dec_target(s, bits);
}

// Byte window of stream b inside a buffer of `total` bytes.
__device__ __forceinline__ void stream_window(int64_t total, const int64_t* offs, int b,
                                              int64_t& off, int64_t& lim) {
    off = offs ? offs[b] : 0;
    lim = total - off;
}

}  // namespace kb
