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
struct BitWriter {
    uint8_t* base;       // stream base
    int64_t limit;       // bytes writable from base (<= 0: nothing writable)
    uint32_t bit_offset; // absolute bit position inside the stream
    uint32_t acc;        // bits of the current partial byte (right-aligned)
    int nb;              // number of bits in acc

    __device__ void open(uint8_t* b, int64_t lim, uint32_t off) {
        base = b;
        limit = lim;
        bit_offset = off;
        nb = (int)(off & 7u);
        const int64_t byte = off >> 3;
        acc = (nb && byte < limit) ? (uint32_t)(base[byte] >> (8 - nb)) : 0u;
    }
    __device__ __forceinline__ void put(uint32_t bit) {
        acc = (acc << 1) | (bit & 1u);
        ++nb;
        ++bit_offset;
        if (nb == 8) {
            const int64_t byte = (int64_t)((bit_offset - 1) >> 3);
            if (byte < limit) base[byte] = (uint8_t)acc;
            acc = 0;
            nb = 0;
        }
    }
    // Emit `bit` followed by `pending` copies of its complement
    // (cpu_reference._emit, cpu_reference.py:150-154).
    __device__ __forceinline__ void emit(uint32_t bit, uint32_t pending) {
        put(bit);
        const uint32_t inv = bit ^ 1u;
        for (uint32_t i = 0; i < pending; ++i) put(inv);
    }
    // Store the trailing partial byte, zero-padded on the right.
    __device__ void close() {
        if (nb) {
            const int64_t byte = (int64_t)(bit_offset >> 3);
            if (byte < limit) base[byte] = (uint8_t)(acc << (8 - nb));
        }
    }
};

struct BitReader {
    const uint8_t* base;
    int64_t limit;
    uint32_t bit_offset;

    __device__ __forceinline__ uint32_t get() {
        const int64_t byte = (int64_t)(bit_offset >> 3);
        const uint32_t sh = 7u - (bit_offset & 7u);
        ++bit_offset;
        if (byte >= limit) return 0u;  // past the buffer: zero bits
        return (uint32_t)(base[byte] >> sh) & 1u;
    }
};

// ----------------------------------------------------------------------------
// Encoder / decoder steps
// ----------------------------------------------------------------------------
struct Enc {
    uint32_t low, high, pending;
};

__device__ __forceinline__ void enc_symbol(Enc& s, BitWriter& w, uint32_t lo, uint32_t hi,
                                           int bits) {
    const uint64_t rng = (uint64_t)(s.high - s.low) + 1ull;
    s.high = s.low + (uint32_t)((rng * (uint64_t)hi) >> bits) - 1u;
    s.low = s.low + (uint32_t)((rng * (uint64_t)lo) >> bits);
    for (;;) {
        if (s.high < RC_HALF) {
            w.emit(0u, s.pending);
            s.pending = 0;
            s.low <<= 1;
            s.high = (s.high << 1) | 1u;
        } else if (s.low >= RC_HALF) {
            w.emit(1u, s.pending);
            s.pending = 0;
            s.low = (s.low - RC_HALF) << 1;
            s.high = ((s.high - RC_HALF) << 1) | 1u;
        } else if (s.low >= RC_QTR && s.high < RC_THREE_QTR) {
            ++s.pending;
            s.low = (s.low - RC_QTR) << 1;
            s.high = ((s.high - RC_QTR) << 1) | 1u;
        } else {
            break;
        }
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
    for (;;) {
        if (s.high < RC_HALF) {
        } else if (s.low >= RC_HALF) {
            s.low -= RC_HALF;
            s.high -= RC_HALF;
            s.value -= RC_HALF;
        } else if (s.low >= RC_QTR && s.high < RC_THREE_QTR) {
            s.low -= RC_QTR;
            s.high -= RC_QTR;
            s.value -= RC_QTR;
        } else {
            break;
        }
        s.low <<= 1;
        s.high = (s.high << 1) | 1u;
        s.value = (s.value << 1) | r.get();
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
