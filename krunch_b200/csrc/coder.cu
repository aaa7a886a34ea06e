// Range coder kernels: one lane per stream.
//
// The arithmetic (coder.cuh) follows krunch_ac/cpu_reference.py exactly.
//
// Differences from the reference kernels (encode_kernel.cu, decode_kernel.cu)
// are in execution only: bits are gathered in a register and stored a byte at
// a time instead of a global read-modify-write per bit, many streams run in
// parallel (one thread each), and the encoder can consume pre-narrowed
// (lo, hi) intervals so the full [rows, V+1] CDF never exists in memory.
#include "coder.cuh"
#include "profile.cuh"

namespace kb {

// ----------------------------------------------------------------------------
// Kernels
// ----------------------------------------------------------------------------
__global__ void k_encode_init(uint32_t* st, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        st[4 * i + 0] = 0u;
        st[4 * i + 1] = 0xFFFFFFFFu;
        st[4 * i + 2] = 0u;
        st[4 * i + 3] = 0u;
    }
}

// Full-CDF encode: stream b consumes rows [b*rows_per, (b+1)*rows_per) when
// batched with one row per stream, or all n rows for the single-stream case.
__global__ void k_encode_cdf(const int32_t* __restrict__ cdf, int64_t stride,
                             const int32_t* __restrict__ sym, int rows_per_stream, int B,
                             int bits, uint8_t* out, int64_t out_bytes,
                             const int64_t* __restrict__ offs, uint32_t* st) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    int64_t off, lim;
    stream_window(out_bytes, offs, b, off, lim);
    uint32_t* s4 = st + 4 * b;
    Enc e{s4[0], s4[1], s4[2]};
    BitWriter w;
    w.open(out + off, lim, s4[3]);
    for (int i = 0; i < rows_per_stream; ++i) {
        const int64_t row = (int64_t)b * rows_per_stream + i;
        const int s = sym[row];
        const int32_t* c = cdf + row * stride;
        enc_symbol(e, w, (uint32_t)c[s], (uint32_t)c[s + 1], bits);
    }
    w.close();
    s4[0] = e.low;
    s4[1] = e.high;
    s4[2] = e.pending;
    s4[3] = w.bit_offset;
}

__global__ void k_encode_lohi(const uint32_t* __restrict__ lohi, int B, int T,
                              const int32_t* __restrict__ n_valid, int bits, uint8_t* out,
                              int64_t out_bytes, const int64_t* __restrict__ offs,
                              uint32_t* st) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const int n = n_valid ? min(max(n_valid[b], 0), T) : T;
    int64_t off, lim;
    stream_window(out_bytes, offs, b, off, lim);
    uint32_t* s4 = st + 4 * b;
    Enc e{s4[0], s4[1], s4[2]};
    BitWriter w;
    w.open(out + off, lim, s4[3]);
    const uint2* p = reinterpret_cast<const uint2*>(lohi) + (int64_t)b * T;
    // Intervals are fetched 16 at a time into registers so that the loads of
    // a block are in flight together instead of one per symbol.
    constexpr int BLK = 16;
    int t = 0;
    for (; t + BLK <= n; t += BLK) {
        uint2 iv[BLK];
#pragma unroll
        for (int j = 0; j < BLK; ++j) iv[j] = __ldg(p + t + j);
#pragma unroll
        for (int j = 0; j < BLK; ++j) enc_symbol(e, w, iv[j].x, iv[j].y, bits);
    }
    for (; t < n; ++t) {
        const uint2 iv = __ldg(p + t);
        enc_symbol(e, w, iv.x, iv.y, bits);
    }
    w.close();
    s4[0] = e.low;
    s4[1] = e.high;
    s4[2] = e.pending;
    s4[3] = w.bit_offset;
}

// Flush: pending+1 bits of (low < QTR ? 0 : 1) (cpu_reference.py:141-146).
__global__ void k_encode_finalize(uint8_t* out, int64_t out_bytes,
                                  const int64_t* __restrict__ offs, uint32_t* st, int B) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    int64_t off, lim;
    stream_window(out_bytes, offs, b, off, lim);
    uint32_t* s4 = st + 4 * b;
    BitWriter w;
    w.open(out + off, lim, s4[3]);
    const uint32_t bit = (s4[0] < RC_QTR) ? 0u : 1u;
    w.emit(bit, s4[2] + 1u);  // one bit, then pending+1 inverted bits
    w.close();
    s4[2] = 0u;
    s4[3] = w.bit_offset;
}

__global__ void k_decode_init(const uint8_t* in, int64_t in_bytes,
                              const int64_t* __restrict__ offs, uint32_t* st, int B) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    int64_t off, lim;
    stream_window(in_bytes, offs, b, off, lim);
    BitReader r{in + off, lim, 0u};
    uint32_t v = 0;
    v = r.get(32);
    uint32_t* s4 = st + 4 * b;
    s4[0] = 0u;
    s4[1] = 0xFFFFFFFFu;
    s4[2] = v;
    s4[3] = r.bit_offset;
}

__global__ void k_decode_cdf(const int32_t* __restrict__ cdfs, int64_t stride, int V, int bits,
                             const uint8_t* in, int64_t in_bytes,
                             const int64_t* __restrict__ offs, uint32_t* st,
                             int32_t* out_syms, int B) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    int64_t off, lim;
    stream_window(in_bytes, offs, b, off, lim);
    uint32_t* s4 = st + 4 * b;
    Dec d{s4[0], s4[1], s4[2]};
    BitReader r{in + off, lim, s4[3]};
    const int32_t* c = cdfs + (int64_t)b * stride;
    const uint32_t target = dec_target(d, bits);
    const int sym = cdf_search(c, V, target);
    dec_narrow(d, r, (uint32_t)c[sym], (uint32_t)c[sym + 1], bits);
    out_syms[b] = sym;
    s4[0] = d.low;
    s4[1] = d.high;
    s4[2] = d.value;
    s4[3] = r.bit_offset;
}

static inline bool bits_ok(int bits) { return bits >= 1 && bits <= 30; }

}  // namespace kb

using namespace kb;

static inline int grid_for(int n, int block) { return (n + block - 1) / block; }

extern "C" int kb_coder_encode_init(uint32_t* states, int n, void* stream) {
    if (!states || n < 0) return KB_ERR_ARG;
    if (n == 0) return KB_OK;
    k_encode_init<<<grid_for(n, 128), 128, 0, as_stream(stream)>>>(states, n);
    return launch_status();
}

extern "C" int kb_coder_encode_cdf(const int32_t* cdf, int64_t stride, const int32_t* symbols,
                                   int n, int bits, uint8_t* out, int64_t out_bytes,
                                   uint32_t* state, void* stream) {
    if (!cdf || !symbols || !out || !state || n < 0 || stride < 2 || !bits_ok(bits))
        return KB_ERR_ARG;
    if (n == 0) return KB_OK;
    k_encode_cdf<<<1, 1, 0, as_stream(stream)>>>(cdf, stride, symbols, n, 1, bits, out,
                                                 out_bytes, nullptr, state);
    return launch_status();
}

extern "C" int kb_coder_encode_cdf_batched(const int32_t* cdfs, int64_t stride,
                                           const int32_t* symbols, int B, int bits,
                                           uint8_t* out, int64_t out_bytes,
                                           const int64_t* offs, uint32_t* states,
                                           void* stream) {
    if (!cdfs || !symbols || !out || !states || B < 0 || stride < 2 || !bits_ok(bits))
        return KB_ERR_ARG;
    if (B > 1 && !offs) return KB_ERR_ARG;
    if (B == 0) return KB_OK;
    k_encode_cdf<<<grid_for(B, 64), 64, 0, as_stream(stream)>>>(
        cdfs, stride, symbols, 1, B, bits, out, out_bytes, offs, states);
    return launch_status();
}

extern "C" int kb_coder_encode_lohi(const uint32_t* lohi, int B, int T, const int32_t* n_valid,
                                    int bits, uint8_t* out, int64_t out_bytes,
                                    const int64_t* offs, uint32_t* states, void* stream) {
    if (!lohi || !out || !states || B < 0 || T < 0 || !bits_ok(bits)) return KB_ERR_ARG;
    if (B > 1 && !offs) return KB_ERR_ARG;
    if (B == 0 || T == 0) return KB_OK;
    if (((uintptr_t)lohi & 7u) != 0) return KB_ERR_ALIGN;
    ProfScope ps(PH_ENCODE, as_stream(stream), (double)B * T * 8.0);
    k_encode_lohi<<<grid_for(B, 32), 32, 0, as_stream(stream)>>>(lohi, B, T, n_valid, bits, out,
                                                                 out_bytes, offs, states);
    return launch_status();
}

extern "C" int kb_coder_encode_finalize(uint8_t* out, int64_t out_bytes, const int64_t* offs,
                                        uint32_t* states, int B, void* stream) {
    if (!out || !states || B < 0) return KB_ERR_ARG;
    if (B > 1 && !offs) return KB_ERR_ARG;
    if (B == 0) return KB_OK;
    k_encode_finalize<<<grid_for(B, 64), 64, 0, as_stream(stream)>>>(out, out_bytes, offs,
                                                                      states, B);
    return launch_status();
}

extern "C" int kb_coder_decode_init(const uint8_t* in, int64_t in_bytes, const int64_t* offs,
                                    uint32_t* states, int B, void* stream) {
    if (!in || !states || B < 0) return KB_ERR_ARG;
    if (B > 1 && !offs) return KB_ERR_ARG;
    if (B == 0) return KB_OK;
    k_decode_init<<<grid_for(B, 64), 64, 0, as_stream(stream)>>>(in, in_bytes, offs, states, B);
    return launch_status();
}

extern "C" int kb_coder_decode_cdf(const int32_t* cdfs, int64_t stride, int V, int bits,
                                   const uint8_t* in, int64_t in_bytes, const int64_t* offs,
                                   uint32_t* states, int32_t* out_syms, int B, void* stream) {
    if (!cdfs || !in || !states || !out_syms || B < 0 || V < 1 || stride < V + 1 ||
        !bits_ok(bits))
        return KB_ERR_ARG;
    if (B > 1 && !offs) return KB_ERR_ARG;
    if (B == 0) return KB_OK;
    k_decode_cdf<<<grid_for(B, 64), 64, 0, as_stream(stream)>>>(cdfs, stride, V, bits, in,
                                                                in_bytes, offs, states,
                                                                out_syms, B);
    return launch_status();
}
