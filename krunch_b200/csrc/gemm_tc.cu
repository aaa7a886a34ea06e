// tcgen05 GEMM for sm_100a: out[M,N] = epi(A[M,K] @ W[N,K]^T), fp16 in,
// fp32 accumulation in TMEM, fused RWKV epilogues.
//
// Persistent, warp-specialised CTA (one per SM):
//   warp 0      TMA producer: A 128x64 and W 256x64 tiles (128-byte swizzle)
//               into a 4-stage shared-memory ring, no cluster multicast;
//   warp 1      MMA issuer: 4 x tcgen05.mma 128x256x16 per stage into one of
//               two TMEM accumulators (2 x 256 fp32 columns);
//   warps 2..17 epilogue: each warp owns 32 TMEM lanes (warp % 4) and one
//               64-column quarter of the tile; tcgen05.ld, the fused epilogue,
//               16-byte stores.  Draining accumulator i overlaps the MMAs of
//               tile i+1.  The head's epilogue stores, instead of the logits,
//               e^(x - m_u) in fp16 for every 32-column subtile u together
//               with the subtile's (m_u, sum), so the CDF kernel needs no exp
//               per element (softmax_stats.cuh).
// Output tile (m, n) walks K from 0 to K in 64-wide blocks, 16 per MMA, for
// every M: a row's result does not depend on M or on the other rows (the
// M-invariance the decoder relies on, krunch_ac/cuda/det_matmul_tc*.cu).
// Every mbarrier wait is bounded; on expiry the CTA records an error code in
// g_tc_error, stops issuing work, frees its TMEM and returns.
#include <cudaTypedefs.h>

#include <mutex>

#include "epi_math.cuh"
#include "rwkv_ops.cuh"
#include "softmax_stats.cuh"
#include "tc_common.cuh"

namespace kb {

constexpr int TC_BM = 128, TC_BK = 64, TC_NT = 576;
constexpr int TC_EPI_WARPS = 16;
#ifndef TC_OUT_BUFS
#define TC_OUT_BUFS 1
#endif
#ifndef TC_HEAD_PAIRCVT
#define TC_HEAD_PAIRCVT 1  // head numerators converted two at a time
#endif
#ifndef TC_PAIR_AUTO
#define TC_PAIR_AUTO 1
#endif
#ifndef TC_MAX_BN
#define TC_MAX_BN 256
#endif
#ifndef TC_STAGE_BUDGET
#define TC_STAGE_BUDGET 196608
#endif
// Output staging per epilogue warp: a ring of TC_OUT_BUFS 2 KB tiles, so a
// warp stages the next chunk while the TMA store of the previous one still
// reads shared memory.
constexpr int TC_OUT_RING = TC_OUT_BUFS;
constexpr uint32_t TC_OUT_TILE = 2048;
constexpr uint32_t TC_STAGE_OUT = TC_OUT_TILE * TC_OUT_RING;
constexpr uint32_t TC_A_BYTES = TC_BM * TC_BK * 2;  // 16 KB

// Tile width BN in {256, 128, 64, 32}: 256 for large M; narrower tiles give
// a small-M launch (the decoder's B rows) more CTAs.  The K walk of an output
// element is the same for every BN.
// operand kinds: fp16, int8 (w8a8), bf16 (KB_BF16 model: bf16 weights and
// GEMM inputs; the kernel's tensor maps move 2-byte elements either way)
enum { TC_F16 = 0, TC_I8 = 1, TC_BF16 = 2 };

// PAIR: a cluster of two CTAs computes a 256-row x BN tile with cta_group::2
// MMAs; each CTA stages its 128 rows of A and BN / 2 rows of B.
template <int BN, int KIND, bool PAIR = false>
struct TcCfg {
    static_assert(BN == 256 || BN == 128 || BN == 64 || BN == 32, "tile width");
    static_assert(!PAIR || BN == 256, "CTA pairs use 256-column tiles");
    // a K block is one 128-byte swizzle row: 64 fp16 or 128 int8 elements
    static constexpr int KEL = KIND == TC_I8 ? 128 : 64;
    static constexpr int B_ROWS = PAIR ? BN / 2 : BN;  // rows of B staged by this CTA
    static constexpr int BM = PAIR ? 2 * TC_BM : TC_BM;  // rows of an output tile
    static constexpr uint32_t B_BYTES = B_ROWS * 128;
    static constexpr uint32_t STAGE_BYTES = TC_A_BYTES + B_BYTES;
    static constexpr int STAGES =
        (TC_STAGE_BUDGET / STAGE_BYTES) < 8 ? (TC_STAGE_BUDGET / STAGE_BYTES) : 8;
    static constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulators
    static constexpr size_t SMEM = (size_t)STAGES * STAGE_BYTES +
                                   TC_EPI_WARPS * TC_STAGE_OUT /*output staging*/ +
                                   1024 /*align*/ + 256 /*bars*/;
    static_assert(SMEM <= 232448, "shared memory per block");
    static constexpr uint32_t IDESC =
        KIND == TC_I8 ? tc::idesc_i8(BM, BN) : tc::idesc_f16(BM, BN, KIND == TC_BF16);
};

// Launch parameters of one GEMM (a __grid_constant__ kernel argument).
struct TcArgs {
    int M, N, K;
    void* out;
    int64_t ldo;
    const uint16_t* resid;
    const uint16_t* gate;
    int V;                    // head: valid vocabulary columns
    float2* stats;            // head: subtile partials
    int stats_stride;
    const float* a_scale[3];     // int8: dequantisation factor per row of A (per GEMM)
    const uint16_t* w_scale[3];  // int8: fp16 dequantisation factor per row of W (per GEMM)
};

// Tensor maps of a launch: A, W and output per GEMM.  One GEMM uses entry 0;
// the grouped k/v/r launch (TC_EPI_KVR) runs three GEMMs of the same shape
// over one tile space.
struct TcMaps {
    CUtensorMap a[3], b[3], o[3];
};

// Internal epilogue id of the grouped k/v/r launch: GEMMs 0 and 1 store
// fp32 (KB_EPI_F32: k and v), GEMM 2 stores fp16 sigmoid (KB_EPI_SIGMOID: r),
// as the reference's 3-way kernel does (det_matmul_tc_3way_async.cu:50-251).
constexpr int TC_EPI_KVR = 7;

__device__ int g_tc_error = 0;

struct TcBars {
    uint64_t full[8];
    uint64_t empty[8];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint32_t tmem_base;
    int abort;
};

__device__ __forceinline__ void tc_fail(TcBars* b, int code) {
    atomicExch(&g_tc_error, code);
    *reinterpret_cast<volatile int*>(&b->abort) = 1;
}
__device__ __forceinline__ bool tc_aborted(TcBars* b) {
    return *reinterpret_cast<volatile int*>(&b->abort) != 0;
}

__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

#ifdef TC_DIAG
// cycles spent in each wait, summed over the threads that wait:
// 0 producer/empty, 1 mma/tempty, 2 mma/full, 3 epilogue/tfull,
// 4 epilogue/staging, 5 epilogue busy (tfull done -> tempty arrive), 6 mma loop
__device__ unsigned long long g_tc_diag[8];
}  // namespace kb
// diagnostic build only: copy (and optionally clear) the wait-cycle sums
extern "C" int kb_tc_diag(unsigned long long* host_out, int reset) {
    cudaDeviceSynchronize();
    if (cudaMemcpyFromSymbol(host_out, kb::g_tc_diag, sizeof(kb::g_tc_diag)) != cudaSuccess)
        return -1;
    if (reset) {
        static const unsigned long long z[8] = {};
        cudaMemcpyToSymbol(kb::g_tc_diag, z, sizeof(z));
    }
    return 0;
}
namespace kb {
#define DIAG_T0(v) const long long v = clock64()
#define DIAG_ADD(acc, v) acc += (unsigned long long)(clock64() - (v))
#define DIAG_FLUSH(i, acc) atomicAdd(&g_tc_diag[i], acc)
#else
#define DIAG_T0(v)
#define DIAG_ADD(acc, v)
#define DIAG_FLUSH(i, acc)
#endif

// Tile order: groups of TC_GROUP_M row blocks; inside a group the row block
// changes fastest, so the CTAs running at the same time share a few weight
// tiles (read from L2) and a few activation row blocks.
constexpr int TC_GROUP_M = 16;
template <int BN, int BM = TC_BM>
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& m0, int& n0) {
    const int per_group = TC_GROUP_M * num_n;
    const int g = t / per_group, r = t - g * per_group;
    const int gm = min(TC_GROUP_M, num_m - g * TC_GROUP_M);
    m0 = (g * TC_GROUP_M + r % gm) * BM;
    n0 = (r / gm) * BN;
}

// Output staging: each epilogue warp owns 2 KB of shared memory holding a
// 32-row x 64-byte tile in the 64-byte swizzle TMA expects (16-byte chunk j
// of row r at chunk position j ^ ((r >> 1) & 3)); one elected lane writes the
// tile to global memory with a TMA store.  Rows past M are clipped by TMA.
__device__ __forceinline__ void stage_row64(unsigned char* st, int r, const uint32_t (&w)[16]) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(st + r * 64 + ((j ^ ((r >> 1) & 3)) << 4)) =
            make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
}

// Warp-wide: the next tile of this warp's staging ring, once the store
// issued from it TC_OUT_RING stores ago has finished reading it.
__device__ __forceinline__ unsigned char* out_tile(unsigned char* ring, uint32_t& n, int lane) {
    if (lane == 0) {
        DIAG_T0(t0);
        tc::bulk_wait_read_max<TC_OUT_RING - 1>();
#ifdef TC_DIAG
        atomicAdd(&g_tc_diag[4], (unsigned long long)(clock64() - t0));
#endif
    }
    __syncwarp();
    return ring + (n++ % TC_OUT_RING) * TC_OUT_TILE;
}

// Warp-wide: stage this lane's row in a free staging tile (out_tile()),
// store the tile at (c0, r0).
__device__ __forceinline__ void stage_and_store(unsigned char* st, int lane,
                                                const uint32_t (&w)[16], const CUtensorMap* map,
                                                int c0, int r0) {
    stage_row64(st, lane, w);
    tc::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        tc::tma_store_2d(map, st, c0, r0);
        tc::bulk_commit();
    }
}

// Warp-wide coalesced read of a 32-row x 32-column fp16 tile (rows from r0,
// rows >= M read as zero) through a free staging tile; lane i gets row r0 + i.
__device__ __forceinline__ void load_tile_rows(const uint16_t* src, int64_t ld, int64_t r0, int c0,
                                               int M, unsigned char* st, int lane,
                                               uint4 (&out)[4]) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int idx = k * 32 + lane, r = idx >> 2, j = idx & 3;
        const int64_t gr = r0 + r;
        const uint4 v = gr < M ? *reinterpret_cast<const uint4*>(src + gr * ld + c0 + j * 8)
                               : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(st + r * 64 + ((j ^ ((r >> 1) & 3)) << 4)) = v;
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 4; ++j)
        out[j] = *reinterpret_cast<const uint4*>(st + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4));
    __syncwarp();
}

// Epilogue values of 32 consecutive columns of one row as 16 words of fp16
// pairs (bf16 pairs when OUT_BF; non-F32 epilogues); rv / gv: the row's
// residual / gate values.
template <int EPI, bool OUT_BF = false>
__device__ __forceinline__ void tc_epi_pack(const uint32_t (&acc)[32], const uint4 (&rv)[4],
                                            const uint4 (&gv)[4], uint32_t (&w)[16]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t* rw = reinterpret_cast<const uint32_t*>(&rv[j]);
        const uint32_t* gw = reinterpret_cast<const uint32_t*>(&gv[j]);
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            float y0 = u2f(acc[8 * j + 2 * h]), y1 = u2f(acc[8 * j + 2 * h + 1]);
            if (EPI == KB_EPI_SIGMOID) {
                y0 = epi_sigmoid(y0);
                y1 = epi_sigmoid(y1);
            } else if (EPI == KB_EPI_RELU_SQ) {
                y0 = epi_relu_sq(y0);
                y1 = epi_relu_sq(y1);
            } else if (EPI == KB_EPI_RESID || EPI == KB_EPI_GATE_RESID) {
                const __half2 rr = *reinterpret_cast<const __half2*>(&rw[h]);
                float g0 = 1.0f, g1 = 1.0f;
                if (EPI == KB_EPI_GATE_RESID) {
                    const __half2 gg = *reinterpret_cast<const __half2*>(&gw[h]);
                    g0 = __low2float(gg);
                    g1 = __high2float(gg);
                }
                y0 = epi_gate_resid(g0, y0, __low2float(rr));
                y1 = epi_gate_resid(g1, y1, __high2float(rr));
            }
            if (OUT_BF) {
                const __nv_bfloat162 p = __floats2bfloat162_rn(y0, y1);
                w[4 * j + h] = *reinterpret_cast<const uint32_t*>(&p);
            } else {
                const __half2 p = __floats2half2_rn(y0, y1);
                w[4 * j + h] = *reinterpret_cast<const uint32_t*>(&p);
            }
        }
    }
}

// int8 accumulators of 32 columns -> fp32 values in place:
// y = (float(acc) * a_scale[row]) * float(w_scale[col]), rounded at each step.
__device__ __forceinline__ void dequant32(uint32_t (&v)[32], float sa, const uint16_t* ws) {
    const uint4* w4 = reinterpret_cast<const uint4*>(ws);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint4 q = __ldg(w4 + j);
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            const float2 sw = __half22float2(*reinterpret_cast<const __half2*>(&qw[h]));
            const int c = 8 * j + 2 * h;
            v[c] = __float_as_uint(epi_dequant((int)v[c], sa, sw.x));
            v[c + 1] = __float_as_uint(epi_dequant((int)v[c + 1], sa, sw.y));
        }
    }
}

// Non-head epilogue of one tile: this warp's 32-column chunks [c_lo, c_hi)
// of TMEM lane quadrant q, epilogue E, stored through mapO.
template <int E, int KIND>
__device__ __forceinline__ void epi_chunks(int c_lo, int c_hi, int n0, int N, int M, int m0,
                                           int q, int lane, uint32_t tbase, float sa,
                                           const uint16_t* w_scale, const CUtensorMap* mapO,
                                           const TcArgs& args, int64_t ldo, unsigned char* ring,
                                           uint32_t& nst) {
#pragma unroll 1
    for (int c = c_lo; c < c_hi; ++c) {
        const int col0 = n0 + c * 32;
        if (col0 >= N) break;
        uint32_t v[32];
        tc::tmem_ld32(tbase + (uint32_t)(c * 32), v);
        tc::tmem_ld_wait();
        if (KIND == TC_I8) dequant32(v, sa, w_scale + col0);
        if (E == KB_EPI_F32) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {  // two 16-column (64-byte) halves
                uint32_t w[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) w[j] = v[16 * h + j];
                stage_and_store(out_tile(ring, nst, lane), lane, w, mapO,
                                col0 + 16 * h, m0 + q * 32);
            }
        } else {
            uint32_t w[16];
            uint4 rv[4], gv[4];
            unsigned char* const st = out_tile(ring, nst, lane);
            if (E == KB_EPI_RESID || E == KB_EPI_GATE_RESID)
                load_tile_rows(args.resid, ldo, m0 + q * 32, col0, M, st, lane, rv);
            if (E == KB_EPI_GATE_RESID)
                load_tile_rows(args.gate, ldo, m0 + q * 32, col0, M, st, lane, gv);
            // a bf16 model's relu(k)^2 is the next GEMM's bf16 operand
            tc_epi_pack<E, KIND == TC_BF16 && E == KB_EPI_RELU_SQ>(v, rv, gv, w);
            stage_and_store(st, lane, w, mapO, col0, m0 + q * 32);
        }
    }
}

template <int EPI, int BN, int KIND, bool PAIR>
__global__ void __launch_bounds__(TC_NT, 1)
    k_gemm_tc(const __grid_constant__ TcMaps maps, const __grid_constant__ TcArgs args) {
    using Cfg = TcCfg<BN, KIND, PAIR>;
    constexpr int G = EPI == TC_EPI_KVR ? 3 : 1;  // GEMMs sharing the tile space
    const int M = args.M, N = args.N, K = args.K;
    const int64_t ldo = args.ldo;
    const int V = args.V, stats_stride = args.stats_stride;
    float2* const stats = args.stats;
    constexpr int TC_STAGES = Cfg::STAGES;
    constexpr uint32_t TC_STAGE_BYTES = Cfg::STAGE_BYTES;
    extern __shared__ unsigned char tc_smem_raw[];
    const uint32_t raw = tc::smem_addr(tc_smem_raw);
    unsigned char* smem = tc_smem_raw + (((raw + 1023u) & ~1023u) - raw);
    unsigned char* stage_out = smem + TC_STAGES * TC_STAGE_BYTES;  // 16 x TC_STAGE_OUT
    TcBars* bars = reinterpret_cast<TcBars*>(stage_out + TC_EPI_WARPS * TC_STAGE_OUT);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_n = (N + BN - 1) / BN;
    const int num_m = (M + Cfg::BM - 1) / Cfg::BM;
    const int tiles = num_m * num_n * G;  // tile t: GEMM t % G, position t / G
    const int KB = K / Cfg::KEL;
    // a pair walks the tiles as one unit; rank 1 holds rows 128..255 of each
    const uint32_t rank = PAIR ? tc::cluster_ctarank() : 0u;
    const int unit0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < TC_STAGES; ++s) {
            tc::mbar_init(&bars->full[s], 1);
            tc::mbar_init(&bars->empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            tc::mbar_init(&bars->tfull[a], 1);
            tc::mbar_init(&bars->tempty[a], PAIR ? 2 * TC_EPI_WARPS : TC_EPI_WARPS);
        }
        bars->abort = 0;
        tc::fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        for (int g = 0; g < G; ++g) {
            tc::prefetch_tmap(&maps.a[g]);
            tc::prefetch_tmap(&maps.b[g]);
            tc::prefetch_tmap(&maps.o[g]);
        }
    }
    if (warp == 1) {
        if (PAIR) tc::tmem_alloc_pair(&bars->tmem_base, Cfg::TMEM_COLS);
        else tc::tmem_alloc(&bars->tmem_base, Cfg::TMEM_COLS);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (PAIR) tc::cluster_sync();  // the peer's barriers are initialised
    tc::fence_after_sync();
    const uint32_t tmem = bars->tmem_base;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0, issued_parity = 0;  // per-stage bit masks
#ifdef TC_DIAG
            unsigned long long d_empty = 0;
#endif
            for (int t = unit0; t < tiles && !tc_aborted(bars); t += units) {
                int m0, n0;
                const int g = t % G;
                tile_coords<BN, Cfg::BM>(t / G, num_m, num_n, m0, n0);
                const CUtensorMap* mapA = &maps.a[g];
                const CUtensorMap* mapB = &maps.b[g];
                for (int kb = 0; kb < KB; ++kb) {
                    DIAG_T0(tw);
                    const bool okw = tc::mbar_wait(&bars->empty[stage], phase ^ 1u);
                    DIAG_ADD(d_empty, tw);
                    if (!okw) {
                        tc_fail(bars, 1);
                        break;
                    }
                    unsigned char* sa = smem + stage * TC_STAGE_BYTES;
                    if (PAIR) {
                        // both CTAs' bytes complete on the leader's barrier
                        const uint32_t fb = tc::mapa_shared(tc::smem_addr(&bars->full[stage]), 0);
                        if (rank == 0) tc::mbar_expect_tx(&bars->full[stage], 2 * TC_STAGE_BYTES);
                        tc::tma_load_2d_pair(sa, mapA, fb, kb * Cfg::KEL, m0 + (int)rank * TC_BM);
                        tc::tma_load_2d_pair(sa + TC_A_BYTES, mapB, fb, kb * Cfg::KEL,
                                             n0 + (int)rank * Cfg::B_ROWS);
                    } else {
                        tc::mbar_expect_tx(&bars->full[stage], TC_STAGE_BYTES);
                        tc::tma_load_2d(sa, mapA, &bars->full[stage], kb * Cfg::KEL, m0);
                        tc::tma_load_2d(sa + TC_A_BYTES, mapB, &bars->full[stage], kb * Cfg::KEL,
                                        n0);
                    }
                    issued |= 1u << stage;
                    issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == TC_STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            DIAG_FLUSH(0, d_empty);
            // Drain: every load this thread issued has landed before the CTA
            // exits (immediate on the normal path; bounded after an abort).
            // A pair's rank 1 sees its loads through the leader's barrier, so
            // it waits for the MMAs that consumed them.
            for (int s = 0; s < TC_STAGES; ++s)
                if (issued & (1u << s)) {
                    if (PAIR && rank != 0) tc::mbar_wait(&bars->empty[s], (issued_parity >> s) & 1u);
                    else tc::mbar_wait(&bars->full[s], (issued_parity >> s) & 1u);
                }
            // After an abort the leader may never consume (or see land) what
            // rank 1 loaded into its own shared memory: rank 1 then keeps its
            // shared memory alive for a bounded 100 us, far beyond a tile
            // load's flight time, before it may leave.
            if (PAIR && rank != 0 && tc_aborted(bars)) {
                unsigned long long t0, t1;
                asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
                do {
                    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
                } while (t1 - t0 < 100000ull);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (a pair's leader) ----------------
        if (lane == 0 && rank == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int i = 0;
#ifdef TC_DIAG
            unsigned long long d_tempty = 0, d_full = 0, d_loop = 0;
            DIAG_T0(tl);
#endif
            for (int t = unit0; t < tiles && !tc_aborted(bars); t += units, ++i) {
                const int a = i & 1;
                const uint32_t use = (uint32_t)(i >> 1);
                DIAG_T0(tw);
                const bool okt = tc::mbar_wait(&bars->tempty[a], (use & 1u) ^ 1u);
                DIAG_ADD(d_tempty, tw);
                if (!okt) {
                    tc_fail(bars, 2);
                    break;
                }
                tc::fence_after_sync();
                const uint32_t d = tmem + (uint32_t)(a * BN);
                bool ok = true;
                for (int kb = 0; kb < KB; ++kb) {
                    DIAG_T0(tf);
                    const bool okf = tc::mbar_wait(&bars->full[stage], phase);
                    DIAG_ADD(d_full, tf);
                    if (!okf) {
                        tc_fail(bars, 3);
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t sa = tc::smem_addr(smem + stage * TC_STAGE_BYTES);
                    const uint32_t sb = sa + TC_A_BYTES;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {  // 32 bytes of K per MMA
                        const uint64_t ad = tc::sdesc_k128(sa + 32u * j);
                        const uint64_t bd = tc::sdesc_k128(sb + 32u * j);
                        const uint32_t acc = (kb | j) != 0;
                        if (PAIR) {
                            if (KIND == TC_I8) tc::mma_i8_pair(d, ad, bd, Cfg::IDESC, acc);
                            else tc::mma_f16_pair(d, ad, bd, Cfg::IDESC, acc);
                        } else {
                            if (KIND == TC_I8) tc::mma_i8(d, ad, bd, Cfg::IDESC, acc);
                            else tc::mma_f16(d, ad, bd, Cfg::IDESC, acc);
                        }
                    }
                    if (PAIR) {  // the stage is free in both CTAs
                        const uint32_t eb = tc::smem_addr(&bars->empty[stage]);
                        tc::mma_commit_pair(tc::mapa_shared(eb, 0));
                        tc::mma_commit_pair(tc::mapa_shared(eb, 1));
                    } else {
                        tc::mma_commit(&bars->empty[stage]);
                    }
                    if (++stage == TC_STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                if (PAIR) {
                    const uint32_t fb = tc::smem_addr(&bars->tfull[a]);
                    tc::mma_commit_pair(tc::mapa_shared(fb, 0));
                    tc::mma_commit_pair(tc::mapa_shared(fb, 1));
                } else {
                    tc::mma_commit(&bars->tfull[a]);
                }
            }
            DIAG_ADD(d_loop, tl);
            DIAG_FLUSH(1, d_tempty);
            DIAG_FLUSH(2, d_full);
            DIAG_FLUSH(6, d_loop);
        }
    } else {
        // ---------------- epilogue (warps 2..17) ----------------
        const int q = warp & 3;          // TMEM lane quadrant this warp may access
        const int g = (warp - 2) >> 2;   // quarter of the tile's columns
        unsigned char* const ring = stage_out + (warp - 2) * TC_STAGE_OUT;
        uint32_t nst = 0;  // stores issued from the ring
        int i = 0;
#ifdef TC_DIAG
        unsigned long long d_tfull = 0, d_busy = 0;
#endif
        for (int t = unit0; t < tiles && !tc_aborted(bars); t += units, ++i) {
            const int a = i & 1;
            const uint32_t use = (uint32_t)(i >> 1);
            int mt, n0;
            const int gi = t % G;  // GEMM of this tile
            tile_coords<BN, Cfg::BM>(t / G, num_m, num_n, mt, n0);
            const int m0 = mt + (int)rank * TC_BM;  // this CTA's 128 rows
            DIAG_T0(tw);
            const bool okt = tc::mbar_wait(&bars->tfull[a], use & 1u);
            DIAG_ADD(d_tfull, tw);
            DIAG_T0(tb);
            if (!okt) {
                tc_fail(bars, 4);
                break;
            }
            tc::fence_after_sync();
            const int64_t row = m0 + q * 32 + lane;
            const float sa = (KIND == TC_I8 && row < M) ? args.a_scale[gi][row] : 0.0f;
            const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * BN);
            // 32-column chunks [c_lo, c_hi) of this warp
            constexpr int NCH = BN / 32;
            const int c_lo = NCH >= 4 ? g * (NCH / 4) : g;
            const int c_hi = NCH >= 4 ? c_lo + NCH / 4 : (g < NCH ? g + 1 : g);
            if (EPI == KB_EPI_LOGITS_STATS) {
                // one pass per 32-column subtile: max of the fp16-rounded
                // logits (columns < V), e = fp16(e^(x - m)), left-to-right sum
#pragma unroll 1
                for (int c = c_lo; c < c_hi; ++c) {
                    const int col0 = n0 + c * 32;
                    if (col0 >= N) break;
                    uint32_t v[32];
                    tc::tmem_ld32(tbase + (uint32_t)(c * 32), v);
                    tc::tmem_ld_wait();
                    if (KIND == TC_I8) dequant32(v, sa, args.w_scale[0] + col0);
                    float xr[32];
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        const float2 f = __half22float2(__floats2half2_rn(u2f(v[j]), u2f(v[j + 1])));
                        xr[j] = f.x;
                        xr[j + 1] = f.y;
                    }
                    const int nv = V - col0;  // valid columns in this subtile
                    float m = -INFINITY, s = 0.0f;
                    uint32_t packed[16];
                    if (nv >= 32) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) m = fmaxf(m, xr[j]);
#pragma unroll
                        for (int j = 0; j < 32; j += 2) {
#if TC_HEAD_PAIRCVT
                            float f0, f1;
                            packed[j / 2] = exp_rel_pair(xr[j], xr[j + 1], m, f0, f1);
                            s = __fadd_rn(__fadd_rn(s, f0), f1);
#else
                            const uint16_t e0 = exp_rel_f16(xr[j], m);
                            const uint16_t e1 = exp_rel_f16(xr[j + 1], m);
                            s = __fadd_rn(s, h2f(e0));
                            s = __fadd_rn(s, h2f(e1));
                            packed[j / 2] = (uint32_t)e0 | ((uint32_t)e1 << 16);
#endif
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (j < nv) m = fmaxf(m, xr[j]);
#pragma unroll
                        for (int j = 0; j < 32; j += 2) {
                            uint16_t e0 = 0, e1 = 0;
                            if (j < nv) {
                                e0 = exp_rel_f16(xr[j], m);
                                s = __fadd_rn(s, h2f(e0));
                            }
                            if (j + 1 < nv) {
                                e1 = exp_rel_f16(xr[j + 1], m);
                                s = __fadd_rn(s, h2f(e1));
                            }
                            packed[j / 2] = (uint32_t)e0 | ((uint32_t)e1 << 16);
                        }
                    }
                    stage_and_store(out_tile(ring, nst, lane), lane, packed, &maps.o[0], col0,
                                    m0 + q * 32);
                    if (row < M) {
                        const int u = col0 / SUBTILE;
                        if (u < stats_stride) stats[row * stats_stride + u] = make_float2(m, s);
                    }
                }
            } else if (EPI == TC_EPI_KVR) {
                if (gi < 2)
                    epi_chunks<KB_EPI_F32, KIND>(c_lo, c_hi, n0, N, M, m0, q, lane, tbase, sa,
                                                 args.w_scale[gi], &maps.o[gi], args, ldo, ring,
                                                 nst);
                else
                    epi_chunks<KB_EPI_SIGMOID, KIND>(c_lo, c_hi, n0, N, M, m0, q, lane, tbase, sa,
                                                     args.w_scale[gi], &maps.o[gi], args, ldo,
                                                     ring, nst);
            } else {
                epi_chunks<EPI, KIND>(c_lo, c_hi, n0, N, M, m0, q, lane, tbase, sa, args.w_scale[0],
                                      &maps.o[0], args, ldo, ring, nst);
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) {
                if (PAIR) tc::mbar_arrive_cluster(tc::mapa_shared(tc::smem_addr(&bars->tempty[a]), 0));
                else tc::mbar_arrive(&bars->tempty[a]);
            }
            DIAG_ADD(d_busy, tb);
        }
        if (lane == 0) {
            DIAG_FLUSH(3, d_tfull);
            DIAG_FLUSH(5, d_busy);
        }
        if (lane == 0) tc::bulk_wait_all();  // staged stores done before exit
    }

    tc::fence_before_sync();
    __syncthreads();
    if (PAIR) tc::cluster_sync();  // no CTA leaves while its peer may still signal it
    if (warp == 1) {
        tc::fence_after_sync();
        if (PAIR) tc::tmem_dealloc_pair(tmem, Cfg::TMEM_COLS);
        else tc::tmem_dealloc(tmem, Cfg::TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

// Row-major [rows, cols] fp16 (elem 2) or int8 (elem 1) with row stride ld
// elements, boxed box_rows x 128 bytes with the 128-byte swizzle; out-of-range
// rows read as zero.
bool make_map(CUtensorMap* map, const void* base, int rows, int cols, int64_t ld, int box_rows,
              int elem) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * elem};
    cuuint32_t box[2] = {(cuuint32_t)(128 / elem), (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, elem == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
              const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Output [rows, cols] (fp32: elem 4, fp16: elem 2), row stride ld elements,
// box 64 bytes x 32 rows with the 64-byte swizzle of the staging tiles.
bool make_out_map(CUtensorMap* map, void* base, int rows, int cols, int64_t ld, int elem) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * elem};
    cuuint32_t box[2] = {(cuuint32_t)(64 / elem), 32};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, elem == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
              base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
    static int cache[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

// Clusters of two CTAs of a pair kernel that fit on the device at once (the
// pair kernel's grid), cached per device.
template <class Kern>
int pair_clusters(Kern kern, size_t smem, std::atomic<int>* cache) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    int n = cache[dev].load();
    if (n) return n;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 74);
    cfg.blockDim = dim3(TC_NT);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = -1;  // pairs unavailable: callers fall back to single CTAs
    }
    cache[dev].store(n);
    return n;
}

template <int EPI, int BN, int KIND, bool PAIR>
int launch_tc_bn(TcMaps& maps, const void* const* W, int64_t ldw, void* const* outs,
                 const TcArgs& args, cudaStream_t st) {
    using Cfg = TcCfg<BN, KIND, PAIR>;
    constexpr int G = EPI == TC_EPI_KVR ? 3 : 1;
    static std::atomic<unsigned long long> done{0};
    const cudaError_t attr_err = once_per_device(done, [] {
        return cudaFuncSetAttribute(k_gemm_tc<EPI, BN, KIND, PAIR>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::SMEM);
    });
    if (attr_err != cudaSuccess) {
        set_cuda_error(attr_err);
        return KB_ERR_CUDA;
    }
    for (int g = 0; g < G; ++g) {
        const bool f32 = EPI == KB_EPI_F32 || (EPI == TC_EPI_KVR && g < 2);
        if (!make_map(&maps.b[g], W[g], args.N, args.K, ldw, Cfg::B_ROWS, KIND == TC_I8 ? 1 : 2) ||
            !make_out_map(&maps.o[g], outs[g], args.M, args.N, args.ldo, f32 ? 4 : 2))
            return KB_ERR_UNSUPPORTED;
    }
    const int tiles = ((args.M + Cfg::BM - 1) / Cfg::BM) * ((args.N + BN - 1) / BN) * G;
    if constexpr (!PAIR) {
        const int grid = tiles < sm_count() ? tiles : sm_count();
        k_gemm_tc<EPI, BN, KIND, false><<<grid, TC_NT, Cfg::SMEM, st>>>(maps, args);
        return launch_status();
    } else {
    static std::atomic<int> clusters[64];
    const int nc = pair_clusters(k_gemm_tc<EPI, BN, KIND, true>, Cfg::SMEM, clusters);
    if (nc <= 0) return KB_ERR_UNSUPPORTED;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (tiles < nc ? tiles : nc));
    cfg.blockDim = dim3(TC_NT);
    cfg.dynamicSmemBytes = Cfg::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemm_tc<EPI, BN, KIND, true>, maps, args);
    if (e != cudaSuccess) {
        set_cuda_error(e);
        return KB_ERR_CUDA;
    }
    return launch_status();
    }
}

// Tile width for a launch: the widest whose tile count fills the SMs, else
// the narrowest.  Every width gives the same bits (one K walk per element).
int pick_bn(int M, int N) {
    const int mt = (M + TC_BM - 1) / TC_BM, sms = sm_count();
    for (int bn = TC_MAX_BN; bn > 32; bn >>= 1)
        if (mt * ((N + bn - 1) / bn) >= sms) return bn;
    return 32;
}

// Library choice: CTA pairs (256 x 256 tiles) once their tiles fill every
// pair of SMs at least twice over, else pick_bn's single-CTA width.  The head
// (softmax-numerator epilogue, bound by its exponentials) measured faster on
// single CTAs and keeps them.
int pick_tile(int M, int N, bool logits) {
    const int bn = pick_bn(M, N);
    if (TC_PAIR_AUTO && bn == 256 && ((M + 255) / 256) * ((N + 255) / 256) >= sm_count() &&
        !logits)
        return KB_TILE_PAIR;
    return bn;
}

// A / W / outs: one pointer per GEMM of the launch (three for TC_EPI_KVR).
template <int EPI, int KIND>
int launch_tc(const void* const* A, int64_t lda, const void* const* W, int64_t ldw,
              void* const* outs, const TcArgs& args, cudaStream_t st, int bn) {
    constexpr int G = EPI == TC_EPI_KVR ? 3 : 1;
    TcMaps maps;
    for (int g = 0; g < G; ++g)
        if (!make_map(&maps.a[g], A[g], args.M, args.K, lda, TC_BM, KIND == TC_I8 ? 1 : 2))
            return KB_ERR_UNSUPPORTED;
    if (bn == 0) bn = pick_tile(args.M, args.N * G, EPI == KB_EPI_LOGITS_STATS);
    switch (bn) {
        case KB_TILE_PAIR: {
            const int r = launch_tc_bn<EPI, 256, KIND, true>(maps, W, ldw, outs, args, st);
            if (r != KB_ERR_UNSUPPORTED) return r;
            return launch_tc_bn<EPI, 256, KIND, false>(maps, W, ldw, outs, args, st);
        }
        case 256: return launch_tc_bn<EPI, 256, KIND, false>(maps, W, ldw, outs, args, st);
        case 128: return launch_tc_bn<EPI, 128, KIND, false>(maps, W, ldw, outs, args, st);
        case 64: return launch_tc_bn<EPI, 64, KIND, false>(maps, W, ldw, outs, args, st);
        case 32: return launch_tc_bn<EPI, 32, KIND, false>(maps, W, ldw, outs, args, st);
        default: return KB_ERR_ARG;
    }
}

template <int KIND>
int launch_epi(const void* A, int64_t lda, const void* W, int64_t ldw, int epi,
               const TcArgs& args, cudaStream_t st, int bn) {
    const void* const a[1] = {A};
    const void* const w[1] = {W};
    void* const o[1] = {args.out};
    switch (epi) {
        case KB_EPI_F32: return launch_tc<KB_EPI_F32, KIND>(a, lda, w, ldw, o, args, st, bn);
        case KB_EPI_F16: return launch_tc<KB_EPI_F16, KIND>(a, lda, w, ldw, o, args, st, bn);
        case KB_EPI_SIGMOID: return launch_tc<KB_EPI_SIGMOID, KIND>(a, lda, w, ldw, o, args, st, bn);
        case KB_EPI_RELU_SQ: return launch_tc<KB_EPI_RELU_SQ, KIND>(a, lda, w, ldw, o, args, st, bn);
        case KB_EPI_RESID: return launch_tc<KB_EPI_RESID, KIND>(a, lda, w, ldw, o, args, st, bn);
        case KB_EPI_GATE_RESID: return launch_tc<KB_EPI_GATE_RESID, KIND>(a, lda, w, ldw, o, args, st, bn);
        case KB_EPI_LOGITS_STATS: return launch_tc<KB_EPI_LOGITS_STATS, KIND>(a, lda, w, ldw, o, args, st, bn);
        default: return KB_ERR_ARG;
    }
}

}  // namespace

int launch_gemm_tc(const uint16_t* A, int64_t lda, const uint16_t* W, int64_t ldw, int M, int N,
                   int K, int epi, void* out, int64_t ldo, const uint16_t* resid,
                   const uint16_t* gate, cudaStream_t st, int bn) {
    if (M == 0) return KB_OK;
    if (epi == KB_EPI_LOGITS_STATS) return KB_ERR_ARG;
    const TcArgs args{M, N, K, out, ldo, resid, gate, 0, nullptr, 0, {}, {}};
    return launch_epi<TC_F16>(A, lda, W, ldw, epi, args, st, bn);
}

int launch_gemm_bf16(const uint16_t* A, int64_t lda, const uint16_t* W, int64_t ldw, int M,
                     int N, int K, int epi, void* out, int64_t ldo, const uint16_t* resid,
                     const uint16_t* gate, cudaStream_t st, int bn) {
    if (M == 0) return KB_OK;
    if (epi == KB_EPI_LOGITS_STATS) return KB_ERR_ARG;
    const TcArgs args{M, N, K, out, ldo, resid, gate, 0, nullptr, 0, {}, {}};
    return launch_epi<TC_BF16>(A, lda, W, ldw, epi, args, st, bn);
}

int launch_gemm_logits_bf16(const uint16_t* A, int64_t lda, const uint16_t* W, int64_t ldw,
                            int M, int N, int K, uint16_t* out, int64_t ldo, int V, float* stats,
                            int stats_stride, cudaStream_t st) {
    if (M == 0) return KB_OK;
    const TcArgs args{M, N, K, out, ldo, nullptr, nullptr, V, reinterpret_cast<float2*>(stats),
                      stats_stride, {}, {}};
    return launch_epi<TC_BF16>(A, lda, W, ldw, KB_EPI_LOGITS_STATS, args, st, 0);
}

int launch_gemm_i8(const int8_t* A, int64_t lda, const float* a_scale, const int8_t* W,
                   int64_t ldw, const uint16_t* w_scale, int M, int N, int K, int epi, void* out,
                   int64_t ldo, const uint16_t* resid, const uint16_t* gate, cudaStream_t st,
                   int bn) {
    if (M == 0) return KB_OK;
    if (epi == KB_EPI_LOGITS_STATS) return KB_ERR_ARG;
    const TcArgs args{M, N, K, out, ldo, resid, gate, 0, nullptr, 0, {a_scale}, {w_scale}};
    return launch_epi<TC_I8>(A, lda, W, ldw, epi, args, st, bn);
}

int launch_gemm_logits(const uint16_t* A, int64_t lda, const uint16_t* W, int64_t ldw, int M,
                       int N, int K, uint16_t* out, int64_t ldo, int V, float* stats,
                       int stats_stride, cudaStream_t st) {
    if (M == 0) return KB_OK;
    const TcArgs args{M, N, K, out, ldo, nullptr, nullptr, V, reinterpret_cast<float2*>(stats),
                      stats_stride, {}, {}};
    return launch_epi<TC_F16>(A, lda, W, ldw, KB_EPI_LOGITS_STATS, args, st, 0);
}

int launch_gemm_logits_i8(const int8_t* A, int64_t lda, const float* a_scale, const int8_t* W,
                          int64_t ldw, const uint16_t* w_scale, int M, int N, int K,
                          uint16_t* out, int64_t ldo, int V, float* stats, int stats_stride,
                          cudaStream_t st) {
    if (M == 0) return KB_OK;
    const TcArgs args{M, N, K, out, ldo, nullptr, nullptr, V, reinterpret_cast<float2*>(stats),
                      stats_stride, {a_scale}, {w_scale}};
    return launch_epi<TC_I8>(A, lda, W, ldw, KB_EPI_LOGITS_STATS, args, st, 0);
}

// k = kx @ Kw^T (fp32), v = vx @ Vw^T (fp32), r = sigmoid(rx @ Rw^T) (fp16)
// in one launch; same shapes, same bits as three launch_gemm_* calls.
int launch_gemm_kvr(int kind, const void* const (&A)[3], int64_t lda,
                    const float* const (&a_scale)[3], const void* const (&W)[3], int64_t ldw,
                    const uint16_t* const (&w_scale)[3], int M, int N, int K,
                    void* const (&out)[3], int64_t ldo, cudaStream_t st, int bn) {
    if (M == 0) return KB_OK;
    TcArgs args{M, N, K, nullptr, ldo, nullptr, nullptr, 0, nullptr, 0,
                {a_scale[0], a_scale[1], a_scale[2]}, {w_scale[0], w_scale[1], w_scale[2]}};
    switch (kind) {
        case KB_F16: return launch_tc<TC_EPI_KVR, TC_F16>(A, lda, W, ldw, out, args, st, bn);
        case KB_BF16: return launch_tc<TC_EPI_KVR, TC_BF16>(A, lda, W, ldw, out, args, st, bn);
        case KB_I8: return launch_tc<TC_EPI_KVR, TC_I8>(A, lda, W, ldw, out, args, st, bn);
        default: return KB_ERR_ARG;
    }
}

int read_tc_error(int reset) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int)) != cudaSuccess) return -1;
    if (reset && v) {
        const int z = 0;
        cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int));
    }
    return v;
}

}  // namespace kb
