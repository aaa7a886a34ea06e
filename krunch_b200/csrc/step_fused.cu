// Fused stepped decode forward of the w8a8 model: the whole T = 1 layer stack
// (embedding -> n_layer x (time mix, channel mix) -> ln_out + quantisation of
// the head input) in ONE persistent cooperative launch, one CTA per SM.  It
// replaces the reference's fused single-token layer kernels
// (krunch_ac/cuda/rwkv_step*.cu, rwkv_step_v3.cu:83-480) and the per-op
// launch chain of forward_stepped_batched (krunch/cpp_path.py:428-460).
//
// The step alternates two kinds of phase, separated by a grid barrier:
//   tile phase  every GEMM of the phase is cut into units (128-row M tile,
//               64-column N tile, K slice of <= 768): TMA brings the int8
//               weight tile and the int8 activation tile into shared memory,
//               one thread issues tcgen05.mma kind::i8 into a TMEM
//               accumulator, and the exact int32 partial sum goes to a
//               [slice][B][N] buffer.  The weight tile of a CTA's next tile
//               phase is prefetched before the barrier (weights never change).
//   row phase   one warp per stream row: sum the slices (exact integers),
//               dequantise, apply the GEMM epilogue, then the row-local ops
//               (WKV, LayerNorm, token-shift mix, quantisation).
// Per layer: [k,v,r] -> WKV -> [o] -> +x, LN2, mix -> [ffn k, ffn r] ->
// relu^2 / sigmoid -> [ffn v] -> +x, next LN1, mix: 8 phases.
//
// Integer partial sums make the result independent of how K is sliced, and
// every floating-point step (epi_math.cuh, rwkv_dev.cuh, quant.cuh) is the
// code the per-op kernels run, so the fused step reproduces
// kb_forward_window(T = 1) — and hence the packed encoder — bit for bit.
//
// Every wait is bounded: mbarrier waits (tc::mbar_wait) and the grid barrier
// spin.  On expiry a CTA records an error, raises the abort flag that the
// other CTAs poll at the barrier, frees its TMEM and returns.
#include <cudaTypedefs.h>

#include <cstring>
#include <memory>
#include <mutex>

#include "epi_math.cuh"
#include "model_impl.h"
#include "profile.cuh"
#include "quant.cuh"
#include "rwkv_dev.cuh"
#include "rwkv_ops.cuh"
#include "tc_common.cuh"

namespace kb {

constexpr int SF_NT = 256;                       // 8 warps
constexpr int SF_BN = 64;                        // N columns per unit
constexpr int SF_MAX_KB = 6;                     // 128-byte K blocks per unit
constexpr int SF_MAX_LAYERS = 24;
constexpr uint32_t SF_A_BLK = 128 * 128;         // A tile, one K block: 16 KB
constexpr uint32_t SF_W_BLK = SF_BN * 128;       // W tile, one K block: 8 KB
constexpr uint32_t SF_A_BYTES = SF_MAX_KB * SF_A_BLK;
constexpr uint32_t SF_W_BYTES = SF_MAX_KB * SF_W_BLK;
constexpr int SF_MAX_C = 2048;                   // row staging per group
constexpr size_t SF_ROW_OFF = SF_A_BYTES + 2 * SF_W_BYTES + 256;
constexpr uint32_t SF_IDESC = tc::idesc_i8(128, SF_BN);
constexpr int SF_TRACE_TILE = 512;  // + 4 tp: SM clock of CTA 0's first unit
constexpr int SF_TRACE_CLK = 768;   // + epoch: SM clock at barrier exit
constexpr int SF_TRACE_TILE2 = 1536;  // + 4 tp: tile phase entry, unit found, W issued
constexpr int SF_TRACE_ARR = 2048;  // + epoch * grid + cta: %globaltimer at each CTA's arrival
constexpr unsigned long long SF_SPIN_NS = 2000000000ull;  // grid-barrier wait bound: 2 s

// GEMMs of a layer, in weight-map order
enum { G_K = 0, G_V, G_R, G_O, G_FK, G_FR, G_FV, G_NUM };
// activation (A operand) maps
enum { A_KX = 0, A_VX, A_RX, A_RY, A_KK, A_NUM };

struct SfLayer {
    const float *ln1_w, *ln1_b, *ln2_w, *ln2_b;
    const float *mix_k, *mix_v, *mix_r, *decay, *first, *fmix_k, *fmix_r;
    const uint16_t* wscale[G_NUM];
};

// Everything but the tensor maps; copied to shared memory at kernel start so
// the phases read it without constant-cache misses.
struct SfHot {
    SfLayer layer[SF_MAX_LAYERS];
    int L, B, C, F, V, conv;
    int ks[G_NUM];   // K slices per GEMM
    const int32_t* tokens;
    const uint16_t* emb;
    const float *ln_out_w, *ln_out_b;
    float* state;    // [L][5][B][C]
    uint16_t *x, *kk, *r2;
    int8_t *q_kx, *q_vx, *q_rx, *q_ry, *q_kk;
    float *s_kx, *s_vx, *s_rx, *s_ry, *s_kk;
    int32_t* part[G_NUM];  // [ks][B][N]
    unsigned* bar;         // [0] arrivals, [1] abort flag; zeroed before launch
    unsigned long long* trace;  // optional: CTA 0's %globaltimer at barrier entry/exit
    unsigned long long spin_ns; // grid-barrier wait bound
    int withhold_arrival;       // test: CTA 0 does not arrive at the first barrier
};

struct SfParams {
    CUtensorMap wmap[SF_MAX_LAYERS][G_NUM];  // int8 weights, box 128 B x 64 rows
    CUtensorMap amap[A_NUM];                 // int8 activations, box 128 B x 128 rows
    CUtensorMap pmap[G_NUM];                 // int32 partials [slice][B][N], box 32 x 128 x 1
    SfHot h;
};

constexpr int SF_RED = 24;  // per-group reduction scratch (floats)
constexpr size_t SF_HOT_OFF = SF_ROW_OFF + 2 * (SF_MAX_C + SF_RED) * 4;
constexpr size_t SF_SMEM = SF_HOT_OFF + sizeof(SfHot) + 1024 /*align*/;
static_assert(SF_SMEM <= 232448, "shared memory per block");

__device__ int g_step_error = 0;

struct Unit {
    int g, amap, N, mt, nt, k0, nkb, ks;
};

struct SfBars {
    uint64_t a_full, w_full[2], mma_done;
    uint32_t tmem_base;
    int ok;
    // this CTA's first unit of each tile-phase kind (kvr, o, ffn, fv): the
    // same for every layer, found once at kernel start
    Unit first[4];
    int has_first[4];
};
static_assert(sizeof(SfBars) <= 256, "SfBars fits its shared-memory slot");

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ void sf_fail(const SfHot& p, int code) {
    atomicExch(&g_step_error, code);
    atomicExch(p.bar + 1, 1u);
}

// Grid barrier number `epoch` (1, 2, ...): every CTA arrives once; returns
// false if any CTA aborted or the wait expired.
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// ---- tile phases -----------------------------------------------------------

struct Job {
    int g;       // GEMM id
    int amap;    // A operand map
    int N, K, ks;
};

// The jobs of tile phase tp (4 per layer).
__device__ __forceinline__ int phase_jobs(const SfHot& p, int tp, Job (&j)[3]) {
    const int C = p.C, F = p.F;
    switch (tp & 3) {
        case 0:
            j[0] = {G_K, A_KX, C, C, p.ks[G_K]};
            j[1] = {G_V, A_VX, C, C, p.ks[G_V]};
            j[2] = {G_R, A_RX, C, C, p.ks[G_R]};
            return 3;
        case 1:
            j[0] = {G_O, A_RY, C, C, p.ks[G_O]};
            return 1;
        case 2:
            j[0] = {G_FK, A_KX, F, C, p.ks[G_FK]};
            j[1] = {G_FR, A_RX, C, C, p.ks[G_FR]};
            return 2;
        default:
            j[0] = {G_FV, A_KK, C, F, p.ks[G_FV]};
            return 1;
    }
}

__device__ __forceinline__ int units_of(const SfHot& p, const Job& jb) {
    return ((p.B + 127) / 128) * (jb.N / SF_BN) * jb.ks;
}

// Unit u of tile phase tp; false past the last unit.
__device__ bool unit_at(const SfHot& p, int tp, int u, Unit& out) {
    Job j[3];
    const int nj = phase_jobs(p, tp, j);
    for (int i = 0; i < nj; ++i) {
        const int n = units_of(p, j[i]);
        if (u < n) {
            const int nt_n = j[i].N / SF_BN;
            const int nkb = j[i].K / 128 / j[i].ks;
            out.g = j[i].g;
            out.amap = j[i].amap;
            out.N = j[i].N;
            out.nt = u % nt_n;
            out.ks = (u / nt_n) % j[i].ks;
            out.mt = u / (nt_n * j[i].ks);
            out.nkb = nkb;
            out.k0 = out.ks * nkb * 128;
            return true;
        }
        u -= n;
    }
    return false;
}

// thread 0: weight tile of unit `un` (layer l) into W buffer `wb`
__device__ __forceinline__ void issue_w(const SfParams& P, const SfHot& p, SfBars* sb, unsigned char* wbuf, int wb,
                                        int l, const Unit& un) {
    tc::mbar_expect_tx(&sb->w_full[wb], (uint32_t)un.nkb * SF_W_BLK);
    for (int kb = 0; kb < un.nkb; ++kb)
        tc::tma_load_2d(wbuf + kb * SF_W_BLK, &P.wmap[l][un.g], &sb->w_full[wb], un.k0 + kb * 128,
                        un.nt * SF_BN);
}

struct SfState {
    uint32_t w_uses[2];   // completed waits per W buffer (thread 0)
    uint32_t a_uses;      // (thread 0)
    uint32_t mma_uses;    // (all threads)
    int w_pending[2];     // a prefetched W load is in flight in this buffer (thread 0)
};

// thread 0: activation tile of unit `un` into the A buffer
__device__ __forceinline__ void issue_a(const SfParams& P, SfBars* sb, unsigned char* abuf,
                                        const Unit& un) {
    tc::mbar_expect_tx(&sb->a_full, (uint32_t)un.nkb * SF_A_BLK);
    for (int kb = 0; kb < un.nkb; ++kb)
        tc::tma_load_2d(abuf + kb * SF_A_BLK, &P.amap[un.amap], &sb->a_full, un.k0 + kb * 128,
                        un.mt * 128);
}

__device__ bool grid_sync(const SfHot& p, SfBars* sb, unsigned epoch) {
    __syncthreads();
    if (threadIdx.x == 0 && blockIdx.x == 0 && p.trace) p.trace[2 * epoch] = gtimer();
    if (threadIdx.x == 0) {
        // release: the CTA's writes (ordered before this thread by the
        // __syncthreads above) become visible with the arrival; the proxy
        // fences order them with the TMA reads of the next tile phase
        fence_proxy_async_global();
        if (p.trace) p.trace[SF_TRACE_ARR + epoch * gridDim.x + blockIdx.x] = gtimer();
        if (!(p.withhold_arrival && epoch == 1 && blockIdx.x == 0))
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.bar) : "memory");
        const unsigned target = epoch * gridDim.x;
        int ok = 1;
        const unsigned long long t0 = gtimer();
        for (uint32_t it = 0;; ++it) {
            if (ld_acquire(p.bar) >= target) break;
            if ((it & 15u) == 15u) {
                if (*reinterpret_cast<volatile unsigned*>(p.bar + 1)) {
                    ok = 0;
                    break;
                }
                if (gtimer() - t0 > p.spin_ns) {
                    sf_fail(p, 5);
                    ok = 0;
                    break;
                }
            }
        }
        fence_proxy_async_global();
        sb->ok = ok;
        if (blockIdx.x == 0 && p.trace) {
            p.trace[2 * epoch + 1] = gtimer();
            p.trace[SF_TRACE_CLK + epoch] = clock64();
        }
    }
    __syncthreads();
    return sb->ok != 0;
}

// Runs this CTA's units of tile phase tp (layer l).  The first unit's weights
// were prefetched into buffer (tp & 1) at the end of the previous tile phase.
__device__ bool tile_phase(const SfParams& P, const SfHot& p, SfBars* sb, unsigned char* smem, uint32_t tmem,
                           int tp, SfState& st) {
    const int l = tp >> 2;
    const int wb = tp & 1;
    unsigned char* abuf = smem;
    unsigned char* wbuf = smem + SF_A_BYTES + wb * SF_W_BYTES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    bool first = true;
    if (p.trace && blockIdx.x == 0 && threadIdx.x == 0) p.trace[SF_TRACE_TILE2 + 4 * tp] = clock64();
    for (int u = blockIdx.x;; u += gridDim.x) {
        Unit un;
        if (first) {
            if (!sb->has_first[tp & 3]) break;
            un = sb->first[tp & 3];
        } else if (!unit_at(p, tp, u, un)) {
            break;
        }
        if (threadIdx.x == 0) {
            if (p.trace && blockIdx.x == 0 && first) p.trace[SF_TRACE_TILE2 + 4 * tp + 1] = clock64();
            if (!(first && st.w_pending[wb])) issue_w(P, p, sb, wbuf, wb, l, un);
            if (p.trace && blockIdx.x == 0 && first) p.trace[SF_TRACE_TILE2 + 4 * tp + 2] = clock64();
            st.w_pending[wb] = 0;
            issue_a(P, sb, abuf, un);
            const bool tr = p.trace && blockIdx.x == 0 && first;
            if (tr) p.trace[SF_TRACE_TILE + 4 * tp] = clock64();
            bool ok = tc::mbar_wait(&sb->w_full[wb], st.w_uses[wb] & 1u);
            ok = tc::mbar_wait(&sb->a_full, st.a_uses & 1u) && ok;
            st.w_uses[wb]++;
            st.a_uses++;
            if (tr) p.trace[SF_TRACE_TILE + 4 * tp + 1] = clock64();
            if (!ok) {
                sf_fail(p, 1);
            } else {
                tc::fence_after_sync();
                const uint32_t sa = tc::smem_addr(abuf), sw = tc::smem_addr(wbuf);
                for (int kb = 0; kb < un.nkb; ++kb)
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        tc::mma_i8(tmem, tc::sdesc_k128(sa + kb * SF_A_BLK + 32u * j),
                                   tc::sdesc_k128(sw + kb * SF_W_BLK + 32u * j), SF_IDESC,
                                   (kb | j) != 0);
            }
            tc::mma_commit(&sb->mma_done);
        }
        __syncwarp();
        // epilogue: warp w drains TMEM lanes 32*(w%4).. and columns 32*(w/4)..
        // (thread 0 waits for the MMAs; the others wait at the CTA barrier)
        if (threadIdx.x == 0) {
            if (!tc::mbar_wait(&sb->mma_done, st.mma_uses & 1u)) sf_fail(p, 2);
            if (p.trace && blockIdx.x == 0 && first) p.trace[SF_TRACE_TILE + 4 * tp + 2] = clock64();
        }
        st.mma_uses++;
        __syncwarp();
        __syncthreads();
        tc::fence_after_sync();
        {
            // stage the 128 x 64 int32 tile in the (now free) A buffer: two
            // 128-row x 128-byte halves in the 128-byte swizzle, then two TMA
            // stores into the [slice][B][N] partials (rows >= B clipped)
            const int q = warp & 3, ch = warp >> 2;
            uint32_t v[32];
            tc::tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ch * 32), v);
            tc::tmem_ld_wait();
            const int r = q * 32 + lane;
            unsigned char* stg = abuf + ch * 16384 + r * 128;
#pragma unroll
            for (int k = 0; k < 8; ++k)
                *reinterpret_cast<uint4*>(stg + ((k ^ (r & 7)) << 4)) =
                    make_uint4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
        }
        tc::fence_before_sync();
        tc::fence_proxy_async_smem();
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int ch = 0; ch < 2; ++ch)
                tc::tma_store_3d(&P.pmap[un.g], abuf + ch * 16384, un.nt * SF_BN + ch * 32,
                                 un.mt * 128, un.ks);
            tc::bulk_commit();
            tc::bulk_wait_all();  // before the grid barrier and before abuf is reused
        }
        if (p.trace && blockIdx.x == 0 && threadIdx.x == 0 && first)
            p.trace[SF_TRACE_TILE + 4 * tp + 3] = clock64();
        first = false;
    }
    // prefetch the weights of this CTA's first unit of the next tile phase
    if (threadIdx.x == 0 && tp + 1 < 4 * p.L) {
        if (sb->has_first[(tp + 1) & 3]) {
            const Unit& nx = sb->first[(tp + 1) & 3];
            const int nb = (tp + 1) & 1;
            issue_w(P, p, sb, smem + SF_A_BYTES + nb * SF_W_BYTES, nb, (tp + 1) >> 2, nx);
            tc::prefetch_tmap(&P.amap[nx.amap]);
            st.w_pending[nb] = 1;
        }
    }
    return true;
}

// ---- row phases ------------------------------------------------------------
// A stream row is handled by a group of 4 warps (two groups per CTA): the
// element-wise work (slice sums, dequantisation, epilogues, WKV, mixes,
// quantisation) is spread over the group's 128 threads, element c on thread
// c % 128; the LayerNorm statistics are computed by the group's first warp
// from the row staged in shared memory, in exactly the lane order and
// butterfly of ln_warp (rwkv_dev.cuh), so the result is the per-op kernel's.
// Every load of a phase is issued before its first global store.

constexpr int SF_GT = 128;  // threads per row group

struct Grp {
    int id, t, w, lane;  // group in CTA, thread / warp / lane in group
    float* xs;           // row staging [C]
    float* red;          // reduction scratch [SF_RED]
};

__device__ __forceinline__ void gsync(const Grp& g) {
    asm volatile("bar.sync %0, %1;" ::"r"(1 + g.id), "r"(SF_GT) : "memory");
}


// mean and 1/std of the row in g.xs, bit-identical to ln_warp<EPL>
template <int EPL>
__device__ __forceinline__ void group_ln_stats(const Grp& g, int C, float& mean, float& rstd) {
    gsync(g);
    if (g.w == 0) {
        float s = 0.0f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) s = __fadd_rn(s, g.xs[RowIdx<EPL>::col(g.lane, e)]);
        const float mn = __fdiv_rn(warp_sum(s), (float)C);
        float q = 0.0f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
            const float d = __fsub_rn(g.xs[RowIdx<EPL>::col(g.lane, e)], mn);
            q = __fmaf_rn(d, d, q);
        }
        const float rs = __frsqrt_rn(__fadd_rn(__fdiv_rn(warp_sum(q), (float)C), LN_EPS));
        if (g.lane == 0) {
            g.red[4] = mn;
            g.red[5] = rs;
        }
    }
    gsync(g);
    mean = g.red[4];
    rstd = g.red[5];
}

__device__ __forceinline__ float f16r(float v) { return __half2float(__float2half_rn(v)); }

// Largest row amax of NQ value sets of this thread, over the group, in one
// exchange (max is exact, so merging the reductions keeps the bits).
template <int NQ>
__device__ __forceinline__ void group_max_n(const Grp& g, float (&m)[NQ]) {
#pragma unroll
    for (int j = 0; j < NQ; ++j) {
        m[j] = warp_max(m[j]);
        if (g.lane == 0) g.red[8 + 4 * j + g.w] = m[j];
    }
    gsync(g);
#pragma unroll
    for (int j = 0; j < NQ; ++j) {
        const float* r = g.red + 8 + 4 * j;
        m[j] = fmaxf(fmaxf(r[0], r[1]), fmaxf(r[2], r[3]));
    }
    gsync(g);
}

// quantise NV values of this thread (fp16-rounded) with the group's row
// amax; element i goes to q[t + 128 i]
template <int NV>
__device__ __forceinline__ void group_quant_store(const Grp& g, const float (&a)[NV], int8_t* q,
                                                  float* qs) {
    float m[1] = {0.0f};
#pragma unroll
    for (int i = 0; i < NV; ++i) m[0] = fmaxf(m[0], fabsf(a[i]));
    group_max_n<1>(g, m);
    const float inv = q_inv(m[0]);
#pragma unroll
    for (int i = 0; i < NV; ++i) q[g.t + SF_GT * i] = (int8_t)q8(a[i], inv);
    if (g.t == 0) *qs = q_factor(m[0]);
}

// Trace marks of row phase rp (CTA 0, group 0, row 0): SM clock at entry,
// when the phase's loaded data has been consumed, after its row reduction,
// and at its end (slots SF_TRACE_ROW + 4 rp + k).
constexpr int SF_TRACE_ROW = 1024;
__device__ __forceinline__ void rmark(const SfHot& p, const Grp& g, int b, int rp, int k) {
    if (p.trace && b == 0 && g.t == 0 && blockIdx.x == 0) p.trace[SF_TRACE_ROW + 4 * rp + k] = clock64();
}

// The int32 K-slice partial sums of row b of one GEMM, columns t + 128 i.
// issue() puts the loads of the first MAXKS slices in flight at once (all
// loads of a row phase go out before its first use); sum() adds them and
// any further slices (exact integers: the order does not matter).
template <int NV, int MAXKS>
struct PartLd {
    int v[MAXKS][NV];
    __device__ __forceinline__ void issue(const Grp& g, const int32_t* part, int ks, int B, int N,
                                          int b) {
#pragma unroll
        for (int s = 0; s < MAXKS; ++s) {
            const int32_t* rp = part + ((int64_t)s * B + b) * N + g.t;
#pragma unroll
            for (int i = 0; i < NV; ++i) v[s][i] = s < ks ? __ldcg(rp + SF_GT * i) : 0;
        }
    }
    __device__ __forceinline__ void sum(const Grp& g, const int32_t* part, int ks, int B, int N,
                                        int b, int (&acc)[NV]) const {
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            acc[i] = v[0][i];
#pragma unroll
            for (int s = 1; s < MAXKS; ++s) acc[i] += v[s][i];
        }
        for (int s = MAXKS; s < ks; ++s) {
            const int32_t* rp = part + ((int64_t)s * B + b) * N + g.t;
#pragma unroll
            for (int i = 0; i < NV; ++i) acc[i] += __ldcg(rp + SF_GT * i);
        }
    }
};

// Inputs of a LayerNorm + NMIX token-shift mixes of one row that do not
// depend on the previous phase (parameters, carried state row), loaded at
// the start of the row phase.
template <int EPL, int NMIX>
struct LnMixIn {
    static constexpr int NE = EPL / 4;
    float prev[NE], w[NE], bi[NE], mk[NMIX > 0 ? NMIX : 1][NE];
    __device__ __forceinline__ void load(const Grp& g, const float* lw, const float* lb,
                                         const float* const (&mix)[3], const float* srow) {
#pragma unroll
        for (int i = 0; i < NE; ++i) {
            const int c = g.t + SF_GT * i;
            if (NMIX > 0) prev[i] = srow[c];
            w[i] = __ldg(lw + c);
            bi[i] = __ldg(lb + c);
#pragma unroll
            for (int m = 0; m < NMIX; ++m) mk[m][i] = __ldg(mix[m] + c);
        }
    }
};

// LN of the row (v: this thread's elements, also staged in g.xs), NMIX
// token-shift mixes against the carried state row srow (overwritten with
// LN(v)), each quantised; NMIX = 0 quantises LN(v) itself.
template <int EPL, int NMIX, int M>
__device__ __forceinline__ void ln_mix_g(const Grp& g, const float (&v)[EPL / 4], int C,
                                         const LnMixIn<EPL, M>& in, float* srow,
                                         int8_t* const (&q)[3], float* const (&qs)[3]) {
    constexpr int NE = EPL / 4;
    constexpr int NQ = NMIX > 0 ? NMIX : 1;
    float mean, rstd;
    group_ln_stats<EPL>(g, C, mean, rstd);
    float cur[NE];
#pragma unroll
    for (int i = 0; i < NE; ++i)
        cur[i] = f16r(__fmaf_rn(__fmul_rn(__fsub_rn(v[i], mean), rstd), in.w[i], in.bi[i]));
    float a[NQ][NE], m[NQ];
#pragma unroll
    for (int j = 0; j < NQ; ++j) {
        m[j] = 0.0f;
#pragma unroll
        for (int i = 0; i < NE; ++i) {
            a[j][i] = NMIX == 0 ? cur[i]
                                : f16r(__fmaf_rn(cur[i], in.mk[j][i],
                                                 __fmul_rn(in.prev[i], __fsub_rn(1.0f, in.mk[j][i]))));
            m[j] = fmaxf(m[j], fabsf(a[j][i]));
        }
    }
    group_max_n<NQ>(g, m);
#pragma unroll
    for (int j = 0; j < NQ; ++j) {
        const float inv = q_inv(m[j]);
#pragma unroll
        for (int i = 0; i < NE; ++i) q[j][g.t + SF_GT * i] = (int8_t)q8(a[j][i], inv);
        if (g.t == 0) *qs[j] = q_factor(m[j]);
    }
    if constexpr (NMIX > 0) {
#pragma unroll
        for (int i = 0; i < NE; ++i) srow[g.t + SF_GT * i] = cur[i];
    }
}

// the LN1 + time-mix inputs of layer l for row b; returns the att_xx state row
template <int EPL, int M>
__device__ __forceinline__ float* ln1_in(const Grp& g, const SfHot& p, int l, int b,
                                         LnMixIn<EPL, M>& in) {
    const size_t BC = (size_t)p.B * p.C;
    const SfLayer& ly = p.layer[l];
    const float* const mix[3] = {ly.mix_k, ly.mix_v, ly.mix_r};
    float* srow = p.state + (size_t)l * 5 * BC + (size_t)b * p.C;
    in.load(g, ly.ln1_w, ly.ln1_b, mix, srow);
    return srow;
}

template <int EPL>
__device__ __forceinline__ void ln1_mix_g(const Grp& g, const SfHot& p, int b,
                                          const float (&v)[EPL / 4], const LnMixIn<EPL, 3>& in,
                                          float* srow) {
    const int C = p.C;
    int8_t* const q[3] = {p.q_kx + (size_t)b * C, p.q_vx + (size_t)b * C, p.q_rx + (size_t)b * C};
    float* const qs[3] = {p.s_kx + b, p.s_vx + b, p.s_rx + b};
    ln_mix_g<EPL, 3>(g, v, C, in, srow, q, qs);
}

// embedding + LN1 of layer 0
template <int EPL>
__device__ void row_embed(const Grp& g, const SfHot& p, int b) {
    constexpr int NE = EPL / 4;
    const int C = p.C;
    LnMixIn<EPL, 3> in;
    float* srow = ln1_in<EPL>(g, p, 0, b, in);
    int t = p.tokens[b];
    t = t < 0 ? 0 : (t >= p.V ? p.V - 1 : t);
    uint16_t e16[NE];
    float v[NE];
#pragma unroll
    for (int i = 0; i < NE; ++i) {
        e16[i] = __ldg(p.emb + (size_t)t * C + g.t + SF_GT * i);
        v[i] = h2f(e16[i]);
        g.xs[g.t + SF_GT * i] = v[i];
    }
    ln1_mix_g<EPL>(g, p, b, v, in, srow);
#pragma unroll
    for (int i = 0; i < NE; ++i) p.x[(size_t)b * C + g.t + SF_GT * i] = e16[i];
}

// Slices of the partial sums loaded in one go, per GEMM group (more slices
// are summed by a second pass): k/v/r, o, ffn key/receptance, ffn value.
// The 2048-wide rows (EPL 64) hold too many values per thread for that.
template <int EPL> struct SfKs {
    static constexpr int KVR = EPL >= 64 ? 1 : 3, O = EPL >= 64 ? 1 : 6;
    static constexpr int FKR = EPL >= 64 ? 1 : 2, FV = EPL >= 64 ? 1 : 6;
};

// Each row phase reads (1) inputs that no phase of this step writes before it
// (carried state, parameters, rows written two or more barriers earlier) and
// (2) the partial sums of the tile phase just before it.  The *In structs
// hold (1) and are loaded at the start of the phase, beside the loads of (2).
// (Loading them before the opening barrier was measured slower: the
// arriving thread's release then waits for its own outstanding loads.)

template <int EPL>
struct WkvIn {
    static constexpr int NE = EPL / 4;
    float aa[NE], bb[NE], pp[NE], u[NE], dec[NE], wk[NE], wv[NE], wr[NE];
    __device__ __forceinline__ void load(const Grp& g, const SfHot& p, int l, int b) {
        const size_t BC = (size_t)p.B * p.C;
        const SfLayer& ly = p.layer[l];
        const float* s = p.state + (size_t)l * 5 * BC + (size_t)b * p.C + g.t;
#pragma unroll
        for (int i = 0; i < NE; ++i) {
            const int c = g.t + SF_GT * i;
            aa[i] = s[BC + SF_GT * i];
            bb[i] = s[2 * BC + SF_GT * i];
            pp[i] = s[3 * BC + SF_GT * i];
            u[i] = __ldg(ly.first + c);
            dec[i] = __ldg(ly.decay + c);
            wk[i] = h2f(__ldg(ly.wscale[G_K] + c));
            wv[i] = h2f(__ldg(ly.wscale[G_V] + c));
            wr[i] = h2f(__ldg(ly.wscale[G_R] + c));
        }
    }
};

// k, v, r -> WKV -> r*y, quantised
template <int EPL>
__device__ void row_wkv(const Grp& g, const SfHot& p, int l, int b, WkvIn<EPL>& in) {
    rmark(p, g, b, 1 + 4 * l, 0);
    constexpr int NE = EPL / 4;
    const int C = p.C;
    const size_t BC = (size_t)p.B * C;
    float* s = p.state + (size_t)l * 5 * BC + (size_t)b * C + g.t;
    const float sk = __ldcg(p.s_kx + b), sv = __ldcg(p.s_vx + b), sr = __ldcg(p.s_rx + b);
    PartLd<NE, SfKs<EPL>::KVR> lk, lv, lr;
    const int ks = p.ks[G_K];
    lk.issue(g, p.part[G_K], ks, p.B, C, b);
    lv.issue(g, p.part[G_V], ks, p.B, C, b);
    lr.issue(g, p.part[G_R], ks, p.B, C, b);
    int ak[NE], av[NE], ar[NE];
    lk.sum(g, p.part[G_K], ks, p.B, C, b, ak);
    lv.sum(g, p.part[G_V], ks, p.B, C, b, av);
    lr.sum(g, p.part[G_R], ks, p.B, C, b, ar);
    float ry[NE];
#pragma unroll
    for (int i = 0; i < NE; ++i) {
        const float k = epi_dequant(ak[i], sk, in.wk[i]);
        const float v = epi_dequant(av[i], sv, in.wv[i]);
        const float r = f16r(epi_sigmoid(epi_dequant(ar[i], sr, in.wr[i])));
        const float y = p.conv == KB_WKV_STEP_REF
                            ? wkv_step<KB_WKV_STEP_REF>(in.aa[i], in.bb[i], in.pp[i], k, v, in.u[i], in.dec[i])
                            : wkv_step<KB_WKV_PRODUCTION>(in.aa[i], in.bb[i], in.pp[i], k, v, in.u[i], in.dec[i]);
        ry[i] = f16r(__fmul_rn(r, y));
    }
    rmark(p, g, b, 1 + 4 * l, 1);
    group_quant_store<NE>(g, ry, p.q_ry + (size_t)b * C, p.s_ry + b);
    rmark(p, g, b, 1 + 4 * l, 2);
#pragma unroll
    for (int i = 0; i < NE; ++i) {
        s[BC + SF_GT * i] = in.aa[i];
        s[2 * BC + SF_GT * i] = in.bb[i];
        s[3 * BC + SF_GT * i] = in.pp[i];
    }
    rmark(p, g, b, 1 + 4 * l, 3);
}

template <int EPL>
struct AttIn {
    static constexpr int NE = EPL / 4;
    LnMixIn<EPL, 2> ln;
    float* srow;
    float x[NE], wo[NE];
    __device__ __forceinline__ void load(const Grp& g, const SfHot& p, int l, int b) {
        const size_t BC = (size_t)p.B * p.C;
        const SfLayer& ly = p.layer[l];
        const float* const mix[3] = {ly.fmix_k, ly.fmix_r, nullptr};
        srow = p.state + (size_t)l * 5 * BC + 4 * BC + (size_t)b * p.C;
        ln.load(g, ly.ln2_w, ly.ln2_b, mix, srow);
        const uint16_t* xr = p.x + (size_t)b * p.C + g.t;
#pragma unroll
        for (int i = 0; i < NE; ++i) {
            x[i] = h2f(xr[SF_GT * i]);
            wo[i] = h2f(__ldg(ly.wscale[G_O] + g.t + SF_GT * i));
        }
    }
};

// x += (r*y) @ Ow; LN2 + the two channel-mix outputs, quantised; ffn_xx <- LN2(x)
template <int EPL>
__device__ void row_att_out(const Grp& g, const SfHot& p, int l, int b, AttIn<EPL>& in) {
    rmark(p, g, b, 2 + 4 * l, 0);
    constexpr int NE = EPL / 4;
    const int C = p.C;
    uint16_t* xr = p.x + (size_t)b * C + g.t;
    const float sa = __ldcg(p.s_ry + b);
    PartLd<NE, SfKs<EPL>::O> lo;
    lo.issue(g, p.part[G_O], p.ks[G_O], p.B, C, b);
    int acc[NE];
    lo.sum(g, p.part[G_O], p.ks[G_O], p.B, C, b, acc);
    float v[NE];
#pragma unroll
    for (int i = 0; i < NE; ++i) {
        v[i] = f16r(epi_gate_resid(1.0f, epi_dequant(acc[i], sa, in.wo[i]), in.x[i]));
        g.xs[g.t + SF_GT * i] = v[i];
    }
    rmark(p, g, b, 2 + 4 * l, 1);
    int8_t* const q[3] = {p.q_kx + (size_t)b * C, p.q_rx + (size_t)b * C, nullptr};
    float* const qs[3] = {p.s_kx + b, p.s_rx + b, nullptr};
    ln_mix_g<EPL, 2>(g, v, C, in.ln, in.srow, q, qs);
    rmark(p, g, b, 2 + 4 * l, 2);
#pragma unroll
    for (int i = 0; i < NE; ++i) xr[SF_GT * i] = f2h(v[i]);
    rmark(p, g, b, 2 + 4 * l, 3);
}

// the ffn-mid phase has no early inputs worth holding in registers (its
// per-channel scales are loaded beside the partial sums)
template <int EPL>
struct MidIn {
    __device__ __forceinline__ void load(const Grp&, const SfHot&, int, int) {}
};

// kk = relu(k)^2 quantised per row (F = 4C: EPL values per thread);
// r2 = sigmoid(r) (fp16)
template <int EPL>
__device__ void row_ffn_mid(const Grp& g, const SfHot& p, int l, int b, MidIn<EPL>&) {
    rmark(p, g, b, 3 + 4 * l, 0);
    constexpr int NE = EPL / 4, NF = EPL;
    const int C = p.C, F = p.F;
    const SfLayer& ly = p.layer[l];
    float wk[NF], wr[NE];
#pragma unroll
    for (int i = 0; i < NF; ++i) wk[i] = h2f(__ldg(ly.wscale[G_FK] + g.t + SF_GT * i));
#pragma unroll
    for (int i = 0; i < NE; ++i) wr[i] = h2f(__ldg(ly.wscale[G_FR] + g.t + SF_GT * i));
    const float sk = __ldcg(p.s_kx + b), sr = __ldcg(p.s_rx + b);
    const int ks = p.ks[G_FK];
    PartLd<NF, SfKs<EPL>::FKR> lk;
    PartLd<NE, SfKs<EPL>::FKR> lr;
    lk.issue(g, p.part[G_FK], ks, p.B, F, b);
    lr.issue(g, p.part[G_FR], ks, p.B, C, b);
    int ak[NF], ar[NE];
    lk.sum(g, p.part[G_FK], ks, p.B, F, b, ak);
    lr.sum(g, p.part[G_FR], ks, p.B, C, b, ar);
    float kk[NF];
#pragma unroll
    for (int i = 0; i < NF; ++i) kk[i] = f16r(epi_relu_sq(epi_dequant(ak[i], sk, wk[i])));
    rmark(p, g, b, 3 + 4 * l, 1);
    group_quant_store<NF>(g, kk, p.q_kk + (size_t)b * F, p.s_kk + b);
    rmark(p, g, b, 3 + 4 * l, 2);
#pragma unroll
    for (int i = 0; i < NE; ++i)
        p.r2[(size_t)b * C + g.t + SF_GT * i] = f2h(epi_sigmoid(epi_dequant(ar[i], sr, wr[i])));
    rmark(p, g, b, 3 + 4 * l, 3);
}

template <int EPL>
struct OutIn {
    static constexpr int NE = EPL / 4;
    LnMixIn<EPL, 3> ln;  // LN1 of layer l+1, or ln_out (mixes unused)
    float* srow;
    float x[NE], gt[NE], wv[NE];
    __device__ __forceinline__ void load(const Grp& g, const SfHot& p, int l, int b) {
        const SfLayer& ly = p.layer[l];
        if (l + 1 < p.L) {
            srow = ln1_in<EPL>(g, p, l + 1, b, ln);
        } else {
            srow = nullptr;
#pragma unroll
            for (int i = 0; i < NE; ++i) {
                ln.w[i] = __ldg(p.ln_out_w + g.t + SF_GT * i);
                ln.bi[i] = __ldg(p.ln_out_b + g.t + SF_GT * i);
            }
        }
        const uint16_t* xr = p.x + (size_t)b * p.C + g.t;
        const uint16_t* r2 = p.r2 + (size_t)b * p.C + g.t;
#pragma unroll
        for (int i = 0; i < NE; ++i) {
            x[i] = h2f(xr[SF_GT * i]);
            gt[i] = h2f(r2[SF_GT * i]);
            wv[i] = h2f(__ldg(ly.wscale[G_FV] + g.t + SF_GT * i));
        }
    }
};

// x += r2 * (kk @ Vw); then LN1 + mix of layer l+1, or ln_out + quantisation
template <int EPL>
__device__ void row_ffn_out(const Grp& g, const SfHot& p, int l, int b, OutIn<EPL>& in) {
    rmark(p, g, b, 4 + 4 * l, 0);
    constexpr int NE = EPL / 4;
    const int C = p.C;
    uint16_t* xr = p.x + (size_t)b * C + g.t;
    const float sa = __ldcg(p.s_kk + b);
    PartLd<NE, SfKs<EPL>::FV> lf;
    lf.issue(g, p.part[G_FV], p.ks[G_FV], p.B, C, b);
    int acc[NE];
    lf.sum(g, p.part[G_FV], p.ks[G_FV], p.B, C, b, acc);
    float v[NE];
#pragma unroll
    for (int i = 0; i < NE; ++i) {
        v[i] = f16r(epi_gate_resid(in.gt[i], epi_dequant(acc[i], sa, in.wv[i]), in.x[i]));
        g.xs[g.t + SF_GT * i] = v[i];
    }
    rmark(p, g, b, 4 + 4 * l, 1);
    if (l + 1 < p.L) {
        ln1_mix_g<EPL>(g, p, b, v, in.ln, in.srow);
    } else {
        int8_t* const q[3] = {p.q_kx + (size_t)b * C, nullptr, nullptr};
        float* const qs[3] = {p.s_kx + b, nullptr, nullptr};
        ln_mix_g<EPL, 0>(g, v, C, in.ln, nullptr, q, qs);
    }
    rmark(p, g, b, 4 + 4 * l, 2);
#pragma unroll
    for (int i = 0; i < NE; ++i) xr[SF_GT * i] = f2h(v[i]);
    rmark(p, g, b, 4 + 4 * l, 3);
}

template <int EPL>
__global__ void __launch_bounds__(SF_NT, 1) k_step_fused(const __grid_constant__ SfParams P) {
    extern __shared__ unsigned char sf_smem_raw[];
    const uint32_t raw = tc::smem_addr(sf_smem_raw);
    unsigned char* smem = sf_smem_raw + (((raw + 1023u) & ~1023u) - raw);
    SfHot& p = *reinterpret_cast<SfHot*>(smem + SF_HOT_OFF);
    {
        static_assert(sizeof(SfHot) % 4 == 0, "word copy");
        const uint32_t* src = reinterpret_cast<const uint32_t*>(&P.h);
        uint32_t* dst = reinterpret_cast<uint32_t*>(&p);
        for (int i = threadIdx.x; i < (int)(sizeof(SfHot) / 4); i += blockDim.x) dst[i] = src[i];
    }
    SfBars* sb = reinterpret_cast<SfBars*>(smem + SF_A_BYTES + 2 * SF_W_BYTES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        tc::mbar_init(&sb->a_full, 1);
        tc::mbar_init(&sb->w_full[0], 1);
        tc::mbar_init(&sb->w_full[1], 1);
        tc::mbar_init(&sb->mma_done, 1);
        tc::fence_barrier_init();
    }
    if (warp == 0) tc::tmem_alloc(&sb->tmem_base, SF_BN);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = sb->tmem_base;

    SfState st{{0, 0}, 0, 0, {0, 0}};
    // weights of the first tile phase, fetched while the embedding runs
    if (threadIdx.x == 0) {
        // (the other threads read the table after the first grid barrier)
        for (int k = 0; k < 4; ++k) sb->has_first[k] = unit_at(p, k, blockIdx.x, sb->first[k]);
        if (sb->has_first[0]) {
            issue_w(P, p, sb, smem + SF_A_BYTES, 0, 0, sb->first[0]);
            st.w_pending[0] = 1;
        }
    }
    // row groups: group 0 of every CTA takes the first rows, then group 1
    Grp grp;
    grp.id = warp >> 2;
    grp.t = threadIdx.x & (SF_GT - 1);
    grp.w = warp & 3;
    grp.lane = lane;
    grp.xs = reinterpret_cast<float*>(smem + SF_ROW_OFF) + grp.id * (SF_MAX_C + SF_RED);
    grp.red = grp.xs + SF_MAX_C;
    const int gw = grp.id * gridDim.x + blockIdx.x, nw = 2 * gridDim.x;
    unsigned epoch = 0;
    bool ok = true;
    for (int b = gw; b < p.B; b += nw) row_embed<EPL>(grp, p, b);
    ok = grid_sync(p, sb, ++epoch);
// a row phase after its opening barrier, one row per group at a time
#define SF_ROWS(IN, FN)                                                  \
    {                                                                    \
        IN<EPL> in;                                                      \
        if (!(ok = grid_sync(p, sb, ++epoch))) break;                   \
        for (int b = gw; b < p.B; b += nw) {                             \
            in.load(grp, p, l, b);                                       \
            FN<EPL>(grp, p, l, b, in);                                   \
        }                                                                \
    }
    for (int l = 0; l < p.L && ok; ++l) {
        tile_phase(P, p, sb, smem, tmem, 4 * l + 0, st);
        SF_ROWS(WkvIn, row_wkv)
        if (!(ok = grid_sync(p, sb, ++epoch))) break;
        tile_phase(P, p, sb, smem, tmem, 4 * l + 1, st);
        SF_ROWS(AttIn, row_att_out)
        if (!(ok = grid_sync(p, sb, ++epoch))) break;
        tile_phase(P, p, sb, smem, tmem, 4 * l + 2, st);
        SF_ROWS(MidIn, row_ffn_mid)
        if (!(ok = grid_sync(p, sb, ++epoch))) break;
        tile_phase(P, p, sb, smem, tmem, 4 * l + 3, st);
        SF_ROWS(OutIn, row_ffn_out)
        if (l + 1 < p.L && !(ok = grid_sync(p, sb, ++epoch))) break;
    }
#undef SF_ROWS
    // a prefetched weight load that no phase consumed (abort) must land
    // before the CTA exits
    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i)
            if (st.w_pending[i]) tc::mbar_wait(&sb->w_full[i], st.w_uses[i] & 1u);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, SF_BN);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            ptr = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }();
    return fn;
}

// int8 [rows, cols] row-major, box 128 bytes x box_rows, 128-byte swizzle
bool map_i8(CUtensorMap* map, const void* base, int rows, int cols, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols};
    cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// int32 partial sums [slices][B][N], box 32 columns x 128 rows x 1 slice,
// 128-byte swizzle (the staging layout)
bool map_part(CUtensorMap* map, void* base, int N, int B, int slices) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)B, (cuuint64_t)slices};
    cuuint64_t strides[2] = {(cuuint64_t)N * 4, (cuuint64_t)B * N * 4};
    cuuint32_t box[3] = {32, 128, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_INT32, 3, base, dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }

int sm_count_now() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

// K slices of a phase: the most that keeps the phase's units within the
// grid, with at most SF_MAX_KB K blocks per unit and nkb % slices == 0.
int pick_slices(int units_per_slice, int nkb, int grid) {
    int best = 0;
    for (int d = 1; d <= nkb; ++d) {
        if (nkb % d || nkb / d > SF_MAX_KB) continue;
        if (best == 0) best = d;  // smallest admissible
        if ((int64_t)units_per_slice * d <= grid) best = d;
    }
    return best;
}

struct Layout {
    size_t x, kk, r2, q_kx, q_vx, q_rx, q_ry, q_kk, s_kx, s_vx, s_rx, s_ry, s_kk, bar;
    size_t part[G_NUM];
    int ks[G_NUM];
    size_t total;
};

Layout make_layout(const kb_model_desc& d, int B, int grid) {
    Layout o{};
    const size_t C = d.n_embd, F = d.n_ffn;
    const int MT = (B + 127) / 128;
    const int nkbC = (int)(C / 128), nkbF = (int)(F / 128);
    const int ntC = (int)(C / SF_BN), ntF = (int)(F / SF_BN);
    o.ks[G_K] = o.ks[G_V] = o.ks[G_R] = pick_slices(MT * 3 * ntC, nkbC, grid);
    o.ks[G_O] = pick_slices(MT * ntC, nkbC, grid);
    o.ks[G_FK] = o.ks[G_FR] = pick_slices(MT * (ntF + ntC), nkbC, grid);
    o.ks[G_FV] = pick_slices(MT * ntC, nkbF, grid);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off += al256(bytes);
        return at;
    };
    o.bar = take(256);
    o.x = take((size_t)B * C * 2);
    o.kk = take((size_t)B * F * 2);
    o.r2 = take((size_t)B * C * 2);
    o.q_kx = take((size_t)B * C);
    o.q_vx = take((size_t)B * C);
    o.q_rx = take((size_t)B * C);
    o.q_ry = take((size_t)B * C);
    o.q_kk = take((size_t)B * F);
    o.s_kx = take((size_t)B * 4);
    o.s_vx = take((size_t)B * 4);
    o.s_rx = take((size_t)B * 4);
    o.s_ry = take((size_t)B * 4);
    o.s_kk = take((size_t)B * 4);
    const size_t N[G_NUM] = {C, C, C, C, F, C, C};
    for (int g = 0; g < G_NUM; ++g) o.part[g] = take((size_t)o.ks[g] * B * N[g] * 4);
    o.total = off;
    return o;
}

unsigned long long* g_step_trace = nullptr;
struct StepFault {
    unsigned long long spin_ns = 0;
    int withhold = 0;
};
StepFault g_step_fault;

struct StepCache {
    const void* ws = nullptr;
    int B = 0, grid = 0;
    std::unique_ptr<SfParams> p;  // maps and workspace pointers
};

bool supported_epl(int C) { return C == 128 || C == 768 || C == 2048; }

}  // namespace

}  // namespace kb

using namespace kb;

extern "C" size_t kb_step_workspace_bytes(const kb_model* m, int B) {
    if (!m || B <= 0) return 0;
    return make_layout(m->d, B, sm_count_now()).total;
}

extern "C" int kb_step_forward(kb_model* m, const int32_t* tokens, int B, float* state, void* ws,
                               size_t ws_bytes, uint16_t* logits, float* logit_stats,
                               void* stream) {
    if (!m || !tokens || !state || !ws || !logits || B <= 0) return KB_ERR_ARG;
    const kb_model_desc& d = m->d;
    if (d.wdtype != KB_I8) return KB_ERR_UNSUPPORTED;
    if (d.n_layer > SF_MAX_LAYERS || !supported_epl(d.n_embd) || d.n_ffn != 4 * d.n_embd)
        return KB_ERR_SHAPE;
    if (!aligned16(ws) || !aligned16(logits) || ((uintptr_t)logit_stats & 7u)) return KB_ERR_ALIGN;
    const int grid = sm_count_now();
    const Layout lo = make_layout(d, B, grid);
    if (ws_bytes < lo.total) return KB_ERR_WORKSPACE;
    cudaStream_t st = as_stream(stream);
    char* base = reinterpret_cast<char*>(ws);

    SfParams* p = nullptr;
    {
        std::lock_guard<std::mutex> lock(m->step_mu);
        auto cache = std::static_pointer_cast<StepCache>(m->step_cache);
        if (!cache || cache->ws != ws || cache->B != B || cache->grid != grid) {
            auto c = std::make_shared<StepCache>();
            c->ws = ws;
            c->B = B;
            c->grid = grid;
            c->p.reset(new (std::nothrow) SfParams());
            if (!c->p) return KB_ERR_NOMEM;
            SfParams& q = *c->p;
            q.h.L = d.n_layer;
            q.h.B = B;
            q.h.C = d.n_embd;
            q.h.F = d.n_ffn;
            q.h.V = d.n_vocab;
            q.h.conv = d.wkv_convention;
            for (int g = 0; g < G_NUM; ++g) q.h.ks[g] = lo.ks[g];
            for (int l = 0; l < d.n_layer; ++l) {
                const kb_layer_desc& L = d.layers[l];
                const void* W[G_NUM] = {L.att_kw, L.att_vw, L.att_rw, L.att_ow,
                                        L.ffn_kw, L.ffn_rw, L.ffn_vw};
                const uint16_t* S[G_NUM] = {L.att_ks, L.att_vs, L.att_rs, L.att_os,
                                            L.ffn_ks, L.ffn_rs, L.ffn_vs};
                const int Nn[G_NUM] = {q.h.C, q.h.C, q.h.C, q.h.C, q.h.F, q.h.C, q.h.C};
                const int Kk[G_NUM] = {q.h.C, q.h.C, q.h.C, q.h.C, q.h.C, q.h.C, q.h.F};
                for (int g = 0; g < G_NUM; ++g) {
                    if (!map_i8(&q.wmap[l][g], W[g], Nn[g], Kk[g], SF_BN))
                        return KB_ERR_UNSUPPORTED;
                    q.h.layer[l].wscale[g] = S[g];
                }
                SfLayer& y = q.h.layer[l];
                y.ln1_w = L.ln1_w; y.ln1_b = L.ln1_b; y.ln2_w = L.ln2_w; y.ln2_b = L.ln2_b;
                y.mix_k = L.att_mix_k; y.mix_v = L.att_mix_v; y.mix_r = L.att_mix_r;
                y.decay = L.att_decay; y.first = L.att_first;
                y.fmix_k = L.ffn_mix_k; y.fmix_r = L.ffn_mix_r;
            }
            q.h.emb = d.emb;
            q.h.ln_out_w = d.ln_out_w;
            q.h.ln_out_b = d.ln_out_b;
            q.h.x = (uint16_t*)(base + lo.x);
            q.h.kk = (uint16_t*)(base + lo.kk);
            q.h.r2 = (uint16_t*)(base + lo.r2);
            q.h.q_kx = (int8_t*)(base + lo.q_kx);
            q.h.q_vx = (int8_t*)(base + lo.q_vx);
            q.h.q_rx = (int8_t*)(base + lo.q_rx);
            q.h.q_ry = (int8_t*)(base + lo.q_ry);
            q.h.q_kk = (int8_t*)(base + lo.q_kk);
            q.h.s_kx = (float*)(base + lo.s_kx);
            q.h.s_vx = (float*)(base + lo.s_vx);
            q.h.s_rx = (float*)(base + lo.s_rx);
            q.h.s_ry = (float*)(base + lo.s_ry);
            q.h.s_kk = (float*)(base + lo.s_kk);
            for (int g = 0; g < G_NUM; ++g) q.h.part[g] = (int32_t*)(base + lo.part[g]);
            q.h.bar = (unsigned*)(base + lo.bar);
            const void* A[A_NUM] = {q.h.q_kx, q.h.q_vx, q.h.q_rx, q.h.q_ry, q.h.q_kk};
            const int Ak[A_NUM] = {q.h.C, q.h.C, q.h.C, q.h.C, q.h.F};
            for (int a = 0; a < A_NUM; ++a)
                if (!map_i8(&q.amap[a], A[a], B, Ak[a], 128)) return KB_ERR_UNSUPPORTED;
            const int Np[G_NUM] = {q.h.C, q.h.C, q.h.C, q.h.C, q.h.F, q.h.C, q.h.C};
            for (int g = 0; g < G_NUM; ++g)
                if (!map_part(&q.pmap[g], q.h.part[g], Np[g], B, lo.ks[g]))
                    return KB_ERR_UNSUPPORTED;
            m->step_cache = c;
            cache = c;
        }
        p = cache->p.get();
    }
    p->h.tokens = tokens;
    p->h.state = state;
    p->h.trace = g_step_trace;
    p->h.spin_ns = g_step_fault.spin_ns ? g_step_fault.spin_ns : SF_SPIN_NS;
    p->h.withhold_arrival = g_step_fault.withhold;

    static std::atomic<unsigned long long> done{0};
    const cudaError_t attr_err = once_per_device(done, [] {
        const int sm = (int)SF_SMEM;
        cudaError_t e = cudaSuccess;
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k_step_fused<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k_step_fused<24>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k_step_fused<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
        return e;
    });
    if (attr_err != cudaSuccess) {
        set_cuda_error(attr_err);
        return KB_ERR_CUDA;
    }
    {
        ProfScope ps(PH_STEP, st, 2.0 * B * (double)d.n_layer *
                                      (5.0 * d.n_embd * d.n_embd + 2.0 * d.n_embd * d.n_ffn));
        cudaError_t e = cudaMemsetAsync(p->h.bar, 0, 2 * sizeof(unsigned), st);
        if (e != cudaSuccess) {
            set_cuda_error(e);
            return KB_ERR_CUDA;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)grid);
        cfg.blockDim = dim3(SF_NT);
        cfg.dynamicSmemBytes = SF_SMEM;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const int epl = d.n_embd / 32;
        if (epl == 4) e = cudaLaunchKernelEx(&cfg, k_step_fused<4>, *p);
        else if (epl == 24) e = cudaLaunchKernelEx(&cfg, k_step_fused<24>, *p);
        else e = cudaLaunchKernelEx(&cfg, k_step_fused<64>, *p);
        if (e != cudaSuccess) {
            set_cuda_error(e);
            return KB_ERR_CUDA;
        }
    }
    // head: the same kernel as the window forward, on the fused step's output
    {
        ProfScope ps(PH_HEAD, st, 2.0 * B * (double)d.n_vocab * d.n_embd);
        const int8_t* hw = (const int8_t*)d.head;
        if (logit_stats)
            return launch_gemm_logits_i8(p->h.q_kx, d.n_embd, p->h.s_kx, hw, d.n_embd, d.head_scale,
                                         B, d.vocab_pad, d.n_embd, logits, d.vocab_pad, d.n_vocab,
                                         logit_stats, d.vocab_pad / 32, st);
        return launch_gemm_i8(p->h.q_kx, d.n_embd, p->h.s_kx, hw, d.n_embd, d.head_scale, B,
                              d.vocab_pad, d.n_embd, KB_EPI_F16, logits, d.vocab_pad, nullptr,
                              nullptr, st);
    }
}

// Profiling aid: when trace is non-NULL (device, >= 2048 u64), CTA 0 of
// every later kb_step_forward records %globaltimer at each grid barrier's
// entry (even slots) and exit (odd slots), and for its first unit of tile
// phase tp at slots 512 + 4 tp + {loads issued, operands landed, MMAs done,
// partials stored} and at barrier exits at 768 + epoch, as SM clock counts,
// and for row 0 of row phase rp (1 + 4 layer + {wkv, ln2, ffn mid, ln1})
// at slots 1024 + 4 rp + {entry, data consumed, row reduction done, end}.
// NULL turns it off.
extern "C" int kb_step_set_trace(unsigned long long* trace) {
    kb::g_step_trace = trace;
    return KB_OK;
}

// Failure-detection test hook: with withhold != 0, CTA 0 of every later
// kb_step_forward skips its arrival at the first grid barrier, so every CTA's
// bounded wait expires (after spin_ns, default 2 s when 0): the step aborts
// cleanly and kb_step_error_status reports KB_ERR_TIMEOUT.  (0, 0) restores
// normal operation.
extern "C" int kb_step_set_fault(int withhold, long long spin_ns) {
    if (spin_ns < 0) return KB_ERR_ARG;
    kb::g_step_fault.withhold = withhold ? 1 : 0;
    kb::g_step_fault.spin_ns = (unsigned long long)spin_ns;
    return KB_OK;
}

extern "C" int kb_step_error_status(int reset) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, kb::g_step_error, sizeof(int)) != cudaSuccess) return KB_ERR_CUDA;
    if (reset && v) {
        const int z = 0;
        cudaMemcpyToSymbol(kb::g_step_error, &z, sizeof(int));
    }
    return v ? KB_ERR_TIMEOUT : KB_OK;
}
