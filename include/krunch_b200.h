/*
 * krunch_b200 — C ABI of the B200-native krunch compress/decompress hot path.
 *
 * Every entry point takes raw device pointers, explicit sizes and an explicit
 * cudaStream_t (passed as void* so this header needs no CUDA include), enqueues
 * work on that stream and returns without synchronising.  Return value is a
 * kb_status (0 = ok, negative = error).  On KB_ERR_CUDA the CUDA error code is
 * kept in a thread-local slot readable with kb_last_cuda_error().
 *
 * Hot-path calls never allocate device memory: callers size a workspace with
 * the matching *_workspace_bytes() query and pass it in.
 *
 * Each declaration names the reference interface it replaces
 * (paths are relative to the dmatth1/krunch source tree).
 */
#ifndef KRUNCH_B200_H
#define KRUNCH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------- */
/* status                                                                    */
/* ------------------------------------------------------------------------- */
enum kb_status {
    KB_OK = 0,
    KB_ERR_ARG = -1,         /* null pointer / bad enum / bad size            */
    KB_ERR_SHAPE = -2,       /* unsupported shape (e.g. K not multiple of 64) */
    KB_ERR_ALIGN = -3,       /* pointer or stride not aligned as required     */
    KB_ERR_CUDA = -4,        /* CUDA runtime error, see kb_last_cuda_error()  */
    KB_ERR_TIMEOUT = -5,     /* bounded device wait expired                   */
    KB_ERR_UNSUPPORTED = -6, /* feature not built for this device             */
    KB_ERR_WORKSPACE = -7,   /* workspace smaller than the query returned     */
    KB_ERR_NOMEM = -8,       /* host allocation failed (model handle)         */
    KB_ERR_TOO_LARGE = -9    /* request exceeds the fixed no-alloc scratch    */
};

const char* kb_version(void);

/* Phase profiler (the counterpart of the reference's KRUNCH_PHASE_PROFILE
 * event timers, krunch_ac/cuda/layer_cpp.cpp:111-157, read_phase_times
 * 825-836).  Between begin and end every launch of this library is bracketed
 * by CUDA events on its stream.  end() waits for those events and fills, per
 * phase (0 embed, 1 layernorm+mix, 2 layer GEMMs, 3 WKV, 4 head GEMM,
 * 5 CDF, 6 encode, 7 decode step), the summed milliseconds, the launch count
 * and the algorithmic work (FLOPs for GEMM phases, bytes otherwise).
 * Host-thread global; not for use inside stream capture. */
int kb_profile_begin(void);
int kb_profile_end(double* ms, int64_t* launches, double* work, int n_phases);
const char* kb_status_string(int status);
int kb_last_cuda_error(void);

/* ------------------------------------------------------------------------- */
/* range coder — one lane (thread) per stream                                */
/*                                                                           */
/* Per-stream state is 4 x uint32:                                           */
/*   encoder {low, high, pending, bit_offset}                                */
/*   decoder {low, high, value,   bit_offset}                                */
/* Same layout as RangeState / DecodeState in                                */
/* krunch_ac/cuda/range_coder.cuh:24-40.  cdf_bits is the log2 of the CDF     */
/* total (16 or 24; the reference hard-codes 24, range_coder.cuh:19).         */
/* Output bits are MSB-first; output buffers must be zeroed beyond the        */
/* current bit_offset (krunch_ac/cpu_reference.py:91-147 bit order).          */
/* Stream b writes/reads bytes starting at base + offsets[b] (offsets NULL    */
/* means every stream starts at byte 0, used with B == 1).  out_bytes /       */
/* in_bytes bound the whole buffer: writes past it are dropped (bit_offset    */
/* still advances, so the host detects overflow) and reads past it return     */
/* zero bits, the CPU reference's past-EOF rule (cpu_reference.py:68-72).     */
/* ------------------------------------------------------------------------- */

/* low=0, high=0xFFFFFFFF, pending=0, bit_offset=0 for n streams
 * (replaces the host-side state init in krunch/inference.py:325-330). */
int kb_coder_encode_init(uint32_t* states, int n_streams, void* stream);

/* Encode n rows of one stream from full CDF rows:
 * cdf int32 [n, cdf_stride] (cdf[i,0]=0, cdf[i,V]=2^cdf_bits), symbols int32 [n].
 * Replaces encode_step (krunch_ac/cuda/main.cpp:114-143,
 * encode_kernel.cu:53-103). */
int kb_coder_encode_cdf(const int32_t* cdf, int64_t cdf_stride, const int32_t* symbols,
                        int n, int cdf_bits, uint8_t* out, int64_t out_bytes,
                        uint32_t* state, void* stream);

/* One symbol per stream for B streams: cdfs int32 [B, cdf_stride].
 * Replaces encode_step_batched (main.cpp:254-284, encode_kernel.cu:148-197). */
int kb_coder_encode_cdf_batched(const int32_t* cdfs, int64_t cdf_stride,
                                const int32_t* symbols, int B, int cdf_bits,
                                uint8_t* out, int64_t out_bytes, const int64_t* out_offsets,
                                uint32_t* states, void* stream);

/* Lane-per-stream encode of pre-narrowed intervals: lohi uint32 [B, T, 2]
 * holds (cdf[sym], cdf[sym+1]) for every row (written by kb_cdf_rows in
 * KB_CDF_LOHI mode); stream b encodes rows 0..n_valid[b]-1 (n_valid NULL =
 * all T).  This is the fused replacement of the per-chunk serial
 * encode_step<<<1,1>>> loop (krunch/inference.py:331-338). */
int kb_coder_encode_lohi(const uint32_t* lohi, int B, int T, const int32_t* n_valid,
                         int cdf_bits, uint8_t* out, int64_t out_bytes,
                         const int64_t* out_offsets, uint32_t* states, void* stream);

/* Final flush: one bit + pending bits.  Replaces encode_finalize /
 * encode_finalize_batched (encode_kernel.cu:106-119, main.cpp:145-156,286-303). */
int kb_coder_encode_finalize(uint8_t* out, int64_t out_bytes, const int64_t* out_offsets,
                             uint32_t* states, int B, void* stream);

/* Read the first 32 bits of each stream.  Replaces decode_init /
 * decode_init_batched (decode_kernel.cu:28-45,138-160; main.cpp:158-219). */
int kb_coder_decode_init(const uint8_t* in, int64_t in_bytes, const int64_t* in_offsets,
                         uint32_t* states, int B, void* stream);

/* Decode one symbol per stream from full CDF rows cdfs int32 [B, cdf_stride]
 * with V = number of symbols.  Replaces decode_step / decode_step_batched
 * (decode_kernel.cu:49-110,162-216; main.cpp:173-252). */
int kb_coder_decode_cdf(const int32_t* cdfs, int64_t cdf_stride, int V, int cdf_bits,
                        const uint8_t* in, int64_t in_bytes, const int64_t* in_offsets,
                        uint32_t* states, int32_t* out_syms, int B, void* stream);

/* ------------------------------------------------------------------------- */
/* logits -> softmax -> integer CDF (one CTA per row, row-local, bit-identical */
/* for any number of rows).  Spec: krunch_ac/cdf.py:22-74 (count =            */
/* floor(p*(T-V))+1, deficit to argmax with smallest-index tie-break) and     */
/* krunch_ac/cuda/det_softmax_cdf.cu:62-185.                                  */
/* ------------------------------------------------------------------------- */
enum kb_cdf_mode {
    KB_CDF_COUNTS = 0, /* out int32 [rows, V+1]: 0, count_0 .. count_{V-1}
                          (det_softmax_cdf contract, layer_cpp.cpp:1041-1052) */
    KB_CDF_CDF = 1,    /* out int32 [rows, V+1]: cumulative CDF            */
    KB_CDF_LOHI = 2    /* out uint32 [rows, 2]: (cdf[s], cdf[s+1]) for
                          s = symbols[row]; feeds kb_coder_encode_lohi      */
};

/* With logit_stats NULL, logits_f16 holds raw fp16 logits [rows, row_stride]
 * (V valid columns).  With logit_stats non-NULL it holds what
 * kb_forward_window writes when asked for stats: per 32-column subtile u the
 * fp16 numerators e^(x - m_u), and logit_stats float2 [rows, stats_stride]
 * the subtile partials (m_u, sum of the numerators), stats_stride >=
 * ceil(V / 32).  Both inputs give bit-identical CDFs (the kernel derives the
 * numerators and partials from raw logits itself). */
int kb_cdf_rows(const uint16_t* logits_f16, int64_t row_stride, int rows, int V,
                int cdf_bits, int mode, const float* logit_stats, int64_t stats_stride,
                const int32_t* symbols, void* out, void* stream);

/* probs fp32 [rows, V] -> int32 CDF [rows, V+1].  Replaces probs_to_cdf_gpu
 * (krunch_ac/gpu_encode.py:22-48) with a fixed-order row reduction. */
int kb_cdf_from_probs(const float* probs, int rows, int V, int cdf_bits, int32_t* cdf_out,
                      void* stream);

/* Fused decompress step tail: for each of B streams, softmax->CDF of its
 * logits row, target search and range-decoder update, one CTA per stream.
 * Replaces softmax_cdfs_per_row + decode_step_batched
 * (krunch/cpp_path.py:490-512, krunch/inference.py:426-434).
 * counters int32 [B, 2] = {symbols decoded so far, symbols in the stream}
 * (NULL: every stream active).  A finished stream keeps its state and gets
 * symbol 0 (the BOS pad input).  The decoded symbol goes to out_syms[b] (the
 * next step's input token) and, when history is non-NULL, to
 * history[b * hist_stride + counters[b][0]].  All pointers stay fixed from
 * step to step, so a decode step can be captured in a CUDA graph. */
int kb_decode_logits_step(const uint16_t* logits_f16, int64_t row_stride, int B, int V,
                          int cdf_bits, const float* logit_stats, int64_t stats_stride,
                          const uint8_t* in, int64_t in_bytes, const int64_t* in_offsets,
                          uint32_t* states, int32_t* counters, int32_t* out_syms,
                          int32_t* history, int64_t hist_stride, void* stream);

/* ------------------------------------------------------------------------- */
/* GEMM: out[M,N] = epilogue(A[M,K] @ W^T) with W stored K-major as [N,K]    */
/* (the transpose of the reference's [in,out] layout).  One tile schedule and */
/* one K order for every M, so each output row is bit-identical whatever M is */
/* (the M-invariance contract of krunch_ac/cuda/det_matmul_tc*.cu).           */
/* Replaces det_matmul (layer_cpp.cpp:728-822) and gemm_fp16 (206-290).       */
/* ------------------------------------------------------------------------- */
enum kb_epilogue {
    KB_EPI_F32 = 0,        /* out fp32 = acc                                 */
    KB_EPI_F16 = 1,        /* out fp16 = acc                                 */
    KB_EPI_SIGMOID = 2,    /* out fp16 = sigmoid(acc)                        */
    KB_EPI_RELU_SQ = 3,    /* out fp16 = relu(acc)^2                         */
    KB_EPI_RESID = 4,      /* out fp16 = resid + acc                         */
    KB_EPI_GATE_RESID = 5  /* out fp16 = resid + gate * acc                  */
};
enum kb_dtype { KB_F16 = 0, KB_BF16 = 1, KB_I8 = 2 };

/* A, W: both fp16 (dtype KB_F16) or both bf16 (KB_BF16; the relu^2
 * epilogue then writes bf16, the others fp16 / fp32 as for fp16).
 * resid/gate fp16 [M, ldo] (may alias out).
 * Requires N % 32 == 0, K % 64 == 0, 16-byte aligned rows and out. */
int kb_gemm(int dtype, const void* A, int64_t lda, const void* W, int64_t ldw,
            int M, int N, int K, int epilogue, void* out, int64_t ldo,
            const uint16_t* resid, const uint16_t* gate, void* stream);

/* w8a8 GEMM: A int8 [M, lda] with a fp32 dequantisation factor per row
 * (a_scale [M]), W int8 [N, ldw] with a fp16 factor per row of W (w_scale
 * [N], per output channel).  Exact int32 accumulation (tcgen05 kind::i8), then
 * y = (acc * a_scale[m]) * w_scale[n] and the epilogue as in kb_gemm.  Any
 * tiling gives the same bits.  Requires K % 128 == 0, N % 32 == 0.  The
 * reference's int8 GEMM is w8a16 (det_matmul_tc_uint8.cu:43-254); this is the
 * w8a8 scheme with per-output-channel scales. */
int kb_gemm_i8(const int8_t* A, int64_t lda, const float* a_scale, const int8_t* W,
               int64_t ldw, const uint16_t* w_scale, int M, int N, int K, int epilogue,
               void* out, int64_t ldo, const uint16_t* resid, const uint16_t* gate,
               int tile_n, void* stream);

/* The three attention projections of a layer in ONE launch over a shared
 * tile space: k = kx @ Kw^T (fp32), v = vx @ Vw^T (fp32),
 * r = sigmoid(rx @ Rw^T) (fp16), all [M, N] with row stride ldo.  dtype
 * KB_F16 / KB_BF16 (scales NULL) or KB_I8 (per-row A factors, per-output
 * channel W factors as in kb_gemm_i8).  Each output element has the bits of
 * the corresponding single kb_gemm / kb_gemm_i8 call.  Replaces
 * det_matmul_tc_3way_async (krunch_ac/cuda/det_matmul_tc_3way_async.cu:50-251,
 * routed at layer_cpp.cpp:531-556). */
int kb_gemm_kvr(int dtype, const void* kx, const void* vx, const void* rx, int64_t lda,
                const float* kx_scale, const float* vx_scale, const float* rx_scale,
                const void* kw, const void* vw, const void* rw, int64_t ldw,
                const uint16_t* kw_scale, const uint16_t* vw_scale, const uint16_t* rw_scale,
                int M, int N, int K, float* k, float* v, uint16_t* r, int64_t ldo, int tile_n,
                void* stream);

/* Per-output-channel int8 weight quantisation of fp16 W [N, K]:
 * scale[n] = fp16(max_k |W[n,k]| / 127), q = clamp(rint(W / scale), -127, 127). */
int kb_quantize_weight(const uint16_t* w, int N, int K, int8_t* q, uint16_t* scale,
                       void* stream);

/* Per-row int8 activation quantisation of fp16 x [R, K] (K % 8 == 0):
 * amax = max |x[r,:]|, q = clamp(rint(x * (127 / amax)), -127, 127),
 * scale[r] = amax / 127 (fp32; 0 for an all-zero row). */
int kb_quantize_rows(const uint16_t* x, int R, int K, int8_t* q, float* scale, void* stream);

/* kb_gemm with the output tile fixed: tile_n in {32, 64, 128, 256} for one
 * CTA per 128-row x tile_n tile, KB_TILE_PAIR for a cluster of two CTAs per
 * 256-row x 256-column tile (cta_group::2 MMAs; the library's choice for
 * large M), or 0 for the library's choice.  Every tiling gives bit-identical
 * results: an output element's K walk does not depend on the tile shape. */
#define KB_TILE_PAIR 512
int kb_gemm_tiled(int dtype, const void* A, int64_t lda, const void* W, int64_t ldw,
                  int M, int N, int K, int epilogue, void* out, int64_t ldo,
                  const uint16_t* resid, const uint16_t* gate, int tile_n, void* stream);

/* Device-side failure report of the tcgen05 kernels: every mbarrier wait in
 * them is bounded, and a wait that expires records an error and makes the
 * kernel unwind (no hang).  Returns KB_OK or KB_ERR_TIMEOUT (KB_ERR_CUDA if the
 * flag cannot be read); reset != 0 clears the flag.  Synchronises the device. */
int kb_device_error_status(int reset);

/* ------------------------------------------------------------------------- */
/* RWKV-4 model                                                               */
/* ------------------------------------------------------------------------- */
enum kb_wkv_convention {
    KB_WKV_STEP_REF = 0,   /* scripts/rwkv4_step_ref.py:76-94 (default)       */
    KB_WKV_PRODUCTION = 1  /* krunch_ac/cuda/wkv_kernel.cu:57-72               */
};

typedef struct kb_layer_desc {
    const float* ln1_w; const float* ln1_b;       /* [C] */
    const float* ln2_w; const float* ln2_b;       /* [C] */
    const float* att_mix_k; const float* att_mix_v; const float* att_mix_r; /* [C] */
    const float* att_decay;  /* [C] exp(time_decay): ww2 = pp - decay           */
    const float* att_first;  /* [C] time_first                                  */
    const void* att_kw; const void* att_vw; const void* att_rw; const void* att_ow; /* [C,C] K-major */
    const float* ffn_mix_k; const float* ffn_mix_r; /* [C] */
    const void* ffn_kw;  /* [F,C] */
    const void* ffn_vw;  /* [C,F] */
    const void* ffn_rw;  /* [C,C] */
    /* KB_I8 only: fp16 dequantisation factor per output channel (per row of
     * the K-major matrix above), 16-byte aligned; NULL for KB_F16. */
    const uint16_t* att_ks; const uint16_t* att_vs; const uint16_t* att_rs; const uint16_t* att_os;
    const uint16_t* ffn_ks; const uint16_t* ffn_vs; const uint16_t* ffn_rs;
} kb_layer_desc;

typedef struct kb_model_desc {
    int n_layer, n_embd, n_ffn, n_vocab;
    int vocab_pad;       /* head rows, multiple of 128, >= n_vocab           */
    int wdtype;          /* kb_dtype of the matrices                          */
    int wkv_convention;  /* kb_wkv_convention                                 */
    const uint16_t* emb; /* fp16 [n_vocab, C]                                 */
    const float* ln_out_w; const float* ln_out_b;
    const void* head;    /* [vocab_pad, C] K-major, rows >= n_vocab zero       */
    const kb_layer_desc* layers; /* n_layer entries (copied at create)        */
    const uint16_t* head_scale;  /* KB_I8: fp16 [vocab_pad] factors, else NULL  */
} kb_model_desc;

typedef struct kb_model kb_model;

/* Validates the description and copies it into an opaque host-side handle
 * (no device allocation).  Replaces cpp_path.init_weights
 * (krunch/cpp_path.py:26-91) on the native side. */
int kb_model_create(const kb_model_desc* desc, kb_model** out);
void kb_model_destroy(kb_model* model);

/* exp(time_decay) with the library's own fixed-order exp, so encoder and
 * decoder hosts derive identical decay constants. */
int kb_prepare_decay(const float* time_decay, float* decay_out, int n, void* stream);

/* Recurrent state: fp32 [n_layer][5][B][C]; slot 0 att_xx, 1 aa, 2 bb, 3 pp,
 * 4 ffn_xx (the 5-per-layer contract of cpp_path.fresh_state,
 * krunch/cpp_path.py:94-106, init_state_batched batched_rwkv4.py:60-82). */
int kb_state_init(const kb_model* model, float* state, int B, void* stream);

size_t kb_forward_workspace_bytes(const kb_model* model, int B, int T);

/* Packed forward of a window: tokens int32 [B, T] (inputs), state as above
 * (read and updated), logits fp16 [B*T, vocab_pad] (row b*T+t).  When
 * logit_stats is non-NULL the head writes, instead of raw logits, the softmax
 * numerators and partials kb_cdf_rows takes (stats float2 [B*T, vocab_pad/32]).
 * T = 1 is the stepped decompress forward; the same kernels run for every T,
 * which makes packed and stepped results bit-identical.  Replaces
 * forward_packed_window / forward_stepped_batched
 * (krunch/cpp_path.py:131-163,428-460) and rwkv4_layer_step_cpp
 * (layer_cpp.cpp:456-637). */
int kb_forward_window(const kb_model* model, const int32_t* tokens, int B, int T,
                      float* state, void* workspace, size_t workspace_bytes,
                      uint16_t* logits, float* logit_stats, void* stream);

/* One layer of the model on a window: x fp16 [B*T, C] (rows b*T + t, 16-byte
 * aligned) is read and replaced by the layer's output; layer_state is that
 * layer's fp32 [5][B][C] slice of the state above (advanced in place);
 * workspace as for kb_forward_window.  kb_forward_window is embed, this for
 * every layer, then LayerNorm + head, so a chain of kb_layer_forward calls
 * gives the same bits.  Replaces rwkv4_layer_step_cpp and
 * rwkv4_layer_step_cpp_t1 (krunch_ac/cuda/layer_cpp.cpp:294-307,456-637). */
int kb_layer_forward(const kb_model* model, int layer, uint16_t* x, int B, int T,
                     float* layer_state, void* workspace, size_t workspace_bytes, void* stream);

/* Fused stepped decode forward (T = 1) of a KB_I8 model: the whole layer
 * stack in one persistent cooperative launch (one CTA per SM, grid barriers
 * between phases, tcgen05 kind::i8 GEMM tiles with int8 weights staged
 * through shared memory by TMA), then the head GEMM.  Same contract and the
 * same bits as kb_forward_window(model, tokens, B, 1, ...): logits (or
 * numerators + stats) and the state it advances.  Replaces the reference's
 * fused single-token layers (krunch_ac/cuda/rwkv_step_v3.cu:83-480) and the
 * launch chain of forward_stepped_batched (krunch/cpp_path.py:428-460).
 * The workspace (kb_step_workspace_bytes) must stay the same buffer across
 * calls to reuse the cached launch parameters; n_layer <= 24,
 * n_embd in {128, 768, 2048}.  KB_ERR_UNSUPPORTED for fp16 models. */
size_t kb_step_workspace_bytes(const kb_model* model, int B);
int kb_step_forward(kb_model* model, const int32_t* tokens, int B, float* state,
                    void* workspace, size_t workspace_bytes, uint16_t* logits,
                    float* logit_stats, void* stream);
/* Profiling aid: a device buffer of >= 2048 u64 receives, for CTA 0 of each
 * later kb_step_forward, %globaltimer at every grid barrier's entry (slot
 * 2e) and exit (slot 2e+1), per tile phase tp the SM clocks when its first
 * unit's loads were issued, landed, multiplied and stored (slots
 * 512 + 4 tp ..), the SM clock at each barrier exit (768 + e), and per row
 * phase rp the SM clocks of row 0 at entry, data consumed, row reduction
 * done and end (1024 + 4 rp ..);
 * NULL turns it off. */
int kb_step_set_trace(unsigned long long* trace);
/* Failure-detection test hook of the fused step: withhold != 0 makes CTA 0
 * skip its arrival at the first grid barrier of later calls, so every CTA's
 * bounded wait (spin_ns; 0 = the default 2 s) expires and the launch unwinds
 * with KB_ERR_TIMEOUT in kb_step_error_status; no GPU fault is involved.
 * (0, 0) restores normal operation. */
int kb_step_set_fault(int withhold, long long spin_ns);
/* Device-side failure report of the fused step (bounded mbarrier and grid
 * barrier waits): KB_OK or KB_ERR_TIMEOUT; reset != 0 clears it. */
int kb_step_error_status(int reset);

/* Allocation-free variant of kb_forward_window.  No counterpart in the
 * reference: it exists for hosts that cannot allocate device memory when they
 * run a forward, e.g. a foreign-language host (Go/JNI/Rust over this ABI)
 * whose process runs under a fixed device-memory budget handed out at
 * start-up, or a caller without a CUDA allocator of its own.  The caller
 * still passes tokens, state and logits; the activation workspace lives in a
 * file-scope __device__ array of KB_NOALLOC_SCRATCH_BYTES that every GPU
 * loading this library keeps until process exit.
 *   - The first call on a device resolves that array's device address (with
 *     the device current), so make it before any stream capture begins.
 *   - Windows whose workspace (kb_forward_workspace_bytes) exceeds the array
 *     return KB_ERR_TOO_LARGE.  At RWKV-4-169M the 8 MiB hold one stream of
 *     up to 389 tokens or up to 303 streams of one token with fp16 / bf16
 *     weights, and 302 tokens or 248 streams with int8 weights; ask
 *     kb_forward_workspace_bytes for other shapes.
 *   - All calls share the one array and it keeps the previous call's
 *     contents; nothing in it needs to start at zero.  Calls that can overlap
 *     on the GPU (other streams, other host threads) race on it: serialise
 *     them on one stream.
 * Makes no cudaMalloc / cudaFree or allocating library call. */
#define KB_NOALLOC_SCRATCH_BYTES ((size_t)8 << 20)
int kb_forward_window_noalloc(const kb_model* model, const int32_t* tokens, int B, int T,
                              float* state, uint16_t* logits, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* KRUNCH_B200_H */
