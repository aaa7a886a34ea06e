// Launchers of the RWKV-4 row-local / recurrent kernels (rwkv_ops.cu) and
// the GEMM family (gemm.cu), used by the forward orchestration (forward.cu).
#pragma once
#include <algorithm>

#include "kb_common.cuh"

namespace kb {

struct MixArgs {
    const float* mix[3];  // time-mix vectors [C]
    uint16_t* out[3];     // fp16 [rows, C] outputs
    int8_t* q[3];         // w8a8: int8 [rows, C] outputs instead (quant.cuh) ...
    float* qs[3];         // ... with their per-row dequantisation factors
    int bf16;             // out[] (and xx_out) in bf16 instead of fp16 (KB_BF16 model)
};

int launch_embed(const int32_t* tok, int64_t rows, int V, int C, const uint16_t* emb, uint16_t* x,
                 cudaStream_t st);
int launch_ln_mix(int nmix, const uint16_t* x, int B, int T, int C, const float* lw,
                  const float* lb, const MixArgs& ma, const float* state_in, float* state_out,
                  uint16_t* xx_out, cudaStream_t st);
// ry in fp16, or bf16 when ry_bf16 (the GEMM operand of a KB_BF16 model)
int launch_wkv(int conv, int B, int T, int C, const float* k, const float* v, const uint16_t* r,
               const float* decay, const float* first, float* aa, float* bb, float* pp,
               uint16_t* ry, cudaStream_t st, bool ry_bf16 = false);
int launch_state_init(float* st, int L, int B, int C, cudaStream_t s);

// out[M,N] = epi(A[M,K] @ W[N,K]^T); see kb_gemm in the public header.
// tile_n 0 = the widest tile width whose tiles fill the SMs.
int launch_gemm_tc(const uint16_t* A, int64_t lda, const uint16_t* W, int64_t ldw, int M, int N,
                   int K, int epi, void* out, int64_t ldo, const uint16_t* resid,
                   const uint16_t* gate, cudaStream_t st, int tile_n = 0);
// Head GEMM: per row and 32-column subtile u, out holds fp16 e^(x - m_u) of
// the fp16-rounded logits x (0 past column V) and stats[row * stats_stride + u]
// = (m_u, sum of those e), as defined in softmax_stats.cuh.
constexpr int KB_EPI_LOGITS_STATS = 6;
int launch_gemm_logits(const uint16_t* A, int64_t lda, const uint16_t* W, int64_t ldw, int M,
                       int N, int K, uint16_t* out, int64_t ldo, int V, float* stats,
                       int stats_stride, cudaStream_t st);
// w8a8: A int8 [M, K] with a fp32 dequantisation factor per row, W int8
// [N, K] with a fp16 factor per row of W (per output channel); exact int32
// accumulation, then y = (acc * a_scale[m]) * w_scale[n] and the epilogue.
// Requires K % 128 == 0.
int launch_gemm_i8(const int8_t* A, int64_t lda, const float* a_scale, const int8_t* W,
                   int64_t ldw, const uint16_t* w_scale, int M, int N, int K, int epi, void* out,
                   int64_t ldo, const uint16_t* resid, const uint16_t* gate, cudaStream_t st,
                   int tile_n = 0);
int launch_gemm_logits_i8(const int8_t* A, int64_t lda, const float* a_scale, const int8_t* W,
                          int64_t ldw, const uint16_t* w_scale, int M, int N, int K,
                          uint16_t* out, int64_t ldo, int V, float* stats, int stats_stride,
                          cudaStream_t st);
// bf16 A and W (KB_BF16 model); outputs fp16 except relu^2 (bf16: the next
// GEMM's operand) and fp32
int launch_gemm_bf16(const uint16_t* A, int64_t lda, const uint16_t* W, int64_t ldw, int M,
                     int N, int K, int epi, void* out, int64_t ldo, const uint16_t* resid,
                     const uint16_t* gate, cudaStream_t st, int tile_n = 0);
int launch_gemm_logits_bf16(const uint16_t* A, int64_t lda, const uint16_t* W, int64_t ldw,
                            int M, int N, int K, uint16_t* out, int64_t ldo, int V, float* stats,
                            int stats_stride, cudaStream_t st);
// The three attention projections of a layer in one launch: out[0] = fp32
// A[0] @ W[0]^T, out[1] = fp32 A[1] @ W[1]^T, out[2] = fp16 sigmoid(A[2] @
// W[2]^T); kind KB_F16 / KB_BF16 / KB_I8 (a_scale / w_scale used for KB_I8
// only).  Bit-identical to three single launches.
int launch_gemm_kvr(int kind, const void* const (&A)[3], int64_t lda,
                    const float* const (&a_scale)[3], const void* const (&W)[3], int64_t ldw,
                    const uint16_t* const (&w_scale)[3], int M, int N, int K,
                    void* const (&out)[3], int64_t ldo, cudaStream_t st, int tile_n = 0);
// Row-wise symmetric int8 quantisation of fp16 [R, K] (quant.cuh).
int launch_quant_rows(const uint16_t* x, int R, int K, int8_t* q, float* scale, cudaStream_t st);
// Device-side error code of the tcgen05 kernels (0 = none); optionally reset.
int read_tc_error(int reset);
// The same for the bulk-copy LayerNorm kernel's bounded waits.
int read_ln_error(int reset);

}  // namespace kb
