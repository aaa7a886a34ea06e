// Public GEMM entry point (kb_gemm) and the device error report; the kernel
// itself is the tcgen05 GEMM in gemm_tc.cu.
#include "profile.cuh"
#include "rwkv_ops.cuh"

namespace kb {

}  // namespace kb

extern "C" int kb_gemm_tiled(int dtype, const void* A, int64_t lda, const void* W, int64_t ldw,
                             int M, int N, int K, int epilogue, void* out, int64_t ldo,
                             const uint16_t* resid, const uint16_t* gate, int tile_n,
                             void* stream) {
    using namespace kb;
    if (!A || !W || !out || M < 0 || N <= 0 || K <= 0) return KB_ERR_ARG;
    if (epilogue < KB_EPI_F32 || epilogue > KB_EPI_GATE_RESID) return KB_ERR_ARG;
    if (tile_n != 0 && tile_n != 32 && tile_n != 64 && tile_n != 128 && tile_n != 256 &&
        tile_n != KB_TILE_PAIR)
        return KB_ERR_ARG;
    if (dtype != KB_F16 && dtype != KB_BF16) return KB_ERR_UNSUPPORTED;
    if (N % 32 || K % 64) return KB_ERR_SHAPE;
    if ((epilogue == KB_EPI_RESID || epilogue == KB_EPI_GATE_RESID) && !resid) return KB_ERR_ARG;
    if (epilogue == KB_EPI_GATE_RESID && !gate) return KB_ERR_ARG;
    if (!aligned16(A) || !aligned16(W) || (lda % 8) || (ldw % 8) || lda < K || ldw < K ||
        ldo < N || (ldo % 8) || !aligned16(out))
        return KB_ERR_ALIGN;
    ProfScope ps(PH_GEMM, as_stream(stream), 2.0 * M * (double)N * K);
    if (dtype == KB_BF16)
        return launch_gemm_bf16(reinterpret_cast<const uint16_t*>(A), lda,
                                reinterpret_cast<const uint16_t*>(W), ldw, M, N, K, epilogue, out,
                                ldo, resid, gate, as_stream(stream), tile_n);
    return launch_gemm_tc(reinterpret_cast<const uint16_t*>(A), lda,
                          reinterpret_cast<const uint16_t*>(W), ldw, M, N, K, epilogue, out, ldo,
                          resid, gate, as_stream(stream), tile_n);
}

extern "C" int kb_gemm(int dtype, const void* A, int64_t lda, const void* W, int64_t ldw, int M,
                       int N, int K, int epilogue, void* out, int64_t ldo, const uint16_t* resid,
                       const uint16_t* gate, void* stream) {
    return kb_gemm_tiled(dtype, A, lda, W, ldw, M, N, K, epilogue, out, ldo, resid, gate, 0,
                         stream);
}

extern "C" int kb_gemm_i8(const int8_t* A, int64_t lda, const float* a_scale, const int8_t* W,
                          int64_t ldw, const uint16_t* w_scale, int M, int N, int K, int epilogue,
                          void* out, int64_t ldo, const uint16_t* resid, const uint16_t* gate,
                          int tile_n, void* stream) {
    using namespace kb;
    if (!A || !W || !out || !a_scale || !w_scale || M < 0 || N <= 0 || K <= 0) return KB_ERR_ARG;
    if (tile_n != 0 && tile_n != 32 && tile_n != 64 && tile_n != 128 && tile_n != 256 &&
        tile_n != KB_TILE_PAIR)
        return KB_ERR_ARG;
    if (epilogue < KB_EPI_F32 || epilogue > KB_EPI_GATE_RESID) return KB_ERR_ARG;
    if (N % 32 || K % 128) return KB_ERR_SHAPE;
    if ((epilogue == KB_EPI_RESID || epilogue == KB_EPI_GATE_RESID) && !resid) return KB_ERR_ARG;
    if (epilogue == KB_EPI_GATE_RESID && !gate) return KB_ERR_ARG;
    if (!aligned16(A) || !aligned16(W) || !aligned16(w_scale) || (lda % 16) || (ldw % 16) ||
        lda < K || ldw < K || ldo < N || (ldo % 8) || !aligned16(out))
        return KB_ERR_ALIGN;
    ProfScope ps(PH_GEMM, as_stream(stream), 2.0 * M * (double)N * K);
    return launch_gemm_i8(A, lda, a_scale, W, ldw, w_scale, M, N, K, epilogue, out, ldo, resid,
                          gate, as_stream(stream), tile_n);
}

extern "C" int kb_gemm_kvr(int dtype, const void* kx, const void* vx, const void* rx, int64_t lda,
                           const float* kx_scale, const float* vx_scale, const float* rx_scale,
                           const void* kw, const void* vw, const void* rw, int64_t ldw,
                           const uint16_t* kw_scale, const uint16_t* vw_scale,
                           const uint16_t* rw_scale, int M, int N, int K, float* k, float* v,
                           uint16_t* r, int64_t ldo, int tile_n, void* stream) {
    using namespace kb;
    if (!kx || !vx || !rx || !kw || !vw || !rw || !k || !v || !r || M < 0 || N <= 0 || K <= 0)
        return KB_ERR_ARG;
    if (tile_n != 0 && tile_n != 32 && tile_n != 64 && tile_n != 128 && tile_n != 256 &&
        tile_n != KB_TILE_PAIR)
        return KB_ERR_ARG;
    if (dtype != KB_F16 && dtype != KB_BF16 && dtype != KB_I8) return KB_ERR_UNSUPPORTED;
    const bool i8 = dtype == KB_I8;
    if (i8 && (!kx_scale || !vx_scale || !rx_scale || !kw_scale || !vw_scale || !rw_scale))
        return KB_ERR_ARG;
    if (N % 32 || K % (i8 ? 128 : 64)) return KB_ERR_SHAPE;
    const int el = i8 ? 16 : 8;  // elements per 16 bytes of A / W
    const void* ptrs[9] = {kx, vx, rx, kw, vw, rw, k, v, r};
    for (const void* q : ptrs)
        if (!aligned16(q)) return KB_ERR_ALIGN;
    if (i8 && (!aligned16(kw_scale) || !aligned16(vw_scale) || !aligned16(rw_scale)))
        return KB_ERR_ALIGN;
    if ((lda % el) || (ldw % el) || lda < K || ldw < K || ldo < N || (ldo % 8)) return KB_ERR_ALIGN;
    const void* const A[3] = {kx, vx, rx};
    const void* const W[3] = {kw, vw, rw};
    const float* const as[3] = {kx_scale, vx_scale, rx_scale};
    const uint16_t* const ws[3] = {kw_scale, vw_scale, rw_scale};
    void* const out[3] = {k, v, r};
    ProfScope ps(PH_GEMM, as_stream(stream), 3.0 * 2.0 * M * (double)N * K);
    return launch_gemm_kvr(dtype, A, lda, as, W, ldw, ws, M, N, K, out, ldo, as_stream(stream),
                           tile_n);
}

extern "C" int kb_device_error_status(int reset) {
    const int e = kb::read_tc_error(reset);
    const int f = kb::read_ln_error(reset);
    if (e < 0 || f < 0) return KB_ERR_CUDA;
    return (e || f) ? KB_ERR_TIMEOUT : KB_OK;
}
