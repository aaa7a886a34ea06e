// fp16 GEMM with fused RWKV epilogues: out[M,N] = epi(A[M,K] @ W[N,K]^T).
//
// One tile schedule (128x128 CTA tile, K walked in 32-wide steps from 0 to
// K, fp32 accumulation) serves every M, so each output element is summed in
// the same order whatever M is: rows are bit-identical between the packed
// encoder (M = B*T) and the stepped decoder (M = B).  This is the M-invariance
// contract of the reference's det_matmul_tc kernels
// (krunch_ac/cuda/det_matmul_tc_async.cu:48-194).
//
// Tensor-core path: mma.sync m16n8k16, cp.async 4-stage pipeline, XOR-swizzled
// shared memory for conflict-free ldmatrix.
#include "rwkv_ops.cuh"

namespace kb {

constexpr int G_BM = 128, G_BN = 128, G_BK = 32, G_STAGES = 4, G_NT = 256;
constexpr int G_STAGE_HALVES = (G_BM + G_BN) * G_BK;
constexpr size_t G_SMEM = (size_t)G_STAGES * G_STAGE_HALVES * 2;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
    const int n = pred ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 16-byte chunk `ch` (0..3) of tile row `row`, swizzled.
__device__ __forceinline__ int sw_off(int row, int ch) {
    return row * G_BK + ((ch ^ ((row >> 1) & 3)) << 3);
}

// Epilogue on two adjacent columns (c, c+1) of row r.
template <int EPI>
__device__ __forceinline__ void epi_store(void* out, int64_t ldo, const uint16_t* resid,
                                          const uint16_t* gate, int64_t r, int c, float a0,
                                          float a1) {
    const int64_t o = r * ldo + c;
    if (EPI == KB_EPI_F32) {
        *reinterpret_cast<float2*>(reinterpret_cast<float*>(out) + o) = make_float2(a0, a1);
        return;
    }
    float y0 = a0, y1 = a1;
    if (EPI == KB_EPI_SIGMOID) {
        y0 = __fdiv_rn(1.0f, __fadd_rn(1.0f, __expf(-a0)));
        y1 = __fdiv_rn(1.0f, __fadd_rn(1.0f, __expf(-a1)));
    } else if (EPI == KB_EPI_RELU_SQ) {
        y0 = fmaxf(a0, 0.0f);
        y1 = fmaxf(a1, 0.0f);
        y0 = __fmul_rn(y0, y0);
        y1 = __fmul_rn(y1, y1);
    } else if (EPI == KB_EPI_RESID || EPI == KB_EPI_GATE_RESID) {
        const __half2 rr = *reinterpret_cast<const __half2*>(resid + o);
        float g0 = 1.0f, g1 = 1.0f;
        if (EPI == KB_EPI_GATE_RESID) {
            const __half2 gg = *reinterpret_cast<const __half2*>(gate + o);
            g0 = __low2float(gg);
            g1 = __high2float(gg);
        }
        y0 = __fmaf_rn(g0, a0, __low2float(rr));
        y1 = __fmaf_rn(g1, a1, __high2float(rr));
    }
    *reinterpret_cast<__half2*>(reinterpret_cast<uint16_t*>(out) + o) = __floats2half2_rn(y0, y1);
}

template <int EPI>
__global__ void __launch_bounds__(G_NT) k_gemm_f16(const uint16_t* __restrict__ A, int64_t lda,
                                                   const uint16_t* __restrict__ W, int64_t ldw,
                                                   int M, int N, int K, void* out, int64_t ldo,
                                                   const uint16_t* resid, const uint16_t* gate) {
    extern __shared__ __align__(128) uint16_t gsm[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int wm = warp >> 2, wn = warp & 3;  // 2 x 4 warps, 64 x 32 each
    const int m0 = blockIdx.y * G_BM, n0 = blockIdx.x * G_BN;
    const int KT = K / G_BK;

    auto load_stage = [&](int s, int kt) {
        uint16_t* sa = gsm + s * G_STAGE_HALVES;
        uint16_t* sb = sa + G_BM * G_BK;
        const int k0 = kt * G_BK;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int id = tid + j * G_NT;
            const int row = id >> 2, ch = id & 3;
            const int gm = m0 + row;
            const bool ok = gm < M;
            const uint16_t* src = A + (int64_t)(ok ? gm : 0) * lda + k0 + ch * 8;
            cp_async16(smem_u32(sa + sw_off(row, ch)), src, ok);
            const uint16_t* srcb = W + (int64_t)(n0 + row) * ldw + k0 + ch * 8;
            cp_async16(smem_u32(sb + sw_off(row, ch)), srcb, true);
        }
    };

    float acc[4][4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[i][j][q] = 0.0f;

#pragma unroll
    for (int s = 0; s < G_STAGES - 1; ++s) {
        if (s < KT) load_stage(s, s);
        cp_commit();
    }

    for (int kt = 0; kt < KT; ++kt) {
        cp_wait<G_STAGES - 2>();
        __syncthreads();
        const int nk = kt + G_STAGES - 1;
        if (nk < KT) load_stage(nk % G_STAGES, nk);
        cp_commit();

        const uint16_t* sa = gsm + (kt % G_STAGES) * G_STAGE_HALVES;
        const uint16_t* sb = sa + G_BM * G_BK;
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            uint32_t af[4][4];
#pragma unroll
            for (int mi = 0; mi < 4; ++mi) {
                const int row = wm * 64 + mi * 16 + (lane & 15);
                const int ch = kk * 2 + (lane >> 4);
                ldsm_x4(smem_u32(sa + sw_off(row, ch)), af[mi][0], af[mi][1], af[mi][2], af[mi][3]);
            }
            uint32_t bf[4][2];
#pragma unroll
            for (int nj = 0; nj < 2; ++nj) {
                const int row = wn * 32 + nj * 16 + (lane & 7) + ((lane >> 4) << 3);
                const int ch = kk * 2 + ((lane >> 3) & 1);
                uint32_t r0, r1, r2, r3;
                ldsm_x4(smem_u32(sb + sw_off(row, ch)), r0, r1, r2, r3);
                bf[nj * 2 + 0][0] = r0;
                bf[nj * 2 + 0][1] = r1;
                bf[nj * 2 + 1][0] = r2;
                bf[nj * 2 + 1][1] = r3;
            }
#pragma unroll
            for (int mi = 0; mi < 4; ++mi)
#pragma unroll
                for (int ni = 0; ni < 4; ++ni) mma16816(acc[mi][ni], af[mi], bf[ni][0], bf[ni][1]);
        }
    }
    cp_wait<0>();

#pragma unroll
    for (int mi = 0; mi < 4; ++mi) {
        const int r = m0 + wm * 64 + mi * 16 + (lane >> 2);
#pragma unroll
        for (int ni = 0; ni < 4; ++ni) {
            const int c = n0 + wn * 32 + ni * 8 + (lane & 3) * 2;
            if (r < M) epi_store<EPI>(out, ldo, resid, gate, r, c, acc[mi][ni][0], acc[mi][ni][1]);
            if (r + 8 < M)
                epi_store<EPI>(out, ldo, resid, gate, r + 8, c, acc[mi][ni][2], acc[mi][ni][3]);
        }
    }
}

template <int EPI>
static int launch_epi(const uint16_t* A, int64_t lda, const uint16_t* W, int64_t ldw, int M, int N,
                      int K, void* out, int64_t ldo, const uint16_t* resid, const uint16_t* gate,
                      cudaStream_t st) {
    static int configured = 0;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(k_gemm_f16<EPI>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)G_SMEM);
        if (e != cudaSuccess) {
            set_cuda_error(e);
            return KB_ERR_CUDA;
        }
        configured = 1;
    }
    dim3 grid(N / G_BN, (M + G_BM - 1) / G_BM);
    k_gemm_f16<EPI><<<grid, G_NT, G_SMEM, st>>>(A, lda, W, ldw, M, N, K, out, ldo, resid, gate);
    return launch_status();
}

int launch_gemm_f16(const uint16_t* A, int64_t lda, const uint16_t* W, int64_t ldw, int M, int N,
                    int K, int epi, void* out, int64_t ldo, const uint16_t* resid,
                    const uint16_t* gate, cudaStream_t st) {
    if (M == 0) return KB_OK;
    switch (epi) {
        case KB_EPI_F32: return launch_epi<KB_EPI_F32>(A, lda, W, ldw, M, N, K, out, ldo, resid, gate, st);
        case KB_EPI_F16: return launch_epi<KB_EPI_F16>(A, lda, W, ldw, M, N, K, out, ldo, resid, gate, st);
        case KB_EPI_SIGMOID: return launch_epi<KB_EPI_SIGMOID>(A, lda, W, ldw, M, N, K, out, ldo, resid, gate, st);
        case KB_EPI_RELU_SQ: return launch_epi<KB_EPI_RELU_SQ>(A, lda, W, ldw, M, N, K, out, ldo, resid, gate, st);
        case KB_EPI_RESID: return launch_epi<KB_EPI_RESID>(A, lda, W, ldw, M, N, K, out, ldo, resid, gate, st);
        case KB_EPI_GATE_RESID: return launch_epi<KB_EPI_GATE_RESID>(A, lda, W, ldw, M, N, K, out, ldo, resid, gate, st);
        default: return KB_ERR_ARG;
    }
}

}  // namespace kb

extern "C" int kb_gemm(int dtype, const void* A, int64_t lda, const void* W, int64_t ldw, int M,
                       int N, int K, int epilogue, void* out, int64_t ldo, const uint16_t* resid,
                       const uint16_t* gate, void* stream) {
    using namespace kb;
    if (!A || !W || !out || M < 0 || N <= 0 || K <= 0) return KB_ERR_ARG;
    if (dtype != KB_F16) return KB_ERR_UNSUPPORTED;
    if (N % G_BN || K % 64) return KB_ERR_SHAPE;
    if ((epilogue == KB_EPI_RESID || epilogue == KB_EPI_GATE_RESID) && !resid) return KB_ERR_ARG;
    if (epilogue == KB_EPI_GATE_RESID && !gate) return KB_ERR_ARG;
    if (!aligned16(A) || !aligned16(W) || (lda % 8) || (ldw % 8) || lda < K || ldw < K ||
        ldo < N || (ldo % 2))
        return KB_ERR_ALIGN;
    return launch_gemm_f16(reinterpret_cast<const uint16_t*>(A), lda,
                           reinterpret_cast<const uint16_t*>(W), ldw, M, N, K, epilogue, out, ldo,
                           resid, gate, as_stream(stream));
}
