// RWKV-4 window forward: the orchestration that replaces cpp_path.py's
// forward_packed_window / forward_stepped_batched and layer_cpp.cpp's
// rwkv4_layer_step_cpp.  One code path for every window length T: T = 1 is
// the stepped decoder, T > 1 the packed encoder.
#include <mutex>
#include <new>
#include <vector>

#include "model_impl.h"
#include "profile.cuh"
#include "rwkv_ops.cuh"

namespace kb {

static thread_local int g_last_cuda_error = 0;
void set_cuda_error(cudaError_t e) { g_last_cuda_error = (int)e; }

// ---- phase profiler (single host thread) ----------------------------------
namespace {
struct ProfRec {
    int phase;
    cudaEvent_t a, b;
    double work;
};
struct Prof {
    bool on = false;
    std::vector<cudaEvent_t> pool;
    size_t used = 0;
    std::vector<ProfRec> recs;
};
Prof g_prof;
}  // namespace

bool prof_on() { return g_prof.on; }
cudaEvent_t prof_event() {
    if (g_prof.used == g_prof.pool.size()) {
        cudaEvent_t e;
        if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
        g_prof.pool.push_back(e);
    }
    return g_prof.pool[g_prof.used++];
}
void prof_push(int phase, cudaEvent_t a, cudaEvent_t b, double work) {
    g_prof.recs.push_back({phase, a, b, work});
}

}  // namespace kb


using namespace kb;

extern "C" int kb_profile_begin(void) {
    g_prof.on = true;
    g_prof.used = 0;
    g_prof.recs.clear();
    return KB_OK;
}

extern "C" int kb_profile_end(double* ms, int64_t* launches, double* work, int n_phases) {
    g_prof.on = false;
    if (n_phases < 0 || ((!ms || !launches || !work) && n_phases > 0)) return KB_ERR_ARG;
    for (int i = 0; i < n_phases; ++i) {
        ms[i] = 0.0;
        launches[i] = 0;
        work[i] = 0.0;
    }
    for (const ProfRec& r : g_prof.recs) {
        if (cudaEventSynchronize(r.b) != cudaSuccess) return launch_status();
        float t = 0.f;
        if (cudaEventElapsedTime(&t, r.a, r.b) != cudaSuccess) return launch_status();
        if (r.phase < n_phases) {
            ms[r.phase] += t;
            launches[r.phase] += 1;
            work[r.phase] += r.work;
        }
    }
    g_prof.recs.clear();
    g_prof.used = 0;
    return KB_OK;
}

extern "C" const char* kb_version(void) { return "krunch_b200 0.1.0 (sm_100a)"; }

extern "C" int kb_last_cuda_error(void) { return g_last_cuda_error; }

extern "C" const char* kb_status_string(int s) {
    switch (s) {
        case KB_OK: return "ok";
        case KB_ERR_ARG: return "invalid argument";
        case KB_ERR_SHAPE: return "unsupported shape";
        case KB_ERR_ALIGN: return "misaligned pointer or stride";
        case KB_ERR_CUDA: return "CUDA error";
        case KB_ERR_TIMEOUT: return "device wait timed out";
        case KB_ERR_UNSUPPORTED: return "unsupported on this build";
        case KB_ERR_WORKSPACE: return "workspace too small";
        case KB_ERR_NOMEM: return "host allocation failed";
        case KB_ERR_TOO_LARGE: return "request exceeds the fixed no-alloc scratch";
        default: return "unknown status";
    }
}

static bool al16(const void* p) { return p && aligned16(p); }

extern "C" int kb_model_create(const kb_model_desc* d, kb_model** out) {
    if (!d || !out) return KB_ERR_ARG;
    *out = nullptr;
    const int C = d->n_embd, F = d->n_ffn;
    if (d->n_layer < 1 || C < 128 || F < 128 || d->n_vocab < 2) return KB_ERR_ARG;
    if (C % 128 || F % 128 || C > 4096) return KB_ERR_SHAPE;
    if (d->vocab_pad < d->n_vocab || d->vocab_pad % 128 || d->n_vocab > 65536) return KB_ERR_SHAPE;
    if (d->wdtype != KB_F16 && d->wdtype != KB_I8 && d->wdtype != KB_BF16) return KB_ERR_UNSUPPORTED;
    const bool i8 = d->wdtype == KB_I8;
    if (i8 && !al16(d->head_scale)) return KB_ERR_ALIGN;
    if (d->wkv_convention != KB_WKV_STEP_REF && d->wkv_convention != KB_WKV_PRODUCTION)
        return KB_ERR_ARG;
    if (!al16(d->emb) || !d->ln_out_w || !d->ln_out_b || !al16(d->head) || !d->layers)
        return KB_ERR_ARG;
    for (int l = 0; l < d->n_layer; ++l) {
        const kb_layer_desc& L = d->layers[l];
        if (!L.ln1_w || !L.ln1_b || !L.ln2_w || !L.ln2_b || !L.att_mix_k || !L.att_mix_v ||
            !L.att_mix_r || !L.att_decay || !L.att_first || !L.ffn_mix_k || !L.ffn_mix_r)
            return KB_ERR_ARG;
        if (!al16(L.att_kw) || !al16(L.att_vw) || !al16(L.att_rw) || !al16(L.att_ow) ||
            !al16(L.ffn_kw) || !al16(L.ffn_vw) || !al16(L.ffn_rw))
            return KB_ERR_ALIGN;
        if (i8 && (!al16(L.att_ks) || !al16(L.att_vs) || !al16(L.att_rs) || !al16(L.att_os) ||
                   !al16(L.ffn_ks) || !al16(L.ffn_vs) || !al16(L.ffn_rs)))
            return KB_ERR_ALIGN;
    }
    kb_model* m = new (std::nothrow) kb_model;
    if (!m) return KB_ERR_NOMEM;
    m->d = *d;
    m->layers.assign(d->layers, d->layers + d->n_layer);
    m->d.layers = m->layers.data();
    *out = m;
    return KB_OK;
}

extern "C" void kb_model_destroy(kb_model* m) { delete m; }

extern "C" int kb_state_init(const kb_model* m, float* state, int B, void* stream) {
    if (!m || !state || B < 0) return KB_ERR_ARG;
    return launch_state_init(state, m->d.n_layer, B, m->d.n_embd, as_stream(stream));
}

namespace {

struct Workspace {
    uint16_t *x, *kx, *vx, *rx, *r, *ry, *kk;
    float *k, *v, *xx_att, *xx_ffn;
    // w8a8 operands (KB_I8 models only): int8 rows and per-row factors
    int8_t *q_kx, *q_vx, *q_rx, *q_ry, *q_kk;
    float *s_kx, *s_vx, *s_rx, *s_ry, *s_kk;
};

inline size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }

size_t layout(const kb_model_desc& d, int B, int T, char* base, Workspace* w) {
    const size_t R = (size_t)B * T, C = d.n_embd, F = d.n_ffn;
    size_t off = 0;
    auto take = [&](size_t bytes) -> char* {
        char* p = base ? base + off : nullptr;
        off += al256(bytes);
        return p;
    };
    Workspace t;
    t.x = (uint16_t*)take(R * C * 2);
    t.kx = (uint16_t*)take(R * C * 2);
    t.vx = (uint16_t*)take(R * C * 2);
    t.rx = (uint16_t*)take(R * C * 2);
    t.r = (uint16_t*)take(R * C * 2);
    t.ry = (uint16_t*)take(R * C * 2);
    t.kk = (uint16_t*)take(R * F * 2);
    t.k = (float*)take(R * C * 4);
    t.v = (float*)take(R * C * 4);
    t.xx_att = (float*)take((size_t)B * C * 4);
    t.xx_ffn = (float*)take((size_t)B * C * 4);
    if (d.wdtype == KB_I8) {
        t.q_kx = (int8_t*)take(R * C);
        t.q_vx = (int8_t*)take(R * C);
        t.q_rx = (int8_t*)take(R * C);
        t.q_ry = (int8_t*)take(R * C);
        t.q_kk = (int8_t*)take(R * F);
        t.s_kx = (float*)take(R * 4);
        t.s_vx = (float*)take(R * 4);
        t.s_rx = (float*)take(R * 4);
        t.s_ry = (float*)take(R * 4);
        t.s_kk = (float*)take(R * 4);
    } else {
        t.q_kx = t.q_vx = t.q_rx = t.q_ry = t.q_kk = nullptr;
        t.s_kx = t.s_vx = t.s_rx = t.s_ry = t.s_kk = nullptr;
    }
    if (w) *w = t;
    return off;
}

#define KB_TRY(expr)                 \
    do {                             \
        const int _s = (expr);       \
        if (_s != KB_OK) return _s;  \
    } while (0)

}  // namespace

namespace {

// One RWKV-4 layer over a window of B x T rows, residual stream in w.x
// (fp16 [B*T, C], read and updated), layer state s fp32 [5][B][C].  The
// body of the reference's rwkv4_layer_step_cpp (layer_cpp.cpp:456-637).
int run_layer(const kb_model_desc& d, const kb_layer_desc& L, const Workspace& w, int B, int T,
              float* s, cudaStream_t st) {
    const int C = d.n_embd, F = d.n_ffn;
    const int R = B * T;
    const size_t BC = (size_t)B * C;
    const bool i8 = d.wdtype == KB_I8;
    const bool bf = d.wdtype == KB_BF16;  // GEMM operands (mix outputs, r*y, relu^2) in bf16
    const double bpe = 2.0;  // fp16 bytes per activation element
    auto gemm = [&](const uint16_t* A, const void* W, int M, int Nn, int K, int epi, void* out,
                    const uint16_t* resid, const uint16_t* gate, int phase) -> int {
        ProfScope ps(phase, st, 2.0 * M * (double)Nn * K);
        if (bf)
            return launch_gemm_bf16(A, K, (const uint16_t*)W, K, M, Nn, K, epi, out, Nn, resid,
                                    gate, st);
        return launch_gemm_tc(A, K, (const uint16_t*)W, K, M, Nn, K, epi, out, Nn, resid, gate, st);
    };
    auto gemm8 = [&](const int8_t* A, const float* sa, const void* W, const uint16_t* sw, int M,
                     int Nn, int K, int epi, void* out, const uint16_t* resid,
                     const uint16_t* gate, int phase) -> int {
        ProfScope ps(phase, st, 2.0 * M * (double)Nn * K);
        return launch_gemm_i8(A, K, sa, (const int8_t*)W, K, sw, M, Nn, K, epi, out, Nn, resid,
                              gate, st);
    };
    auto quant = [&](const uint16_t* x, int K, int8_t* q, float* qs) -> int {
        ProfScope ps(PH_LN_MIX, st, (double)R * K * 3.0);
        return launch_quant_rows(x, R, K, q, qs, st);
    };
    float *s_att = s, *s_aa = s + BC, *s_bb = s + 2 * BC, *s_pp = s + 3 * BC,
          *s_ffn = s + 4 * BC;

    // ---- time mix -------------------------------------------------------
    MixArgs ma{{L.att_mix_k, L.att_mix_v, L.att_mix_r}, {w.kx, w.vx, w.rx},
               {w.q_kx, w.q_vx, w.q_rx}, {w.s_kx, w.s_vx, w.s_rx}, bf ? 1 : 0};
    {
        ProfScope ps(PH_LN_MIX, st, (double)R * C * (i8 ? 2 * bpe + 3 : 4 * bpe));
        KB_TRY(launch_ln_mix(3, w.x, B, T, C, L.ln1_w, L.ln1_b, ma, s_att, w.xx_att, nullptr, st));
    }
    {
        // k, v, r projections in one launch (the reference's 3-way kernel)
        ProfScope ps(PH_GEMM, st, 3.0 * 2.0 * R * (double)C * C);
        const void* const A[3] = {i8 ? (const void*)w.q_kx : w.kx, i8 ? (const void*)w.q_vx : w.vx,
                                  i8 ? (const void*)w.q_rx : w.rx};
        const float* const as[3] = {w.s_kx, w.s_vx, w.s_rx};
        const void* const W[3] = {L.att_kw, L.att_vw, L.att_rw};
        const uint16_t* const ws[3] = {L.att_ks, L.att_vs, L.att_rs};
        void* const out[3] = {w.k, w.v, w.r};
        KB_TRY(launch_gemm_kvr(d.wdtype, A, C, as, W, C, ws, R, C, C, out, C, st));
    }
    {
        ProfScope ps(PH_WKV, st, (double)R * C * 12.0);
        KB_TRY(launch_wkv(d.wkv_convention, B, T, C, w.k, w.v, w.r, L.att_decay, L.att_first,
                          s_aa, s_bb, s_pp, w.ry, st, bf));
    }
    if (i8) {
        KB_TRY(quant(w.ry, C, w.q_ry, w.s_ry));
        KB_TRY(gemm8(w.q_ry, w.s_ry, L.att_ow, L.att_os, R, C, C, KB_EPI_RESID, w.x, w.x, nullptr, PH_GEMM));
    } else {
        KB_TRY(gemm(w.ry, L.att_ow, R, C, C, KB_EPI_RESID, w.x, w.x, nullptr, PH_GEMM));
    }
    if (cudaMemcpyAsync(s_att, w.xx_att, BC * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return launch_status();

    // ---- channel mix ----------------------------------------------------
    MixArgs mf{{L.ffn_mix_k, L.ffn_mix_r, nullptr}, {w.kx, w.rx, nullptr},
               {w.q_kx, w.q_rx, nullptr}, {w.s_kx, w.s_rx, nullptr}, bf ? 1 : 0};
    {
        ProfScope ps(PH_LN_MIX, st, (double)R * C * (i8 ? bpe + 2 : 3 * bpe));
        KB_TRY(launch_ln_mix(2, w.x, B, T, C, L.ln2_w, L.ln2_b, mf, s_ffn, w.xx_ffn, nullptr, st));
    }
    if (i8) {
        KB_TRY(gemm8(w.q_rx, w.s_rx, L.ffn_rw, L.ffn_rs, R, C, C, KB_EPI_SIGMOID, w.r, nullptr, nullptr, PH_GEMM));
        KB_TRY(gemm8(w.q_kx, w.s_kx, L.ffn_kw, L.ffn_ks, R, F, C, KB_EPI_RELU_SQ, w.kk, nullptr, nullptr, PH_GEMM));
        KB_TRY(quant(w.kk, F, w.q_kk, w.s_kk));
        KB_TRY(gemm8(w.q_kk, w.s_kk, L.ffn_vw, L.ffn_vs, R, C, F, KB_EPI_GATE_RESID, w.x, w.x, w.r, PH_GEMM));
    } else {
        KB_TRY(gemm(w.rx, L.ffn_rw, R, C, C, KB_EPI_SIGMOID, w.r, nullptr, nullptr, PH_GEMM));
        KB_TRY(gemm(w.kx, L.ffn_kw, R, F, C, KB_EPI_RELU_SQ, w.kk, nullptr, nullptr, PH_GEMM));
        KB_TRY(gemm(w.kk, L.ffn_vw, R, C, F, KB_EPI_GATE_RESID, w.x, w.x, w.r, PH_GEMM));
    }
    if (cudaMemcpyAsync(s_ffn, w.xx_ffn, BC * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return launch_status();
    return KB_OK;
}

}  // namespace

extern "C" size_t kb_forward_workspace_bytes(const kb_model* m, int B, int T) {
    if (!m || B <= 0 || T <= 0) return 0;
    return layout(m->d, B, T, nullptr, nullptr);
}

extern "C" int kb_forward_window(const kb_model* m, const int32_t* tokens, int B, int T,
                                 float* state, void* ws, size_t ws_bytes, uint16_t* logits,
                                 float* logit_stats, void* stream) {
    if (!m || !tokens || !state || !ws || !logits || B <= 0 || T <= 0) return KB_ERR_ARG;
    const kb_model_desc& d = m->d;
    if (ws_bytes < layout(d, B, T, nullptr, nullptr)) return KB_ERR_WORKSPACE;
    if (!aligned16(ws) || !aligned16(logits) || ((uintptr_t)logit_stats & 7u)) return KB_ERR_ALIGN;
    cudaStream_t st = as_stream(stream);
    Workspace w;
    layout(d, B, T, reinterpret_cast<char*>(ws), &w);
    const int C = d.n_embd;
    const int R = B * T;
    const size_t BC = (size_t)B * C;

    const bool i8 = d.wdtype == KB_I8;
    const bool bf = d.wdtype == KB_BF16;
    const double bpe = 2.0;  // fp16 bytes per activation element
    {
        ProfScope ps(PH_EMBED, st, (double)R * C * 2 * bpe);
        KB_TRY(launch_embed(tokens, R, d.n_vocab, C, d.emb, w.x, st));
    }
    for (int l = 0; l < d.n_layer; ++l)
        KB_TRY(run_layer(d, d.layers[l], w, B, T, state + (size_t)l * 5 * BC, st));
    MixArgs none{{nullptr, nullptr, nullptr}, {nullptr, nullptr, nullptr},
                 {w.q_kx, nullptr, nullptr}, {w.s_kx, nullptr, nullptr}, bf ? 1 : 0};
    {
        ProfScope ps(PH_LN_MIX, st, (double)R * C * (i8 ? bpe + 1 : 2 * bpe));
        KB_TRY(launch_ln_mix(0, w.x, B, T, C, d.ln_out_w, d.ln_out_b, none, nullptr, nullptr,
                             i8 ? nullptr : w.kx, st));
    }
    {
        ProfScope ps(PH_HEAD, st, 2.0 * R * (double)d.n_vocab * C);
        if (i8) {
            const int8_t* hw = (const int8_t*)d.head;
            if (logit_stats)
                KB_TRY(launch_gemm_logits_i8(w.q_kx, C, w.s_kx, hw, C, d.head_scale, R,
                                             d.vocab_pad, C, logits, d.vocab_pad, d.n_vocab,
                                             logit_stats, d.vocab_pad / 32, st));
            else
                KB_TRY(launch_gemm_i8(w.q_kx, C, w.s_kx, hw, C, d.head_scale, R, d.vocab_pad, C,
                                      KB_EPI_F16, logits, d.vocab_pad, nullptr, nullptr, st));
        } else if (bf) {
            if (logit_stats)
                KB_TRY(launch_gemm_logits_bf16(w.kx, C, (const uint16_t*)d.head, C, R, d.vocab_pad,
                                               C, logits, d.vocab_pad, d.n_vocab, logit_stats,
                                               d.vocab_pad / 32, st));
            else
                KB_TRY(launch_gemm_bf16(w.kx, C, (const uint16_t*)d.head, C, R, d.vocab_pad, C,
                                        KB_EPI_F16, logits, d.vocab_pad, nullptr, nullptr, st));
        } else if (logit_stats) {
            KB_TRY(launch_gemm_logits(w.kx, C, (const uint16_t*)d.head, C, R, d.vocab_pad, C,
                                      logits, d.vocab_pad, d.n_vocab, logit_stats,
                                      d.vocab_pad / 32, st));
        } else {
            KB_TRY(launch_gemm_tc(w.kx, C, (const uint16_t*)d.head, C, R, d.vocab_pad, C,
                                   KB_EPI_F16, logits, d.vocab_pad, nullptr, nullptr, st));
        }
    }
    return KB_OK;
}

extern "C" int kb_layer_forward(const kb_model* m, int layer, uint16_t* x, int B, int T,
                                float* layer_state, void* ws, size_t ws_bytes, void* stream) {
    if (!m || !x || !layer_state || !ws || B <= 0 || T <= 0) return KB_ERR_ARG;
    const kb_model_desc& d = m->d;
    if (layer < 0 || layer >= d.n_layer) return KB_ERR_ARG;
    if (ws_bytes < layout(d, B, T, nullptr, nullptr)) return KB_ERR_WORKSPACE;
    if (!aligned16(ws) || !aligned16(x)) return KB_ERR_ALIGN;
    Workspace w;
    layout(d, B, T, reinterpret_cast<char*>(ws), &w);
    w.x = x;  // the caller's residual rows are read and updated in place
    return run_layer(d, d.layers[layer], w, B, T, layer_state, as_stream(stream));
}

// ---------------------------------------------------------------------------
// kb_forward_window_noalloc: the same forward with its workspace in a fixed
// device array, for callers that cannot allocate device memory.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_noalloc_scratch[KB_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device, resolved once
// per device (host code must not use the symbol itself as a pointer).
int noalloc_scratch(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        set_cuda_error(e);
        return KB_ERR_CUDA;
    }
    if (dev < 0 || dev >= kMaxDevices) return KB_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            set_cuda_error(e);
            return KB_ERR_CUDA;
        }
        g_noalloc_addr[dev] = p;
    }
    *out = g_noalloc_addr[dev];
    return KB_OK;
}
}  // namespace

extern "C" int kb_forward_window_noalloc(const kb_model* m, const int32_t* tokens, int B, int T,
                                         float* state, uint16_t* logits, void* stream) {
    if (!m || !tokens || !state || !logits || B <= 0 || T <= 0) return KB_ERR_ARG;
    if (layout(m->d, B, T, nullptr, nullptr) > KB_NOALLOC_SCRATCH_BYTES) return KB_ERR_TOO_LARGE;
    void* ws = nullptr;
    const int rc = noalloc_scratch(&ws);
    if (rc != KB_OK) return rc;
    return kb_forward_window(m, tokens, B, T, state, ws, KB_NOALLOC_SCRATCH_BYTES, logits, nullptr,
                             stream);
}
