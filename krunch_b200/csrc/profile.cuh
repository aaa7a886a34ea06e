// CUDA-event phase profiler (the counterpart of the reference's
// KRUNCH_PHASE_PROFILE timers, krunch_ac/cuda/layer_cpp.cpp:111-157).
// Off by default; when on, every launch of the library is bracketed by two
// events on its stream and tagged with a phase and its algorithmic work.
#pragma once
#include "kb_common.cuh"

namespace kb {

enum Phase { PH_EMBED = 0, PH_LN_MIX, PH_GEMM, PH_WKV, PH_HEAD, PH_CDF, PH_ENCODE, PH_DECODE, PH_STEP, PH_N };

bool prof_on();
void prof_push(int phase, cudaEvent_t a, cudaEvent_t b, double work);
cudaEvent_t prof_event();

struct ProfScope {
    int phase;
    double work;
    cudaStream_t st;
    cudaEvent_t a = nullptr;
    ProfScope(int p, cudaStream_t s, double w = 0.0) : phase(p), work(w), st(s) {
        if (prof_on()) {
            a = prof_event();
            if (a) cudaEventRecord(a, st);
        }
    }
    ~ProfScope() {
        if (a) {
            cudaEvent_t b = prof_event();
            if (b) {
                cudaEventRecord(b, st);
                prof_push(phase, a, b, work);
            }
        }
    }
};

}  // namespace kb
