// Host-side definition of the opaque kb_model handle, shared by the window
// forward (forward.cu) and the fused decode step (step_fused.cu).
#pragma once
#include <memory>
#include <mutex>
#include <vector>

#include "krunch_b200.h"

struct kb_model {
    kb_model_desc d;
    std::vector<kb_layer_desc> layers;
    // fused decode step: launch parameters (tensor maps) cached per
    // workspace; built on first use, type-erased here
    std::mutex step_mu;
    std::shared_ptr<void> step_cache;
};
