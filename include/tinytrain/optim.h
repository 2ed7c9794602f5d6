#pragma once

// Gradient-based optimizers (same API as the reference's optim.h,
// optim.h:14-42 of seampm/tinytrain). They update parameters in place on the
// device; AdamW runs as one fused multi-tensor kernel.

#include <cstdint>
#include <vector>

#include "tinytrain/tensor.h"

namespace tt {

// AdamW: Adam with decoupled weight decay (the modern default).
class AdamW {
public:
    AdamW(const std::vector<Tensor*>& params, float lr, float beta1 = 0.9f,
          float beta2 = 0.999f, float eps = 1e-8f, float weight_decay = 0.0f);
    ~AdamW();
    void step();
    void zero_grad();
    void set_lr(float lr) { lr_ = lr; }

    // ---- extensions (not in the reference) ----
    // Global-norm gradient clipping folded into step(): gradients are scaled
    // by max_norm / (||g|| + 1e-6) when that is < 1. 0 disables it.
    void set_clip_norm(float max_norm) { clip_ = max_norm; }
    // Multiplier applied to every gradient inside step() (e.g. 1/world after
    // an all-reduce sum); the clip norm is measured after it.
    void set_grad_scale(float s) { grad_scale_ = s; }
    // Norm measured by the last step() with clipping on (reads the device).
    float last_grad_norm() const;
    // The same without a host read: the device sum of squares behind it
    // (null before the first clipped step) and the scale it is taken at;
    // norm = sqrt(sum) * scale.
    const double* grad_sumsq_device() const { return sumsq_; }
    float grad_scale() const { return grad_scale_; }
    int64_t step_count() const { return step_; }
    // Optimizer state for checkpoints: first (which = 0) or second (1) moment
    // of parameter i on the device, allocated zeroed if it does not exist yet;
    // and the step counter behind the bias correction.
    float* moment(size_t i, int which);
    void set_step_count(int64_t t) { step_ = t; }
    // Learning rate and bias-corrected rate read from the device ({lr,
    // lr_t} at `sched`, written by ttk_adamw_sched_set) instead of passed
    // with the launch: for a step recorded in a CUDA graph and replayed.
    // nullptr returns to the host values.
    void set_device_schedule(const float* sched) { sched_ = sched; }

private:
    std::vector<Tensor*> params_;
    float lr_, beta1_, beta2_, eps_, weight_decay_;
    float clip_ = 0.0f, grad_scale_ = 1.0f;
    int64_t step_ = 0;
    // per-parameter state, allocated lazily on the device, keyed by index
    std::vector<float*> m_, v_;
    double* sumsq_ = nullptr;
    const float* sched_ = nullptr;
};

// SGD with optional momentum and weight decay.
class SGD {
public:
    SGD(const std::vector<Tensor*>& params, float lr, float momentum = 0.0f,
        float weight_decay = 0.0f);
    ~SGD();
    void step();
    void zero_grad();

private:
    std::vector<Tensor*> params_;
    float lr_, momentum_, weight_decay_;
    std::vector<float*> vel_;
};

} // namespace tt
