// Optimizers on device state (the reference's optim.cpp of seampm/tinytrain:
// AdamW optim.cpp:17-48, SGD optim.cpp:58-82). AdamW::step is one fused
// multi-tensor kernel (ttk_adamw_multi) preceded, when clipping is on, by one
// multi-tensor sum-of-squares kernel; moments are allocated lazily per
// parameter on its first step with a gradient, as in the reference.
#include <cmath>
#include <stdexcept>

#include "internal.h"
#include "tinytrain/optim.h"

namespace tt {

using namespace detail;

namespace {
float* zeroed(int64_t n) {
    void* p = nullptr;
    check(ttk_malloc(&p, static_cast<size_t>(n) * 4, stream()), "optimizer state");
    check(ttk_memset(p, 0, static_cast<size_t>(n) * 4, stream()), "optimizer state");
    return static_cast<float*>(p);
}

void mark_written(Tensor* p) {
    p->impl()->data->host_valid = false;
    ++p->impl()->data->version;
}
}  // namespace

AdamW::AdamW(const std::vector<Tensor*>& params, float lr, float beta1, float beta2, float eps,
             float weight_decay)
    : params_(params), lr_(lr), beta1_(beta1), beta2_(beta2), eps_(eps),
      weight_decay_(weight_decay), m_(params.size(), nullptr), v_(params.size(), nullptr) {}

AdamW::~AdamW() {
    void* s = stream_if_ready();
    for (float* p : m_)
        ttk_free(p, s);
    for (float* p : v_)
        ttk_free(p, s);
    ttk_free(sumsq_, s);
}

void AdamW::zero_grad() {
    for (Tensor* p : params_)
        p->zero_grad();
}

void AdamW::step() {
    ++step_;
    std::vector<float*> ps, ms, vs;
    std::vector<const float*> gs;
    std::vector<int64_t> ns;
    for (size_t i = 0; i < params_.size(); ++i) {
        Tensor* p = params_[i];
        if (!p->has_grad())
            continue;  // optim.cpp:28-29
        if (!m_[i]) {
            m_[i] = zeroed(p->numel());
            v_[i] = zeroed(p->numel());
        }
        ps.push_back(dwrite(p->impl()));
        gs.push_back(p->device_grad());
        ms.push_back(m_[i]);
        vs.push_back(v_[i]);
        ns.push_back(p->numel());
        mark_written(p);
    }
    if (ps.empty())
        return;
    const double* ss = nullptr;
    if (clip_ > 0.0f) {
        if (!sumsq_)
            check(ttk_malloc(reinterpret_cast<void**>(&sumsq_), 8, stream()), "sumsq");
        check(ttk_memset(sumsq_, 0, 8, stream()), "sumsq zero");
        check(ttk_sumsq_multi(gs.data(), ns.data(), static_cast<int>(gs.size()), sumsq_, stream()),
              "sumsq");
        ss = sumsq_;
    }
    if (sched_)
        check(ttk_adamw_multi_sched(ps.data(), gs.data(), ms.data(), vs.data(), ns.data(),
                                    static_cast<int>(ps.size()), beta1_, beta2_, eps_,
                                    weight_decay_, sched_, ss, clip_, grad_scale_, stream()),
              "adamw");
    else
        check(ttk_adamw_multi(ps.data(), gs.data(), ms.data(), vs.data(), ns.data(),
                              static_cast<int>(ps.size()), lr_, beta1_, beta2_, eps_,
                              weight_decay_, step_, ss, clip_, grad_scale_, stream()),
              "adamw");
}

float* AdamW::moment(size_t i, int which) {
    if (i >= params_.size())
        throw std::out_of_range("AdamW::moment: parameter index");
    if (!m_[i]) {
        m_[i] = zeroed(params_[i]->numel());
        v_[i] = zeroed(params_[i]->numel());
    }
    return which == 0 ? m_[i] : v_[i];
}

float AdamW::last_grad_norm() const {
    if (!sumsq_)
        return 0.0f;
    double ss = 0.0;
    check(ttk_memcpy_d2h(&ss, sumsq_, 8, stream()), "norm read");
    return static_cast<float>(std::sqrt(ss) * grad_scale_);
}

SGD::SGD(const std::vector<Tensor*>& params, float lr, float momentum, float weight_decay)
    : params_(params), lr_(lr), momentum_(momentum), weight_decay_(weight_decay),
      vel_(params.size(), nullptr) {}

SGD::~SGD() {
    void* s = stream_if_ready();
    for (float* p : vel_)
        ttk_free(p, s);
}

void SGD::zero_grad() {
    for (Tensor* p : params_)
        p->zero_grad();
}

void SGD::step() {
    for (size_t i = 0; i < params_.size(); ++i) {
        Tensor* p = params_[i];
        if (!p->has_grad())
            continue;
        if (momentum_ != 0.0f && !vel_[i])
            vel_[i] = zeroed(p->numel());
        float* d = dwrite(p->impl());
        check(ttk_sgd(d, p->device_grad(), vel_[i], p->numel(), lr_, momentum_, weight_decay_,
                      stream()),
              "sgd");
        mark_written(p);
    }
}

}  // namespace tt
