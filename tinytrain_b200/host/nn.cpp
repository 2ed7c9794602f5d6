// NN modules (the reference's nn.cpp of seampm/tinytrain: same initializers,
// so a given seed yields the same weights). Linear::forward calls the fused
// linear op, which reads W as a transposed GEMM operand instead of copying
// W^T as the reference's matmul(x, transpose(W)) does.
#include <cmath>
#include <vector>

#include "internal.h"
#include "nn_init.h"
#include "tinytrain/nn.h"
#include "tinytrain/ops.h"

namespace tt {

namespace {
thread_local bool t_skip_host_init = false;

// randn(seed) * scale computed on the host in float, like nn.cpp:16-20.
void init_scaled_normal(Tensor& w, uint64_t seed, float scale) {
    if (t_skip_host_init)
        return;
    std::vector<float> h(static_cast<size_t>(w.numel()));
    detail::host_randn(h.data(), w.numel(), seed);
    for (auto& x : h)
        x = x * scale;
    w.copy_from_host(h.data());
}
}  // namespace

namespace detail {
HostInitScope::HostInitScope(bool host_init) : prev(t_skip_host_init) {
    t_skip_host_init = !host_init;
}
HostInitScope::~HostInitScope() { t_skip_host_init = prev; }
}  // namespace detail

void Module::zero_grad() {
    for (Tensor* p : parameters())
        p->zero_grad();
}

Linear::Linear(int64_t in_features, int64_t out_features, uint64_t seed)
    : weight({out_features, in_features}, true) {
    // Xavier-style: Var(W) = 2 / (in + out)
    const float scale = std::sqrt(2.0f / static_cast<float>(in_features + out_features));
    init_scaled_normal(weight, seed, scale);
}

Tensor Linear::forward(const Tensor& x) { return linear(x, weight); }

Embedding::Embedding(int64_t vocab_size, int64_t dim, uint64_t seed)
    : weight({vocab_size, dim}, true) {
    const float scale = 1.0f / std::sqrt(static_cast<float>(dim));
    init_scaled_normal(weight, seed, scale);
}

Tensor Embedding::forward(const std::vector<int64_t>& idx) { return embedding(weight, idx); }

RMSNorm::RMSNorm(int64_t dim, float eps) : weight({dim}, 1.0f, true), eps(eps) {}

Tensor RMSNorm::forward(const Tensor& x) { return rmsnorm(x, weight, eps); }

}  // namespace tt
