// Deferred attention-score chain: semantics check on the device.
//
// Runs the reference's attention op chain (model.cpp:133-138) twice on the
// same inputs through this library's tt:: API:
//   A: untouched, so bmm(probs, v) runs the fused kernel; afterwards the
//      deferred probs are read, which computes them with the ordinary kernels;
//   B: the scores are read right after bmm(q, transpose(k)), which computes
//      them and breaks the chain, so every op runs eagerly.
// Checks: A fused one chain and B none; A's probs (computed on demand) equal
// B's bit for bit; outputs and q, k, v gradients agree within 1e-4
// (max |a - b| / max |b|). Prints "ok" and exits 0 on success.
#include <cmath>
#include <cstdio>
#include <vector>

#include "tinytrain/ops.h"
#include "tinytrain/tensor.h"

namespace {

double rel(const float* a, const float* b, int64_t n) {
    double num = 0, den = 1e-30;
    for (int64_t i = 0; i < n; ++i) {
        num = std::fmax(num, std::fabs(double(a[i]) - b[i]));
        den = std::fmax(den, std::fabs(double(b[i])));
    }
    return num / den;
}

struct Out {
    std::vector<float> att, probs, dq, dk, dv;
};

Out run(bool break_chain, int64_t N, int64_t T, int64_t hd) {
    tt::Tensor q = tt::randn({N, T, hd}, 1), k = tt::randn({N, T, hd}, 2),
               v = tt::randn({N, T, hd}, 3), G = tt::randn({N, T, hd}, 4);
    q.set_requires_grad(true);
    k.set_requires_grad(true);
    v.set_requires_grad(true);
    tt::Tensor mask = tt::full({T, T}, 0.0f);
    for (int64_t i = 0; i < T; ++i)
        for (int64_t j = i + 1; j < T; ++j)
            mask.data()[i * T + j] = -1e9f;
    const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
    tt::Tensor scores = tt::bmm(q, tt::transpose(k, 1, 2));
    if (break_chain)
        (void)static_cast<const tt::Tensor&>(scores).data();
    tt::Tensor s2 = tt::add(tt::mul(scores, tt::full(scores.shape(), scale)), mask);
    tt::Tensor probs = tt::softmax(s2, -1);
    tt::Tensor att = tt::bmm(probs, v);
    tt::Tensor loss = tt::sum_all(tt::mul(att, G));
    loss.backward();
    Out o;
    const tt::Tensor& ca = att;
    const tt::Tensor& cp = probs;
    o.att.assign(ca.data(), ca.data() + att.numel());
    o.probs.assign(cp.data(), cp.data() + probs.numel());
    o.dq.assign(q.grad_data(), q.grad_data() + q.numel());
    o.dk.assign(k.grad_data(), k.grad_data() + k.numel());
    o.dv.assign(v.grad_data(), v.grad_data() + v.numel());
    return o;
}

}  // namespace

int main() {
    try {
        const int64_t N = 6, T = 200, hd = 64;
        const int64_t f0 = tt::fused_attention_chains();
        Out a = run(false, N, T, hd);
        const int64_t f1 = tt::fused_attention_chains();
        Out b = run(true, N, T, hd);
        const int64_t f2 = tt::fused_attention_chains();
        int bad = 0;
        if (f1 - f0 != 1 || f2 - f1 != 0) {
            std::printf("fused chains: %lld then %lld (want 1, 0)\n", (long long)(f1 - f0),
                        (long long)(f2 - f1));
            ++bad;
        }
        if (a.probs != b.probs) {
            std::printf("probs computed on demand differ from the eager ones\n");
            ++bad;
        }
        const double e[4] = {rel(a.att.data(), b.att.data(), (int64_t)a.att.size()),
                             rel(a.dq.data(), b.dq.data(), (int64_t)a.dq.size()),
                             rel(a.dk.data(), b.dk.data(), (int64_t)a.dk.size()),
                             rel(a.dv.data(), b.dv.data(), (int64_t)a.dv.size())};
        for (double x : e)
            if (!(x <= 1e-4))
                ++bad;
        std::printf("att %.2e dq %.2e dk %.2e dv %.2e\n", e[0], e[1], e[2], e[3]);
        if (bad)
            return 1;
        std::printf("ok\n");
        return 0;
    } catch (const std::exception& ex) {
        std::printf("exception: %s\n", ex.what());
        return 2;
    }
}
