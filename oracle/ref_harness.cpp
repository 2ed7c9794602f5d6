// Oracle harness: a C ABI over the tinytrain reference's own CPU library.
//
// TEST INFRASTRUCTURE ONLY. This file is compiled together with the
// reference sources (src/tensor.cpp, src/ops.cpp, src/nn.cpp, src/optim.cpp,
// src/model.cpp of seampm/tinytrain) by oracle/Makefile into
// oracle/_ref/libttref.so. Tests, the smoke check and the CPU-baseline leg of
// bench.py load it through oracle/refbind.py to obtain the reference's own
// results on the same seeded inputs the CUDA path receives. Nothing in the
// product links or calls it.
//
// Every entry point builds reference tt::Tensors from caller buffers, runs the
// reference op (or op chain) forward, seeds the backward pass with an upstream
// gradient G through loss = sum_all(mul(y, G)) (whose backward hands exactly G
// to y: ops.cpp:253-255 bwd_mul gives g*G with g = 1), and copies outputs and
// input gradients back. All return 0 on success, 1 on a reference exception
// (message retrievable through ref_last_error).

#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "tinytrain/model.h"
#include "tinytrain/nn.h"
#include "tinytrain/ops.h"
#include "tinytrain/optim.h"
#include "tinytrain/tensor.h"

namespace {

std::string g_err;

tt::Tensor from_buf(const std::vector<int64_t>& shape, const float* src, bool rg) {
    tt::Tensor t(shape, rg);
    std::memcpy(t.data(), src, sizeof(float) * static_cast<size_t>(t.numel()));
    return t;
}

void to_buf(const tt::Tensor& t, float* dst) {
    if (dst)
        std::memcpy(dst, t.data(), sizeof(float) * static_cast<size_t>(t.numel()));
}

void grad_to_buf(const tt::Tensor& t, float* dst) {
    if (!dst)
        return;
    if (t.has_grad())
        std::memcpy(dst, t.grad_data(), sizeof(float) * static_cast<size_t>(t.numel()));
    else
        std::memset(dst, 0, sizeof(float) * static_cast<size_t>(t.numel()));
}

// loss = sum_all(y * G); backward seeds y.grad = G.
void seed_backward(const tt::Tensor& y, const float* G) {
    tt::Tensor g = from_buf(y.shape(), G, false);
    tt::Tensor loss = tt::sum_all(tt::mul(y, g));
    loss.backward();
}

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return 1;
    }
}

struct RefCfg {
    int64_t vocab, dim, layers, heads, ffn, max_seq;
    float norm_eps, rope_theta;
};

tt::GPTConfig to_cfg(const RefCfg* c) {
    tt::GPTConfig cfg;
    cfg.vocab_size = c->vocab;
    cfg.dim = c->dim;
    cfg.n_layers = c->layers;
    cfg.n_heads = c->heads;
    cfg.n_kv_heads = c->heads;
    cfg.ffn_dim = c->ffn;
    cfg.max_seq_len = c->max_seq;
    cfg.norm_eps = c->norm_eps;
    cfg.rope_theta = c->rope_theta;
    return cfg;
}

void load_params(tt::GPTModel& m, const float* w) {
    size_t off = 0;
    for (tt::Tensor* p : m.parameters()) {
        std::memcpy(p->data(), w + off, sizeof(float) * static_cast<size_t>(p->numel()));
        off += static_cast<size_t>(p->numel());
    }
}

void store_params(tt::GPTModel& m, float* w) {
    size_t off = 0;
    for (tt::Tensor* p : m.parameters()) {
        std::memcpy(w + off, p->data(), sizeof(float) * static_cast<size_t>(p->numel()));
        off += static_cast<size_t>(p->numel());
    }
}

void store_grads(tt::GPTModel& m, float* g) {
    size_t off = 0;
    for (tt::Tensor* p : m.parameters()) {
        grad_to_buf(*p, g + off);
        off += static_cast<size_t>(p->numel());
    }
}

// Global-norm gradient clipping. The reference has no clipping (its README
// claims it, but no symbol exists); this restates the conventional rule
// (torch.nn.utils.clip_grad_norm_): total = sqrt(sum over all grads of g^2),
// coef = max_norm / (total + 1e-6), grads *= coef when coef < 1. The sum is
// accumulated in double, like the reference's other full reductions
// (ops.cpp:441-460 sum_all).
double clip_grads(const std::vector<tt::Tensor*>& ps, float max_norm) {
    double ss = 0.0;
    for (tt::Tensor* p : ps) {
        if (!p->has_grad())
            continue;
        const float* g = p->grad_data();
        for (int64_t i = 0; i < p->numel(); ++i)
            ss += static_cast<double>(g[i]) * g[i];
    }
    double total = std::sqrt(ss);
    if (max_norm > 0.0f) {
        float coef = static_cast<float>(max_norm / (total + 1e-6));
        if (coef < 1.0f) {
            for (tt::Tensor* p : ps) {
                if (!p->has_grad())
                    continue;
                float* g = p->grad_data();
                for (int64_t i = 0; i < p->numel(); ++i)
                    g[i] *= coef;
            }
        }
    }
    return total;
}

// The reference's backward closures capture their own node by shared_ptr
// (e.g. ops.cpp:169-171), so every graph is a reference cycle and is never
// freed; a multi-step run would exhaust host memory. After a step, walk the
// graph from the loss and drop each node's closure and edges (both public
// members of the reference's Tensor::Impl, tensor.h:21-32). Values already
// computed are unaffected.
void release_graph(const tt::Tensor& root) {
    std::vector<std::shared_ptr<tt::Tensor::Impl>> stack{root.impl()}, seen;
    std::vector<tt::Tensor::Impl*> visited;
    while (!stack.empty()) {
        auto n = stack.back();
        stack.pop_back();
        bool dup = false;
        for (auto* v : visited)
            if (v == n.get()) {
                dup = true;
                break;
            }
        if (dup)
            continue;
        visited.push_back(n.get());
        seen.push_back(n);
        for (auto& p : n->prev)
            stack.push_back(p);
    }
    for (auto& n : seen) {
        n->backward_fn = [] {};
        n->prev.clear();
    }
}

} // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

// C = A[M,K] @ B[K,N] (ops.cpp:661-697); dA, dB from upstream G[M,N].
int ref_matmul(int64_t M, int64_t K, int64_t N, const float* A, const float* B,
               const float* G, float* C, float* dA, float* dB) {
    return guarded([&] {
        tt::Tensor a = from_buf({M, K}, A, true), b = from_buf({K, N}, B, true);
        tt::Tensor c = tt::matmul(a, b);
        to_buf(c, C);
        if (G) {
            seed_backward(c, G);
            grad_to_buf(a, dA);
            grad_to_buf(b, dB);
        }
    });
}

// Linear layer y = x @ W^T with W [out,in] (nn.cpp:23-26): the transpose is a
// permute copy whose backward scatters dW^T back into W's layout.
int ref_linear(int64_t R, int64_t in, int64_t out, const float* X, const float* W,
               const float* G, float* Y, float* dX, float* dW) {
    return guarded([&] {
        tt::Tensor x = from_buf({R, in}, X, true), w = from_buf({out, in}, W, true);
        tt::Tensor y = tt::matmul(x, tt::transpose(w, 0, 1));
        to_buf(y, Y);
        if (G) {
            seed_backward(y, G);
            grad_to_buf(x, dX);
            grad_to_buf(w, dW);
        }
    });
}

// C = A[Bt,M,K] @ B[Bt,K,N] (ops.cpp:699-742).
int ref_bmm(int64_t Bt, int64_t M, int64_t K, int64_t N, const float* A, const float* B,
            const float* G, float* C, float* dA, float* dB) {
    return guarded([&] {
        tt::Tensor a = from_buf({Bt, M, K}, A, true), b = from_buf({Bt, K, N}, B, true);
        tt::Tensor c = tt::bmm(a, b);
        to_buf(c, C);
        if (G) {
            seed_backward(c, G);
            grad_to_buf(a, dA);
            grad_to_buf(b, dB);
        }
    });
}

// y = rmsnorm(x [R,D], w [D], eps) (ops.cpp:932-942).
int ref_rmsnorm(int64_t R, int64_t D, const float* X, const float* Wt, float eps,
                const float* G, float* Y, float* dX, float* dW) {
    return guarded([&] {
        tt::Tensor x = from_buf({R, D}, X, true), w = from_buf({D}, Wt, true);
        tt::Tensor y = tt::rmsnorm(x, w, eps);
        to_buf(y, Y);
        if (G) {
            seed_backward(y, G);
            grad_to_buf(x, dX);
            grad_to_buf(w, dW);
        }
    });
}

// y = silu(a) * b, the SwiGLU product of model.cpp:149-151.
int ref_swiglu(int64_t R, int64_t F, const float* Ain, const float* Bin, const float* G,
               float* Y, float* dA, float* dB) {
    return guarded([&] {
        tt::Tensor a = from_buf({R, F}, Ain, true), b = from_buf({R, F}, Bin, true);
        tt::Tensor y = tt::mul(tt::silu(a), b);
        to_buf(y, Y);
        if (G) {
            seed_backward(y, G);
            grad_to_buf(a, dA);
            grad_to_buf(b, dB);
        }
    });
}

// loss = cross_entropy(logits [N,C], targets) (ops.cpp:928-930) and its
// gradient with respect to the logits for d(loss) = 1.
int ref_cross_entropy(int64_t N, int64_t C, const float* logits, const int64_t* targets,
                      float* loss, float* dlogits) {
    return guarded([&] {
        tt::Tensor x = from_buf({N, C}, logits, true);
        std::vector<int64_t> t(targets, targets + N);
        tt::Tensor l = tt::cross_entropy(x, t);
        *loss = l.data()[0];
        if (dlogits) {
            l.backward();
            grad_to_buf(x, dlogits);
        }
    });
}

// out = embedding(W [V,D], idx [N]) (ops.cpp:746-775).
int ref_embedding(int64_t V, int64_t D, const float* Wt, int64_t N, const int64_t* idx,
                  const float* G, float* out, float* dW) {
    return guarded([&] {
        tt::Tensor w = from_buf({V, D}, Wt, true);
        std::vector<int64_t> ix(idx, idx + N);
        tt::Tensor y = tt::embedding(w, ix);
        to_buf(y, out);
        if (G) {
            seed_backward(y, G);
            grad_to_buf(w, dW);
        }
    });
}

// out = rope(x [B,T,H,D], cos [T,D/2], sin [T,D/2]) (ops.cpp:970-1052).
int ref_rope(int64_t B, int64_t T, int64_t H, int64_t D, const float* X, const float* cs,
             const float* sn, const float* G, float* Y, float* dX) {
    return guarded([&] {
        tt::Tensor x = from_buf({B, T, H, D}, X, true);
        tt::Tensor c = from_buf({T, D / 2}, cs, false), s = from_buf({T, D / 2}, sn, false);
        tt::Tensor y = tt::rope(x, c, s);
        to_buf(y, Y);
        if (G) {
            seed_backward(y, G);
            grad_to_buf(x, dX);
        }
    });
}

// The reference's dropout mask for n elements (ops.cpp:944-968): dropout of
// a tensor of ones, whose output is mask / (1 - p); mask[i] = (out[i] != 0).
int ref_dropout_mask(int64_t n, float p, uint64_t seed, float* mask) {
    return guarded([&] {
        tt::Tensor ones = tt::full({n}, 1.0f);
        tt::Tensor y = tt::dropout(ones, p, seed);
        const float* d = y.data();
        for (int64_t i = 0; i < n; ++i)
            mask[i] = d[i] != 0.0f ? 1.0f : 0.0f;
    });
}

// y = softmax(x [R,C], -1) (ops.cpp:777-838).
int ref_softmax(int64_t R, int64_t C, const float* X, const float* G, float* Y, float* dX) {
    return guarded([&] {
        tt::Tensor x = from_buf({R, C}, X, true);
        tt::Tensor y = tt::softmax(x, -1);
        to_buf(y, Y);
        if (G) {
            seed_backward(y, G);
            grad_to_buf(x, dX);
        }
    });
}

// The attention block of GPTModel::forward (model.cpp:127-141) on q, k, v
// given as [B,T,H,hd] projections: rope(q), rope(k) with the model's own
// tables (model.cpp:43-53), permute to [B*H,T,hd], bmm, scale, causal mask,
// softmax, bmm, permute back to [B,T,H*hd].
int ref_attention(int64_t B, int64_t T, int64_t H, int64_t hd, float theta, const float* Q,
                  const float* K, const float* V, const float* G, float* O, float* dQ,
                  float* dK, float* dV) {
    return guarded([&] {
        int64_t Dh = hd / 2;
        tt::Tensor cos = tt::full({T, Dh}, 0.0f), sin = tt::full({T, Dh}, 0.0f);
        for (int64_t pos = 0; pos < T; ++pos)
            for (int64_t i = 0; i < Dh; ++i) {
                float inv_freq =
                    1.0f / std::pow(theta, (2.0f * i) / static_cast<float>(hd));
                float angle = static_cast<float>(pos) * inv_freq;
                cos.data()[pos * Dh + i] = std::cos(angle);
                sin.data()[pos * Dh + i] = std::sin(angle);
            }
        tt::Tensor mask = tt::full({T, T}, 0.0f);
        for (int64_t i = 0; i < T; ++i)
            for (int64_t j = i + 1; j < T; ++j)
                mask.data()[i * T + j] = -1e9f;
        float scale = 1.0f / std::sqrt(static_cast<float>(hd));
        tt::Tensor q = from_buf({B, T, H, hd}, Q, true);
        tt::Tensor k = from_buf({B, T, H, hd}, K, true);
        tt::Tensor v = from_buf({B, T, H, hd}, V, true);
        tt::Tensor qr = tt::rope(q, cos, sin), kr = tt::rope(k, cos, sin);
        tt::Tensor qb = tt::reshape(tt::permute(qr, {0, 2, 1, 3}), {B * H, T, hd});
        tt::Tensor kb = tt::reshape(tt::permute(kr, {0, 2, 1, 3}), {B * H, T, hd});
        tt::Tensor vb = tt::reshape(tt::permute(v, {0, 2, 1, 3}), {B * H, T, hd});
        tt::Tensor scores = tt::bmm(qb, tt::transpose(kb, 1, 2));
        scores = tt::mul(scores, tt::full(scores.shape(), scale));
        scores = tt::add(scores, mask);
        tt::Tensor probs = tt::softmax(scores, -1);
        tt::Tensor att = tt::bmm(probs, vb);
        tt::Tensor out = tt::reshape(
            tt::permute(tt::reshape(att, {B, H, T, hd}), {0, 2, 1, 3}), {B, T, H * hd});
        to_buf(out, O);
        if (G) {
            seed_backward(out, G);
            grad_to_buf(q, dQ);
            grad_to_buf(k, dK);
            grad_to_buf(v, dV);
        }
    });
}

// K steps of the reference AdamW (optim.cpp:17-48) on one parameter of n
// elements, with the gradient of step s taken from grads[s*n .. s*n+n).
int ref_adamw(int64_t n, float* p, const float* grads, int64_t K, float lr, float b1,
              float b2, float eps, float wd) {
    return guarded([&] {
        tt::Tensor x = from_buf({n}, p, true);
        tt::AdamW opt({&x}, lr, b1, b2, eps, wd);
        for (int64_t s = 0; s < K; ++s) {
            opt.zero_grad();
            std::memcpy(x.grad_data(), grads + s * n, sizeof(float) * static_cast<size_t>(n));
            opt.step();
        }
        to_buf(x, p);
    });
}

// Number of parameters of GPTModel for a config (model.cpp:56-85 order).
int64_t ref_param_count(const RefCfg* c) {
    try {
        tt::GPTConfig cfg = to_cfg(c);
        int64_t hd = cfg.dim / cfg.n_heads;
        int64_t per_layer = 2 * cfg.dim + 4 * cfg.dim * cfg.n_heads * hd + 3 * cfg.dim * cfg.ffn_dim;
        return cfg.vocab_size * cfg.dim + cfg.n_layers * per_layer + cfg.dim;
    } catch (...) {
        return -1;
    }
}

// Parameter shapes in GPTModel::parameters() order: writes (rows, cols) pairs
// (cols = 0 for 1-D) into shapes[2*i], returns the count.
int64_t ref_param_shapes(const RefCfg* c, int64_t* shapes, int64_t cap) {
    try {
        tt::GPTConfig cfg = to_cfg(c);
        cfg.vocab_size = c->vocab;
        tt::GPTModel m(cfg, 1);
        auto ps = m.parameters();
        int64_t i = 0;
        for (tt::Tensor* p : ps) {
            if (i < cap) {
                shapes[2 * i] = p->dim(0);
                shapes[2 * i + 1] = p->ndim() > 1 ? p->dim(1) : 0;
            }
            ++i;
        }
        return i;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

// The reference's own initialization of GPTModel(cfg, seed) (model.cpp:14-54,
// nn.cpp:14-44), flattened in parameters() order.
int ref_init_params(const RefCfg* c, uint64_t seed, float* out) {
    return guarded([&] {
        tt::GPTModel m(to_cfg(c), seed);
        store_params(m, out);
    });
}

// Parameters of a GPTModel after the reference's load_checkpoint(dir)
// (model.cpp:229-280), flat in parameters() order.
int ref_load_checkpoint(const RefCfg* c, const char* dir, float* out) {
    return guarded([&] {
        tt::GPTModel m(to_cfg(c), 1);
        m.load_checkpoint(dir);
        store_params(m, out);
    });
}

// logits = GPTModel::forward(idx, B, T) (model.cpp:87-160) with the given
// flat parameters; optionally the loss and every parameter gradient of
// cross_entropy(logits, targets).
int ref_model_fwd_bwd(const RefCfg* c, const float* params, const int64_t* idx,
                      const int64_t* targets, int64_t B, int64_t T, float* logits,
                      float* loss, float* grads) {
    return guarded([&] {
        tt::GPTModel m(to_cfg(c), 1);
        load_params(m, params);
        std::vector<int64_t> ix(idx, idx + B * T);
        m.zero_grad();
        tt::Tensor lg = m.forward(ix, B, T);
        to_buf(lg, logits);
        if (targets) {
            std::vector<int64_t> tg(targets, targets + B * T);
            tt::Tensor l = tt::cross_entropy(lg, tg);
            if (loss)
                *loss = l.data()[0];
            if (grads) {
                l.backward();
                store_grads(m, grads);
            }
        }
    });
}

// The training loop of apps/train.cpp:212-256 with fixed batches: per step
// zero_grad, forward, cross_entropy, backward, optional global-norm clipping
// (restated above), AdamW step at lrs[s]. idx/targets hold steps*B*T ids.
// Writes losses[steps], grad_norms[steps] (pre-clip) and the final params.
int ref_train(const RefCfg* c, float* params, const int64_t* idx, const int64_t* targets,
              int64_t B, int64_t T, int64_t steps, const float* lrs, float b1, float b2,
              float eps, float wd, float clip, float* losses, float* grad_norms) {
    return guarded([&] {
        tt::GPTModel m(to_cfg(c), 1);
        load_params(m, params);
        auto ps = m.parameters();
        tt::AdamW opt(ps, lrs[0], b1, b2, eps, wd);
        for (int64_t s = 0; s < steps; ++s) {
            std::vector<int64_t> ix(idx + s * B * T, idx + (s + 1) * B * T);
            std::vector<int64_t> tg(targets + s * B * T, targets + (s + 1) * B * T);
            opt.zero_grad();
            tt::Tensor lg = m.forward(ix, B, T);
            tt::Tensor l = tt::cross_entropy(lg, tg);
            losses[s] = l.data()[0];
            l.backward();
            double gn = clip_grads(ps, clip);
            if (grad_norms)
                grad_norms[s] = static_cast<float>(gn);
            opt.set_lr(lrs[s]);
            opt.step();
            release_graph(l);
        }
        store_params(m, params);
    });
}

// CPU baseline: one full training step (forward, cross-entropy, backward,
// AdamW) of the reference at the given config on B x T random tokens, timed
// with steady_clock over `steps` steps after `warmup` untimed ones. Model
// construction (the reference's own Xavier init) is not timed. Returns the
// mean seconds per timed step in *secs.
int ref_time_train(const RefCfg* c, int64_t B, int64_t T, int64_t warmup, int64_t steps,
                   uint64_t seed, double* secs) {
    return guarded([&] {
        tt::GPTModel m(to_cfg(c), seed);
        auto ps = m.parameters();
        tt::AdamW opt(ps, 3e-4f, 0.9f, 0.95f, 1e-8f, 0.1f);
        uint64_t s = seed ? seed : 1;
        auto next = [&]() {
            s ^= s >> 12;
            s ^= s << 25;
            s ^= s >> 27;
            return s * 0x2545F4914F6CDD1DULL;
        };
        std::vector<int64_t> ix(static_cast<size_t>(B * T)), tg(static_cast<size_t>(B * T));
        double total = 0.0;
        for (int64_t it = 0; it < warmup + steps; ++it) {
            for (auto& v : ix)
                v = static_cast<int64_t>(next() % static_cast<uint64_t>(c->vocab));
            for (auto& v : tg)
                v = static_cast<int64_t>(next() % static_cast<uint64_t>(c->vocab));
            auto t0 = std::chrono::steady_clock::now();
            opt.zero_grad();
            tt::Tensor lg = m.forward(ix, B, T);
            tt::Tensor l = tt::cross_entropy(lg, tg);
            volatile float lv = l.data()[0];
            (void)lv;
            l.backward();
            clip_grads(ps, 1.0f);
            opt.step();
            auto t1 = std::chrono::steady_clock::now();
            release_graph(l);
            if (it >= warmup)
                total += std::chrono::duration<double>(t1 - t0).count();
        }
        *secs = total / static_cast<double>(steps > 0 ? steps : 1);
    });
}

// CPU baseline by phase, on one micro-batch of B x T random tokens: the mean
// seconds of (zero_grad, forward, cross_entropy, backward) over `steps`
// micro-steps after `warmup` untimed ones, and of one optimizer step (global
// -norm clip as restated above, then AdamW::step) timed once after them. The
// caller amortizes the optimizer over as many micro-batches as a global
// batch holds, as gradient accumulation does. Model construction is untimed.
int ref_time_phases(const RefCfg* c, int64_t B, int64_t T, int64_t warmup, int64_t steps,
                    uint64_t seed, double* fb_secs, double* opt_secs) {
    return guarded([&] {
        tt::GPTModel m(to_cfg(c), seed);
        auto ps = m.parameters();
        tt::AdamW opt(ps, 3e-4f, 0.9f, 0.95f, 1e-8f, 0.1f);
        uint64_t s = seed ? seed : 1;
        auto next = [&]() {
            s ^= s >> 12;
            s ^= s << 25;
            s ^= s >> 27;
            return s * 0x2545F4914F6CDD1DULL;
        };
        std::vector<int64_t> ix(static_cast<size_t>(B * T)), tg(static_cast<size_t>(B * T));
        double total = 0.0;
        for (int64_t it = 0; it < warmup + steps; ++it) {
            for (auto& v : ix)
                v = static_cast<int64_t>(next() % static_cast<uint64_t>(c->vocab));
            for (auto& v : tg)
                v = static_cast<int64_t>(next() % static_cast<uint64_t>(c->vocab));
            auto t0 = std::chrono::steady_clock::now();
            opt.zero_grad();
            tt::Tensor lg = m.forward(ix, B, T);
            tt::Tensor l = tt::cross_entropy(lg, tg);
            volatile float lv = l.data()[0];
            (void)lv;
            l.backward();
            auto t1 = std::chrono::steady_clock::now();
            release_graph(l);
            if (it >= warmup)
                total += std::chrono::duration<double>(t1 - t0).count();
        }
        *fb_secs = total / static_cast<double>(steps > 0 ? steps : 1);
        auto t0 = std::chrono::steady_clock::now();
        clip_grads(ps, 1.0f);
        opt.step();
        auto t1 = std::chrono::steady_clock::now();
        *opt_secs = std::chrono::duration<double>(t1 - t0).count();
    });
}

} // extern "C"
