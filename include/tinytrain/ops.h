#pragma once

// Differentiable ops on device tensors. Same signatures and argument checks
// as the reference's ops.h (ops.h:15-59 of seampm/tinytrain); every op runs
// as CUDA kernels through the ttk C ABI, and its backward rule accumulates
// into the inputs' gradients like the reference's closures (ops.cpp:12-15).
//
// Composite ops of the reference (rmsnorm, cross_entropy, softmax-based
// attention) are single fused nodes here; their gradients match the
// composites' to fp32 rounding.

#include <cstdint>
#include <vector>

#include "tinytrain/tensor.h"

namespace tt {

// ---- elementwise (NumPy-style trailing broadcasting) ----
Tensor add(const Tensor& a, const Tensor& b);
Tensor sub(const Tensor& a, const Tensor& b);
Tensor mul(const Tensor& a, const Tensor& b);
Tensor div(const Tensor& a, const Tensor& b);
Tensor neg(const Tensor& a);

// ---- unary ----
Tensor exp(const Tensor& a);
Tensor log(const Tensor& a);
Tensor sqrt(const Tensor& a);
Tensor tanh(const Tensor& a);
Tensor silu(const Tensor& a); // x * sigmoid(x)
Tensor sin(const Tensor& a);
Tensor cos(const Tensor& a);
Tensor pow(const Tensor& a, float p);

// ---- reductions ----
Tensor sum(const Tensor& a, int64_t dim, bool keepdim = false);
Tensor sum_all(const Tensor& a);
Tensor mean(const Tensor& a);

// ---- shape ----
Tensor reshape(const Tensor& a, const std::vector<int64_t>& shape);
Tensor transpose(const Tensor& a, int64_t d0, int64_t d1);
Tensor permute(const Tensor& a, const std::vector<int64_t>& dims);
Tensor expand(const Tensor& a, const std::vector<int64_t>& shape);
Tensor squeeze(const Tensor& a, int64_t dim);
Tensor unsqueeze(const Tensor& a, int64_t dim);

// ---- linear algebra ----
Tensor matmul(const Tensor& a, const Tensor& b); // 2D @ 2D
Tensor bmm(const Tensor& a, const Tensor& b);    // [B,M,K] @ [B,K,N]

// ---- neural nets ----
Tensor embedding(const Tensor& weight, const std::vector<int64_t>& idx); // [V,D] -> [N,D]
Tensor softmax(const Tensor& a, int64_t dim);
Tensor log_softmax(const Tensor& a, int64_t dim);
// mean negative log-likelihood; log_probs [N,C]
Tensor nll_loss(const Tensor& log_probs, const std::vector<int64_t>& targets);
Tensor cross_entropy(const Tensor& logits, const std::vector<int64_t>& targets);
// x normalized over last dim, scaled by weight; eps for stability
Tensor rmsnorm(const Tensor& a, const Tensor& weight, float eps);
Tensor dropout(const Tensor& a, float p, uint64_t seed);
// Rotary position embeddings: x [B,T,H,D] (D even), cos/sin [T,D/2]
Tensor rope(const Tensor& x, const Tensor& cos, const Tensor& sin);

// ---- fused ops (extensions; not in the reference) ----

// Token ids resident on the device (int64), for inputs uploaded once per
// step instead of per op.
struct DeviceIds {
    DeviceIds() = default;
    explicit DeviceIds(const std::vector<int64_t>& host);
    DeviceIds(const int64_t* host, int64_t n);
    // Adopt device memory holding n ids (not owned).
    static DeviceIds borrow(const int64_t* dev, int64_t n);
    int64_t size() const { return n; }
    const int64_t* data() const;
    std::shared_ptr<void> buf;
    const int64_t* dev = nullptr;
    int64_t n = 0;
};

// y = x @ W^T with W [out, in] (nn.cpp:23-26 without the transpose copy).
Tensor linear(const Tensor& x, const Tensor& weight);
// Causal self-attention with RoPE on q, k, v [B,T,H,hd] (pre-RoPE), scale
// 1/sqrt(hd); returns [B,T,H*hd]. Replaces model.cpp:127-141.
Tensor causal_attention(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& cos,
                        const Tensor& sin);
// The reference's own op chain for attention, bmm(q, transpose(k)) [N,T,T]
// with q, k [N,T,hd] (hd 32, 64 or 128), mul by a full() constant, add of a
// [T,T] causal mask (0 on/below the diagonal, <= -1e9 above), softmax(-1),
// bmm(., v), also runs as the fused kernel: the intermediate results are
// deferred and computed only if something else reads them. Number of chains
// fused so far:
int64_t fused_attention_chains();
Tensor embedding(const Tensor& weight, const DeviceIds& idx);
// cross_entropy with device-resident, range-checked targets.
Tensor cross_entropy(const Tensor& logits, const DeviceIds& targets);
// silu(a) * b fused (model.cpp:149-151).
Tensor swiglu(const Tensor& a, const Tensor& b);
// The SwiGLU feed-forward block linear(swiglu(linear(x, w_gate),
// linear(x, w_up)), w_down) as one op (model.cpp:148-152), same results.
Tensor ffn_swiglu(const Tensor& x, const Tensor& w_gate, const Tensor& w_up,
                  const Tensor& w_down);
// Global L2 norm of the gradients of `params`; when max_norm > 0 the
// gradients are scaled by max_norm / (norm + 1e-6) if that is < 1
// (the conventional rule; the reference has no clipping). Returns the norm.
float clip_grad_norm(const std::vector<Tensor*>& params, float max_norm);

} // namespace tt
