// Internals shared by the host translation units of libtinytrain.
#pragma once

#include <functional>
#include <stdexcept>
#include <string>
#include <vector>

#include "tinytrain/tensor.h"
#include "ttk.h"

namespace tt {
namespace detail {

using ImplPtr = std::shared_ptr<Tensor::Impl>;

// Throws std::runtime_error carrying ttk_last_error() when rc != TTK_OK.
inline void check(int rc, const char* what) {
    if (rc != TTK_OK)
        throw std::runtime_error(std::string(what) + ": " + ttk_last_error());
}

void* stream();
void ensure_runtime();
// The library stream if the runtime is up, else null; never throws (for
// destructors).
void* stream_if_ready();

// Row-major strides of a shape.
std::vector<int64_t> row_major(const std::vector<int64_t>& shape);
int64_t numel_of(const std::vector<int64_t>& shape);

// New tensor with an uninitialized device buffer of the given shape.
Tensor make_out(const std::vector<int64_t>& shape, bool requires_grad);
// View sharing `src`'s data buffer with another shape (same numel).
Tensor make_view(const Tensor& src, const std::vector<int64_t>& shape, bool requires_grad);

// Data of an impl materialized on the device (resolves lazy transposes).
const float* dread(Tensor::Impl* p);
float* dwrite(Tensor::Impl* p);
inline const float* dread(const ImplPtr& p) { return dread(p.get()); }
inline float* dwrite(const ImplPtr& p) { return dwrite(p.get()); }

// Gradient destination for an accumulation: returns the device pointer and
// sets `overwrite` when the gradient is still logically zero, so the caller
// may write instead of read-modify-write.
float* grad_target(const ImplPtr& p, bool& overwrite);
// Gradient for read-modify-write (materializes pending zeros).
float* grad_rmw(const ImplPtr& p);
// Upstream gradient of a node (null when nothing flowed into it). Backward
// closures refer to their own node by raw pointer: the node owns the
// closure, so a shared_ptr capture would be a cycle and leak the graph.
const float* grad_in(const Tensor::Impl* p);

// Scratch device memory released (stream-ordered) when it goes out of scope.
struct Scratch {
    explicit Scratch(size_t bytes);
    ~Scratch();
    Scratch(const Scratch&) = delete;
    Scratch& operator=(const Scratch&) = delete;
    void* ptr = nullptr;
    size_t bytes = 0;
    template <class T>
    T* as() const { return static_cast<T*>(ptr); }
};

// The reference's randn stream (xorshift64* + Box-Muller) on the host.
void host_randn(float* out, int64_t n, uint64_t seed);

// Give `p` its own data: materializes a lazy transpose or computes a
// deferred result (no-op when the data exists).
void materialize(Tensor::Impl* p);
inline void materialize(const ImplPtr& p) { materialize(p.get()); }

}  // namespace detail

// Recipe of a deferred node of the attention-score chain (model.cpp:133-137):
// scores = bmm(q, transpose(k)) [N, T, T], then optionally * constant,
// + causal mask, softmax(-1). `compute` writes the node's value into its
// (already allocated) buffer with the ordinary kernels; the closing
// bmm(probs, v) reads q, k, scale instead and never computes it.
struct Deferred {
    detail::ImplPtr q, k;         // [N, T, hd] operands of bmm(q, transpose(k))
    uint64_t vq = 0, vk = 0;      // their buffer versions when the chain began
    float scale = 1.0f;           // product of the constant factors so far
    bool masked = false;          // causal mask added
    bool softmax = false;         // row softmax applied
    std::function<void(Tensor::Impl*)> compute;
};

namespace detail {

// The chain recipe of `p` when it is an uncomputed deferred node.
inline const Deferred* pending_chain(const ImplPtr& p) {
    return (p && p->deferred && !p->data) ? p->deferred.get() : nullptr;
}

}  // namespace detail
}  // namespace tt
