#pragma once

// tinytrain Tensor on B200 device storage.
//
// Same public API as the reference's tensor.h (tensor.h:19-78 of
// seampm/tinytrain): a Tensor is a cheap shared handle to an Impl holding the
// shape, the data, an optional accumulated gradient and the graph edges of the
// op that produced it; backward() topologically sorts from a scalar and runs
// each node's closure in reverse, accumulating gradients.
//
// What changes underneath: data and grad live in HBM (fp32, row-major), and
// every op runs as a CUDA kernel through the ttk C ABI (include/ttk.h).
// data() / grad_data() still return writable host pointers: they bring the
// device copy into a host mirror, and a write through them is uploaded before
// the next device use (the mirror-on-access contract that lets host code such
// as tests and checkpoint I/O keep indexing element by element). There is no
// host compute path: without a CUDA device every op throws.
//
// Differences from the reference, all invisible to its model.cpp/train.cpp:
//  - reshape / squeeze / unsqueeze return views sharing the input's storage
//    (the reference copies); their gradients are still separate.
//  - a 2-D transpose (and the last-two-dims transpose of a 3-D tensor) is
//    lazy: matmul/bmm read it as a transposed operand without a copy.
//  - the attention-score chain of model.cpp:133-138, bmm(q, transpose(k)),
//    mul by a constant, add of a causal mask, softmax, is deferred: each of
//    those results keeps a recipe instead of a [B*H, T, T] buffer, and the
//    closing bmm(probs, v) runs the fused causal attention kernel. A deferred
//    result read any other way (data(), another op) is computed then, with
//    the reference's own op sequence, so every value stays observable.

#include <cstdint>
#include <functional>
#include <memory>
#include <vector>

namespace tt {

struct Deferred;  // recipe of a deferred result (see Tensor::Impl::deferred)

// Device buffer of fp32 values with a host mirror. Shared between views.
struct Buffer {
    explicit Buffer(int64_t n);
    ~Buffer();
    Buffer(const Buffer&) = delete;
    Buffer& operator=(const Buffer&) = delete;

    int64_t n = 0;
    float* dev = nullptr;        // device storage (owned unless `external`)
    std::vector<float> host;     // mirror, valid when host_valid
    bool dev_valid = false;      // device copy is current
    bool host_valid = false;     // host mirror is current
    bool pending_fill = false;   // logically filled with fill_value, not yet written
    float fill_value = 0.0f;
    bool external = false;       // dev points into memory owned elsewhere
    uint64_t version = 0;        // bumped on every device-side write
    // Cached three-term split of the contents as a GEMM operand (ttk_gemm_split
    // layout; device memory owned by the buffer), valid while split_version ==
    // version and the key (offset, batch, rows, cols, ld, batch stride,
    // precision) matches: a tensor read by several GEMMs is split once.
    void* split_dev = nullptr;
    size_t split_bytes = 0;
    uint64_t split_version = ~0ull;
    int64_t split_key[7] = {};
    // Whether the contents form a causal attention mask (0 on and below the
    // diagonal, <= -1e9 above), valid while mask_version == version.
    uint64_t mask_version = ~0ull;
    bool causal_mask = false;

    float* device();             // make the device copy current, return it
    float* device_for_overwrite();  // caller overwrites everything: skip uploads
    float* host_ptr();           // make the mirror current (device -> host)
    void host_written();         // the mirror was written: device is stale
    void fill(float v);          // lazy fill (materialized on first use)
    void touch() { ++version; }
};

class Tensor {
public:
    struct Impl {
        std::vector<int64_t> shape;
        std::vector<int64_t> strides;  // row-major
        int64_t numel = 0;
        std::shared_ptr<Buffer> data;

        bool requires_grad = false;
        std::shared_ptr<Buffer> grad;  // null until the first accumulation
        bool grad_fresh = false;       // grad holds zeros not yet written

        // Lazy transpose: this tensor is `base` with its last two dims
        // swapped; `data` stays null until someone needs it materialized.
        std::shared_ptr<Impl> transpose_of;
        // Deferred value: `data` stays null until the recipe is computed
        // (or an op consumes the recipe without ever computing it).
        std::shared_ptr<Deferred> deferred;

        std::function<void()> backward_fn = [] {};
        std::vector<std::shared_ptr<Impl>> prev;
    };

    Tensor() = default;
    explicit Tensor(std::vector<int64_t> shape, bool requires_grad = false);
    Tensor(std::vector<int64_t> shape, float fill, bool requires_grad = false);

    static Tensor from_impl(std::shared_ptr<Impl> impl);

    // ---- storage / shape ----
    const std::vector<int64_t>& shape() const { return impl_->shape; }
    int64_t ndim() const { return static_cast<int64_t>(impl_->shape.size()); }
    int64_t numel() const { return impl_->numel; }
    int64_t dim(int64_t i) const { return impl_->shape.at(static_cast<size_t>(i)); }
    float* data();
    const float* data() const;
    int64_t offset(const std::vector<int64_t>& idx) const;

    // ---- autograd ----
    bool requires_grad() const { return impl_->requires_grad; }
    void set_requires_grad(bool v);
    bool has_grad() const { return impl_->grad != nullptr; }
    float* grad_data();
    const float* grad_data() const;
    void zero_grad();

    // Reverse-mode differentiation. Must be called on a scalar tensor.
    // Accumulates gradients into every requires_grad leaf/input.
    void backward();

    // Same storage, detached from the graph.
    Tensor detach() const;

    std::shared_ptr<Impl> impl() { return impl_; }
    const std::shared_ptr<Impl>& impl() const { return impl_; }

    // ---- device access (extensions) ----
    // Device pointer of the data / gradient (materializing lazy state).
    float* device_data() const;
    float* device_grad() const;
    // Copy host values in / out without going through the mirror.
    void copy_from_host(const float* src);
    void copy_to_host(float* dst) const;

private:
    std::shared_ptr<Impl> impl_;
};

// ---- construction helpers ----
Tensor zeros(const std::vector<int64_t>& shape, bool requires_grad = false);
Tensor ones(const std::vector<int64_t>& shape, bool requires_grad = false);
Tensor full(const std::vector<int64_t>& shape, float v, bool requires_grad = false);
// Standard-normal samples, deterministic for a given seed (the reference's
// xorshift64* + Box-Muller stream, generated on the host and uploaded).
Tensor randn(const std::vector<int64_t>& shape, uint64_t seed);
// Uniform samples in [lo, hi), deterministic for a given seed.
Tensor rand_uniform(const std::vector<int64_t>& shape, float lo, float hi, uint64_t seed);

// ---- runtime (extensions) ----
// The CUDA stream every op is issued on (default: a stream owned by the
// library). Set it to share ordering with another runtime (e.g. torch).
void set_stream(void* stream);
void* get_stream();
// Blocks until all issued work finished; throws on a device error.
void synchronize();
// Called with each leaf whose gradient is final during backward(), in
// completion order (used to launch gradient all-reduce buckets early).
void set_grad_ready_hook(std::function<void(const std::shared_ptr<Tensor::Impl>&)> hook);

} // namespace tt
