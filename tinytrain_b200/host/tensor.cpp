// Tensor storage on the device, the host mirror, and the autograd engine.
//
// The graph engine follows the reference's design (tensor.cpp:83-113 of
// seampm/tinytrain): a DFS topological order from the scalar loss, non-leaf
// gradients cleared, seed 1.0, closures run in reverse. Two additions: each
// non-leaf gradient buffer is released right after its node's closure ran
// (activation gradients would otherwise stay resident until the graph dies),
// and an optional hook reports each leaf whose gradient is final, so a
// data-parallel driver can start reducing finished buckets during backward.
#include <cmath>
#include <cstring>
#include <functional>
#include <mutex>
#include <numeric>
#include <stdexcept>
#include <unordered_map>
#include <unordered_set>

#include "internal.h"
#include "tinytrain/tensor.h"
#include "ttk.h"

namespace tt {

namespace {

void* g_stream = nullptr;
bool g_stream_set = false;
std::once_flag g_init_once;
std::function<void(const std::shared_ptr<Tensor::Impl>&)> g_grad_hook;

}  // namespace

namespace detail {

void ensure_runtime() {
    std::call_once(g_init_once, [] {
        int n = 0;
        if (ttk_device_count(&n) != TTK_OK || n < 1)
            throw std::runtime_error(
                "tinytrain: no CUDA device (the device kernels are the only implementation)");
        // The device the calling thread already has current (selected by the
        // application, e.g. one GPU per rank), device 0 otherwise.
        int dev = 0;
        check(ttk_current_device(&dev), "current device");
        check(ttk_init(dev), "ttk_init");
        if (!g_stream_set)
            check(ttk_stream_create(&g_stream), "stream create");
    });
}

void* stream() {
    ensure_runtime();
    return g_stream;
}

void* stream_if_ready() { return g_stream; }

std::vector<int64_t> row_major(const std::vector<int64_t>& shape) {
    std::vector<int64_t> st(shape.size());
    int64_t s = 1;
    for (int64_t i = static_cast<int64_t>(shape.size()) - 1; i >= 0; --i) {
        st[static_cast<size_t>(i)] = s;
        s *= shape[static_cast<size_t>(i)];
    }
    return st;
}

int64_t numel_of(const std::vector<int64_t>& shape) {
    int64_t n = 1;
    for (int64_t d : shape)
        n *= d;
    return n;
}

Scratch::Scratch(size_t b) : bytes(b) {
    if (b)
        check(ttk_malloc(&ptr, b, stream()), "scratch alloc");
}

Scratch::~Scratch() {
    if (ptr)
        ttk_free(ptr, stream_if_ready());
}

}  // namespace detail

using namespace detail;

// ------------------------------------------------------------------ Buffer --

Buffer::Buffer(int64_t n_) : n(n_) {}

Buffer::~Buffer() {
    if (dev && !external)
        ttk_free(dev, g_stream);
    if (split_dev)
        ttk_free(split_dev, g_stream);
}

static void alloc_dev(Buffer& b) {
    if (!b.dev && b.n > 0)
        check(ttk_malloc(reinterpret_cast<void**>(&b.dev), static_cast<size_t>(b.n) * 4, stream()),
              "device alloc");
}

float* Buffer::device() {
    if (dev_valid && !pending_fill)
        return dev;
    alloc_dev(*this);
    if (pending_fill) {
        check(ttk_fill(dev, fill_value, n, stream()), "fill");
        pending_fill = false;
    } else if (host_valid) {
        check(ttk_memcpy_h2d(dev, host.data(), static_cast<size_t>(n) * 4, stream()), "upload");
    } else if (n > 0) {
        throw std::runtime_error("Buffer::device: buffer was never written");
    }
    dev_valid = true;
    return dev;
}

float* Buffer::device_for_overwrite() {
    alloc_dev(*this);
    pending_fill = false;
    dev_valid = true;
    host_valid = false;
    ++version;
    return dev;
}

float* Buffer::host_ptr() {
    if (host_valid)
        return host.data();
    host.resize(static_cast<size_t>(n));
    if (pending_fill) {
        std::fill(host.begin(), host.end(), fill_value);
    } else if (dev_valid && n > 0) {
        check(ttk_memcpy_d2h(host.data(), dev, static_cast<size_t>(n) * 4, stream()), "download");
    }
    host_valid = true;
    return host.data();
}

void Buffer::host_written() {
    pending_fill = false;
    dev_valid = false;
    ++version;
}

void Buffer::fill(float v) {
    pending_fill = true;
    fill_value = v;
    host_valid = false;
    dev_valid = false;
    ++version;
}

namespace detail {

Tensor make_out(const std::vector<int64_t>& shape, bool requires_grad) {
    return Tensor(shape, requires_grad);
}

Tensor make_view(const Tensor& src, const std::vector<int64_t>& shape, bool requires_grad) {
    auto impl = std::make_shared<Tensor::Impl>();
    impl->shape = shape;
    impl->strides = row_major(shape);
    impl->numel = numel_of(shape);
    materialize(src.impl());
    impl->data = src.impl()->data;
    impl->requires_grad = requires_grad;
    return Tensor::from_impl(impl);
}

void materialize(Tensor::Impl* p) {
    if (p->data)
        return;
    if (p->deferred) {
        // Computed with the ordinary kernels; the recipe stays attached (its
        // inputs stay alive like graph edges) but no longer fuses: a chain
        // continues only from uncomputed nodes.
        auto buf = std::make_shared<Buffer>(p->numel);
        buf->device_for_overwrite();
        p->data = buf;
        p->deferred->compute(p);
        return;
    }
    if (!p->transpose_of)
        return;
    const ImplPtr& base = p->transpose_of;
    const int64_t nd = static_cast<int64_t>(p->shape.size());
    // p's shape is base's with the last two dims swapped; gather from base.
    std::vector<int64_t> in_strides(static_cast<size_t>(nd));
    const auto bst = base->strides;
    for (int64_t d = 0; d < nd; ++d)
        in_strides[static_cast<size_t>(d)] = bst[static_cast<size_t>(d)];
    std::swap(in_strides[static_cast<size_t>(nd - 1)], in_strides[static_cast<size_t>(nd - 2)]);
    auto buf = std::make_shared<Buffer>(p->numel);
    float* out = buf->device_for_overwrite();
    check(ttk_strided_copy(dread(base), in_strides.data(), out, p->shape.data(),
                           static_cast<int>(nd), 0, 0, stream()),
          "transpose copy");
    p->data = buf;
}

const float* dread(Tensor::Impl* p) {
    if (!p->data)
        materialize(p);
    return p->data->device();
}

float* dwrite(Tensor::Impl* p) {
    if (!p->data)
        materialize(p);
    float* d = p->data->device();
    p->data->host_valid = false;
    ++p->data->version;
    return d;
}

float* grad_target(const ImplPtr& p, bool& overwrite) {
    if (!p->grad) {
        p->grad = std::make_shared<Buffer>(p->numel);
        p->grad->fill(0.0f);
    }
    Buffer& g = *p->grad;
    if (g.pending_fill && g.fill_value == 0.0f) {
        overwrite = true;
        return g.device_for_overwrite();
    }
    overwrite = false;
    float* d = g.device();
    g.host_valid = false;
    ++g.version;
    return d;
}

float* grad_rmw(const ImplPtr& p) {
    bool ow = false;
    float* d = grad_target(p, ow);
    if (ow)
        check(ttk_memset(d, 0, static_cast<size_t>(p->numel) * 4, stream()), "grad zero");
    return d;
}

const float* grad_in(const Tensor::Impl* p) {
    if (!p->grad)
        return nullptr;
    return p->grad->device();
}

}  // namespace detail

// ------------------------------------------------------------------ Tensor --

namespace {

std::shared_ptr<Tensor::Impl> make_impl(std::vector<int64_t> shape, bool requires_grad) {
    if (shape.empty())
        throw std::invalid_argument("Tensor: shape must have at least one dim");
    for (int64_t d : shape)
        if (d <= 0)
            throw std::invalid_argument("Tensor: dims must be positive");
    auto impl = std::make_shared<Tensor::Impl>();
    impl->shape = std::move(shape);
    impl->strides = row_major(impl->shape);
    impl->numel = numel_of(impl->shape);
    impl->data = std::make_shared<Buffer>(impl->numel);
    impl->requires_grad = requires_grad;
    return impl;
}

}  // namespace

Tensor::Tensor(std::vector<int64_t> shape, bool requires_grad)
    : impl_(make_impl(std::move(shape), requires_grad)) {
    // The reference zero-fills every new tensor (tensor.cpp:28); a lazy fill
    // costs nothing when the tensor is then overwritten by an op.
    impl_->data->fill(0.0f);
}

Tensor::Tensor(std::vector<int64_t> shape, float fill, bool requires_grad)
    : impl_(make_impl(std::move(shape), requires_grad)) {
    impl_->data->fill(fill);
}

Tensor Tensor::from_impl(std::shared_ptr<Impl> impl) {
    Tensor t;
    t.impl_ = std::move(impl);
    return t;
}

float* Tensor::data() {
    materialize(impl_);
    float* h = impl_->data->host_ptr();
    impl_->data->host_written();  // the caller may write through the pointer
    return h;
}

const float* Tensor::data() const {
    materialize(impl_);
    return impl_->data->host_ptr();
}

int64_t Tensor::offset(const std::vector<int64_t>& idx) const {
    if (idx.size() != impl_->shape.size())
        throw std::invalid_argument("Tensor::offset: rank mismatch");
    int64_t off = 0;
    for (size_t i = 0; i < idx.size(); ++i) {
        if (idx[i] < 0 || idx[i] >= impl_->shape[i])
            throw std::out_of_range("Tensor::offset: index out of range");
        off += idx[i] * impl_->strides[i];
    }
    return off;
}

void Tensor::set_requires_grad(bool v) {
    impl_->requires_grad = v;
    if (!v)
        impl_->grad.reset();
}

float* Tensor::grad_data() {
    if (!impl_->grad)
        return nullptr;
    float* h = impl_->grad->host_ptr();
    impl_->grad->host_written();
    return h;
}

const float* Tensor::grad_data() const {
    if (!impl_->grad)
        return nullptr;
    return impl_->grad->host_ptr();
}

void Tensor::zero_grad() {
    if (!impl_->requires_grad)
        return;
    if (!impl_->grad)
        impl_->grad = std::make_shared<Buffer>(impl_->numel);
    impl_->grad->fill(0.0f);
}

Tensor Tensor::detach() const {
    auto impl = std::make_shared<Impl>();
    impl->shape = impl_->shape;
    impl->strides = impl_->strides;
    impl->numel = impl_->numel;
    materialize(impl_);
    // The reference copies the storage (tensor.cpp:73-81).
    impl->data = std::make_shared<Buffer>(impl->numel);
    float* dst = impl->data->device_for_overwrite();
    check(ttk_memcpy_d2d(dst, impl_->data->device(), static_cast<size_t>(impl->numel) * 4,
                         stream()),
          "detach copy");
    return from_impl(impl);
}

float* Tensor::device_data() const {
    return const_cast<float*>(dread(impl_));
}

float* Tensor::device_grad() const {
    if (!impl_->grad)
        return nullptr;
    return impl_->grad->device();
}

void Tensor::copy_from_host(const float* src) {
    materialize(impl_);
    float* d = impl_->data->device_for_overwrite();
    check(ttk_memcpy_h2d(d, src, static_cast<size_t>(impl_->numel) * 4, stream()), "upload");
}

void Tensor::copy_to_host(float* dst) const {
    const float* d = dread(impl_);
    check(ttk_memcpy_d2h(dst, d, static_cast<size_t>(impl_->numel) * 4, stream()), "download");
}

void Tensor::backward() {
    if (impl_->numel != 1)
        throw std::invalid_argument("Tensor::backward: only scalar tensors");

    // Topological order via an iterative DFS over prev edges.
    std::vector<std::shared_ptr<Impl>> topo;
    std::unordered_set<Impl*> visited;
    std::vector<std::pair<std::shared_ptr<Impl>, size_t>> stack;
    stack.emplace_back(impl_, 0);
    visited.insert(impl_.get());
    while (!stack.empty()) {
        auto& [node, next] = stack.back();
        if (next < node->prev.size()) {
            auto child = node->prev[next++];
            if (visited.insert(child.get()).second)
                stack.emplace_back(child, 0);
        } else {
            topo.push_back(node);
            stack.pop_back();
        }
    }

    // Fresh backward pass: intermediate gradients are stale; leaf gradients
    // accumulate across calls (the reference's convention).
    for (auto& n : topo)
        if (!n->prev.empty())
            n->grad.reset();

    // Last consumer (in execution order) of each leaf, for the ready hook.
    std::unordered_map<Impl*, size_t> last_use;
    if (g_grad_hook) {
        size_t k = 0;
        for (auto it = topo.rbegin(); it != topo.rend(); ++it, ++k)
            for (auto& p : (*it)->prev)
                if (p->prev.empty() && p->requires_grad)
                    last_use[p.get()] = k;
    }

    impl_->grad = std::make_shared<Buffer>(1);
    impl_->grad->fill(1.0f);

    size_t k = 0;
    for (auto it = topo.rbegin(); it != topo.rend(); ++it, ++k) {
        auto& n = *it;
        n->backward_fn();
        if (!n->prev.empty() && n.get() != impl_.get())
            n->grad.reset();  // consumed: release the activation gradient
        if (g_grad_hook) {
            for (auto& p : n->prev)
                if (p->prev.empty() && p->requires_grad) {
                    auto f = last_use.find(p.get());
                    if (f != last_use.end() && f->second == k) {
                        g_grad_hook(p);
                        last_use.erase(f);
                    }
                }
        }
    }
}

// ---------------------------------------------------------- construction --

Tensor zeros(const std::vector<int64_t>& shape, bool requires_grad) {
    return Tensor(shape, 0.0f, requires_grad);
}

Tensor ones(const std::vector<int64_t>& shape, bool requires_grad) {
    return Tensor(shape, 1.0f, requires_grad);
}

Tensor full(const std::vector<int64_t>& shape, float v, bool requires_grad) {
    return Tensor(shape, v, requires_grad);
}

namespace {
// xorshift64* with Box-Muller, the reference's generator (tensor.cpp:132-149):
// kept identical so that randn(shape, seed) gives the same values.
struct Rng {
    explicit Rng(uint64_t seed) : s(seed ? seed : 0x9E3779B97F4A7C15ULL) {}
    uint64_t next() {
        s ^= s >> 12;
        s ^= s << 25;
        s ^= s >> 27;
        return s * 0x2545F4914F6CDD1DULL;
    }
    double uniform01() { return (next() >> 11) * (1.0 / 9007199254740992.0); }
    double normal() {
        double u1 = uniform01(), u2 = uniform01();
        return std::sqrt(-2.0 * std::log(u1 + 1e-300)) * std::cos(2.0 * 3.141592653589793 * u2);
    }
    uint64_t s;
};
}  // namespace

void detail::host_randn(float* out, int64_t n, uint64_t seed) {
    Rng rng(seed);
    for (int64_t i = 0; i < n; ++i)
        out[i] = static_cast<float>(rng.normal());
}

Tensor randn(const std::vector<int64_t>& shape, uint64_t seed) {
    Tensor t(shape);
    std::vector<float> h(static_cast<size_t>(t.numel()));
    host_randn(h.data(), t.numel(), seed);
    t.copy_from_host(h.data());
    return t;
}

Tensor rand_uniform(const std::vector<int64_t>& shape, float lo, float hi, uint64_t seed) {
    Tensor t(shape);
    std::vector<float> h(static_cast<size_t>(t.numel()));
    Rng rng(seed);
    for (auto& x : h)
        x = lo + static_cast<float>(rng.uniform01()) * (hi - lo);
    t.copy_from_host(h.data());
    return t;
}

// ----------------------------------------------------------------- runtime --

void set_stream(void* s) {
    // Work already issued on the previous stream completes first, so buffers
    // allocated there are safe to use and free on the new one.
    if (g_stream)
        ttk_stream_synchronize(g_stream);
    g_stream = s;
    g_stream_set = true;
    ensure_runtime();
    g_stream = s;
}

void* get_stream() { return stream(); }

void synchronize() {
    check(ttk_stream_synchronize(stream()), "synchronize");
    unsigned bits = 0;
    check(ttk_device_status(&bits), "device status");
    if (bits)
        throw std::runtime_error("tinytrain: a kernel reported device status 0x" +
                                 std::to_string(bits));
}

void set_grad_ready_hook(std::function<void(const std::shared_ptr<Tensor::Impl>&)> hook) {
    g_grad_hook = std::move(hook);
}

}  // namespace tt
