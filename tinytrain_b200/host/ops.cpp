// Ops of the reference's ops.h on device tensors, with their reverse-mode
// rules (the reference's ops.cpp of seampm/tinytrain is the model: argument
// checks throw the same std::invalid_argument messages, and every backward
// closure accumulates into its inputs' gradients). Every computation is a
// ttk_* kernel call on the library stream.
//
// Gradient writes: a gradient buffer that is still logically zero is
// overwritten instead of read-modified-written (grad_target), which saves a
// memset and a read per first contribution.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <stdexcept>

#include "internal.h"
#include "tinytrain/ops.h"
#include "ttk.h"

namespace tt {

using namespace detail;

namespace {

// ------------------------------------------------------------- helpers --

std::vector<int64_t> broadcast_shape(const std::vector<int64_t>& a,
                                     const std::vector<int64_t>& b) {
    int64_t ar = static_cast<int64_t>(a.size()), br = static_cast<int64_t>(b.size());
    int64_t r = std::max(ar, br);
    std::vector<int64_t> out(static_cast<size_t>(r));
    for (int64_t i = 0; i < r; ++i) {
        int64_t ad = (i < r - ar) ? 1 : a[static_cast<size_t>(i - (r - ar))];
        int64_t bd = (i < r - br) ? 1 : b[static_cast<size_t>(i - (r - br))];
        if (ad != bd && ad != 1 && bd != 1)
            throw std::invalid_argument("broadcast: incompatible shapes");
        out[static_cast<size_t>(i)] = std::max(ad, bd);
    }
    return out;
}

int64_t norm_dim(int64_t dim, int64_t rank) {
    if (dim < 0)
        dim += rank;
    if (dim < 0 || dim >= rank)
        throw std::invalid_argument("dim out of range");
    return dim;
}

// Strides of `in` viewed in the index space of `out_shape` (trailing
// alignment, 0 on broadcast dims).
std::vector<int64_t> bcast_strides(const ImplPtr& in, const std::vector<int64_t>& out_shape) {
    const int64_t r = static_cast<int64_t>(out_shape.size());
    const int64_t ir = static_cast<int64_t>(in->shape.size());
    std::vector<int64_t> st(static_cast<size_t>(r), 0);
    for (int64_t d = 0; d < r; ++d) {
        const int64_t di = d - (r - ir);
        if (di >= 0 && in->shape[static_cast<size_t>(di)] != 1)
            st[static_cast<size_t>(d)] = in->strides[static_cast<size_t>(di)];
    }
    return st;
}

// keep mask for reducing a gradient of shape out_shape back onto `in`.
unsigned keep_mask(const ImplPtr& in, const std::vector<int64_t>& out_shape) {
    const int64_t r = static_cast<int64_t>(out_shape.size());
    const int64_t ir = static_cast<int64_t>(in->shape.size());
    unsigned m = 0;
    for (int64_t d = 0; d < r; ++d) {
        const int64_t di = d - (r - ir);
        if (di >= 0 && in->shape[static_cast<size_t>(di)] == out_shape[static_cast<size_t>(d)])
            m |= 1u << d;
    }
    return m;
}

bool same_shape(const ImplPtr& a, const std::vector<int64_t>& s) { return a->shape == s; }

// A constant-filled operand is read as one element with zero strides instead
// of materializing it (e.g. the reference's full(scores.shape(), scale)).
struct Operand {
    const float* ptr;
    std::vector<int64_t> strides;
    std::shared_ptr<Scratch> holder;
};

Operand operand(const ImplPtr& p, const std::vector<int64_t>& out_shape) {
    Operand o;
    if (p->data && !p->transpose_of && p->data->pending_fill) {
        o.holder = std::make_shared<Scratch>(16);
        check(ttk_fill(o.holder->as<float>(), p->data->fill_value, 1, stream()), "const");
        o.ptr = o.holder->as<float>();
        o.strides.assign(out_shape.size(), 0);
        return o;
    }
    o.ptr = dread(p);
    o.strides = bcast_strides(p, out_shape);
    return o;
}

// dst.grad += src (numel elements), overwriting a still-zero gradient.
void accum_grad(const ImplPtr& dst, const float* src) {
    bool ow = false;
    float* g = grad_target(dst, ow);
    if (ow)
        check(ttk_memcpy_d2d(g, src, static_cast<size_t>(dst->numel) * 4, stream()), "grad copy");
    else
        check(ttk_axpy(1.0f, src, g, dst->numel, stream()), "grad axpy");
}

float* out_ptr(Tensor& t) { return t.impl()->data->device_for_overwrite(); }

// ------------------------------------------------- deferred attention chain --
// bmm(q, transpose(k)) -> mul(., constant) -> add(., causal mask) ->
// softmax(., -1) -> bmm(., v), the attention of model.cpp:133-138. The first
// four results are deferred (no [N, T, T] buffer); the closing bmm runs the
// fused causal attention on q, k, v and the accumulated scale. Any other read
// of a deferred result computes it with the ordinary kernels.

int64_t g_chains_fused = 0;

// Turns the freshly made `out` into a deferred node computed by `fwd`.
void defer(Tensor& out, std::shared_ptr<Deferred> d, std::function<void(Tensor::Impl*)> fwd) {
    d->compute = std::move(fwd);
    out.impl()->data.reset();
    out.impl()->deferred = std::move(d);
}

// A tensor with its own (possibly still lazily filled) storage.
bool plain(const ImplPtr& p) { return p->data && !p->transpose_of && !p->deferred; }

// Constant tensor: a full() that nobody wrote into since.
bool constant_value(const ImplPtr& p, float& v) {
    if (!plain(p) || !p->data->pending_fill || !std::isfinite(p->data->fill_value))
        return false;
    v = p->data->fill_value;
    return true;
}

// [T, T] (or [1, T, T]) holding 0 on and below the diagonal and <= -1e9
// above it (model.cpp:97-101). Under it the composite softmax gives every
// masked entry exactly 0, as the fused kernel's causal skip does. Checked on
// the host mirror once per buffer version.
bool causal_mask(const ImplPtr& m, int64_t T) {
    const auto& sh = m->shape;
    const bool shape_ok = (sh.size() == 2 && sh[0] == T && sh[1] == T) ||
                          (sh.size() == 3 && sh[0] == 1 && sh[1] == T && sh[2] == T);
    if (!shape_ok || !plain(m))
        return false;
    Buffer& b = *m->data;
    if (b.mask_version == b.version)
        return b.causal_mask;
    const float* h = b.host_ptr();
    bool ok = true;
    for (int64_t i = 0; i < T && ok; ++i)
        for (int64_t j = 0; j < T; ++j) {
            const float x = h[i * T + j];
            if (j <= i ? x != 0.0f : !(x <= -1e9f)) {
                ok = false;
                break;
            }
        }
    b.mask_version = b.version;
    b.causal_mask = ok;
    return ok;
}

uint64_t version_of(const ImplPtr& p) {
    if (p->data)
        return p->data->version;
    if (p->transpose_of && p->transpose_of->data)
        return p->transpose_of->data->version;
    return ~0ull;
}

void check_chain_inputs(const Deferred& d) {
    if (version_of(d.q) != d.vq || version_of(d.k) != d.vk)
        throw std::logic_error(
            "attention scores: q or k was modified after bmm(q, transpose(k)) and before its "
            "result was used");
}

// --------------------------------------------------------- elementwise --

Tensor elem_binary(const Tensor& a, const Tensor& b, int op) {
    auto shape = broadcast_shape(a.shape(), b.shape());
    Tensor out = make_out(shape, a.requires_grad() || b.requires_grad());
    std::shared_ptr<Deferred> chain;
    if (const Deferred* d = pending_chain(a.impl());
        d && !d->masked && !d->softmax && shape == a.shape()) {
        float c = 0.0f;
        if (op == 2 && constant_value(b.impl(), c)) {  // scores * scale (model.cpp:134)
            chain = std::make_shared<Deferred>(*d);
            chain->scale = d->scale * c;
        } else if (op == 0 && causal_mask(b.impl(), shape[1])) {  // + mask (model.cpp:135)
            chain = std::make_shared<Deferred>(*d);
            chain->masked = true;
        }
    }
    auto fwd = [ai = a.impl(), bi = b.impl(), shape, op](Tensor::Impl* o) {
        Operand oa = operand(ai, shape), ob = operand(bi, shape);
        check(ttk_binary(op, oa.ptr, oa.strides.data(), ob.ptr, ob.strides.data(),
                         o->data->device_for_overwrite(), shape.data(),
                         static_cast<int>(shape.size()), stream()),
              "binary");
    };
    if (chain)
        defer(out, chain, fwd);
    else
        fwd(out.impl().get());
    if (out.requires_grad()) {
        auto ao = a.impl(), bo = b.impl();
        Tensor::Impl* oo = out.impl().get();  // own node: raw, no cycle
        oo->prev = {ao, bo};
        oo->backward_fn = [ao, bo, oo, shape, op]() {
            const float* g = grad_in(oo);
            if (!g)
                return;
            bool handed = false;  // the output gradient's buffer went to an input
            for (int which = 0; which < 2; ++which) {
                const ImplPtr& X = which ? bo : ao;
                if (!X->requires_grad)
                    continue;
                const bool full = same_shape(X, shape);
                if (full && (op == 0 || (op == 1 && which == 0))) {
                    // d(a+b)/da = d(a+b)/db = d(a-b)/da = 1. The first input
                    // whose gradient is still logically zero takes the output
                    // gradient's buffer itself (this node is its last reader);
                    // any other gets a copy or an accumulation.
                    Buffer* xg = X->grad.get();
                    const bool fresh =
                        !xg || (xg->pending_fill && xg->fill_value == 0.0f && !xg->external);
                    // (numel > 1: never the backward root, whose seed stays.)
                    if (!handed && fresh && !oo->grad->external && oo->grad->n == X->numel &&
                        oo->numel > 1) {
                        X->grad = oo->grad;
                        handed = true;
                        continue;
                    }
                    accum_grad(X, g);
                    continue;
                }
                Operand oa = operand(ao, shape), ob = operand(bo, shape);
                Scratch tmp(static_cast<size_t>(oo->numel) * 4);
                check(ttk_binary_bwd(op, which, oa.ptr, oa.strides.data(), ob.ptr,
                                     ob.strides.data(), g, tmp.as<float>(), shape.data(),
                                     static_cast<int>(shape.size()), stream()),
                      "binary_bwd");
                if (full)
                    accum_grad(X, tmp.as<float>());
                else
                    check(ttk_reduce_to(tmp.as<float>(), shape.data(),
                                        static_cast<int>(shape.size()), keep_mask(X, shape),
                                        grad_rmw(X), 1, stream()),
                          "reduce_to");
            }
        };
    }
    return out;
}

Tensor elem_unary(const Tensor& a, int op, float p = 0.0f) {
    Tensor out = make_out(a.shape(), a.requires_grad());
    check(ttk_unary(op, dread(a.impl()), out_ptr(out), a.numel(), p, stream()), "unary");
    if (out.requires_grad()) {
        auto ao = a.impl();
        Tensor::Impl* oo = out.impl().get();  // own node: raw, no cycle
        oo->prev = {ao};
        oo->backward_fn = [ao, oo, op, p]() {
            const float* g = grad_in(oo);
            if (!g || !ao->requires_grad)
                return;
            check(ttk_unary_bwd(op, dread(ao), g, grad_rmw(ao), ao->numel, p, stream()),
                  "unary_bwd");
        };
    }
    return out;
}

// Matrix operand of a GEMM: storage pointer, transposed flag, row length.
struct MatOp {
    ImplPtr base;   // tensor whose storage is read (the lazy transpose's source)
    const float* ptr;
    int trans;      // 1: the logical matrix is base^T
};

MatOp mat_operand(const ImplPtr& p) {
    if (p->transpose_of && !p->data)
        return {p->transpose_of, dread(p->transpose_of), 1};
    return {p, dread(p), 0};
}

// The split of a GEMM operand stored in `buf` at `ptr` (batch x rows x cols,
// leading dimension ld, batch stride bs), from the buffer's cache when its
// contents and the geometry are unchanged since the last split. The same
// activation is read by the forward GEMM and by dW, the same output gradient
// by dX and dW, and a weight by every micro-batch until the optimizer writes
// it; each is split once.
const void* operand_split(Buffer* buf, const float* ptr, int64_t batch, int64_t rows,
                          int64_t cols, int64_t ld, int64_t bs) {
    const int64_t key[7] = {ptr - buf->dev, batch, rows, cols, ld, bs, ttk_gemm_get_precision()};
    if (buf->split_dev && buf->split_version == buf->version &&
        std::equal(key, key + 7, buf->split_key))
        return buf->split_dev;
    const size_t bytes = ttk_gemm_split_bytes(batch, rows, cols);
    if (buf->split_bytes < bytes) {
        ttk_free(buf->split_dev, stream());
        buf->split_dev = nullptr;
        buf->split_bytes = 0;
        check(ttk_malloc(&buf->split_dev, bytes, stream()), "gemm split");
        buf->split_bytes = bytes;
    }
    check(ttk_gemm_split(ptr, rows, cols, ld, bs, batch, buf->split_dev, stream()), "gemm split");
    buf->split_version = buf->version;
    std::copy(key, key + 7, buf->split_key);
    return buf->split_dev;
}

// GEMM operand: storage buffer, pointer into it, leading dimension and batch
// stride (elements) of the stored (not transposed) matrix.
struct GemmArg {
    Buffer* buf;
    const float* ptr;
    int64_t ld, bs;
};

void gemm(int ta, int tb, int64_t batch, int64_t M, int64_t N, int64_t K, GemmArg A, GemmArg B,
          float beta, float* C, int64_t ldc, int64_t sC) {
    if (M == 0 || N == 0 || batch == 0)
        return;
    // K = 0 (C = beta * C) and small problems (the exact fp32 kernel) take no
    // operand split.
    if (K == 0 || ttk_gemm_uses_fp32(batch, M, N, K)) {
        check(ttk_gemm(ta, tb, batch, M, N, K, 1.0f, A.ptr, A.ld, A.bs, B.ptr, B.ld, B.bs, beta, C,
                       ldc, sC, nullptr, 0, stream()),
              "gemm");
        return;
    }
    const void* sa = operand_split(A.buf, A.ptr, batch, ta ? K : M, ta ? M : K, A.ld, A.bs);
    const int64_t brows = tb ? N : K, bcols = tb ? K : N;
    const void* sb = nullptr;
    std::unique_ptr<Scratch> own;  // both operands in one buffer, other geometry: B uncached
    const int64_t bkey[7] = {B.ptr - B.buf->dev, batch, brows, bcols, B.ld, B.bs,
                             ttk_gemm_get_precision()};
    if (B.buf == A.buf && !std::equal(bkey, bkey + 7, A.buf->split_key)) {
        own = std::make_unique<Scratch>(ttk_gemm_split_bytes(batch, brows, bcols));
        check(ttk_gemm_split(B.ptr, brows, bcols, B.ld, B.bs, batch, own->ptr, stream()),
              "gemm split");
        sb = own->ptr;
    } else {
        sb = operand_split(B.buf, B.ptr, batch, brows, bcols, B.ld, B.bs);
    }
    check(ttk_gemm_splits(ta, tb, batch, M, N, K, 1.0f, sa, sb, beta, C, ldc, sC, stream()),
          "gemm");
}

// The buffer holding an operand's storage: the tensor's data, or a gradient.
GemmArg data_arg(Tensor::Impl* p, int64_t ld, int64_t bs) {
    const float* d = dread(p);
    return {p->data.get(), d, ld, bs};
}

}  // namespace

Tensor add(const Tensor& a, const Tensor& b) { return elem_binary(a, b, 0); }
Tensor sub(const Tensor& a, const Tensor& b) { return elem_binary(a, b, 1); }
Tensor mul(const Tensor& a, const Tensor& b) { return elem_binary(a, b, 2); }
Tensor div(const Tensor& a, const Tensor& b) { return elem_binary(a, b, 3); }
Tensor neg(const Tensor& a) { return elem_unary(a, 0); }

Tensor exp(const Tensor& a) { return elem_unary(a, 1); }
Tensor log(const Tensor& a) { return elem_unary(a, 2); }
Tensor sqrt(const Tensor& a) { return elem_unary(a, 3); }
Tensor tanh(const Tensor& a) { return elem_unary(a, 4); }
Tensor silu(const Tensor& a) { return elem_unary(a, 5); }
Tensor sin(const Tensor& a) { return elem_unary(a, 6); }
Tensor cos(const Tensor& a) { return elem_unary(a, 7); }
Tensor pow(const Tensor& a, float p) { return elem_unary(a, 8, p); }

// ----------------------------------------------------------- reductions --

Tensor sum(const Tensor& a, int64_t dim, bool keepdim) {
    dim = norm_dim(dim, a.ndim());
    std::vector<int64_t> oshape;
    int64_t outer = 1, inner = 1;
    for (int64_t d = 0; d < a.ndim(); ++d) {
        if (d < dim)
            outer *= a.dim(d);
        if (d > dim)
            inner *= a.dim(d);
        if (d == dim) {
            if (keepdim)
                oshape.push_back(1);
        } else {
            oshape.push_back(a.dim(d));
        }
    }
    if (oshape.empty())
        oshape.push_back(1);
    const int64_t K = a.dim(dim);
    Tensor out = make_out(oshape, a.requires_grad());
    check(ttk_reduce_mid(dread(a.impl()), out_ptr(out), outer, K, inner, 0, stream()), "sum");
    if (out.requires_grad()) {
        auto ao = a.impl();
        Tensor::Impl* oo = out.impl().get();  // own node: raw, no cycle
        oo->prev = {ao};
        oo->backward_fn = [ao, oo, outer, K, inner]() {
            const float* g = grad_in(oo);
            if (!g || !ao->requires_grad)
                return;
            const int64_t shp[3] = {outer, K, inner};
            const int64_t st[3] = {inner, 0, 1};
            check(ttk_strided_copy(g, st, grad_rmw(ao), shp, 3, 1, 0, stream()), "sum bwd");
        };
    }
    return out;
}

Tensor sum_all(const Tensor& a) {
    Tensor out = make_out({1}, a.requires_grad());
    check(ttk_sum_all(dread(a.impl()), a.numel(), out_ptr(out), 0, stream()), "sum_all");
    if (out.requires_grad()) {
        auto ao = a.impl();
        Tensor::Impl* oo = out.impl().get();  // own node: raw, no cycle
        oo->prev = {ao};
        oo->backward_fn = [ao, oo]() {
            const float* g = grad_in(oo);
            if (!g || !ao->requires_grad)
                return;
            const int64_t shp[1] = {ao->numel};
            const int64_t st[1] = {0};
            check(ttk_strided_copy(g, st, grad_rmw(ao), shp, 1, 1, 0, stream()), "sum_all bwd");
        };
    }
    return out;
}

Tensor mean(const Tensor& a) {
    // The reference's mean is sum_all followed by a division by numel whose
    // backward is og / numel (ops.cpp:462-479): the same as div by a constant.
    return div(sum_all(a), full({1}, static_cast<float>(a.numel())));
}

// ---------------------------------------------------------------- shape --

Tensor reshape(const Tensor& a, const std::vector<int64_t>& shape) {
    int64_t n = 1;
    int64_t infer = -1;
    for (size_t i = 0; i < shape.size(); ++i) {
        if (shape[i] == -1) {
            if (infer != -1)
                throw std::invalid_argument("reshape: only one -1 allowed");
            infer = static_cast<int64_t>(i);
        } else {
            if (shape[i] <= 0)
                throw std::invalid_argument("reshape: dims must be positive");
            n *= shape[i];
        }
    }
    std::vector<int64_t> out_shape = shape;
    if (infer != -1) {
        if (a.numel() % n != 0)
            throw std::invalid_argument("reshape: incompatible size");
        out_shape[static_cast<size_t>(infer)] = a.numel() / n;
        n = a.numel();
    }
    if (n != a.numel() || out_shape.empty())
        throw std::invalid_argument("reshape: incompatible size");
    Tensor out = make_view(a, out_shape, a.requires_grad());
    if (out.requires_grad()) {
        auto ao = a.impl();
        Tensor::Impl* oo = out.impl().get();  // own node: raw, no cycle
        oo->prev = {ao};
        oo->backward_fn = [ao, oo]() {
            const float* g = grad_in(oo);
            if (!g || !ao->requires_grad)
                return;
            // The view's gradient has the input's size and element order: when
            // the input's gradient is still logically zero, hand over the
            // buffer itself (with any operand split cached on it) instead of
            // copying it. The view's own reference is dropped once this node
            // has run, so the buffer then belongs to the input alone (a scalar
            // view may be the backward root, whose seed stays: copied).
            Buffer* ig = ao->grad.get();
            const bool fresh = !ig || (ig->pending_fill && ig->fill_value == 0.0f && !ig->external);
            if (fresh && !oo->grad->external && oo->grad->n == ao->numel && oo->numel > 1) {
                ao->grad = oo->grad;
                return;
            }
            accum_grad(ao, g);
        };
    }
    return out;
}

Tensor transpose(const Tensor& a, int64_t d0, int64_t d1) {
    d0 = norm_dim(d0, a.ndim());
    d1 = norm_dim(d1, a.ndim());
    std::vector<int64_t> dims(static_cast<size_t>(a.ndim()));
    for (int64_t d = 0; d < a.ndim(); ++d)
        dims[static_cast<size_t>(d)] = d;
    std::swap(dims[static_cast<size_t>(d0)], dims[static_cast<size_t>(d1)]);
    return permute(a, dims);
}

Tensor permute(const Tensor& a, const std::vector<int64_t>& dims) {
    const int64_t rank = a.ndim();
    if (static_cast<int64_t>(dims.size()) != rank)
        throw std::invalid_argument("permute: rank mismatch");
    std::vector<int64_t> oshape(static_cast<size_t>(rank)), src(static_cast<size_t>(rank));
    std::vector<bool> seen(static_cast<size_t>(rank), false);
    for (int64_t d = 0; d < rank; ++d) {
        const int64_t s = norm_dim(dims[static_cast<size_t>(d)], rank);
        if (seen[static_cast<size_t>(s)])
            throw std::invalid_argument("permute: repeated dim");
        seen[static_cast<size_t>(s)] = true;
        src[static_cast<size_t>(d)] = s;
        oshape[static_cast<size_t>(d)] = a.dim(s);
    }
    auto ao = a.impl();
    // Swap of the last two dims of a 2-D or 3-D tensor: lazy (read by
    // matmul/bmm as a transposed operand, materialized only if needed).
    const bool lazy = (rank == 2 || rank == 3) && src[static_cast<size_t>(rank - 1)] == rank - 2 &&
                      src[static_cast<size_t>(rank - 2)] == rank - 1 && (rank == 2 || src[0] == 0) &&
                      !ao->transpose_of;
    Tensor out;
    // Element strides of the source, listed in output dim order.
    std::vector<int64_t> in_strides(static_cast<size_t>(rank));
    for (int64_t d = 0; d < rank; ++d)
        in_strides[static_cast<size_t>(d)] = ao->strides[static_cast<size_t>(src[static_cast<size_t>(d)])];
    if (lazy) {
        auto impl = std::make_shared<Tensor::Impl>();
        impl->shape = oshape;
        impl->strides = row_major(oshape);
        impl->numel = a.numel();
        impl->transpose_of = ao;
        impl->requires_grad = a.requires_grad();
        out = Tensor::from_impl(impl);
    } else {
        out = make_out(oshape, a.requires_grad());
        check(ttk_strided_copy(dread(ao), in_strides.data(), out_ptr(out), oshape.data(),
                               static_cast<int>(rank), 0, 0, stream()),
              "permute");
    }
    if (out.requires_grad()) {
        Tensor::Impl* oo = out.impl().get();  // own node: raw, no cycle
        oo->prev = {ao};
        oo->backward_fn = [ao, oo, in_strides]() {
            const float* g = grad_in(oo);
            if (!g || !ao->requires_grad)
                return;
            // permute backward: scatter the gradient back through the same
            // (bijective) index map.
            check(ttk_strided_copy(g, in_strides.data(), grad_rmw(ao), oo->shape.data(),
                                   static_cast<int>(oo->shape.size()), 1, 1, stream()),
                  "permute bwd");
        };
    }
    return out;
}

Tensor expand(const Tensor& a, const std::vector<int64_t>& shape) {
    (void)broadcast_shape(a.shape(), shape);
    const int64_t ar = a.ndim(), r = static_cast<int64_t>(shape.size());
    if (r < ar)
        throw std::invalid_argument("expand: incompatible shape");
    for (int64_t i = 0; i < r; ++i) {
        const int64_t ad = (i < r - ar) ? 1 : a.dim(i - (r - ar));
        if (ad != 1 && ad != shape[static_cast<size_t>(i)])
            throw std::invalid_argument("expand: incompatible shape");
    }
    Tensor out = make_out(shape, a.requires_grad());
    auto ao = a.impl();
    auto st = bcast_strides(ao, shape);
    check(ttk_strided_copy(dread(ao), st.data(), out_ptr(out), shape.data(), static_cast<int>(r),
                           0, 0, stream()),
          "expand");
    if (out.requires_grad()) {
        Tensor::Impl* oo = out.impl().get();  // own node: raw, no cycle
        oo->prev = {ao};
        oo->backward_fn = [ao, oo, shape]() {
            const float* g = grad_in(oo);
            if (!g || !ao->requires_grad)
                return;
            check(ttk_reduce_to(g, shape.data(), static_cast<int>(shape.size()),
                                keep_mask(ao, shape), grad_rmw(ao), 1, stream()),
                  "expand bwd");
        };
    }
    return out;
}

Tensor squeeze(const Tensor& a, int64_t dim) {
    dim = norm_dim(dim, a.ndim());
    if (a.dim(dim) != 1)
        throw std::invalid_argument("squeeze: dim size != 1");
    std::vector<int64_t> oshape;
    for (int64_t d = 0; d < a.ndim(); ++d)
        if (d != dim)
            oshape.push_back(a.dim(d));
    if (oshape.empty())
        oshape.push_back(1);
    return reshape(a, oshape);
}

Tensor unsqueeze(const Tensor& a, int64_t dim) {
    const int64_t rank = a.ndim() + 1;
    if (dim < 0)
        dim += rank;
    if (dim < 0 || dim > a.ndim())
        throw std::invalid_argument("unsqueeze: dim out of range");
    std::vector<int64_t> oshape;
    for (int64_t d = 0; d < a.ndim(); ++d) {
        if (d == dim)
            oshape.push_back(1);
        oshape.push_back(a.dim(d));
    }
    if (dim == a.ndim())
        oshape.push_back(1);
    return reshape(a, oshape);
}

// ------------------------------------------------------- linear algebra --

namespace {

Tensor fused_attention(const ImplPtr& qo, const ImplPtr& ko, const ImplPtr& vo, ImplPtr co,
                       ImplPtr so, int64_t B, int64_t T, int64_t H, int64_t hd, float scale,
                       std::vector<int64_t> oshape, bool planes = false);

// C (batch x [M,N]) = op(A) op(B) and its backward, for matmul and bmm. A is
// [M,K] (storage [K,M] when A.trans), B is [K,N] (storage [N,K] when B.trans).
Tensor batched_matmul(const Tensor& a, const Tensor& b, int64_t Bt, int64_t M, int64_t K,
                      int64_t N, std::vector<int64_t> oshape,
                      std::shared_ptr<Deferred> chain = nullptr) {
    Tensor out = make_out(oshape, a.requires_grad() || b.requires_grad());
    auto fwd = [ai = a.impl(), bi = b.impl(), Bt, M, K, N, chain](Tensor::Impl* o) {
        if (chain)
            check_chain_inputs(*chain);
        MatOp A = mat_operand(ai), Bm = mat_operand(bi);
        const int64_t lda = A.trans ? M : K, ldb = Bm.trans ? K : N;
        gemm(A.trans, Bm.trans, Bt, M, N, K, {A.base->data.get(), A.ptr, lda, M * K},
             {Bm.base->data.get(), Bm.ptr, ldb, K * N}, 0.0f, o->data->device_for_overwrite(),
             N, M * N);
    };
    if (chain)
        defer(out, chain, fwd);
    else
        fwd(out.impl().get());
    if (out.requires_grad()) {
        auto ao = a.impl(), bo = b.impl();
        Tensor::Impl* oo = out.impl().get();  // own node: raw, no cycle
        oo->prev = {ao, bo};
        oo->backward_fn = [ao, bo, oo, Bt, M, K, N]() {
            const float* g = grad_in(oo);
            if (!g)
                return;
            MatOp A = mat_operand(ao), Bm = mat_operand(bo);
            const int64_t lda = A.trans ? M : K, ldb = Bm.trans ? K : N;
            const GemmArg ga{oo->grad.get(), g, N, M * N};
            const GemmArg aa{A.base->data.get(), A.ptr, lda, M * K};
            const GemmArg ba{Bm.base->data.get(), Bm.ptr, ldb, K * N};
            if (ao->requires_grad) {
                // dA = g B^T. For a lazy transpose A = X^T the gradient goes
                // straight into X: dX = B g^T.
                bool ow = false;
                if (!A.trans) {
                    float* d = grad_target(ao, ow);
                    gemm(0, Bm.trans ? 0 : 1, Bt, M, K, N, ga, ba, ow ? 0.0f : 1.0f, d, K, M * K);
                } else if (A.base->requires_grad) {
                    float* d = grad_target(A.base, ow);
                    gemm(Bm.trans ? 1 : 0, 1, Bt, K, M, N, ba, ga, ow ? 0.0f : 1.0f, d, M, M * K);
                }
            }
            if (bo->requires_grad) {
                // dB = A^T g. For B = W^T: dW = g^T A.
                bool ow = false;
                if (!Bm.trans) {
                    float* d = grad_target(bo, ow);
                    gemm(A.trans ? 0 : 1, 0, Bt, K, N, M, aa, ga, ow ? 0.0f : 1.0f, d, N, K * N);
                } else if (Bm.base->requires_grad) {
                    float* d = grad_target(Bm.base, ow);
                    gemm(1, A.trans ? 1 : 0, Bt, N, K, M, ga, aa, ow ? 0.0f : 1.0f, d, K, K * N);
                }
            }
        };
    }
    return out;
}

}  // namespace

Tensor matmul(const Tensor& a, const Tensor& b) {
    if (a.ndim() != 2 || b.ndim() != 2)
        throw std::invalid_argument("matmul: both inputs must be 2D");
    const int64_t M = a.dim(0), K = a.dim(1), K2 = b.dim(0), N = b.dim(1);
    if (K != K2)
        throw std::invalid_argument("matmul: inner dims mismatch");
    return batched_matmul(a, b, 1, M, K, N, {M, N});
}

Tensor bmm(const Tensor& a, const Tensor& b) {
    if (a.ndim() != 3 || b.ndim() != 3)
        throw std::invalid_argument("bmm: both inputs must be 3D");
    const int64_t B = a.dim(0), M = a.dim(1), K = a.dim(2);
    if (b.dim(0) != B || b.dim(1) != K)
        throw std::invalid_argument("bmm: batch/inner dims mismatch");
    const int64_t N = b.dim(2);
    // probs @ v closing a deferred causal chain (model.cpp:138): fused.
    if (const Deferred* d = pending_chain(a.impl());
        d && d->masked && d->softmax && plain(b.impl()) && b.shape() == d->q->shape) {
        check_chain_inputs(*d);
        ++g_chains_fused;
        return fused_attention(d->q, d->k, b.impl(), nullptr, nullptr, B, M, 1, N, d->scale,
                               {B, M, N});
    }
    // q @ k^T of an attention block (model.cpp:133): deferred.
    const ImplPtr& bi = b.impl();
    if (plain(a.impl()) && bi->transpose_of && !bi->data && plain(bi->transpose_of) &&
        bi->transpose_of->shape == a.shape() && M == N && (K == 32 || K == 64 || K == 128) &&
        B <= 65535) {
        auto d = std::make_shared<Deferred>();
        d->q = a.impl();
        d->k = bi->transpose_of;
        d->vq = version_of(d->q);
        d->vk = version_of(d->k);
        return batched_matmul(a, b, B, M, K, N, {B, M, N}, d);
    }
    return batched_matmul(a, b, B, M, K, N, {B, M, N});
}

int64_t fused_attention_chains() { return g_chains_fused; }

Tensor linear(const Tensor& x, const Tensor& weight) {
    if (x.ndim() != 2 || weight.ndim() != 2)
        throw std::invalid_argument("linear: x and weight must be 2D");
    if (x.dim(1) != weight.dim(1))
        throw std::invalid_argument("matmul: inner dims mismatch");
    const int64_t R = x.dim(0), In = x.dim(1), Out = weight.dim(0);
    Tensor out = make_out({R, Out}, x.requires_grad() || weight.requires_grad());
    gemm(0, 1, 1, R, Out, In, data_arg(x.impl().get(), In, 0), data_arg(weight.impl().get(), In, 0),
         0.0f, out_ptr(out), Out, 0);
    if (out.requires_grad()) {
        auto xo = x.impl(), wo = weight.impl();
        Tensor::Impl* oo = out.impl().get();  // own node: raw, no cycle
        oo->prev = {xo, wo};
        oo->backward_fn = [xo, wo, oo, R, In, Out]() {
            const float* g = grad_in(oo);
            if (!g)
                return;
            const GemmArg ga{oo->grad.get(), g, Out, 0};
            if (xo->requires_grad) {  // dX = g W
                bool ow = false;
                float* d = grad_target(xo, ow);
                gemm(0, 0, 1, R, In, Out, ga, data_arg(wo.get(), In, 0), ow ? 0.0f : 1.0f, d, In,
                     0);
            }
            if (wo->requires_grad) {  // dW = g^T X
                bool ow = false;
                float* d = grad_target(wo, ow);
                gemm(1, 0, 1, Out, In, R, ga, data_arg(xo.get(), In, 0), ow ? 0.0f : 1.0f, d, In,
                     0);
            }
        };
    }
    return out;
}

// out = linear(swiglu(linear(x, w_gate), linear(x, w_up)), w_down) with the
// activation y = silu(x W_g^T) * (x W_u^T) and its gradients dA, dB held only
// as bf16x3 operand planes (ttk_swiglu_*_split): the projection GEMMs take
// them through ttk_gemm_splits, and the fp32 y, dA and dB of the composed ops
// never exist. The planes equal the split of those fp32 tensors, so every
// result equals the composition's bit for bit. The composition runs instead
// when the operands are not in the bf16x3 precision, when a projection is
// small enough for the exact fp32 GEMM, or when TT_FUSED_FFN=0.
Tensor ffn_swiglu(const Tensor& x, const Tensor& w_gate, const Tensor& w_up,
                  const Tensor& w_down) {
    if (x.ndim() != 2 || w_gate.ndim() != 2 || w_up.ndim() != 2 || w_down.ndim() != 2)
        throw std::invalid_argument("ffn_swiglu: x and weights must be 2D");
    const int64_t R = x.dim(0), d = x.dim(1), F = w_gate.dim(0);
    if (w_gate.dim(1) != d || w_up.dim(0) != F || w_up.dim(1) != d || w_down.dim(0) != d ||
        w_down.dim(1) != F)
        throw std::invalid_argument("ffn_swiglu: weight shapes do not match");
    const char* env = std::getenv("TT_FUSED_FFN");
    const bool fused = !(env && env[0] == '0') && ttk_gemm_get_precision() == 0 && F % 4 == 0 &&
                       !ttk_gemm_uses_fp32(1, R, F, d) && !ttk_gemm_uses_fp32(1, R, d, F) &&
                       !ttk_gemm_uses_fp32(1, F, d, R) && !ttk_gemm_uses_fp32(1, d, F, R);
    if (!fused)
        return linear(swiglu(linear(x, w_gate), linear(x, w_up)), w_down);
    const bool rg = x.requires_grad() || w_gate.requires_grad() || w_up.requires_grad() ||
                    w_down.requires_grad();
    // a, b: the projections, kept in fp32 for the backward (not graph nodes)
    Tensor a = make_out({R, F}, false), b = make_out({R, F}, false);
    gemm(0, 1, 1, R, F, d, data_arg(x.impl().get(), d, 0), data_arg(w_gate.impl().get(), d, 0),
         0.0f, out_ptr(a), F, 0);
    gemm(0, 1, 1, R, F, d, data_arg(x.impl().get(), d, 0), data_arg(w_up.impl().get(), d, 0),
         0.0f, out_ptr(b), F, 0);
    const size_t split_bytes = ttk_gemm_split_bytes(1, R, F);
    auto ys = std::make_shared<Scratch>(split_bytes);
    check(ttk_swiglu_fwd_split(dread(a.impl()), dread(b.impl()), ys->ptr, R, F, stream()),
          "ffn swiglu");
    Tensor out = make_out({R, d}, rg);
    {
        const GemmArg wd = data_arg(w_down.impl().get(), F, 0);
        const void* wds = operand_split(wd.buf, wd.ptr, 1, d, F, F, 0);
        check(ttk_gemm_splits(0, 1, 1, R, d, F, 1.0f, ys->ptr, wds, 0.0f, out_ptr(out), d, 0,
                              stream()),
              "ffn down");
    }
    if (rg) {
        auto xo = x.impl(), go = w_gate.impl(), uo = w_up.impl(), wo = w_down.impl();
        auto ao = a.impl(), bo = b.impl();
        Tensor::Impl* oo = out.impl().get();  // own node: raw, no cycle
        oo->prev = {xo, go, uo, wo};
        oo->backward_fn = [xo, go, uo, wo, ao, bo, oo, ys, R, d, F, split_bytes]() {
            const float* g = grad_in(oo);
            if (!g)
                return;
            const GemmArg ga{oo->grad.get(), g, d, 0};
            // dY = dOut W_d  [R, F]
            Scratch dy(static_cast<size_t>(R * F) * 4);
            gemm(0, 0, 1, R, F, d, ga, data_arg(wo.get(), F, 0), 0.0f, dy.as<float>(), F, 0);
            if (wo->requires_grad) {  // dW_d = dOut^T Y  [d, F]
                bool ow = false;
                float* gw = grad_target(wo, ow);
                const void* gs = operand_split(ga.buf, ga.ptr, 1, R, d, d, 0);
                check(ttk_gemm_splits(1, 0, 1, d, F, R, 1.0f, gs, ys->ptr, ow ? 0.0f : 1.0f, gw,
                                      F, 0, stream()),
                      "ffn dW down");
            }
            if (!(xo->requires_grad || go->requires_grad || uo->requires_grad))
                return;
            Scratch das(split_bytes), dbs(split_bytes);
            check(ttk_swiglu_bwd_split(dread(ao), dread(bo), dy.as<float>(), das.ptr, dbs.ptr, R,
                                       F, stream()),
                  "ffn swiglu bwd");
            if (xo->requires_grad) {  // dX = dA W_g + dB W_u  [R, d]
                bool ow = false;
                float* gx = grad_target(xo, ow);
                const GemmArg wg = data_arg(go.get(), d, 0), wu = data_arg(uo.get(), d, 0);
                const void* wgs = operand_split(wg.buf, wg.ptr, 1, F, d, d, 0);
                check(ttk_gemm_splits(0, 0, 1, R, d, F, 1.0f, das.ptr, wgs, ow ? 0.0f : 1.0f, gx,
                                      d, 0, stream()),
                      "ffn dX");
                const void* wus = operand_split(wu.buf, wu.ptr, 1, F, d, d, 0);
                check(ttk_gemm_splits(0, 0, 1, R, d, F, 1.0f, dbs.ptr, wus, 1.0f, gx, d, 0,
                                      stream()),
                      "ffn dX");
            }
            if (go->requires_grad || uo->requires_grad) {  // dW_g = dA^T X, dW_u = dB^T X
                const GemmArg xa = data_arg(xo.get(), d, 0);
                const void* xs = operand_split(xa.buf, xa.ptr, 1, R, d, d, 0);
                if (go->requires_grad) {
                    bool ow = false;
                    float* gw = grad_target(go, ow);
                    check(ttk_gemm_splits(1, 0, 1, F, d, R, 1.0f, das.ptr, xs, ow ? 0.0f : 1.0f,
                                          gw, d, 0, stream()),
                          "ffn dW gate");
                }
                if (uo->requires_grad) {
                    bool ow = false;
                    float* gw = grad_target(uo, ow);
                    check(ttk_gemm_splits(1, 0, 1, F, d, R, 1.0f, dbs.ptr, xs, ow ? 0.0f : 1.0f,
                                          gw, d, 0, stream()),
                          "ffn dW up");
                }
            }
        };
    }
    return out;
}

// ---------------------------------------------------------- neural nets --

DeviceIds::DeviceIds(const std::vector<int64_t>& host) : DeviceIds(host.data(),
                                                                    static_cast<int64_t>(host.size())) {}

DeviceIds::DeviceIds(const int64_t* host, int64_t n_) : n(n_) {
    if (n <= 0)
        return;
    auto s = std::make_shared<Scratch>(static_cast<size_t>(n) * 8);
    check(ttk_memcpy_h2d(s->ptr, host, static_cast<size_t>(n) * 8, stream()), "ids upload");
    dev = s->as<int64_t>();
    buf = std::shared_ptr<void>(s, s->ptr);
}

DeviceIds DeviceIds::borrow(const int64_t* d, int64_t n) {
    DeviceIds ids;
    ids.dev = d;
    ids.n = n;
    return ids;
}

const int64_t* DeviceIds::data() const { return dev; }

Tensor embedding(const Tensor& weight, const std::vector<int64_t>& idx) {
    const int64_t V = weight.dim(0);
    for (int64_t t : idx)
        if (t < 0 || t >= V)
            throw std::invalid_argument("embedding: index out of range");
    return embedding(weight, DeviceIds(idx));
}

Tensor embedding(const Tensor& weight, const DeviceIds& idx) {
    if (weight.ndim() != 2)
        throw std::invalid_argument("embedding: weight must be 2D");
    const int64_t V = weight.dim(0), D = weight.dim(1), N = idx.size();
    if (N <= 0)
        throw std::invalid_argument("Tensor: dims must be positive");
    Tensor out = make_out({N, D}, weight.requires_grad());
    check(ttk_embedding_fwd(dread(weight.impl()), idx.data(), out_ptr(out), N, D, V, stream()),
          "embedding");
    if (out.requires_grad()) {
        auto wo = weight.impl();
        Tensor::Impl* oo = out.impl().get();  // own node: raw, no cycle
        oo->prev = {wo};
        oo->backward_fn = [wo, oo, idx, N, D, V]() {
            const float* g = grad_in(oo);
            if (!g || !wo->requires_grad)
                return;
            const size_t ws = ttk_embedding_bwd_workspace_size(N);
            Scratch w(ws);
            check(ttk_embedding_bwd(g, idx.data(), grad_rmw(wo), N, D, V, w.ptr, ws, stream()),
                  "embedding bwd");
        };
    }
    return out;
}

namespace {

Tensor softmax_impl(const Tensor& a, int64_t dim, int log) {
    dim = norm_dim(dim, a.ndim());
    if (dim != a.ndim() - 1) {
        // Move `dim` last, apply, move it back (autograd flows through).
        std::vector<int64_t> p(static_cast<size_t>(a.ndim()));
        for (int64_t d = 0; d < a.ndim(); ++d)
            p[static_cast<size_t>(d)] = d;
        std::swap(p[static_cast<size_t>(dim)], p[static_cast<size_t>(a.ndim() - 1)]);
        Tensor moved = permute(a, p);
        Tensor r = softmax_impl(moved, -1, log);
        return permute(r, p);
    }
    const int64_t C = a.dim(a.ndim() - 1), R = a.numel() / C;
    Tensor out = make_out(a.shape(), a.requires_grad());
    auto fwd = [ai = a.impl(), R, C, log](Tensor::Impl* o) {
        check(ttk_softmax_fwd(dread(ai), o->data->device_for_overwrite(), R, C, log, stream()),
              "softmax");
    };
    const Deferred* d = pending_chain(a.impl());
    if (d && d->masked && !d->softmax && !log) {  // softmax(masked scores) (model.cpp:136)
        auto chain = std::make_shared<Deferred>(*d);
        chain->softmax = true;
        defer(out, chain, fwd);
    } else {
        fwd(out.impl().get());
    }
    if (out.requires_grad()) {
        auto ao = a.impl();
        Tensor::Impl* oo = out.impl().get();  // own node: raw, no cycle
        oo->prev = {ao};
        oo->backward_fn = [ao, oo, R, C, log]() {
            const float* g = grad_in(oo);
            if (!g || !ao->requires_grad)
                return;
            bool ow = false;
            float* d = grad_target(ao, ow);
            check(ttk_softmax_bwd(dread(oo), g, d, ow ? 0 : 1, R, C, log, stream()),
                  "softmax bwd");
        };
    }
    return out;
}

void check_targets(const std::vector<int64_t>& targets, int64_t N, int64_t C, const char* who) {
    if (static_cast<int64_t>(targets.size()) != N)
        throw std::invalid_argument(std::string(who) + ": targets size mismatch");
    for (int64_t t : targets)
        if (t < 0 || t >= C)
            throw std::invalid_argument(std::string(who) + ": target out of range");
}

}  // namespace

Tensor softmax(const Tensor& a, int64_t dim) { return softmax_impl(a, dim, 0); }
Tensor log_softmax(const Tensor& a, int64_t dim) { return softmax_impl(a, dim, 1); }

Tensor nll_loss(const Tensor& log_probs, const std::vector<int64_t>& targets) {
    if (log_probs.ndim() != 2)
        throw std::invalid_argument("nll_loss: log_probs must be 2D");
    const int64_t N = log_probs.dim(0), C = log_probs.dim(1);
    check_targets(targets, N, C, "nll_loss");
    DeviceIds ids(targets);
    Tensor out = make_out({1}, log_probs.requires_grad());
    check(ttk_nll_fwd(dread(log_probs.impl()), ids.data(), N, C, out_ptr(out), stream()), "nll");
    if (out.requires_grad()) {
        auto lo = log_probs.impl();
        Tensor::Impl* oo = out.impl().get();  // own node: raw, no cycle
        oo->prev = {lo};
        oo->backward_fn = [lo, oo, ids, N, C]() {
            const float* g = grad_in(oo);
            if (!g || !lo->requires_grad)
                return;
            check(ttk_nll_bwd(ids.data(), N, C, g, grad_rmw(lo), stream()), "nll bwd");
        };
    }
    return out;
}

Tensor cross_entropy(const Tensor& logits, const std::vector<int64_t>& targets) {
    if (logits.ndim() != 2)
        throw std::invalid_argument("nll_loss: log_probs must be 2D");
    check_targets(targets, logits.dim(0), logits.dim(1), "nll_loss");
    return cross_entropy(logits, DeviceIds(targets));
}

Tensor cross_entropy(const Tensor& logits, const DeviceIds& targets) {
    if (logits.ndim() != 2)
        throw std::invalid_argument("nll_loss: log_probs must be 2D");
    const int64_t N = logits.dim(0), C = logits.dim(1);
    if (targets.size() != N)
        throw std::invalid_argument("nll_loss: targets size mismatch");
    Tensor out = make_out({1}, logits.requires_grad());
    Scratch acc(8);
    check(ttk_memset(acc.ptr, 0, 8, stream()), "ce zero");
    // The gradient for d(loss) = 1 is produced in the same pass (the row is
    // still in registers) and kept for the backward.
    std::shared_ptr<Buffer> dlog;
    if (logits.requires_grad())
        dlog = std::make_shared<Buffer>(N * C);
    const float inv_n = 1.0f / static_cast<float>(N);
    check(ttk_cross_entropy(dread(logits.impl()), targets.data(), N, C, acc.as<double>(),
                            dlog ? dlog->device_for_overwrite() : nullptr, inv_n, stream()),
          "cross_entropy");
    check(ttk_loss_finalize(acc.as<double>(), inv_n, out_ptr(out), stream()), "loss");
    if (out.requires_grad()) {
        auto lo = logits.impl();
        Tensor::Impl* oo = out.impl().get();  // own node: raw, no cycle
        oo->prev = {lo};
        oo->backward_fn = [lo, oo, dlog, N, C]() {
            if (!oo->grad || !lo->requires_grad)
                return;
            Buffer& og = *oo->grad;
            const bool unit = og.pending_fill && og.fill_value == 1.0f;
            if (unit && (!lo->grad || (lo->grad->pending_fill && lo->grad->fill_value == 0.0f))) {
                lo->grad = dlog;  // adopt the precomputed gradient, no copy
                return;
            }
            bool ow = false;
            float* d = grad_target(lo, ow);
            if (unit) {
                if (ow)
                    check(ttk_memcpy_d2d(d, dlog->device(), static_cast<size_t>(N * C) * 4,
                                         stream()),
                          "ce grad copy");
                else
                    check(ttk_axpy(1.0f, dlog->device(), d, N * C, stream()), "ce grad");
            } else {
                check(ttk_axpy_dev(og.device(), dlog->device(), d, N * C, ow ? 0 : 1, stream()),
                      "ce grad scale");
            }
        };
    }
    return out;
}

Tensor rmsnorm(const Tensor& a, const Tensor& weight, float eps) {
    const int64_t D = a.dim(a.ndim() - 1);
    if (weight.ndim() != 1 || weight.dim(0) != D)
        throw std::invalid_argument("broadcast: incompatible shapes");
    const int64_t R = a.numel() / D;
    Tensor out = make_out(a.shape(), a.requires_grad() || weight.requires_grad());
    auto rstd = std::make_shared<Buffer>(R);
    // Outputs large enough to feed tensor-core GEMMs get their bf16x3 operand
    // planes from the same kernel, cached on the output buffer as a GEMM
    // operand split of [R, D] rows (what linear() looks up): the projections
    // that read the output skip their split pass. Same planes, same results.
    const bool planes = D % 256 == 0 && R * D >= (1 << 20) && ttk_gemm_get_precision() == 0;
    if (planes) {
        float* y = out_ptr(out);
        Buffer& ob = *out.impl()->data;
        const size_t bytes = ttk_gemm_split_bytes(1, R, D);
        if (ob.split_bytes < bytes) {
            ttk_free(ob.split_dev, stream());
            ob.split_dev = nullptr;
            ob.split_bytes = 0;
            check(ttk_malloc(&ob.split_dev, bytes, stream()), "rmsnorm planes");
            ob.split_bytes = bytes;
        }
        check(ttk_rmsnorm_fwd_split(dread(a.impl()), dread(weight.impl()), y,
                                    rstd->device_for_overwrite(), R, D, eps, ob.split_dev,
                                    stream()),
              "rmsnorm");
        const int64_t key[7] = {0, 1, R, D, D, 0, 0};
        ob.split_version = ob.version;
        std::copy(key, key + 7, ob.split_key);
    } else {
        check(ttk_rmsnorm_fwd(dread(a.impl()), dread(weight.impl()), out_ptr(out),
                              rstd->device_for_overwrite(), R, D, eps, stream()),
              "rmsnorm");
    }
    if (out.requires_grad()) {
        auto ao = a.impl(), wo = weight.impl();
        Tensor::Impl* oo = out.impl().get();  // own node: raw, no cycle
        oo->prev = {ao, wo};
        oo->backward_fn = [ao, wo, oo, rstd, R, D]() {
            const float* g = grad_in(oo);
            if (!g)
                return;
            bool ow = false;
            float* dx = ao->requires_grad ? grad_target(ao, ow) : nullptr;
            float* dw = wo->requires_grad ? grad_rmw(wo) : nullptr;
            const size_t ws = ttk_rmsnorm_bwd_workspace_size(R, D);
            Scratch w(ws);
            check(ttk_rmsnorm_bwd(dread(ao), dread(wo), rstd->device(), g, dx, ow ? 0 : 1, dw, R,
                                  D, w.ptr, ws, stream()),
                  "rmsnorm bwd");
        };
    }
    return out;
}

Tensor dropout(const Tensor& a, float p, uint64_t seed) {
    if (p <= 0.0f)
        return a;
    if (p >= 1.0f)
        throw std::invalid_argument("dropout: p must be < 1");
    // The reference's mask stream (xorshift64*, ops.cpp:949-963), generated on
    // the device bit for bit, so that a given seed drops the same elements.
    Tensor mask = make_out(a.shape(), false);
    check(ttk_dropout_mask(out_ptr(mask), mask.numel(), p, seed, stream()), "dropout");
    const float scale = 1.0f / (1.0f - p);
    return mul(mul(a, mask), full(a.shape(), scale));
}

Tensor rope(const Tensor& x, const Tensor& cos, const Tensor& sin) {
    if (x.ndim() != 4 || cos.ndim() != 2 || sin.ndim() != 2)
        throw std::invalid_argument("rope: rank mismatch");
    const int64_t B = x.dim(0), T = x.dim(1), H = x.dim(2), D = x.dim(3);
    if (D % 2 != 0)
        throw std::invalid_argument("rope: head dim must be even");
    const int64_t Dh = D / 2;
    if (cos.dim(0) != T || cos.dim(1) != Dh || sin.dim(0) != T || sin.dim(1) != Dh)
        throw std::invalid_argument("rope: cos/sin shape mismatch");
    Tensor out = make_out(x.shape(), x.requires_grad());
    check(ttk_rope_fwd(dread(x.impl()), dread(cos.impl()), dread(sin.impl()), out_ptr(out), B, T,
                       H, D, stream()),
          "rope");
    if (out.requires_grad() || cos.requires_grad() || sin.requires_grad()) {
        out.impl()->requires_grad = true;
        auto xo = x.impl(), co = cos.impl(), so = sin.impl();
        Tensor::Impl* oo = out.impl().get();  // own node: raw, no cycle
        oo->prev = {xo, co, so};
        oo->backward_fn = [xo, co, so, oo, B, T, H, D]() {
            const float* g = grad_in(oo);
            if (!g)
                return;
            if (xo->requires_grad) {
                bool ow = false;
                float* d = grad_target(xo, ow);
                check(ttk_rope_bwd(g, dread(co), dread(so), d, ow ? 0 : 1, B, T, H, D, stream()),
                      "rope bwd");
            }
            if (co->requires_grad || so->requires_grad)
                check(ttk_rope_table_grad(dread(xo), g, B, T, H, D,
                                          co->requires_grad ? grad_rmw(co) : nullptr,
                                          so->requires_grad ? grad_rmw(so) : nullptr, stream()),
                      "rope table grad");
        };
    }
    return out;
}

// ------------------------------------------------------------ fused ops --

namespace {

// The fused causal attention as one graph node: q, k, v [B,T,H,hd] (any
// logical shape with that storage), RoPE from the tables co/so (identity
// when null: the deferred chain's q and k are already rotated), output of
// shape `oshape` holding [B,T,H*hd]. With `planes` (and the bf16x3
// precision, an output big enough for tensor-core GEMMs) the kernel also
// writes the output's operand planes, cached on the output buffer as the
// [B*T, H*hd] GEMM operand split that the output projection looks up.
Tensor fused_attention(const ImplPtr& qo, const ImplPtr& ko, const ImplPtr& vo, ImplPtr co,
                       ImplPtr so, int64_t B, int64_t T, int64_t H, int64_t hd, float scale,
                       std::vector<int64_t> oshape, bool planes) {
    if (!co) {
        co = full({T, hd / 2}, 1.0f).impl();
        so = full({T, hd / 2}, 0.0f).impl();
    }
    const bool rg = qo->requires_grad || ko->requires_grad || vo->requires_grad;
    Tensor out = make_out(oshape, rg);
    auto lse = std::make_shared<Buffer>(B * H * T);
    // The forward's workspace holds q, k, v split into bf16 planes; it is kept
    // for the backward, which reuses them while q, k, v are unchanged.
    const size_t fws = ttk_attention_fwd_workspace_size(B, T, H, hd);
    auto fw = std::make_shared<Scratch>(fws);
    const int64_t R = B * T, D = H * hd;
    if (planes && ttk_gemm_get_precision() == 0 && R * D >= (1 << 20)) {
        float* o = out_ptr(out);
        Buffer& ob = *out.impl()->data;
        const size_t bytes = ttk_gemm_split_bytes(1, R, D);
        if (ob.split_bytes < bytes) {
            ttk_free(ob.split_dev, stream());
            ob.split_dev = nullptr;
            ob.split_bytes = 0;
            check(ttk_malloc(&ob.split_dev, bytes, stream()), "attention planes");
            ob.split_bytes = bytes;
        }
        check(ttk_attention_fwd_split(dread(qo), dread(ko), dread(vo), dread(co), dread(so), o,
                                      lse->device_for_overwrite(), ob.split_dev, B, T, H, hd,
                                      scale, fw->ptr, fws, stream()),
              "attention");
        const int64_t key[7] = {0, 1, R, D, D, 0, 0};
        ob.split_version = ob.version;
        std::copy(key, key + 7, ob.split_key);
    } else {
        check(ttk_attention_fwd(dread(qo), dread(ko), dread(vo), dread(co), dread(so),
                                out_ptr(out), lse->device_for_overwrite(), B, T, H, hd, scale,
                                fw->ptr, fws, stream()),
              "attention");
    }
    if (!rg)
        return out;
    // Contents of q, k, v as the forward read them (buffer versions).
    const uint64_t vq = version_of(qo), vk = version_of(ko), vv = version_of(vo);
    Tensor::Impl* oo = out.impl().get();  // own node: raw, no cycle
    oo->prev = {qo, ko, vo};
    const bool grad_planes = planes && ttk_gemm_get_precision() == 0 && R * D >= (1 << 20);
    oo->backward_fn = [qo, ko, vo, co, so, oo, lse, B, T, H, hd, scale, fw, vq, vk, vv,
                       grad_planes]() mutable {
        const float* g = grad_in(oo);
        if (!g)
            return;
        // Gradients that are not wanted go to scratch.
        std::vector<std::unique_ptr<Scratch>> junk;
        auto dst = [&](const ImplPtr& p, bool& ow) -> float* {
            if (p->requires_grad)
                return grad_target(p, ow);
            junk.emplace_back(new Scratch(static_cast<size_t>(p->numel) * 4));
            ow = true;
            return junk.back()->as<float>();
        };
        bool oq = false, ok = false, ov = false;
        float* dq = dst(qo, oq);
        float* dk = dst(ko, ok);
        float* dv = dst(vo, ov);
        const bool all_fresh = oq && ok && ov;
        if (!all_fresh) {  // one accumulate flag covers all three
            if (oq)
                check(ttk_memset(dq, 0, static_cast<size_t>(qo->numel) * 4, stream()), "zero");
            if (ok)
                check(ttk_memset(dk, 0, static_cast<size_t>(ko->numel) * 4, stream()), "zero");
            if (ov)
                check(ttk_memset(dv, 0, static_cast<size_t>(vo->numel) * 4, stream()), "zero");
        }
        const float *qd = dread(qo), *kd = dread(ko), *vd = dread(vo);
        const bool reuse = fw && fw->ptr && vq != ~0ull && version_of(qo) == vq &&
                           version_of(ko) == vk && version_of(vo) == vv;
        if (grad_planes) {
            // The gradients' operand planes, cached on their buffers as the
            // [B*T, H*hd] GEMM operand split the projections' backward reads.
            const int64_t R = B * T, D = H * hd;
            const size_t bytes = ttk_gemm_split_bytes(1, R, D);
            auto planes_of = [&](const ImplPtr& p) -> Buffer* {
                if (!p->requires_grad || !p->grad || p->grad->external)
                    return nullptr;
                Buffer& gb = *p->grad;
                if (gb.split_bytes < bytes) {
                    ttk_free(gb.split_dev, stream());
                    gb.split_dev = nullptr;
                    gb.split_bytes = 0;
                    check(ttk_malloc(&gb.split_dev, bytes, stream()), "gradient planes");
                    gb.split_bytes = bytes;
                }
                return &gb;
            };
            Buffer *pq = planes_of(qo), *pk = planes_of(ko), *pv = planes_of(vo);
            const size_t ws = reuse ? ttk_attention_bwd_ex_workspace_size(B, T, H, hd)
                                    : ttk_attention_bwd_workspace_size(B, T, H, hd);
            Scratch w(ws);
            check(ttk_attention_bwd_split(qd, kd, vd, dread(co), dread(so), dread(oo),
                                          lse->device(), g, dq, dk, dv, all_fresh ? 0 : 1, B, T,
                                          H, hd, scale, reuse ? fw->ptr : nullptr, w.ptr, ws,
                                          pq ? pq->split_dev : nullptr,
                                          pk ? pk->split_dev : nullptr,
                                          pv ? pv->split_dev : nullptr, stream()),
                  "attention bwd");
            const int64_t key[7] = {0, 1, R, D, D, 0, 0};
            for (Buffer* b : {pq, pk, pv})
                if (b) {
                    b->split_version = b->version;
                    std::copy(key, key + 7, b->split_key);
                }
        } else if (reuse) {
            const size_t ws = ttk_attention_bwd_ex_workspace_size(B, T, H, hd);
            Scratch w(ws);
            check(ttk_attention_bwd_ex(qd, kd, vd, dread(co), dread(so), dread(oo),
                                       lse->device(), g, dq, dk, dv, all_fresh ? 0 : 1, B, T, H,
                                       hd, scale, fw->ptr, w.ptr, ws, stream()),
                  "attention bwd");
        } else {
            const size_t ws = ttk_attention_bwd_workspace_size(B, T, H, hd);
            Scratch w(ws);
            check(ttk_attention_bwd(qd, kd, vd, dread(co), dread(so), dread(oo), lse->device(),
                                    g, dq, dk, dv, all_fresh ? 0 : 1, B, T, H, hd, scale, w.ptr,
                                    ws, stream()),
                  "attention bwd");
        }
        fw.reset();  // planes no longer needed (stream-ordered free)
    };
    return out;
}

}  // namespace

Tensor causal_attention(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& cos,
                        const Tensor& sin) {
    if (q.ndim() != 4 || q.shape() != k.shape() || q.shape() != v.shape())
        throw std::invalid_argument("causal_attention: q, k, v must be [B,T,H,hd] alike");
    const int64_t B = q.dim(0), T = q.dim(1), H = q.dim(2), hd = q.dim(3);
    if (cos.ndim() != 2 || cos.dim(0) < T || cos.dim(1) != hd / 2 || sin.shape() != cos.shape())
        throw std::invalid_argument("rope: cos/sin shape mismatch");
    const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
    return fused_attention(q.impl(), k.impl(), v.impl(), cos.impl(), sin.impl(), B, T, H, hd,
                           scale, {B, T, H * hd}, true);
}

Tensor swiglu(const Tensor& a, const Tensor& b) {
    if (a.shape() != b.shape())
        throw std::invalid_argument("swiglu: shape mismatch");
    Tensor out = make_out(a.shape(), a.requires_grad() || b.requires_grad());
    check(ttk_swiglu_fwd(dread(a.impl()), dread(b.impl()), out_ptr(out), a.numel(), stream()),
          "swiglu");
    if (out.requires_grad()) {
        auto ao = a.impl(), bo = b.impl();
        Tensor::Impl* oo = out.impl().get();  // own node: raw, no cycle
        oo->prev = {ao, bo};
        oo->backward_fn = [ao, bo, oo]() {
            const float* g = grad_in(oo);
            if (!g)
                return;
            std::unique_ptr<Scratch> ja, jb;
            bool owa = true, owb = true;
            float* da;
            float* db;
            if (ao->requires_grad) {
                da = grad_target(ao, owa);
            } else {
                ja.reset(new Scratch(static_cast<size_t>(ao->numel) * 4));
                da = ja->as<float>();
            }
            if (bo->requires_grad) {
                db = grad_target(bo, owb);
            } else {
                jb.reset(new Scratch(static_cast<size_t>(bo->numel) * 4));
                db = jb->as<float>();
            }
            if (owa != owb) {
                if (owa)
                    check(ttk_memset(da, 0, static_cast<size_t>(ao->numel) * 4, stream()), "zero");
                if (owb)
                    check(ttk_memset(db, 0, static_cast<size_t>(bo->numel) * 4, stream()), "zero");
            }
            check(ttk_swiglu_bwd(dread(ao), dread(bo), g, da, db, (owa && owb) ? 0 : 1, ao->numel,
                                 stream()),
                  "swiglu bwd");
        };
    }
    return out;
}

float clip_grad_norm(const std::vector<Tensor*>& params, float max_norm) {
    std::vector<const float*> ptrs;
    std::vector<int64_t> sizes;
    for (Tensor* p : params)
        if (p->has_grad()) {
            ptrs.push_back(p->device_grad());
            sizes.push_back(p->numel());
        }
    Scratch acc(8);
    check(ttk_memset(acc.ptr, 0, 8, stream()), "zero");
    check(ttk_sumsq_multi(ptrs.data(), sizes.data(), static_cast<int>(ptrs.size()),
                          acc.as<double>(), stream()),
          "sumsq");
    double ss = 0.0;
    check(ttk_memcpy_d2h(&ss, acc.ptr, 8, stream()), "norm read");
    const double total = std::sqrt(ss);
    if (max_norm > 0.0f) {
        const float coef = static_cast<float>(max_norm / (total + 1e-6));
        if (coef < 1.0f) {
            Scratch c(16);
            check(ttk_fill(c.as<float>(), coef, 1, stream()), "coef");
            const int64_t zero = 0, one = 1;
            for (Tensor* p : params)
                if (p->has_grad()) {
                    const int64_t n = p->numel();
                    float* g = p->impl()->grad->device();
                    check(ttk_binary(2, g, &one, c.as<float>(), &zero, g, &n, 1, stream()),
                          "clip scale");
                    p->impl()->grad->host_valid = false;
                    p->impl()->grad->touch();
                }
        }
    }
    return static_cast<float>(total);
}

}  // namespace tt
