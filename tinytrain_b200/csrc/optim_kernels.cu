// Optimizer kernels: multi-tensor sum of squares (the global gradient norm)
// and one fused AdamW step with global-norm clipping folded in, over a list
// of parameter tensors in a single launch (the reference's AdamW::step,
// optim.cpp:17-48, runs a sequential host loop per parameter).
//
// HBM traffic per parameter element: sumsq reads g (4 B); AdamW reads p, g, m,
// v and writes p, m, v (28 B): 32 B in total.
#include <cuda_runtime.h>
#include <stdint.h>

#include "ttk_common.cuh"
#include "ttk_internal.h"

namespace ttk {
namespace opt {

constexpr int kMaxTensors = 96;  // per launch; longer lists are split

struct TensorList {
    float* p[kMaxTensors];
    const float* g[kMaxTensors];
    float* m[kMaxTensors];
    float* v[kMaxTensors];
    int64_t start4[kMaxTensors + 1];  // prefix sums of ceil(n/4)
    int64_t n[kMaxTensors];
    int count;
};

__device__ __forceinline__ int find_tensor(const TensorList& L, int64_t q) {
    int lo = 0, hi = L.count - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (L.start4[mid] <= q)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}

__global__ void sumsq_kernel(TensorList L, double* __restrict__ acc) {
    const int64_t total4 = L.start4[L.count];
    double s = 0.0;
    for (int64_t q = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; q < total4;
         q += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int t = find_tensor(L, q);
        const int64_t e0 = (q - L.start4[t]) * 4;
        const float* g = L.g[t];
        const int64_t n = L.n[t];
        if (e0 + 4 <= n && (reinterpret_cast<uintptr_t>(g) & 15) == 0) {
            const float4 v = *reinterpret_cast<const float4*>(g + e0);
            s += static_cast<double>(v.x * v.x + v.y * v.y) + static_cast<double>(v.z * v.z + v.w * v.w);
        } else {
            for (int64_t e = e0; e < n && e < e0 + 4; ++e)
                s += static_cast<double>(g[e]) * g[e];
        }
    }
    s = warp_sum_d(s);
    __shared__ double sh[32];
    if ((threadIdx.x & 31) == 0)
        sh[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        s = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0;
        s = warp_sum_d(s);
        if (threadIdx.x == 0)
            atomicAdd(acc, s);
    }
}

struct AdamArgs {
    float lr, b1, b2, eps, wd, lr_t, grad_scale, max_norm;
    const double* sumsq;
    // Device schedule {lr, lr_t} read at kernel start when set (a step
    // replayed from a CUDA graph takes its learning rate and bias correction
    // from here instead of from the launch arguments recorded once).
    const float* sched;
};

// lr_t of optim.cpp:22-24 in float, as the reference computes it.
static float adam_lr_t(float lr, float beta1, float beta2, int64_t step) {
    const float bc1 = 1.0f - std::pow(beta1, static_cast<float>(step));
    const float bc2 = 1.0f - std::pow(beta2, static_cast<float>(step));
    return lr * std::sqrt(bc2) / bc1;
}

__global__ void adam_sched_kernel(float* __restrict__ sched, float lr, float lr_t) {
    sched[0] = lr;
    sched[1] = lr_t;
}

// One element of optim.cpp:36-45, gradient pre-multiplied by the clip
// coefficient and grad_scale.
__device__ __forceinline__ void adam_elem(float& d, float gi, float& m, float& v,
                                          const AdamArgs& a) {
    d -= a.lr * a.wd * d;
    m = a.b1 * m + (1.0f - a.b1) * gi;
    v = a.b2 * v + (1.0f - a.b2) * gi * gi;
    d -= a.lr_t * m / (sqrtf(v) + a.eps);
}

__global__ void adamw_kernel(TensorList L, AdamArgs a) {
    if (a.sched) {
        a.lr = a.sched[0];
        a.lr_t = a.sched[1];
    }
    float coef = a.grad_scale;
    if (a.sumsq && a.max_norm > 0.0f) {
        // coef = max_norm / (||g|| + 1e-6), applied when < 1 (the norm is of
        // the gradients as accumulated, before grad_scale).
        const double total = sqrt(*a.sumsq) * static_cast<double>(a.grad_scale);
        const float c = static_cast<float>(static_cast<double>(a.max_norm) / (total + 1e-6));
        if (c < 1.0f)
            coef = a.grad_scale * c;
    }
    const int64_t total4 = L.start4[L.count];
    for (int64_t q = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; q < total4;
         q += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int t = find_tensor(L, q);
        const int64_t e0 = (q - L.start4[t]) * 4;
        float* p = L.p[t];
        const float* g = L.g[t];
        float* m = L.m[t];
        float* v = L.v[t];
        const int64_t n = L.n[t];
        const bool vec = e0 + 4 <= n &&
                         ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(g) |
                           reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v)) &
                          15) == 0;
        if (vec) {
            float4 pd = *reinterpret_cast<float4*>(p + e0);
            const float4 gd = *reinterpret_cast<const float4*>(g + e0);
            float4 md = *reinterpret_cast<float4*>(m + e0);
            float4 vd = *reinterpret_cast<float4*>(v + e0);
            adam_elem(pd.x, gd.x * coef, md.x, vd.x, a);
            adam_elem(pd.y, gd.y * coef, md.y, vd.y, a);
            adam_elem(pd.z, gd.z * coef, md.z, vd.z, a);
            adam_elem(pd.w, gd.w * coef, md.w, vd.w, a);
            *reinterpret_cast<float4*>(p + e0) = pd;
            *reinterpret_cast<float4*>(m + e0) = md;
            *reinterpret_cast<float4*>(v + e0) = vd;
        } else {
            for (int64_t e = e0; e < n && e < e0 + 4; ++e)
                adam_elem(p[e], g[e] * coef, m[e], v[e], a);
        }
    }
}

// SGD (optim.cpp:58-82).
__global__ void sgd_kernel(float* __restrict__ p, const float* __restrict__ g,
                           float* __restrict__ vel, int64_t n, float lr, float mom, float wd) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        if (mom == 0.0f || !vel) {
            p[i] -= lr * (g[i] + wd * p[i]);
        } else {
            const float gi = g[i] + wd * p[i];
            vel[i] = mom * vel[i] + gi;
            p[i] -= lr * vel[i];
        }
    }
}

}  // namespace opt
}  // namespace ttk

using namespace ttk;
using namespace ttk::opt;

static inline cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

extern "C" {

int ttk_sumsq_multi(const float* const* ptrs, const int64_t* sizes, int n_tensors, double* acc,
                    void* stream) {
    if (n_tensors < 0 || (n_tensors && (!ptrs || !sizes)) || !acc)
        return set_error(TTK_ERR_ARG, "sumsq_multi: bad arguments");
    for (int base = 0; base < n_tensors; base += kMaxTensors) {
        TensorList L{};
        L.count = std::min(kMaxTensors, n_tensors - base);
        L.start4[0] = 0;
        for (int i = 0; i < L.count; ++i) {
            L.g[i] = ptrs[base + i];
            L.n[i] = sizes[base + i];
            if (L.n[i] < 0)
                return set_error(TTK_ERR_ARG, "sumsq_multi: negative size");
            L.start4[i + 1] = L.start4[i] + (L.n[i] + 3) / 4;
        }
        const int64_t total4 = L.start4[L.count];
        if (!total4)
            continue;
        sumsq_kernel<<<grid_for(total4, 256, 148 * 4), 256, 0, S(stream)>>>(L, acc);
        int rc = check_launch("sumsq_kernel");
        if (rc)
            return rc;
    }
    return TTK_OK;
}

static int adamw_multi(float* const* params, const float* const* grads, float* const* m,
                       float* const* v, const int64_t* sizes, int n_tensors, float lr, float beta1,
                       float beta2, float eps, float weight_decay, int64_t step,
                       const double* sumsq, float max_norm, float grad_scale, const float* sched,
                       void* stream) {
    if (n_tensors < 0 || step < 1)
        return set_error(TTK_ERR_ARG, "adamw_multi: bad arguments");
    AdamArgs a;
    a.lr = lr, a.b1 = beta1, a.b2 = beta2, a.eps = eps, a.wd = weight_decay;
    a.lr_t = adam_lr_t(lr, beta1, beta2, step);
    a.grad_scale = grad_scale;
    a.max_norm = max_norm;
    a.sumsq = sumsq;
    a.sched = sched;
    for (int base = 0; base < n_tensors; base += kMaxTensors) {
        TensorList L{};
        L.count = std::min(kMaxTensors, n_tensors - base);
        L.start4[0] = 0;
        for (int i = 0; i < L.count; ++i) {
            const int j = base + i;
            if (!params[j] || !grads[j] || !m[j] || !v[j] || sizes[j] < 0)
                return set_error(TTK_ERR_ARG, "adamw_multi: null tensor");
            L.p[i] = params[j], L.g[i] = grads[j], L.m[i] = m[j], L.v[i] = v[j];
            L.n[i] = sizes[j];
            L.start4[i + 1] = L.start4[i] + (L.n[i] + 3) / 4;
        }
        const int64_t total4 = L.start4[L.count];
        if (!total4)
            continue;
        adamw_kernel<<<grid_for(total4, 256, 148 * 8), 256, 0, S(stream)>>>(L, a);
        int rc = check_launch("adamw_kernel");
        if (rc)
            return rc;
    }
    return TTK_OK;
}

int ttk_adamw_multi(float* const* params, const float* const* grads, float* const* m,
                    float* const* v, const int64_t* sizes, int n_tensors, float lr, float beta1,
                    float beta2, float eps, float weight_decay, int64_t step,
                    const double* sumsq, float max_norm, float grad_scale, void* stream) {
    return adamw_multi(params, grads, m, v, sizes, n_tensors, lr, beta1, beta2, eps, weight_decay,
                       step, sumsq, max_norm, grad_scale, nullptr, stream);
}

int ttk_adamw_multi_sched(float* const* params, const float* const* grads, float* const* m,
                          float* const* v, const int64_t* sizes, int n_tensors, float beta1,
                          float beta2, float eps, float weight_decay, const float* sched,
                          const double* sumsq, float max_norm, float grad_scale, void* stream) {
    if (!sched)
        return set_error(TTK_ERR_ARG, "adamw_multi_sched: null schedule");
    // lr and step are placeholders: the kernel reads lr and lr_t from sched.
    return adamw_multi(params, grads, m, v, sizes, n_tensors, 0.0f, beta1, beta2, eps,
                       weight_decay, 1, sumsq, max_norm, grad_scale, sched, stream);
}

int ttk_adamw_sched_set(float* sched, float lr, float beta1, float beta2, int64_t step,
                        void* stream) {
    if (!sched || step < 1)
        return set_error(TTK_ERR_ARG, "adamw_sched_set: bad arguments");
    adam_sched_kernel<<<1, 1, 0, S(stream)>>>(sched, lr, adam_lr_t(lr, beta1, beta2, step));
    return check_launch("adam_sched_kernel");
}

int ttk_sgd(float* p, const float* g, float* vel, int64_t n, float lr, float momentum,
            float weight_decay, void* stream) {
    if (n < 0)
        return set_error(TTK_ERR_ARG, "sgd: negative size");
    if (!n)
        return TTK_OK;
    sgd_kernel<<<grid_for(n, 256), 256, 0, S(stream)>>>(p, g, vel, n, lr, momentum, weight_decay);
    return check_launch("sgd_kernel");
}

}  // extern "C"
