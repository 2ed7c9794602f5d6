// Generic tensor kernels behind the rest of the reference op set
// (ops.cpp:139-657): broadcast elementwise binary / unary ops with their
// gradient rules, reductions, strided (permute / expand) copies, fill, axpy,
// and a counter-based normal initializer.
//
// Shapes are passed as up to TTK_MAX_DIMS extents with per-input element
// strides expressed in the output's index space (0 on broadcast dims), so the
// reference's per-element multi-index decode (ops.cpp:150-158) happens once
// per element on the device. Reductions assign one thread per output element
// and sum in a fixed order: results are deterministic.
#include <cuda_runtime.h>
#include <stdint.h>

#include "ttk_common.cuh"
#include "ttk_internal.h"

namespace ttk {
namespace gen {

struct Shape8 {
    int64_t n[TTK_MAX_DIMS];
    int64_t sa[TTK_MAX_DIMS];
    int64_t sb[TTK_MAX_DIMS];
    int ndim;
};

__device__ __forceinline__ void decode(const Shape8& s, int64_t l, int64_t& oa, int64_t& ob) {
    oa = 0, ob = 0;
    for (int d = s.ndim - 1; d >= 0; --d) {
        const int64_t i = l % s.n[d];
        l /= s.n[d];
        oa += i * s.sa[d];
        ob += i * s.sb[d];
    }
}

__device__ __forceinline__ float bin_fwd(int op, float a, float b) {
    switch (op) {
        case 0: return a + b;
        case 1: return a - b;
        case 2: return a * b;
        default: return a / b;
    }
}

// d(out)/d(a) * g or d(out)/d(b) * g (ops.cpp:253-259).
__device__ __forceinline__ float bin_grad(int op, int which, float a, float b, float g) {
    switch (op) {
        case 0: return g;
        case 1: return which ? -g : g;
        case 2: return which ? g * a : g * b;
        default: return which ? -g * a / (b * b) : g / b;
    }
}

__global__ void binary_kernel(int op, const float* __restrict__ a, const float* __restrict__ b,
                              float* __restrict__ out, Shape8 s, int64_t total) {
    for (int64_t l = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; l < total;
         l += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t oa, ob;
        decode(s, l, oa, ob);
        out[l] = bin_fwd(op, a[oa], b[ob]);
    }
}

// Same-shape contiguous operands (the residual adds of a transformer block):
// 16-byte vector loads and stores, no index decode. Same arithmetic as
// binary_kernel, element for element.
template <int OP>
__global__ void binary_contig_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                     float* __restrict__ out, int64_t n) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t n4 = n / 4;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
         i += stride) {
        const float4 x = reinterpret_cast<const float4*>(a)[i];
        const float4 y = reinterpret_cast<const float4*>(b)[i];
        float4 r;
        r.x = bin_fwd(OP, x.x, y.x);
        r.y = bin_fwd(OP, x.y, y.y);
        r.z = bin_fwd(OP, x.z, y.z);
        r.w = bin_fwd(OP, x.w, y.w);
        reinterpret_cast<float4*>(out)[i] = r;
    }
    for (int64_t i = n4 * 4 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += stride)
        out[i] = bin_fwd(OP, a[i], b[i]);
}

__global__ void binary_grad_kernel(int op, int which, const float* __restrict__ a,
                                   const float* __restrict__ b, const float* __restrict__ g,
                                   float* __restrict__ gf, Shape8 s, int64_t total) {
    for (int64_t l = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; l < total;
         l += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t oa, ob;
        decode(s, l, oa, ob);
        gf[l] = bin_grad(op, which, a[oa], b[ob], g[l]);
    }
}

// Unary ops and derivatives (ops.cpp:314-363).
__device__ __forceinline__ float un_fwd(int op, float x, float p) {
    switch (op) {
        case 0: return -x;
        case 1: return expf(x);
        case 2: return logf(x);
        case 3: return sqrtf(x);
        case 4: return tanhf(x);
        case 5: return x / (1.0f + expf(-x));
        case 6: return sinf(x);
        case 7: return cosf(x);
        default: return powf(x, p);
    }
}

__device__ __forceinline__ float un_grad(int op, float x, float p) {
    switch (op) {
        case 0: return -1.0f;
        case 1: return expf(x);
        case 2: return 1.0f / x;
        case 3: return 0.5f / sqrtf(x);
        case 4: {
            const float t = tanhf(x);
            return 1.0f - t * t;
        }
        case 5: {
            const float s = 1.0f / (1.0f + expf(-x));
            return s * (1.0f + x * (1.0f - s));
        }
        case 6: return cosf(x);
        case 7: return -sinf(x);
        default: return p * powf(x, p - 1.0f);
    }
}

__global__ void unary_kernel(int op, const float* __restrict__ x, float* __restrict__ y, int64_t n,
                             float p) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] = un_fwd(op, x[i], p);
}

__global__ void unary_bwd_kernel(int op, const float* __restrict__ x, const float* __restrict__ dy,
                                 float* __restrict__ dx, int64_t n, float p) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        // neg's rule is a subtraction in the reference (ops.cpp:281); the
        // others multiply dy by f'(x).
        dx[i] += op == 0 ? -dy[i] : dy[i] * un_grad(op, x[i], p);
    }
}

// out[o*inner + i] (+)= sum_k in[(o*K + k)*inner + i], k ascending.
__global__ void reduce_mid_kernel(const float* __restrict__ in, float* __restrict__ out,
                                  int64_t outer, int64_t K, int64_t inner, int accumulate) {
    const int64_t total = outer * inner;
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t o = t / inner, i = t % inner;
        const float* p = in + o * K * inner + i;
        float s = 0.0f;
        for (int64_t k = 0; k < K; ++k)
            s += p[k * inner];
        out[t] = accumulate ? out[t] + s : s;
    }
}

// General reduction to the kept dims (bit d of keep set: dim d kept).
struct ReduceGeo {
    int64_t n[TTK_MAX_DIMS];
    int ndim;
    unsigned keep;
};

__global__ void reduce_to_kernel(const float* __restrict__ g, float* __restrict__ out,
                                 ReduceGeo r, int64_t out_total, int64_t red_total,
                                 int accumulate) {
    for (int64_t o = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; o < out_total;
         o += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        // Multi-index of the kept dims from o.
        int64_t kidx[TTK_MAX_DIMS];
        int64_t rem = o;
        for (int d = r.ndim - 1; d >= 0; --d) {
            if (r.keep & (1u << d)) {
                kidx[d] = rem % r.n[d];
                rem /= r.n[d];
            } else {
                kidx[d] = 0;
            }
        }
        float s = 0.0f;
        for (int64_t q = 0; q < red_total; ++q) {
            int64_t rq = q, off = 0, stride = 1;
            int64_t idx[TTK_MAX_DIMS];
            for (int d = r.ndim - 1; d >= 0; --d) {
                if (r.keep & (1u << d)) {
                    idx[d] = kidx[d];
                } else {
                    idx[d] = rq % r.n[d];
                    rq /= r.n[d];
                }
            }
            for (int d = r.ndim - 1; d >= 0; --d) {
                off += idx[d] * stride;
                stride *= r.n[d];
            }
            s += g[off];
        }
        out[o] = accumulate ? out[o] + s : s;
    }
}

__global__ void sum_all_kernel(const float* __restrict__ in, int64_t n, double* __restrict__ acc) {
    double s = 0.0;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        s += static_cast<double>(in[i]);
    s = warp_sum_d(s);
    __shared__ double sh[32];
    if ((threadIdx.x & 31) == 0)
        sh[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        s = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0;
        s = warp_sum_d(s);
        if (threadIdx.x == 0)
            acc[blockIdx.x] = s;
    }
}

__global__ void sum_all_finish_kernel(const double* __restrict__ part, int nb, float* out,
                                      int accumulate) {
    double s = 0.0;
    for (int i = 0; i < nb; ++i)
        s += part[i];
    out[0] = accumulate ? out[0] + static_cast<float>(s) : static_cast<float>(s);
}

// Gather: out[l] (+)= in[view(l)]; scatter: out[view(l)] += in[l] (the view
// must be injective, as permute's is).
__global__ void strided_copy_kernel(const float* __restrict__ in, float* __restrict__ out,
                                    Shape8 s, int64_t total, int accumulate, int scatter) {
    for (int64_t l = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; l < total;
         l += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t oa, ob;
        decode(s, l, oa, ob);
        if (scatter)
            out[oa] += in[l];
        else
            out[l] = accumulate ? out[l] + in[oa] : in[oa];
    }
}

__global__ void fill_kernel(float* __restrict__ x, float v, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        x[i] = v;
}

__global__ void axpy_kernel(float alpha, const float* __restrict__ x, float* __restrict__ y,
                            int64_t n) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const bool vec = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
    int64_t start = 0;
    if (vec) {
        const int64_t n4 = n / 4;
        for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
             i += stride) {
            const float4 a = reinterpret_cast<const float4*>(x)[i];
            float4 b = reinterpret_cast<float4*>(y)[i];
            if (alpha == 1.0f) {
                b.x += a.x, b.y += a.y, b.z += a.z, b.w += a.w;
            } else {
                b.x += alpha * a.x, b.y += alpha * a.y, b.z += alpha * a.z, b.w += alpha * a.w;
            }
            reinterpret_cast<float4*>(y)[i] = b;
        }
        start = n4 * 4;
    }
    for (int64_t i = start + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += stride)
        y[i] += alpha == 1.0f ? x[i] : alpha * x[i];
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// x[i] = std * N(0,1) from a counter-based generator (splitmix64 of the
// seed and index, Box-Muller): any element is computable independently.
__global__ void init_normal_kernel(float* __restrict__ x, int64_t n, float stdv, uint64_t seed) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const uint64_t r1 = splitmix64(seed * 0x632BE59BD9B4E019ull + 2 * static_cast<uint64_t>(i));
        const uint64_t r2 = splitmix64(seed * 0x632BE59BD9B4E019ull + 2 * static_cast<uint64_t>(i) + 1);
        const double u1 = (r1 >> 11) * (1.0 / 9007199254740992.0);
        const double u2 = (r2 >> 11) * (1.0 / 9007199254740992.0);
        const double z = sqrt(-2.0 * log(u1 + 1e-300)) * cos(6.283185307179586 * u2);
        x[i] = stdv * static_cast<float>(z);
    }
}

int fill_shape(Shape8& s, const int64_t* shape, int ndim, const int64_t* sa, const int64_t* sb,
               int64_t& total) {
    if (ndim < 1 || ndim > TTK_MAX_DIMS)
        return set_error(TTK_ERR_ARG, "rank must be 1..8");
    s.ndim = ndim;
    total = 1;
    for (int d = 0; d < ndim; ++d) {
        if (shape[d] < 0)
            return set_error(TTK_ERR_ARG, "negative extent");
        s.n[d] = shape[d];
        s.sa[d] = sa ? sa[d] : 0;
        s.sb[d] = sb ? sb[d] : 0;
        total *= shape[d];
    }
    return TTK_OK;
}

}  // namespace gen
}  // namespace ttk

using namespace ttk;
using namespace ttk::gen;

static inline cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

extern "C" {

int ttk_binary(int op, const float* a, const int64_t* a_strides, const float* b,
               const int64_t* b_strides, float* out, const int64_t* shape, int ndim,
               void* stream) {
    if (op < 0 || op > 3)
        return set_error(TTK_ERR_ARG, "binary: unknown op");
    Shape8 s;
    int64_t total;
    int rc = fill_shape(s, shape, ndim, a_strides, b_strides, total);
    if (rc || !total)
        return rc;
    // Row-major contiguous strides on both inputs (extent-1 dims may carry any
    // stride) and 16-byte aligned pointers: the vector path.
    bool contig = ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                    reinterpret_cast<uintptr_t>(out)) & 15) == 0;
    int64_t expect = 1;
    for (int d = ndim - 1; d >= 0 && contig; --d) {
        if (s.n[d] != 1 && (s.sa[d] != expect || s.sb[d] != expect))
            contig = false;
        expect *= s.n[d];
    }
    if (contig) {
        const unsigned grid = grid_for(total / 4 + 1, 256);
        switch (op) {
            case 0: binary_contig_kernel<0><<<grid, 256, 0, S(stream)>>>(a, b, out, total); break;
            case 1: binary_contig_kernel<1><<<grid, 256, 0, S(stream)>>>(a, b, out, total); break;
            case 2: binary_contig_kernel<2><<<grid, 256, 0, S(stream)>>>(a, b, out, total); break;
            default: binary_contig_kernel<3><<<grid, 256, 0, S(stream)>>>(a, b, out, total); break;
        }
        return check_launch("binary_contig_kernel");
    }
    binary_kernel<<<grid_for(total, 256), 256, 0, S(stream)>>>(op, a, b, out, s, total);
    return check_launch("binary_kernel");
}

int ttk_binary_bwd(int op, int which, const float* a, const int64_t* a_strides, const float* b,
                   const int64_t* b_strides, const float* dout, float* g_full,
                   const int64_t* shape, int ndim, void* stream) {
    if (op < 0 || op > 3 || which < 0 || which > 1)
        return set_error(TTK_ERR_ARG, "binary_bwd: bad op");
    Shape8 s;
    int64_t total;
    int rc = fill_shape(s, shape, ndim, a_strides, b_strides, total);
    if (rc || !total)
        return rc;
    binary_grad_kernel<<<grid_for(total, 256), 256, 0, S(stream)>>>(op, which, a, b, dout,
                                                                    g_full, s, total);
    return check_launch("binary_grad_kernel");
}

int ttk_unary(int op, const float* x, float* y, int64_t n, float p, void* stream) {
    if (op < 0 || op > 8 || n < 0)
        return set_error(TTK_ERR_ARG, "unary: bad op");
    if (!n)
        return TTK_OK;
    unary_kernel<<<grid_for(n, 256), 256, 0, S(stream)>>>(op, x, y, n, p);
    return check_launch("unary_kernel");
}

int ttk_unary_bwd(int op, const float* x, const float* dy, float* dx, int64_t n, float p,
                  void* stream) {
    if (op < 0 || op > 8 || n < 0)
        return set_error(TTK_ERR_ARG, "unary_bwd: bad op");
    if (!n)
        return TTK_OK;
    unary_bwd_kernel<<<grid_for(n, 256), 256, 0, S(stream)>>>(op, x, dy, dx, n, p);
    return check_launch("unary_bwd_kernel");
}

int ttk_reduce_mid(const float* in, float* out, int64_t outer, int64_t K, int64_t inner,
                   int accumulate, void* stream) {
    if (outer < 0 || K < 0 || inner < 0)
        return set_error(TTK_ERR_ARG, "reduce_mid: negative size");
    if (!outer || !inner)
        return TTK_OK;
    reduce_mid_kernel<<<grid_for(outer * inner, 256), 256, 0, S(stream)>>>(in, out, outer, K,
                                                                          inner, accumulate);
    return check_launch("reduce_mid_kernel");
}

int ttk_reduce_to(const float* g, const int64_t* shape, int ndim, unsigned keep_mask, float* out,
                  int accumulate, void* stream) {
    if (ndim < 1 || ndim > TTK_MAX_DIMS)
        return set_error(TTK_ERR_ARG, "reduce_to: rank must be 1..8");
    ReduceGeo r;
    r.ndim = ndim;
    r.keep = keep_mask;
    int64_t out_total = 1, red_total = 1;
    for (int d = 0; d < ndim; ++d) {
        r.n[d] = shape[d];
        if (keep_mask & (1u << d))
            out_total *= shape[d];
        else
            red_total *= shape[d];
    }
    if (!out_total)
        return TTK_OK;
    reduce_to_kernel<<<grid_for(out_total, 128), 128, 0, S(stream)>>>(g, out, r, out_total,
                                                                     red_total, accumulate);
    return check_launch("reduce_to_kernel");
}

int ttk_sum_all(const float* in, int64_t n, float* out, int accumulate, void* stream) {
    if (n < 0)
        return set_error(TTK_ERR_ARG, "sum_all: negative size");
    const int nb = static_cast<int>(std::min<int64_t>(std::max<int64_t>((n + 1023) / 1024, 1), 296));
    double* part = nullptr;
    int rc = check_cuda(cudaMallocAsync(reinterpret_cast<void**>(&part), nb * sizeof(double),
                                        S(stream)),
                        "sum_all alloc");
    if (rc)
        return rc;
    sum_all_kernel<<<nb, 256, 0, S(stream)>>>(in, n, part);
    sum_all_finish_kernel<<<1, 1, 0, S(stream)>>>(part, nb, out, accumulate);
    cudaFreeAsync(part, S(stream));
    return check_launch("sum_all_kernel");
}

int ttk_strided_copy(const float* in, const int64_t* in_strides, float* out,
                     const int64_t* shape, int ndim, int accumulate, int scatter_add,
                     void* stream) {
    Shape8 s;
    int64_t total;
    int rc = fill_shape(s, shape, ndim, in_strides, nullptr, total);
    if (rc || !total)
        return rc;
    strided_copy_kernel<<<grid_for(total, 256), 256, 0, S(stream)>>>(in, out, s, total,
                                                                    accumulate, scatter_add);
    return check_launch("strided_copy_kernel");
}

int ttk_fill(float* x, float v, int64_t n, void* stream) {
    if (n < 0)
        return set_error(TTK_ERR_ARG, "fill: negative size");
    if (!n)
        return TTK_OK;
    fill_kernel<<<grid_for(n, 256), 256, 0, S(stream)>>>(x, v, n);
    return check_launch("fill_kernel");
}

int ttk_axpy(float alpha, const float* x, float* y, int64_t n, void* stream) {
    if (n < 0)
        return set_error(TTK_ERR_ARG, "axpy: negative size");
    if (!n)
        return TTK_OK;
    axpy_kernel<<<grid_for(n / 4 + 1, 256), 256, 0, S(stream)>>>(alpha, x, y, n);
    return check_launch("axpy_kernel");
}

int ttk_init_normal(float* x, int64_t n, float std, uint64_t seed, void* stream) {
    if (n < 0)
        return set_error(TTK_ERR_ARG, "init_normal: negative size");
    if (!n)
        return TTK_OK;
    init_normal_kernel<<<grid_for(n, 256), 256, 0, S(stream)>>>(x, n, std, seed);
    return check_launch("init_normal_kernel");
}

}  // extern "C"
