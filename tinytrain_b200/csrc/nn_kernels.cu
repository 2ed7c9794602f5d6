// Bandwidth-bound NN kernels: RMSNorm, SwiGLU, fused cross-entropy,
// embedding gather / deterministic scatter-add, RoPE, row softmax.
//
// All are HBM-bound: float4 coalesced access, warp-shuffle reductions, one
// read and one write of each tensor where the algorithm allows (the fused
// cross-entropy keeps its 32000-wide row in registers between the reduction
// and the gradient write).
#include <algorithm>
#include <atomic>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ttk_common.cuh"
#include "ttk_internal.h"

namespace ttk {
namespace nn {

// ------------------------------------------------------------- RMSNorm --
// One warp per row (ops.cpp:932-942: r = (sum(x^2)/D + eps)^-1/2, y = x*r*w).
__global__ void rmsnorm_fwd_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                   float* __restrict__ y, float* __restrict__ rstd, int64_t R,
                                   int64_t D, float eps) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    const bool vec = (D & 3) == 0;
    for (int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
         row < R; row += warps) {
        const float* xr = x + row * D;
        float ss = 0.0f;
        if (vec) {
            for (int64_t c = lane * 4; c < D; c += 128) {
                float4 v = *reinterpret_cast<const float4*>(xr + c);
                ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            }
        } else {
            for (int64_t c = lane; c < D; c += 32)
                ss += xr[c] * xr[c];
        }
        ss = warp_sum(ss);
        const float r = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
        if (lane == 0 && rstd)
            rstd[row] = r;
        float* yr = y + row * D;
        if (vec) {
            for (int64_t c = lane * 4; c < D; c += 128) {
                float4 v = *reinterpret_cast<const float4*>(xr + c);
                float4 g = *reinterpret_cast<const float4*>(w + c);
                float4 o = make_float4(v.x * r * g.x, v.y * r * g.y, v.z * r * g.z, v.w * r * g.w);
                *reinterpret_cast<float4*>(yr + c) = o;
            }
        } else {
            for (int64_t c = lane; c < D; c += 32)
                yr[c] = xr[c] * r * w[c];
        }
    }
}

// dx = r*(dy*w) - x * r^3/D * sum(dy*w*x); dw partial per block (fixed order).
// Block: 8 warps; block b owns rows [b*rpb, (b+1)*rpb); partial[b][D].
__global__ void rmsnorm_bwd_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                   const float* __restrict__ rstd, const float* __restrict__ dy,
                                   float* __restrict__ dx, int accumulate,
                                   float* __restrict__ partial, int64_t R, int64_t D,
                                   int64_t rpb) {
    extern __shared__ float sdw[];  // [8][D]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r0 = blockIdx.x * rpb;
    const int64_t r1 = min(R, r0 + rpb);
    for (int64_t c = threadIdx.x; c < 8 * D; c += blockDim.x)
        sdw[c] = 0.0f;
    __syncthreads();
    float* mydw = sdw + warp * D;
    for (int64_t row = r0 + warp; row < r1; row += 8) {
        const float* xr = x + row * D;
        const float* gr = dy + row * D;
        const float r = rstd[row];
        float dot = 0.0f;
        for (int64_t c = lane; c < D; c += 32)
            dot += gr[c] * w[c] * xr[c];
        dot = warp_sum(dot);
        const float k = r * r * r / static_cast<float>(D) * dot;
        for (int64_t c = lane; c < D; c += 32) {
            const float gx = gr[c];
            const float xv = xr[c];
            if (dx) {
                float v = r * (gx * w[c]) - xv * k;
                dx[row * D + c] = accumulate ? dx[row * D + c] + v : v;
            }
            mydw[c] += gx * xv * r;
        }
    }
    __syncthreads();
    if (partial) {
        for (int64_t c = threadIdx.x; c < D; c += blockDim.x) {
            float s = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                s += sdw[i * D + c];
            partial[blockIdx.x * D + c] = s;
        }
    }
}

// Row-parallel variants for D a multiple of 256: a row is spread over TPR =
// D/8 threads holding 8 elements each (two float4 at columns 4t and
// 4(t + TPR)), so x and dy are read once and kept in registers; row sums meet
// in shared memory. A block holds RPB = blockDim.x / TPR row slots.
constexpr int RMS_EPT = 8;

__device__ __forceinline__ float block_row_sum(float v, float* red, int slot, int t, int tpr,
                                               int parity) {
    v = warp_sum(v);
    const int wpr = tpr >> 5;  // warps per row
    float* rs = red + (parity * 8 + slot) * 32;
    if ((t & 31) == 0)
        rs[t >> 5] = v;
    __syncthreads();
    float tot = 0.0f;
    for (int i = 0; i < wpr; ++i)
        tot += rs[i];
    return tot;
}

// With `split` (bf16x3 GEMM operand planes [2][R][D], the ttk_gemm_split
// layout for D a multiple of 32) the kernel also writes the split of y, with
// the split kernel's arithmetic (split_bf16), so the planes equal
// ttk_gemm_split(y) bit for bit and the split pass before the GEMMs that
// read y is skipped.
__global__ void rmsnorm_fwd_rows_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                        float* __restrict__ y, float* __restrict__ rstd,
                                        int64_t R, int64_t D, float eps,
                                        __nv_bfloat16* __restrict__ split) {
    __shared__ float red[2 * 8 * 32];
    const int tpr = static_cast<int>(D / RMS_EPT);
    const int rpb = blockDim.x / tpr;
    const int slot = threadIdx.x / tpr, t = threadIdx.x % tpr;
    const int64_t c0 = 4 * static_cast<int64_t>(t), c1 = 4 * static_cast<int64_t>(t + tpr);
    const float4 w0 = *reinterpret_cast<const float4*>(w + c0);
    const float4 w1 = *reinterpret_cast<const float4*>(w + c1);
    // The next row's x is loaded before this row's reduction (two rows of
    // loads in flight per thread).
    auto load = [&](int64_t row, float4& a, float4& b) {
        a = b = make_float4(0.f, 0.f, 0.f, 0.f);
        if (row < R) {
            a = *reinterpret_cast<const float4*>(x + row * D + c0);
            b = *reinterpret_cast<const float4*>(x + row * D + c1);
        }
    };
    const int64_t step = static_cast<int64_t>(gridDim.x) * rpb;
    int parity = 0;
    float4 a, b;
    load(static_cast<int64_t>(blockIdx.x) * rpb + slot, a, b);
    for (int64_t base = static_cast<int64_t>(blockIdx.x) * rpb; base < R;
         base += step, parity ^= 1) {
        const int64_t row = base + slot;
        const bool ok = row < R;
        float4 na, nb;
        load(row + step, na, nb);
        const float ss = block_row_sum(a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w + b.x * b.x +
                                           b.y * b.y + b.z * b.z + b.w * b.w,
                                       red, slot, t, tpr, parity);
        if (ok) {
            const float r = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
            if (t == 0 && rstd)
                rstd[row] = r;
            const float4 y0 =
                make_float4(a.x * r * w0.x, a.y * r * w0.y, a.z * r * w0.z, a.w * r * w0.w);
            const float4 y1 =
                make_float4(b.x * r * w1.x, b.y * r * w1.y, b.z * r * w1.z, b.w * r * w1.w);
            *reinterpret_cast<float4*>(y + row * D + c0) = y0;
            *reinterpret_cast<float4*>(y + row * D + c1) = y1;
            if (split) {
                const int64_t plane = R * D;
                const float4 ys[2] = {y0, y1};
                const int64_t cs[2] = {c0, c1};
#pragma unroll
                for (int g = 0; g < 2; ++g) {
                    const float v[4] = {ys[g].x, ys[g].y, ys[g].z, ys[g].w};
                    __nv_bfloat16 hi[4], lo[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        split_bf16(v[j], hi[j], lo[j]);
                    __nv_bfloat16* d = split + row * D + cs[g];
                    *reinterpret_cast<uint2*>(d) = *reinterpret_cast<const uint2*>(hi);
                    *reinterpret_cast<uint2*>(d + plane) = *reinterpret_cast<const uint2*>(lo);
                }
            }
        }
        a = na, b = nb;
    }
}

// dx as rmsnorm_bwd_kernel; dw partial per row slot of each block:
// partial[blockIdx.x * RPB + slot][D] (rows in a fixed order).
__global__ void rmsnorm_bwd_rows_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                        const float* __restrict__ rstd,
                                        const float* __restrict__ dy, float* __restrict__ dx,
                                        int accumulate, float* __restrict__ partial, int64_t R,
                                        int64_t D) {
    __shared__ float red[2 * 8 * 32];
    const int tpr = static_cast<int>(D / RMS_EPT);
    const int rpb = blockDim.x / tpr;
    const int slot = threadIdx.x / tpr, t = threadIdx.x % tpr;
    const int64_t c0 = 4 * static_cast<int64_t>(t), c1 = 4 * static_cast<int64_t>(t + tpr);
    const float4 w0 = *reinterpret_cast<const float4*>(w + c0);
    const float4 w1 = *reinterpret_cast<const float4*>(w + c1);
    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    const bool acc = dx && accumulate;
    float dw[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    // One row's operands: x, dy, the dx being accumulated into, and rstd. The
    // next row's are loaded before this row's reduction, so two rows of loads
    // are in flight per thread.
    struct RowIn {
        float4 x0, x1, g0, g1, q0, q1;
        float r;
    };
    auto load = [&](int64_t row) {
        RowIn v;
        const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
        v.x0 = v.x1 = v.g0 = v.g1 = v.q0 = v.q1 = z;
        v.r = 0.0f;
        if (row < R) {
            v.x0 = *reinterpret_cast<const float4*>(x + row * D + c0);
            v.x1 = *reinterpret_cast<const float4*>(x + row * D + c1);
            v.g0 = *reinterpret_cast<const float4*>(dy + row * D + c0);
            v.g1 = *reinterpret_cast<const float4*>(dy + row * D + c1);
            if (acc) {
                v.q0 = *reinterpret_cast<const float4*>(dx + row * D + c0);
                v.q1 = *reinterpret_cast<const float4*>(dx + row * D + c1);
            }
            v.r = rstd[row];
        }
        return v;
    };
    const int64_t step = static_cast<int64_t>(gridDim.x) * rpb;
    int parity = 0;
    RowIn cur = load(static_cast<int64_t>(blockIdx.x) * rpb + slot);
    for (int64_t base = static_cast<int64_t>(blockIdx.x) * rpb; base < R;
         base += step, parity ^= 1) {
        const int64_t row = base + slot;
        const bool ok = row < R;
        const RowIn nxt = load(row + step);
        const float xv[8] = {cur.x0.x, cur.x0.y, cur.x0.z, cur.x0.w,
                             cur.x1.x, cur.x1.y, cur.x1.z, cur.x1.w};
        const float gv[8] = {cur.g0.x, cur.g0.y, cur.g0.z, cur.g0.w,
                             cur.g1.x, cur.g1.y, cur.g1.z, cur.g1.w};
        const float r = cur.r;
        float dot = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e)
            dot += gv[e] * wv[e] * xv[e];
        dot = block_row_sum(dot, red, slot, t, tpr, parity);
        if (ok) {
            const float k = r * r * r / static_cast<float>(D) * dot;
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                o[e] = r * (gv[e] * wv[e]) - xv[e] * k;
                dw[e] += gv[e] * xv[e] * r;
            }
            if (dx) {
                if (acc) {
                    o[0] += cur.q0.x, o[1] += cur.q0.y, o[2] += cur.q0.z, o[3] += cur.q0.w;
                    o[4] += cur.q1.x, o[5] += cur.q1.y, o[6] += cur.q1.z, o[7] += cur.q1.w;
                }
                *reinterpret_cast<float4*>(dx + row * D + c0) = make_float4(o[0], o[1], o[2], o[3]);
                *reinterpret_cast<float4*>(dx + row * D + c1) = make_float4(o[4], o[5], o[6], o[7]);
            }
        }
        cur = nxt;
    }
    if (partial) {
        float* pr = partial + (static_cast<int64_t>(blockIdx.x) * rpb + slot) * D;
        *reinterpret_cast<float4*>(pr + c0) = make_float4(dw[0], dw[1], dw[2], dw[3]);
        *reinterpret_cast<float4*>(pr + c1) = make_float4(dw[4], dw[5], dw[6], dw[7]);
    }
}

// dw[c] += sum_b partial[b][c] over nb partial rows. A block of 16 warps owns
// 32 adjacent columns (one per lane, 128-byte row segments); warp w sums rows
// b = w, w + 16, ... in ascending order and the sixteen warp sums are added
// in warp order: a fixed summation order, so the result is deterministic.
constexpr int COLSUM_THREADS = 512;
__global__ void __launch_bounds__(COLSUM_THREADS) colsum_kernel(const float* __restrict__ partial,
                                                                int64_t nb, int64_t D,
                                                                float* __restrict__ out) {
    constexpr int NW = COLSUM_THREADS / 32;
    __shared__ float red[NW][32];
    const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
    for (int64_t cb = static_cast<int64_t>(blockIdx.x) * 32; cb < D;
         cb += static_cast<int64_t>(gridDim.x) * 32) {
        const int64_t c = cb + lane;
        float s = 0.0f;
        if (c < D) {
#pragma unroll 8
            for (int64_t b = wp; b < nb; b += NW)
                s += partial[b * D + c];
        }
        red[wp][lane] = s;
        __syncthreads();
        if (wp == 0 && c < D) {
            float tot = 0.0f;
#pragma unroll
            for (int i = 0; i < NW; ++i)
                tot += red[i][lane];
            out[c] += tot;
        }
        __syncthreads();
    }
}

// -------------------------------------------------------------- SwiGLU --
__device__ __forceinline__ float silu_f(float a) { return a / (1.0f + expf(-a)); }

__global__ void swiglu_fwd_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                  float* __restrict__ y, int64_t n) {
    const int64_t n4 = n / 4;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
         i += stride) {
        float4 av = reinterpret_cast<const float4*>(a)[i];
        float4 bv = reinterpret_cast<const float4*>(b)[i];
        reinterpret_cast<float4*>(y)[i] = make_float4(silu_f(av.x) * bv.x, silu_f(av.y) * bv.y,
                                                      silu_f(av.z) * bv.z, silu_f(av.w) * bv.w);
    }
    for (int64_t i = n4 * 4 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += stride)
        y[i] = silu_f(a[i]) * b[i];
}

__device__ __forceinline__ void swiglu_grad(float a, float b, float g, float& da, float& db) {
    const float s = 1.0f / (1.0f + expf(-a));
    da = (g * b) * (s * (1.0f + a * (1.0f - s)));
    db = g * (a / (1.0f + expf(-a)));
}

// SwiGLU forward / backward writing their results only as bf16x3 GEMM
// operand planes: [2][R][ldp] bf16 (hi plane, then lo), ldp = F rounded up to
// 32, columns [F, ldp) zero; the layout of ttk_gemm_split. The fp32 values
// are computed exactly as swiglu_fwd_kernel / swiglu_bwd_kernel compute them,
// and split with split_bf16 as the split kernel does, so the planes equal
// those of the unfused pair bit for bit. Launch shape: TPR threads per row,
// 256 / TPR rows per block sweep (F % 4 == 0).
__device__ __forceinline__ void store_split4(__nv_bfloat16* hi, int64_t plane, const float (&v)[4]) {
    __nv_bfloat16 h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
        split_bf16(v[j], h[j], l[j]);
    *reinterpret_cast<uint2*>(hi) = *reinterpret_cast<const uint2*>(h);
    *reinterpret_cast<uint2*>(hi + plane) = *reinterpret_cast<const uint2*>(l);
}

__global__ void swiglu_fwd_split_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                        __nv_bfloat16* __restrict__ ys, int64_t R, int64_t F,
                                        int64_t ldp, int tpr) {
    const int rpb = blockDim.x / tpr;
    const int lr = threadIdx.x / tpr, lg = threadIdx.x % tpr;
    const int64_t plane = R * ldp;
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * rpb + lr; r < R;
         r += static_cast<int64_t>(gridDim.x) * rpb) {
        for (int64_t g = lg; g < ldp / 4; g += tpr) {
            const int64_t c = g * 4;
            float y[4] = {0.f, 0.f, 0.f, 0.f};
            if (c < F) {
                const float4 av = *reinterpret_cast<const float4*>(a + r * F + c);
                const float4 bv = *reinterpret_cast<const float4*>(b + r * F + c);
                y[0] = silu_f(av.x) * bv.x, y[1] = silu_f(av.y) * bv.y;
                y[2] = silu_f(av.z) * bv.z, y[3] = silu_f(av.w) * bv.w;
            }
            store_split4(ys + r * ldp + c, plane, y);
        }
    }
}

__global__ void swiglu_bwd_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                  const float* __restrict__ dy, float* __restrict__ da,
                                  float* __restrict__ db, int accumulate, int64_t n) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t n4 = n / 4;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
         i += stride) {
        float4 av = reinterpret_cast<const float4*>(a)[i];
        float4 bv = reinterpret_cast<const float4*>(b)[i];
        float4 gv = reinterpret_cast<const float4*>(dy)[i];
        float4 oa, ob;
        swiglu_grad(av.x, bv.x, gv.x, oa.x, ob.x);
        swiglu_grad(av.y, bv.y, gv.y, oa.y, ob.y);
        swiglu_grad(av.z, bv.z, gv.z, oa.z, ob.z);
        swiglu_grad(av.w, bv.w, gv.w, oa.w, ob.w);
        if (accumulate) {
            float4 pa = reinterpret_cast<float4*>(da)[i];
            float4 pb = reinterpret_cast<float4*>(db)[i];
            oa.x += pa.x, oa.y += pa.y, oa.z += pa.z, oa.w += pa.w;
            ob.x += pb.x, ob.y += pb.y, ob.z += pb.z, ob.w += pb.w;
        }
        reinterpret_cast<float4*>(da)[i] = oa;
        reinterpret_cast<float4*>(db)[i] = ob;
    }
    for (int64_t i = n4 * 4 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += stride) {
        float oa, ob;
        swiglu_grad(a[i], b[i], dy[i], oa, ob);
        da[i] = accumulate ? da[i] + oa : oa;
        db[i] = accumulate ? db[i] + ob : ob;
    }
}

__global__ void swiglu_bwd_split_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                        const float* __restrict__ dy,
                                        __nv_bfloat16* __restrict__ das,
                                        __nv_bfloat16* __restrict__ dbs, int64_t R, int64_t F,
                                        int64_t ldp, int tpr) {
    const int rpb = blockDim.x / tpr;
    const int lr = threadIdx.x / tpr, lg = threadIdx.x % tpr;
    const int64_t plane = R * ldp;
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * rpb + lr; r < R;
         r += static_cast<int64_t>(gridDim.x) * rpb) {
        for (int64_t g = lg; g < ldp / 4; g += tpr) {
            const int64_t c = g * 4;
            float da[4] = {0.f, 0.f, 0.f, 0.f}, db[4] = {0.f, 0.f, 0.f, 0.f};
            if (c < F) {
                const float4 av = *reinterpret_cast<const float4*>(a + r * F + c);
                const float4 bv = *reinterpret_cast<const float4*>(b + r * F + c);
                const float4 gv = *reinterpret_cast<const float4*>(dy + r * F + c);
                swiglu_grad(av.x, bv.x, gv.x, da[0], db[0]);
                swiglu_grad(av.y, bv.y, gv.y, da[1], db[1]);
                swiglu_grad(av.z, bv.z, gv.z, da[2], db[2]);
                swiglu_grad(av.w, bv.w, gv.w, da[3], db[3]);
            }
            store_split4(das + r * ldp + c, plane, da);
            store_split4(dbs + r * ldp + c, plane, db);
        }
    }
}

// ------------------------------------------------------- cross-entropy --
// One 1024-thread block per row; the row (C <= 32768) stays in registers
// between the max / sum-exp reduction and the gradient write.
constexpr int CE_THREADS = 1024;
constexpr int CE_VEC = 8;  // float4 per thread -> 32768 floats per row

template <bool IN_REGS>
__global__ void __launch_bounds__(CE_THREADS, 1)
    cross_entropy_kernel(const float* __restrict__ logits, const int64_t* __restrict__ targets,
                         int64_t N, int64_t C, double* __restrict__ loss_acc,
                         float* __restrict__ dlogits, float grad_scale) {
    __shared__ float s_red[32];
    __shared__ double s_redd[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool vec = (C & 3) == 0;
    for (int64_t row = blockIdx.x; row < N; row += gridDim.x) {
        const float* xr = logits + row * C;
        const int64_t t = targets[row];
        const bool t_ok = t >= 0 && t < C;
        // The target's logit is read before the first barrier of the row: no
        // thread writes the row's gradient before the second one, so the
        // read sees the logit even when dlogits aliases logits.
        const float x_t = (threadIdx.x == 0 && t_ok) ? xr[t] : 0.0f;
        float v[IN_REGS ? CE_VEC * 4 : 1];
        float m = -INFINITY;
        if (IN_REGS) {
#pragma unroll
            for (int j = 0; j < CE_VEC; ++j) {
                const int64_t c = (static_cast<int64_t>(j) * CE_THREADS + threadIdx.x) * 4;
                float4 t4;
                if (vec && c + 4 <= C) {
                    t4 = __ldg(reinterpret_cast<const float4*>(xr + c));
                } else {
                    t4.x = c < C ? xr[c] : -INFINITY;
                    t4.y = c + 1 < C ? xr[c + 1] : -INFINITY;
                    t4.z = c + 2 < C ? xr[c + 2] : -INFINITY;
                    t4.w = c + 3 < C ? xr[c + 3] : -INFINITY;
                }
                v[4 * j] = t4.x, v[4 * j + 1] = t4.y, v[4 * j + 2] = t4.z, v[4 * j + 3] = t4.w;
                m = fmaxf(m, fmaxf(fmaxf(t4.x, t4.y), fmaxf(t4.z, t4.w)));
            }
        } else {
            for (int64_t c = threadIdx.x; c < C; c += CE_THREADS)
                m = fmaxf(m, xr[c]);
        }
        m = warp_max(m);
        if (lane == 0)
            s_red[warp] = m;
        __syncthreads();
        m = s_red[lane];
        m = warp_max(m);
        __syncthreads();
        double s = 0.0;
        if (IN_REGS) {
#pragma unroll
            for (int j = 0; j < CE_VEC * 4; ++j)
                s += static_cast<double>(expf(v[j] - m));  // exp(-inf) = 0 for padding
        } else {
            for (int64_t c = threadIdx.x; c < C; c += CE_THREADS)
                s += static_cast<double>(expf(xr[c] - m));
        }
        s = warp_sum_d(s);
        if (lane == 0)
            s_redd[warp] = s;
        __syncthreads();
        s = s_redd[lane];
        s = warp_sum_d(s);
        const float lse = m + static_cast<float>(log(s));
        if (threadIdx.x == 0) {
            if (t_ok)
                atomicAdd(loss_acc, static_cast<double>(-(x_t - lse)));
            else
                report(kErrBadIndex);
        }
        if (dlogits) {
            float* dr = dlogits + row * C;
            if (IN_REGS) {
#pragma unroll
                for (int j = 0; j < CE_VEC; ++j) {
                    const int64_t c = (static_cast<int64_t>(j) * CE_THREADS + threadIdx.x) * 4;
                    float o[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float p = expf(v[4 * j + q] - lse);
                        o[q] = grad_scale * (c + q == t ? p - 1.0f : p);
                    }
                    if (vec && c + 4 <= C) {
                        *reinterpret_cast<float4*>(dr + c) = make_float4(o[0], o[1], o[2], o[3]);
                    } else {
                        for (int q = 0; q < 4; ++q)
                            if (c + q < C)
                                dr[c + q] = o[q];
                    }
                }
            } else {
                for (int64_t c = threadIdx.x; c < C; c += CE_THREADS) {
                    const float p = expf(xr[c] - lse);
                    dr[c] = grad_scale * (c == t ? p - 1.0f : p);
                }
            }
        }
        __syncthreads();
    }
}

// Rows of at most 32768 logits with C a multiple of 4: the same arithmetic as
// cross_entropy_kernel<true> (identical results), with the next row streamed
// into shared memory by one bulk copy while the current row is reduced and
// its gradient written, so the row reads overlap the gradient writes. One
// 1024-thread block per SM. Thread 0 waits on the copy's mbarrier with the
// bounded wait; on expiry the block stops (device status set) after waiting
// once more for the copy it issued.
__global__ void __launch_bounds__(CE_THREADS, 1)
    cross_entropy_bulk_kernel(const float* __restrict__ logits,
                              const int64_t* __restrict__ targets, int64_t N, int64_t C,
                              double* __restrict__ loss_acc, float* __restrict__ dlogits,
                              float grad_scale) {
    extern __shared__ __align__(16) float srow[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ float s_red[32];
    __shared__ double s_redd[32];
    __shared__ int s_ok;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t bytes = static_cast<uint32_t>(C) * 4u;
    int64_t row = blockIdx.x;
    if (row >= N)
        return;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
        mbar_arrive_expect_tx(&bar, bytes);
        bulk_load(srow, logits + row * C, bytes, &bar);
    }
    uint32_t phase = 0;
    for (; row < N; row += gridDim.x) {
        if (threadIdx.x == 0)
            s_ok = mbar_wait(&bar, phase, 80) ? 1 : 0;
        __syncthreads();
        if (!s_ok) {
            if (threadIdx.x == 0)
                mbar_wait(&bar, phase, 81);  // the copy in flight lands before exit
            return;
        }
        phase ^= 1u;
        const int64_t t = targets[row];
        const bool t_ok = t >= 0 && t < C;
        const float x_t = (threadIdx.x == 0 && t_ok) ? srow[t] : 0.0f;
        float v[CE_VEC * 4];
        float m = -INFINITY;
#pragma unroll
        for (int j = 0; j < CE_VEC; ++j) {
            const int64_t c = (static_cast<int64_t>(j) * CE_THREADS + threadIdx.x) * 4;
            float4 t4 = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
            if (c < C)
                t4 = *reinterpret_cast<const float4*>(srow + c);
            v[4 * j] = t4.x, v[4 * j + 1] = t4.y, v[4 * j + 2] = t4.z, v[4 * j + 3] = t4.w;
            m = fmaxf(m, fmaxf(fmaxf(t4.x, t4.y), fmaxf(t4.z, t4.w)));
        }
        __syncthreads();  // every thread has its part of the row: the buffer is free
        if (threadIdx.x == 0 && row + gridDim.x < N) {
            fence_async_smem();
            mbar_arrive_expect_tx(&bar, bytes);
            bulk_load(srow, logits + (row + gridDim.x) * C, bytes, &bar);
        }
        m = warp_max(m);
        if (lane == 0)
            s_red[warp] = m;
        __syncthreads();
        m = s_red[lane];
        m = warp_max(m);
        __syncthreads();
        double sd = 0.0;
#pragma unroll
        for (int j = 0; j < CE_VEC * 4; ++j)
            sd += static_cast<double>(expf(v[j] - m));  // exp(-inf) = 0 for padding
        sd = warp_sum_d(sd);
        if (lane == 0)
            s_redd[warp] = sd;
        __syncthreads();
        sd = s_redd[lane];
        sd = warp_sum_d(sd);
        const float lse = m + static_cast<float>(log(sd));
        if (threadIdx.x == 0) {
            if (t_ok)
                atomicAdd(loss_acc, static_cast<double>(-(x_t - lse)));
            else
                report(kErrBadIndex);
        }
        if (dlogits) {
            float* dr = dlogits + row * C;
#pragma unroll
            for (int j = 0; j < CE_VEC; ++j) {
                const int64_t c = (static_cast<int64_t>(j) * CE_THREADS + threadIdx.x) * 4;
                if (c < C) {
                    float o[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float p = expf(v[4 * j + q] - lse);
                        o[q] = grad_scale * (c + q == t ? p - 1.0f : p);
                    }
                    *reinterpret_cast<float4*>(dr + c) = make_float4(o[0], o[1], o[2], o[3]);
                }
            }
        }
        __syncthreads();  // s_red / s_redd reused by the next row
    }
}

__global__ void loss_finalize_kernel(const double* acc, float scale, float* out) {
    out[0] = static_cast<float>(acc[0] * static_cast<double>(scale));
}

// ----------------------------------------------------------- embedding --
__global__ void embedding_fwd_kernel(const float* __restrict__ W, const int64_t* __restrict__ idx,
                                     float* __restrict__ out, int64_t N, int64_t D, int64_t V) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    const bool vec = (D & 3) == 0;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
         i < N; i += warps) {
        const int64_t t = idx[i];
        if (t < 0 || t >= V) {
            if (lane == 0)
                report(kErrBadIndex);
            continue;
        }
        const float* src = W + t * D;
        float* dst = out + i * D;
        if (vec) {
            for (int64_t c = lane * 4; c < D; c += 128)
                *reinterpret_cast<float4*>(dst + c) = *reinterpret_cast<const float4*>(src + c);
        } else {
            for (int64_t c = lane; c < D; c += 32)
                dst[c] = src[c];
        }
    }
}

// Keys (id << 32 | position) sorted ascending give, per id, its positions in
// ascending order: the reference's accumulation order (ops.cpp:766-771).
__global__ void make_keys_kernel(const int64_t* __restrict__ idx, int64_t N, int64_t Npow2,
                                 uint64_t* __restrict__ keys) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < Npow2;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        keys[i] = i < N ? (static_cast<uint64_t>(idx[i]) << 32) | static_cast<uint64_t>(i)
                        : ~0ull;
}

// Bitonic sort of Npow2 keys held in shared memory by one block.
__global__ void bitonic_smem_kernel(uint64_t* __restrict__ keys, int64_t Npow2) {
    extern __shared__ uint64_t sk[];
    for (int64_t i = threadIdx.x; i < Npow2; i += blockDim.x)
        sk[i] = keys[i];
    __syncthreads();
    for (int64_t k = 2; k <= Npow2; k <<= 1) {
        for (int64_t j = k >> 1; j > 0; j >>= 1) {
            for (int64_t i = threadIdx.x; i < Npow2; i += blockDim.x) {
                const int64_t p = i ^ j;
                if (p > i) {
                    const bool up = (i & k) == 0;
                    const uint64_t a = sk[i], b = sk[p];
                    if ((a > b) == up) {
                        sk[i] = b;
                        sk[p] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
    for (int64_t i = threadIdx.x; i < Npow2; i += blockDim.x)
        keys[i] = sk[i];
}

// Stages of a global bitonic sort that stay inside chunks of BITONIC_CHUNK
// keys, each chunk in one block's shared memory. Directions use the global
// index (i & k), so the passes are those of the global network:
//   first = 1: every stage k <= BITONIC_CHUNK (the chunks sorted in
//              alternating directions);
//   first = 0: the passes j < BITONIC_CHUNK of stage k (after the global
//              passes j >= BITONIC_CHUNK of that stage).
constexpr int64_t BITONIC_CHUNK = 8192;

__global__ void __launch_bounds__(1024)
    bitonic_chunk_kernel(uint64_t* __restrict__ keys, int64_t k_stage, int first) {
    extern __shared__ uint64_t ck[];
    const int64_t base = static_cast<int64_t>(blockIdx.x) * BITONIC_CHUNK;
    for (int64_t i = threadIdx.x; i < BITONIC_CHUNK; i += blockDim.x)
        ck[i] = keys[base + i];
    __syncthreads();
    auto pass = [&](int64_t k, int64_t j) {
        for (int64_t i = threadIdx.x; i < BITONIC_CHUNK; i += blockDim.x) {
            const int64_t p = i ^ j;
            if (p > i) {
                const bool up = ((base + i) & k) == 0;
                const uint64_t a = ck[i], b = ck[p];
                if ((a > b) == up) {
                    ck[i] = b;
                    ck[p] = a;
                }
            }
        }
        __syncthreads();
    };
    if (first) {
        for (int64_t k = 2; k <= BITONIC_CHUNK; k <<= 1)
            for (int64_t j = k >> 1; j > 0; j >>= 1)
                pass(k, j);
    } else {
        for (int64_t j = BITONIC_CHUNK >> 1; j > 0; j >>= 1)
            pass(k_stage, j);
    }
    for (int64_t i = threadIdx.x; i < BITONIC_CHUNK; i += blockDim.x)
        keys[base + i] = ck[i];
}

// One compare-exchange pass (k, j) of a global-memory bitonic sort.
__global__ void bitonic_global_kernel(uint64_t* __restrict__ keys, int64_t Npow2, int64_t k,
                                      int64_t j) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < Npow2;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t p = i ^ j;
        if (p > i) {
            const bool up = (i & k) == 0;
            const uint64_t a = keys[i], b = keys[p];
            if ((a > b) == up) {
                keys[i] = b;
                keys[p] = a;
            }
        }
    }
}

// One warp per sorted position; the warp that starts a run of equal ids adds
// the run's gradient rows into dW[id] sequentially, in position order.
__global__ void embedding_segment_kernel(const uint64_t* __restrict__ keys, int64_t N,
                                         const float* __restrict__ dout, float* __restrict__ dW,
                                         int64_t D, int64_t V) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
         p < N; p += warps) {
        const uint64_t id = keys[p] >> 32;
        if (p > 0 && (keys[p - 1] >> 32) == id)
            continue;
        if (id >= static_cast<uint64_t>(V)) {
            if (lane == 0)
                report(kErrBadIndex);
            continue;
        }
        int64_t end = p + 1;
        while (end < N && (keys[end] >> 32) == id)
            ++end;
        float* drow = dW + static_cast<int64_t>(id) * D;
        for (int64_t c = lane; c < D; c += 32) {
            float acc = drow[c];
            for (int64_t q = p; q < end; ++q) {
                const int64_t pos = static_cast<int64_t>(keys[q] & 0xffffffffull);
                acc += dout[pos * D + c];
            }
            drow[c] = acc;
        }
    }
}

__global__ void index_check_kernel(const int64_t* __restrict__ idx, int64_t n, int64_t V,
                                   unsigned long long* __restrict__ bad) {
    unsigned long long cnt = 0;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        cnt += (idx[i] < 0 || idx[i] >= V) ? 1 : 0;
    if (cnt)
        atomicAdd(bad, cnt);
}

// ---------------------------------------------------------------- RoPE --
// x [B,T,H,D], cos/sin [T,D/2]; pair (d, d + D/2) rotated (ops.cpp:970-999).
__global__ void rope_kernel(const float* __restrict__ x, const float* __restrict__ cs,
                            const float* __restrict__ sn, float* __restrict__ y, int accumulate,
                            int backward, int64_t B, int64_t T, int64_t H, int64_t D) {
    const int64_t Dh = D / 2;
    const int64_t total = B * T * H * Dh;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t d = i % Dh;
        const int64_t bth = i / Dh;
        const int64_t t = (bth / H) % T;
        const int64_t base = bth * D;
        const float x1 = x[base + d], x2 = x[base + Dh + d];
        const float c = cs[t * Dh + d], s = sn[t * Dh + d];
        float o1, o2;
        if (!backward) {
            o1 = x1 * c - x2 * s;
            o2 = x1 * s + x2 * c;
        } else {  // transpose rotation (ops.cpp:1020-1021)
            o1 = x1 * c + x2 * s;
            o2 = -x1 * s + x2 * c;
        }
        if (accumulate) {
            y[base + d] += o1;
            y[base + Dh + d] += o2;
        } else {
            y[base + d] = o1;
            y[base + Dh + d] = o2;
        }
    }
}

// -------------------------------------------------------------- softmax --
// One warp per row; two passes over the row (max; sum in double; write).
__global__ void softmax_fwd_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t R,
                                   int64_t C, int log_out) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
         row < R; row += warps) {
        const float* xr = x + row * C;
        float* yr = y + row * C;
        float m = -1e30f;  // the reference's initial max (ops.cpp:794)
        for (int64_t c = lane; c < C; c += 32)
            m = fmaxf(m, xr[c]);
        m = warp_max(m);
        double s = 0.0;
        for (int64_t c = lane; c < C; c += 32)
            s += static_cast<double>(expf(xr[c] - m));
        s = warp_sum_d(s);
        if (log_out) {
            const float lse = m + static_cast<float>(log(s));
            for (int64_t c = lane; c < C; c += 32)
                yr[c] = xr[c] - lse;
        } else {
            const float inv = static_cast<float>(1.0 / s);
            for (int64_t c = lane; c < C; c += 32)
                yr[c] = expf(xr[c] - m) * inv;
        }
    }
}

// softmax: dx (+)= y*(dy - sum(dy*y)); log_softmax: dx (+)= dy - exp(y)*sum(dy).
__global__ void softmax_bwd_kernel(const float* __restrict__ y, const float* __restrict__ dy,
                                   float* __restrict__ dx, int accumulate, int64_t R, int64_t C,
                                   int log_in) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
         row < R; row += warps) {
        const float* yr = y + row * C;
        const float* gr = dy + row * C;
        float* dr = dx + row * C;
        double s = 0.0;
        for (int64_t c = lane; c < C; c += 32)
            s += log_in ? static_cast<double>(gr[c])
                        : static_cast<double>(gr[c]) * static_cast<double>(yr[c]);
        s = warp_sum_d(s);
        const float sf = static_cast<float>(s);
        for (int64_t c = lane; c < C; c += 32) {
            const float v = log_in ? gr[c] - expf(yr[c]) * sf : yr[c] * (gr[c] - sf);
            dr[c] = accumulate ? dr[c] + v : v;
        }
    }
}

// ----------------------------------------------------------------- NLL --
// loss = -sum_i lp[i, t_i] / N with a double accumulator in i order
// (ops.cpp:905-912); one block, deterministic.
__global__ void nll_fwd_kernel(const float* __restrict__ lp, const int64_t* __restrict__ t,
                               int64_t N, int64_t C, float* __restrict__ out) {
    __shared__ double sh[32];
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < N; i += blockDim.x) {
        const int64_t c = t[i];
        if (c >= 0 && c < C)
            s -= static_cast<double>(lp[i * C + c]);
        else
            report(kErrBadIndex);
    }
    s = warp_sum_d(s);
    if ((threadIdx.x & 31) == 0)
        sh[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        s = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0;
        s = warp_sum_d(s);
        if (threadIdx.x == 0)
            out[0] = static_cast<float>(s / static_cast<double>(N));
    }
}

// dlp[i, t_i] -= g[0] / N (ops.cpp:918-923).
__global__ void nll_bwd_kernel(const int64_t* __restrict__ t, int64_t N, int64_t C,
                               const float* __restrict__ g, float* __restrict__ dlp) {
    const float gv = g[0] / static_cast<float>(N);
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < N;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t c = t[i];
        if (c >= 0 && c < C)
            dlp[i * C + c] -= gv;
    }
}

// Gradients of the RoPE tables (ops.cpp:1024-1048): per (t, d), summed over
// b and h in ascending order.
__global__ void rope_table_grad_kernel(const float* __restrict__ x, const float* __restrict__ g,
                                       int64_t B, int64_t T, int64_t H, int64_t D,
                                       float* __restrict__ dcos, float* __restrict__ dsin) {
    const int64_t Dh = D / 2;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < T * Dh;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = i / Dh, d = i % Dh;
        float sc = 0.0f, ss = 0.0f;
        for (int64_t b = 0; b < B; ++b)
            for (int64_t h = 0; h < H; ++h) {
                const int64_t base = ((b * T + t) * H + h) * D;
                const float x1 = x[base + d], x2 = x[base + Dh + d];
                const float g1 = g[base + d], g2 = g[base + Dh + d];
                sc += g1 * x1 + g2 * x2;
                ss += -g1 * x2 + g2 * x1;
            }
        if (dcos)
            dcos[i] += sc;
        if (dsin)
            dsin[i] += ss;
    }
}

// y (+)= alpha[0] * x with alpha read on the device.
__global__ void axpy_dev_kernel(const float* __restrict__ alpha, const float* __restrict__ x,
                                float* __restrict__ y, int64_t n, int accumulate) {
    const float a = alpha[0];
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] = accumulate ? y[i] + a * x[i] : a * x[i];
}

}  // namespace nn
}  // namespace ttk

using namespace ttk;
using namespace ttk::nn;

static inline cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Row-parallel RMSNorm applies when D is a multiple of 256 (whole warps per
// row) and a row fits one block of at most 1024 threads.
static inline bool rms_rows_ok(int64_t D) { return D % 256 == 0 && D / RMS_EPT <= 1024; }
static inline int rms_block(int64_t D) {  // threads per block: whole rows, up to 256 (or one row)
    const int tpr = static_cast<int>(D / RMS_EPT);
    return tpr >= 256 ? tpr : tpr * (256 / tpr);
}

// Blocks of `kernel` (bs threads, static shared memory only) that are
// resident at once on all SMs of the current device: the row kernels loop
// over rows with a grid stride, so a grid of exactly one resident wave keeps
// every SM busy to the end (a grid of 1.6 waves left 40% of the SMs idle for
// the second wave's duration). Cached per device and block size.
template <class Kernel>
static int64_t resident_grid(Kernel kernel, int bs, int slot) {
    constexpr int kDevs = 16, kSlots = 2, kSizes = 33;
    static std::atomic<int> cache[kDevs][kSlots][kSizes];  // zero-initialized (static)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess)
        dev = 0;
    const int bi = bs / 32;
    std::atomic<int>* c =
        (dev < kDevs && slot < kSlots && bi < kSizes && bs % 32 == 0) ? &cache[dev][slot][bi]
                                                                      : nullptr;
    if (c) {
        const int v = c->load(std::memory_order_relaxed);
        if (v > 0)
            return v;
    }
    int sms = 0, per = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        sms <= 0)
        sms = 148;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kernel, bs, 0) != cudaSuccess ||
        per <= 0) {
        cudaGetLastError();
        per = 2;
    }
    const int n = sms * per;
    if (c)
        c->store(n, std::memory_order_relaxed);
    return n;
}

extern "C" {

int ttk_rmsnorm_fwd(const float* x, const float* w, float* y, float* rstd, int64_t R, int64_t D,
                    float eps, void* stream) {
    if (R < 0 || D <= 0 || !x || !w || !y)
        return set_error(TTK_ERR_ARG, "rmsnorm_fwd: bad arguments");
    if (R == 0)
        return TTK_OK;
    if ((D & 3) == 0 && !(aligned16(x) && aligned16(w) && aligned16(y)))
        return set_error(TTK_ERR_ARG, "rmsnorm_fwd: tensors must be 16-byte aligned");
    if (rms_rows_ok(D)) {
        const int tpr = static_cast<int>(D / RMS_EPT), bs = rms_block(D);
        const int64_t blocks = std::min<int64_t>((R + bs / tpr - 1) / (bs / tpr),
                                                 resident_grid(rmsnorm_fwd_rows_kernel, bs, 0));
        rmsnorm_fwd_rows_kernel<<<static_cast<int>(blocks), bs, 0, S(stream)>>>(x, w, y, rstd, R,
                                                                                 D, eps, nullptr);
        return check_launch("rmsnorm_fwd_rows_kernel");
    }
    rmsnorm_fwd_kernel<<<grid_for(R, 8), 256, 0, S(stream)>>>(x, w, y, rstd, R, D, eps);
    return check_launch("rmsnorm_fwd_kernel");
}

int ttk_rmsnorm_fwd_split(const float* x, const float* w, float* y, float* rstd, int64_t R,
                          int64_t D, float eps, void* split, void* stream) {
    if (R < 0 || D <= 0 || !x || !w || !y || !split)
        return set_error(TTK_ERR_ARG, "rmsnorm_fwd_split: bad arguments");
    if (!rms_rows_ok(D))
        return set_error(TTK_ERR_ARG, "rmsnorm_fwd_split: D must be a multiple of 256");
    if (ttk_gemm_get_precision() != 0)
        return set_error(TTK_ERR_ARG, "rmsnorm_fwd_split: planes exist for the bf16x3 precision");
    if (!(aligned16(x) && aligned16(w) && aligned16(y) && aligned16(split)))
        return set_error(TTK_ERR_ARG, "rmsnorm_fwd_split: tensors must be 16-byte aligned");
    if (R == 0)
        return TTK_OK;
    const int tpr = static_cast<int>(D / RMS_EPT), bs = rms_block(D);
    const int64_t blocks = std::min<int64_t>((R + bs / tpr - 1) / (bs / tpr),
                                             resident_grid(rmsnorm_fwd_rows_kernel, bs, 0));
    rmsnorm_fwd_rows_kernel<<<static_cast<int>(blocks), bs, 0, S(stream)>>>(
        x, w, y, rstd, R, D, eps, static_cast<__nv_bfloat16*>(split));
    return check_launch("rmsnorm_fwd_rows_kernel");
}

static int colsum_grid(int64_t D) {
    return static_cast<int>(std::min<int64_t>((D + 31) / 32, 148 * 8));
}

static int64_t rms_blocks(int64_t R) { return std::min<int64_t>(std::max<int64_t>(R / 64, 1), 296); }

// Row-parallel backward: blocks (one resident wave) and dw partial rows (one
// per row slot).
static int64_t rms_rows_blocks(int64_t R, int64_t D) {
    const int bs = rms_block(D);
    const int rpb = bs / static_cast<int>(D / RMS_EPT);
    return std::min<int64_t>((R + rpb - 1) / rpb, resident_grid(rmsnorm_bwd_rows_kernel, bs, 1));
}

size_t ttk_rmsnorm_bwd_workspace_size(int64_t R, int64_t D) {
    if (rms_rows_ok(D)) {
        const int rpb = rms_block(D) / static_cast<int>(D / RMS_EPT);
        return static_cast<size_t>(rms_rows_blocks(R, D) * rpb * D) * sizeof(float);
    }
    return static_cast<size_t>(rms_blocks(R) * D) * sizeof(float);
}

int ttk_rmsnorm_bwd(const float* x, const float* w, const float* rstd, const float* dy, float* dx,
                    int accumulate_dx, float* dw, int64_t R, int64_t D, void* workspace,
                    size_t workspace_bytes, void* stream) {
    if (R < 0 || D <= 0 || !x || !w || !rstd || !dy)
        return set_error(TTK_ERR_ARG, "rmsnorm_bwd: bad arguments");
    if (R == 0)
        return TTK_OK;
    float* partial = nullptr;
    if (dw) {
        if (!workspace || workspace_bytes < ttk_rmsnorm_bwd_workspace_size(R, D))
            return set_error(TTK_ERR_ARG, "rmsnorm_bwd: workspace too small");
        partial = static_cast<float*>(workspace);
    }
    if (rms_rows_ok(D) && aligned16(x) && aligned16(w) && aligned16(dy) && (!dx || aligned16(dx))) {
        const int bs = rms_block(D);
        const int64_t nbk = rms_rows_blocks(R, D);
        rmsnorm_bwd_rows_kernel<<<static_cast<int>(nbk), bs, 0, S(stream)>>>(
            x, w, rstd, dy, dx, accumulate_dx, partial, R, D);
        int rc = check_launch("rmsnorm_bwd_rows_kernel");
        if (rc || !dw)
            return rc;
        const int64_t nparts = nbk * (bs / static_cast<int>(D / RMS_EPT));
        colsum_kernel<<<colsum_grid(D), COLSUM_THREADS, 0, S(stream)>>>(partial, nparts, D, dw);
        return check_launch("colsum_kernel");
    }
    const int64_t nb = rms_blocks(R);
    const int64_t rpb = (R + nb - 1) / nb;
    const size_t smem = static_cast<size_t>(8 * D) * sizeof(float);
    if (smem > 200 * 1024)
        return set_error(TTK_ERR_ARG, "rmsnorm_bwd: D too large");
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(rmsnorm_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    rmsnorm_bwd_kernel<<<static_cast<int>(nb), 256, smem, S(stream)>>>(
        x, w, rstd, dy, dx, accumulate_dx, partial, R, D, rpb);
    int rc = check_launch("rmsnorm_bwd_kernel");
    if (rc || !dw)
        return rc;
    colsum_kernel<<<colsum_grid(D), COLSUM_THREADS, 0, S(stream)>>>(partial, nb, D, dw);
    return check_launch("colsum_kernel");
}

int ttk_swiglu_fwd(const float* a, const float* b, float* y, int64_t n, void* stream) {
    if (n < 0 || (n && (!a || !b || !y)))
        return set_error(TTK_ERR_ARG, "swiglu_fwd: bad arguments");
    if (!n)
        return TTK_OK;
    if (!(aligned16(a) && aligned16(b) && aligned16(y)))
        return set_error(TTK_ERR_ARG, "swiglu_fwd: tensors must be 16-byte aligned");
    swiglu_fwd_kernel<<<grid_for(n / 4 + 1, 256), 256, 0, S(stream)>>>(a, b, y, n);
    return check_launch("swiglu_fwd_kernel");
}

int ttk_swiglu_bwd(const float* a, const float* b, const float* dy, float* da, float* db,
                   int accumulate, int64_t n, void* stream) {
    if (n < 0 || (n && (!a || !b || !dy || !da || !db)))
        return set_error(TTK_ERR_ARG, "swiglu_bwd: bad arguments");
    if (!n)
        return TTK_OK;
    if (!(aligned16(a) && aligned16(b) && aligned16(dy) && aligned16(da) && aligned16(db)))
        return set_error(TTK_ERR_ARG, "swiglu_bwd: tensors must be 16-byte aligned");
    swiglu_bwd_kernel<<<grid_for(n / 4 + 1, 256), 256, 0, S(stream)>>>(a, b, dy, da, db,
                                                                       accumulate, n);
    return check_launch("swiglu_bwd_kernel");
}

static int split_rows_tpr(int64_t ldp) {
    int tpr = 1;
    while (tpr < 256 && tpr < ldp / 4)
        tpr <<= 1;
    return tpr;
}

int ttk_swiglu_fwd_split(const float* a, const float* b, void* y_split, int64_t R, int64_t F,
                         void* stream) {
    if (R < 0 || F <= 0 || (F & 3) || (R && (!a || !b || !y_split)))
        return set_error(TTK_ERR_ARG, "swiglu_fwd_split: bad arguments (F % 4 == 0)");
    if (ttk_gemm_get_precision() != 0)
        return set_error(TTK_ERR_ARG, "swiglu_fwd_split: the planes are bf16x3 operands");
    if (!R)
        return TTK_OK;
    if (!(aligned16(a) && aligned16(b) && aligned16(y_split)))
        return set_error(TTK_ERR_ARG, "swiglu_fwd_split: tensors must be 16-byte aligned");
    const int64_t ldp = (F + 31) / 32 * 32;
    const int tpr = split_rows_tpr(ldp);
    const int64_t rpb = 256 / tpr;
    const int blocks = static_cast<int>(std::min<int64_t>((R + rpb - 1) / rpb, 148 * 16));
    swiglu_fwd_split_kernel<<<blocks, 256, 0, S(stream)>>>(
        a, b, static_cast<__nv_bfloat16*>(y_split), R, F, ldp, tpr);
    return check_launch("swiglu_fwd_split_kernel");
}

int ttk_swiglu_bwd_split(const float* a, const float* b, const float* dy, void* da_split,
                         void* db_split, int64_t R, int64_t F, void* stream) {
    if (R < 0 || F <= 0 || (F & 3) || (R && (!a || !b || !dy || !da_split || !db_split)))
        return set_error(TTK_ERR_ARG, "swiglu_bwd_split: bad arguments (F % 4 == 0)");
    if (ttk_gemm_get_precision() != 0)
        return set_error(TTK_ERR_ARG, "swiglu_bwd_split: the planes are bf16x3 operands");
    if (!R)
        return TTK_OK;
    if (!(aligned16(a) && aligned16(b) && aligned16(dy) && aligned16(da_split) &&
          aligned16(db_split)))
        return set_error(TTK_ERR_ARG, "swiglu_bwd_split: tensors must be 16-byte aligned");
    const int64_t ldp = (F + 31) / 32 * 32;
    const int tpr = split_rows_tpr(ldp);
    const int64_t rpb = 256 / tpr;
    const int blocks = static_cast<int>(std::min<int64_t>((R + rpb - 1) / rpb, 148 * 16));
    swiglu_bwd_split_kernel<<<blocks, 256, 0, S(stream)>>>(
        a, b, dy, static_cast<__nv_bfloat16*>(da_split), static_cast<__nv_bfloat16*>(db_split), R,
        F, ldp, tpr);
    return check_launch("swiglu_bwd_split_kernel");
}

int ttk_cross_entropy(const float* logits, const int64_t* targets, int64_t N, int64_t C,
                      double* loss_acc, float* dlogits, float grad_scale, void* stream) {
    if (N < 0 || C <= 0 || !logits || !targets || !loss_acc)
        return set_error(TTK_ERR_ARG, "cross_entropy: bad arguments");
    if (!N)
        return TTK_OK;
    if ((C & 3) == 0 && !(aligned16(logits) && (!dlogits || aligned16(dlogits))))
        return set_error(TTK_ERR_ARG, "cross_entropy: tensors must be 16-byte aligned");
    if ((C & 3) == 0 && C <= static_cast<int64_t>(CE_THREADS) * CE_VEC * 4) {
        const int smem = static_cast<int>(C * 4);
        cudaFuncSetAttribute(cross_entropy_bulk_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        const int gb = static_cast<int>(std::min<int64_t>(N, 148));
        cross_entropy_bulk_kernel<<<gb, CE_THREADS, smem, S(stream)>>>(
            logits, targets, N, C, loss_acc, dlogits, grad_scale);
        return check_launch("cross_entropy_bulk_kernel");
    }
    const int grid = static_cast<int>(std::min<int64_t>(N, 148 * 2));
    if (C <= static_cast<int64_t>(CE_THREADS) * CE_VEC * 4)
        cross_entropy_kernel<true><<<grid, CE_THREADS, 0, S(stream)>>>(logits, targets, N, C,
                                                                       loss_acc, dlogits,
                                                                       grad_scale);
    else
        cross_entropy_kernel<false><<<grid, CE_THREADS, 0, S(stream)>>>(logits, targets, N, C,
                                                                        loss_acc, dlogits,
                                                                        grad_scale);
    return check_launch("cross_entropy_kernel");
}

int ttk_loss_finalize(const double* loss_acc, float scale, float* loss_out, void* stream) {
    loss_finalize_kernel<<<1, 1, 0, S(stream)>>>(loss_acc, scale, loss_out);
    return check_launch("loss_finalize_kernel");
}

int ttk_embedding_fwd(const float* W, const int64_t* idx, float* out, int64_t N, int64_t D,
                      int64_t V, void* stream) {
    if (N < 0 || D <= 0 || V <= 0 || (N && (!W || !idx || !out)))
        return set_error(TTK_ERR_ARG, "embedding_fwd: bad arguments");
    if (!N)
        return TTK_OK;
    if ((D & 3) == 0 && !(aligned16(W) && aligned16(out)))
        return set_error(TTK_ERR_ARG, "embedding_fwd: tensors must be 16-byte aligned");
    embedding_fwd_kernel<<<grid_for(N, 8), 256, 0, S(stream)>>>(W, idx, out, N, D, V);
    return check_launch("embedding_fwd_kernel");
}

static int64_t pow2_at_least(int64_t n) {
    int64_t p = 1;
    while (p < n)
        p <<= 1;
    return p;
}

size_t ttk_embedding_bwd_workspace_size(int64_t N) {
    return static_cast<size_t>(pow2_at_least(std::max<int64_t>(N, 1))) * sizeof(uint64_t);
}

int ttk_embedding_bwd(const float* dout, const int64_t* idx, float* dW, int64_t N, int64_t D,
                      int64_t V, void* workspace, size_t workspace_bytes, void* stream) {
    if (N < 0 || D <= 0 || V <= 0 || (N && (!dout || !idx || !dW)))
        return set_error(TTK_ERR_ARG, "embedding_bwd: bad arguments");
    if (!N)
        return TTK_OK;
    if (N >= (1ll << 32) || V >= (1ll << 31))
        return set_error(TTK_ERR_ARG, "embedding_bwd: N or V too large");
    const int64_t np2 = pow2_at_least(N);
    if (!workspace || workspace_bytes < static_cast<size_t>(np2) * sizeof(uint64_t))
        return set_error(TTK_ERR_ARG, "embedding_bwd: workspace too small");
    uint64_t* keys = static_cast<uint64_t*>(workspace);
    make_keys_kernel<<<grid_for(np2, 256), 256, 0, S(stream)>>>(idx, N, np2, keys);
    int rc = check_launch("make_keys_kernel");
    if (rc)
        return rc;
    const size_t smem = static_cast<size_t>(np2) * sizeof(uint64_t);
    if (smem <= 128 * 1024) {
        if (smem > 48 * 1024)
            cudaFuncSetAttribute(bitonic_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem));
        bitonic_smem_kernel<<<1, 1024, smem, S(stream)>>>(keys, np2);
        rc = check_launch("bitonic_smem_kernel");
    } else {
        // np2 > 16384 is a multiple of the chunk: stages up to the chunk size
        // in shared memory, then per stage the passes across chunks in global
        // memory and the rest in shared memory again (the same network).
        const int cs = static_cast<int>(BITONIC_CHUNK * sizeof(uint64_t));
        cudaFuncSetAttribute(bitonic_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             cs);
        const unsigned nchunks = static_cast<unsigned>(np2 / BITONIC_CHUNK);
        bitonic_chunk_kernel<<<nchunks, 1024, cs, S(stream)>>>(keys, 0, 1);
        rc = check_launch("bitonic_chunk_kernel");
        for (int64_t k = 2 * BITONIC_CHUNK; k <= np2 && !rc; k <<= 1) {
            for (int64_t j = k >> 1; j >= BITONIC_CHUNK && !rc; j >>= 1) {
                bitonic_global_kernel<<<grid_for(np2, 256), 256, 0, S(stream)>>>(keys, np2, k, j);
                rc = check_launch("bitonic_global_kernel");
            }
            if (!rc) {
                bitonic_chunk_kernel<<<nchunks, 1024, cs, S(stream)>>>(keys, k, 0);
                rc = check_launch("bitonic_chunk_kernel");
            }
        }
    }
    if (rc)
        return rc;
    embedding_segment_kernel<<<grid_for(N, 8), 256, 0, S(stream)>>>(keys, N, dout, dW, D, V);
    return check_launch("embedding_segment_kernel");
}

int ttk_index_check(const int64_t* idx, int64_t n, int64_t V, int64_t* bad_host, void* stream) {
    if (n <= 0) {
        *bad_host = 0;
        return TTK_OK;
    }
    unsigned long long* d = nullptr;
    int rc = check_cuda(cudaMallocAsync(reinterpret_cast<void**>(&d), 8, S(stream)), "alloc");
    if (rc)
        return rc;
    cudaMemsetAsync(d, 0, 8, S(stream));
    index_check_kernel<<<grid_for(n, 256), 256, 0, S(stream)>>>(idx, n, V, d);
    unsigned long long h = 0;
    cudaMemcpyAsync(&h, d, 8, cudaMemcpyDeviceToHost, S(stream));
    cudaFreeAsync(d, S(stream));
    rc = check_cuda(cudaStreamSynchronize(S(stream)), "index_check");
    *bad_host = static_cast<int64_t>(h);
    return rc;
}

int ttk_rope_fwd(const float* x, const float* cos_t, const float* sin_t, float* y, int64_t B,
                 int64_t T, int64_t H, int64_t D, void* stream) {
    if (B < 0 || T < 0 || H < 0 || D <= 0 || (D & 1))
        return set_error(TTK_ERR_ARG, "rope: head dim must be even");
    const int64_t total = B * T * H * (D / 2);
    if (!total)
        return TTK_OK;
    rope_kernel<<<grid_for(total, 256), 256, 0, S(stream)>>>(x, cos_t, sin_t, y, 0, 0, B, T, H, D);
    return check_launch("rope_kernel");
}

int ttk_rope_bwd(const float* dy, const float* cos_t, const float* sin_t, float* dx,
                 int accumulate, int64_t B, int64_t T, int64_t H, int64_t D, void* stream) {
    if (B < 0 || T < 0 || H < 0 || D <= 0 || (D & 1))
        return set_error(TTK_ERR_ARG, "rope: head dim must be even");
    const int64_t total = B * T * H * (D / 2);
    if (!total)
        return TTK_OK;
    rope_kernel<<<grid_for(total, 256), 256, 0, S(stream)>>>(dy, cos_t, sin_t, dx, accumulate, 1,
                                                             B, T, H, D);
    return check_launch("rope_kernel");
}

int ttk_softmax_fwd(const float* x, float* y, int64_t R, int64_t C, int log, void* stream) {
    if (R < 0 || C <= 0)
        return set_error(TTK_ERR_ARG, "softmax: bad shape");
    if (!R)
        return TTK_OK;
    softmax_fwd_kernel<<<grid_for(R, 8), 256, 0, S(stream)>>>(x, y, R, C, log);
    return check_launch("softmax_fwd_kernel");
}

int ttk_softmax_bwd(const float* y, const float* dy, float* dx, int accumulate, int64_t R,
                    int64_t C, int log, void* stream) {
    if (R < 0 || C <= 0)
        return set_error(TTK_ERR_ARG, "softmax: bad shape");
    if (!R)
        return TTK_OK;
    softmax_bwd_kernel<<<grid_for(R, 8), 256, 0, S(stream)>>>(y, dy, dx, accumulate, R, C, log);
    return check_launch("softmax_bwd_kernel");
}

int ttk_nll_fwd(const float* lp, const int64_t* targets, int64_t N, int64_t C, float* loss,
                void* stream) {
    if (N <= 0 || C <= 0 || !lp || !targets || !loss)
        return set_error(TTK_ERR_ARG, "nll_fwd: bad arguments");
    nll_fwd_kernel<<<1, 1024, 0, S(stream)>>>(lp, targets, N, C, loss);
    return check_launch("nll_fwd_kernel");
}

int ttk_nll_bwd(const int64_t* targets, int64_t N, int64_t C, const float* g, float* dlp,
                void* stream) {
    if (N <= 0 || C <= 0 || !targets || !g || !dlp)
        return set_error(TTK_ERR_ARG, "nll_bwd: bad arguments");
    nll_bwd_kernel<<<grid_for(N, 256), 256, 0, S(stream)>>>(targets, N, C, g, dlp);
    return check_launch("nll_bwd_kernel");
}

int ttk_rope_table_grad(const float* x, const float* dy, int64_t B, int64_t T, int64_t H,
                        int64_t D, float* dcos, float* dsin, void* stream) {
    if (B < 0 || T < 0 || H < 0 || D <= 0 || (D & 1))
        return set_error(TTK_ERR_ARG, "rope_table_grad: bad shape");
    if (!B || !T || !H)
        return TTK_OK;
    rope_table_grad_kernel<<<grid_for(T * (D / 2), 256), 256, 0, S(stream)>>>(x, dy, B, T, H, D,
                                                                             dcos, dsin);
    return check_launch("rope_table_grad_kernel");
}

int ttk_axpy_dev(const float* alpha, const float* x, float* y, int64_t n, int accumulate,
                 void* stream) {
    if (n < 0 || (n && (!alpha || !x || !y)))
        return set_error(TTK_ERR_ARG, "axpy_dev: bad arguments");
    if (!n)
        return TTK_OK;
    axpy_dev_kernel<<<grid_for(n, 256), 256, 0, S(stream)>>>(alpha, x, y, n, accumulate);
    return check_launch("axpy_dev_kernel");
}

}  // extern "C"
