// Fused causal self-attention with RoPE, forward and backward, fp32.
//
// Replaces the attention block of GPTModel::forward (model.cpp:127-141):
// rope(q), rope(k) (ops.cpp:970-1052), the [B*H,T,T] score bmm, the scale
// and -1e9 mask (a masked score contributes exp(-1e9 - m) = 0 in fp32, the
// same as skipping it), softmax (ops.cpp:777-838) and the P.V bmm, with their
// backward rules. Scores never reach HBM: flash-style online softmax over
// 64x64 tiles, the log-sum-exp per query row is saved for the backward.
//
// q, k, v, o: [B, T, H, HD] row-major (the Linear outputs' layout).
// cos/sin: [T, HD/2]. lse: [B, H, T].
//
// Thread tiling (256 threads, 16 x 16): a 64 x 64 score tile gives thread
// (tr, tc) rows tr*4 .. tr*4+3 and columns tc + 16*j (j < 4). Shared tiles
// are row-major with a 4-float pad, which makes every float4 read in the
// inner products bank-conflict free. Output columns of HD-wide rows are held
// as float4 groups at g*64 + tc*4 (HD >= 64) or float2 at tc*2 (HD = 32).
//
// Backward: dK/dV kernel per key block (loops over later query blocks) and a
// dQ kernel per query block (loops over earlier key blocks). Both recompute
// the scores; no atomics, so results are deterministic.
#include <cuda_runtime.h>

#include <initializer_list>
#include <stdint.h>

#include <cstdlib>
#include <string>

#include "ttk_common.cuh"
#include "ttk_internal.h"

namespace ttk {
namespace attn {

constexpr int BT = 64;        // rows per tile (queries and keys)
constexpr int NT = 256;       // threads per block
constexpr int LDP = BT + 4;   // padded stride of 64-wide tiles

template <int HD>
struct Geo {
    static constexpr int LD = HD + 4;         // padded stride of HD-wide tiles
    static constexpr int NC = HD >= 64 ? HD / 64 : 1;  // column groups per thread
    static constexpr int CW = HD >= 64 ? 4 : 2;        // columns per group
    static constexpr int OC = NC * CW;                  // output columns per thread
    __device__ static int col(int tc, int g, int e) {
        return HD >= 64 ? g * 64 + tc * 4 + e : tc * 2 + e;
    }
};

__device__ __forceinline__ int64_t row_off(int b, int64_t t, int h, int64_t T, int H, int HD) {
    return ((static_cast<int64_t>(b) * T + t) * H + h) * HD;
}

// Load a 64-row tile of x [B,T,H,HD] (rows t0..t0+63 of head h) into shared
// memory, optionally rotated by RoPE; rows past T are zero.
template <int HD>
__device__ __forceinline__ void load_tile(float* __restrict__ dst, const float* __restrict__ x,
                                          const float* __restrict__ cs,
                                          const float* __restrict__ sn, bool rope, int b,
                                          int64_t t0, int h, int64_t T, int H) {
    constexpr int LD = Geo<HD>::LD;
    constexpr int HH = HD / 2;
    for (int idx = threadIdx.x; idx < BT * HH; idx += NT) {
        const int r = idx / HH, d = idx % HH;
        const int64_t t = t0 + r;
        float a = 0.0f, c2 = 0.0f;
        if (t < T) {
            const float* src = x + row_off(b, t, h, T, H, HD);
            const float x1 = src[d], x2 = src[d + HH];
            if (rope) {
                const float c = cs[t * HH + d], s = sn[t * HH + d];
                a = x1 * c - x2 * s;
                c2 = x1 * s + x2 * c;
            } else {
                a = x1;
                c2 = x2;
            }
        }
        dst[r * LD + d] = a;
        dst[r * LD + d + HH] = c2;
    }
}

// acc[i][j] = sum_d A[tr*4+i][d] * Bm[tc+16j][d] over HD (row-major, padded).
template <int HD>
__device__ __forceinline__ void tile_dot(const float* __restrict__ A, const float* __restrict__ Bm,
                                         int tr, int tc, float (&acc)[4][4]) {
    constexpr int LD = Geo<HD>::LD;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
            acc[i][j] = 0.0f;
#pragma unroll 4
    for (int d = 0; d < HD; d += 4) {
        float4 a[4], bb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            a[i] = *reinterpret_cast<const float4*>(A + (tr * 4 + i) * LD + d);
#pragma unroll
        for (int j = 0; j < 4; ++j)
            bb[j] = *reinterpret_cast<const float4*>(Bm + (tc + 16 * j) * LD + d);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j)
                acc[i][j] += a[i].x * bb[j].x + a[i].y * bb[j].y + a[i].z * bb[j].z +
                             a[i].w * bb[j].w;
    }
}

// out[i][c] += sum_k W[k][r_i] * M[k][col(c)] where W is a 64x64 tile stored
// k-major (W[k*LDP + r]) and rows r_i = tr*4 + i; M is row-major [64][LD].
template <int HD>
__device__ __forceinline__ void tile_accum(const float* __restrict__ W, const float* __restrict__ M,
                                           int tr, int tc, float (&out)[4][Geo<HD>::OC]) {
    using G = Geo<HD>;
#pragma unroll 4
    for (int k = 0; k < BT; ++k) {
        const float4 w = *reinterpret_cast<const float4*>(W + k * LDP + tr * 4);
        const float wv[4] = {w.x, w.y, w.z, w.w};
        float mv[G::OC];
#pragma unroll
        for (int g = 0; g < G::NC; ++g) {
            if (G::CW == 4) {
                const float4 m4 = *reinterpret_cast<const float4*>(M + k * G::LD + G::col(tc, g, 0));
                mv[g * 4] = m4.x, mv[g * 4 + 1] = m4.y, mv[g * 4 + 2] = m4.z, mv[g * 4 + 3] = m4.w;
            } else {
                const float2 m2 = *reinterpret_cast<const float2*>(M + k * G::LD + G::col(tc, g, 0));
                mv[g * 2] = m2.x, mv[g * 2 + 1] = m2.y;
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int c = 0; c < G::OC; ++c)
                out[i][c] += wv[i] * mv[c];
    }
}

__device__ __forceinline__ float half_warp_max(float v) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1)
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float half_warp_sum(float v) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ------------------------------------------------------------- forward --
template <int HD>
__global__ void __launch_bounds__(NT) attn_fwd_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    const float* __restrict__ cs, const float* __restrict__ sn, float* __restrict__ o,
    float* __restrict__ lse, int64_t T, int H, float scale) {
    using G = Geo<HD>;
    extern __shared__ float sm[];
    float* Qs = sm;                  // [64][LD]
    float* Ks = Qs + BT * G::LD;     // [64][LD]
    float* Vs = Ks + BT * G::LD;     // [64][LD]
    float* Pt = Vs + BT * G::LD;     // [64 keys][LDP] (transposed P)
    const int qb = blockIdx.x;
    const int bh = blockIdx.y;
    const int b = bh / H, h = bh % H;
    const int tr = threadIdx.x >> 4, tc = threadIdx.x & 15;
    const int64_t q0 = static_cast<int64_t>(qb) * BT;

    load_tile<HD>(Qs, q, cs, sn, true, b, q0, h, T, H);
    float m[4], l[4], acc[4][G::OC];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
#pragma unroll
        for (int c = 0; c < G::OC; ++c)
            acc[i][c] = 0.0f;
    }
    for (int kb = 0; kb <= qb; ++kb) {
        const int64_t k0 = static_cast<int64_t>(kb) * BT;
        __syncthreads();
        load_tile<HD>(Ks, k, cs, sn, true, b, k0, h, T, H);
        load_tile<HD>(Vs, v, cs, sn, false, b, k0, h, T, H);
        __syncthreads();
        float s[4][4];
        tile_dot<HD>(Qs, Ks, tr, tc, s);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t qr = q0 + tr * 4 + i;
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t kc = k0 + tc + 16 * j;
                s[i][j] = (kc > qr || kc >= T) ? -INFINITY : s[i][j] * scale;
                mx = fmaxf(mx, s[i][j]);
            }
            mx = half_warp_max(mx);
            const float mn = fmaxf(m[i], mx);
            const float alpha = (m[i] == -INFINITY) ? 0.0f : expf(m[i] - mn);
            float rs = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                s[i][j] = (s[i][j] == -INFINITY) ? 0.0f : expf(s[i][j] - mn);
                rs += s[i][j];
            }
            rs = half_warp_sum(rs);
            l[i] = l[i] * alpha + rs;
            m[i] = mn;
#pragma unroll
            for (int c = 0; c < G::OC; ++c)
                acc[i][c] *= alpha;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
            *reinterpret_cast<float4*>(Pt + (tc + 16 * j) * LDP + tr * 4) =
                make_float4(s[0][j], s[1][j], s[2][j], s[3][j]);
        __syncthreads();
        tile_accum<HD>(Pt, Vs, tr, tc, acc);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t t = q0 + tr * 4 + i;
        if (t >= T)
            continue;
        const float inv = 1.0f / l[i];
        float* dst = o + row_off(b, t, h, T, H, HD);
#pragma unroll
        for (int g = 0; g < G::NC; ++g) {
            if (G::CW == 4)
                *reinterpret_cast<float4*>(dst + G::col(tc, g, 0)) =
                    make_float4(acc[i][g * 4] * inv, acc[i][g * 4 + 1] * inv,
                                acc[i][g * 4 + 2] * inv, acc[i][g * 4 + 3] * inv);
            else
                *reinterpret_cast<float2*>(dst + G::col(tc, g, 0)) =
                    make_float2(acc[i][g * 2] * inv, acc[i][g * 2 + 1] * inv);
        }
        if (tc == 0)
            lse[static_cast<int64_t>(bh) * T + t] = m[i] + logf(l[i]);
    }
}

// D[bh][t] = sum_d dO[t][d] * O[t][d]  (the softmax-backward row term).
template <int HD>
__global__ void attn_dot_kernel(const float* __restrict__ o, const float* __restrict__ dout,
                                float* __restrict__ Dv, int64_t B, int64_t T, int H) {
    const int lane = threadIdx.x & 31;
    const int64_t rows = B * T * H;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
         r < rows; r += warps) {
        const float* a = o + r * HD;
        const float* g = dout + r * HD;
        float s = 0.0f;
        for (int d = lane; d < HD; d += 32)
            s += a[d] * g[d];
        s = warp_sum(s);
        if (lane == 0) {
            const int64_t h = r % H, t = (r / H) % T, b = r / (H * T);
            Dv[(b * H + h) * T + t] = s;
        }
    }
}

// Write a [64][HD] gradient tile held in shared memory (w.r.t. the rotated
// operand when `rope`) to dst rows t0.., applying the transpose rotation.
template <int HD>
__device__ __forceinline__ void store_grad_tile(const float* __restrict__ src,
                                                float* __restrict__ dst,
                                                const float* __restrict__ cs,
                                                const float* __restrict__ sn, bool rope,
                                                int accumulate, int b, int64_t t0, int h,
                                                int64_t T, int H) {
    constexpr int LD = Geo<HD>::LD;
    constexpr int HH = HD / 2;
    for (int idx = threadIdx.x; idx < BT * HH; idx += NT) {
        const int r = idx / HH, d = idx % HH;
        const int64_t t = t0 + r;
        if (t >= T)
            continue;
        const float g1 = src[r * LD + d], g2 = src[r * LD + d + HH];
        float o1 = g1, o2 = g2;
        if (rope) {
            const float c = cs[t * HH + d], s = sn[t * HH + d];
            o1 = g1 * c + g2 * s;
            o2 = -g1 * s + g2 * c;
        }
        float* p = dst + row_off(b, t, h, T, H, HD);
        if (accumulate) {
            p[d] += o1;
            p[d + HH] += o2;
        } else {
            p[d] = o1;
            p[d + HH] = o2;
        }
    }
}

template <int HD>
__device__ __forceinline__ void acc_to_smem(float* __restrict__ dst, int tr, int tc,
                                            const float (&acc)[4][Geo<HD>::OC], float mul) {
    using G = Geo<HD>;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int g = 0; g < G::NC; ++g)
#pragma unroll
            for (int e = 0; e < G::CW; ++e)
                dst[(tr * 4 + i) * G::LD + G::col(tc, g, e)] = acc[i][g * G::CW + e] * mul;
}

// dK, dV for one key block: loops over query blocks qb >= kb.
template <int HD>
__global__ void __launch_bounds__(NT) attn_bwd_dkv_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    const float* __restrict__ cs, const float* __restrict__ sn, const float* __restrict__ lse,
    const float* __restrict__ Dv, const float* __restrict__ dout, float* __restrict__ dk,
    float* __restrict__ dv, int accumulate, int64_t T, int H, float scale) {
    using G = Geo<HD>;
    extern __shared__ float sm[];
    float* Ks = sm;                  // [64][LD] rotated keys
    float* Vs = Ks + BT * G::LD;     // [64][LD]
    float* Qs = Vs + BT * G::LD;     // [64][LD] rotated queries (per query block)
    float* dOs = Qs + BT * G::LD;    // [64][LD]
    float* Ps = dOs + BT * G::LD;    // [64 q][LDP]
    float* dSs = Ps + BT * LDP;      // [64 q][LDP]
    float* rl = dSs + BT * LDP;      // [64] lse
    float* rd = rl + BT;             // [64] D
    const int kb = blockIdx.x;
    const int bh = blockIdx.y;
    const int b = bh / H, h = bh % H;
    const int tr = threadIdx.x >> 4, tc = threadIdx.x & 15;
    const int64_t k0 = static_cast<int64_t>(kb) * BT;
    const int nqb = static_cast<int>((T + BT - 1) / BT);

    load_tile<HD>(Ks, k, cs, sn, true, b, k0, h, T, H);
    load_tile<HD>(Vs, v, cs, sn, false, b, k0, h, T, H);
    float dK[4][G::OC], dV[4][G::OC];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < G::OC; ++c)
            dK[i][c] = 0.0f, dV[i][c] = 0.0f;

    for (int qb = kb; qb < nqb; ++qb) {
        const int64_t q0 = static_cast<int64_t>(qb) * BT;
        __syncthreads();
        load_tile<HD>(Qs, q, cs, sn, true, b, q0, h, T, H);
        load_tile<HD>(dOs, dout, cs, sn, false, b, q0, h, T, H);
        for (int r = threadIdx.x; r < BT; r += NT) {
            const int64_t t = q0 + r;
            rl[r] = t < T ? lse[static_cast<int64_t>(bh) * T + t] : 0.0f;
            rd[r] = t < T ? Dv[static_cast<int64_t>(bh) * T + t] : 0.0f;
        }
        __syncthreads();
        float s[4][4], dp[4][4];
        tile_dot<HD>(Qs, Ks, tr, tc, s);
        tile_dot<HD>(dOs, Vs, tr, tc, dp);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = tr * 4 + i;
            const int64_t qr = q0 + r;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int c = tc + 16 * j;
                const int64_t kc = k0 + c;
                const bool live = kc <= qr && qr < T && kc < T;
                const float p = live ? expf(s[i][j] * scale - rl[r]) : 0.0f;
                Ps[r * LDP + c] = p;
                dSs[r * LDP + c] = p * (dp[i][j] - rd[r]);
            }
        }
        __syncthreads();
        // dV[c][d] += sum_r P[r][c] dO[r][d]; dK[c][d] += sum_r dS[r][c] Q[r][d]
        tile_accum<HD>(Ps, dOs, tr, tc, dV);
        tile_accum<HD>(dSs, Qs, tr, tc, dK);
    }
    __syncthreads();
    acc_to_smem<HD>(Qs, tr, tc, dK, scale);
    acc_to_smem<HD>(dOs, tr, tc, dV, 1.0f);
    __syncthreads();
    store_grad_tile<HD>(Qs, dk, cs, sn, true, accumulate, b, k0, h, T, H);
    store_grad_tile<HD>(dOs, dv, cs, sn, false, accumulate, b, k0, h, T, H);
}

// dQ for one query block: loops over key blocks kb <= qb.
template <int HD>
__global__ void __launch_bounds__(NT) attn_bwd_dq_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    const float* __restrict__ cs, const float* __restrict__ sn, const float* __restrict__ lse,
    const float* __restrict__ Dv, const float* __restrict__ dout, float* __restrict__ dq,
    int accumulate, int64_t T, int H, float scale) {
    using G = Geo<HD>;
    extern __shared__ float sm[];
    float* Qs = sm;                  // [64][LD]
    float* dOs = Qs + BT * G::LD;    // [64][LD]
    float* Ks = dOs + BT * G::LD;    // [64][LD]
    float* Vs = Ks + BT * G::LD;     // [64][LD]
    float* dSt = Vs + BT * G::LD;    // [64 keys][LDP] (transposed dS)
    const int qb = blockIdx.x;
    const int bh = blockIdx.y;
    const int b = bh / H, h = bh % H;
    const int tr = threadIdx.x >> 4, tc = threadIdx.x & 15;
    const int64_t q0 = static_cast<int64_t>(qb) * BT;

    load_tile<HD>(Qs, q, cs, sn, true, b, q0, h, T, H);
    load_tile<HD>(dOs, dout, cs, sn, false, b, q0, h, T, H);
    float rl[4], rd[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t t = q0 + tr * 4 + i;
        rl[i] = t < T ? lse[static_cast<int64_t>(bh) * T + t] : 0.0f;
        rd[i] = t < T ? Dv[static_cast<int64_t>(bh) * T + t] : 0.0f;
    }
    float dQ[4][G::OC];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < G::OC; ++c)
            dQ[i][c] = 0.0f;
    for (int kb = 0; kb <= qb; ++kb) {
        const int64_t k0 = static_cast<int64_t>(kb) * BT;
        __syncthreads();
        load_tile<HD>(Ks, k, cs, sn, true, b, k0, h, T, H);
        load_tile<HD>(Vs, v, cs, sn, false, b, k0, h, T, H);
        __syncthreads();
        float s[4][4], dp[4][4];
        tile_dot<HD>(Qs, Ks, tr, tc, s);
        tile_dot<HD>(dOs, Vs, tr, tc, dp);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int c = tc + 16 * j;
            const int64_t kc = k0 + c;
            float ds[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int64_t qr = q0 + tr * 4 + i;
                const bool live = kc <= qr && qr < T && kc < T;
                const float p = live ? expf(s[i][j] * scale - rl[i]) : 0.0f;
                ds[i] = p * (dp[i][j] - rd[i]);
            }
            *reinterpret_cast<float4*>(dSt + c * LDP + tr * 4) = make_float4(ds[0], ds[1], ds[2], ds[3]);
        }
        __syncthreads();
        // dQ[r][d] += sum_c dS[r][c] K[c][d]
        tile_accum<HD>(dSt, Ks, tr, tc, dQ);
    }
    __syncthreads();
    acc_to_smem<HD>(Ks, tr, tc, dQ, scale);
    __syncthreads();
    store_grad_tile<HD>(Ks, dq, cs, sn, true, accumulate, b, q0, h, T, H);
}

template <int HD>
size_t fwd_smem() { return (3 * BT * Geo<HD>::LD + BT * LDP) * sizeof(float); }
template <int HD>
size_t dkv_smem() { return (4 * BT * Geo<HD>::LD + 2 * BT * LDP + 2 * BT) * sizeof(float); }
template <int HD>
size_t dq_smem() { return (4 * BT * Geo<HD>::LD + BT * LDP) * sizeof(float); }

template <int HD>
int launch_fwd(const float* q, const float* k, const float* v, const float* cs, const float* sn,
               float* o, float* lse, int64_t B, int64_t T, int64_t H, float scale,
               cudaStream_t st) {
    const size_t smem = fwd_smem<HD>();
    cudaFuncSetAttribute(attn_fwd_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
    dim3 grid(static_cast<unsigned>((T + BT - 1) / BT), static_cast<unsigned>(B * H));
    attn_fwd_kernel<HD><<<grid, NT, smem, st>>>(q, k, v, cs, sn, o, lse, T, static_cast<int>(H),
                                               scale);
    return check_launch("attn_fwd_kernel");
}

template <int HD>
int launch_bwd(const float* q, const float* k, const float* v, const float* cs, const float* sn,
               const float* o, const float* lse, const float* dout, float* dq, float* dk,
               float* dv, int accumulate, int64_t B, int64_t T, int64_t H, float scale,
               float* Dv, cudaStream_t st) {
    attn_dot_kernel<HD><<<grid_for(B * T * H, 8), 256, 0, st>>>(o, dout, Dv, B, T,
                                                                static_cast<int>(H));
    int rc = check_launch("attn_dot_kernel");
    if (rc)
        return rc;
    dim3 grid(static_cast<unsigned>((T + BT - 1) / BT), static_cast<unsigned>(B * H));
    size_t smem = dkv_smem<HD>();
    cudaFuncSetAttribute(attn_bwd_dkv_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
    attn_bwd_dkv_kernel<HD><<<grid, NT, smem, st>>>(q, k, v, cs, sn, lse, Dv, dout, dk, dv,
                                                   accumulate, T, static_cast<int>(H), scale);
    rc = check_launch("attn_bwd_dkv_kernel");
    if (rc)
        return rc;
    smem = dq_smem<HD>();
    cudaFuncSetAttribute(attn_bwd_dq_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
    attn_bwd_dq_kernel<HD><<<grid, NT, smem, st>>>(q, k, v, cs, sn, lse, Dv, dout, dq, accumulate,
                                                  T, static_cast<int>(H), scale);
    return check_launch("attn_bwd_dq_kernel");
}

}  // namespace attn
}  // namespace ttk

using namespace ttk;
using namespace ttk::attn;

static inline cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

static int attn_check(const void* q, const void* k, const void* v, const void* cs,
                      const void* sn, int64_t B, int64_t T, int64_t H, int64_t hd) {
    if (B < 0 || T < 0 || H < 0)
        return set_error(TTK_ERR_ARG, "attention: negative size");
    if (hd != 32 && hd != 64 && hd != 128)
        return set_error(TTK_ERR_ARG, "attention: head_dim must be 32, 64 or 128");
    if (B * H > 65535 || T > (1ll << 31) / 64)
        return set_error(TTK_ERR_ARG, "attention: B*H or T too large");
    if (B && T && H && (!q || !k || !v || !cs || !sn))
        return set_error(TTK_ERR_ARG, "attention: null pointer");
    return TTK_OK;
}

// The tensor-core engines read q, k, v, dO and the RoPE tables as float4.
static int attn_align_check(std::initializer_list<const void*> ps) {
    for (const void* p : ps)
        if (p && (reinterpret_cast<uintptr_t>(p) & 15))
            return set_error(TTK_ERR_ARG, "attention: tensors must be 16-byte aligned");
    return TTK_OK;
}

namespace {
// 0: tensor cores, tcgen05 forward where the head dim allows (64, 128) and
//    mma.sync otherwise (default); 1: fp32 FMA kernels; 2: mma.sync only.
// TTK_ATTENTION=fma | mma selects 1 | 2 at start-up.
int g_attn_impl = -1;
int attn_impl() {
    if (g_attn_impl < 0) {
        const char* e = std::getenv("TTK_ATTENTION");
        g_attn_impl = (e && std::string(e) == "fma") ? 1 : (e && std::string(e) == "mma") ? 2 : 0;
    }
    return g_attn_impl;
}
inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }
}  // namespace

extern "C" {

int ttk_attention_set_impl(int impl) {
    if (impl < 0 || impl > 2)
        return set_error(TTK_ERR_ARG,
                         "attention impl must be 0 (tensor cores), 1 (fp32 FMA) or 2 (mma.sync)");
    g_attn_impl = impl;
    return TTK_OK;
}

int ttk_attention_get_impl(void) { return attn_impl(); }

size_t ttk_attention_fwd_workspace_size(int64_t B, int64_t T, int64_t H, int64_t hd) {
    if (attn_impl() == 1)
        return 0;
    return static_cast<size_t>(B * T * H * hd) * 6 * 2;  // q, k, v as bf16 hi|lo
}

int ttk_attention_fwd(const float* q, const float* k, const float* v, const float* cos_t,
                      const float* sin_t, float* o, float* lse, int64_t B, int64_t T, int64_t H,
                      int64_t hd, float scale, void* workspace, size_t workspace_bytes,
                      void* stream) {
    int rc = attn_check(q, k, v, cos_t, sin_t, B, T, H, hd);
    if (rc)
        return rc;
    if (!B || !T || !H)
        return TTK_OK;
    if (!o || !lse)
        return set_error(TTK_ERR_ARG, "attention_fwd: null output");
    if (attn_impl() != 1) {
        if (!workspace || workspace_bytes < ttk_attention_fwd_workspace_size(B, T, H, hd))
            return set_error(TTK_ERR_ARG, "attention_fwd: workspace too small");
        rc = attn_align_check({q, k, v, cos_t, sin_t, o});
        if (rc)
            return rc;
        const bool tc = attn_impl() == 0 && attention_tc_supported(static_cast<int>(hd));
        return attention_mma_forward(static_cast<int>(hd), q, k, v, cos_t, sin_t, o, lse, B, T,
                                     H, scale, workspace, tc, S(stream));
    }
    switch (hd) {
        case 32: return launch_fwd<32>(q, k, v, cos_t, sin_t, o, lse, B, T, H, scale, S(stream));
        case 64: return launch_fwd<64>(q, k, v, cos_t, sin_t, o, lse, B, T, H, scale, S(stream));
        default: return launch_fwd<128>(q, k, v, cos_t, sin_t, o, lse, B, T, H, scale, S(stream));
    }
}

size_t ttk_attention_bwd_workspace_size(int64_t B, int64_t T, int64_t H, int64_t hd) {
    const size_t dv = align256(static_cast<size_t>(B * T * H) * sizeof(float));
    if (attn_impl() == 1)
        return dv;
    // q, k, v, dO as bf16 hi|lo, then the (lse, D) table of the tcgen05 path
    return dv + static_cast<size_t>(B * T * H * hd) * 8 * 2 +
           align256(static_cast<size_t>(B * H * ((T + 31) / 32 * 32)) * 8);
}

int ttk_attention_bwd(const float* q, const float* k, const float* v, const float* cos_t,
                      const float* sin_t, const float* o, const float* lse, const float* dout,
                      float* dq, float* dk, float* dv, int accumulate, int64_t B, int64_t T,
                      int64_t H, int64_t hd, float scale, void* workspace,
                      size_t workspace_bytes, void* stream) {
    int rc = attn_check(q, k, v, cos_t, sin_t, B, T, H, hd);
    if (rc)
        return rc;
    if (!B || !T || !H)
        return TTK_OK;
    if (!o || !lse || !dout || !dq || !dk || !dv)
        return set_error(TTK_ERR_ARG, "attention_bwd: null pointer");
    if (!workspace || workspace_bytes < ttk_attention_bwd_workspace_size(B, T, H, hd))
        return set_error(TTK_ERR_ARG, "attention_bwd: workspace too small");
    if (attn_impl() != 1) {
        rc = attn_align_check({q, k, v, cos_t, sin_t, o, dout, dq, dk, dv});
        if (rc)
            return rc;
        const bool tc = attn_impl() == 0 && attention_tc_supported(static_cast<int>(hd));
        return attention_mma_backward(static_cast<int>(hd), q, k, v, cos_t, sin_t, o, lse, dout,
                                      dq, dk, dv, accumulate, B, T, H, scale, workspace, tc,
                                      S(stream));
    }
    float* Dv = static_cast<float*>(workspace);
    switch (hd) {
        case 32:
            return launch_bwd<32>(q, k, v, cos_t, sin_t, o, lse, dout, dq, dk, dv, accumulate, B,
                                  T, H, scale, Dv, S(stream));
        case 64:
            return launch_bwd<64>(q, k, v, cos_t, sin_t, o, lse, dout, dq, dk, dv, accumulate, B,
                                  T, H, scale, Dv, S(stream));
        default:
            return launch_bwd<128>(q, k, v, cos_t, sin_t, o, lse, dout, dq, dk, dv, accumulate, B,
                                   T, H, scale, Dv, S(stream));
    }
}

size_t ttk_attention_bwd_ex_workspace_size(int64_t B, int64_t T, int64_t H, int64_t hd) {
    const size_t dv = align256(static_cast<size_t>(B * T * H) * sizeof(float));
    if (attn_impl() == 1)
        return dv;
    // dO as bf16 hi|lo, then the (lse, D) table; q, k, v come from the forward
    return dv + static_cast<size_t>(B * T * H * hd) * 2 * 2 +
           align256(static_cast<size_t>(B * H * ((T + 31) / 32 * 32)) * 8);
}

int ttk_attention_bwd_ex(const float* q, const float* k, const float* v, const float* cos_t,
                         const float* sin_t, const float* o, const float* lse, const float* dout,
                         float* dq, float* dk, float* dv, int accumulate, int64_t B, int64_t T,
                         int64_t H, int64_t hd, float scale, const void* fwd_workspace,
                         void* workspace, size_t workspace_bytes, void* stream) {
    if (!fwd_workspace || attn_impl() == 1)
        return ttk_attention_bwd(q, k, v, cos_t, sin_t, o, lse, dout, dq, dk, dv, accumulate, B,
                                 T, H, hd, scale, workspace, workspace_bytes, stream);
    int rc = attn_check(q, k, v, cos_t, sin_t, B, T, H, hd);
    if (rc)
        return rc;
    if (!B || !T || !H)
        return TTK_OK;
    if (!o || !lse || !dout || !dq || !dk || !dv)
        return set_error(TTK_ERR_ARG, "attention_bwd: null pointer");
    if (!workspace || workspace_bytes < ttk_attention_bwd_ex_workspace_size(B, T, H, hd))
        return set_error(TTK_ERR_ARG, "attention_bwd: workspace too small");
    rc = attn_align_check({q, k, v, cos_t, sin_t, o, dout, dq, dk, dv, fwd_workspace});
    if (rc)
        return rc;
    const bool tc = attn_impl() == 0 && attention_tc_supported(static_cast<int>(hd));
    return attention_mma_backward(static_cast<int>(hd), q, k, v, cos_t, sin_t, o, lse, dout, dq,
                                  dk, dv, accumulate, B, T, H, scale, workspace, tc,
                                  S(stream), fwd_workspace);
}

}  // extern "C"
