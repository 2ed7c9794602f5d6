// Fused causal attention with RoPE on the tensor cores (warp-level
// mma.sync m16n8k16 bf16 with an fp32 accumulator), fp32-accurate through the
// same three-term bf16 split as the GEMM: every operand x is held as
// hi = bf16_rn(x), lo = bf16_rn(x - hi), and each product is
// lo*hi + hi*lo + hi*hi.
//
// Replaces the attention block of GPTModel::forward (model.cpp:127-141:
// rope(q), rope(k), bmm, scale, -1e9 causal mask, softmax, bmm) and its
// backward. Flash-style: scores never reach HBM; the forward keeps an online
// softmax per query row and saves lse = m + log(l) for the backward.
//
// Data flow:
//   attn_split_kernel  q/k (rotated by RoPE, q also scaled by 1/sqrt(hd)), v,
//                      dO: fp32 [B,T,H,HD] -> bf16 hi|lo planes [B,H,T,HD]
//   attn_fwd_mma       per CTA 128 query rows (8 warps x 16); K/V tiles of 64
//                      keys double-buffered in shared memory by cp.async;
//                      S = Q K^T, online softmax, O += P V
//   (backward: attn_bwd_mma_dkv / attn_bwd_mma_dq, below)
// Shared tiles are [rows][HD] bf16 with the 16-byte chunks of each row XOR
// swizzled so every ldmatrix phase hits 8 distinct bank groups.
#include <algorithm>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ttk_common.cuh"
#include "ttk_internal.h"

namespace ttk {
namespace fa {

// ------------------------------------------------------------ primitives --

// Not volatile: a pure register-to-register op, free for the compiler to
// schedule between independent accumulators.
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Three-term products c[j0 + 2p + {0,1}] += A * B_p for NP pairs of n8 tiles
// (B_p as loaded by frag_b_rows / frag_b_cols: [0],[1] the first tile, [2],[3]
// the second), in pass-major order: every lo*hi term, then every hi*lo, then
// every hi*hi. Each accumulator still sums its terms smallest first, and
// consecutive MMAs go to different accumulators, so the tensor pipe is not
// held up by the latency of a dependent MMA.
template <int NP, int N>
__device__ __forceinline__ void mma3_pairs(float (&c)[N][4], int j0, const uint32_t (&ah)[4],
                                           const uint32_t (&al)[4], const uint32_t (&bh)[NP][4],
                                           const uint32_t (&bl)[NP][4]) {
#pragma unroll
    for (int p = 0; p < NP; ++p) {
        mma16816(c[j0 + 2 * p], al, bh[p][0], bh[p][1]);
        mma16816(c[j0 + 2 * p + 1], al, bh[p][2], bh[p][3]);
    }
#pragma unroll
    for (int p = 0; p < NP; ++p) {
        mma16816(c[j0 + 2 * p], ah, bl[p][0], bl[p][1]);
        mma16816(c[j0 + 2 * p + 1], ah, bl[p][2], bl[p][3]);
    }
#pragma unroll
    for (int p = 0; p < NP; ++p) {
        mma16816(c[j0 + 2 * p], ah, bh[p][0], bh[p][1]);
        mma16816(c[j0 + 2 * p + 1], ah, bh[p][2], bh[p][3]);
    }
}

// Two mma3_pairs groups (different A, B and accumulators) interleaved pass by
// pass: 4*NP independent accumulators per pass.
template <int NP, int N1, int N2>
__device__ __forceinline__ void mma3_dual(float (&c1)[N1][4], int j1, const uint32_t (&a1h)[4],
                                          const uint32_t (&a1l)[4], const uint32_t (&b1h)[NP][4],
                                          const uint32_t (&b1l)[NP][4], float (&c2)[N2][4], int j2,
                                          const uint32_t (&a2h)[4], const uint32_t (&a2l)[4],
                                          const uint32_t (&b2h)[NP][4],
                                          const uint32_t (&b2l)[NP][4]) {
#pragma unroll
    for (int pass = 0; pass < 3; ++pass) {
#pragma unroll
        for (int p = 0; p < NP; ++p) {
            const uint32_t(&x1)[4] = pass == 0 ? a1l : a1h;
            const uint32_t(&x2)[4] = pass == 0 ? a2l : a2h;
            const uint32_t(&y1)[4] = pass == 1 ? b1l[p] : b1h[p];
            const uint32_t(&y2)[4] = pass == 1 ? b2l[p] : b2h[p];
            mma16816(c1[j1 + 2 * p], x1, y1[0], y1[1]);
            mma16816(c1[j1 + 2 * p + 1], x1, y1[2], y1[3]);
            mma16816(c2[j2 + 2 * p], x2, y2[0], y2[1]);
            mma16816(c2[j2 + 2 * p + 1], x2, y2[2], y2[3]);
        }
    }
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    const int n = valid ? 16 : 0;  // 0: zero-fill the 16 bytes
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n)
                 : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// hi|lo bf16 pair of each of two fp32 values, packed as bf16x2 words.
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat16 h0 = __float2bfloat16_rn(x0), h1 = __float2bfloat16_rn(x1);
    const __nv_bfloat16 l0 = __float2bfloat16_rn(x0 - __bfloat162float(h0));
    const __nv_bfloat16 l1 = __float2bfloat16_rn(x1 - __bfloat162float(h1));
    hi = static_cast<uint32_t>(__bfloat16_as_ushort(h0)) |
         (static_cast<uint32_t>(__bfloat16_as_ushort(h1)) << 16);
    lo = static_cast<uint32_t>(__bfloat16_as_ushort(l0)) |
         (static_cast<uint32_t>(__bfloat16_as_ushort(l1)) << 16);
}

// Byte offset of 16-byte chunk c of row r in a [rows][HD] bf16 tile.
template <int HD>
__device__ __forceinline__ uint32_t tile_off(int r, int c) {
    constexpr int C = HD / 8;  // chunks per row
    const int pc = C >= 8 ? (c ^ (r & 7)) : (c ^ ((r >> 1) & 3));
    return static_cast<uint32_t>((r * C + pc) * 16);
}

// Copy rows [t0, t0+ROWS) of one (b,h) slice of a [B,H,T,HD] bf16 plane into
// a swizzled tile (rows past T zero-filled).
template <int HD, int ROWS, int NT>
__device__ __forceinline__ void load_tile(uint32_t sdst, const __nv_bfloat16* __restrict__ plane,
                                          int64_t bh, int64_t t0, int64_t T) {
    constexpr int C = HD / 8;
    for (int i = threadIdx.x; i < ROWS * C; i += NT) {
        const int r = i / C, c = i % C;
        const int64_t t = t0 + r;
        const bool ok = t < T;
        const __nv_bfloat16* src = plane + ((bh * T + (ok ? t : 0)) * HD + c * 8);
        cp_async16(sdst + tile_off<HD>(r, c), src, ok);
    }
}

// A fragment (16 rows x 16 cols at (row0, col0)) of a swizzled tile.
template <int HD>
__device__ __forceinline__ void frag_a(uint32_t (&a)[4], uint32_t tile, int row0, int col0) {
    const int lane = threadIdx.x & 31;
    const int r = row0 + (lane & 7) + ((lane >> 3) & 1) * 8;
    const int c = (col0 >> 3) + (lane >> 4);
    ldsm_x4(a, tile + tile_off<HD>(r, c));
}

// B fragments of two n8 tiles whose n index is the tile ROW (K stored
// [keys][HD], product over HD): rows n0..n0+15, k cols k0..k0+15.
// b[0],b[1]: n-tile n0..n0+7 ; b[2],b[3]: n-tile n0+8..n0+15.
template <int HD>
__device__ __forceinline__ void frag_b_rows(uint32_t (&b)[4], uint32_t tile, int n0, int k0) {
    const int lane = threadIdx.x & 31;
    const int r = n0 + (lane & 7) + (lane >> 4) * 8;
    const int c = (k0 >> 3) + ((lane >> 3) & 1);
    ldsm_x4(b, tile + tile_off<HD>(r, c));
}

// B fragments of two n8 tiles whose k index is the tile ROW (V stored
// [keys][HD], product over keys): k rows k0..k0+15, n cols n0..n0+15.
template <int HD>
__device__ __forceinline__ void frag_b_cols(uint32_t (&b)[4], uint32_t tile, int k0, int n0) {
    const int lane = threadIdx.x & 31;
    const int r = k0 + (lane & 7) + ((lane >> 3) & 1) * 8;
    const int c = (n0 >> 3) + (lane >> 4);
    ldsm_x4_t(b, tile + tile_off<HD>(r, c));
}

// ------------------------------------------------------------- prep pass --
// out_hi/out_lo [B,H,T,HD] = split(rope?(x) * mul) for x [B,T,H,HD]. Each
// thread takes 4 consecutive columns d of the first half and their RoPE
// partners d + HD/2 (float4 loads, 8-byte bf16x4 stores).
__device__ __forceinline__ void split4(const float (&v)[4], uint2& hi, uint2& lo) {
    uint32_t h0, h1, l0, l1;
    split_pair_bf16(v[0], v[1], h0, l0);
    split_pair_bf16(v[2], v[3], h1, l1);
    hi = make_uint2(h0, h1);
    lo = make_uint2(l0, l1);
}

// Launch shape: blockIdx.y strides over the B*H heads, blockIdx.x over time;
// a block of 256 threads covers 256/Q rows (time steps) of one head per
// sweep, Q = HD/8 threads per row, each thread one column quad of each half
// row (the RoPE pair). The head's (b, h) is divided out once per head, not
// per element.
__global__ void attn_split_kernel(const float* __restrict__ x, const float* __restrict__ cs,
                                  const float* __restrict__ sn, int rope, float mul,
                                  __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo,
                                  int64_t B, int64_t T, int64_t H, int64_t HD) {
    const int HH = static_cast<int>(HD / 2), Q = HH / 4;  // column quads per half row
    const int rpb = blockDim.x / Q;
    const int lr = threadIdx.x / Q, d = (threadIdx.x % Q) * 4;
    if (lr >= rpb)
        return;
    for (int64_t bh = blockIdx.y; bh < B * H; bh += gridDim.y) {
        const int64_t b = bh / H, h = bh - b * H;
        for (int64_t t = static_cast<int64_t>(blockIdx.x) * rpb + lr; t < T;
             t += static_cast<int64_t>(gridDim.x) * rpb) {
            const float* src = x + ((b * T + t) * H + h) * HD;
            const float4 a = __ldg(reinterpret_cast<const float4*>(src + d));
            const float4 c = __ldg(reinterpret_cast<const float4*>(src + d + HH));
            float x1[4] = {a.x, a.y, a.z, a.w}, x2[4] = {c.x, c.y, c.z, c.w};
            if (rope) {
                const float4 co = __ldg(reinterpret_cast<const float4*>(cs + t * HH + d));
                const float4 si = __ldg(reinterpret_cast<const float4*>(sn + t * HH + d));
                const float cv[4] = {co.x, co.y, co.z, co.w}, sv[4] = {si.x, si.y, si.z, si.w};
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float r1 = x1[u] * cv[u] - x2[u] * sv[u],
                                r2 = x1[u] * sv[u] + x2[u] * cv[u];
                    x1[u] = r1, x2[u] = r2;
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
                x1[u] *= mul, x2[u] *= mul;
            const int64_t o = (bh * T + t) * HD;
            uint2 h1, l1, h2, l2;
            split4(x1, h1, l1);
            split4(x2, h2, l2);
            *reinterpret_cast<uint2*>(hi + o + d) = h1;
            *reinterpret_cast<uint2*>(lo + o + d) = l1;
            *reinterpret_cast<uint2*>(hi + o + d + HH) = h2;
            *reinterpret_cast<uint2*>(lo + o + d + HH) = l2;
        }
    }
}

// --------------------------------------------------------------- forward --
constexpr int FWD_BQ = 128;  // query rows per CTA (8 warps x 16)
constexpr int BKV = 64;      // keys per tile
constexpr int FWD_THREADS = 256;

template <int HD>
struct FwdSmem {
    static constexpr int TILE = BKV * HD * 2;       // bytes of one [64][HD] bf16 plane tile
    static constexpr int QTILE = FWD_BQ * HD * 2;  // [128][HD]
    static constexpr int KV_STAGE = 4 * TILE;      // K hi, K lo, V hi, V lo
    static constexpr int BYTES = 2 * QTILE + 2 * KV_STAGE;
};

template <int HD>
__global__ void __launch_bounds__(FWD_THREADS) attn_fwd_mma(
    const __nv_bfloat16* __restrict__ qh, const __nv_bfloat16* __restrict__ ql,
    const __nv_bfloat16* __restrict__ kh, const __nv_bfloat16* __restrict__ kl,
    const __nv_bfloat16* __restrict__ vh, const __nv_bfloat16* __restrict__ vl,
    float* __restrict__ o, float* __restrict__ lse, int64_t T, int H) {
    using SM = FwdSmem<HD>;
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t s_base = smem_u32(smem);
    const uint32_t sQh = s_base, sQl = s_base + SM::QTILE;
    const uint32_t sKV = s_base + 2 * SM::QTILE;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, tq = lane & 3;
    const int qb = blockIdx.x;
    const int64_t bh = blockIdx.y;
    const int64_t q0 = static_cast<int64_t>(qb) * FWD_BQ;

    load_tile<HD, FWD_BQ, FWD_THREADS>(sQh, qh, bh, q0, T);
    load_tile<HD, FWD_BQ, FWD_THREADS>(sQl, ql, bh, q0, T);
    const int64_t q_last = min(q0 + FWD_BQ, T) - 1;
    const int nkb = static_cast<int>(q_last / BKV) + 1;  // causal: key blocks <= last query
    auto issue_kv = [&](int kb, int stage) {
        const uint32_t st = sKV + stage * SM::KV_STAGE;
        const int64_t k0 = static_cast<int64_t>(kb) * BKV;
        load_tile<HD, BKV, FWD_THREADS>(st, kh, bh, k0, T);
        load_tile<HD, BKV, FWD_THREADS>(st + SM::TILE, kl, bh, k0, T);
        load_tile<HD, BKV, FWD_THREADS>(st + 2 * SM::TILE, vh, bh, k0, T);
        load_tile<HD, BKV, FWD_THREADS>(st + 3 * SM::TILE, vl, bh, k0, T);
    };
    issue_kv(0, 0);
    cp_async_commit();

    constexpr int NO = HD / 8;  // n8 tiles of the output row
    float acc[NO][4];
#pragma unroll
    for (int j = 0; j < NO; ++j)
        acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
    const int row_lo = warp * 16 + g;  // rows of c0/c1 (g) and c2/c3 (g + 8)
    const int64_t qr0 = q0 + row_lo, qr1 = qr0 + 8;

    for (int kb = 0; kb < nkb; ++kb) {
        if (kb + 1 < nkb)
            issue_kv(kb + 1, (kb + 1) & 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const uint32_t st = sKV + (kb & 1) * SM::KV_STAGE;
        const uint32_t sKh = st, sKl = st + SM::TILE, sVh = st + 2 * SM::TILE,
                       sVl = st + 3 * SM::TILE;
        const int64_t k0 = static_cast<int64_t>(kb) * BKV;
        // Skip warps whose 16 rows all precede this key block.
        const bool active = (q0 + warp * 16 + 15) >= k0;
        if (active) {
            float s[8][4];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
            for (int kk = 0; kk < HD; kk += 16) {
                uint32_t ah[4], al[4];
                frag_a<HD>(ah, sQh, warp * 16, kk);
                frag_a<HD>(al, sQl, warp * 16, kk);
                uint32_t bh[4][4], bl[4][4];  // all 64 keys: 8 n8 tiles
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    frag_b_rows<HD>(bh[p], sKh, p * 16, kk);
                    frag_b_rows<HD>(bl[p], sKl, p * 16, kk);
                }
                mma3_pairs<4>(s, 0, ah, al, bh, bl);
            }
            // mask (causal / past T) and online softmax; q was pre-scaled
            float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                const int64_t kc = k0 + nt * 8 + 2 * tq;
                if (kc > qr0 || kc >= T) s[nt][0] = -INFINITY;
                if (kc + 1 > qr0 || kc + 1 >= T) s[nt][1] = -INFINITY;
                if (kc > qr1 || kc >= T) s[nt][2] = -INFINITY;
                if (kc + 1 > qr1 || kc + 1 >= T) s[nt][3] = -INFINITY;
                mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
                mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
            }
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
            const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
            // A row with no live key yet keeps m = -inf and contributes nothing.
            const float al0 = (m0 == -INFINITY) ? 0.0f : expf(m0 - mn0);
            const float al1 = (m1 == -INFINITY) ? 0.0f : expf(m1 - mn1);
            float rs0 = 0.0f, rs1 = 0.0f;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                s[nt][0] = (s[nt][0] == -INFINITY) ? 0.0f : expf(s[nt][0] - mn0);
                s[nt][1] = (s[nt][1] == -INFINITY) ? 0.0f : expf(s[nt][1] - mn0);
                s[nt][2] = (s[nt][2] == -INFINITY) ? 0.0f : expf(s[nt][2] - mn1);
                s[nt][3] = (s[nt][3] == -INFINITY) ? 0.0f : expf(s[nt][3] - mn1);
                rs0 += s[nt][0] + s[nt][1];
                rs1 += s[nt][2] + s[nt][3];
            }
            rs0 += __shfl_xor_sync(0xffffffffu, rs0, 1);
            rs0 += __shfl_xor_sync(0xffffffffu, rs0, 2);
            rs1 += __shfl_xor_sync(0xffffffffu, rs1, 1);
            rs1 += __shfl_xor_sync(0xffffffffu, rs1, 2);
            l0 = l0 * al0 + rs0;
            l1 = l1 * al1 + rs1;
            m0 = (mn0 == -INFINITY) ? m0 : mn0;
            m1 = (mn1 == -INFINITY) ? m1 : mn1;
#pragma unroll
            for (int j = 0; j < NO; ++j) {
                acc[j][0] *= al0, acc[j][1] *= al0;
                acc[j][2] *= al1, acc[j][3] *= al1;
            }
            // O += P V over the 64 keys: 4 k16 chunks of P (accumulator tiles
            // 2c and 2c+1 form the A fragment of chunk c).
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t ph[4], pl[4];
                split2(s[2 * c][0], s[2 * c][1], ph[0], pl[0]);
                split2(s[2 * c][2], s[2 * c][3], ph[1], pl[1]);
                split2(s[2 * c + 1][0], s[2 * c + 1][1], ph[2], pl[2]);
                split2(s[2 * c + 1][2], s[2 * c + 1][3], ph[3], pl[3]);
                constexpr int NP = NO >= 8 ? 4 : NO / 2;  // tile pairs per batch
#pragma unroll
                for (int j = 0; j < NO; j += 2 * NP) {
                    uint32_t bh[NP][4], bl[NP][4];
#pragma unroll
                    for (int p = 0; p < NP; ++p) {
                        frag_b_cols<HD>(bh[p], sVh, c * 16, (j + 2 * p) * 8);
                        frag_b_cols<HD>(bl[p], sVl, c * 16, (j + 2 * p) * 8);
                    }
                    mma3_pairs<NP>(acc, j, ph, pl, bh, bl);
                }
            }
        }
        __syncthreads();  // this stage is refilled two iterations later
    }
    // O / l to [B,T,H,HD]; lse = m + log(l)
    const int64_t b = bh / H, h = bh % H;
    const float inv0 = l0 > 0.0f ? 1.0f / l0 : 0.0f, inv1 = l1 > 0.0f ? 1.0f / l1 : 0.0f;
    if (qr0 < T) {
        float* dst = o + ((b * T + qr0) * H + h) * HD;
#pragma unroll
        for (int j = 0; j < NO; ++j)
            *reinterpret_cast<float2*>(dst + j * 8 + 2 * tq) =
                make_float2(acc[j][0] * inv0, acc[j][1] * inv0);
        if (tq == 0)
            lse[bh * T + qr0] = m0 + logf(l0);
    }
    if (qr1 < T) {
        float* dst = o + ((b * T + qr1) * H + h) * HD;
#pragma unroll
        for (int j = 0; j < NO; ++j)
            *reinterpret_cast<float2*>(dst + j * 8 + 2 * tq) =
                make_float2(acc[j][2] * inv1, acc[j][3] * inv1);
        if (tq == 0)
            lse[bh * T + qr1] = m1 + logf(l1);
    }
}

}  // namespace fa
}  // namespace ttk

namespace ttk {
namespace fa {

// D[bh][t] = sum_d dO[t][d] * O[t][d] (fp32, [B,T,H,HD] inputs); with `ld`,
// also the table ld[bh][t] = (lse[bh][t] * log2 e, D[bh][t]) with rows padded
// to T32 (the padding is zeroed beforehand).
__global__ void attn_rowdot_kernel(const float* __restrict__ o, const float* __restrict__ dout,
                                   float* __restrict__ Dv, int64_t B, int64_t T, int64_t H,
                                   int64_t HD, const float* __restrict__ lse,
                                   float* __restrict__ ld, int64_t T32) {
    const int lane = threadIdx.x & 31;
    const int64_t rows = B * T * H;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
         r < rows; r += warps) {
        const float* a = o + r * HD;
        const float* g = dout + r * HD;
        float s = 0.0f;
        for (int64_t d = lane; d < HD; d += 32)
            s += a[d] * g[d];
        s = warp_sum(s);
        if (lane == 0) {
            const int64_t h = r % H, t = (r / H) % T, b = r / (H * T);
            Dv[(b * H + h) * T + t] = s;
            if (ld) {
                float* e = ld + ((b * H + h) * T32 + t) * 2;
                e[0] = lse[(b * H + h) * T + t] * 1.4426950408889634f;
                e[1] = s;
            }
        }
    }
}

// Write a gradient held in accumulator fragments (two rows per thread, cols
// j*8 + 2*tq + {0,1}) to dst [B,T,H,HD], scaled, with the RoPE transpose
// rotation when `rope` (pairs d, d + HD/2 live in tiles j, j + HD/16).
template <int HD>
__device__ __forceinline__ void store_grad_rows(const float (&acc)[HD / 8][4], int64_t t_lo,
                                               int64_t T, int64_t b, int64_t h, int64_t H,
                                               const float* __restrict__ cs,
                                               const float* __restrict__ sn, bool rope,
                                               float scale, int accumulate,
                                               float* __restrict__ dst) {
    const int lane = threadIdx.x & 31, tq = lane & 3;
    constexpr int NO = HD / 8, HH = HD / 2;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const int64_t t = t_lo + half * 8;
        if (t >= T)
            continue;
        float* row = dst + ((b * T + t) * H + h) * HD;
#pragma unroll
        for (int j = 0; j < NO / 2; ++j) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int d = j * 8 + 2 * tq + e;
                float g1 = acc[j][half * 2 + e] * scale;
                float g2 = acc[j + NO / 2][half * 2 + e] * scale;
                if (rope) {
                    const float c = cs[t * HH + d], s = sn[t * HH + d];
                    const float r1 = g1 * c + g2 * s, r2 = -g1 * s + g2 * c;
                    g1 = r1, g2 = r2;
                }
                if (accumulate) {
                    row[d] += g1;
                    row[d + HH] += g2;
                } else {
                    row[d] = g1;
                    row[d + HH] = g2;
                }
            }
        }
    }
}

// ---------------------------------------------------------- dK, dV kernel --
// CTA: 128 keys (8 warps x 16), loops over query blocks of 32 rows from the
// diagonal on; S^T = K Q^T and dP^T = V dO^T land in accumulator fragments
// that are directly the A operands of dV += P^T dO and dK += dS^T Q.
constexpr int DKV_BK = 128;
constexpr int DKV_BQ = 32;
constexpr int BWD_THREADS = 256;

template <int HD>
struct DkvSmem {
    static constexpr int KT = DKV_BK * HD * 2;  // one [128][HD] bf16 plane
    static constexpr int QT = DKV_BQ * HD * 2;  // one [32][HD] bf16 plane
    static constexpr int QSTAGE = 4 * QT + 2 * DKV_BQ * 4;  // Q hi|lo, dO hi|lo, lse, D
    static constexpr int BYTES = 4 * KT + 2 * QSTAGE;
};

template <int HD>
__global__ void __launch_bounds__(BWD_THREADS) attn_bwd_mma_dkv(
    const __nv_bfloat16* __restrict__ qh, const __nv_bfloat16* __restrict__ ql,
    const __nv_bfloat16* __restrict__ kh, const __nv_bfloat16* __restrict__ kl,
    const __nv_bfloat16* __restrict__ vh, const __nv_bfloat16* __restrict__ vl,
    const __nv_bfloat16* __restrict__ dh, const __nv_bfloat16* __restrict__ dl,
    const float* __restrict__ lse, const float* __restrict__ Dv, const float* __restrict__ cs,
    const float* __restrict__ sn, float* __restrict__ dk, float* __restrict__ dv, int accumulate,
    int64_t T, int H) {
    using SM = DkvSmem<HD>;
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t base = smem_u32(smem);
    const uint32_t sKh = base, sKl = base + SM::KT, sVh = base + 2 * SM::KT,
                   sVl = base + 3 * SM::KT, sQ = base + 4 * SM::KT;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, tq = lane & 3;
    const int64_t bh = blockIdx.y;
    const int64_t k0 = static_cast<int64_t>(blockIdx.x) * DKV_BK;
    load_tile<HD, DKV_BK, BWD_THREADS>(sKh, kh, bh, k0, T);
    load_tile<HD, DKV_BK, BWD_THREADS>(sKl, kl, bh, k0, T);
    load_tile<HD, DKV_BK, BWD_THREADS>(sVh, vh, bh, k0, T);
    load_tile<HD, DKV_BK, BWD_THREADS>(sVl, vl, bh, k0, T);
    const int qb_first = static_cast<int>(k0 / DKV_BQ);
    const int nqb = static_cast<int>((T + DKV_BQ - 1) / DKV_BQ);
    auto issue_q = [&](int qb, int stage) {
        const uint32_t st = sQ + stage * SM::QSTAGE;
        const int64_t q0 = static_cast<int64_t>(qb) * DKV_BQ;
        load_tile<HD, DKV_BQ, BWD_THREADS>(st, qh, bh, q0, T);
        load_tile<HD, DKV_BQ, BWD_THREADS>(st + SM::QT, ql, bh, q0, T);
        load_tile<HD, DKV_BQ, BWD_THREADS>(st + 2 * SM::QT, dh, bh, q0, T);
        load_tile<HD, DKV_BQ, BWD_THREADS>(st + 3 * SM::QT, dl, bh, q0, T);
        // lse and D for these rows (plain loads: the rows need not be 16-byte
        // aligned); rows past T read as 0. The stage being filled was last
        // read before the previous iteration's closing barrier.
        float* s_l = reinterpret_cast<float*>(smem + (st - base) + 4 * SM::QT);
        for (int i = threadIdx.x; i < DKV_BQ; i += BWD_THREADS) {
            const int64_t q = q0 + i;
            s_l[i] = q < T ? lse[bh * T + q] : 0.0f;
            s_l[DKV_BQ + i] = q < T ? Dv[bh * T + q] : 0.0f;
        }
    };
    if (qb_first < nqb)
        issue_q(qb_first, 0);
    cp_async_commit();

    constexpr int NO = HD / 8;
    float dK[NO][4], dV[NO][4];
#pragma unroll
    for (int j = 0; j < NO; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e)
            dK[j][e] = 0.0f, dV[j][e] = 0.0f;
    const int64_t key0 = k0 + warp * 16 + g, key1 = key0 + 8;  // rows of this thread

    for (int qb = qb_first; qb < nqb; ++qb) {
        const int stage = (qb - qb_first) & 1;
        if (qb + 1 < nqb)
            issue_q(qb + 1, stage ^ 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const uint32_t st = sQ + stage * SM::QSTAGE;
        const uint32_t sQh = st, sQl = st + SM::QT, sDh = st + 2 * SM::QT, sDl = st + 3 * SM::QT;
        const float* s_lse = reinterpret_cast<const float*>(smem + (st - base) + 4 * SM::QT);
        const float* s_D = s_lse + DKV_BQ;
        const int64_t q0 = static_cast<int64_t>(qb) * DKV_BQ;
        // this warp's 16 keys are all after this query block: nothing to do
        if (k0 + warp * 16 <= q0 + DKV_BQ - 1) {
            constexpr int NQ = DKV_BQ / 8;  // n8 tiles over the query block
            float sT[NQ][4], pT[NQ][4];
#pragma unroll
            for (int j = 0; j < NQ; ++j)
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    sT[j][e] = 0.0f, pT[j][e] = 0.0f;
#pragma unroll
            for (int kk = 0; kk < HD; kk += 16) {
                uint32_t akh[4], akl[4], avh[4], avl[4];
                frag_a<HD>(akh, sKh, warp * 16, kk);
                frag_a<HD>(akl, sKl, warp * 16, kk);
                frag_a<HD>(avh, sVh, warp * 16, kk);
                frag_a<HD>(avl, sVl, warp * 16, kk);
#pragma unroll
                for (int nt = 0; nt < NQ; nt += 2) {
                    uint32_t bq[1][4], bql[1][4], bd[1][4], bdl[1][4];
                    frag_b_rows<HD>(bq[0], sQh, nt * 8, kk);
                    frag_b_rows<HD>(bql[0], sQl, nt * 8, kk);
                    frag_b_rows<HD>(bd[0], sDh, nt * 8, kk);
                    frag_b_rows<HD>(bdl[0], sDl, nt * 8, kk);
                    mma3_dual<1>(sT, nt, akh, akl, bq, bql, pT, nt, avh, avl, bd, bdl);
                }
            }
            // P^T = exp(S^T - lse[q]) on live (key <= q < T) entries; dS^T =
            // P^T (dP^T - D[q]). sT becomes P^T, pT becomes dS^T.
#pragma unroll
            for (int nt = 0; nt < NQ; ++nt) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int qi = nt * 8 + 2 * tq + (e & 1);
                    const int64_t q = q0 + qi;
                    const int64_t key = (e < 2) ? key0 : key1;
                    const bool live = key <= q && q < T;
                    const float p = live ? expf(sT[nt][e] - s_lse[qi]) : 0.0f;
                    pT[nt][e] = p * (pT[nt][e] - s_D[qi]);
                    sT[nt][e] = p;
                }
            }
            // dV += P^T dO ; dK += dS^T Q  (k = the 32 query rows)
#pragma unroll
            for (int c = 0; c < DKV_BQ / 16; ++c) {
                uint32_t ph[4], pl[4], sh[4], sl[4];
                split2(sT[2 * c][0], sT[2 * c][1], ph[0], pl[0]);
                split2(sT[2 * c][2], sT[2 * c][3], ph[1], pl[1]);
                split2(sT[2 * c + 1][0], sT[2 * c + 1][1], ph[2], pl[2]);
                split2(sT[2 * c + 1][2], sT[2 * c + 1][3], ph[3], pl[3]);
                split2(pT[2 * c][0], pT[2 * c][1], sh[0], sl[0]);
                split2(pT[2 * c][2], pT[2 * c][3], sh[1], sl[1]);
                split2(pT[2 * c + 1][0], pT[2 * c + 1][1], sh[2], sl[2]);
                split2(pT[2 * c + 1][2], pT[2 * c + 1][3], sh[3], sl[3]);
#pragma unroll
                for (int j = 0; j < NO; j += 2) {
                    uint32_t bd[1][4], bdl[1][4], bq[1][4], bql[1][4];
                    frag_b_cols<HD>(bd[0], sDh, c * 16, j * 8);
                    frag_b_cols<HD>(bdl[0], sDl, c * 16, j * 8);
                    frag_b_cols<HD>(bq[0], sQh, c * 16, j * 8);
                    frag_b_cols<HD>(bql[0], sQl, c * 16, j * 8);
                    mma3_dual<1>(dV, j, ph, pl, bd, bdl, dK, j, sh, sl, bq, bql);
                }
            }
        }
        __syncthreads();
    }
    const int64_t b = bh / H, h = bh % H;
    // dK: q was pre-scaled, so dS^T Q_scaled is already the gradient of the
    // rotated k; dV needs no rotation.
    store_grad_rows<HD>(dK, key0, T, b, h, H, cs, sn, true, 1.0f, accumulate, dk);
    store_grad_rows<HD>(dV, key0, T, b, h, H, cs, sn, false, 1.0f, accumulate, dv);
}

// ---------------------------------------------------------------- dQ kernel --
// CTA: 128 query rows (8 warps x 16); loops over key blocks of 32 up to the
// diagonal: S = Q K^T, dP = dO V^T, dS = P (dP - D), dQ += dS K.
constexpr int DQ_BQ = 128;
constexpr int DQ_BK = 32;

template <int HD>
struct DqSmem {
    static constexpr int QT = DQ_BQ * HD * 2;
    static constexpr int KT = DQ_BK * HD * 2;
    static constexpr int KSTAGE = 4 * KT;  // K hi|lo, V hi|lo
    static constexpr int BYTES = 4 * QT + 2 * KSTAGE;
};

template <int HD>
__global__ void __launch_bounds__(BWD_THREADS) attn_bwd_mma_dq(
    const __nv_bfloat16* __restrict__ qh, const __nv_bfloat16* __restrict__ ql,
    const __nv_bfloat16* __restrict__ kh, const __nv_bfloat16* __restrict__ kl,
    const __nv_bfloat16* __restrict__ vh, const __nv_bfloat16* __restrict__ vl,
    const __nv_bfloat16* __restrict__ dh, const __nv_bfloat16* __restrict__ dl,
    const float* __restrict__ lse, const float* __restrict__ Dv, const float* __restrict__ cs,
    const float* __restrict__ sn, float* __restrict__ dq, int accumulate, float scale, int64_t T,
    int H) {
    using SM = DqSmem<HD>;
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t base = smem_u32(smem);
    const uint32_t sQh = base, sQl = base + SM::QT, sDh = base + 2 * SM::QT,
                   sDl = base + 3 * SM::QT, sK = base + 4 * SM::QT;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, tq = lane & 3;
    const int64_t bh = blockIdx.y;
    const int64_t q0 = static_cast<int64_t>(blockIdx.x) * DQ_BQ;
    load_tile<HD, DQ_BQ, BWD_THREADS>(sQh, qh, bh, q0, T);
    load_tile<HD, DQ_BQ, BWD_THREADS>(sQl, ql, bh, q0, T);
    load_tile<HD, DQ_BQ, BWD_THREADS>(sDh, dh, bh, q0, T);
    load_tile<HD, DQ_BQ, BWD_THREADS>(sDl, dl, bh, q0, T);
    const int64_t qr0 = q0 + warp * 16 + g, qr1 = qr0 + 8;
    const float lse0 = qr0 < T ? lse[bh * T + qr0] : 0.0f;
    const float lse1 = qr1 < T ? lse[bh * T + qr1] : 0.0f;
    const float D0 = qr0 < T ? Dv[bh * T + qr0] : 0.0f;
    const float D1 = qr1 < T ? Dv[bh * T + qr1] : 0.0f;
    const int64_t q_last = min(q0 + DQ_BQ, T) - 1;
    const int nkb = static_cast<int>(q_last / DQ_BK) + 1;
    auto issue_k = [&](int kb, int stage) {
        const uint32_t st = sK + stage * SM::KSTAGE;
        const int64_t k0 = static_cast<int64_t>(kb) * DQ_BK;
        load_tile<HD, DQ_BK, BWD_THREADS>(st, kh, bh, k0, T);
        load_tile<HD, DQ_BK, BWD_THREADS>(st + SM::KT, kl, bh, k0, T);
        load_tile<HD, DQ_BK, BWD_THREADS>(st + 2 * SM::KT, vh, bh, k0, T);
        load_tile<HD, DQ_BK, BWD_THREADS>(st + 3 * SM::KT, vl, bh, k0, T);
    };
    issue_k(0, 0);
    cp_async_commit();
    constexpr int NO = HD / 8;
    float dQ[NO][4];
#pragma unroll
    for (int j = 0; j < NO; ++j)
        dQ[j][0] = dQ[j][1] = dQ[j][2] = dQ[j][3] = 0.0f;
    for (int kb = 0; kb < nkb; ++kb) {
        if (kb + 1 < nkb)
            issue_k(kb + 1, (kb + 1) & 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const uint32_t st = sK + (kb & 1) * SM::KSTAGE;
        const uint32_t sKh = st, sKl = st + SM::KT, sVh = st + 2 * SM::KT, sVl = st + 3 * SM::KT;
        const int64_t k0 = static_cast<int64_t>(kb) * DQ_BK;
        if (q0 + warp * 16 + 15 >= k0) {
            constexpr int NK = DQ_BK / 8;
            float s[NK][4], dp[NK][4];
#pragma unroll
            for (int j = 0; j < NK; ++j)
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    s[j][e] = 0.0f, dp[j][e] = 0.0f;
#pragma unroll
            for (int kk = 0; kk < HD; kk += 16) {
                uint32_t aq[4], aql[4], ad[4], adl[4];
                frag_a<HD>(aq, sQh, warp * 16, kk);
                frag_a<HD>(aql, sQl, warp * 16, kk);
                frag_a<HD>(ad, sDh, warp * 16, kk);
                frag_a<HD>(adl, sDl, warp * 16, kk);
                constexpr int NP = NK / 2;  // all key tiles of the block at once
                uint32_t bk[NP][4], bkl[NP][4], bv[NP][4], bvl[NP][4];
#pragma unroll
                for (int p = 0; p < NP; ++p) {
                    frag_b_rows<HD>(bk[p], sKh, p * 16, kk);
                    frag_b_rows<HD>(bkl[p], sKl, p * 16, kk);
                    frag_b_rows<HD>(bv[p], sVh, p * 16, kk);
                    frag_b_rows<HD>(bvl[p], sVl, p * 16, kk);
                }
                mma3_dual<NP>(s, 0, aq, aql, bk, bkl, dp, 0, ad, adl, bv, bvl);
            }
#pragma unroll
            for (int nt = 0; nt < NK; ++nt) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int64_t key = k0 + nt * 8 + 2 * tq + (e & 1);
                    const int64_t q = (e < 2) ? qr0 : qr1;
                    const bool live = key <= q && q < T;
                    const float p = live ? expf(s[nt][e] - ((e < 2) ? lse0 : lse1)) : 0.0f;
                    s[nt][e] = p * (dp[nt][e] - ((e < 2) ? D0 : D1));  // dS
                }
            }
#pragma unroll
            for (int c = 0; c < DQ_BK / 16; ++c) {
                uint32_t sh[4], sl[4];
                split2(s[2 * c][0], s[2 * c][1], sh[0], sl[0]);
                split2(s[2 * c][2], s[2 * c][3], sh[1], sl[1]);
                split2(s[2 * c + 1][0], s[2 * c + 1][1], sh[2], sl[2]);
                split2(s[2 * c + 1][2], s[2 * c + 1][3], sh[3], sl[3]);
                constexpr int NP = NO >= 8 ? 4 : NO / 2;
#pragma unroll
                for (int j = 0; j < NO; j += 2 * NP) {
                    uint32_t bk[NP][4], bkl[NP][4];
#pragma unroll
                    for (int p = 0; p < NP; ++p) {
                        frag_b_cols<HD>(bk[p], sKh, c * 16, (j + 2 * p) * 8);
                        frag_b_cols<HD>(bkl[p], sKl, c * 16, (j + 2 * p) * 8);
                    }
                    mma3_pairs<NP>(dQ, j, sh, sl, bk, bkl);
                }
            }
        }
        __syncthreads();
    }
    const int64_t b = bh / H, h = bh % H;
    store_grad_rows<HD>(dQ, qr0, T, b, h, H, cs, sn, true, scale, accumulate, dq);
}

// ------------------------------------------------------------- launchers --

struct SplitBufs {
    __nv_bfloat16 *qh, *ql, *kh, *kl, *vh, *vl, *dh, *dl;
};

inline int launch_split(const float* x, const float* cs, const float* sn, int rope, float mul,
                        __nv_bfloat16* hi, __nv_bfloat16* lo, int64_t B, int64_t T, int64_t H,
                        int64_t HD, cudaStream_t st) {
    if (!B || !T || !H)
        return TTK_OK;
    const int64_t rpb = 256 / (HD / 8);  // time steps per block sweep
    const dim3 grid(static_cast<unsigned>(std::min<int64_t>((T + rpb - 1) / rpb, 1024)),
                    static_cast<unsigned>(std::min<int64_t>(B * H, 65535)));
    attn_split_kernel<<<grid, 256, 0, st>>>(x, cs, sn, rope, mul, hi, lo, B, T, H, HD);
    return check_launch("attn_split_kernel");
}

template <int HD>
int fwd(const float* q, const float* k, const float* v, const float* cs, const float* sn,
        float* o, float* lse, int64_t B, int64_t T, int64_t H, float scale, SplitBufs s, bool tc,
        cudaStream_t st, void* o_split) {
    int rc = launch_split(q, cs, sn, 1, scale, s.qh, s.ql, B, T, H, HD, st);
    if (!rc)
        rc = launch_split(k, cs, sn, 1, 1.0f, s.kh, s.kl, B, T, H, HD, st);
    if (!rc)
        rc = launch_split(v, cs, sn, 0, 1.0f, s.vh, s.vl, B, T, H, HD, st);
    if (rc)
        return rc;
    if (tc)
        return attention_tc_forward_core(HD, s.qh, s.kh, s.vh, o, lse, B, T, H, st,
                                         static_cast<__nv_bfloat16*>(o_split));
    const int smem = FwdSmem<HD>::BYTES;
    cudaFuncSetAttribute(attn_fwd_mma<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    dim3 grid(static_cast<unsigned>((T + FWD_BQ - 1) / FWD_BQ), static_cast<unsigned>(B * H));
    attn_fwd_mma<HD><<<grid, FWD_THREADS, smem, st>>>(s.qh, s.ql, s.kh, s.kl, s.vh, s.vl, o, lse,
                                                      T, static_cast<int>(H));
    rc = check_launch("attn_fwd_mma");
    if (rc || !o_split)
        return rc;
    return gemm_split(o, B * T, H * HD, H * HD, 0, 1, o_split, st);
}

// qkv_ready: s.q*, s.k*, s.v* already hold the forward's splits of q, k, v
// (same inputs, same scale), so only dO is split here.
template <int HD>
int bwd(const float* q, const float* k, const float* v, const float* cs, const float* sn,
        const float* o, const float* lse, const float* dout, float* dq, float* dk, float* dv,
        int accumulate, int64_t B, int64_t T, int64_t H, float scale, SplitBufs s, float* Dv,
        float* ld, bool tc, cudaStream_t st, bool qkv_ready = false, void* dq_split = nullptr,
        void* dk_split = nullptr, void* dv_split = nullptr) {
    int rc = TTK_OK;
    if (!qkv_ready) {
        rc = launch_split(q, cs, sn, 1, scale, s.qh, s.ql, B, T, H, HD, st);
        if (!rc)
            rc = launch_split(k, cs, sn, 1, 1.0f, s.kh, s.kl, B, T, H, HD, st);
        if (!rc)
            rc = launch_split(v, cs, sn, 0, 1.0f, s.vh, s.vl, B, T, H, HD, st);
    }
    if (!rc)
        rc = launch_split(dout, cs, sn, 0, 1.0f, s.dh, s.dl, B, T, H, HD, st);
    if (rc)
        return rc;
    const int64_t T32 = (T + 31) / 32 * 32;
    if (tc) {
        rc = check_cuda(cudaMemsetAsync(ld, 0, static_cast<size_t>(B * H * T32) * 8, st),
                        "attention_bwd: ld table");
        if (rc)
            return rc;
    }
    attn_rowdot_kernel<<<grid_for(B * T * H, 8), 256, 0, st>>>(o, dout, Dv, B, T, H, HD, lse,
                                                                tc ? ld : nullptr, T32);
    rc = check_launch("attn_rowdot_kernel");
    if (rc)
        return rc;
    if (tc)
        return attention_tc_backward_core(HD, s.qh, s.kh, s.vh, s.dh, lse, Dv, ld, T32, cs, sn,
                                          dq, dk, dv, accumulate, B, T, H, scale, st,
                                          static_cast<__nv_bfloat16*>(dq_split),
                                          static_cast<__nv_bfloat16*>(dk_split),
                                          static_cast<__nv_bfloat16*>(dv_split));
    int smem = DkvSmem<HD>::BYTES;
    cudaFuncSetAttribute(attn_bwd_mma_dkv<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    dim3 g1(static_cast<unsigned>((T + DKV_BK - 1) / DKV_BK), static_cast<unsigned>(B * H));
    attn_bwd_mma_dkv<HD><<<g1, BWD_THREADS, smem, st>>>(s.qh, s.ql, s.kh, s.kl, s.vh, s.vl, s.dh,
                                                        s.dl, lse, Dv, cs, sn, dk, dv, accumulate,
                                                        T, static_cast<int>(H));
    rc = check_launch("attn_bwd_mma_dkv");
    if (rc)
        return rc;
    smem = DqSmem<HD>::BYTES;
    cudaFuncSetAttribute(attn_bwd_mma_dq<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    dim3 g2(static_cast<unsigned>((T + DQ_BQ - 1) / DQ_BQ), static_cast<unsigned>(B * H));
    attn_bwd_mma_dq<HD><<<g2, BWD_THREADS, smem, st>>>(s.qh, s.ql, s.kh, s.kl, s.vh, s.vl, s.dh,
                                                       s.dl, lse, Dv, cs, sn, dq, accumulate,
                                                       scale, T, static_cast<int>(H));
    rc = check_launch("attn_bwd_mma_dq");
    const int64_t R = B * T, D = H * HD;
    if (!rc && dq_split)
        rc = gemm_split(dq, R, D, D, 0, 1, dq_split, st);
    if (!rc && dk_split)
        rc = gemm_split(dk, R, D, D, 0, 1, dk_split, st);
    if (!rc && dv_split)
        rc = gemm_split(dv, R, D, D, 0, 1, dv_split, st);
    return rc;
}

}  // namespace fa
}  // namespace ttk

namespace ttk {

int attention_mma_forward(int hd, const float* q, const float* k, const float* v,
                          const float* cs, const float* sn, float* o, float* lse, int64_t B,
                          int64_t T, int64_t H, float scale, void* ws, bool tc,
                          cudaStream_t st, void* o_split) {
    const int64_t n = B * T * H * hd;
    __nv_bfloat16* w = static_cast<__nv_bfloat16*>(ws);
    fa::SplitBufs s{w, w + n, w + 2 * n, w + 3 * n, w + 4 * n, w + 5 * n, nullptr, nullptr};
    switch (hd) {
        case 32: return fa::fwd<32>(q, k, v, cs, sn, o, lse, B, T, H, scale, s, tc, st, o_split);
        case 64: return fa::fwd<64>(q, k, v, cs, sn, o, lse, B, T, H, scale, s, tc, st, o_split);
        default:
            return fa::fwd<128>(q, k, v, cs, sn, o, lse, B, T, H, scale, s, tc, st, o_split);
    }
}

// Workspace: Dv [B*T*H] fp32 (256-byte aligned), then the q, k, v, dO planes
// (8n bf16), then the tcgen05 path's (lse, D) table. With fwd_ws (the
// forward's workspace: q, k, v planes, 6n bf16) the q, k, v planes are read
// from there and ws holds Dv, the dO planes and the table.
int attention_mma_backward(int hd, const float* q, const float* k, const float* v,
                           const float* cs, const float* sn, const float* o, const float* lse,
                           const float* dout, float* dq, float* dk, float* dv, int accumulate,
                           int64_t B, int64_t T, int64_t H, float scale, void* ws, bool tc,
                           cudaStream_t st, const void* fwd_ws, void* dq_split, void* dk_split,
                           void* dv_split) {
    const int64_t n = B * T * H * hd;
    float* Dv = static_cast<float*>(ws);
    __nv_bfloat16* w = reinterpret_cast<__nv_bfloat16*>(
        static_cast<char*>(ws) + ((B * T * H * 4 + 255) / 256) * 256);
    fa::SplitBufs s;
    float* ld;
    if (fwd_ws) {
        __nv_bfloat16* f = const_cast<__nv_bfloat16*>(static_cast<const __nv_bfloat16*>(fwd_ws));
        s = fa::SplitBufs{f, f + n, f + 2 * n, f + 3 * n, f + 4 * n, f + 5 * n, w, w + n};
        ld = reinterpret_cast<float*>(w + 2 * n);  // 16-byte aligned: n*4 bytes before it
    } else {
        s = fa::SplitBufs{w, w + n, w + 2 * n, w + 3 * n, w + 4 * n, w + 5 * n, w + 6 * n,
                          w + 7 * n};
        ld = reinterpret_cast<float*>(w + 8 * n);  // 256-byte aligned: n*16 bytes before it
    }
    const bool ready = fwd_ws != nullptr;
    switch (hd) {
        case 32:
            return fa::bwd<32>(q, k, v, cs, sn, o, lse, dout, dq, dk, dv, accumulate, B, T, H,
                               scale, s, Dv, ld, tc, st, ready, dq_split, dk_split, dv_split);
        case 64:
            return fa::bwd<64>(q, k, v, cs, sn, o, lse, dout, dq, dk, dv, accumulate, B, T, H,
                               scale, s, Dv, ld, tc, st, ready, dq_split, dk_split, dv_split);
        default:
            return fa::bwd<128>(q, k, v, cs, sn, o, lse, dout, dq, dk, dv, accumulate, B, T, H,
                                scale, s, Dv, ld, tc, st, ready, dq_split, dk_split, dv_split);
    }
}

}  // namespace ttk
