// Fused causal attention forward on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), fp32-accurate through the three-term bf16 split
// (lo*hi + hi*lo + hi*hi) used by the GEMM and the mma.sync kernels.
//
// Same contract as the mma.sync forward (attention_mma.cu): q, k, v are the
// split planes written by attn_split_kernel ([B,H,T,HD] bf16 hi, then lo, q
// rotated and pre-scaled by 1/sqrt(hd), k rotated); outputs O [B,T,H,HD] fp32
// and lse [B,H,T] (natural log) for the backward. Replaces the attention
// block of GPTModel::forward (model.cpp:127-141).
//
// CTA = one tile of 128 query rows of one (b, h); loops over 64-key blocks
// up to the diagonal. 10 warps:
//   warp 0     TMA producer (one lane): the Q tile once, then K and V tiles
//              through a 3-slot ring in the order the MMAs consume them
//              (K0, K1, V0, K2, V1, ..., V_last)
//   warp 1     TMEM allocator + MMA issuer (one lane):
//                S_j  = Q K_j^T  (M128 N64, K = HD)   -> TMEM S[j % 2]
//                O_j  = P_j V_j  (M128 N=HD, K = 64)  -> TMEM O[j % 2]
//              issued S_{j+1} before O_j so the softmax of block j+1 runs
//              while the tensor core computes O_j
//   warps 2-9  softmax: two warps per TMEM lane quadrant (32 rows), each
//              owning half of the columns of its rows. Per block: read the
//              row's 64 scores (both halves read all 64 so they agree on the
//              running max without exchanging it), mask, p = exp(s - m),
//              split p into bf16 hi|lo and store it to shared memory as the
//              K-major A operand of P V; then fold the previous block's O_j
//              from TMEM into fp32 registers (O = O * exp(m_old - m_new) +
//              O_j). Accumulating O in registers with round-to-nearest adds
//              keeps long key sums free of the tensor-core accumulator's
//              rounding bias.
// Shared-memory tiles are TMA boxes {32 elements, rows, HD/32 chunks, 1, 2
// planes} in the 64-byte swizzle: [plane][chunk][row][64 B], the canonical
// K-major layout for Q, K and P and the MN-major layout for V.
// Every wait is bounded; on expiry the kernel flags the device status, lets
// copies in flight land, waits for issued MMAs, frees TMEM and returns.
// Every TMA load has one destination: the issuing CTA's shared memory.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "ttk_common.cuh"
#include "ttk_internal.h"

namespace ttk {
namespace fatc {

constexpr int BQ = 128;  // query rows per CTA (MMA M, TMEM lanes)
constexpr int BKV = 64;  // keys per block
constexpr int NSLOT = 3;
constexpr int NUM_THREADS = 320;
// Forward: a second MMA-issuing warp (index 10) issues O_j = P_j V_j while
// warp 1 issues the score MMAs.
constexpr int FWD_PV_WARP = 10;
constexpr int FWD_THREADS = 352;
// dK/dV: a second MMA-issuing warp (index 10) after the eight softmax warps.
constexpr int DKV_MMA_B_WARP = 10;
constexpr int DKV_THREADS = 352;
constexpr int SOFTMAX_THREADS = 256;
constexpr uint32_t kSW64 = 4;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

template <int HD>
struct FwdCfg {
    static constexpr int NCH = HD / 32;                 // 32-element chunks per row
    static constexpr int Q_PLANE = NCH * BQ * 64;        // [NCH][128 rows][64 B]
    static constexpr int KV_PLANE = NCH * BKV * 64;      // [NCH][64 rows][64 B]
    static constexpr int P_PLANE = (BKV / 32) * BQ * 64;  // [2 key chunks][128 rows][64 B]
    static constexpr int Q_BYTES = 2 * Q_PLANE;
    static constexpr int SLOT_BYTES = 2 * KV_PLANE;
    static constexpr int P_BYTES = 2 * P_PLANE;
    static constexpr int OFF_SLOT = Q_BYTES;
    static constexpr int OFF_P = OFF_SLOT + NSLOT * SLOT_BYTES;
    static constexpr int OFF_RED = OFF_P + 2 * P_BYTES;  // float [2 halves][128 rows]
    static constexpr int OFF_BAR = OFF_RED + 2 * BQ * 4;
    // q_full, full[3], empty[3], s_full[2], p_full[2], o_full[2], o_free[2], done
    static constexpr int NBARS = 1 + 2 * NSLOT + 8 + 1;
    static constexpr int BYTES = OFF_BAR + 8 * NBARS + 16 /*tmem slot, abort*/ + 1024 /*align*/;
    static constexpr int S_COL = 0;        // S buffers: columns [0, 128)
    static constexpr int O_COL = 2 * BKV;  // O buffers: [128, 128 + 2*HD)
    static constexpr int TMEM_COLS = 512;
    static_assert(O_COL + 2 * HD <= TMEM_COLS, "TMEM budget");
    static_assert(BYTES <= 232448, "shared memory budget");
};

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint32_t pack_bf16x2(__nv_bfloat16 a, __nv_bfloat16 b) {
    return static_cast<uint32_t>(__bfloat16_as_ushort(a)) |
           (static_cast<uint32_t>(__bfloat16_as_ushort(b)) << 16);
}

// K-major operand (Q, K: rows x HD; P: rows x 64 keys), k-step ks of 16
// elements: chunk ks/2 of the plane, 32 B into each 64 B row.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t plane, int rows, int ks) {
    return umma_smem_desc(plane + (ks >> 1) * (rows * 64) + (ks & 1) * 32, 16, 512, kSW64);
}

// MN-major B operand V [64 keys][HD]: k-step ks covers keys 16ks..16ks+15
// (16 rows of 64 B); the HD extent is NCH chunks BKV*64 bytes apart.
__device__ __forceinline__ uint64_t v_desc(uint32_t plane, int ks) {
    return umma_smem_desc(plane + ks * 1024, BKV * 64, 512, kSW64);
}

// Position of K_j / V_j in the producer's ring order (K0, K1, V0, K2, V1, ...,
// V_last): n = 0 for K0, 2j - 1 for K_j (j >= 1), 2j + 2 for V_j before the
// last block and 2 * nblk - 1 for the last V.
__device__ __forceinline__ int ring_pos_k(int j) { return j == 0 ? 0 : 2 * j - 1; }
__device__ __forceinline__ int ring_pos_v(int j, int nblk) {
    return j == nblk - 1 ? 2 * nblk - 1 : 2 * j + 2;
}

template <int HD>
__global__ void __launch_bounds__(FWD_THREADS, 1)
    attn_fwd_tc(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                const __grid_constant__ CUtensorMap map_v, float* __restrict__ o,
                float* __restrict__ lse, int64_t T, int H, __nv_bfloat16* __restrict__ o_split,
                int64_t o_plane) {
    using CF = FwdCfg<HD>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + CF::OFF_BAR);
    uint64_t* q_full = bars;
    uint64_t* full = bars + 1;
    uint64_t* empty = full + NSLOT;
    uint64_t* s_full = empty + NSLOT;
    uint64_t* p_full = s_full + 2;
    uint64_t* o_full = p_full + 2;
    uint64_t* o_free = o_full + 2;
    uint64_t* done = o_free + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nqt = static_cast<int>((T + BQ - 1) / BQ);
    const int qt = nqt - 1 - static_cast<int>(blockIdx.x);  // longest tiles first
    const int64_t q0 = static_cast<int64_t>(qt) * BQ;
    const int64_t bh = blockIdx.y;
    const int64_t q_last = min(q0 + BQ, T) - 1;
    const int nblk = static_cast<int>(q_last / BKV) + 1;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < NSLOT; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_full[b], 1);
            mbar_init(&p_full[b], SOFTMAX_THREADS);
            mbar_init(&o_full[b], 1);
            mbar_init(&o_free[b], SOFTMAX_THREADS);
        }
        mbar_init(done, 2);  // both MMA-issuing warps commit
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&map_q);
        tma_prefetch_desc(&map_k);
        tma_prefetch_desc(&map_v);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, CF::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t s_base = smem_u32(smem);
    // softmax warps: this thread's half row of O, its partial row sum and the
    // final row max (log2 units), kept for the store after the closing barrier
    constexpr int OH = HD / 2;
    float acc[OH];
    float l_own = 0.0f, m_out = -INFINITY;
    float* red = reinterpret_cast<float*>(smem + CF::OFF_RED);

    if (warp == 0) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0) {
            int armed_ph[NSLOT];
#pragma unroll
            for (int i = 0; i < NSLOT; ++i)
                armed_ph[i] = -1;
            mbar_arrive_expect_tx(q_full, CF::Q_BYTES);
            tma_load_5d(smem, &map_q, q_full, 0, static_cast<int>(q0), 0, static_cast<int>(bh), 0);
            int it = 0;
            bool ok = true;
            // consumption order: K0, then (K_i, V_{i-1}) for i >= 1, then V_last
            for (int n = 0; n < 2 * nblk && ok; ++n) {
                const bool is_v = n > 0 && (n == 2 * nblk - 1 || (n & 1) == 0);
                const int j = n == 0 ? 0 : (is_v ? (n == 2 * nblk - 1 ? nblk - 1 : n / 2 - 1)
                                                 : (n + 1) / 2);
                const int slot = it % NSLOT;
                const uint32_t ph = static_cast<uint32_t>((it / NSLOT) & 1);
                if (*abort_flag || !mbar_wait(&empty[slot], ph ^ 1, 21)) {
                    ok = false;
                    break;
                }
                uint8_t* dst = smem + CF::OFF_SLOT + slot * CF::SLOT_BYTES;
                mbar_arrive_expect_tx(&full[slot], CF::SLOT_BYTES);
                tma_load_5d(dst, is_v ? &map_v : &map_k, &full[slot], 0, j * BKV, 0,
                            static_cast<int>(bh), 0);
                armed_ph[slot] = static_cast<int>(ph);
                ++it;
            }
            if (!ok) {
                *abort_flag = 1;
                mbar_wait(q_full, 0, 26);
#pragma unroll
                for (int i = 0; i < NSLOT; ++i)
                    if (armed_ph[i] >= 0)
                        mbar_wait(&full[i], static_cast<uint32_t>(armed_ph[i]), 26);
            }
        }
    } else if (warp == 1 || warp == FWD_PV_WARP) {
        // ------------------------------------------------------- MMA issuers
        // One warp issues at most about one MMA per 64 cycles, so two warps
        // share the work (each loop warp-uniform; lane 0 issues):
        //   warp 1:  S_j = Q K_j^T into S[j % 2], once the softmax of block
        //            j - 2 has read that buffer (p_full);
        //   warp 10: O_j = P_j V_j into O[j % 2], once P_j is written
        //            (p_full) and O_{j-2} was folded (o_free).
        // They touch different TMEM columns and shared-memory tiles; each
        // frees its ring slots as its MMAs complete.
        constexpr uint32_t idesc_s = umma_idesc_bf16(BQ, BKV, 0, 0);
        constexpr uint32_t idesc_o = umma_idesc_bf16(BQ, HD, 0, 1);
        const uint32_t sQ = s_base;
        bool ok = true;
        auto wait_slot = [&](int n, uint32_t& addr, unsigned site) -> bool {
            const int slot = n % NSLOT;
            const uint32_t ph = static_cast<uint32_t>((n / NSLOT) & 1);
            if (*abort_flag || !mbar_wait(&full[slot], ph, site))
                return false;
            addr = s_base + CF::OFF_SLOT + slot * CF::SLOT_BYTES;
            return true;
        };
        if (warp == 1) {
            ok = mbar_wait(q_full, 0, 22);
            for (int j = 0; j < nblk && ok; ++j) {
                const int n = ring_pos_k(j);
                uint32_t sK;
                if (!wait_slot(n, sK, 23) ||
                    (j >= 2 && (*abort_flag ||
                                !mbar_wait(&p_full[j & 1], ((j - 2) >> 1) & 1, 24)))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + CF::S_COL + (j & 1) * BKV;
#pragma unroll
                for (int ks = 0; ks < HD / 16; ++ks) {
                    const uint64_t qh_ = kmajor_desc(sQ, BQ, ks);
                    const uint64_t ql_ = kmajor_desc(sQ + CF::Q_PLANE, BQ, ks);
                    const uint64_t kh_ = kmajor_desc(sK, BKV, ks);
                    const uint64_t kl_ = kmajor_desc(sK + CF::KV_PLANE, BKV, ks);
                    mma_bf16_w(d, ql_, kh_, idesc_s, ks > 0 ? 1u : 0u);
                    mma_bf16_w(d, qh_, kl_, idesc_s, 1u);
                    mma_bf16_w(d, qh_, kh_, idesc_s, 1u);
                }
                mma_commit_w(&s_full[j & 1]);
                mma_commit_w(&empty[n % NSLOT]);
            }
        } else {
            for (int i = 0; i < nblk && ok; ++i) {
                const int n = ring_pos_v(i, nblk);
                uint32_t sV;
                if (!wait_slot(n, sV, 25) ||
                    *abort_flag || !mbar_wait(&p_full[i & 1], (i >> 1) & 1, 26) ||
                    (i >= 2 && (*abort_flag ||
                                !mbar_wait(&o_free[i & 1], ((i - 2) >> 1) & 1, 27)))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t sP = s_base + CF::OFF_P + (i & 1) * CF::P_BYTES;
                const uint32_t d = tmem + CF::O_COL + (i & 1) * HD;
#pragma unroll
                for (int ks = 0; ks < BKV / 16; ++ks) {
                    const uint64_t ph_ = kmajor_desc(sP, BQ, ks);
                    const uint64_t pl_ = kmajor_desc(sP + CF::P_PLANE, BQ, ks);
                    const uint64_t vh_ = v_desc(sV, ks);
                    const uint64_t vl_ = v_desc(sV + CF::KV_PLANE, ks);
                    mma_bf16_w(d, pl_, vh_, idesc_o, ks > 0 ? 1u : 0u);
                    mma_bf16_w(d, ph_, vl_, idesc_o, 1u);
                    mma_bf16_w(d, ph_, vh_, idesc_o, 1u);
                }
                mma_commit_w(&o_full[i & 1]);
                mma_commit_w(&empty[n % NSLOT]);
            }
        }
        if (!ok)
            *abort_flag = 1;
        // Every MMA issued by both warps has retired once this fires (also on
        // abort).
        mma_commit_w(done);
        mbar_wait(done, 0, 28);
    } else {
        // ----------------------------------------------------------- softmax
        const int sw = warp - 2;
        const int quad = warp & 3;  // TMEM lanes 32*quad .. +31
        const int half = sw >> 2;   // columns [half*32, +32) of S, [half*HD/2, +HD/2) of O
        const int r = quad * 32 + lane;
        const int64_t q = q0 + r;
        const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
#pragma unroll
        for (int c = 0; c < OH; ++c)
            acc[c] = 0.0f;
        float m_prev = -INFINITY;  // max (log2 units) used for the previous block
        float m_cur = -INFINITY;   // max for the current block
        float l = 0.0f;            // partial row sum over this thread's columns
        bool ok = true;

        auto fold_o = [&](int i, float scale) -> bool {
            if (*abort_flag || !mbar_wait(&o_full[i & 1], (i >> 1) & 1, 28))
                return false;
            tc_fence_after();
            const uint32_t base = tmem + lane_off + CF::O_COL + (i & 1) * HD + half * OH;
            constexpr int W = OH < 32 ? OH : 32;  // columns per TMEM load
#pragma unroll
            for (int c = 0; c < OH; c += W) {
                float v[W];
                if constexpr (W == 32)
                    tmem_ld_32x32b_x32(base + c, v);
                else
                    tmem_ld_32x32b_x16(base + c, v);
                tmem_ld_wait();
                // acc = acc * scale + v, two lanes per packed FMA (same rounding)
#pragma unroll
                for (int e = 0; e < W; e += 2) {
                    const float2 r = __ffma2_rn(make_float2(acc[c + e], acc[c + e + 1]),
                                                make_float2(scale, scale),
                                                make_float2(v[e], v[e + 1]));
                    acc[c + e] = r.x, acc[c + e + 1] = r.y;
                }
            }
            tc_fence_before();
            mbar_arrive(&o_free[i & 1]);
            return true;
        };

        float m_hist = -INFINITY;  // max of block j-2 (scale of acc before folding O_{j-1})
        for (int j = 0; j < nblk; ++j) {
            if (*abort_flag || !mbar_wait(&s_full[j & 1], (j >> 1) & 1, 29)) {
                ok = false;
                break;
            }
            tc_fence_after();
            // This thread's 32 scores (keys k0 + half*32 + e) and the partner
            // half's 32 (needed only for the row max).
            float s[32], so[32];
            const uint32_t sb = tmem + lane_off + CF::S_COL + (j & 1) * BKV;
            tmem_ld_32x32b_x32(sb + half * 32, s);
            tmem_ld_32x32b_x32(sb + (half ^ 1) * 32, so);
            tmem_ld_wait();
            const int64_t k0 = static_cast<int64_t>(j) * BKV;
            if (k0 + BKV - 1 > q0 || k0 + BKV > T) {
                const int64_t km = k0 + half * 32, ko = k0 + (half ^ 1) * 32;
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    if (km + e > q || km + e >= T)
                        s[e] = -INFINITY;
                    if (ko + e > q || ko + e >= T)
                        so[e] = -INFINITY;
                }
            }
            // Both halves take the maximum of the same 64 values (exact; the
            // two 32-column maxima are combined in column order).
            const float ms = max32(s), mso = max32(so);
            const float mx = half == 0 ? fmaxf(ms, mso) : fmaxf(mso, ms);
            m_prev = m_cur;
            m_cur = fmaxf(m_cur, mx * LOG2E);
            const float mc = m_cur == -INFINITY ? 0.0f : m_cur;  // all masked so far
            const float alpha = exp2_approx(m_prev - mc);        // 0 when m_prev = -inf
            float rs = 0.0f;
            uint32_t hi[16], lo[16];
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
                const float2 t = __ffma2_rn(make_float2(s[e], s[e + 1]), make_float2(LOG2E, LOG2E),
                                            make_float2(-mc, -mc));
                const float p0 = exp2_approx(t.x);
                const float p1 = exp2_approx(t.y);
                rs += p0 + p1;
                split_pair_bf16(p0, p1, hi[e / 2], lo[e / 2]);
            }
            l = l * alpha + rs;
            // P_j -> buffer j % 2, row r, key chunk `half` (64 B per plane),
            // 16-byte pieces XOR-swizzled with (r / 2) % 4. Buffer j % 2 was
            // last read by O_{j-2}, whose completion fold_o(j - 2) observed.
            uint8_t* pb = smem + CF::OFF_P + (j & 1) * CF::P_BYTES + half * (BQ * 64) + r * 64;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int pc = (c ^ ((r >> 1) & 3)) * 16;
                *reinterpret_cast<uint4*>(pb + pc) =
                    make_uint4(hi[4 * c], hi[4 * c + 1], hi[4 * c + 2], hi[4 * c + 3]);
                *reinterpret_cast<uint4*>(pb + CF::P_PLANE + pc) =
                    make_uint4(lo[4 * c], lo[4 * c + 1], lo[4 * c + 2], lo[4 * c + 3]);
            }
            fence_proxy_async_smem();  // P stores -> visible to the tensor core
            tc_fence_before();         // S reads ordered before the S buffer's reuse
            mbar_arrive(&p_full[j & 1]);
            // fold O_{j-1} (computed with max m_prev) into acc (scaled to m_hist)
            if (j >= 1) {
                const float sc = m_prev == -INFINITY ? 0.0f : exp2_approx(m_hist - m_prev);
                if (!fold_o(j - 1, sc)) {
                    ok = false;
                    break;
                }
            }
            m_hist = m_prev;
        }
        if (ok) {
            const float sc = m_cur == -INFINITY ? 0.0f : exp2_approx(m_hist - m_cur);
            ok = fold_o(nblk - 1, sc);
        }
        if (!ok)
            *abort_flag = 1;
        // Row sums of the two halves meet after the closing barrier, which
        // every thread reaches.
        red[half * BQ + r] = l;
        l_own = l;
        m_out = m_cur;
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, CF::TMEM_COLS);
    }
    if (warp >= 2 && warp < 2 + 8 && !*abort_flag) {
        // Epilogue in two phases. (1) Each thread scales its half row of O
        // and puts it in a shared-memory tile [BQ][HD + 4] over the K/V ring
        // (free: every MMA that read it has completed). (2) The eight warps
        // store the tile row by row, HD / 4 lanes per row with one float4
        // each, so a warp's stores (and those of the bf16x3 planes) cover
        // whole contiguous rows instead of 32 rows 4 KB apart.
        constexpr int LD = HD + 4;  // row pitch in floats: conflict-free float4 stores
        static_assert(BQ * LD * 4 <= NSLOT * CF::SLOT_BYTES, "epilogue tile fits the ring");
        float* tile = reinterpret_cast<float*>(smem + CF::OFF_SLOT);
        const int quad = warp & 3, half = (warp - 2) >> 2;
        const int r = quad * 32 + lane;
        const int64_t q = q0 + r;
        const float lt = l_own + red[(half ^ 1) * BQ + r];
        const float inv = lt > 0.0f ? 1.0f / lt : 0.0f;
        float* trow = tile + r * LD + half * OH;
#pragma unroll
        for (int c = 0; c < OH; c += 4)
            *reinterpret_cast<float4*>(trow + c) =
                make_float4(acc[c] * inv, acc[c + 1] * inv, acc[c + 2] * inv, acc[c + 3] * inv);
        if (q < T && half == 0)
            lse[bh * T + q] = m_out * LN2 + logf(lt);
        asm volatile("bar.sync 1, %0;" ::"n"(SOFTMAX_THREADS) : "memory");
        constexpr int LPR = HD / 4;     // lanes per row
        constexpr int RPI = 32 / LPR;   // rows per warp instruction
        const int sw = warp - 2;
        const int c = (lane % LPR) * 4;
        const int64_t b = bh / H, h = bh % H;
        for (int rr = sw * RPI + lane / LPR; rr < BQ; rr += 8 * RPI) {
            const int64_t qq = q0 + rr;
            if (qq >= T)
                break;
            const float4 v = *reinterpret_cast<const float4*>(tile + rr * LD + c);
            const int64_t off = ((b * T + qq) * H + h) * HD + c;
            *reinterpret_cast<float4*>(o + off) = v;
            if (o_split) {  // the split kernel's arithmetic (split_bf16)
                const float ov[4] = {v.x, v.y, v.z, v.w};
                __nv_bfloat16 hi[4], lo[4];
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    split_bf16(ov[u], hi[u], lo[u]);
                *reinterpret_cast<uint2*>(o_split + off) = *reinterpret_cast<const uint2*>(hi);
                *reinterpret_cast<uint2*>(o_split + o_plane + off) =
                    *reinterpret_cast<const uint2*>(lo);
            }
        }
    }
}


// ------------------------------------------------------------ backward --
// Both backward kernels take the split planes of q (rotated, pre-scaled), k
// (rotated), v and dO, and write fp32 gradients in [B,T,H,HD] with the RoPE
// transpose rotation applied to dq and dk. Streamed blocks are 32 rows (keys
// for dQ, queries for dK/dV). Per block the tensor core computes the score
// block S (S^T) and dP (dP^T) into one of NBUF TMEM buffers; a softmax warp
// group reads them and writes the bf16 hi|lo split of dS (of P^T and dS^T)
// back over the same columns, where the accumulation MMAs take it as their A
// operand (row m in lane m, bf16 pairs packed per 32-bit column). Two softmax
// groups of four warps take alternate blocks (one thread per row, all 32
// columns), and the MMA warp issues the scores of block j before the
// accumulation of block j - LOOKAHEAD, so the tensor core never waits on the
// softmax of the block it just produced. dQ, dK and dV accumulate in TMEM
// over every block.
// Column ownership in the epilogues: with HH = HD/2 and QW = HD/4, the thread
// of group g holds columns [g*QW, g*QW + QW) and [HH + g*QW, HH + g*QW + QW),
// so each RoPE pair (d, d + HH) lives in one thread.

constexpr int BWD_BLK = 32;
constexpr int NBUF = 4;  // score buffers in TMEM (64 columns each)
constexpr int GROUP_THREADS = 128;
// Ring depths and lookahead (blocks between a score MMA and its accumulation
// MMA, below NBUF). A ring slot is held from its tile's first MMA to its last;
// each ring leaves about two blocks between a slot's release and its reuse,
// so the copy into it hides behind the tensor core's work.
//   dQ:     K held from S_j to dQ_j (lookahead 2) -> 4 slots; V freed after
//           dP_j -> 2 slots
//   dK, dV: Q_i and dO_i held from S^T_i to the accumulation (lookahead 1)
//           -> 3 slots each
constexpr int DKV_R1 = 3, DKV_R2 = 3, DKV_LOOKAHEAD = 1;
static_assert(DKV_R1 == DKV_R2, "the dK/dV kernel indexes both rings with one slot");
static_assert(DKV_LOOKAHEAD < NBUF, "a score buffer is reused after its accumulation MMA "
              "was issued");
constexpr int LD_BYTES = BWD_BLK * 8;  // (lse * log2 e, D) pairs of one query block

template <int HD, int R1, int R2>
struct BwdCfg {
    static constexpr int NCH = HD / 32;
    static constexpr int BIG_PLANE = NCH * BQ * 64;         // 128-row tile plane
    static constexpr int BIG_BYTES = 2 * BIG_PLANE;
    static constexpr int SMALL_PLANE = NCH * BWD_BLK * 64;  // 32-row tile plane
    static constexpr int SMALL_BYTES = 2 * SMALL_PLANE;
    static constexpr int OFF_BIG1 = BIG_BYTES;                  // second resident tile
    static constexpr int OFF_R1 = 2 * BIG_BYTES;                // ring 1 (K | Q)
    static constexpr int OFF_R2 = OFF_R1 + R1 * SMALL_BYTES;  // ring 2 (V | dO)
    static constexpr int OFF_LD = OFF_R2 + R2 * SMALL_BYTES;  // ring 1's (lse, D) blocks
    static constexpr int OFF_BAR = OFF_LD + R1 * LD_BYTES;
    static constexpr int NBARS = 32;
    static constexpr int BYTES = OFF_BAR + 8 * NBARS + 16 + 1024;
    static constexpr int ACC_COL = NBUF * 64;  // dQ (HD) | dV (HD), dK (HD)
    static constexpr int TMEM_COLS = 512;
    static_assert(ACC_COL + 2 * HD <= TMEM_COLS, "TMEM budget");
    static_assert(BYTES <= 232448, "shared memory budget");
};

// MN-major B operand from a 32-row tile [plane][NCH][32 rows][64 B]: k-step ks
// covers rows 16ks..16ks+15; the HD extent is NCH chunks 2 KB apart.
__device__ __forceinline__ uint64_t small_mn_desc(uint32_t plane, int ks) {
    return umma_smem_desc(plane + ks * 1024, BWD_BLK * 64, 512, kSW64);
}

// Load this thread's 2*QW accumulator columns (see column ownership above).
template <int HD>
__device__ __forceinline__ void load_owned(uint32_t taddr, int grp, float (&v)[HD / 2]) {
    constexpr int QW = HD / 4, HH = HD / 2;
    float a[QW], b[QW];
    if constexpr (QW == 32) {
        tmem_ld_32x32b_x32(taddr + grp * QW, a);
        tmem_ld_32x32b_x32(taddr + HH + grp * QW, b);
    } else if constexpr (QW == 16) {
        tmem_ld_32x32b_x16(taddr + grp * QW, a);
        tmem_ld_32x32b_x16(taddr + HH + grp * QW, b);
    } else {
        static_assert(QW == 8, "head dims 32, 64, 128");
        tmem_ld_32x32b_x8(taddr + grp * QW, a);
        tmem_ld_32x32b_x8(taddr + HH + grp * QW, b);
    }
    tmem_ld_wait();
#pragma unroll
    for (int e = 0; e < QW; ++e)
        v[e] = a[e], v[QW + e] = b[e];
}

// Epilogues stage a 128-row gradient tile in shared memory ([BQ][HD + 4]
// floats: the pitch makes each thread's float4 stores conflict-free) so that
// the global stores cover whole rows per warp.
template <int HD>
__host__ __device__ constexpr int tile_ld() {
    return HD + 4;
}

// Phase 1: this thread's owned columns of one gradient row, scaled, with the
// RoPE transpose rotation when `rope`, into its tile row.
template <int HD>
__device__ __forceinline__ void stage_owned(const float (&g)[HD / 2], float* __restrict__ trow,
                                            int64_t t, const float* __restrict__ cs,
                                            const float* __restrict__ sn, bool rope, float scale,
                                            int grp) {
    constexpr int QW = HD / 4, HH = HD / 2;
#pragma unroll
    for (int e = 0; e < QW; e += 4) {
        const int d = grp * QW + e;
        float a[4], b[4];
        float4 c4 = make_float4(1.f, 1.f, 1.f, 1.f), s4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (rope) {
            c4 = __ldg(reinterpret_cast<const float4*>(cs + t * HH + d));
            s4 = __ldg(reinterpret_cast<const float4*>(sn + t * HH + d));
        }
        const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float g1 = g[e + u] * scale, g2 = g[QW + e + u] * scale;
            a[u] = rope ? g1 * cc[u] + g2 * ss[u] : g1;
            b[u] = rope ? -g1 * ss[u] + g2 * cc[u] : g2;
        }
        *reinterpret_cast<float4*>(trow + d) = make_float4(a[0], a[1], a[2], a[3]);
        *reinterpret_cast<float4*>(trow + HH + d) = make_float4(b[0], b[1], b[2], b[3]);
    }
}

// Phase 2: the eight epilogue warps (sw = 0..7) store the tile's rows row0 +
// rr (rows at or past T skipped), HD / 4 lanes per row with one float4 each,
// into out [B,T,H,HD] for head bh: added to the stored values when
// `accumulate`, and split into bf16x3 planes at `split` (lo `plane` elements
// after hi) after the addition, with the split kernel's arithmetic
// (split_bf16).
template <int HD>
__device__ __forceinline__ void store_rows(const float* __restrict__ tile, float* __restrict__ out,
                                           __nv_bfloat16* __restrict__ split, int64_t plane,
                                           int64_t row0, int64_t T, int H, int64_t bh,
                                           int accumulate, int sw, int lane) {
    constexpr int LD = tile_ld<HD>();
    constexpr int LPR = HD / 4;    // lanes per row
    constexpr int RPI = 32 / LPR;  // rows per warp instruction
    const int c = (lane % LPR) * 4;
    const int64_t b = bh / H, h = bh % H;
    for (int rr = sw * RPI + lane / LPR; rr < BQ; rr += 8 * RPI) {
        const int64_t t = row0 + rr;
        if (t >= T)
            break;
        float4 v = *reinterpret_cast<const float4*>(tile + rr * LD + c);
        const int64_t off = ((b * T + t) * H + h) * HD + c;
        float4* p = reinterpret_cast<float4*>(out + off);
        if (accumulate) {
            const float4 o = *p;
            v.x += o.x, v.y += o.y, v.z += o.z, v.w += o.w;
        }
        *p = v;
        if (split) {
            const float vv[4] = {v.x, v.y, v.z, v.w};
            __nv_bfloat16 hi[4], lo[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                split_bf16(vv[u], hi[u], lo[u]);
            *reinterpret_cast<uint2*>(split + off) = *reinterpret_cast<const uint2*>(hi);
            *reinterpret_cast<uint2*>(split + plane + off) = *reinterpret_cast<const uint2*>(lo);
        }
    }
}

// Barrier 1 over the 256 softmax / epilogue threads, returning whether `ok`
// holds in all of them (every one of them reaches it: their waits are
// bounded), so that they take the epilogue or the abort path together.
__device__ __forceinline__ bool softmax_all(bool ok) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(ok)), "n"(SOFTMAX_THREADS)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void softmax_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(SOFTMAX_THREADS) : "memory");
}

// Packed bf16 hi|lo of 32 values: hi[i], lo[i] hold elements 2i, 2i+1.
__device__ __forceinline__ void split32(const float (&x)[32], uint32_t (&hi)[16],
                                        uint32_t (&lo)[16]) {
#pragma unroll
    for (int i = 0; i < 16; ++i)
        split_pair_bf16(x[2 * i], x[2 * i + 1], hi[i], lo[i]);
}

// dQ: CTA = 128 query rows of one (b, h); key blocks of 64 up to the diagonal.
//   S_j = Q K_j^T (buffer cols [0,64)), dP_j = dO V_j^T ([64,128)); N = 64
//   per MMA, twice the 32-row blocks of dK/dV, which halves the MMA
//   instructions per key (an instruction costs about the same time at N = 32
//   and N = 64). The two softmax warps of a lane quadrant each take 32 keys
//   (half h) of every block and write the split of dS_j over exactly the 32
//   S columns they read: keys 32h..32h+31 -> hi at [32h, 32h+16), lo at
//   [32h+16, 32h+32).
//   Issue order S_j, dQ_{j-1}, dP_j: the K slot of block j-1 frees one
//   product earlier, and V_j's copy hides behind S_j and dQ_{j-1}.
constexpr int DQ_BK = 64;

template <int HD>
struct DqCfg {
    static constexpr int NCH = HD / 32;
    static constexpr int BIG_PLANE = NCH * BQ * 64;      // Q, dO: [NCH][128][64 B]
    static constexpr int BIG_BYTES = 2 * BIG_PLANE;
    static constexpr int TILE_PLANE = NCH * DQ_BK * 64;  // K, V: [NCH][64][64 B]
    static constexpr int TILE_BYTES = 2 * TILE_PLANE;
    static constexpr int KR = HD == 128 ? 2 : 4;          // ring depths (shared-memory bound)
    static constexpr int VR = HD == 128 ? 1 : 3;
    static constexpr int OFF_DO = BIG_BYTES;
    static constexpr int OFF_K = 2 * BIG_BYTES;
    static constexpr int OFF_V = OFF_K + KR * TILE_BYTES;
    static constexpr int OFF_BAR = OFF_V + VR * TILE_BYTES;
    static constexpr int NBARS = 32;
    static constexpr int BYTES = OFF_BAR + 8 * NBARS + 16 + 1024;
    static constexpr int ACC_COL = 256;  // two 128-column block buffers, then dQ
    static constexpr int TMEM_COLS = 512;
    static_assert(ACC_COL + HD <= TMEM_COLS, "TMEM budget");
    static_assert(BYTES <= 232448, "shared memory budget");
    static_assert(1 + 2 * KR + 2 * VR + 2 + 2 + 1 <= NBARS, "barriers");
};

template <int HD>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    attn_bwd_dq_tc(const __grid_constant__ CUtensorMap map_q,
                   const __grid_constant__ CUtensorMap map_do,
                   const __grid_constant__ CUtensorMap map_k,
                   const __grid_constant__ CUtensorMap map_v, const float* __restrict__ lse,
                   const float* __restrict__ Dv, const float* __restrict__ cs,
                   const float* __restrict__ sn, float* __restrict__ dq, int accumulate,
                   float scale, int64_t T, int H, __nv_bfloat16* __restrict__ dq_split,
                   int64_t plane) {
    using CF = DqCfg<HD>;
    constexpr int HH = HD / 2, KR = CF::KR, VR = CF::VR;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + CF::OFF_BAR);
    uint64_t* a_full = bars;
    uint64_t* kfull = bars + 1;
    uint64_t* kempty = kfull + KR;
    uint64_t* vfull = kempty + KR;
    uint64_t* vempty = vfull + VR;
    uint64_t* sd_full = vempty + VR;  // [2]
    uint64_t* ds_full = sd_full + 2;  // [2]
    uint64_t* done = ds_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + CF::NBARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nqt = static_cast<int>((T + BQ - 1) / BQ);
    const int qt = nqt - 1 - static_cast<int>(blockIdx.x);
    const int64_t q0 = static_cast<int64_t>(qt) * BQ;
    const int64_t bh = blockIdx.y;
    const int64_t q_last = min(q0 + BQ, T) - 1;
    const int nblk = static_cast<int>(q_last / DQ_BK) + 1;

    if (threadIdx.x == 0) {
        mbar_init(a_full, 1);
        for (int i = 0; i < KR; ++i) {
            mbar_init(&kfull[i], 1);
            mbar_init(&kempty[i], 1);
        }
        for (int i = 0; i < VR; ++i) {
            mbar_init(&vfull[i], 1);
            mbar_init(&vempty[i], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&sd_full[b], 1);
            mbar_init(&ds_full[b], SOFTMAX_THREADS);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&map_q);
        tma_prefetch_desc(&map_do);
        tma_prefetch_desc(&map_k);
        tma_prefetch_desc(&map_v);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, CF::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t s_base = smem_u32(smem);

    if (warp == 0) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0) {
            int karmed[KR], varmed[VR];
#pragma unroll
            for (int i = 0; i < KR; ++i)
                karmed[i] = -1;
#pragma unroll
            for (int i = 0; i < VR; ++i)
                varmed[i] = -1;
            mbar_arrive_expect_tx(a_full, 2 * CF::BIG_BYTES);
            tma_load_5d(smem, &map_q, a_full, 0, static_cast<int>(q0), 0, static_cast<int>(bh), 0);
            tma_load_5d(smem + CF::OFF_DO, &map_do, a_full, 0, static_cast<int>(q0), 0,
                        static_cast<int>(bh), 0);
            bool ok = true;
            for (int j = 0; j < nblk && ok; ++j) {
                const int ks_ = j % KR, vs_ = j % VR;
                const uint32_t kph = static_cast<uint32_t>((j / KR) & 1);
                const uint32_t vph = static_cast<uint32_t>((j / VR) & 1);
                if (*abort_flag || !mbar_wait(&kempty[ks_], kph ^ 1, 41)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&kfull[ks_], CF::TILE_BYTES);
                tma_load_5d(smem + CF::OFF_K + ks_ * CF::TILE_BYTES, &map_k, &kfull[ks_], 0,
                            j * DQ_BK, 0, static_cast<int>(bh), 0);
                karmed[ks_] = static_cast<int>(kph);
                if (*abort_flag || !mbar_wait(&vempty[vs_], vph ^ 1, 42)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&vfull[vs_], CF::TILE_BYTES);
                tma_load_5d(smem + CF::OFF_V + vs_ * CF::TILE_BYTES, &map_v, &vfull[vs_], 0,
                            j * DQ_BK, 0, static_cast<int>(bh), 0);
                varmed[vs_] = static_cast<int>(vph);
            }
            if (!ok) {
                *abort_flag = 1;
                mbar_wait(a_full, 0, 46);
#pragma unroll
                for (int i = 0; i < KR; ++i)
                    if (karmed[i] >= 0)
                        mbar_wait(&kfull[i], static_cast<uint32_t>(karmed[i]), 46);
#pragma unroll
                for (int i = 0; i < VR; ++i)
                    if (varmed[i] >= 0)
                        mbar_wait(&vfull[i], static_cast<uint32_t>(varmed[i]), 46);
            }
        }
    } else if (warp == 1) {
        // -------------------------------------------------------- MMA issuer
        // The whole warp runs this loop (uniform control flow); lane 0 issues.
        constexpr uint32_t idesc_sd = umma_idesc_bf16(BQ, DQ_BK, 0, 0);
        constexpr uint32_t idesc_q = umma_idesc_bf16(BQ, HD, 0, 1);
        const uint64_t qh0 = kmajor_desc(s_base, BQ, 0);
        const uint64_t ql0 = kmajor_desc(s_base + CF::BIG_PLANE, BQ, 0);
        const uint64_t oh0 = kmajor_desc(s_base + CF::OFF_DO, BQ, 0);
        const uint64_t ol0 = kmajor_desc(s_base + CF::OFF_DO + CF::BIG_PLANE, BQ, 0);
        const uint32_t dQ = tmem + CF::ACC_COL;
        bool ok = mbar_wait(a_full, 0, 43);
        auto issue_dq = [&](int i) -> bool {
            const int b = i & 1;
            if (*abort_flag || !mbar_wait(&ds_full[b], (i >> 1) & 1, 45))
                return false;
            tc_fence_after();
            const uint32_t sK = s_base + CF::OFF_K + (i % KR) * CF::TILE_BYTES;
            // MN-major K_i [64 keys][HD]: k-step of 16 keys = 16 rows of 64 B
            const uint64_t kh = umma_smem_desc(sK, DQ_BK * 64, 512, kSW64);
            const uint64_t kl = umma_smem_desc(sK + CF::TILE_PLANE, DQ_BK * 64, 512, kSW64);
            const uint32_t a = tmem + b * 128;
#pragma unroll
            for (int ks = 0; ks < DQ_BK / 16; ++ks) {
                const uint32_t ah = a + (ks >> 1) * 32 + (ks & 1) * 8, al = ah + 16;
                const uint64_t bh_ = desc_add(kh, ks * 1024), bl_ = desc_add(kl, ks * 1024);
                mma_bf16_ta_w(dQ, al, bh_, idesc_q, (i == 0 && ks == 0) ? 0u : 1u);
                mma_bf16_ta_w(dQ, ah, bl_, idesc_q, 1u);
                mma_bf16_ta_w(dQ, ah, bh_, idesc_q, 1u);
            }
            mma_commit_w(&kempty[i % KR]);
            return true;
        };
        for (int j = 0; j < nblk && ok; ++j) {
            const int ks_ = j % KR, vs_ = j % VR;
            if (*abort_flag || !mbar_wait(&kfull[ks_], (j / KR) & 1, 47)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t sK = s_base + CF::OFF_K + ks_ * CF::TILE_BYTES;
            const uint64_t kh0 = kmajor_desc(sK, DQ_BK, 0);
            const uint64_t kl0 = kmajor_desc(sK + CF::TILE_PLANE, DQ_BK, 0);
            const uint32_t ds = tmem + (j & 1) * 128, dp = ds + 64;
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks) {
                const uint32_t ob = (ks >> 1) * (BQ * 64) + (ks & 1) * 32;
                const uint32_t sb = (ks >> 1) * (DQ_BK * 64) + (ks & 1) * 32;
                mma_bf16_w(ds, desc_add(ql0, ob), desc_add(kh0, sb), idesc_sd, ks > 0 ? 1u : 0u);
                mma_bf16_w(ds, desc_add(qh0, ob), desc_add(kl0, sb), idesc_sd, 1u);
                mma_bf16_w(ds, desc_add(qh0, ob), desc_add(kh0, sb), idesc_sd, 1u);
            }
            if (j >= 1 && !issue_dq(j - 1)) {
                ok = false;
                break;
            }
            if (*abort_flag || !mbar_wait(&vfull[vs_], (j / VR) & 1, 48)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t sV = s_base + CF::OFF_V + vs_ * CF::TILE_BYTES;
            const uint64_t vh0 = kmajor_desc(sV, DQ_BK, 0);
            const uint64_t vl0 = kmajor_desc(sV + CF::TILE_PLANE, DQ_BK, 0);
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks) {
                const uint32_t ob = (ks >> 1) * (BQ * 64) + (ks & 1) * 32;
                const uint32_t sb = (ks >> 1) * (DQ_BK * 64) + (ks & 1) * 32;
                mma_bf16_w(dp, desc_add(ol0, ob), desc_add(vh0, sb), idesc_sd, ks > 0 ? 1u : 0u);
                mma_bf16_w(dp, desc_add(oh0, ob), desc_add(vl0, sb), idesc_sd, 1u);
                mma_bf16_w(dp, desc_add(oh0, ob), desc_add(vh0, sb), idesc_sd, 1u);
            }
            mma_commit_w(&sd_full[j & 1]);
            mma_commit_w(&vempty[vs_]);
        }
        if (ok && !issue_dq(nblk - 1))
            ok = false;
        if (!ok)
            *abort_flag = 1;
        // fires once every MMA issued has retired (also on abort)
        mma_commit_w(done);
        mbar_wait(done, 0, 49);
    } else {
        // --------------------------------------------------- softmax / dS
        // Every block goes through all eight warps: the two warps of a TMEM
        // lane quadrant take keys [32h, 32h+32) of their rows (h = half).
        const int grp = (warp - 2) >> 2;  // column half; also the dQ column owner
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        const int64_t q = q0 + r;
        const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
        const float lse2 = q < T ? lse[bh * T + q] * LOG2E : 0.0f;
        const float Dq = q < T ? Dv[bh * T + q] : 0.0f;
        bool ok = true;
        for (int j = 0; j < nblk; ++j) {
            const int b = j & 1;
            if (*abort_flag || !mbar_wait(&sd_full[b], (j >> 1) & 1, 51)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t buf = tmem + lane_off + b * 128 + grp * 32;
            const int64_t k0 = static_cast<int64_t>(j) * DQ_BK + grp * 32;
            const bool diag = k0 + 31 > q0;
            float sv[32], dpv[32];
            tmem_ld_32x32b_x32(buf, sv);
            tmem_ld_32x32b_x32(buf + 64, dpv);
            tmem_ld_wait();
            // p = exp2(s log2e - lse), dS = p (dP - D); two lanes per packed
            // instruction (the same roundings as the scalar forms)
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
                const float2 t = __ffma2_rn(make_float2(sv[e], sv[e + 1]),
                                            make_float2(LOG2E, LOG2E), make_float2(-lse2, -lse2));
                const bool l0 = q < T && (!diag || k0 + e <= q);
                const bool l1 = q < T && (!diag || k0 + e + 1 <= q);
                const float2 pp = make_float2(l0 ? exp2_approx(t.x) : 0.0f,
                                              l1 ? exp2_approx(t.y) : 0.0f);
                const float2 d = __fadd2_rn(make_float2(dpv[e], dpv[e + 1]), make_float2(-Dq, -Dq));
                const float2 r = __fmul2_rn(pp, d);
                sv[e] = r.x, sv[e + 1] = r.y;
            }
            uint32_t hi[16], lo[16];
            split32(sv, hi, lo);
            tmem_st_32x32b_x16(buf, hi);
            tmem_st_32x32b_x16(buf + 16, lo);
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(&ds_full[b]);
        }
        if (ok && (*abort_flag || !mbar_wait(done, 0, 52)))
            ok = false;
        if (!softmax_all(ok)) {
            *abort_flag = 1;
        } else {
            // dQ tile staged over the Q / dO tiles (every MMA has completed),
            // then stored row by row.
            static_assert(BQ * tile_ld<HD>() * 4 <= 2 * CF::BIG_BYTES, "dQ tile fits");
            float* tile = reinterpret_cast<float*>(smem);
            tc_fence_after();
            float g[HH];
            load_owned<HD>(tmem + lane_off + CF::ACC_COL, grp, g);
            if (q < T)
                stage_owned<HD>(g, tile + r * tile_ld<HD>(), q, cs, sn, true, scale, grp);
            softmax_sync();
            store_rows<HD>(tile, dq, dq_split, plane, q0, T, H, bh, accumulate, warp - 2, lane);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, CF::TMEM_COLS);
    }
}

// dK, dV: CTA = 128 keys of one (b, h); query blocks of 32 from the diagonal.
//   S^T_i = K Q_i^T (buffer cols [0,32)), dP^T_i = V dO_i^T ([32,64)); the
//   softmax group writes P^T over S^T (hi [0,16), lo [16,32)) and dS^T =
//   P^T (dP^T - D) over dP^T ([32,48), [48,64)); dV += P^T dO_i, dK += dS^T Q_i.
//   lse (pre-multiplied by log2 e) and D of each query block arrive with Q_i
//   by a bulk copy from the padded (lse, D) table `ld` [B*H][T32][2].
template <int HD>
__global__ void __launch_bounds__(DKV_THREADS, 1)
    attn_bwd_dkv_tc(const __grid_constant__ CUtensorMap map_k,
                    const __grid_constant__ CUtensorMap map_v,
                    const __grid_constant__ CUtensorMap map_q,
                    const __grid_constant__ CUtensorMap map_do, const float* __restrict__ ld,
                    int64_t T32, const float* __restrict__ cs, const float* __restrict__ sn,
                    float* __restrict__ dk, float* __restrict__ dv, int accumulate, int64_t T,
                    int H, __nv_bfloat16* __restrict__ dk_split,
                    __nv_bfloat16* __restrict__ dv_split, int64_t plane) {
    using CF = BwdCfg<HD, DKV_R1, DKV_R2>;
    constexpr int HH = HD / 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + CF::OFF_BAR);
    uint64_t* a_full = bars;
    uint64_t* qfull = bars + 1;
    uint64_t* qempty = qfull + DKV_R1;
    uint64_t* ofull = qempty + DKV_R1;
    uint64_t* oempty = ofull + DKV_R1;
    uint64_t* sd_full = oempty + DKV_R1;    // [NBUF]
    uint64_t* pds_full = sd_full + NBUF;  // [NBUF]
    uint64_t* done = pds_full + NBUF;
    uint64_t* bfree = done + 1;  // [NBUF]: a score buffer's accumulation MMAs done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + CF::NBARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t k0 = static_cast<int64_t>(blockIdx.x) * BQ;  // most query blocks first
    const int64_t bh = blockIdx.y;
    const int i_first = static_cast<int>(k0 / BWD_BLK);
    const int nblk = static_cast<int>((T + BWD_BLK - 1) / BWD_BLK) - i_first;

    if (threadIdx.x == 0) {
        mbar_init(a_full, 1);
        for (int i = 0; i < DKV_R1; ++i) {
            mbar_init(&qfull[i], 1);
            mbar_init(&qempty[i], 1);
            mbar_init(&ofull[i], 1);
            mbar_init(&oempty[i], 1);
        }
        // Two MMA-issuing warps: commits from both complete sd_full, bfree and done.
        for (int b = 0; b < NBUF; ++b) {
            mbar_init(&sd_full[b], 2);
            mbar_init(&pds_full[b], GROUP_THREADS);
            mbar_init(&bfree[b], 2);
        }
        mbar_init(done, 2);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&map_k);
        tma_prefetch_desc(&map_v);
        tma_prefetch_desc(&map_q);
        tma_prefetch_desc(&map_do);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, CF::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t s_base = smem_u32(smem);

    if (warp == 0) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0) {
            int qarmed[DKV_R1], oarmed[DKV_R1];
#pragma unroll
            for (int i = 0; i < DKV_R1; ++i)
                qarmed[i] = oarmed[i] = -1;
            mbar_arrive_expect_tx(a_full, 2 * CF::BIG_BYTES);
            tma_load_5d(smem, &map_k, a_full, 0, static_cast<int>(k0), 0, static_cast<int>(bh), 0);
            tma_load_5d(smem + CF::OFF_BIG1, &map_v, a_full, 0, static_cast<int>(k0), 0,
                        static_cast<int>(bh), 0);
            bool ok = true;
            for (int n = 0; n < nblk && ok; ++n) {
                const int slot = n % DKV_R1;
                const uint32_t ph = static_cast<uint32_t>((n / DKV_R1) & 1);
                const int row = (i_first + n) * BWD_BLK;
                if (*abort_flag || !mbar_wait(&qempty[slot], ph ^ 1, 61)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&qfull[slot], CF::SMALL_BYTES + LD_BYTES);
                tma_load_5d(smem + CF::OFF_R1 + slot * CF::SMALL_BYTES, &map_q, &qfull[slot], 0,
                            row, 0, static_cast<int>(bh), 0);
                bulk_load(smem + CF::OFF_LD + slot * LD_BYTES, ld + (bh * T32 + row) * 2,
                          LD_BYTES, &qfull[slot]);
                qarmed[slot] = static_cast<int>(ph);
                if (*abort_flag || !mbar_wait(&oempty[slot], ph ^ 1, 62)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&ofull[slot], CF::SMALL_BYTES);
                tma_load_5d(smem + CF::OFF_R2 + slot * CF::SMALL_BYTES, &map_do, &ofull[slot], 0,
                            row, 0, static_cast<int>(bh), 0);
                oarmed[slot] = static_cast<int>(ph);
            }
            if (!ok) {
                *abort_flag = 1;
                mbar_wait(a_full, 0, 66);
#pragma unroll
                for (int i = 0; i < DKV_R1; ++i) {
                    if (qarmed[i] >= 0)
                        mbar_wait(&qfull[i], static_cast<uint32_t>(qarmed[i]), 66);
                    if (oarmed[i] >= 0)
                        mbar_wait(&ofull[i], static_cast<uint32_t>(oarmed[i]), 66);
                }
            }
        }
    } else if (warp == 1 || warp == DKV_MMA_B_WARP) {
        // -------------------------------------------------------- MMA issuers
        // One warp issues at most about one MMA per 64 cycles, so two warps
        // share the work (each loop warp-uniform; lane 0 issues):
        //   warp A (1):  S^T = K Q^T  and  dK += dS^T Q   (the Q slot)
        //   warp B (10): dP^T = V dO^T  and  dV += P^T dO  (the dO slot)
        // Their MMAs are not ordered against each other, so a score buffer is
        // rewritten only after both warps' accumulation MMAs on its previous
        // block completed (bfree).
        const bool wa = warp == 1;
        constexpr uint32_t idesc_sd = umma_idesc_bf16(BQ, BWD_BLK, 0, 0);
        constexpr uint32_t idesc_acc = umma_idesc_bf16(BQ, HD, 0, 1);
        const uint32_t big = wa ? 0u : static_cast<uint32_t>(CF::OFF_BIG1);  // K | V
        const uint64_t xh0 = kmajor_desc(s_base + big, BQ, 0);
        const uint64_t xl0 = kmajor_desc(s_base + big + CF::BIG_PLANE, BQ, 0);
        const uint32_t ring = wa ? static_cast<uint32_t>(CF::OFF_R1) : static_cast<uint32_t>(CF::OFF_R2);
        uint64_t* rfull = wa ? qfull : ofull;
        uint64_t* rempty = wa ? qempty : oempty;
        const uint32_t acc_d = tmem + CF::ACC_COL + (wa ? HD : 0);  // dK | dV
        const uint32_t half = wa ? 32u : 0u;  // A operand of the accumulation: dS^T | P^T
        bool ok = mbar_wait(a_full, 0, 63);
        auto issue_acc = [&](int i) -> bool {
            const int b = i % NBUF;
            if (*abort_flag || !mbar_wait(&pds_full[b], (i / NBUF) & 1, 64))
                return false;
            tc_fence_after();
            const int slot = i % DKV_R1;
            const uint32_t sR = s_base + ring + slot * CF::SMALL_BYTES;
            const uint64_t rh = small_mn_desc(sR, 0), rl = small_mn_desc(sR + CF::SMALL_PLANE, 0);
            const uint32_t x = tmem + b * 64 + half;
#pragma unroll
            for (int ks = 0; ks < BWD_BLK / 16; ++ks) {
                const uint32_t first = (i == 0 && ks == 0) ? 0u : 1u;
                const uint32_t o = ks * 1024;
                mma_bf16_ta_w(acc_d, x + 16 + ks * 8, desc_add(rh, o), idesc_acc, first);
                mma_bf16_ta_w(acc_d, x + ks * 8, desc_add(rl, o), idesc_acc, 1u);
                mma_bf16_ta_w(acc_d, x + ks * 8, desc_add(rh, o), idesc_acc, 1u);
            }
            mma_commit_w(&rempty[slot]);
            mma_commit_w(&bfree[b]);
            return true;
        };
        for (int n = 0; n < nblk && ok; ++n) {
            const int slot = n % DKV_R1;
            const uint32_t ph = static_cast<uint32_t>((n / DKV_R1) & 1);
            const int b = n % NBUF;
            if (*abort_flag || !mbar_wait(&rfull[slot], ph, wa ? 67 : 68) ||
                (n >= NBUF && !mbar_wait(&bfree[b], static_cast<uint32_t>((n / NBUF - 1) & 1), 65))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t sR = s_base + ring + slot * CF::SMALL_BYTES;
            const uint64_t rh0 = kmajor_desc(sR, BWD_BLK, 0);
            const uint64_t rl0 = kmajor_desc(sR + CF::SMALL_PLANE, BWD_BLK, 0);
            const uint32_t dst = tmem + b * 64 + (wa ? 0u : 32u);  // S^T | dP^T
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks) {
                const uint32_t bb = (ks >> 1) * (BQ * 64) + (ks & 1) * 32;
                const uint32_t sb = (ks >> 1) * (BWD_BLK * 64) + (ks & 1) * 32;
                const uint32_t acc = ks > 0 ? 1u : 0u;
                mma_bf16_w(dst, desc_add(xl0, bb), desc_add(rh0, sb), idesc_sd, acc);
                mma_bf16_w(dst, desc_add(xh0, bb), desc_add(rl0, sb), idesc_sd, 1u);
                mma_bf16_w(dst, desc_add(xh0, bb), desc_add(rh0, sb), idesc_sd, 1u);
            }
            mma_commit_w(&sd_full[b]);
            if (n >= DKV_LOOKAHEAD && !issue_acc(n - DKV_LOOKAHEAD))
                ok = false;
        }
        for (int i = max(0, nblk - DKV_LOOKAHEAD); i < nblk && ok; ++i)
            if (!issue_acc(i))
                ok = false;
        if (!ok)
            *abort_flag = 1;
        mma_commit_w(done);
        mbar_wait(done, 0, 69);
    } else if (warp >= 2 && warp < 2 + 8) {
        // ------------------------------------------------ P^T, dS^T, epilogue
        const int grp = (warp - 2) >> 2;  // query blocks n with n % 2 == grp
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        const int64_t key = k0 + r;
        const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
        bool ok = true;
        for (int n = grp; n < nblk; n += 2) {
            const int b = n % NBUF;
            if (*abort_flag || !mbar_wait(&sd_full[b], (n / NBUF) & 1, 70)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float sv[32], dpv[32];
            tmem_ld_32x32b_x32(tmem + lane_off + b * 64, sv);
            tmem_ld_32x32b_x32(tmem + lane_off + b * 64 + 32, dpv);
            tmem_ld_wait();
            // (lse * log2 e, D) of this query block landed with Q_i: observe
            // that copy's completion here too (already complete; the slot is
            // refilled only after this block's pds_full).
            if (*abort_flag || !mbar_wait(&qfull[n % DKV_R1], (n / DKV_R1) & 1, 73)) {
                ok = false;
                break;
            }
            const float2* ldv =
                reinterpret_cast<const float2*>(smem + CF::OFF_LD + (n % DKV_R1) * LD_BYTES);
            const int64_t qb = static_cast<int64_t>(i_first + n) * BWD_BLK;
            const bool diag = qb < k0 + BQ - 1 || qb + BWD_BLK > T;
            float pv[32];
            // P^T = exp2(s log2e - lse), dS^T = P^T (dP^T - D); two lanes per
            // packed instruction (the same roundings as the scalar forms)
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
                const float2 l0 = ldv[e], l1 = ldv[e + 1];
                const float2 t = __ffma2_rn(make_float2(sv[e], sv[e + 1]),
                                            make_float2(LOG2E, LOG2E), make_float2(-l0.x, -l1.x));
                const bool a0 = !diag || (key <= qb + e && qb + e < T);
                const bool a1 = !diag || (key <= qb + e + 1 && qb + e + 1 < T);
                const float2 pp = make_float2(a0 ? exp2_approx(t.x) : 0.0f,
                                              a1 ? exp2_approx(t.y) : 0.0f);
                const float2 d = __fadd2_rn(make_float2(dpv[e], dpv[e + 1]),
                                            make_float2(-l0.y, -l1.y));
                const float2 r = __fmul2_rn(pp, d);
                pv[e] = pp.x, pv[e + 1] = pp.y;
                sv[e] = r.x, sv[e + 1] = r.y;
            }
            uint32_t phi[16], plo[16], shi[16], slo[16];
            split32(pv, phi, plo);
            split32(sv, shi, slo);
            tmem_st_32x32b_x16(tmem + lane_off + b * 64, phi);
            tmem_st_32x32b_x16(tmem + lane_off + b * 64 + 16, plo);
            tmem_st_32x32b_x16(tmem + lane_off + b * 64 + 32, shi);
            tmem_st_32x32b_x16(tmem + lane_off + b * 64 + 48, slo);
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(&pds_full[b]);
        }
        if (ok && (*abort_flag || !mbar_wait(done, 0, 72)))
            ok = false;
        if (!softmax_all(ok)) {
            *abort_flag = 1;
        } else {
            // dV and dK tiles staged over the K / V tiles and the first ring
            // (every MMA and copy has completed), then stored row by row.
            constexpr int TILE = BQ * tile_ld<HD>();
            static_assert(2 * TILE * 4 <= CF::OFF_BAR, "dK/dV tiles fit");
            float* tile_v = reinterpret_cast<float*>(smem);
            float* tile_k = tile_v + TILE;
            tc_fence_after();
            float g[HH];
            load_owned<HD>(tmem + lane_off + CF::ACC_COL, grp, g);
            if (key < T)
                stage_owned<HD>(g, tile_v + r * tile_ld<HD>(), key, cs, sn, false, 1.0f, grp);
            load_owned<HD>(tmem + lane_off + CF::ACC_COL + HD, grp, g);
            if (key < T)
                stage_owned<HD>(g, tile_k + r * tile_ld<HD>(), key, cs, sn, true, 1.0f, grp);
            softmax_sync();
            store_rows<HD>(tile_v, dv, dv_split, plane, k0, T, H, bh, accumulate, warp - 2, lane);
            store_rows<HD>(tile_k, dk, dk_split, plane, k0, T, H, bh, accumulate, warp - 2, lane);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, CF::TMEM_COLS);
    }
}

}  // namespace fatc

// Tensor map over a pair of split planes (hi at `hi`, lo n elements later),
// each [BH][T][HD] bf16, as 5-D {32, T, HD/32, BH, 2} with a box of
// {32, rows, HD/32, 1, 2}: one copy brings both planes of a rows x HD tile.
static int make_plane_map(CUtensorMap* map, const __nv_bfloat16* hi, int64_t n, int64_t BH,
                          int64_t T, int hd, int rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc)
        return set_error(TTK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[5] = {32, static_cast<cuuint64_t>(T), static_cast<cuuint64_t>(hd / 32),
                          static_cast<cuuint64_t>(BH), 2};
    cuuint64_t strides[4] = {static_cast<cuuint64_t>(hd) * 2, 64,
                             static_cast<cuuint64_t>(T) * hd * 2, static_cast<cuuint64_t>(n) * 2};
    cuuint32_t box[5] = {32, static_cast<cuuint32_t>(rows), static_cast<cuuint32_t>(hd / 32), 1, 2};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<__nv_bfloat16*>(hi),
                     dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(TTK_ERR_CUDA, "cuTensorMapEncodeTiled failed (attention planes)");
    return TTK_OK;
}

bool attention_tc_supported(int hd) { return hd == 32 || hd == 64 || hd == 128; }

int attention_tc_forward_core(int hd, const __nv_bfloat16* qh, const __nv_bfloat16* kh,
                              const __nv_bfloat16* vh, float* o, float* lse, int64_t B, int64_t T,
                              int64_t H, cudaStream_t st, __nv_bfloat16* o_split) {
    const int64_t n = B * T * H * hd;
    CUtensorMap mq, mk, mv;
    int rc = make_plane_map(&mq, qh, n, B * H, T, hd, fatc::BQ);
    if (!rc)
        rc = make_plane_map(&mk, kh, n, B * H, T, hd, fatc::BKV);
    if (!rc)
        rc = make_plane_map(&mv, vh, n, B * H, T, hd, fatc::BKV);
    if (rc)
        return rc;
    dim3 grid(static_cast<unsigned>((T + fatc::BQ - 1) / fatc::BQ), static_cast<unsigned>(B * H));
    auto launch = [&](auto hd_tag) {
        constexpr int HD = decltype(hd_tag)::value;
        const int smem = fatc::FwdCfg<HD>::BYTES;
        cudaFuncSetAttribute(fatc::attn_fwd_tc<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem);
        fatc::attn_fwd_tc<HD><<<grid, fatc::FWD_THREADS, smem, st>>>(
            mq, mk, mv, o, lse, T, static_cast<int>(H), o_split, n);
    };
    if (hd == 128)
        launch(std::integral_constant<int, 128>{});
    else if (hd == 64)
        launch(std::integral_constant<int, 64>{});
    else
        launch(std::integral_constant<int, 32>{});
    return check_launch("attn_fwd_tc");
}

int attention_tc_backward_core(int hd, const __nv_bfloat16* qh, const __nv_bfloat16* kh,
                               const __nv_bfloat16* vh, const __nv_bfloat16* dh,
                               const float* lse, const float* Dv, const float* ld, int64_t T32,
                               const float* cs, const float* sn, float* dq, float* dk, float* dv,
                               int accumulate, int64_t B, int64_t T, int64_t H, float scale,
                               cudaStream_t st, __nv_bfloat16* dq_split,
                               __nv_bfloat16* dk_split, __nv_bfloat16* dv_split) {
    const int64_t n = B * T * H * hd;
    const int64_t BH = B * H;
    CUtensorMap q128, d128, k64, v64, k128, v128, q32, d32;
    int rc = make_plane_map(&q128, qh, n, BH, T, hd, fatc::BQ);
    if (!rc) rc = make_plane_map(&d128, dh, n, BH, T, hd, fatc::BQ);
    if (!rc) rc = make_plane_map(&k64, kh, n, BH, T, hd, fatc::DQ_BK);
    if (!rc) rc = make_plane_map(&v64, vh, n, BH, T, hd, fatc::DQ_BK);
    if (!rc) rc = make_plane_map(&k128, kh, n, BH, T, hd, fatc::BQ);
    if (!rc) rc = make_plane_map(&v128, vh, n, BH, T, hd, fatc::BQ);
    if (!rc) rc = make_plane_map(&q32, qh, n, BH, T, hd, fatc::BWD_BLK);
    if (!rc) rc = make_plane_map(&d32, dh, n, BH, T, hd, fatc::BWD_BLK);
    if (rc)
        return rc;
    dim3 grid(static_cast<unsigned>((T + fatc::BQ - 1) / fatc::BQ), static_cast<unsigned>(BH));
    auto launch = [&](auto hd_tag) -> int {
        constexpr int HD = decltype(hd_tag)::value;
        int smem = fatc::BwdCfg<HD, fatc::DKV_R1, fatc::DKV_R2>::BYTES;
        cudaFuncSetAttribute(fatc::attn_bwd_dkv_tc<HD>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        fatc::attn_bwd_dkv_tc<HD><<<grid, fatc::DKV_THREADS, smem, st>>>(
            k128, v128, q32, d32, ld, T32, cs, sn, dk, dv, accumulate, T, static_cast<int>(H),
            dk_split, dv_split, n);
        int r = check_launch("attn_bwd_dkv_tc");
        if (r)
            return r;
        smem = fatc::DqCfg<HD>::BYTES;
        cudaFuncSetAttribute(fatc::attn_bwd_dq_tc<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem);
        fatc::attn_bwd_dq_tc<HD><<<grid, fatc::NUM_THREADS, smem, st>>>(
            q128, d128, k64, v64, lse, Dv, cs, sn, dq, accumulate, scale, T, static_cast<int>(H),
            dq_split, n);
        return check_launch("attn_bwd_dq_tc");
    };
    if (hd == 128)
        return launch(std::integral_constant<int, 128>{});
    if (hd == 64)
        return launch(std::integral_constant<int, 64>{});
    return launch(std::integral_constant<int, 32>{});
}

}  // namespace ttk
