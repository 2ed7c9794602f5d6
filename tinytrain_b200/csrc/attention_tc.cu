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
// No load uses .multicast::cluster.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ttk_common.cuh"
#include "ttk_internal.h"

namespace ttk {
namespace fatc {

constexpr int BQ = 128;  // query rows per CTA (MMA M, TMEM lanes)
constexpr int BKV = 64;  // keys per block
constexpr int NSLOT = 3;
constexpr int NUM_THREADS = 320;
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

template <int HD>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    attn_fwd_tc(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                const __grid_constant__ CUtensorMap map_v, float* __restrict__ o,
                float* __restrict__ lse, int64_t T, int H) {
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
        mbar_init(done, 1);
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
    } else if (warp == 1) {
        // -------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc_s = umma_idesc_bf16(BQ, BKV, 0, 0);
            constexpr uint32_t idesc_o = umma_idesc_bf16(BQ, HD, 0, 1);
            const uint32_t sQ = s_base;
            int it = 0;
            bool ok = mbar_wait(q_full, 0, 22);
            auto next_slot = [&](uint32_t& addr) -> bool {
                const int slot = it % NSLOT;
                const uint32_t ph = static_cast<uint32_t>((it / NSLOT) & 1);
                if (*abort_flag || !mbar_wait(&full[slot], ph, 23))
                    return false;
                addr = s_base + CF::OFF_SLOT + slot * CF::SLOT_BYTES;
                ++it;
                return true;
            };
            auto issue_pv = [&](int i) -> bool {
                uint32_t sV;
                const int slot = it % NSLOT;
                if (!next_slot(sV))
                    return false;
                if (*abort_flag || !mbar_wait(&p_full[i & 1], (i >> 1) & 1, 24))
                    return false;
                if (i >= 2 && (*abort_flag || !mbar_wait(&o_free[i & 1], ((i - 2) >> 1) & 1, 25)))
                    return false;
                tc_fence_after();
                const uint32_t sP = s_base + CF::OFF_P + (i & 1) * CF::P_BYTES;
                const uint32_t d = tmem + CF::O_COL + (i & 1) * HD;
#pragma unroll
                for (int ks = 0; ks < BKV / 16; ++ks) {
                    const uint64_t ph_ = kmajor_desc(sP, BQ, ks);
                    const uint64_t pl_ = kmajor_desc(sP + CF::P_PLANE, BQ, ks);
                    const uint64_t vh_ = v_desc(sV, ks);
                    const uint64_t vl_ = v_desc(sV + CF::KV_PLANE, ks);
                    mma_bf16(d, pl_, vh_, idesc_o, ks > 0 ? 1u : 0u);
                    mma_bf16(d, ph_, vl_, idesc_o, 1u);
                    mma_bf16(d, ph_, vh_, idesc_o, 1u);
                }
                mma_commit(&o_full[i & 1]);
                mma_commit(&empty[slot]);
                return true;
            };
            for (int j = 0; j < nblk && ok; ++j) {
                uint32_t sK;
                const int slot = it % NSLOT;
                if (!next_slot(sK)) {
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
                    mma_bf16(d, ql_, kh_, idesc_s, ks > 0 ? 1u : 0u);
                    mma_bf16(d, qh_, kl_, idesc_s, 1u);
                    mma_bf16(d, qh_, kh_, idesc_s, 1u);
                }
                mma_commit(&s_full[j & 1]);
                mma_commit(&empty[slot]);
                if (j >= 1 && !issue_pv(j - 1))
                    ok = false;
            }
            if (ok && !issue_pv(nblk - 1))
                ok = false;
            if (!ok)
                *abort_flag = 1;
            // Every MMA issued has retired once this fires (also on abort).
            mma_commit(done);
            mbar_wait(done, 0, 27);
        }
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
#pragma unroll
            for (int c = 0; c < OH; c += 32) {
                float v[32];
                tmem_ld_32x32b_x32(base + c, v);
                tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 32; ++e)
                    acc[c + e] = fmaf(acc[c + e], scale, v[e]);
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
            // Both halves fold the same 64 values in the same order, so they
            // hold bit-identical maxima.
            float mx0 = half == 0 ? s[0] : so[0];
            float mx1 = half == 0 ? so[0] : s[0];
#pragma unroll
            for (int e = 1; e < 32; ++e) {
                mx0 = fmaxf(mx0, half == 0 ? s[e] : so[e]);
                mx1 = fmaxf(mx1, half == 0 ? so[e] : s[e]);
            }
            const float mx = fmaxf(mx0, mx1);
            m_prev = m_cur;
            m_cur = fmaxf(m_cur, mx * LOG2E);
            const float mc = m_cur == -INFINITY ? 0.0f : m_cur;  // all masked so far
            const float alpha = exp2f(m_prev - mc);              // 0 when m_prev = -inf
            float rs = 0.0f;
            uint32_t hi[16], lo[16];
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
                const float p0 = exp2f(fmaf(s[e], LOG2E, -mc));
                const float p1 = exp2f(fmaf(s[e + 1], LOG2E, -mc));
                rs += p0 + p1;
                const __nv_bfloat16 h0 = __float2bfloat16_rn(p0), h1 = __float2bfloat16_rn(p1);
                hi[e / 2] = pack_bf16x2(h0, h1);
                lo[e / 2] = pack_bf16x2(__float2bfloat16_rn(p0 - __bfloat162float(h0)),
                                        __float2bfloat16_rn(p1 - __bfloat162float(h1)));
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
                const float sc = m_prev == -INFINITY ? 0.0f : exp2f(m_hist - m_prev);
                if (!fold_o(j - 1, sc)) {
                    ok = false;
                    break;
                }
            }
            m_hist = m_prev;
        }
        if (ok) {
            const float sc = m_cur == -INFINITY ? 0.0f : exp2f(m_hist - m_cur);
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
    if (warp >= 2 && !*abort_flag) {
        const int quad = warp & 3, half = (warp - 2) >> 2;
        const int r = quad * 32 + lane;
        const int64_t q = q0 + r;
        const float lt = l_own + red[(half ^ 1) * BQ + r];
        if (q < T) {
            const int64_t b = bh / H, h = bh % H;
            const float inv = lt > 0.0f ? 1.0f / lt : 0.0f;
            float* dst = o + ((b * T + q) * H + h) * HD + half * OH;
#pragma unroll
            for (int c = 0; c < OH; c += 4)
                *reinterpret_cast<float4*>(dst + c) = make_float4(
                    acc[c] * inv, acc[c + 1] * inv, acc[c + 2] * inv,
                    acc[c + 3] * inv);
            if (half == 0)
                lse[bh * T + q] = m_out * LN2 + logf(lt);
        }
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

bool attention_tc_supported(int hd) { return hd == 64 || hd == 128; }

int attention_tc_forward_core(int hd, const __nv_bfloat16* qh, const __nv_bfloat16* kh,
                              const __nv_bfloat16* vh, float* o, float* lse, int64_t B, int64_t T,
                              int64_t H, cudaStream_t st) {
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
    if (hd == 128) {
        const int smem = fatc::FwdCfg<128>::BYTES;
        cudaFuncSetAttribute(fatc::attn_fwd_tc<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem);
        fatc::attn_fwd_tc<128><<<grid, fatc::NUM_THREADS, smem, st>>>(mq, mk, mv, o, lse, T,
                                                                       static_cast<int>(H));
    } else {
        const int smem = fatc::FwdCfg<64>::BYTES;
        cudaFuncSetAttribute(fatc::attn_fwd_tc<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem);
        fatc::attn_fwd_tc<64><<<grid, fatc::NUM_THREADS, smem, st>>>(mq, mk, mv, o, lse, T,
                                                                      static_cast<int>(H));
    }
    return check_launch("attn_fwd_tc");
}

}  // namespace ttk
