// fp32-accurate GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
//   C[b] = alpha * op(A[b]) @ op(B[b]) + beta * C[b]      (row-major fp32)
//
// Replaces the reference's CPU sgemm (ops.cpp:96-125) under matmul
// (ops.cpp:661-697: forward, dA = G @ B^T, dB = A^T @ G) and bmm
// (ops.cpp:699-742). op(X) = X or X^T is taken by reading the operand
// K-major or MN-major straight from its storage; no transposed copies.
//
// Precision: a three-term split. Each operand is split once (split kernels)
// into a high part and the rounded remainder, stored as two planes; the MMA
// accumulates lo*hi + hi*lo + hi*hi in an fp32 TMEM accumulator:
//   PREC_BF16X3 (default): hi = bf16_rn(x), lo = bf16_rn(x - hi), three
//     tcgen05.mma.kind::f16 (bf16) products: ~2^-17 per product, ~4e-6
//     normalized max error over any K (emulated and measured), at half the
//     tensor-core time of the TF32 split.
//   PREC_TF32X3: hi = rna_tf32(x), lo = x - hi, three kind::tf32 products:
//     ~2^-21 per product.
// Both smem layouts have 64-byte rows per k-slice (BK = 16 fp32 or 32 bf16),
// so the pipeline geometry is shared.
//
// CTA pairs (bf16 split, large problems): a cluster of two CTAs computes a
// 256 x 256 tile with tcgen05.mma.cta_group::2 (M = 256) issued by rank 0.
// Each CTA loads its 128 rows of A and 128 of the 256 rows of B into its own
// shared memory (a 6-stage ring of 32 KB stages), both CTAs' TMA loads complete
// on rank 0's barrier, the MMA commits arrive on both CTAs' barriers, and each
// CTA drains its own 128 accumulator rows from its own TMEM. Per SM this halves
// the B traffic of a 128 x 256 tile; results equal the single-CTA kernel's.
//
// Kernel structure (persistent, one CTA per SM, 64 + 32*EPI_WARPS threads):
//   warp 0      TMA producer: 4-stage ring of {A hi|lo, B hi|lo} K-slices
//               (64 B rows), one TMA per operand per stage (hi and lo planes
//               are one extra tensor dimension)
//   warp 1      TMEM allocator + MMA issuer (one lane): 2 k-steps x 3 products
//               of tcgen05.mma M128 x BN x (K8 tf32 | K16 bf16) per stage; commit
//               frees the stage. Each 256-wide K chunk accumulates into its own
//               TMEM buffer (a ring of 512/BN buffers of BN columns)
//   warps 2..   epilogue: drain each chunk buffer with tcgen05.ld into fp32
//               registers (each thread: one row x 128 columns), free it, and
//               store the finished tile with alpha/beta; the ring lets the
//               MMAs of the next chunk / tile run while a chunk is drained
// Every TMA load has one destination: the issuing CTA's shared memory.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <string>
#include <stdint.h>

#include <vector>

#include "ttk_common.cuh"
#include "ttk_internal.h"

namespace ttk {

namespace gemm {

constexpr int BM = 128;
constexpr int ROW_BYTES = 64;  // one k-slice row of an operand tile (SW64)
// Tile raster: bands of group_m M-tiles sweep the N tiles (Params.group_m,
// chosen per problem on the host so that a band's A rows stay in L2 while
// the band's N tiles read them).
// K extent accumulated inside TMEM before the partial sum is promoted to the
// epilogue's fp32 registers. The tensor-core accumulator rounds with a bias
// (its error grows linearly with K), so long sums are built from 256-wide
// chunks added with round-to-nearest FADD; error then grows like sqrt(K/256).
constexpr int KCHUNK = 256;

enum { PREC_BF16X3 = 0, PREC_TF32X3 = 1 };

template <int PREC>
struct Prec {
    static constexpr int ELT = PREC == PREC_TF32X3 ? 4 : 2;  // bytes per split element
    static constexpr int BK = ROW_BYTES / ELT;                // k per stage: 16 | 32
    static constexpr int UK = PREC == PREC_TF32X3 ? 8 : 16;   // k per MMA instruction
    static constexpr int KCHUNK_BLOCKS = KCHUNK / BK;
    // MN-major smem layout: tf32 admits only 128B swizzle with 32B atoms
    // (32 elements = 128 B per row); bf16 uses plain 64B swizzle (32
    // elements = 64 B per row). Both: 32-element chunks of the M/N extent.
    static constexpr uint32_t MN_LAYOUT = PREC == PREC_TF32X3 ? 1 : 4;
    static constexpr int MN_ROW_BYTES = 32 * ELT;
};

// PAIR: a CTA pair (cluster of two, cta_group::2) computes a 256 x BN tile
// with M = 256 MMAs issued by rank 0; each CTA loads its 128 rows of A and
// BN/2 rows of B (half the operand traffic per SM of a 128 x BN tile) and
// drains its own 128 accumulator rows.
template <int BN, bool PAIR = false>
struct Cfg {
    static constexpr int B_ROWS = PAIR ? BN / 2 : BN;  // rows of B held by one CTA
    static constexpr int A_PLANE = BM * ROW_BYTES;
    static constexpr int B_PLANE = B_ROWS * ROW_BYTES;
    static constexpr int A_BYTES = 2 * A_PLANE;  // hi | lo
    static constexpr int B_BYTES = 2 * B_PLANE;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = PAIR ? 6 : 4;
    static constexpr int NBUF = 512 / BN;            // TMEM chunk buffers
    static constexpr int TMEM_COLS = 512;
    static constexpr int EPI_WARPS = 4 * (BN / 128);  // each thread: 1 row x 128 columns
    static constexpr int NUM_THREADS = 64 + 32 * EPI_WARPS;
    // per epilogue warp: a 32 x 32 fp32 staging tile for the TMA store (128B swizzle)
    static constexpr int EPI_STAGE_BYTES = EPI_WARPS * 4096;
    static constexpr int SMEM_BYTES =
        STAGES * STAGE_BYTES + EPI_STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
    static_assert(!PAIR || BN == 256, "CTA pairs use 256 x 256 tiles");
};

// C write mode of the epilogue: direct stores (any layout, any beta), or a
// TMA store (beta = 0) / TMA reduce-add (beta = 1) of 32 x 32 staged tiles.
enum { C_DIRECT = 0, C_TMA_STORE = 1, C_TMA_ADD = 2 };

struct Params {
    int64_t M, N, K, batch;
    int a_mn, b_mn;  // 1: operand is MN-major in its storage
    int c_mode;
    float alpha, beta;
    float* C;
    int64_t ldc, strideC;
    int num_m, num_n, num_k;
    int64_t num_tiles;
    int group_m;
};

__device__ __forceinline__ void tile_coords(const Params& p, int64_t t, int& b, int& m, int& n) {
    int64_t per_batch = static_cast<int64_t>(p.num_m) * p.num_n;
    b = static_cast<int>(t / per_batch);
    int64_t r = t % per_batch;
    int64_t band = static_cast<int64_t>(p.group_m) * p.num_n;
    int64_t g = r / band;
    int first_m = static_cast<int>(g * p.group_m);
    int gsize = min(p.num_m - first_m, p.group_m);
    int64_t rr = r % band;
    m = first_m + static_cast<int>(rr % gsize);
    n = static_cast<int>(rr / gsize);
}

// Descriptor of one MMA k-step (ks = 0, 1) of an operand tile plane.
// K-major, 64B swizzle: rows of 64 B, 8-row groups 512 B apart (SBO); one
// k-step (8 tf32 | 16 bf16 = 32 B) is a 32 B offset inside the swizzled row.
// MN-major: 32-element chunks of the M/N extent, BK k-rows each, so chunks are
// BK*MN_ROW_BYTES = 2048 B apart (LBO); 8-row (bf16) / 4-row (tf32) swizzle
// groups 512 B apart (SBO); one k-step is 1024 B further (8 rows of 128 B for
// tf32, 16 rows of 64 B for bf16).
constexpr uint32_t kLayoutSW64 = 4;
template <int PREC>
__device__ __forceinline__ uint64_t operand_desc(uint32_t plane_addr, int mn_major, int ks) {
    using P = Prec<PREC>;
    if (mn_major)
        return umma_smem_desc(plane_addr + ks * 1024, P::BK * P::MN_ROW_BYTES, 512, P::MN_LAYOUT);
    return umma_smem_desc(plane_addr + ks * 32, 16, 512, kLayoutSW64);
}

// Issued by the whole MMA warp (warp-uniform loop); lane 0 performs it.
template <int PREC>
__device__ __forceinline__ void mma_split(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                          uint32_t acc) {
    if (PREC == PREC_TF32X3)
        mma_tf32_w(d, a, b, idesc, acc);
    else
        mma_bf16_w(d, a, b, idesc, acc);
}

template <int BN, int PREC, bool PAIR>
__global__ void __launch_bounds__(Cfg<BN, PAIR>::NUM_THREADS, 1)
    gemm_split3_kernel(const __grid_constant__ CUtensorMap map_a,
                       const __grid_constant__ CUtensorMap map_b,
                       const __grid_constant__ CUtensorMap map_c, const Params p) {
    using CF = Cfg<BN, PAIR>;
    using PR = Prec<PREC>;
    constexpr int BK = PR::BK;
    constexpr int KCHUNK_BLOCKS = PR::KCHUNK_BLOCKS;
    constexpr int NBUF = CF::NBUF;
    constexpr int STAGES = CF::STAGES;
    constexpr int TILE_M = PAIR ? 2 * BM : BM;  // rows of C per tile (per pair)
    static_assert(!PAIR || PREC == PREC_BF16X3, "CTA pairs run the bf16 split");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * CF::STAGE_BYTES +
                                                 CF::EPI_STAGE_BYTES);
    uint64_t* full = bars;
    uint64_t* empty = bars + STAGES;
    uint64_t* cfull = bars + 2 * STAGES;
    uint64_t* cempty = bars + 2 * STAGES + NBUF;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 2 * NBUF);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // Pair rank (0 issues the MMAs); tiles are dealt per pair.
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
    const int64_t tile0 = PAIR ? (blockIdx.x >> 1) : blockIdx.x;
    const int64_t tile_step = PAIR ? (gridDim.x >> 1) : gridDim.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < NBUF; ++b) {
            mbar_init(&cfull[b], 1);
            // one arrive per epilogue warp; rank 0's barrier collects both CTAs'
            mbar_init(&cempty[b], (PAIR ? 2 : 1) * CF::EPI_WARPS);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&map_a);
        tma_prefetch_desc(&map_b);
    }
    if (warp == 1) {
        if constexpr (PAIR) {
            tmem_alloc_pair(tmem_slot, CF::TMEM_COLS);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, CF::TMEM_COLS);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR)
        cluster_sync();  // the peer's barriers are initialized before any remote use
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            // Parity each stage was last armed with (-1: never), so that an
            // abort can wait for copies still landing in shared memory.
            int armed_ph[STAGES];
#pragma unroll
            for (int i = 0; i < STAGES; ++i)
                armed_ph[i] = -1;
            for (int64_t t = tile0; t < p.num_tiles && !*abort_flag; t += tile_step) {
                int b, mt, nt;
                tile_coords(p, t, b, mt, nt);
                const int a_row = mt * TILE_M + static_cast<int>(rank) * BM;
                const int b_row = nt * BN + static_cast<int>(rank) * CF::B_ROWS;
                for (int kb = 0; kb < p.num_k; ++kb) {
                    if (!mbar_wait(&empty[s], ph ^ 1, 1)) {
                        *abort_flag = 1;
                        break;
                    }
                    uint8_t* sa = smem + s * CF::STAGE_BYTES;
                    uint8_t* sb = sa + CF::A_BYTES;
                    const int k0 = kb * BK;
                    if constexpr (PAIR) {
                        // Rank 0 expects both CTAs' bytes on its barrier; each
                        // CTA loads its own halves into its own shared memory.
                        if (rank == 0)
                            mbar_arrive_expect_tx(&full[s], 2 * CF::STAGE_BYTES);
                        const uint32_t fb = smem_in_cta(&full[s], 0);
                        if (p.a_mn)
                            tma_load_5d_pair(sa, &map_a, fb, 0, k0, a_row / 32, 0, b);
                        else
                            tma_load_4d_pair(sa, &map_a, fb, k0, a_row, 0, b);
                        if (p.b_mn)
                            tma_load_5d_pair(sb, &map_b, fb, 0, k0, b_row / 32, 0, b);
                        else
                            tma_load_4d_pair(sb, &map_b, fb, k0, b_row, 0, b);
                    } else {
                        mbar_arrive_expect_tx(&full[s], CF::STAGE_BYTES);
                        if (p.a_mn)
                            tma_load_5d(sa, &map_a, &full[s], 0, k0, a_row / 32, 0, b);
                        else
                            tma_load_4d(sa, &map_a, &full[s], k0, a_row, 0, b);
                        if (p.b_mn)
                            tma_load_5d(sb, &map_b, &full[s], 0, k0, b_row / 32, 0, b);
                        else
                            tma_load_4d(sb, &map_b, &full[s], k0, b_row, 0, b);
                    }
                    armed_ph[s] = static_cast<int>(ph);
                    if (++s == STAGES) {
                        s = 0;
                        ph ^= 1;
                    }
                }
            }
            // On abort, let armed copies land before the CTA's smem is
            // released (rank 0 holds the barriers both CTAs' copies complete on).
            if (*abort_flag && rank == 0) {
#pragma unroll
                for (int i = 0; i < STAGES; ++i)
                    if (armed_ph[i] >= 0)
                        mbar_wait(&full[i], static_cast<uint32_t>(armed_ph[i]), 5);
            }
        }
    } else if (warp == 1 && rank == 0) {
        // -------------------------------------------------------- MMA issuer
        // The whole warp runs this loop (uniform control flow); lane 0 issues.
        const uint32_t idesc = PREC == PREC_TF32X3
                                   ? umma_idesc_tf32(TILE_M, BN, p.a_mn, p.b_mn)
                                   : umma_idesc_bf16(TILE_M, BN, p.a_mn, p.b_mn);
        int s = 0;
        uint32_t ph = 0;
        int64_t g = 0;  // chunk counter across this CTA's tiles
        bool ok = true;
        for (int64_t t = tile0; t < p.num_tiles && ok && !*abort_flag; t += tile_step) {
            for (int kc = 0; kc < p.num_k && ok; kc += KCHUNK_BLOCKS, ++g) {
                const int buf = static_cast<int>(g % NBUF);
                const uint32_t cph = static_cast<uint32_t>((g / NBUF) & 1);
                if (!mbar_wait(&cempty[buf], cph ^ 1, 2)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + buf * BN;
                const int kend = min(p.num_k, kc + KCHUNK_BLOCKS);
                for (int kb = kc; kb < kend; ++kb) {
                    if (!mbar_wait(&full[s], ph, 3)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + s * CF::STAGE_BYTES);
                    const uint32_t sb = sa + CF::A_BYTES;
#pragma unroll
                    for (int ks = 0; ks < BK / PR::UK; ++ks) {
                        const uint64_t a_hi = operand_desc<PREC>(sa, p.a_mn, ks);
                        const uint64_t a_lo = operand_desc<PREC>(sa + CF::A_PLANE, p.a_mn, ks);
                        const uint64_t b_hi = operand_desc<PREC>(sb, p.b_mn, ks);
                        const uint64_t b_lo = operand_desc<PREC>(sb + CF::B_PLANE, p.b_mn, ks);
                        const uint32_t acc = (kb > kc || ks > 0) ? 1u : 0u;
                        if constexpr (PAIR) {
                            mma_bf16_pair_w(d_tmem, a_lo, b_hi, idesc, acc);
                            mma_bf16_pair_w(d_tmem, a_hi, b_lo, idesc, 1u);
                            mma_bf16_pair_w(d_tmem, a_hi, b_hi, idesc, 1u);
                        } else {
                            mma_split<PREC>(d_tmem, a_lo, b_hi, idesc, acc);
                            mma_split<PREC>(d_tmem, a_hi, b_lo, idesc, 1u);
                            mma_split<PREC>(d_tmem, a_hi, b_hi, idesc, 1u);
                        }
                    }
                    // frees the stage in both CTAs of a pair
                    if constexpr (PAIR)
                        mma_commit_pair_w(&empty[s]);
                    else
                        mma_commit_w(&empty[s]);
                    if (++s == STAGES) {
                        s = 0;
                        ph ^= 1;
                    }
                }
                // Fires once every MMA issued so far has retired, also on
                // abort, so TMEM is quiescent before the epilogue / dealloc.
                if constexpr (PAIR)
                    mma_commit_pair_w(&cfull[buf]);
                else
                    mma_commit_w(&cfull[buf]);
            }
        }
        if (!ok)
            *abort_flag = 1;
    } else if (warp >= 2) {
        // ---------------------------------------------------------- epilogue
        // Waits are taken by lane 0 and broadcast, so every branch below is
        // warp-uniform and __syncwarp is always reached by the whole warp.
        const int e = warp - 2;
        const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
        const int col_base = (e >> 2) * 128;
        const int row_in_tile = quarter * 32 + lane;
        uint8_t* stage_c = smem + STAGES * CF::STAGE_BYTES + e * 4096;  // 32 rows x 128 B
        const bool vec_ok = ((p.ldc & 3) == 0) &&
                            ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0) &&
                            ((p.strideC & 3) == 0);
        int64_t g = 0;
        bool ok = true;
        bool pending = false;  // lane 0 has a bulk store reading stage_c
        for (int64_t t = tile0; t < p.num_tiles && ok; t += tile_step) {
            float acc[128];
#pragma unroll
            for (int j = 0; j < 128; ++j)
                acc[j] = 0.0f;
            for (int kc = 0; kc < p.num_k; kc += KCHUNK_BLOCKS, ++g) {
                const int buf = static_cast<int>(g % NBUF);
                const uint32_t cph = static_cast<uint32_t>((g / NBUF) & 1);
                int got = 0;
                if (lane == 0)
                    got = !*abort_flag && mbar_wait(&cfull[buf], cph, 4);
                if (!__shfl_sync(0xffffffffu, got, 0)) {
                    ok = false;
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float v[32];
                    tmem_ld_32x32b_x32(tmem_base + buf * BN + col_base + c * 32 +
                                           (static_cast<uint32_t>(quarter * 32) << 16),
                                       v);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        acc[c * 32 + j] += v[j];
                }
                // Each thread's TMEM reads are complete (tcgen05.wait::ld) and
                // fenced; after the warp sync one lane releases the buffer.
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if constexpr (PAIR)
                        mbar_arrive_cluster(smem_in_cta(&cempty[buf], 0));
                    else
                        mbar_arrive(&cempty[buf]);
                }
            }
            if (!ok)
                break;
            int b, mt, nt;
            tile_coords(p, t, b, mt, nt);
            const int row0 = mt * TILE_M + static_cast<int>(rank) * BM;  // this CTA's rows
            if (p.c_mode != C_DIRECT) {
                // 4 subtiles of 32 columns: registers -> 128B-swizzled staging
                // tile -> one TMA store (or reduce-add) per warp; rows and
                // columns outside C are clipped by the tensor map.
#pragma unroll
                for (int qd = 0; qd < 4; ++qd) {
                    if (lane == 0 && pending)
                        bulk_wait_read_all();
                    __syncwarp();
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const int j = qd * 32 + c * 4;
                        *reinterpret_cast<float4*>(stage_c + lane * 128 + ((c ^ (lane & 7)) << 4)) =
                            make_float4(p.alpha * acc[j], p.alpha * acc[j + 1], p.alpha * acc[j + 2],
                                        p.alpha * acc[j + 3]);
                    }
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        const int x = nt * BN + col_base + qd * 32, y = row0 + quarter * 32;
                        if (p.c_mode == C_TMA_ADD)
                            tma_reduce_add_3d(&map_c, stage_c, x, y, b);
                        else
                            tma_store_3d(&map_c, stage_c, x, y, b);
                        bulk_commit_group();
                        pending = true;
                    }
                }
                continue;
            }
            const int64_t row = static_cast<int64_t>(row0) + row_in_tile;
            if (row >= p.M)
                continue;
            const int64_t col0 = static_cast<int64_t>(nt) * BN + col_base;
            float* dst = p.C + b * p.strideC + row * p.ldc + col0;
            if (vec_ok && col0 + 128 <= p.N) {
#pragma unroll
                for (int j = 0; j < 128; j += 4) {
                    float4 o = make_float4(p.alpha * acc[j], p.alpha * acc[j + 1],
                                           p.alpha * acc[j + 2], p.alpha * acc[j + 3]);
                    if (p.beta != 0.0f) {
                        const float4 ci = *reinterpret_cast<const float4*>(dst + j);
                        o.x += p.beta * ci.x;
                        o.y += p.beta * ci.y;
                        o.z += p.beta * ci.z;
                        o.w += p.beta * ci.w;
                    }
                    *reinterpret_cast<float4*>(dst + j) = o;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 128; ++j) {
                    if (col0 + j < p.N) {
                        float o = p.alpha * acc[j];
                        if (p.beta != 0.0f)
                            o += p.beta * dst[j];
                        dst[j] = o;
                    }
                }
            }
        }
        // Bulk stores complete before the kernel ends.
        if (lane == 0 && pending)
            bulk_wait_all();
    }

    tc_fence_before();
    __syncthreads();
    // Neither CTA of a pair leaves (or frees TMEM) while the other may still
    // signal its barriers or read its shared memory.
    if constexpr (PAIR)
        cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        if constexpr (PAIR)
            tmem_dealloc_pair(tmem_base, CF::TMEM_COLS);
        else
            tmem_dealloc(tmem_base, CF::TMEM_COLS);
    }
}

// Split of src (rows x cols per batch, leading dim ld) into planes
// dst[b][0|1][r][0..ld_pad) = hi | lo, zeros in the padding [cols, ld_pad):
//   float dst: hi = rna_tf32(x), lo = x - hi (exact in fp32)
//   bf16 dst:  hi = bf16_rn(x), lo = bf16_rn(x - hi)
__device__ __forceinline__ void split_one(float x, float& hi, float& lo) {
    uint32_t h;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
    hi = __uint_as_float(h);
    lo = x - hi;
}

__device__ __forceinline__ void split_one(float x, __nv_bfloat16& hi, __nv_bfloat16& lo) {
    split_bf16(x, hi, lo);
}

// Launch shape: TPR threads per row (a power of two covering the row's
// 4-element groups, at most the block), 256 / TPR rows per block sweep, rows
// strided over the grid; the batch index is divided out once per row.
template <class T>
__global__ void split_kernel(const float* __restrict__ src, int64_t rows, int64_t cols,
                             int64_t ld, int64_t bstride, int64_t batch, T* __restrict__ dst,
                             int64_t ld_pad, int tpr) {
    const int64_t per_row = ld_pad / 4;  // 4-element groups per padded row
    const int64_t nrows = batch * rows;
    const int64_t plane = rows * ld_pad;
    const int rpb = blockDim.x / tpr;
    const int lr = threadIdx.x / tpr, lg = threadIdx.x % tpr;
    const bool vec = ((ld & 3) == 0) && ((bstride & 3) == 0) &&
                     ((reinterpret_cast<uintptr_t>(src) & 15) == 0);
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * rpb + lr; row < nrows;
         row += static_cast<int64_t>(gridDim.x) * rpb) {
        const int64_t b = row / rows, r = row - b * rows;
        const float* s_row = src + b * bstride + r * ld;
        T* d_row = dst + b * 2 * plane + r * ld_pad;
        for (int64_t g = lg; g < per_row; g += tpr) {
            const int64_t c0 = g * 4;
            float x[4];
            if (vec && c0 + 4 <= cols) {
                const float4 t = __ldg(reinterpret_cast<const float4*>(s_row + c0));
                x[0] = t.x, x[1] = t.y, x[2] = t.z, x[3] = t.w;
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    x[j] = (c0 + j < cols) ? __ldg(s_row + c0 + j) : 0.0f;
            }
            T hi[4], lo[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                split_one(x[j], hi[j], lo[j]);
            T* d = d_row + c0;
            if (sizeof(T) == 4) {
                *reinterpret_cast<float4*>(d) = *reinterpret_cast<const float4*>(hi);
                *reinterpret_cast<float4*>(d + plane) = *reinterpret_cast<const float4*>(lo);
            } else {
                *reinterpret_cast<uint2*>(d) = *reinterpret_cast<const uint2*>(hi);
                *reinterpret_cast<uint2*>(d + plane) = *reinterpret_cast<const uint2*>(lo);
            }
        }
    }
}

__global__ void scale_kernel(float* C, int64_t batch, int64_t M, int64_t N, int64_t ldc,
                             int64_t strideC, float beta) {
    const int64_t total = batch * M * N;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t n = i % N, m = (i / N) % M, b = i / (M * N);
        float* c = C + b * strideC + m * ldc + n;
        *c = beta == 0.0f ? 0.0f : beta * *c;
    }
}

// Split-K finish: C = alpha * sum_s W[s] + beta * C over S partial products
// W[s] (M x N, leading dimension ldw, slices M*ldw apart), s ascending: a
// fixed summation order, so the result is deterministic.
__global__ void splitk_reduce_kernel(const float* __restrict__ W, int S, int64_t M, int64_t N,
                                     int64_t ldw, float alpha, float beta, float* __restrict__ C,
                                     int64_t ldc) {
    const int64_t slice = M * ldw;
    const bool vec = ((N & 3) == 0) && ((ldc & 3) == 0) &&
                     ((reinterpret_cast<uintptr_t>(C) & 15) == 0);
    if (vec) {
        const int64_t n4 = N / 4, total = M * n4;
        for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
             i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
            const int64_t m = i / n4, c = (i % n4) * 4;
            const float* w = W + m * ldw + c;
            float4 acc = *reinterpret_cast<const float4*>(w);
            for (int s = 1; s < S; ++s) {
                const float4 v = *reinterpret_cast<const float4*>(w + s * slice);
                acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
            }
            float4* dst = reinterpret_cast<float4*>(C + m * ldc + c);
            float4 o = make_float4(alpha * acc.x, alpha * acc.y, alpha * acc.z, alpha * acc.w);
            if (beta != 0.0f) {
                const float4 ci = *dst;
                o.x += beta * ci.x, o.y += beta * ci.y, o.z += beta * ci.z, o.w += beta * ci.w;
            }
            *dst = o;
        }
        return;
    }
    const int64_t total = M * N;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t m = i / N, c = i % N;
        float acc = W[m * ldw + c];
        for (int s = 1; s < S; ++s)
            acc += W[s * slice + m * ldw + c];
        float* dst = C + m * ldc + c;
        float o = alpha * acc;
        if (beta != 0.0f)
            o += beta * *dst;
        *dst = o;
    }
}

// Exact fp32 GEMM for small problems (at most gemm_fp32_max_macs()
// multiply-adds): C = alpha * op(A) op(B) + beta * C with one fp32 fused
// multiply-add per product in ascending k, the reference's sgemm arithmetic
// (ops.cpp:96-125). A 256-thread block owns a 32 x 32 tile of C (a column
// per lane, four rows per warp) and stages 32-deep slices of op(A) and op(B)
// in shared memory, zero outside the matrix. Below this size the operand
// split's extra launches cost more than the products, and the result is
// as smooth in the inputs as an fp32 loop: finite-difference gradient checks
// see no split truncation steps.
constexpr int F32_T = 32;
__global__ void __launch_bounds__(256) gemm_fp32_kernel(
    int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float* __restrict__ A,
    int64_t lda, int64_t sA, const float* __restrict__ B, int64_t ldb, int64_t sB, float beta,
    float* __restrict__ C, int64_t ldc, int64_t sC) {
    __shared__ float as[F32_T][F32_T + 1];  // [m][k]
    __shared__ float bs[F32_T][F32_T + 1];  // [k][n]
    const int64_t bat = blockIdx.z;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * F32_T;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * F32_T;
    A += bat * sA, B += bat * sB, C += bat * sC;
    const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int64_t k0 = 0; k0 < K; k0 += F32_T) {
        for (int i = threadIdx.x; i < F32_T * F32_T; i += 256) {
            const int r = i >> 5, c = i & 31;
            // op(A)[m][k]: r = m offset, c = k offset (k-contiguous for ta = 0)
            const int64_t am = m0 + (ta ? c : r), ak = k0 + (ta ? r : c);
            float av = 0.0f;
            if (am < M && ak < K)
                av = ta ? A[ak * lda + am] : A[am * lda + ak];
            if (ta)
                as[c][r] = av;
            else
                as[r][c] = av;
            // op(B)[k][n]: r = k offset, c = n offset (n-contiguous for tb = 0)
            const int64_t bk = k0 + (tb ? c : r), bn = n0 + (tb ? r : c);
            float bv = 0.0f;
            if (bk < K && bn < N)
                bv = tb ? B[bn * ldb + bk] : B[bk * ldb + bn];
            if (tb)
                bs[c][r] = bv;
            else
                bs[r][c] = bv;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < F32_T; ++kk) {
            const float bv = bs[kk][lane];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                acc[i] = fmaf(as[wp + 8 * i][kk], bv, acc[i]);
        }
        __syncthreads();
    }
    const int64_t n = n0 + lane;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t m = m0 + wp + 8 * i;
        if (m < M && n < N) {
            float* c = C + m * ldc + n;
            const float r = alpha * acc[i];
            *c = beta == 0.0f ? r : r + beta * *c;
        }
    }
}

}  // namespace gemm

// ------------------------------------------------------------- host side --

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

namespace {

inline int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

// Storage geometry of one split operand: rows x cols per batch, padded to
// ld_pad elements, planes hi|lo of elt-byte elements.
struct SplitGeom {
    int64_t rows, cols, ld_pad;
    int elt;
    size_t bytes(int64_t batch) const {
        return static_cast<size_t>(batch) * 2 * rows * ld_pad * elt;
    }
};

// K-major map: dims {cols(K), rows(M|N), plane, batch}, box {BK, tile, 2, 1},
//               64B swizzle (64-byte rows).
// MN-major map: dims {32, rows(K), cols/32 chunks, plane, batch},
//               box {32, BK, tile/32, 2, 1}: tf32 128B swizzle with 32B atoms
//               (128-byte rows), bf16 64B swizzle (64-byte rows).
// kslices > 1 (split-K; batch 1): the K extent is cut into kslices equal
// slices that the map presents as its batch dimension, so batch index s of the
// kernel reads K range [s*K/kslices, (s+1)*K/kslices).
template <int PREC>
int make_operand_map(CUtensorMap* map, const void* base, const SplitGeom& g, int64_t batch,
                     int mn_major, int tile, int kslices = 1) {
    using PR = gemm::Prec<PREC>;
    EncodeTiledFn enc = encode_fn();
    if (!enc)
        return set_error(TTK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const CUtensorMapDataType dt = PREC == gemm::PREC_TF32X3 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                              : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const cuuint64_t plane = static_cast<cuuint64_t>(g.rows * g.ld_pad * PR::ELT);
    CUresult r;
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    if (!mn_major) {
        // K is the column extent
        const int64_t kc = g.cols / kslices;
        cuuint64_t dims[4] = {static_cast<cuuint64_t>(kc), static_cast<cuuint64_t>(g.rows), 2,
                              static_cast<cuuint64_t>(kslices > 1 ? kslices : batch)};
        cuuint64_t strides[3] = {static_cast<cuuint64_t>(g.ld_pad * PR::ELT), plane,
                                 kslices > 1 ? static_cast<cuuint64_t>(kc * PR::ELT) : 2 * plane};
        cuuint32_t box[4] = {PR::BK, static_cast<cuuint32_t>(tile), 2, 1};
        r = enc(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
        // K is the row extent
        const int64_t kr = g.rows / kslices;
        cuuint64_t dims[5] = {32, static_cast<cuuint64_t>(kr),
                              static_cast<cuuint64_t>(g.ld_pad / 32), 2,
                              static_cast<cuuint64_t>(kslices > 1 ? kslices : batch)};
        cuuint64_t strides[4] = {static_cast<cuuint64_t>(g.ld_pad * PR::ELT),
                                 static_cast<cuuint64_t>(32 * PR::ELT), plane,
                                 kslices > 1 ? static_cast<cuuint64_t>(kr * g.ld_pad * PR::ELT)
                                             : 2 * plane};
        cuuint32_t box[5] = {32, PR::BK, static_cast<cuuint32_t>(tile / 32), 2, 1};
        r = enc(map, dt, 5, const_cast<void*>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE,
                PREC == gemm::PREC_TF32X3 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                          : CU_TENSOR_MAP_SWIZZLE_64B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r != CUDA_SUCCESS)
        return set_error(TTK_ERR_CUDA, "cuTensorMapEncodeTiled failed");
    return TTK_OK;
}

int num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0)
            n = 148;
    }
    return n;
}

// Optional live timing of the tcgen05 kernel (ttk_profile_enable): an event
// pair around each launch, read back and summed by ttk_profile_read.
struct ProfRec {
    cudaEvent_t a, b;
    double flops;
};
struct Profiler {
    bool on = false;
    std::vector<ProfRec> recs;
    std::vector<cudaEvent_t> pool;
    cudaEvent_t get() {
        if (!pool.empty()) {
            cudaEvent_t e = pool.back();
            pool.pop_back();
            return e;
        }
        cudaEvent_t e;
        cudaEventCreate(&e);
        return e;
    }
};
Profiler& prof() {
    static thread_local Profiler p;
    return p;
}

// Second step of a split-K GEMM: C = alpha * sum_s W[s] + beta * C.
struct SplitKFinish {
    const float* W;
    int S;
    int64_t M, N, ldw;
    float alpha, beta;
    float* C;
    int64_t ldc;
};

// Band height of the tile raster (bands of group_m M tiles, each band sweeping
// the N tiles with M fastest). Operand bytes per batch entry (hi and lo
// planes): A = M x K, B = N x K.
//   B within 48 MB: group 1, rows of N tiles; B stays in L2 and each A block
//     is read once.
//   else A <= B: one band over all M tiles (up to 16); the B column tile is
//     read once and the smaller A is what gets re-read.
//   else: bands whose A rows total about 48 MB.
// TTK_GEMM_GROUP_M overrides the choice.
int raster_group(int tile_m, int num_m, int64_t M, int64_t N, int64_t K, int elt) {
    static int env = -1;
    if (env < 0) {
        const char* e = std::getenv("TTK_GEMM_GROUP_M");
        env = e ? std::max(0, std::atoi(e)) : 0;
    }
    if (env > 0)
        return env;
    const double budget = 48.0 * (1 << 20);
    const double a_total = static_cast<double>(M) * K * 2 * elt;
    const double b_total = static_cast<double>(N) * K * 2 * elt;
    if (b_total <= budget)
        return 1;
    if (a_total <= b_total)
        return std::max(1, std::min(16, num_m));
    const double band_row_bytes = static_cast<double>(tile_m) * K * 2 * elt;
    return std::max(1, std::min(16, static_cast<int>(budget / band_row_bytes)));
}

template <int BN, int PREC, bool PAIR>
int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc,
                gemm::Params p, cudaStream_t stream, const SplitKFinish* fin = nullptr) {
    using CF = gemm::Cfg<BN, PAIR>;
    auto kern = gemm::gemm_split3_kernel<BN, PREC, PAIR>;
    static bool attr_set[64] = {};
    static int max_pairs[64] = {};  // co-resident clusters of two (PAIR)
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64)
        return set_error(TTK_ERR_ARG, "gemm: device ordinal out of range");
    cudaLaunchAttribute cluster_attr;
    cluster_attr.id = cudaLaunchAttributeClusterDimension;
    cluster_attr.val.clusterDim.x = 2;
    cluster_attr.val.clusterDim.y = 1;
    cluster_attr.val.clusterDim.z = 1;
    if (!attr_set[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 CF::SMEM_BYTES) != cudaSuccess)
            return set_error(TTK_ERR_CUDA, "cudaFuncSetAttribute(gemm) failed");
        if (PAIR) {
            // Persistent grid: as many pairs as can be resident at once (a
            // cluster's two CTAs share a GPC, so this can be below SMs / 2).
            cudaLaunchConfig_t q = {};
            q.gridDim = dim3(2);
            q.blockDim = dim3(CF::NUM_THREADS);
            q.dynamicSmemBytes = CF::SMEM_BYTES;
            q.attrs = &cluster_attr;
            q.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, kern, &q) != cudaSuccess || n <= 0) {
                cudaGetLastError();
                n = num_sms() / 2;
            }
            max_pairs[dev] = std::min(n, num_sms() / 2);
        }
        attr_set[dev] = true;
    }
    p.num_n = static_cast<int>((p.N + BN - 1) / BN);
    p.num_tiles = static_cast<int64_t>(p.num_m) * p.num_n * p.batch;
    p.group_m = raster_group(PAIR ? 2 * gemm::BM : gemm::BM, p.num_m, p.M, p.N, p.K,
                             PREC == gemm::PREC_TF32X3 ? 4 : 2);
    Profiler& pr = prof();
    ProfRec rec{};
    // No timing events inside a stream capture: a replayed graph would not
    // add records, and the recorded pair would be read as a launch.
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    const bool timed = pr.on && cudaStreamIsCapturing(stream, &cap) == cudaSuccess &&
                       cap == cudaStreamCaptureStatusNone;
    if (timed) {
        rec.a = pr.get();
        rec.b = pr.get();
        rec.flops = 2.0 * static_cast<double>(p.M) * p.N * p.K * p.batch;
        cudaEventRecord(rec.a, stream);
    }
    if (PAIR) {
        const int pairs = static_cast<int>(std::min<int64_t>(p.num_tiles, max_pairs[dev]));
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * pairs);
        cfg.blockDim = dim3(CF::NUM_THREADS);
        cfg.dynamicSmemBytes = CF::SMEM_BYTES;
        cfg.stream = stream;
        cfg.attrs = &cluster_attr;
        cfg.numAttrs = 1;
        cudaLaunchKernelEx(&cfg, kern, ma, mb, mc, p);
    } else {
        const int grid = static_cast<int>(std::min<int64_t>(p.num_tiles, num_sms()));
        kern<<<grid, CF::NUM_THREADS, CF::SMEM_BYTES, stream>>>(ma, mb, mc, p);
    }
    int rc = check_launch("gemm_split3_kernel");
    if (!rc && fin) {
        const int64_t work = fin->M * ((fin->N & 3) == 0 ? fin->N / 4 : fin->N);
        const int blocks = static_cast<int>(std::min<int64_t>((work + 255) / 256, 148 * 8));
        gemm::splitk_reduce_kernel<<<blocks, 256, 0, stream>>>(fin->W, fin->S, fin->M, fin->N,
                                                             fin->ldw, fin->alpha, fin->beta,
                                                             fin->C, fin->ldc);
        rc = check_launch("splitk_reduce_kernel");
    }
    if (timed) {
        cudaEventRecord(rec.b, stream);
        pr.recs.push_back(rec);
    }
    return rc;
}

// CTA-pair tiles for the bf16 split: 0 never, 1 when the pair tiles occupy
// every pair (default), 2 whenever N > 128 (covers edge tiles on small
// problems). TTK_GEMM_PAIRS=0|1|2 sets it at start-up.
int g_pairs = -1;

int cta_pairs_mode() {
    if (g_pairs < 0) {
        const char* e = std::getenv("TTK_GEMM_PAIRS");
        g_pairs = (e && (e[0] == '0' || e[0] == '2') && e[1] == 0) ? e[0] - '0' : 1;
    }
    return g_pairs;
}

// Tile configuration the kernel uses for (batch, M, N): CTA pairs with
// 256 x 256 tiles, or single CTAs with 128 x BN tiles; `slots` tiles run at
// once on the persistent grid.
struct TilePlan {
    bool pair;
    int bn;
    int64_t tiles, slots;
};

TilePlan tile_plan(int prec, int64_t batch, int64_t M, int64_t N) {
    const int64_t pair_tiles = ((M + 2 * gemm::BM - 1) / (2 * gemm::BM)) * ((N + 255) / 256) * batch;
    const int pmode = cta_pairs_mode();
    if (prec == gemm::PREC_BF16X3 && N > 128 &&
        (pmode == 2 || (pmode == 1 && pair_tiles >= num_sms() / 2)))
        return {true, 256, pair_tiles, num_sms() / 2};
    const int64_t mt = (M + gemm::BM - 1) / gemm::BM;
    const int64_t tiles256 = mt * ((N + 255) / 256) * batch;
    const int bn = (N <= 128 || tiles256 < num_sms()) ? 128 : 256;
    return {false, bn, mt * ((N + bn - 1) / bn) * batch, num_sms()};
}

// Fraction of the slots busy over the waves needed for `units` tiles.
double wave_eff(int64_t units, int64_t slots) {
    const int64_t waves = (units + slots - 1) / slots;
    return static_cast<double>(units) / static_cast<double>(waves * slots);
}

// Split-K (TTK_GEMM_SPLITK=0 disables): a single long-K problem whose tiles
// fill the machine's slots poorly (the weight gradients dW = dY^T X, whose
// M x N is small against K = tokens) runs as S K-slices, each writing a
// partial product, and one pass sums the partials in slice order.
int g_splitk = -1;

bool splitk_enabled() {
    if (g_splitk < 0) {
        const char* e = std::getenv("TTK_GEMM_SPLITK");
        g_splitk = (e && e[0] == '0' && e[1] == 0) ? 0 : 1;
    }
    return g_splitk != 0;
}

constexpr int64_t kSplitKMaxBytes = int64_t(512) << 20;

int64_t splitk_ldw(int64_t N) { return round_up(N, 4); }

size_t splitk_bytes(int S, int64_t M, int64_t N) {
    return S > 1 ? static_cast<size_t>(S) * M * splitk_ldw(N) * 4 : 0;
}

// Slices: the smallest S (K divisible by S, slices a multiple of 256 long)
// that lifts the wave efficiency clearly; 1 when the problem fills the
// machine already.
int choose_split_k(int prec, int64_t batch, int64_t M, int64_t N, int64_t K) {
    if (!splitk_enabled() || batch != 1 || K < 2048)
        return 1;
    const TilePlan t1 = tile_plan(prec, 1, M, N);
    double best = wave_eff(t1.tiles, t1.slots);
    if (best >= 0.9)
        return 1;
    int best_s = 1;
    for (int S = 2; S <= 16; ++S) {
        if (K % S || (K / S) % 256)
            continue;
        if (static_cast<int64_t>(splitk_bytes(S, M, N)) > kSplitKMaxBytes)
            break;
        const TilePlan t = tile_plan(prec, S, M, N);
        const double e = wave_eff(t.tiles, t.slots);
        if (e > best + 0.05) {
            best = e;
            best_s = S;
        }
        if (best >= 0.95)
            break;
    }
    return best_s;
}

struct GemmPlan {
    SplitGeom ga, gb;
    size_t off_b, total;
    size_t off_w, w_bytes;  // split-K partials (0 bytes when not split)
};

GemmPlan plan(int prec, int transA, int transB, int64_t batch, int64_t M, int64_t N, int64_t K,
              bool allow_splitk = true) {
    GemmPlan pl;
    const int elt = prec == gemm::PREC_TF32X3 ? 4 : 2;
    // op(A) = A [M,K] (K-major) or A^T with A stored [K,M] (MN-major).
    // K-major rows are padded to 16 elements, MN-major rows to 32 (whole chunks).
    pl.ga = transA ? SplitGeom{K, M, round_up(M, 32), elt} : SplitGeom{M, K, round_up(K, 16), elt};
    // op(B) = B [K,N] (MN-major) or B^T with B stored [N,K] (K-major).
    pl.gb = transB ? SplitGeom{N, K, round_up(K, 16), elt} : SplitGeom{K, N, round_up(N, 32), elt};
    pl.off_b = static_cast<size_t>(round_up(static_cast<int64_t>(pl.ga.bytes(batch)), 256));
    pl.total = pl.off_b + pl.gb.bytes(batch);
    const int S = allow_splitk ? choose_split_k(prec, batch, M, N, K) : 1;
    pl.off_w = static_cast<size_t>(round_up(static_cast<int64_t>(pl.total), 256));
    pl.w_bytes = splitk_bytes(S, M, N);
    if (pl.w_bytes)
        pl.total = pl.off_w + pl.w_bytes;
    return pl;
}

}  // namespace

int gemm_profile_enable(int on) {
    prof().on = on != 0;
    return TTK_OK;
}

int gemm_profile_read(double* ms, double* flops, int64_t* launches) {
    Profiler& pr = prof();
    double tms = 0.0, tfl = 0.0;
    for (auto& r : pr.recs) {
        float m = 0.0f;
        if (cudaEventSynchronize(r.b) != cudaSuccess ||
            cudaEventElapsedTime(&m, r.a, r.b) != cudaSuccess)
            return set_error(TTK_ERR_CUDA, "profile: event read failed");
        tms += m;
        tfl += r.flops;
        pr.pool.push_back(r.a);
        pr.pool.push_back(r.b);
    }
    if (ms)
        *ms = tms;
    if (flops)
        *flops = tfl;
    if (launches)
        *launches = static_cast<int64_t>(pr.recs.size());
    pr.recs.clear();
    return TTK_OK;
}

namespace {

// Process-wide precision of ttk_gemm (TTK_GEMM_PRECISION=tf32x3 selects the
// TF32 split; default bf16x3).
int g_prec = -1;


int current_prec() {
    if (g_prec < 0) {
        const char* e = std::getenv("TTK_GEMM_PRECISION");
        g_prec = (e && (std::string(e) == "tf32x3" || std::string(e) == "1"))
                     ? gemm::PREC_TF32X3
                     : gemm::PREC_BF16X3;
    }
    return g_prec;
}

template <int PREC>
int launch_split(const float* src, int64_t rows, int64_t cols, int64_t ld, int64_t bstride,
                 int64_t batch, void* dst, int64_t ld_pad, cudaStream_t stream) {
    const int64_t per_row = ld_pad / 4, nrows = batch * rows;
    if (per_row == 0 || nrows == 0)
        return TTK_OK;
    const int threads = 256;
    int tpr = 1;  // threads per row: a power of two covering the row, at most the block
    while (tpr < threads && tpr < per_row)
        tpr <<= 1;
    const int64_t rpb = threads / tpr;
    const int64_t blocks = std::min<int64_t>((nrows + rpb - 1) / rpb, 148 * 16);
    if (PREC == gemm::PREC_TF32X3)
        gemm::split_kernel<float><<<static_cast<int>(blocks), threads, 0, stream>>>(
            src, rows, cols, ld, bstride, batch, static_cast<float*>(dst), ld_pad, tpr);
    else
        gemm::split_kernel<__nv_bfloat16><<<static_cast<int>(blocks), threads, 0, stream>>>(
            src, rows, cols, ld, bstride, batch, static_cast<__nv_bfloat16*>(dst), ld_pad, tpr);
    return check_launch("split_kernel");
}

// Tensor map over C (fp32 [batch][M][ldc]) for the epilogue's TMA stores:
// boxes of 32 x 32 in the 128B swizzle. Returns the epilogue mode: a TMA store
// for beta = 0, a TMA reduce-add (C += tile, one fp32 add per element) for
// beta = 1, and direct stores otherwise or when C's layout does not satisfy
// the TMA alignment rules (16-byte base, row and batch strides).
int c_tensor_map(CUtensorMap* map, float* C, int64_t M, int64_t N, int64_t ldc, int64_t strideC,
                 int64_t batch, float beta) {
    if (beta != 0.0f && beta != 1.0f)
        return gemm::C_DIRECT;
    const int64_t bstride = batch > 1 ? strideC : M * ldc;
    if ((reinterpret_cast<uintptr_t>(C) & 15) || (ldc & 3) || (bstride & 3) || N < 1 || M < 1)
        return gemm::C_DIRECT;
    EncodeTiledFn enc = encode_fn();
    if (!enc)
        return gemm::C_DIRECT;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M),
                          static_cast<cuuint64_t>(batch)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(ldc) * 4, static_cast<cuuint64_t>(bstride) * 4};
    cuuint32_t box[3] = {32, 32, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    if (enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, C, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return gemm::C_DIRECT;
    return beta == 0.0f ? gemm::C_TMA_STORE : gemm::C_TMA_ADD;
}

// kmode: 0 = no split-K; 1 = split-K partials in the caller's workspace kws
// (kws_bytes; falls back to one pass if too small); 2 = partials from the
// stream-ordered pool.
template <int PREC>
int run_presplit(int transA, int transB, int64_t batch, int64_t M, int64_t N, int64_t K,
                 float alpha, const void* a_split, int64_t lda_pad, const void* b_split,
                 int64_t ldb_pad, float beta, float* C, int64_t ldc, int64_t strideC,
                 cudaStream_t stream, int kmode = 0, void* kws = nullptr,
                 size_t kws_bytes = 0) {
    using PR = gemm::Prec<PREC>;
    if (M <= 0 || N <= 0 || K <= 0 || batch <= 0)
        return set_error(TTK_ERR_ARG, "gemm_presplit: sizes must be positive");
    // K-major planes: leading dimension a multiple of 16; MN-major: of 32.
    if ((reinterpret_cast<uintptr_t>(a_split) & 15) || (reinterpret_cast<uintptr_t>(b_split) & 15) ||
        (lda_pad & (transA ? 31 : 15)) || (ldb_pad & (transB ? 15 : 31)))
        return set_error(TTK_ERR_ARG, "gemm_presplit: split planes misaligned or badly padded");
    SplitGeom ga = transA ? SplitGeom{K, M, lda_pad, PR::ELT} : SplitGeom{M, K, lda_pad, PR::ELT};
    SplitGeom gb = transB ? SplitGeom{N, K, ldb_pad, PR::ELT} : SplitGeom{K, N, ldb_pad, PR::ELT};
    if (ga.ld_pad < ga.cols || gb.ld_pad < gb.cols)
        return set_error(TTK_ERR_ARG, "gemm_presplit: padded leading dimension too small");
    // Split-K: S slices of K, each a batch entry writing its partial product
    // to W[s]; the finish step adds them in slice order into C.
    int S = kmode ? choose_split_k(PREC, batch, M, N, K) : 1;
    float* W = nullptr;
    bool own_w = false;
    if (S > 1) {
        const size_t need = splitk_bytes(S, M, N);
        if (kmode == 1) {
            if (kws && kws_bytes >= need && !(reinterpret_cast<uintptr_t>(kws) & 15))
                W = static_cast<float*>(kws);
        } else if (cudaMallocAsync(reinterpret_cast<void**>(&W), need, stream) == cudaSuccess) {
            own_w = true;
        } else {
            cudaGetLastError();
            W = nullptr;
        }
        if (!W)
            S = 1;
    }
    const int64_t kb = K / S, nb = S > 1 ? S : batch;
    gemm::Params p{};
    p.M = M, p.N = N, p.K = kb, p.batch = nb;
    p.a_mn = transA ? 1 : 0;
    p.b_mn = transB ? 0 : 1;
    p.num_m = static_cast<int>((M + gemm::BM - 1) / gemm::BM);
    p.num_k = static_cast<int>((kb + PR::BK - 1) / PR::BK);
    SplitKFinish fin{};
    if (S > 1) {
        const int64_t ldw = splitk_ldw(N);
        p.alpha = 1.0f, p.beta = 0.0f;
        p.C = W, p.ldc = ldw, p.strideC = M * ldw;
        fin = SplitKFinish{W, S, M, N, ldw, alpha, beta, C, ldc};
    } else {
        p.alpha = alpha, p.beta = beta;
        p.C = C, p.ldc = ldc, p.strideC = strideC;
    }
    const TilePlan tp = tile_plan(PREC, nb, M, N);
    const int bn = tp.bn;
    CUtensorMap ma, mb, mc;
    int rc = make_operand_map<PREC>(&ma, a_split, ga, batch, p.a_mn, gemm::BM, S);
    // a CTA of a pair holds half of B's 256 rows
    if (!rc)
        rc = make_operand_map<PREC>(&mb, b_split, gb, batch, p.b_mn, tp.pair ? bn / 2 : bn, S);
    if (!rc) {
        std::memset(&mc, 0, sizeof(mc));
        p.c_mode = c_tensor_map(&mc, p.C, M, N, p.ldc, p.strideC, nb, p.beta);
        const SplitKFinish* f = S > 1 ? &fin : nullptr;
        rc = -1;
        if constexpr (PREC == gemm::PREC_BF16X3) {
            if (tp.pair) {
                p.num_m = static_cast<int>((M + 2 * gemm::BM - 1) / (2 * gemm::BM));
                rc = launch_gemm<256, PREC, true>(ma, mb, mc, p, stream, f);
            }
        }
        if (rc == -1)
            rc = bn == 128 ? launch_gemm<128, PREC, false>(ma, mb, mc, p, stream, f)
                           : launch_gemm<256, PREC, false>(ma, mb, mc, p, stream, f);
    }
    if (own_w)
        cudaFreeAsync(W, stream);
    return rc;
}

}  // namespace

int gemm_set_precision(int prec) {
    if (prec != gemm::PREC_BF16X3 && prec != gemm::PREC_TF32X3)
        return set_error(TTK_ERR_ARG, "gemm precision must be 0 (bf16x3) or 1 (tf32x3)");
    g_prec = prec;
    return TTK_OK;
}

int gemm_get_precision() { return current_prec(); }

int gemm_set_cta_pairs(int mode) {
    if (mode < 0 || mode > 2)
        return set_error(TTK_ERR_ARG, "gemm: CTA-pair mode must be 0, 1 or 2");
    g_pairs = mode;
    return TTK_OK;
}

int gemm_get_cta_pairs() { return cta_pairs_mode(); }

int gemm_set_split_k(int on) {
    g_splitk = on ? 1 : 0;
    return TTK_OK;
}

int gemm_get_split_k() { return splitk_enabled() ? 1 : 0; }

int gemm_split_k_slices(int transA, int transB, int64_t batch, int64_t M, int64_t N, int64_t K) {
    (void)transA, (void)transB;
    if (M <= 0 || N <= 0 || K <= 0 || batch <= 0 || gemm_uses_fp32(batch, M, N, K))
        return 1;
    return choose_split_k(current_prec(), batch, M, N, K);
}

namespace {
int64_t g_fp32_max_macs = int64_t(1) << 24;
}

int gemm_set_fp32_max_macs(int64_t macs) {
    if (macs < 0)
        return set_error(TTK_ERR_ARG, "gemm: fp32 size limit must be >= 0");
    g_fp32_max_macs = macs;
    return TTK_OK;
}

int64_t gemm_fp32_max_macs() { return g_fp32_max_macs; }

bool gemm_uses_fp32(int64_t batch, int64_t M, int64_t N, int64_t K) {
    if (batch <= 0 || M <= 0 || N <= 0 || K <= 0 || batch > 65535 ||
        (M + gemm::F32_T - 1) / gemm::F32_T > 65535)
        return false;
    // Overflow-safe batch * M * N * K <= limit.
    double macs = static_cast<double>(batch) * M * N * K;
    return macs <= static_cast<double>(g_fp32_max_macs);
}

size_t gemm_workspace_size(int transA, int transB, int64_t batch, int64_t M, int64_t N,
                           int64_t K, bool allow_splitk) {
    if (M <= 0 || N <= 0 || K <= 0 || batch <= 0 || gemm_uses_fp32(batch, M, N, K))
        return 0;
    return plan(current_prec(), transA, transB, batch, M, N, K, allow_splitk).total;
}

int split_tf32(const float* src, int64_t rows, int64_t cols, int64_t ld, int64_t bstride,
               int64_t batch, float* dst, int64_t ld_pad, cudaStream_t stream) {
    return launch_split<gemm::PREC_TF32X3>(src, rows, cols, ld, bstride, batch, dst, ld_pad,
                                           stream);
}

int gemm_run(int transA, int transB, int64_t batch, int64_t M, int64_t N, int64_t K, float alpha,
             const float* A, int64_t lda, int64_t strideA, const float* B, int64_t ldb,
             int64_t strideB, float beta, float* C, int64_t ldc, int64_t strideC, void* ws,
             size_t ws_bytes, cudaStream_t stream, bool allow_splitk) {
    if (M < 0 || N < 0 || K < 0 || batch < 0)
        return set_error(TTK_ERR_ARG, "gemm: negative size");
    if (M == 0 || N == 0 || batch == 0)
        return TTK_OK;
    if (!C || (K > 0 && (!A || !B)))
        return set_error(TTK_ERR_ARG, "gemm: null pointer");
    if (ldc < N)
        return set_error(TTK_ERR_ARG, "gemm: ldc < N");
    if (K == 0 || alpha == 0.0f) {
        if (beta == 1.0f)
            return TTK_OK;
        const int64_t total = batch * M * N;
        const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 16);
        gemm::scale_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(C, batch, M, N, ldc,
                                                                         strideC, beta);
        return check_launch("scale_kernel");
    }
    if (M > (1ll << 31) / 2 || N > (1ll << 31) / 2 || K > (1ll << 31) / 2)
        return set_error(TTK_ERR_ARG, "gemm: dimension too large");
    if ((transA ? lda < M : lda < K) || (transB ? ldb < K : ldb < N))
        return set_error(TTK_ERR_ARG, "gemm: leading dimension too small");
    if (gemm_uses_fp32(batch, M, N, K)) {
        const dim3 grid(static_cast<unsigned>((N + gemm::F32_T - 1) / gemm::F32_T),
                        static_cast<unsigned>((M + gemm::F32_T - 1) / gemm::F32_T),
                        static_cast<unsigned>(batch));
        gemm::gemm_fp32_kernel<<<grid, 256, 0, stream>>>(transA, transB, M, N, K, alpha, A, lda,
                                                         strideA, B, ldb, strideB, beta, C, ldc,
                                                         strideC);
        return check_launch("gemm_fp32_kernel");
    }
    const int prec = current_prec();
    const GemmPlan pl = plan(prec, transA, transB, batch, M, N, K, allow_splitk);
    if (!ws || ws_bytes < pl.total)
        return set_error(TTK_ERR_ARG, "gemm: workspace too small");
    void* wa = ws;
    void* wb = static_cast<char*>(ws) + pl.off_b;
    if (prec == gemm::PREC_TF32X3) {
        int rc = launch_split<gemm::PREC_TF32X3>(A, pl.ga.rows, pl.ga.cols, lda, strideA, batch,
                                                 wa, pl.ga.ld_pad, stream);
        if (!rc)
            rc = launch_split<gemm::PREC_TF32X3>(B, pl.gb.rows, pl.gb.cols, ldb, strideB, batch,
                                                 wb, pl.gb.ld_pad, stream);
        if (rc)
            return rc;
        return run_presplit<gemm::PREC_TF32X3>(transA, transB, batch, M, N, K, alpha, wa,
                                               pl.ga.ld_pad, wb, pl.gb.ld_pad, beta, C, ldc,
                                               strideC, stream, pl.w_bytes ? 1 : 0,
                                               static_cast<char*>(ws) + pl.off_w,
                                               pl.w_bytes ? ws_bytes - pl.off_w : 0);
    }
    int rc = launch_split<gemm::PREC_BF16X3>(A, pl.ga.rows, pl.ga.cols, lda, strideA, batch, wa,
                                             pl.ga.ld_pad, stream);
    if (!rc)
        rc = launch_split<gemm::PREC_BF16X3>(B, pl.gb.rows, pl.gb.cols, ldb, strideB, batch, wb,
                                             pl.gb.ld_pad, stream);
    if (rc)
        return rc;
    return run_presplit<gemm::PREC_BF16X3>(transA, transB, batch, M, N, K, alpha, wa,
                                           pl.ga.ld_pad, wb, pl.gb.ld_pad, beta, C, ldc, strideC,
                                           stream, pl.w_bytes ? 1 : 0,
                                           static_cast<char*>(ws) + pl.off_w,
                                           pl.w_bytes ? ws_bytes - pl.off_w : 0);
}

// Caller-held operand splits in the current precision: [batch][2][rows][ld]
// with ld = cols rounded up to 32, which serves both K-major and MN-major use.
size_t gemm_split_bytes(int64_t batch, int64_t rows, int64_t cols) {
    if (batch <= 0 || rows <= 0 || cols <= 0)
        return 0;
    const int elt = current_prec() == gemm::PREC_TF32X3 ? 4 : 2;
    return static_cast<size_t>(batch) * 2 * rows * round_up(cols, 32) * elt;
}

int gemm_split(const float* src, int64_t rows, int64_t cols, int64_t ld, int64_t bstride,
               int64_t batch, void* dst, cudaStream_t stream) {
    if (rows < 0 || cols < 0 || batch < 0 || ld < cols)
        return set_error(TTK_ERR_ARG, "gemm_split: bad geometry");
    if (rows == 0 || cols == 0 || batch == 0)
        return TTK_OK;
    if (!src || !dst || (reinterpret_cast<uintptr_t>(dst) & 15))
        return set_error(TTK_ERR_ARG, "gemm_split: null or misaligned pointer");
    const int64_t ld_pad = round_up(cols, 32);
    if (current_prec() == gemm::PREC_TF32X3)
        return launch_split<gemm::PREC_TF32X3>(src, rows, cols, ld, bstride, batch, dst, ld_pad,
                                               stream);
    return launch_split<gemm::PREC_BF16X3>(src, rows, cols, ld, bstride, batch, dst, ld_pad,
                                           stream);
}

int gemm_on_splits(int transA, int transB, int64_t batch, int64_t M, int64_t N, int64_t K,
                   float alpha, const void* a_split, const void* b_split, float beta, float* C,
                   int64_t ldc, int64_t strideC, cudaStream_t stream) {
    if (M < 0 || N < 0 || K < 0 || batch < 0)
        return set_error(TTK_ERR_ARG, "gemm_on_splits: negative size");
    if (M == 0 || N == 0 || batch == 0)
        return TTK_OK;
    if (!C || (K > 0 && (!a_split || !b_split)))
        return set_error(TTK_ERR_ARG, "gemm_on_splits: null pointer");
    if (ldc < N)
        return set_error(TTK_ERR_ARG, "gemm_on_splits: ldc < N");
    if (K == 0 || alpha == 0.0f) {
        if (beta == 1.0f)
            return TTK_OK;
        const int64_t total = batch * M * N;
        const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 16);
        gemm::scale_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(C, batch, M, N, ldc,
                                                                         strideC, beta);
        return check_launch("scale_kernel");
    }
    if (M > (1ll << 31) / 2 || N > (1ll << 31) / 2 || K > (1ll << 31) / 2)
        return set_error(TTK_ERR_ARG, "gemm_on_splits: dimension too large");
    const int64_t lda_pad = round_up(transA ? M : K, 32);
    const int64_t ldb_pad = round_up(transB ? K : N, 32);
    if (current_prec() == gemm::PREC_TF32X3)
        return run_presplit<gemm::PREC_TF32X3>(transA, transB, batch, M, N, K, alpha, a_split,
                                               lda_pad, b_split, ldb_pad, beta, C, ldc, strideC,
                                               stream, 2);
    return run_presplit<gemm::PREC_BF16X3>(transA, transB, batch, M, N, K, alpha, a_split,
                                           lda_pad, b_split, ldb_pad, beta, C, ldc, strideC,
                                           stream, 2);
}

int gemm_tf32x3_presplit(int transA, int transB, int64_t batch, int64_t M, int64_t N, int64_t K,
                         float alpha, const float* a_split, int64_t lda_pad,
                         const float* b_split, int64_t ldb_pad, float beta, float* C,
                         int64_t ldc, int64_t strideC, cudaStream_t stream) {
    return run_presplit<gemm::PREC_TF32X3>(transA, transB, batch, M, N, K, alpha, a_split,
                                           lda_pad, b_split, ldb_pad, beta, C, ldc, strideC,
                                           stream);
}

}  // namespace ttk
