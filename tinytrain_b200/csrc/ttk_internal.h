// Host-side internals shared by the ttk translation units.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <algorithm>

#include "ttk.h"

namespace ttk {

// Records a message for ttk_last_error() and returns the code.
int set_error(int code, const char* msg);
// Converts a pending launch error into a status.
int check_launch(const char* what);
int check_cuda(cudaError_t e, const char* what);
const char* last_error_cstr();

// cuTensorMapEncodeTiled, resolved once through the runtime's driver entry
// point query (null if unavailable).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn();

inline int grid_for(int64_t n, int threads, int max_blocks = 148 * 16) {
    int64_t b = (n + threads - 1) / threads;
    if (b < 1)
        b = 1;
    return static_cast<int>(std::min<int64_t>(b, max_blocks));
}

// GEMM entry points (gemm_split3.cu), shared with the C ABI wrappers.
int gemm_profile_enable(int on);
int gemm_profile_read(double* ms, double* flops, int64_t* launches);
// allow_splitk: include (and use) split-K partials in the workspace.
size_t gemm_workspace_size(int transA, int transB, int64_t batch, int64_t M, int64_t N,
                           int64_t K, bool allow_splitk = true);
int split_tf32(const float* src, int64_t rows, int64_t cols, int64_t ld, int64_t bstride,
               int64_t batch, float* dst, int64_t ld_pad, cudaStream_t stream);
int gemm_set_precision(int prec);
int gemm_get_precision();
int gemm_set_cta_pairs(int mode);
int gemm_get_cta_pairs();
int gemm_set_split_k(int on);
int gemm_get_split_k();
int gemm_split_k_slices(int transA, int transB, int64_t batch, int64_t M, int64_t N, int64_t K);
int gemm_set_fp32_max_macs(int64_t macs);
int64_t gemm_fp32_max_macs();
bool gemm_uses_fp32(int64_t batch, int64_t M, int64_t N, int64_t K);
int gemm_run(int transA, int transB, int64_t batch, int64_t M, int64_t N, int64_t K, float alpha,
             const float* A, int64_t lda, int64_t strideA, const float* B, int64_t ldb,
             int64_t strideB, float beta, float* C, int64_t ldc, int64_t strideC, void* ws,
             size_t ws_bytes, cudaStream_t stream, bool allow_splitk = true);
size_t gemm_split_bytes(int64_t batch, int64_t rows, int64_t cols);
int gemm_split(const float* src, int64_t rows, int64_t cols, int64_t ld, int64_t bstride,
               int64_t batch, void* dst, cudaStream_t stream);
int gemm_on_splits(int transA, int transB, int64_t batch, int64_t M, int64_t N, int64_t K,
                   float alpha, const void* a_split, const void* b_split, float beta, float* C,
                   int64_t ldc, int64_t strideC, cudaStream_t stream);
int gemm_tf32x3_presplit(int transA, int transB, int64_t batch, int64_t M, int64_t N, int64_t K,
                         float alpha, const float* a_split, int64_t lda_pad,
                         const float* b_split, int64_t ldb_pad, float beta, float* C,
                         int64_t ldc, int64_t strideC, cudaStream_t stream);

// Tensor-core attention (attention_mma.cu); ws sized by the C ABI's
// workspace functions.
// o_split (optional): bf16x3 GEMM operand planes of o as [B*T, H*hd] rows
// (the ttk_gemm_split layout), written by the tcgen05 epilogue or, for the
// mma.sync engine, by a split pass after it.
int attention_mma_forward(int hd, const float* q, const float* k, const float* v,
                          const float* cs, const float* sn, float* o, float* lse, int64_t B,
                          int64_t T, int64_t H, float scale, void* ws, bool tc,
                          cudaStream_t st, void* o_split = nullptr);
// d*_split (optional, each): bf16x3 operand planes of dq / dk / dv as
// [B*T, H*hd] rows, written by the tcgen05 epilogues or by split passes.
int attention_mma_backward(int hd, const float* q, const float* k, const float* v,
                           const float* cs, const float* sn, const float* o, const float* lse,
                           const float* dout, float* dq, float* dk, float* dv, int accumulate,
                           int64_t B, int64_t T, int64_t H, float scale, void* ws, bool tc,
                           cudaStream_t st, const void* fwd_ws = nullptr,
                           void* dq_split = nullptr, void* dk_split = nullptr,
                           void* dv_split = nullptr);

// tcgen05 attention forward / backward (attention_tc.cu) over split planes
// written by the mma.sync path's split pass; head dims 32, 64 and 128.
bool attention_tc_supported(int hd);
int attention_tc_forward_core(int hd, const __nv_bfloat16* qh, const __nv_bfloat16* kh,
                              const __nv_bfloat16* vh, float* o, float* lse, int64_t B, int64_t T,
                              int64_t H, cudaStream_t st, __nv_bfloat16* o_split = nullptr);
// ld: [B*H][T32][2] table of (lse * log2 e, D), T32 = T rounded up to 32,
// zero in the padding rows.
int attention_tc_backward_core(int hd, const __nv_bfloat16* qh, const __nv_bfloat16* kh,
                               const __nv_bfloat16* vh, const __nv_bfloat16* dh,
                               const float* lse, const float* Dv, const float* ld, int64_t T32,
                               const float* cs, const float* sn, float* dq, float* dk, float* dv,
                               int accumulate, int64_t B, int64_t T, int64_t H, float scale,
                               cudaStream_t st, __nv_bfloat16* dq_split = nullptr,
                               __nv_bfloat16* dk_split = nullptr,
                               __nv_bfloat16* dv_split = nullptr);

}  // namespace ttk
