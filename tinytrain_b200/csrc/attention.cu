// Fused causal self-attention with RoPE, forward and backward: the C ABI.
//
// Replaces the attention block of GPTModel::forward (model.cpp:127-141):
// rope(q), rope(k) (ops.cpp:970-1052), the [B*H,T,T] score bmm, the scale
// and -1e9 mask (a masked score contributes exp(-1e9 - m) = 0 in fp32, the
// same as skipping it), softmax (ops.cpp:777-838) and the P.V bmm, with their
// backward rules. Scores never reach HBM.
//
// q, k, v, o: [B, T, H, HD] row-major (the Linear outputs' layout).
// cos/sin: [T, HD/2]. lse: [B, H, T].
//
// Engines (both on the bf16x3 operand split, attention_mma.cu):
//   0  tcgen05 kernels (attention_tc.cu) where the head dim allows, the
//      mma.sync kernels otherwise (default);
//   2  the mma.sync kernels only.
// Engine 1, a scalar fp32-FMA implementation, was removed: nothing used it.
#include <cuda_runtime.h>

#include <initializer_list>
#include <stdint.h>

#include <cstdlib>
#include <string>

#include "ttk_internal.h"

using namespace ttk;

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
// 0: tcgen05 where the head dim allows and mma.sync otherwise (default);
// 2: mma.sync only. TTK_ATTENTION=mma selects 2 at start-up.
int g_attn_impl = -1;
int attn_impl() {
    if (g_attn_impl < 0) {
        const char* e = std::getenv("TTK_ATTENTION");
        g_attn_impl = (e && std::string(e) == "mma") ? 2 : 0;
    }
    return g_attn_impl;
}
inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }
}  // namespace

extern "C" {

int ttk_attention_set_impl(int impl) {
    if (impl != 0 && impl != 2)
        return set_error(TTK_ERR_ARG,
                         "attention impl must be 0 (tcgen05 where the head dim allows) or 2 "
                         "(mma.sync); the fp32 FMA engine (1) was removed");
    g_attn_impl = impl;
    return TTK_OK;
}

int ttk_attention_get_impl(void) { return attn_impl(); }

size_t ttk_attention_fwd_workspace_size(int64_t B, int64_t T, int64_t H, int64_t hd) {
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
    if (!workspace || workspace_bytes < ttk_attention_fwd_workspace_size(B, T, H, hd))
        return set_error(TTK_ERR_ARG, "attention_fwd: workspace too small");
    rc = attn_align_check({q, k, v, cos_t, sin_t, o});
    if (rc)
        return rc;
    const bool tc = attn_impl() == 0 && attention_tc_supported(static_cast<int>(hd));
    return attention_mma_forward(static_cast<int>(hd), q, k, v, cos_t, sin_t, o, lse, B, T, H,
                                 scale, workspace, tc, S(stream));
}

int ttk_attention_fwd_split(const float* q, const float* k, const float* v, const float* cos_t,
                            const float* sin_t, float* o, float* lse, void* o_split, int64_t B,
                            int64_t T, int64_t H, int64_t hd, float scale, void* workspace,
                            size_t workspace_bytes, void* stream) {
    if (!o_split)
        return set_error(TTK_ERR_ARG, "attention_fwd_split: null o_split");
    if (ttk_gemm_get_precision() != 0)
        return set_error(TTK_ERR_ARG, "attention_fwd_split: planes exist for the bf16x3 precision");
    int rc = attn_check(q, k, v, cos_t, sin_t, B, T, H, hd);
    if (rc)
        return rc;
    if (!B || !T || !H)
        return TTK_OK;
    if (!o || !lse)
        return set_error(TTK_ERR_ARG, "attention_fwd: null output");
    if (!workspace || workspace_bytes < ttk_attention_fwd_workspace_size(B, T, H, hd))
        return set_error(TTK_ERR_ARG, "attention_fwd: workspace too small");
    rc = attn_align_check({q, k, v, cos_t, sin_t, o, o_split});
    if (rc)
        return rc;
    const bool tc = attn_impl() == 0 && attention_tc_supported(static_cast<int>(hd));
    return attention_mma_forward(static_cast<int>(hd), q, k, v, cos_t, sin_t, o, lse, B, T, H,
                                 scale, workspace, tc, S(stream), o_split);
}

size_t ttk_attention_bwd_workspace_size(int64_t B, int64_t T, int64_t H, int64_t hd) {
    const size_t dv = align256(static_cast<size_t>(B * T * H) * sizeof(float));
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
    rc = attn_align_check({q, k, v, cos_t, sin_t, o, dout, dq, dk, dv});
    if (rc)
        return rc;
    const bool tc = attn_impl() == 0 && attention_tc_supported(static_cast<int>(hd));
    return attention_mma_backward(static_cast<int>(hd), q, k, v, cos_t, sin_t, o, lse, dout, dq,
                                  dk, dv, accumulate, B, T, H, scale, workspace, tc, S(stream));
}

size_t ttk_attention_bwd_ex_workspace_size(int64_t B, int64_t T, int64_t H, int64_t hd) {
    const size_t dv = align256(static_cast<size_t>(B * T * H) * sizeof(float));
    // dO as bf16 hi|lo, then the (lse, D) table; q, k, v come from the forward
    return dv + static_cast<size_t>(B * T * H * hd) * 2 * 2 +
           align256(static_cast<size_t>(B * H * ((T + 31) / 32 * 32)) * 8);
}

int ttk_attention_bwd_ex(const float* q, const float* k, const float* v, const float* cos_t,
                         const float* sin_t, const float* o, const float* lse, const float* dout,
                         float* dq, float* dk, float* dv, int accumulate, int64_t B, int64_t T,
                         int64_t H, int64_t hd, float scale, const void* fwd_workspace,
                         void* workspace, size_t workspace_bytes, void* stream) {
    if (!fwd_workspace)
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

int ttk_attention_bwd_split(const float* q, const float* k, const float* v, const float* cos_t,
                            const float* sin_t, const float* o, const float* lse,
                            const float* dout, float* dq, float* dk, float* dv, int accumulate,
                            int64_t B, int64_t T, int64_t H, int64_t hd, float scale,
                            const void* fwd_workspace, void* workspace, size_t workspace_bytes,
                            void* dq_split, void* dk_split, void* dv_split, void* stream) {
    if (ttk_gemm_get_precision() != 0)
        return set_error(TTK_ERR_ARG, "attention_bwd_split: planes exist for the bf16x3 precision");
    int rc = attn_check(q, k, v, cos_t, sin_t, B, T, H, hd);
    if (rc)
        return rc;
    if (!B || !T || !H)
        return TTK_OK;
    if (!o || !lse || !dout || !dq || !dk || !dv)
        return set_error(TTK_ERR_ARG, "attention_bwd: null pointer");
    const size_t need = fwd_workspace ? ttk_attention_bwd_ex_workspace_size(B, T, H, hd)
                                      : ttk_attention_bwd_workspace_size(B, T, H, hd);
    if (!workspace || workspace_bytes < need)
        return set_error(TTK_ERR_ARG, "attention_bwd: workspace too small");
    rc = attn_align_check({q, k, v, cos_t, sin_t, o, dout, dq, dk, dv, fwd_workspace, dq_split,
                           dk_split, dv_split});
    if (rc)
        return rc;
    const bool tc = attn_impl() == 0 && attention_tc_supported(static_cast<int>(hd));
    return attention_mma_backward(static_cast<int>(hd), q, k, v, cos_t, sin_t, o, lse, dout, dq,
                                  dk, dv, accumulate, B, T, H, scale, workspace, tc,
                                  S(stream), fwd_workspace, dq_split, dk_split, dv_split);
}

}  // extern "C"
