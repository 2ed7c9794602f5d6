/* ttk: the C ABI of the B200 (sm_100a) kernel layer under tinytrain's
 * Tensor / ops / nn / optim API.
 *
 * Plain pointers and sizes only. Every float* / int64_t* argument named as a
 * tensor is DEVICE memory; `stream` is a cudaStream_t passed as void* (NULL =
 * the legacy default stream). Every function returns TTK_OK (0) or a
 * TTK_ERR_* code; ttk_last_error() gives the message of the last failure on
 * the calling thread. Argument checks mirror the reference's
 * std::invalid_argument throws and run before any launch.
 *
 * Tensors are row-major fp32 (the reference's only dtype, tensor.h:25).
 * "accumulate" flags select out += result (the reference's grad +=
 * semantics, ops.cpp:12-15) instead of out = result.
 *
 * The reference (seampm/tinytrain) has no FFI; each entry point names the
 * reference function whose arithmetic it replaces.
 */
#ifndef TTK_H
#define TTK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TTK_OK 0
#define TTK_ERR_ARG 1     /* invalid argument (shape, range, null, alignment) */
#define TTK_ERR_CUDA 2    /* CUDA runtime / driver failure */
#define TTK_ERR_NCCL 3    /* collective library failure */
#define TTK_ERR_DEVICE 4  /* a kernel reported an error through the status word */

/* ------------------------------------------------------------------ runtime */

const char* ttk_last_error(void);
const char* ttk_version(void);
/* Sets the calling thread's device and creates its stream-ordered memory pool. */
int ttk_init(int device);
int ttk_device_count(int* n);
/* The calling thread's current device (the one another runtime in the
 * process, e.g. torch.cuda.set_device, made current; 0 by default). */
int ttk_current_device(int* device);
/* Reads and clears the device status word (bit 0: a bounded wait expired,
 * bit 1: an out-of-range index was skipped). Synchronizes the device. */
int ttk_device_status(unsigned* bits);
int ttk_synchronize(void);
/* Failure-path self test, no counterpart in the reference (whose CPU code has
 * no device waits): one thread waits on an mbarrier that nothing arrives on,
 * through the bounded wait every pipeline kernel here uses, with a limit of
 * limit_ns (at most the pipelines' 2 s). The kernel gives up, sets bit 0 of
 * the device status word and the wait site (bits 8..15), and returns; the
 * context stays usable. */
int ttk_selftest_wait_timeout(unsigned site, uint64_t limit_ns, void* stream);
/* Number of kernels launched through this library so far (all streams). */
int64_t ttk_launch_count(void);

/* Stream-ordered allocation from the device's pool (cached, never released to
 * the driver until exit). The caching allocator under tt::Tensor storage. */
int ttk_malloc(void** ptr, size_t bytes, void* stream);
int ttk_free(void* ptr, void* stream);
int ttk_pool_stats(size_t* reserved, size_t* used);
/* High-water marks of the device pool's reserved and used bytes since the
 * last reset (reset != 0 resets them after reading). */
int ttk_pool_high_water(size_t* reserved_high, size_t* used_high, int reset);
int ttk_host_alloc(void** ptr, size_t bytes); /* pinned host memory */
int ttk_host_free(void* ptr);

int ttk_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream);
int ttk_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream);
/* Stream-ordered device-to-host copy that returns without waiting (dst
 * pinned for the copy to be asynchronous); ttk_memcpy_d2h waits for it. */
int ttk_memcpy_d2h_async(void* dst, const void* src, size_t bytes, void* stream);
int ttk_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream);
int ttk_memset(void* dst, int value, size_t bytes, void* stream);

int ttk_stream_create(void** stream);
int ttk_stream_destroy(void* stream);
int ttk_stream_synchronize(void* stream);
int ttk_event_create(void** event);
int ttk_event_destroy(void* event);
int ttk_event_record(void* event, void* stream);
int ttk_stream_wait_event(void* stream, void* event);
int ttk_event_elapsed_ms(void* start, void* end, float* ms);
int ttk_event_synchronize(void* event);
/* *done = 1 when the work before the event's record has completed, else 0;
 * never blocks. */
int ttk_event_query(void* event, int* done);

/* CUDA graphs (no counterpart in the reference, which has no device):
 * ttk_stream_begin_capture starts recording `stream` (not the legacy default
 * stream) in thread-local mode; ttk_stream_end_capture ends it and returns an
 * instantiated graph (memory the graph allocates and leaves allocated is
 * freed at its next launch); ttk_graph_launch replays it on any stream;
 * ttk_graph_destroy releases it. ttk_pool_trim waits for `stream` and
 * returns the device pool's unused memory to the device. */
int ttk_stream_begin_capture(void* stream);
int ttk_stream_end_capture(void* stream, void** graph_exec);
int ttk_graph_launch(void* graph_exec, void* stream);
int ttk_graph_destroy(void* graph_exec);
int ttk_pool_trim(void* stream);
/* Host-side cache of freed device blocks over the pool (on != 0; off by
 * default): a block that ttk_free returns on a stream is handed out again by
 * a later ttk_malloc of the same size on the same device and stream (stream
 * order makes the reuse safe), so a training loop's repeating pattern of
 * allocations stops reaching the pool. Allocations made while a stream is
 * being captured into a graph bypass it; when a ttk_malloc finds the device
 * out of memory the cached blocks are returned to the pool and it retries;
 * ttk_pool_trim and turning the cache off return them too. No counterpart in
 * the reference. */
int ttk_set_block_cache(int on);

/* ------------------------------------------------------------ dense algebra */

/* C[b] = alpha * op(A[b]) @ op(B[b]) + beta * C[b] on the tcgen05 tensor
 * cores, fp32-accurate through a three-term operand split (see
 * ttk_gemm_set_precision). op(A) is A [M,K] (lda) when transA = 0, or A^T with A stored
 * [K,M] when transA = 1; op(B) is B [K,N] (ldb) when transB = 0, or B^T with B
 * stored [N,K] when transB = 1. stride* are the batch strides (elements).
 * `workspace` (device, 16-byte aligned) holds the split operands and must be
 * at least ttk_gemm_workspace_size(...) bytes.
 * Replaces: sgemm + matmul fwd/bwd (ops.cpp:96-125, 661-697) and bmm
 * (ops.cpp:699-742). */
/* Split used by ttk_gemm (process-wide): 0 = bf16x3 (default; hi/lo bf16
 * halves, three kind::f16 MMAs, ~4e-6 normalized error), 1 = tf32x3 (hi/lo
 * TF32, three kind::tf32 MMAs, twice the tensor time). The environment
 * variable TTK_GEMM_PRECISION=tf32x3 selects 1 at start-up. Workspace sizes
 * depend on the choice. */
int ttk_gemm_set_precision(int prec);
int ttk_gemm_get_precision(void);
/* Large bf16-split problems run 256 x 256 tiles on CTA pairs (clusters of two
 * SMs sharing one M = 256 tcgen05 MMA; each SM loads half the operand tiles
 * of a 128 x 256 tile). Mode 1 (default): pairs when N > 128 and the 256 x 256
 * tiles occupy every resident pair; 0: single-CTA tiles only; 2: pairs
 * whenever N > 128. TTK_GEMM_PAIRS=0|1|2 selects the mode at start-up. */
int ttk_gemm_set_cta_pairs(int mode);
int ttk_gemm_get_cta_pairs(void);
/* Split-K (default on; TTK_GEMM_SPLITK=0 turns it off at start-up): a single
 * GEMM with a long K whose output tiles would leave many SMs idle in the last
 * wave (the weight gradients dY^T X: M x N small against K = tokens) runs as
 * S K-slices that write partial products, then one pass sums them in slice
 * order (deterministic) into alpha * sum + beta * C. ttk_gemm_workspace_size
 * includes the partials; ttk_gemm_noalloc never splits. ttk_gemm_split_k_slices
 * reports S for one problem (1 = not split). */
int ttk_gemm_set_split_k(int on);
int ttk_gemm_get_split_k(void);
int ttk_gemm_split_k_slices(int transA, int transB, int64_t batch, int64_t M, int64_t N,
                            int64_t K);
/* Problems of at most `macs` multiply-adds (batch*M*N*K; default 2^24) run
 * as an exact fp32 SIMT GEMM, one fused multiply-add per product in
 * ascending k, with no workspace: below that size the split's extra launches
 * cost more than the products, and the result carries no split truncation
 * (finite-difference gradient checks, as in the reference's
 * tests/test_autograd.cpp, rely on that). 0 sends every size to the tensor
 * cores. ttk_gemm_uses_fp32 reports the choice for one problem. */
int ttk_gemm_set_fp32_max_macs(int64_t macs);
int64_t ttk_gemm_get_fp32_max_macs(void);
int ttk_gemm_uses_fp32(int64_t batch, int64_t M, int64_t N, int64_t K);
size_t ttk_gemm_workspace_size(int transA, int transB, int64_t batch, int64_t M, int64_t N,
                               int64_t K);
int ttk_gemm(int transA, int transB, int64_t batch, int64_t M, int64_t N, int64_t K, float alpha,
             const float* A, int64_t lda, int64_t strideA, const float* B, int64_t ldb,
             int64_t strideB, float beta, float* C, int64_t ldc, int64_t strideC,
             void* workspace, size_t workspace_bytes, void* stream);
/* ttk_gemm without a workspace argument, for callers that cannot allocate
 * device memory: code running under another framework's fixed memory budget,
 * paths that must not fail with out-of-memory after start-up, or host
 * programs that own only their input and output buffers. No counterpart in
 * the reference (its CPU sgemm needs no device scratch).
 * The split operands go to a fixed scratch array compiled into libttk.so
 * (ttk_gemm_noalloc_max_workspace() bytes, 32 MiB, held by every GPU that
 * loads the library until exit); operands needing more scratch than that
 * (see ttk_gemm_workspace_size) are rejected with TTK_ERR_ARG. No memory is
 * allocated. The first call on each device looks up the array's device
 * address; make that first call before any stream capture. All calls share
 * the one array, so calls that overlap on the GPU (different streams, or
 * different host threads, without ordering between them) race on it; the
 * caller must serialize them. The looked-up address is cached for the life
 * of the process: do not call it on a device after cudaDeviceReset there.
 * Inputs and outputs are as for ttk_gemm. */
size_t ttk_gemm_noalloc_max_workspace(void);
int ttk_gemm_noalloc(int transA, int transB, int64_t batch, int64_t M, int64_t N, int64_t K,
                     float alpha, const float* A, int64_t lda, int64_t strideA, const float* B,
                     int64_t ldb, int64_t strideB, float beta, float* C, int64_t ldc,
                     int64_t strideC, void* stream);
/* Operand splits that a caller keeps and reuses across the GEMMs reading the
 * same tensor (matmul forward, dA and dB of ops.cpp:661-697 read each operand
 * twice; weights are read by every micro-batch until the optimizer writes
 * them). In the current precision (bf16 planes for bf16x3, fp32 for tf32x3),
 * layout [batch][hi|lo][rows][round_up(cols, 32)]: one split serves K-major
 * and MN-major reads alike. ttk_gemm_split writes the split of src
 * [batch][rows][cols] (leading dimension ld, batch stride bstride) into dst
 * (16-byte aligned, ttk_gemm_split_bytes long); ttk_gemm_splits runs
 * C = alpha op(A) op(B) + beta C on two splits holding op(A)'s storage
 * (transA ? [K,M] : [M,K]) and op(B)'s (transB ? [N,K] : [K,N]). A split is
 * valid only for the precision it was made in. */
size_t ttk_gemm_split_bytes(int64_t batch, int64_t rows, int64_t cols);
int ttk_gemm_split(const float* src, int64_t rows, int64_t cols, int64_t ld, int64_t bstride,
                   int64_t batch, void* dst, void* stream);
int ttk_gemm_splits(int transA, int transB, int64_t batch, int64_t M, int64_t N, int64_t K,
                    float alpha, const void* a_split, const void* b_split, float beta, float* C,
                    int64_t ldc, int64_t strideC, void* stream);

/* The operand split alone: dst[b][0|1][r][0..ld_pad) = hi | lo of
 * src[b][r][0..cols) (ld, batch stride bstride), zero in [cols, ld_pad).
 * ld_pad must be a multiple of 16 (32 for an operand read MN-major by
 * ttk_gemm_presplit: A with transA = 1, B with transB = 0). */
int ttk_split_tf32(const float* src, int64_t rows, int64_t cols, int64_t ld, int64_t bstride,
                   int64_t batch, float* dst, int64_t ld_pad, void* stream);
/* GEMM on operands already split by ttk_split_tf32 (TF32 planes, always the
 * tf32x3 kernel; e.g. weights split once per optimizer step). a_split holds op(A)'s storage ([M,K] or [K,M]) with
 * padded leading dimension lda_pad, likewise b_split. */
int ttk_gemm_presplit(int transA, int transB, int64_t batch, int64_t M, int64_t N, int64_t K,
                      float alpha, const float* a_split, int64_t lda_pad, const float* b_split,
                      int64_t ldb_pad, float beta, float* C, int64_t ldc, int64_t strideC,
                      void* stream);

/* Live timing of the tcgen05 GEMM kernel on the calling thread: when enabled,
 * each launch is bracketed by CUDA events on its stream; ttk_profile_read
 * synchronizes, returns the summed kernel time (ms), the summed algorithmic
 * FLOPs (2*M*N*K per GEMM) and the launch count since the last read, and
 * resets them. Off by default. */
int ttk_profile_enable(int on);
int ttk_profile_read(double* gemm_ms, double* gemm_flops, int64_t* launches);

/* ------------------------------------------------------------ fused NN ops */

/* y = x * rstd * w, rstd = (mean(x^2) + eps)^-1/2 per row; x, y [R,D], w [D],
 * rstd [R] (saved for the backward). Replaces the 7-op composite rmsnorm
 * (ops.cpp:932-942). */
int ttk_rmsnorm_fwd(const float* x, const float* w, float* y, float* rstd, int64_t R, int64_t D,
                    float eps, void* stream);
/* ttk_rmsnorm_fwd that also writes the bf16x3 GEMM operand planes of y into
 * `split` (ttk_gemm_split_bytes(1, R, D) bytes, the ttk_gemm_split layout),
 * equal bit for bit to ttk_gemm_split(y, R, D, D, 0, 1, split): the split
 * pass before the GEMMs that read y (the q/k/v, gate/up and LM-head
 * projections of the model) is saved. D a multiple of 256, the bf16x3
 * precision; no counterpart in the reference. */
int ttk_rmsnorm_fwd_split(const float* x, const float* w, float* y, float* rstd, int64_t R,
                          int64_t D, float eps, void* split, void* stream);
/* dx (+)= rstd*w*dy - x*rstd^3/D*sum(dy*w*x); dw += sum_rows(dy*x*rstd).
 * dx may be NULL. dw (when not NULL) is always accumulated; `workspace`
 * (device) must hold ttk_rmsnorm_bwd_workspace_size(R, D) bytes. */
size_t ttk_rmsnorm_bwd_workspace_size(int64_t R, int64_t D);
int ttk_rmsnorm_bwd(const float* x, const float* w, const float* rstd, const float* dy, float* dx,
                    int accumulate_dx, float* dw, int64_t R, int64_t D, void* workspace,
                    size_t workspace_bytes, void* stream);

/* y = silu(a) * b (model.cpp:149-151, ops.cpp:324); n elements. */
int ttk_swiglu_fwd(const float* a, const float* b, float* y, int64_t n, void* stream);
/* da (+)= dy*b*s*(1+a*(1-s)), db (+)= dy*silu(a) (ops.cpp:325-328, :256). */
int ttk_swiglu_bwd(const float* a, const float* b, const float* dy, float* da, float* db,
                   int accumulate, int64_t n, void* stream);
/* SwiGLU forward / backward producing their results only as bf16x3 GEMM
 * operand planes in the layout of ttk_gemm_split ([2][R][round_up(F, 32)]
 * bf16, hi then lo, padding zero), for a projection GEMM that consumes them
 * through ttk_gemm_splits: y = silu(a) * b, and da, db for dy, equal bit for
 * bit to ttk_swiglu_fwd / ttk_swiglu_bwd followed by ttk_gemm_split, without
 * the fp32 tensors. a, b, dy are [R, F] row-major with F % 4 == 0; requires
 * the bf16x3 precision. */
int ttk_swiglu_fwd_split(const float* a, const float* b, void* y_split, int64_t R, int64_t F,
                         void* stream);
int ttk_swiglu_bwd_split(const float* a, const float* b, const float* dy, void* da_split,
                         void* db_split, int64_t R, int64_t F, void* stream);

/* Fused log_softmax + nll_loss (ops.cpp:840-930) over logits [N,C]:
 * loss_sum[0] (+)= sum_i (lse_i - x[i,t_i]) accumulated in fp64 into
 * loss_acc (device double), and, when dlogits is not NULL,
 * dlogits = grad_scale * (softmax(x) - onehot(t)) (dlogits may alias logits).
 * Targets out of [0, C) are rejected before launch. */
int ttk_cross_entropy(const float* logits, const int64_t* targets, int64_t N, int64_t C,
                      double* loss_acc, float* dlogits, float grad_scale, void* stream);
/* loss_out[0] = (float)(loss_acc[0] * scale) (the mean of ops.cpp:911-912). */
int ttk_loss_finalize(const double* loss_acc, float scale, float* loss_out, void* stream);

/* Causal self-attention with RoPE, fused (model.cpp:127-141: rope(q), rope(k),
 * softmax(q k^T * scale + causal mask) v). q, k, v, o are [B,T,H,hd] (the
 * layout the projections produce; o is ready for the output projection);
 * cos/sin [T, hd/2] are the model's RoPE tables (model.cpp:43-53); lse
 * [B,H,T] is saved for the backward. hd in {32, 64, 128}. `workspace` must
 * hold ttk_attention_fwd_workspace_size(B,T,H,hd) bytes (the split
 * operands). */
size_t ttk_attention_fwd_workspace_size(int64_t B, int64_t T, int64_t H, int64_t hd);
int ttk_attention_fwd(const float* q, const float* k, const float* v, const float* cos_t,
                      const float* sin_t, float* o, float* lse, int64_t B, int64_t T, int64_t H,
                      int64_t hd, float scale, void* workspace, size_t workspace_bytes,
                      void* stream);
/* ttk_attention_fwd that also writes the bf16x3 GEMM operand planes of o,
 * viewed as [B*T, H*hd] rows, into o_split (ttk_gemm_split_bytes(1, B*T,
 * H*hd) bytes): equal bit for bit to ttk_gemm_split of o, so the output
 * projection skips its split pass. bf16x3 precision only; no counterpart in
 * the reference. */
int ttk_attention_fwd_split(const float* q, const float* k, const float* v, const float* cos_t,
                            const float* sin_t, float* o, float* lse, void* o_split, int64_t B,
                            int64_t T, int64_t H, int64_t hd, float scale, void* workspace,
                            size_t workspace_bytes, void* stream);
/* dq, dk, dv (+)= gradients w.r.t. the pre-RoPE q, k and v. `workspace` must
 * hold ttk_attention_bwd_workspace_size(B,T,H,hd) bytes. */
size_t ttk_attention_bwd_workspace_size(int64_t B, int64_t T, int64_t H, int64_t hd);
int ttk_attention_bwd(const float* q, const float* k, const float* v, const float* cos_t,
                      const float* sin_t, const float* o, const float* lse, const float* dout,
                      float* dq, float* dk, float* dv, int accumulate, int64_t B, int64_t T,
                      int64_t H, int64_t hd, float scale, void* workspace,
                      size_t workspace_bytes, void* stream);
/* ttk_attention_bwd reusing the forward's operand planes: fwd_workspace is
 * the workspace of the ttk_attention_fwd call that produced o and lse (same
 * q, k, v, tables, scale and engine, and q, k, v unchanged since), kept by the
 * caller. Only dO is split here, and `workspace` needs only
 * ttk_attention_bwd_ex_workspace_size bytes. A null fwd_workspace (or the
 * FMA engine, whose forward keeps no planes) runs ttk_attention_bwd. */
size_t ttk_attention_bwd_ex_workspace_size(int64_t B, int64_t T, int64_t H, int64_t hd);
int ttk_attention_bwd_ex(const float* q, const float* k, const float* v, const float* cos_t,
                         const float* sin_t, const float* o, const float* lse, const float* dout,
                         float* dq, float* dk, float* dv, int accumulate, int64_t B, int64_t T,
                         int64_t H, int64_t hd, float scale, const void* fwd_workspace,
                         void* workspace, size_t workspace_bytes, void* stream);
/* ttk_attention_bwd_ex (fwd_workspace may be NULL: then as ttk_attention_bwd,
 * with its workspace size) that also writes the bf16x3 GEMM operand planes of
 * dq, dk and dv, each viewed as [B*T, H*hd] rows, into dq_split / dk_split /
 * dv_split (each NULL or ttk_gemm_split_bytes(1, B*T, H*hd) bytes): equal bit
 * for bit to ttk_gemm_split of the stored gradients (after accumulation), so
 * the q/k/v projections' backward GEMMs skip their split passes. bf16x3
 * precision only; no counterpart in the reference. */
int ttk_attention_bwd_split(const float* q, const float* k, const float* v, const float* cos_t,
                            const float* sin_t, const float* o, const float* lse,
                            const float* dout, float* dq, float* dk, float* dv, int accumulate,
                            int64_t B, int64_t T, int64_t H, int64_t hd, float scale,
                            const void* fwd_workspace, void* workspace, size_t workspace_bytes,
                            void* dq_split, void* dk_split, void* dv_split, void* stream);
/* Attention engine (process-wide), all fp32-accurate:
 *   0 = tensor cores (default): tcgen05 forward and backward for head dims
 *       32, 64 and 128, mma.sync m16n8k16 elsewhere, both with the bf16x3
 *       operand split;
 *   2 = mma.sync m16n8k16 kernels only.
 * Engine 1 (scalar fp32 FMA kernels) was removed; asking for it fails with
 * TTK_ERR_ARG. The environment variable TTK_ATTENTION=mma selects 2 at
 * start-up. Workspace sizes depend on the choice. */
int ttk_attention_set_impl(int impl);
int ttk_attention_get_impl(void);

/* out[i,:] = W[idx[i],:] (ops.cpp:746-759); idx validated against V. */
int ttk_embedding_fwd(const float* W, const int64_t* idx, float* out, int64_t N, int64_t D,
                      int64_t V, void* stream);
/* dW[idx[i],:] += dout[i,:] in ascending i per row, deterministic and
 * bit-identical to the reference's sequential loop (ops.cpp:761-772).
 * `workspace` must hold ttk_embedding_bwd_workspace_size(N) bytes. */
size_t ttk_embedding_bwd_workspace_size(int64_t N);
int ttk_embedding_bwd(const float* dout, const int64_t* idx, float* dW, int64_t N, int64_t D,
                      int64_t V, void* workspace, size_t workspace_bytes, void* stream);
/* Range check of ids on the device: *bad = number of ids outside [0, V). */
int ttk_index_check(const int64_t* idx, int64_t n, int64_t V, int64_t* bad_host, void* stream);

/* RoPE on x [B,T,H,D] with cos/sin [T,D/2] (ops.cpp:970-999) and its
 * transpose rotation for the backward (ops.cpp:1011-1023). */
int ttk_rope_fwd(const float* x, const float* cos_t, const float* sin_t, float* y, int64_t B,
                 int64_t T, int64_t H, int64_t D, void* stream);
int ttk_rope_bwd(const float* dy, const float* cos_t, const float* sin_t, float* dx,
                 int accumulate, int64_t B, int64_t T, int64_t H, int64_t D, void* stream);

/* The reference's dropout mask (ops.cpp:944-968): mask[i] = 1.0f when the
 * (i+1)-th output r of its xorshift64* stream (seed 0 -> 0x9E3779B97F4A7C15)
 * gives (r >> 11) * 2^-53 >= p, else 0.0f; bit-identical to the sequential
 * loop at any n (each thread jumps ahead to its chunk of the stream). */
int ttk_dropout_mask(float* mask, int64_t n, float p, uint64_t seed, void* stream);

/* Training windows from a device-resident int32 token stream
 * (apps/train.cpp:225-232): for w < count, idx[w*T + t] = tokens[starts[w] + t]
 * and targets[w*T + t] = tokens[starts[w] + t + 1], widened to int64. starts
 * (device) must satisfy starts[w] + T < token count (checked by the caller). */
int ttk_gather_windows(const int32_t* tokens, const int64_t* starts, int64_t count, int64_t T,
                       int64_t* idx, int64_t* targets, void* stream);

/* nll_loss over log-probabilities [N,C] (ops.cpp:898-926): *loss =
 * -sum_i lp[i,t_i] / N (fp64, i ascending); backward dlp[i,t_i] -= g[0]/N with
 * the upstream gradient g read on the device. */
int ttk_nll_fwd(const float* lp, const int64_t* targets, int64_t N, int64_t C, float* loss,
                void* stream);
int ttk_nll_bwd(const int64_t* targets, int64_t N, int64_t C, const float* g, float* dlp,
                void* stream);
/* Gradients of the RoPE tables (ops.cpp:1024-1048): dcos/dsin [T,D/2] +=
 * sums over b, h (either may be NULL). */
int ttk_rope_table_grad(const float* x, const float* dy, int64_t B, int64_t T, int64_t H,
                        int64_t D, float* dcos, float* dsin, void* stream);

/* Row softmax / log-softmax over the last dim of [R,C] (ops.cpp:777-896);
 * backward: dx (+)= y*(dy - sum(dy*y)) resp. dy - exp(y)*sum(dy). */
int ttk_softmax_fwd(const float* x, float* y, int64_t R, int64_t C, int log, void* stream);
int ttk_softmax_bwd(const float* y, const float* dy, float* dx, int accumulate, int64_t R,
                    int64_t C, int log, void* stream);

/* --------------------------------------------------------------- optimizer */

/* Sum of squares of a list of tensors, accumulated in fp64 into *acc
 * (device double); the global grad norm for clipping. */
int ttk_sumsq_multi(const float* const* ptrs, const int64_t* sizes, int n_tensors, double* acc,
                    void* stream);
/* One fused AdamW step over a list of tensors (optim.cpp:17-48: decoupled
 * decay with lr before the moments, bias correction folded into lr_t, eps on
 * the uncorrected sqrt(v)), with global-norm clipping folded in: the gradient
 * is multiplied by min(1, max_norm / (sqrt(*sumsq) + 1e-6)) read on the
 * device (max_norm <= 0 disables it) and by grad_scale (e.g. 1/world for an
 * all-reduced sum). step is the 1-based step count. */
int ttk_adamw_multi(float* const* params, const float* const* grads, float* const* m,
                    float* const* v, const int64_t* sizes, int n_tensors, float lr, float beta1,
                    float beta2, float eps, float weight_decay, int64_t step,
                    const double* sumsq, float max_norm, float grad_scale, void* stream);
/* The same step taking the learning rate and the bias-corrected rate from
 * the device (sched = {lr, lr_t}, read when the kernel starts), so a step
 * recorded once in a CUDA graph can be replayed with each step's values;
 * ttk_adamw_sched_set writes them for a 1-based step count (the arithmetic
 * of ttk_adamw_multi, so both give the same update). No counterpart in the
 * reference. */
int ttk_adamw_multi_sched(float* const* params, const float* const* grads, float* const* m,
                          float* const* v, const int64_t* sizes, int n_tensors, float beta1,
                          float beta2, float eps, float weight_decay, const float* sched,
                          const double* sumsq, float max_norm, float grad_scale, void* stream);
int ttk_adamw_sched_set(float* sched, float lr, float beta1, float beta2, int64_t step,
                        void* stream);
/* SGD with momentum / L2 decay (optim.cpp:58-82) on one tensor. */
int ttk_sgd(float* p, const float* g, float* vel, int64_t n, float lr, float momentum,
            float weight_decay, void* stream);

/* -------------------------------------------------- generic tensor kernels */

/* Elementwise ops on up-to-8-D broadcast views. shape[] is the output shape;
 * a_strides / b_strides are element strides of each input expressed in the
 * output's index space (0 on broadcast dims). Binary ops: 0 add, 1 sub,
 * 2 mul, 3 div (ops.cpp:139-266). */
#define TTK_MAX_DIMS 8
int ttk_binary(int op, const float* a, const int64_t* a_strides, const float* b,
               const int64_t* b_strides, float* out, const int64_t* shape, int ndim,
               void* stream);
/* Gradient of a binary op w.r.t. one input, accumulated into grad (which has
 * the output's shape when `reduce` is 0). which = 0: d/da, 1: d/db. */
int ttk_binary_bwd(int op, int which, const float* a, const int64_t* a_strides, const float* b,
                   const int64_t* b_strides, const float* dout, float* g_full,
                   const int64_t* shape, int ndim, void* stream);
/* Unary ops: 0 neg, 1 exp, 2 log, 3 sqrt, 4 tanh, 5 silu, 6 sin, 7 cos,
 * 8 pow(p) (ops.cpp:268-363); y = f(x). */
int ttk_unary(int op, const float* x, float* y, int64_t n, float p, void* stream);
/* dx += dy * f'(x) (the b_* rules of ops.cpp:314-363; always accumulates,
 * like the reference's backward closures). */
int ttk_unary_bwd(int op, const float* x, const float* dy, float* dx, int64_t n, float p,
                  void* stream);
/* out[o, i] (+)= sum_k in[o, k, i] over [outer, K, inner] (ops.cpp:367-439 sum). */
int ttk_reduce_mid(const float* in, float* out, int64_t outer, int64_t K, int64_t inner,
                   int accumulate, void* stream);
/* *out (+)= sum of n elements (fp64 accumulate, like ops.cpp:441-460). */
int ttk_sum_all(const float* in, int64_t n, float* out, int accumulate, void* stream);
/* out = in viewed through (shape, in_strides) made contiguous; accumulate
 * adds instead. Implements permute/transpose/expand copies
 * (ops.cpp:534-629). scatter_add = 1 performs the reverse: out[in_view] +=
 * in_contiguous (permute/expand backward). */
int ttk_strided_copy(const float* in, const int64_t* in_strides, float* out,
                     const int64_t* shape, int ndim, int accumulate, int scatter_add,
                     void* stream);
int ttk_fill(float* x, float v, int64_t n, void* stream);
/* y += alpha * x. */
int ttk_axpy(float alpha, const float* x, float* y, int64_t n, void* stream);
/* y (+)= alpha[0] * x with alpha a device scalar (an upstream gradient). */
int ttk_axpy_dev(const float* alpha, const float* x, float* y, int64_t n, int accumulate,
                 void* stream);
/* out[k] (+)= sum over the dims of `shape` whose bit is clear in keep_mask of
 * g[...] (g contiguous with shape `shape`; out contiguous over the kept
 * dims). The broadcast-gradient reduction (ops.cpp:35-61 bcast_add). */
int ttk_reduce_to(const float* g, const int64_t* shape, int ndim, unsigned keep_mask, float* out,
                  int accumulate, void* stream);

/* ---------------------------------------------------------------- training */

/* Counter-based N(0, std) init on the device (seeded; not the reference's
 * sequential xorshift stream, which is generated on the host instead). */
int ttk_init_normal(float* x, int64_t n, float std, uint64_t seed, void* stream);

/* -------------------------------------------------------------- collectives */

/* NCCL over NVLink / NVSwitch, one communicator per rank (one process per
 * GPU). The library is loaded on first use. */
int ttk_dist_unique_id(unsigned char out[128]);
int ttk_dist_init(int rank, int world, const unsigned char id[128], void** comm);
int ttk_dist_destroy(void* comm);
/* In-place sum over ranks of n fp32 values. */
int ttk_dist_allreduce_f32(void* comm, float* buf, int64_t n, void* stream);
int ttk_dist_allreduce_f64(void* comm, double* buf, int64_t n, void* stream);
/* Non-zero when the communicator reported an asynchronous error. */
int ttk_dist_async_error(void* comm, int* err);
int ttk_dist_abort(void* comm);

#ifdef __cplusplus
}
#endif

#endif /* TTK_H */
