/* tt_trainer: C ABI over the tinytrain training step on B200.
 *
 * Drives the reference's hot loop (apps/train.cpp:212-256 of
 * seampm/tinytrain: zero_grad, forward, cross_entropy, loss read, backward,
 * set_lr, AdamW step) for a GPTModel held on the device, with two additions
 * the data-parallel configurations need: gradient accumulation over
 * micro-batches, and a bucketed NCCL all-reduce of the gradients overlapped
 * with the last micro-batch's backward (one process per GPU). Global-norm
 * clipping is folded into the fused AdamW kernel.
 *
 * Every function returns 0 on success; tt_last_error() holds the message of
 * the last failure on the calling thread. Host arrays are plain pointers.
 */
#ifndef TT_TRAINER_H
#define TT_TRAINER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int64_t vocab, dim, layers, heads, ffn, max_seq;
    float norm_eps, rope_theta;
} tt_model_config;

typedef struct {
    float lr, beta1, beta2, eps, weight_decay, clip_norm;
} tt_adamw_config;

const char* tt_last_error(void);

/* host_init = 1: the reference's initialization for `seed` (nn.cpp:14-38, on
 * the host, identical weights); 0: parameters left for tt_trainer_init_normal
 * or tt_trainer_set_params. */
int tt_trainer_create(const tt_model_config* cfg, uint64_t seed, int host_init, void** handle);
int tt_trainer_destroy(void* handle);
/* Issue all work on this CUDA stream (cudaStream_t as void*). */
int tt_trainer_set_stream(void* handle, void* stream);
int64_t tt_trainer_param_count(void* handle);
/* Matrices ~ N(0, std) from a counter-based device generator, norms = 1. */
int tt_trainer_init_normal(void* handle, float std, uint64_t seed);
/* Flat parameter vector in GPTModel::parameters() order (model.cpp:56-85). */
int tt_trainer_set_params(void* handle, const float* host, int64_t n);
int tt_trainer_get_params(void* handle, float* host, int64_t n);
int tt_trainer_get_grads(void* handle, float* host, int64_t n);
int tt_trainer_set_optimizer(void* handle, const tt_adamw_config* cfg);

/* One optimizer step over n_micro micro-batches of B x T tokens each:
 * idx/targets hold n_micro*B*T ids (host memory). The loss of the step (mean
 * over all its tokens, and over ranks when distributed) is written to *loss;
 * *grad_norm (may be NULL) gets the global gradient norm before clipping. */
int tt_trainer_step(void* handle, const int64_t* idx, const int64_t* targets, int64_t B,
                    int64_t T, int64_t n_micro, float lr, float* loss, float* grad_norm);
/* The same with ids already in device memory; the loss stays on the device
 * (read it with tt_trainer_last_loss) so no host synchronization happens. */
int tt_trainer_step_device(void* handle, const int64_t* idx, const int64_t* targets, int64_t B,
                           int64_t T, int64_t n_micro, float lr);
/* tt_trainer_step_device replayed from a CUDA graph (single GPU; no
 * counterpart in the reference, whose step is host code). The first call
 * with given id pointers and sizes runs an ordinary step; the second records
 * a step into a graph and launches it; later calls with the same pointers
 * and sizes launch the graph again, after writing that step's learning rate
 * and AdamW bias correction to the device. Each call is one optimizer step
 * with the same arithmetic as tt_trainer_step_device (identical results).
 * The caller puts each step's ids into the same two device buffers before
 * the call (stream-ordered). Other pointers or sizes drop the graph and
 * start over, as do tt_trainer_set_params, tt_trainer_init_normal,
 * tt_trainer_load, tt_trainer_set_optimizer and tt_trainer_dist_init (they
 * rewrite or replace state the graph reads). A failed recording leaves the
 * step count as it was. Recording returns the device pool's unused memory first: the
 * graph allocates its activations from its own pool. Fails on a trainer
 * with a communicator. */
int tt_trainer_step_graph(void* handle, const int64_t* idx, const int64_t* targets, int64_t B,
                          int64_t T, int64_t n_micro, float lr);
int tt_trainer_last_loss(void* handle, float* loss);
/* tt_trainer_step in two halves, so that the host prepares and enqueues step
 * i + 1 while the device runs step i. submit copies the host ids into one of
 * two pinned staging slots of the trainer (the caller may reuse its arrays on
 * return), uploads them, enqueues the step and the copy of its loss and
 * gradient norm into pinned memory, and returns without waiting. result waits
 * for the oldest submitted step and returns its loss and norm (as
 * tt_trainer_step does). At most two steps are in flight: a third submit
 * before a result fails. */
int tt_trainer_step_submit(void* handle, const int64_t* idx, const int64_t* targets, int64_t B,
                           int64_t T, int64_t n_micro, float lr);
int tt_trainer_step_result(void* handle, float* loss, float* grad_norm);
/* Forward + cross-entropy + backward only (gradients accumulate into the
 * parameters' gradients, zeroed first); logits (host, may be NULL) receives
 * [B*T, vocab]. */
int tt_trainer_forward_backward(void* handle, const int64_t* idx, const int64_t* targets,
                                int64_t B, int64_t T, float* loss, float* logits);

/* ---- data feed (apps/train.cpp:162-174, 225-232) ----
 * A token stream is the int32 token file written by apps/prepare_data.cpp
 * (raw little-endian int32), held in device memory for the whole run. */
int tt_tokens_from_file(const char* path, void** tokens);
int tt_tokens_from_host(const int32_t* host, int64_t n, void** tokens);
int64_t tt_tokens_count(void* tokens);
int tt_tokens_destroy(void* tokens);
/* The reference's window sampler: `count` draws of its xorshift64* Rng
 * (apps/train.cpp:145-153; the state starts at the seed, apps/train.cpp uses
 * seed + 999, and 0 stands for 0x9E3779B97F4A7C15), each start = next() %
 * (ntok - T - 1). *rng_state advances, so consecutive calls continue the
 * stream exactly as consecutive training steps do. Host only. */
int tt_sample_windows(uint64_t* rng_state, int64_t ntok, int64_t T, int64_t count,
                      int64_t* starts);
/* One optimizer step on windows of a device token stream: `starts` (host)
 * holds the n_micro*B window starts of this rank (for data parallelism, rank
 * r takes draws [r*n_micro*B, (r+1)*n_micro*B) of the global batch); only
 * they cross to the device, where a gather kernel builds ids and targets.
 * loss / grad_norm as in tt_trainer_step (either may be NULL). */
int tt_trainer_step_tokens(void* handle, void* tokens, const int64_t* starts, int64_t B,
                           int64_t T, int64_t n_micro, float lr, float* loss, float* grad_norm);

/* The learning-rate schedule of apps/train.cpp:214-222: linear warmup over
 * `warmup` steps, then cosine decay to 10% of base_lr at total_steps (float
 * arithmetic in the reference's order). The result is the lr argument of the
 * step functions, i.e. a scalar argument of the fused AdamW kernel. */
float tt_lr_at(float base_lr, int64_t step, int64_t warmup, int64_t total_steps);

/* ---- checkpoints ----
 * <dir>/model.safetensors + config.json exactly as GPTModel::save_checkpoint
 * writes them (model.cpp:162-227; the reference's load_checkpoint reads them),
 * plus <dir>/optimizer.safetensors with AdamW's moments ("m.<i>", "v.<i>",
 * parameters() order) and its step count, so that a run resumes bit for bit
 * (the reference restores weights only). tt_trainer_load restores the
 * optimizer state when the file is present. */
int tt_trainer_save(void* handle, const char* dir);
int tt_trainer_load(void* handle, const char* dir);

/* Deadline for a distributed step's collectives (default 300 s). Before each
 * distributed step the previous one's completion is awaited with this bound
 * (one step in flight), polling ncclCommGetAsyncError; tt_trainer_step also
 * awaits its own step before reading the loss. On an asynchronous error or
 * an overrun (a peer left or hangs) the communicator is aborted
 * (ncclCommAbort ends its pending collectives), the step fails with the
 * reason, and later distributed steps are refused. No counterpart in the
 * reference (which has no distributed code). */
int tt_trainer_set_collective_timeout(void* handle, double seconds);
/* Timing of the gradient all-reduce (off by default): with profiling on,
 * every bucket's all-reduce is bracketed by events on the comm stream, and
 * each distributed step records the end of its last backward on the compute
 * stream against the end of its last all-reduce. tt_trainer_comm_stats
 * returns, since the last read, the summed all-reduce time, the summed
 * exposed tail (all-reduce end minus backward end, when positive: the time
 * the optimizer waits for the collective), and the counts; it synchronizes. */
int tt_trainer_comm_profile(void* handle, int on);
int tt_trainer_comm_stats(void* handle, double* allreduce_ms, double* tail_ms,
                          int64_t* n_allreduce, int64_t* n_steps);
/* The watchdog's wait loop on caller-supplied probes, for testing it without
 * a communicator: done(ctx) != 0 ends the wait (outcome 0); async_error(ctx)
 * != 0 calls abort(ctx) once (outcome 1); so does passing timeout_s
 * (outcome 2). */
int tt_watchdog_selftest(int (*done)(void*), int (*async_error)(void*), int (*abort)(void*),
                         void* ctx, double timeout_s, int* outcome);
/* Data parallelism: join an NCCL communicator (id from rank 0's
 * ttk_dist_unique_id, shared out of band) and reduce gradients in buckets of
 * about bucket_bytes during backward. */
int tt_trainer_dist_init(void* handle, int rank, int world, const unsigned char id[128],
                         int64_t bucket_bytes);
/* The gradient arena / bucket plan used by a data-parallel trainer (host
 * only, no device needed): for n parameters of the given sizes in
 * parameters() order, writes each one's arena offset (elements) and bucket
 * id, and per bucket its offset and length (buckets ordered as backward
 * finishes them; arrays sized n). */
int tt_plan_buckets(const int64_t* sizes, int n, int64_t bucket_bytes, int64_t* offsets,
                    int* bucket_of_param, int64_t* bucket_offset, int64_t* bucket_count,
                    int* n_buckets);
/* Number of CUDA kernels this library launched so far (all streams). */
int64_t tt_kernel_launches(void);
/* Number of attention-score chains (bmm(q, transpose(k)), * constant,
 * + causal mask, softmax, bmm(., v): model.cpp:133-138 of the reference)
 * that ran as the fused causal attention kernel since start-up. */
int64_t tt_fused_attention_chains(void);

#ifdef __cplusplus
}
#endif

#endif /* TT_TRAINER_H */
