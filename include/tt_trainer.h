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
int tt_trainer_last_loss(void* handle, float* loss);
/* Forward + cross-entropy + backward only (gradients accumulate into the
 * parameters' gradients, zeroed first); logits (host, may be NULL) receives
 * [B*T, vocab]. */
int tt_trainer_forward_backward(void* handle, const int64_t* idx, const int64_t* targets,
                                int64_t B, int64_t T, float* loss, float* logits);

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

#ifdef __cplusplus
}
#endif

#endif /* TT_TRAINER_H */
