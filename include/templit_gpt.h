/*
 * templit_gpt.h - C ABI of the GPT training step built from TempLit's own
 * model and compiler (include/nn/GPT.h, include/passes/compile.h in
 * JTPuffer/TempLit) on the `cuda` runtime.
 *
 * One handle owns a compiled `nn::GPT<Mat, vocab, max_seq, d_model, heads>`
 * with its cross-entropy loss and AdamW optimiser, exactly as
 * src/train.cpp:89-157 builds it, with the backend alias switched to
 * RTensor<cuda::CUDA, float>.  tlg_train_step runs one iteration of the
 * reference training loop: set inputs, zero_grad, forward, read the losses,
 * backward with root gradient 1/(rank-local tokens * world), step(clip).
 *
 * Model families: `family` 4 is the reference's 4-block GPT (d_model 384,
 * 6 heads, vocab 2048, max sequence 192); `family` 12 the 12-block,
 * d_model 768, 12-head, FFN 3072, max-sequence-1024 variant of the
 * data-parallel configuration (the reference's decoder blocks, embedding
 * and projection, generalised from GPT.h's four blocks).  All calls return
 * 0 on success; tlg_last_error() explains a failure.
 */
#ifndef TEMPLIT_GPT_H
#define TEMPLIT_GPT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct tlg_config {
  uint32_t family;       /* 4 or 12 (see above)                                */
  uint32_t batch;        /* sequences per rank                                 */
  uint32_t seq;          /* tokens per sequence (<= the family's max sequence) */
  uint32_t seed;         /* std::mt19937 seed of the reference initialiser     */
  float init_std;        /* > 0: re-draw every weight N(0, init_std), biases 0 */
  float lr, beta1, beta2, eps, weight_decay;
  float clip;            /* > 0: Compiled::step(clip), else Compiled::step()    */
  uint32_t world;        /* data-parallel ranks sharing the global batch       */
  int32_t fusion;        /* runtime program fusion on/off                      */
  int32_t graphs;        /* CUDA-graph replay on/off                           */
  int32_t gemm_precision; /* TL_GEMM_TF32 (0, tensor cores), TL_GEMM_FP32 (1) or
                             TL_GEMM_3XTF32 (2, split tf32 operands)            */
  int32_t deferred_wait; /* cuda::Runtime::set_deferred_wait: the host records the
                            next window while the GPU runs the current one     */
  uint32_t micro_batches; /* > 1: a train step is this many forward / backward
                             passes of `batch` sequences, their gradients
                             summed (the reference's gradient accumulation
                             across backward calls, include/passes/context.h:
                             74-89), then one optimiser step; tlg_set_batch
                             takes micro_batches * batch sequences           */
  int32_t flash_attention; /* attention on the flash kernels: 0 where the short-
                              sequence fused kernels cannot run (T > 192), 1
                              always, -1 never (cuda::Runtime::
                              set_flash_attention modes 1, 2, 0)               */
} tlg_config;

const char *tlg_last_error(void);
int tlg_create(const tlg_config *config, void **handle);
int tlg_destroy(void *handle);
/* Host token ids and targets, micro_batches*batch*seq each (row-major
 * [micro_batches * batch, seq]; micro_batches 0 counts as 1). */
int tlg_set_batch(void *handle, const uint32_t *tokens, const uint32_t *targets);
/* One training iteration; *mean_loss receives the mean loss of this rank's batch. */
int tlg_train_step(void *handle, float *mean_loss);
/* Forward only; losses receives batch*seq per-token losses. */
int tlg_forward(void *handle, float *losses);
/* Parameters in the compiler's gradient-path order, concatenated. */
int tlg_param_count(void *handle, uint64_t *count, uint32_t *tensors);
int tlg_get_params(void *handle, float *out, uint64_t count);
int tlg_set_params(void *handle, const float *in, uint64_t count);
/* The backend stream (cudaStream_t) every launch of this handle uses. */
void *tlg_stream(void *handle);
/* Runtime counters: [0] windows, [1] recorded ops, [2] launched ops,
 * [3] kernels, [4] graph replays, [5] graph captures, [6] fused ops,
 * [7] peak device bytes, [8] host ns recording, [9] host ns in submit,
 * [10] optimiser cache hits (totals since creation). */
#define TLG_STATS 11
int tlg_stats(void *handle, uint64_t out[TLG_STATS]);
/* Data parallelism: NCCL unique id (128 bytes) made on rank 0 and shared
 * by the caller, then a communicator on every rank. */
int tlg_nccl_unique_id(uint8_t id[128]);
int tlg_set_communicator(void *handle, const uint8_t id[128], int nranks, int rank);
/* Per-op device timing of the next `steps` train steps, written as JSON. */
int tlg_profile(void *handle, const char *path, int steps);

/* Configuration 1: the MLP loss sqe(linear(sigmoid(linear(X, W1, b1)), W2, b2), Y)
 * compiled by passes::compile with SGD(lr) and trained `steps` iterations
 * with a constant root gradient, on cuda::Runtime.  X [batch, in],
 * W1 [in, hidden], b1 [1, hidden], W2 [hidden, out], b2 [1, out],
 * Y [batch, out] are host arrays; the weights are updated in place,
 * losses[s] receives the summed loss of step s, *seconds the loop time.
 * gemm_precision selects TL_GEMM_TF32 (0) or TL_GEMM_FP32 (1). */
/* Checkpoints in the reference's archive format (src/model_utils/
 * archive.cpp:33-73, Compiled::save / load, include/passes/compile.h:
 * 259-298): the parameters and, with `optimiser`, the AdamW moments and
 * step count (saving those needs at least one step). */
int tlg_save(void *handle, const char *path, int optimiser);
int tlg_load(void *handle, const char *path, int optimiser);

/* Training input pipeline (src/train.cpp:75-77,142-144): a raw uint32 token
 * file split as the reference's Dataset (training part, or with
 * `validation` the rest) and sampled as its Loader::get_batch with
 * std::mt19937(seed); a background thread draws the next batch into pinned
 * memory.  tlg_loader_next hands out [batch, seq] inputs and targets, valid
 * until the next call - pass them to tlg_set_batch. */
int tlg_loader_create(const char *path, double training_fraction, int validation,
                      uint32_t batch, uint32_t seq, uint32_t seed, void **handle);
int tlg_loader_next(void *handle, const uint32_t **inputs, const uint32_t **targets);
int tlg_loader_destroy(void *handle);

/* Forward-only inference as src/generate.cpp sets it up: a batch-1 model of
 * config->seq tokens (family 4; init_std/seed as for training) whose logits
 * graph is compiled on its own, driven by the reference's
 * inference::autoregression (include/inference.h:45-97).  Parameters in the
 * order of tlg_get_params. */
int tlg_infer_create(const tlg_config *config, void **handle);
int tlg_infer_destroy(void *handle);
int tlg_infer_param_count(void *handle, uint64_t *count);
int tlg_infer_get_params(void *handle, float *out, uint64_t count);
int tlg_infer_set_params(void *handle, const float *in, uint64_t count);
/* logits [seq, 2048] of one window of seq tokens */
int tlg_infer_logits(void *handle, const uint32_t *tokens, float *logits);
/* tokens emitted by inference::autoregression for this prompt (top-k
 * sampling with std::mt19937(seed)); *n_out = how many were emitted, of
 * which the first max_out are stored */
int tlg_infer_generate(void *handle, const uint32_t *prompt, uint32_t n_prompt, uint32_t eos,
                       uint32_t seed, uint32_t top_k, float temperature, uint32_t min_length,
                       uint32_t *out, uint32_t max_out, uint32_t *n_out);

int tlg_mlp_train(const float *X, uint32_t batch, uint32_t in, uint32_t hidden, uint32_t out,
                  float *W1, float *b1, float *W2, float *b2, const float *Y, float root,
                  float lr, int steps, int gemm_precision, float *losses, double *seconds);
const char *tlg_mlp_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* TEMPLIT_GPT_H */
