/*
 * templit_cuda.h - C ABI of the B200 (sm_100a) kernel library behind the
 * TempLit `cuda` runtime.
 *
 * Every entry point takes plain pointers and sizes, returns an int status
 * (TL_OK == 0) and never throws.  Device pointers are CUDA device memory;
 * `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 * All launches are asynchronous on `stream`; argument errors are reported
 * before anything is launched, launch errors through the return value, and
 * data-dependent errors (an embedding id outside the table) through the
 * device status word read by tl_device_status().  Text for the last failure
 * on the calling thread is returned by tl_last_error().
 *
 * Each function names the reference interface it replaces: the
 * `metal::Runtime` method (src/my_metal/runtime.cpp) and the Metal kernel it
 * dispatches (include/my_metal/math.metal) in JTPuffer/TempLit.  Tensors are
 * dense row-major fp32 (uint32 for token ids), the only layout
 * RTensor produces (include/RTensor/RTensor.h:110-137,245-281).
 */
#ifndef TEMPLIT_CUDA_H
#define TEMPLIT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TL_MAX_RANK 8

enum tl_status_code {
  TL_OK = 0,
  TL_ERR_INVALID = 1,     /* bad argument: shape, rank, null pointer      */
  TL_ERR_CUDA = 2,        /* CUDA runtime or launch failure               */
  TL_ERR_UNSUPPORTED = 3, /* valid request this build cannot serve        */
  TL_ERR_RANGE = 4        /* axis / size outside the supported range      */
};

/* Bits of the device status word (tl_device_status). */
enum tl_device_flag {
  TL_FLAG_INDEX_RANGE = 1u, /* an id >= table rows reached a gather/scatter */
  TL_FLAG_TIMEOUT = 2u      /* a bounded on-device wait gave up (kernel returned early) */
};

/* ---------------------------------------------------------------- library */

/* ABI version of this library (bumped on any signature change). */
int tl_version(void);
/* Message of the last failing call on this thread ("" if none). */
const char *tl_last_error(void);
/* Select and initialise `device`; replaces metal::init() (src/my_metal/metal.cpp:18-30). */
int tl_device_init(int device);
/* Synchronise `stream`, then read and clear the device status word. */
int tl_device_status(uint32_t *flags, void *stream);
/* Without synchronising: enqueue on `stream` a move of the status word into
 * *host_flags (pinned host memory, valid once the stream reaches this point)
 * and clear it.  Backs cuda::Runtime's deferred wait(). */
int tl_device_status_enqueue(uint32_t *host_flags, void *stream);

/* ------------------------------------------- memory (Storage<Metal,T> ops) */
/* Device allocation; replaces MTL::Device::newBuffer (include/my_metal/storage.h:13-16). */
int tl_malloc(void **ptr, size_t bytes);
int tl_free(void *ptr);
/* Pinned host allocation for staging host<->device copies. */
int tl_host_alloc(void **ptr, size_t bytes);
int tl_host_free(void *ptr);
int tl_stream_create(void **stream);
int tl_stream_destroy(void *stream);
int tl_stream_sync(void *stream);
/* Stream-ordered copies; replace Storage::write/read/clone memcpy (include/my_metal/storage.h:25-52). */
int tl_memcpy_h2d(void *dst, const void *src, size_t bytes, void *stream);
int tl_memcpy_d2h(void *dst, const void *src, size_t bytes, void *stream);
int tl_memcpy_d2d(void *dst, const void *src, size_t bytes, void *stream);
/* Fill with a 32-bit pattern; replaces Storage::fill (include/my_metal/storage.h:41-43). */
int tl_fill_u32(void *dst, uint32_t pattern, size_t count, void *stream);

/* ---------------------- command recording (MTL::CommandBuffer counterparts) */
/* Events for device-side timing; replace the Metal capture-manager profile
 * hooks (src/my_metal/runtime.cpp:42-63). */
int tl_event_create(void **event);
int tl_event_destroy(void *event);
int tl_event_record(void *event, void *stream);
/* Milliseconds between two recorded events (waits for `end`). */
int tl_event_elapsed_ms(float *ms, void *start, void *end);
/* *done = 1 when all work before the event's record has completed. */
int tl_event_query(void *event, int *done);
/* Stream capture into a replayable graph: the counterpart of encoding a
 * command buffer once and committing it again (src/my_metal/runtime.cpp:290-317). */
int tl_graph_capture_begin(void *stream);
/* Ends the capture on `stream`; *graph_exec receives an instantiated graph
 * (NULL and an error status if anything in the capture failed). */
int tl_graph_capture_end(void *stream, void **graph_exec);
int tl_graph_launch(void *graph_exec, void *stream);
int tl_graph_destroy(void *graph_exec);
/* Kernels this library has launched on this host thread so far (stream
 * captures included): the runtime's launch accounting. */
uint64_t tl_kernel_launches(void);

/* ------------------------------------------------------------ elementwise */
enum tl_binary_op { TL_ADD = 0, TL_SUB = 1, TL_MUL = 2, TL_DIV = 3 };
/*
 * out = a (op) b with trailing-aligned size-1 broadcasting against
 * out_shape.  Replaces Runtime::add/sub/hadamard/divide
 * (src/my_metal/runtime.cpp:18-39,65-95,321-353; math.metal:401-510).
 * out may alias a or b element-for-element.
 */
int tl_binary(int op, const float *a, const uint32_t *a_shape, int a_rank,
              const float *b, const uint32_t *b_shape, int b_rank, float *out,
              const uint32_t *out_shape, int out_rank, void *stream);

enum tl_scalar_op { TL_SCALAR_ADD = 0, TL_SCALAR_DIV = 1, TL_SCALAR_POW = 2 };
/* out = x (op) s.  Replaces Runtime::add(a,s)/divide(a,s)/pow
 * (src/my_metal/runtime.cpp:116-136,327-330,350-353,365-368; math.metal:427-434,511-518,527-534). */
int tl_scalar(int op, const float *x, float s, float *out, size_t count,
              void *stream);

enum tl_unary_op {
  TL_SIGMOID = 0,
  TL_SQRT = 1,
  TL_EXP = 2,
  TL_GELU = 3,
  TL_GELU_DERIVATIVE = 4
};
/* out = f(x).  Replaces Runtime::sigmoid/sqrt/exp/GELU/GELU_derivative
 * (src/my_metal/runtime.cpp:97-114,355-373,1073-1081; math.metal:519-548,821-855). */
int tl_unary(int op, const float *x, float *out, size_t count, void *stream);

/* out = GELU'(x) * grad in one pass: the executor's GELU_derivative followed
 * by its chain-rule hadamard (include/passes/autograd.h GELU rule;
 * math.metal:835-855,461-485). */
int tl_gelu_backward(const float *x, const float *grad, float *out,
                     size_t count, void *stream);

/* out = x.  Replaces Runtime::copy (src/my_metal/runtime.cpp:1170-1186; math.metal:1045-1051). */
int tl_copy(const float *x, float *out, size_t count, void *stream);

/* ------------------------------------------------------------- reductions */
enum tl_reduce_op { TL_REDUCE_SUM = 0, TL_REDUCE_MAX = 1 };
/*
 * Reduce x to out_shape (trailing-aligned; every out dim equal to the x dim
 * or 1).  Replaces Runtime::sum_to_shape / max_to_shape / reduce_to_shape
 * (src/my_metal/runtime.cpp:595-745; math.metal:618-714).  Deterministic.
 * A column reduction split over many CTAs folds its partials in the same
 * launch, counting arrivals in counters inside the library: reductions of
 * one process must not run concurrently on several streams. 
 * workspace may be NULL when tl_reduce_workspace_size() returns 0.
 */
int tl_reduce(int op, const float *x, const uint32_t *x_shape, int x_rank,
              float *out, const uint32_t *out_shape, int out_rank,
              void *workspace, size_t workspace_bytes, void *stream);
size_t tl_reduce_workspace_size(const uint32_t *x_shape, int x_rank,
                                const uint32_t *out_shape, int out_rank);

/*
 * tl_reduce of up to TL_REDUCE_MAX_GROUPS tensors of one shape, x[i] ->
 * out[i], each result bit-identical to tl_reduce(x[i]); the column
 * reductions that fold their partials in-launch run as one launch for all
 * groups.  Replaces consecutive Runtime::sum_to_shape calls on same-shape
 * tensors (src/my_metal/runtime.cpp:595-745), which the runtime's optimiser
 * groups: the bias gradients of the query, key and value projections.
 * Workspace: tl_reduce_group_workspace_size() (groups x the single one).
 */
#define TL_REDUCE_MAX_GROUPS 4
int tl_reduce_group(int op, uint32_t groups, const float *const *x, const uint32_t *x_shape,
                    int x_rank, float *const *out, const uint32_t *out_shape, int out_rank,
                    void *workspace, size_t workspace_bytes, void *stream);
size_t tl_reduce_group_workspace_size(uint32_t groups, const uint32_t *x_shape, int x_rank,
                                      const uint32_t *out_shape, int out_rank);

/*
 * tl_reduce without a workspace argument; it allocates nothing.  No
 * counterpart in the reference: it exists for callers that cannot allocate
 * device memory when they reduce - code running while a CUDA stream is
 * captured into a graph (cudaMalloc is not allowed there), hosts whose
 * device memory is wholly owned by another allocator (a framework pool or a
 * fixed arena), and foreign-language callers without a CUDA allocator.
 * Partial sums go to a 4 MiB array in the library's device memory
 * (tl_reduce_noalloc_max_workspace() bytes), held by every GPU that loads
 * the library until the process exits.  A reduction whose
 * tl_reduce_workspace_size() exceeds that returns TL_ERR_RANGE.  The first
 * call on each device looks up the array's device address (make it before
 * any stream capture); first calls from several host threads at once are
 * safe.  The address stays cached for the process, so do not call this
 * again on a device after cudaDeviceReset.  All calls share the array:
 * calls that can overlap on the GPU (other streams, other host threads)
 * race on it; calls ordered on one stream do not.
 */
int tl_reduce_noalloc(int op, const float *x, const uint32_t *x_shape, int x_rank,
                      float *out, const uint32_t *out_shape, int out_rank, void *stream);
size_t tl_reduce_noalloc_max_workspace(void);

/* First index of the maximum of x[0..count) (NaN ignored, 0 if none).
 * Replaces Runtime::argmax (src/my_metal/runtime.cpp:850-918; math.metal:715-777). */
int tl_argmax(const float *x, size_t count, uint32_t *out_index,
              void *workspace, size_t workspace_bytes, void *stream);
size_t tl_argmax_workspace_size(size_t count);

/* Materialised swap of axes dim_a, dim_b of a dense tensor.
 * Replaces Runtime::transpose (src/my_metal/runtime.cpp:529-569; math.metal:566-584). */
int tl_transpose(const float *x, const uint32_t *shape, int rank, int dim_a,
                 int dim_b, float *out, void *stream);

/* --------------------------------------------------------- row operators */
/* Row softmax over the last dim.  Replaces Runtime::softmax
 * (src/my_metal/runtime.cpp:747-766; math.metal:857-882). */
int tl_softmax_rows(const float *x, float *out, uint32_t rows, uint32_t cols,
                    void *stream);
/* out = softmax(x / divisor[0] + mask[r % mask_rows, :]) (divisor and mask
 * optional, mask of mask_rows x cols): the score chain of
 * nn::MultiHeadAttention (include/nn/multi_head.h: divide by
 * sqrt(HeadSize), add the causal mask, soft_max) in one pass, bit-identical
 * to the three separate ops. */
int tl_softmax_scaled_masked_rows(const float *x, const float *divisor, const float *mask,
                                  uint32_t mask_rows, float *out, uint32_t rows,
                                  uint32_t cols, void *stream);
/* dx = y * (g - sum_row(g * y)) (then / divisor[0] when divisor is not
 * NULL): the SFTMX_DERIVATIVE rule (include/passes/execute.h:291-308) in one
 * pass, optionally with the derivative of the preceding score division. */
int tl_softmax_backward_rows(const float *grad, const float *y, const float *divisor,
                             float *dx, uint32_t rows, uint32_t cols, void *stream);
/* rms[r] = sqrt(sum(x^2)/cols + 1e-6).  Replaces Runtime::RMS
 * (src/my_metal/runtime.cpp:1031-1059). */
int tl_rms_rows(const float *x, float *rms, uint32_t rows, uint32_t cols,
                void *stream);
/* out = x / rms(x) (rms_out optional).  Replaces Runtime::RMSNorm
 * (src/my_metal/runtime.cpp:1061-1072). */
int tl_rmsnorm_rows(const float *x, float *out, float *rms_out, uint32_t rows,
                    uint32_t cols, void *stream);
/* dx = (g - y * mean(g * y)) / rms(x) (+ addend when not NULL; addend may
 * equal dx): the RMSN_DERIVATIVE rule (include/passes/execute.h:330-356) in
 * one pass, optionally with the residual gradient added after it. */
int tl_rmsnorm_backward_rows(const float *grad, const float *x, const float *y,
                             const float *addend, float *dx, uint32_t rows, uint32_t cols,
                             void *stream);
/* loss[r] = max + log(sum(exp(z - max))) - z[t]; +inf when t >= vocab.
 * Replaces Runtime::cross_entropy (src/my_metal/runtime.cpp:768-804; math.metal:884-910). */
int tl_xent_rows(const float *logits, const uint32_t *targets, float *loss,
                 uint32_t rows, uint32_t vocab, void *stream);
/* dz = (softmax(z) - onehot(t)) * row_scale[r] (row_scale NULL => 1); a row
 * with t >= vocab is +inf.  Replaces Runtime::cross_entropy_derivative
 * (src/my_metal/runtime.cpp:806-841; math.metal:912-953), optionally fused
 * with the executor's hadamard by the root gradient. */
int tl_xent_backward_rows(const float *logits, const uint32_t *targets,
                          const float *row_scale, float *dlogits,
                          uint32_t rows, uint32_t vocab, void *stream);

/* -------------------------------------------------------------- embedding */
/* out[i,:] = weights[ids[i],:].  Replaces Runtime::embedding_lookup /
 * gather_rows (src/my_metal/runtime.cpp:920-950; math.metal:778-793).
 * An id >= n_rows yields a zero row and sets TL_FLAG_INDEX_RANGE. */
int tl_embedding_gather(const float *weights, uint32_t n_rows, uint32_t dim,
                        const uint32_t *ids, uint32_t n_ids, float *out,
                        void *stream);
/* dst[r,:] = base[r,:] + sum of values[i,:] over i with ids[i] == r
 * (base NULL => zeros; base may equal dst).  Replaces
 * Runtime::scatter_add_rows (base given) and Runtime::scatter_index (base
 * NULL) (src/my_metal/runtime.cpp:952-1030; math.metal:794-820).
 * Deterministic: each chunk of 256 ids is summed per id in input order, and
 * each row folds its chunk sums in chunk order.  The workspace holds one
 * partial row per id (tl_embedding_scatter_workspace_size).
 * An id >= n_rows is skipped and sets TL_FLAG_INDEX_RANGE. */
int tl_embedding_scatter_add(const float *values, const uint32_t *ids,
                             uint32_t n_ids, uint32_t dim, const float *base,
                             float *dst, uint32_t n_rows, void *workspace,
                             size_t workspace_bytes, void *stream);
size_t tl_embedding_scatter_workspace_size(uint32_t n_ids, uint32_t n_rows, uint32_t dim);

/* -------------------------------------------------------------- optimiser */
/* sqnorm[0] += sum(grad^2).  Replaces Runtime::accumulate_gradient_squared_norm
 * (src/my_metal/runtime.cpp:1083-1101; math.metal:955-983).  Deterministic. */
int tl_grad_sqnorm_accumulate(const float *grad, size_t count, float *sqnorm,
                              void *workspace, size_t workspace_bytes,
                              void *stream);
size_t tl_grad_sqnorm_workspace_size(size_t count);
/* out = grad * min(1, max_norm * rsqrt(max(sqnorm, 1e-12))).  Replaces
 * Runtime::clip_gradient (src/my_metal/runtime.cpp:1103-1127; math.metal:985-1006). */
int tl_clip_gradient(const float *grad, const float *sqnorm, float max_norm,
                     float *out, size_t count, void *stream);
/* AdamW with decoupled decay p*decay (decay = 1 - lr*wd).  Replaces
 * Runtime::adamW (src/my_metal/runtime.cpp:1129-1168; math.metal:1008-1043;
 * include/optimiser/AdamW.h:75-82).  beta1/beta2/decay/lr are device scalars. */
int tl_adamw(const float *param, const float *grad, float *out, float *m1,
             float *m2, const float *beta1, const float *beta2,
             const float *decay, const float *lr, float epsilon, uint32_t step,
             size_t count, void *stream);

/* One parameter tensor of a fused multi-tensor optimiser pass. */
typedef struct tl_param_slot {
  const float *param; /* parameter read                                  */
  float *out;         /* destination (may equal param)                   */
  float *grad;        /* gradient (clipped in place when clipping)       */
  float *m1;          /* first moment                                    */
  float *m2;          /* second moment                                   */
  uint64_t count;     /* elements                                        */
  uint32_t chunk0;    /* index of this slot's first chunk: the sum of
                         ceil(count / TL_OPT_CHUNK) over earlier slots   */
  uint32_t step;      /* per-tensor AdamW step (>= 1)                    */
} tl_param_slot;
/* Elements per work chunk of the multi-tensor optimiser kernels. */
#define TL_OPT_CHUNK 8192u
/*
 * The whole `Compiled::step(max_norm)` program (include/passes/compile.h:236-258)
 * in two launches: sqnorm[0] += sum over all slots of grad^2, then for every
 * slot grad = clip(grad), and the AdamW update.  max_norm <= 0 skips the norm
 * and the clip (Compiled::step() without clipping, compile.h:223-234).
 * `slots` is device memory holding n_slots records.  The norm's CTAs count
 * their arrivals in a counter inside the library (the last one adds the
 * partials): calls of one process must not run concurrently on several
 * streams.
 */
int tl_multi_clip_adamw(const tl_param_slot *slots, uint32_t n_slots,
                        uint32_t n_chunks, float *sqnorm, float max_norm,
                        const float *beta1, const float *beta2,
                        const float *decay, const float *lr, float epsilon,
                        void *workspace, size_t workspace_bytes, void *stream);
size_t tl_multi_clip_adamw_workspace_size(uint32_t n_chunks);
/*
 * Copies every slot's gradient into one flat buffer (unpack = 0) or back
 * out of it (unpack = 1), in the slots' chunk layout: slot i's element e at
 * flat[chunk0 * TL_OPT_CHUNK + e]; `flat` holds n_chunks * TL_OPT_CHUNK
 * floats (16-byte aligned) and the padding after each slot is left as it
 * is.  Only `grad`, `count` and `chunk0` of the (device) slots are read.
 * No counterpart in the reference, which has no multi-device path: the
 * data-parallel gradient exchange runs as one NCCL all-reduce over `flat`
 * instead of one per tensor.
 */
int tl_multi_grad_flat(const tl_param_slot *slots, uint32_t n_slots, uint32_t n_chunks,
                       float *flat, int unpack, void *stream);

/* ------------------------------------------------------------------- GEMM */
enum tl_gemm_precision {
  TL_GEMM_TF32 = 0,   /* tcgen05 kind::tf32 tensor cores, fp32 accumulate */
  TL_GEMM_FP32 = 1,   /* CUDA-core fp32 FMA (exact fp32 products)         */
  TL_GEMM_3XTF32 = 2  /* tcgen05 with split big/small tf32 operands: each
                         product is big*big + big*small + small*big of the
                         operands' tf32 halves, about fp32's accuracy   */
};
#define TL_GEMM_MAX_BATCH_RANK 6
#define TL_GEMM_MAX_GROUPS 4
enum tl_gemm_group_mode {
  TL_GEMM_GROUP_NONE = 0,
  TL_GEMM_GROUP_N = 1,  /* C_g = op(A) op(B_g) (+ bias_g), A shared           */
  TL_GEMM_GROUP_K = 2   /* C = sum_g op(A_g) op(B_g) (+ bias) (+ addend / C)   */
};
/*
 * C[b] = op(A[b]) * op(B[b]) (+ bias) (+ beta * C[b]) for every batch index
 * b of batch_shape, with per-operand batch strides in elements (0 =
 * broadcast).  trans_a = 0: A[b] is [M,K] row-major, 1: stored [K,M].
 * trans_b = 0: B[b] is [K,N] row-major, 1: stored [N,K].  Replaces
 * Runtime::mult (src/my_metal/runtime.cpp:375-505; math.metal:13-400) and,
 * through trans_a/trans_b, the executor's transpose+mult pairs of
 * EXPR_MULT_{LHS,RHS}_DERIVATIVE (include/passes/execute.h:187-232).
 * gelu_out (optional) receives GELU of the final value.  addend (optional,
 * C's layout) is added to the product: C = addend + (A*B + bias), the
 * executor's add of a product into a gradient or residual stream folded
 * into the epilogue; beta = 1 is the same with addend = C.
 */
typedef struct tl_gemm_desc {
  const float *a;
  const float *b;
  float *c;
  const float *bias; /* optional [N], added to every row               */
  float *gelu_out;   /* optional, same layout as c                     */
  uint32_t m, n, k;
  int32_t trans_a, trans_b;
  int32_t precision; /* tl_gemm_precision                               */
  float beta;        /* 0 or 1                                          */
  uint32_t batch_rank;
  uint32_t batch_shape[TL_GEMM_MAX_BATCH_RANK];
  uint64_t a_batch_stride[TL_GEMM_MAX_BATCH_RANK];
  uint64_t b_batch_stride[TL_GEMM_MAX_BATCH_RANK];
  uint64_t c_batch_stride[TL_GEMM_MAX_BATCH_RANK];
  /* Scratch for split-K slices (tl_gemm_workspace_size bytes).  A product
   * with few output tiles and a long K (a weight gradient) is cut into K
   * slices summed in order by a second kernel; with a smaller workspace it
   * runs unsplit, with the same result. */
  void *workspace;
  uint64_t workspace_bytes;
  const float *addend;
  /* Row strides (elements) of the stored A, B and C matrices; 0 = dense
   * (the stored row length: K or M for A, N or K for B, N for C).  C,
   * gelu_out and addend share ldc.  With the batch strides they address
   * strided views, e.g. one attention head of a [B, T, H, D] tensor. */
  uint64_t lda, ldb, ldc;
  /* Grouped products (group_mode != TL_GEMM_GROUP_NONE, 2 <= groups <=
   * TL_GEMM_MAX_GROUPS) sharing every other field: the Q, K and V
   * projections of one input (GROUP_N: b_group[g], c_group[g],
   * bias_group[g] per product, `a` shared, c_group[0] == c; no GELU,
   * addend or beta), or a sum of products into one output over their
   * concatenated K (GROUP_K: a_group[g], b_group[g], each product of depth
   * k; bias, addend and beta apply once; no GELU).  One launch instead of
   * `groups`. */
  int32_t group_mode;
  uint32_t groups;
  const float *a_group[TL_GEMM_MAX_GROUPS];
  const float *b_group[TL_GEMM_MAX_GROUPS];
  float *c_group[TL_GEMM_MAX_GROUPS];
  const float *bias_group[TL_GEMM_MAX_GROUPS];
  /* Optional, C's layout: C = GELU'(gelu_grad_x) * (A*B (+ bias)), the GELU
   * backward (GELU_derivative(x) hadamard the incoming gradient,
   * include/passes/execute.h) folded into the epilogue of the product that
   * makes the gradient.  Not with addend, beta, gelu_out or groups. */
  const float *gelu_grad_x;
  /* Optional head-split store (c_heads > 0): the [M, N] result is written
   * as [M / R, H, R, N / H] with H = c_heads, R = c_head_rows, i.e. the
   * transpose(split_last_dim(mult(x, w)), 1, 2) of nn::MultiHeadAttention's
   * query / key / value projections (include/nn/multi_head.h) done by the
   * product's store: element (m, n) at c[((m / R) * H + n / Dh) * R * Dh +
   * (m % R) * Dh + n % Dh], Dh = N / H.  Unbatched, TF32 / 3xTF32, dense C
   * (ldc 0 or N), no addend, beta, GELU or GELU backward; N % H == 0,
   * M % R == 0, Dh and R multiples of 32, every C 16-byte aligned.  Groups
   * (GROUP_N) share the layout. */
  uint32_t c_heads, c_head_rows;
} tl_gemm_desc;
int tl_gemm(const tl_gemm_desc *desc, void *stream);
size_t tl_gemm_workspace_size(const tl_gemm_desc *desc);
/* 1 when tl_gemm runs this descriptor on the tcgen05 tensor-core kernel, 0
 * when it would take the CUDA-core kernel (TL_GEMM_FP32, fewer than 2^20
 * multiply-adds, operands TMA cannot address) or the descriptor is invalid.
 * Products that only the tensor-core path accepts (a head-split store) are
 * formed only when this holds.  No counterpart in the reference (its mult
 * has one Metal kernel, src/my_metal/runtime.cpp:375-505). */
int tl_gemm_on_tensor_cores(const tl_gemm_desc *desc);
/* Launch counts of tl_gemm since the library loaded: on the tensor cores,
 * on the CUDA cores, and the CUDA-core launches of products that asked for
 * tensor cores but whose operands that path refused (a layout regression
 * shows here instead of only as a slowdown).  NULL pointers are skipped. */
void tl_gemm_counters(uint64_t *tensor_core, uint64_t *cuda_core, uint64_t *cuda_core_refused);

/* -------------------------------------------------------------- attention */
/* The attention core of nn::MultiHeadAttention (include/nn/multi_head.h:
 * 45-52) after the projections, for every batch b and head h:
 *   S = Q_bh K_bh^T / divisor[0] + mask        (mask optional, [T, T])
 *   P = softmax_rows(S)   -> p [B, H, T, T]    (kept for the backward)
 *   O_bh = P V_bh         -> o (q's layout)
 * q, k, v, o and the gradients share one layout: [B, H, T, D] (the tensors
 * the reference's head split produces) or [B, T, H, D] (the projections
 * before the split; each head is then read and written in place).  divisor
 * is a device scalar (sqrt(D) in the reference), mask is added after the
 * divide (causal_mask, include/nn/attention.h:10-22: -inf above the
 * diagonal).  Products in `precision` (tl_gemm_precision), softmax fp32. */
enum tl_attention_layout { TL_ATTN_BHTD = 0, TL_ATTN_BTHD = 1 };
int tl_attention_fwd(const float *q, const float *k, const float *v, const float *divisor,
                     const float *mask, float *p, float *o, uint32_t B, uint32_t T, uint32_t H,
                     uint32_t D, int32_t layout, int32_t precision, void *workspace,
                     size_t workspace_bytes, void *stream);
/* Its backward (the product rules and SFTMX_DERIVATIVE, include/passes/
 * execute.h:187-232,291-308): dq, dk, dv from d_o and the forward's p. */
int tl_attention_bwd(const float *q, const float *k, const float *v, const float *p,
                     const float *divisor, const float *d_o, float *dq, float *dk, float *dv,
                     uint32_t B, uint32_t T, uint32_t H, uint32_t D, int32_t layout,
                     int32_t precision, void *workspace, size_t workspace_bytes, void *stream);
/* Scratch of either call: the scores (forward), their gradient and the
 * softmax gradient (backward). */
size_t tl_attention_workspace_size(uint32_t B, uint32_t T, uint32_t H, uint32_t D);

/* Fused passes of the same attention for T <= 192 and D == 64 on operands
 * with their own strides (the runtime's fused attention ops).  A view is
 * one [T, D] block per (batch b, head h): element (t, d) of block (b, h) at
 * p + b * batch_stride + h * head_stride + t * row_stride + d, or, when
 * `transposed`, at p + b * batch_stride + h * head_stride + d * row_stride
 * + t (only k may be transposed).  p and ds are dense [B, H, T, T].
 *   TL_ATTN_FORWARD      q, k, v, divisor, mask (optional) -> p, o
 *   TL_ATTN_BACKWARD_Q   d_o, v, k, p, divisor -> ds = P * (dP - rowsum(dP
 *                        * P)) / divisor with dP = dO V^T, dq = ds K
 *   TL_ATTN_PRODUCT_TN   dk = ds^T q: one [T, T]^T x [T, D] product per
 *                        block (dK = dS^T Q, dV = P^T dO) */
enum tl_attn_pass { TL_ATTN_FORWARD = 0, TL_ATTN_BACKWARD_Q = 1, TL_ATTN_PRODUCT_TN = 2 };
typedef struct tl_attn_view {
  const float *p;
  uint64_t batch_stride, head_stride, row_stride; /* elements */
  int32_t transposed;
  int32_t reserved;
} tl_attn_view;
typedef struct tl_attn_desc {
  int32_t pass; /* tl_attn_pass */
  uint32_t B, T, H, D;
  tl_attn_view q, k, v, o, d_o, dq, dk;
  const float *divisor, *mask;
  float *p, *ds;
  /* forward scratch (>= 16 bytes, optional): a word recording whether the
   * mask is the causal one (-inf above the diagonal, 0 elsewhere), which
   * the kernel then applies without reading it and skips the fully masked
   * key blocks */
  void *workspace;
  uint64_t workspace_bytes;
  /* optional: a word tl_attention_mask_check has already set for `mask`;
   * the forward then reads it and runs no check of its own (a program
   * checks its mask once, not once per layer) */
  const uint32_t *mask_flag;
} tl_attn_desc;
/* 1 when the fused kernels take this descriptor, 0 when not (no launch). */
int tl_attention_fused_supported(const tl_attn_desc *d);
/* TL_ERR_UNSUPPORTED when they do not. */
int tl_attention_fused(const tl_attn_desc *d, void *stream);

/* Test of the bounded on-device waits (no counterpart in the reference):
 * one CTA allocates TMEM, waits on an mbarrier nothing arrives at for at
 * most limit_ns (<= 1 s), raises TL_FLAG_TIMEOUT, frees TMEM and returns;
 * *waited_us (device memory) receives how long it waited.  The path every
 * tensor-core kernel of this library takes when a wait gives up. */
int tl_check_wait_timeout(uint64_t limit_ns, uint32_t *waited_us, void *stream);

/* Flash attention for any T and 64-wide heads: the same attention as
 * tl_attention_fused (the executor's composite of include/nn/multi_head.h:
 * 45-52 and its backward through SFTMX_DERIVATIVE, include/passes/
 * execute.h:187-232,291-308) without a [T, T] tensor in HBM.  The forward
 * leaves O and the row log-sum-exp lse[b, h, t] = ln sum_k e^{S[t, k]} of
 * the scores S = Q K^T / divisor + mask; the backward recomputes P = e^(S -
 * lse) on the tensor cores and uses delta[b, h, t] = sum_d dO * O (scratch)
 * for the softmax derivative's row sum.  Views as in tl_attn_desc (only k
 * may be stored transposed).  mask is optional ([T, T], added after the
 * divide); mask_flag (optional device word, tl_attention_mask_check) marks
 * it as the causal mask, which the kernels then apply by position and whose
 * zero blocks they skip.  TF32 products, fp32 softmax; deterministic. */
typedef struct tl_flash_desc {
  uint32_t B, T, H, D; /* D must be 64 */
  tl_attn_view q, k, v, o, d_o, dq, dk, dv;
  const float *divisor;       /* device scalar (sqrt(D) in the reference)  */
  const float *mask;          /* optional [T, T]                            */
  const uint32_t *mask_flag;  /* optional: nonzero = mask is causal         */
  float *lse;                 /* [B, H, T]                                  */
  float *delta;               /* [B, H, T] backward scratch                 */
} tl_flash_desc;
/* 1 when the flash kernels take this descriptor (16-byte aligned operands
 * and strides, D == 64), else 0. */
int tl_flash_attention_supported(const tl_flash_desc *d);
/* q, k, v, divisor, mask -> o, lse */
int tl_flash_attention_fwd(const tl_flash_desc *d, void *stream);
/* q, k, v, o, d_o, lse, divisor, mask -> dq, dk, dv (delta scratch) */
int tl_flash_attention_bwd(const tl_flash_desc *d, void *stream);
/* P = softmax of the scores ([B, H, T, T] dense) from q, k and lse: the
 * forward's probabilities for a reader other than the flash backward. */
int tl_flash_attention_probs(const tl_flash_desc *d, float *p, void *stream);
/* *flag (device word) = 1 when mask ([T, T]) is nn::causal_mask's (-inf
 * above the diagonal, 0 elsewhere; include/nn/attention.h:10-22), else 0. */
int tl_attention_mask_check(const float *mask, uint32_t T, uint32_t *flag, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* TEMPLIT_CUDA_H */
