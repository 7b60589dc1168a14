// cuda::Runtime: the TempLit runtime backend for NVIDIA B200 (sm_100a).
//
// Drop-in counterpart of metal::Runtime (include/my_metal/runtime.h:10-181
// in JTPuffer/TempLit): the same public method set, the same
// destination-tensor calling convention and the same exception types, so
// that passes::Compiled's typed executor (include/passes/execute.h) and the
// optimisers (include/optimiser/AdamW.h, sgd.h) run on it unchanged:
//
//   static_assert(passes::Runnable<RTensor<cuda::CUDA, float>, cuda::Runtime>);
//
// Execution model.  Like a Metal command buffer, start() opens a recording
// window; every op method validates its arguments (throwing exactly where
// the Metal runtime throws) and appends one entry to the window's program.
// submit() optimises the program (fusing the executor's op patterns into
// single kernels) and launches it on the backend stream, replaying a CUDA
// graph when the same program was seen before; wait() blocks until it has
// finished and surfaces device-side errors as exceptions.
#pragma once

#include "RTensor/RTensor.h"
#include "my_cuda/cuda.h"
#include "my_cuda/storage.h"

#include <cstddef>
#include <cstdint>
#include <memory>
#include <span>
#include <string>
#include <string_view>

namespace cuda {

enum class ReduceKind { Sum, Max };

// Counters of the last submitted programs (for benchmarks and tests).
struct RuntimeStats {
  uint64_t windows = 0;         // submitted programs
  uint64_t ops_recorded = 0;    // runtime calls recorded in total
  uint64_t ops_launched = 0;    // ops launched after fusion, in total
  uint64_t kernel_launches = 0; // kernels this runtime launched (graph replays count their nodes)
  uint64_t graph_replays = 0;   // programs served by replaying a captured graph
  uint64_t graph_captures = 0;  // graphs captured
  uint64_t fused_ops = 0;       // recorded ops folded into fused kernels
  uint64_t host_record_ns = 0;  // host time from start() to submit(), in total
  uint64_t host_submit_ns = 0;  // host time inside submit() (optimise + launch), in total
  uint64_t optimiser_cache_hits = 0;  // programs whose optimised form was reused
  uint64_t flash_forward = 0;   // flash attention forwards launched (P left virtual)
  uint64_t flash_backward = 0;  // flash attention backwards launched (P recomputed)
  uint64_t flash_rebuilt = 0;   // virtual P tensors written out for another reader
};

class Runtime {
public:
  using Mat = RTensor<CUDA, kernel_type>;
  using IndexMat = RTensor<CUDA, index_type>;

  Runtime();
  Runtime(const Runtime &) = delete;
  Runtime &operator=(const Runtime &) = delete;
  ~Runtime();

  void start();
  void submit();
  void wait();
  void abort() noexcept;
  void cleanup() noexcept;

  // Per-op device timing of every submitted program until end_profile(),
  // written as JSON to output_path.
  void start_profile(std::string_view output_path);
  void end_profile();

  void reduce_to_shape(const Mat &a, std::span<const uint32_t> output_shape, Mat &output,
                       ReduceKind kind = ReduceKind::Max);
  void add(const Mat &, const Mat &, Mat &);
  void add(const Mat &, kernel_type, Mat &);
  void sub(const Mat &, const Mat &, Mat &);
  void mult(const Mat &, const Mat &, Mat &);
  void hadamard(const Mat &, const Mat &, Mat &);
  void divide(const Mat &, const Mat &, Mat &);
  void divide(const Mat &, kernel_type, Mat &);
  void sigmoid(const Mat &, Mat &);
  void sqrt(const Mat &, Mat &);
  void pow(const Mat &, kernel_type, Mat &);
  void exp(const Mat &, Mat &);
  void sum(const Mat &, Mat &);
  void sum(const Mat &, size_t axis, Mat &);
  void transpose(const Mat &, Mat &, int32_t dim_a = -2, int32_t dim_b = -1);
  void split_last_dim(const Mat &, Mat &, uint32_t outer, uint32_t inner);
  void merge_last_dims(const Mat &, Mat &, uint32_t outer, uint32_t inner);
  void sum_to_shape(const Mat &, std::span<const uint32_t>, Mat &);
  void max_to_shape(const Mat &, std::span<const uint32_t>, Mat &);
  void softmax(const Mat &, Mat &);
  void cross_entropy(const Mat &, const IndexMat &, Mat &);
  void cross_entropy_derivative(const Mat &, const IndexMat &, Mat &);
  void sqe(const Mat &, const Mat &, Mat &);
  void argmax(const Mat &, IndexMat &);
  void embedding_lookup(const Mat &, const IndexMat &, Mat &);
  void gather_rows(const Mat &, const IndexMat &, Mat &);
  void scatter_add_rows(const Mat &, const IndexMat &, const Mat &, Mat &);
  void scatter_index(const Mat &, const IndexMat &, Mat &);
  void RMS(const Mat &, Mat &);
  void RMSNorm(const Mat &, Mat &);
  void GELU(const Mat &, Mat &);
  void GELU_derivative(const Mat &, Mat &);
  void accumulate_gradient_squared_norm(const Mat &gradient, Mat &squared_norm);
  void clip_gradient(const Mat &gradient, const Mat &squared_norm, kernel_type max_norm,
                     Mat &destination);
  void adamW(const Mat &parameter, const Mat &gradient, Mat &destination, Mat &momentum1,
             Mat &momentum2, const Mat &beta1, const Mat &beta2, const Mat &decay,
             const Mat &learning_rate, kernel_type epsilon, uint32_t step);
  void copy(const Mat &a, Mat &output);

  // ---- B200 additions (no Metal counterpart) -------------------------
  // Program optimisation switches (all on by default).
  void set_fusion(bool enabled);
  void set_graphs(bool enabled);
  // GEMM arithmetic of mult: TL_GEMM_TF32 (tcgen05 tensor cores, default)
  // or TL_GEMM_FP32 (exact fp32 products on CUDA cores).
  void set_gemm_precision(int precision);
  // Attention composites on the flash kernels: the forward keeps the
  // softmax output P as its recipe (row log-sum-exp) instead of writing it,
  // the backward recomputes it, and any other reader gets it rebuilt first.
  // Mode 0: never; 1 (default): sequences longer than the short-sequence
  // fused kernels take (T > 192), which are faster up to there; 2: always.
  // The environment variable TL_FLASH_ATTENTION sets the initial mode.
  void set_flash_attention(int mode);
  // Data parallelism: an NCCL communicator (ncclComm_t as void*).  When set,
  // the program of a window that updates parameters (AdamW) first
  // sum-reduces every gradient it reads across the communicator's ranks, so
  // all ranks clip and step with the same global gradient.
  void set_communicator(void *nccl_comm);
  // Deferred wait (off by default): wait() returns without synchronising,
  // so the host records the next window while the GPU runs this one.
  // Storage reads still synchronise; a device error (embedding id out of
  // range, kernel timeout) is raised by a later wait() instead of this one.
  void set_deferred_wait(bool enabled);
  const RuntimeStats &stats() const;

  struct Impl;

private:
  std::unique_ptr<Impl> impl_;
};

}  // namespace cuda
