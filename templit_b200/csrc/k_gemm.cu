// tl_gemm: validates the descriptor and routes to the tcgen05 tensor-core
// kernel (TL_GEMM_TF32, TL_GEMM_3XTF32) or the CUDA-core fp32 kernel
// (TL_GEMM_FP32, tiny problems, and operands TMA cannot address).
#include "gemm_common.cuh"

#include <atomic>
#include <cstdlib>
#include <cstring>

namespace tl {
namespace {

// Problems below this many multiply-adds finish faster on CUDA cores than a
// persistent tensor-core launch can be set up.
constexpr uint64_t kTcMinMacs = 1ull << 20;

bool force_fp32_from_env() {
  static const bool v = [] {
    const char *e = std::getenv("TL_GEMM_FORCE_FP32");
    return e && std::strcmp(e, "0") != 0;
  }();
  return v;
}

int to_args(const tl_gemm_desc *d, GemmArgs &g) {
  if (!d) return fail(TL_ERR_INVALID, "tl_gemm: null descriptor");
  if (d->batch_rank > TL_GEMM_MAX_BATCH_RANK)
    return fail(TL_ERR_INVALID, "tl_gemm: batch rank too large");
  if (d->beta != 0.0f && d->beta != 1.0f)
    return fail(TL_ERR_INVALID, "tl_gemm: beta must be 0 or 1");
  if (d->precision < TL_GEMM_TF32 || d->precision > TL_GEMM_3XTF32)
    return fail(TL_ERR_INVALID, "tl_gemm: unknown precision");
  g = GemmArgs{};
  g.a = d->a;
  g.b = d->b;
  g.c = d->c;
  g.bias = d->bias;
  g.gelu_out = d->gelu_out;
  g.m = d->m;
  g.n = d->n;
  g.k = d->k;
  g.trans_a = d->trans_a != 0;
  g.trans_b = d->trans_b != 0;
  g.split_tf32 = d->precision == TL_GEMM_3XTF32;
  g.beta = d->beta;
  if (d->addend && d->beta != 0.0f && d->addend != d->c)
    return fail(TL_ERR_INVALID, "tl_gemm: addend with beta = 1 must be C");
  g.addend = d->addend ? d->addend : (d->beta != 0.0f ? d->c : nullptr);
  g.gelu_grad_x = d->gelu_grad_x;
  if (g.gelu_grad_x && (g.addend || d->gelu_out || d->group_mode != TL_GEMM_GROUP_NONE))
    return fail(TL_ERR_INVALID, "tl_gemm: gelu_grad_x takes no addend, beta, gelu_out or groups");
  g.c_heads = d->c_heads;
  g.c_head_rows = d->c_heads ? d->c_head_rows : 0;
  if (d->c_heads) {
    const uint32_t H = d->c_heads, R = d->c_head_rows;
    if (g.addend || d->gelu_out || g.gelu_grad_x || d->batch_rank ||
        d->group_mode == TL_GEMM_GROUP_K || (d->ldc && d->ldc != d->n) ||
        d->precision == TL_GEMM_FP32)
      return fail(TL_ERR_INVALID, "tl_gemm: a head-split store takes an unbatched TF32 product "
                                  "with dense C and no addend, beta or GELU");
    if (R == 0 || d->n % H || d->m % R || (d->n / H) % 32 || R % 32)
      return fail(TL_ERR_INVALID, "tl_gemm: head-split store needs N % heads == 0, "
                                  "M % rows == 0 and head width and rows multiples of 32");
  }
  g.group_mode = d->group_mode;
  g.groups = 1;
  if (d->group_mode != TL_GEMM_GROUP_NONE) {
    if (d->group_mode != TL_GEMM_GROUP_N && d->group_mode != TL_GEMM_GROUP_K)
      return fail(TL_ERR_INVALID, "tl_gemm: unknown group mode");
    if (d->groups < 2 || d->groups > TL_GEMM_MAX_GROUPS)
      return fail(TL_ERR_INVALID, "tl_gemm: group count out of range");
    g.groups = d->groups;
    for (uint32_t i = 0; i < g.groups; ++i) {
      g.ag[i] = d->group_mode == TL_GEMM_GROUP_K ? d->a_group[i] : d->a;
      g.bg[i] = d->b_group[i];
      g.cg[i] = d->group_mode == TL_GEMM_GROUP_N ? d->c_group[i] : d->c;
      g.biasg[i] = d->group_mode == TL_GEMM_GROUP_N ? d->bias_group[i] : d->bias;
      if (!g.ag[i] || !g.bg[i] || !g.cg[i])
        return fail(TL_ERR_INVALID, "tl_gemm: null group operand");
    }
    if (d->group_mode == TL_GEMM_GROUP_N && (d->gelu_out || d->addend || d->beta != 0.0f))
      return fail(TL_ERR_INVALID, "tl_gemm: N-grouped products take no GELU, addend or beta");
    if (d->group_mode == TL_GEMM_GROUP_K && d->gelu_out)
      return fail(TL_ERR_INVALID, "tl_gemm: K-grouped products take no GELU");
    if (d->group_mode == TL_GEMM_GROUP_N && d->c_group[0] != d->c)
      return fail(TL_ERR_INVALID, "tl_gemm: c_group[0] must be c");
    g.a = g.ag[0];
    g.b = g.bg[0];
  }
  g.lda = d->lda ? d->lda : (g.trans_a ? g.m : g.k);
  g.ldb = d->ldb ? d->ldb : (g.trans_b ? g.k : g.n);
  g.ldc = d->ldc ? d->ldc : g.n;
  if (g.lda < (g.trans_a ? g.m : g.k) || g.ldb < (g.trans_b ? g.k : g.n) || g.ldc < g.n)
    return fail(TL_ERR_INVALID, "tl_gemm: row stride shorter than the row");
  // batch dims, merging neighbours that every operand walks as one (the
  // outer stride is the inner stride times the inner extent)
  g.batch_rank = 0;
  g.batch_count = 1;
  for (uint32_t i = 0; i < d->batch_rank; ++i) {
    const uint32_t n = d->batch_shape[i];
    g.batch_count *= n;
    if (n == 1) continue;
    const uint64_t sa = d->a_batch_stride[i], sb = d->b_batch_stride[i],
                   sc = d->c_batch_stride[i];
    if (g.batch_rank > 0) {
      const uint32_t j = g.batch_rank - 1;
      if (g.sa[j] == sa * n && g.sb[j] == sb * n && g.sc[j] == sc * n) {
        g.batch_shape[j] *= n;
        g.sa[j] = sa;
        g.sb[j] = sb;
        g.sc[j] = sc;
        continue;
      }
    }
    g.batch_shape[g.batch_rank] = n;
    g.sa[g.batch_rank] = sa;
    g.sb[g.batch_rank] = sb;
    g.sc[g.batch_rank] = sc;
    ++g.batch_rank;
  }
  return TL_OK;
}

bool wants_tc(const tl_gemm_desc *d, const GemmArgs &g) {
  const uint64_t macs = static_cast<uint64_t>(g.m) * g.n * g.k * g.batch_count;
  return d->precision != TL_GEMM_FP32 && !force_fp32_from_env() && macs >= kTcMinMacs &&
         g.k > 0;
}

// Launch counters by path (tl_gemm_counters): tensor-core launches, CUDA-core
// launches, and the CUDA-core launches of products that asked for tensor
// cores but whose operands the tensor-core path refused.
std::atomic<uint64_t> g_tc_launches{0}, g_simt_launches{0}, g_simt_refused{0};

}  // namespace
}  // namespace tl

using namespace tl;

extern "C" size_t tl_gemm_workspace_size(const tl_gemm_desc *d) {
  GemmArgs g;
  if (to_args(d, g) || g.m == 0 || g.n == 0 || g.batch_count == 0) return 0;
  if (!wants_tc(d, g)) return 0;
  size_t ws = tc_gemm_workspace(g);
  if (g.groups > 1) {  // split fallback: each product's own plan
    for (uint32_t i = 0; i < g.groups; ++i) {
      tl_gemm_desc one = *d;
      one.group_mode = TL_GEMM_GROUP_NONE;
      one.groups = 0;
      const size_t w = tl_gemm_workspace_size(&one);
      if (w > ws) ws = w;
    }
  }
  return ws;
}

extern "C" int tl_gemm_on_tensor_cores(const tl_gemm_desc *d) {
  GemmArgs g;
  if (to_args(d, g) || g.m == 0 || g.n == 0 || g.batch_count == 0) return 0;
  return wants_tc(d, g) && tc_gemm_supported(g) ? 1 : 0;
}

extern "C" void tl_gemm_counters(uint64_t *tensor_core, uint64_t *cuda_core,
                                 uint64_t *cuda_core_refused) {
  if (tensor_core) *tensor_core = g_tc_launches.load();
  if (cuda_core) *cuda_core = g_simt_launches.load();
  if (cuda_core_refused) *cuda_core_refused = g_simt_refused.load();
}

extern "C" int tl_gemm(const tl_gemm_desc *d, void *stream) {
  GemmArgs g;
  int rc = to_args(d, g);
  if (rc) return rc;
  if (g.m == 0 || g.n == 0 || g.batch_count == 0) return TL_OK;
  if (!g.c || (g.k && (!g.a || !g.b))) return fail(TL_ERR_INVALID, "tl_gemm: null pointer");
  cudaStream_t s = as_stream(stream);
  const bool tc = wants_tc(d, g);
  if (tc) {
    rc = launch_tc_gemm(g, d->workspace, d->workspace_bytes, s);
    if (rc != TL_ERR_UNSUPPORTED) {
      if (rc == TL_OK) ++g_tc_launches;
      return rc;
    }
  }
  if (g.c_heads)
    return fail(TL_ERR_UNSUPPORTED,
                "tl_gemm: a head-split store runs on the tensor-core path only (16-byte "
                "aligned operands and rows)");
  if (g.groups > 1) {
    // one product per group: N groups independently; K groups as a chain
    // accumulating into C (bias and addend with the first)
    for (uint32_t i = 0; i < g.groups; ++i) {
      tl_gemm_desc one = *d;
      one.group_mode = TL_GEMM_GROUP_NONE;
      one.groups = 0;
      one.a = g.ag[i];
      one.b = g.bg[i];
      one.c = g.cg[i];
      if (d->group_mode == TL_GEMM_GROUP_N) {
        one.bias = g.biasg[i];
      } else if (i > 0) {
        one.bias = nullptr;
        one.addend = nullptr;
        one.beta = 1.0f;
        one.gelu_out = nullptr;
      } else {
        one.gelu_out = nullptr;
      }
      rc = tl_gemm(&one, stream);
      if (rc) return rc;
    }
    return TL_OK;
  }
  ++g_simt_launches;
  if (tc) ++g_simt_refused;
  return launch_sgemm(g, s);
}
