// CUDA-core fp32 GEMM: the exact-fp32 path of tl_gemm (TL_GEMM_FP32) and the
// path for operands the tensor-core kernel cannot take (rows whose byte
// length is not a multiple of 16, which TMA cannot address).  Operands and
// C are addressed through their row strides (lda, ldb, ldc).
//
// 128x128x8 CTA tile, 256 threads, 8x8 outputs per thread, operands staged
// through shared memory in k-major order so every thread reads its 8 rows
// and 8 columns as two float4 each.  Transposed operands (trans_a/trans_b)
// are read in their stored order and transposed on the way into shared
// memory, so the executor's materialised transposes are not needed.
#include "gemm_common.cuh"

namespace tl {
namespace {

constexpr int BM = 128, BN = 128, BK = 8, TM = 8, TN = 8;

__global__ void __launch_bounds__(256)
sgemm_kernel(GemmArgs g) {
  pdl_enter();
  __shared__ __align__(16) float As[2][BK][BM];
  __shared__ __align__(16) float Bs[2][BK][BN];
  const uint32_t batch = blockIdx.z;
  uint64_t oa, ob, oc;
  batch_offsets(g, batch, oa, ob, oc);
  const float *A = g.a + oa;
  const float *B = g.b + ob;
  float *C = g.c + oc;
  const uint32_t M = g.m, N = g.n, K = g.k;
  const uint32_t m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

  // each thread stages 4 elements of A and 4 of B per k-tile
  auto load_tiles = [&](int buf, uint32_t k0) {
    if (!g.trans_a) {  // A[m][k] at A[m*K + k]: thread -> (row tid/2, k half)
      const uint32_t r = tid / 2, kc = (tid % 2) * 4;
      const uint32_t m = m0 + r;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t k = k0 + kc + q;
        As[buf][kc + q][r] = (m < M && k < K) ? A[static_cast<size_t>(m) * g.lda + k] : 0.0f;
      }
    } else {  // A stored [K][M]: thread -> (k row tid/32, 4 consecutive m)
      const uint32_t kr = tid / 32, mc = (tid % 32) * 4;
      const uint32_t k = k0 + kr;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t m = m0 + mc + q;
        As[buf][kr][mc + q] = (m < M && k < K) ? A[static_cast<size_t>(k) * g.lda + m] : 0.0f;
      }
    }
    if (!g.trans_b) {  // B[k][n] at B[k*N + n]
      const uint32_t kr = tid / 32, nc = (tid % 32) * 4;
      const uint32_t k = k0 + kr;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t n = n0 + nc + q;
        Bs[buf][kr][nc + q] = (n < N && k < K) ? B[static_cast<size_t>(k) * g.ldb + n] : 0.0f;
      }
    } else {  // B stored [N][K]
      const uint32_t r = tid / 2, kc = (tid % 2) * 4;
      const uint32_t n = n0 + r;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t k = k0 + kc + q;
        Bs[buf][kc + q][r] = (n < N && k < K) ? B[static_cast<size_t>(n) * g.ldb + k] : 0.0f;
      }
    }
  };

  const uint32_t ktiles = (K + BK - 1) / BK;
  load_tiles(0, 0);
  __syncthreads();
  for (uint32_t kt = 0; kt < ktiles; ++kt) {
    const int cur = kt & 1;
    if (kt + 1 < ktiles) load_tiles(cur ^ 1, (kt + 1) * BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[TM], b[TN];
      const float4 a0 = *reinterpret_cast<const float4 *>(&As[cur][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4 *>(&As[cur][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4 *>(&Bs[cur][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4 *>(&Bs[cur][kk][64 + tx * 4]);
      a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
      a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
      b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
      b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }

  // thread owns rows {ty*4+i, 64+ty*4+i} and cols {tx*4+j, 64+tx*4+j}
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const uint32_t m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const uint32_t n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (n >= N) continue;
      const size_t idx = static_cast<size_t>(m) * g.ldc + n;
      epilogue_store(g, C, oc, idx, n, acc[i][j]);
    }
  }
}

}  // namespace

int launch_sgemm(const GemmArgs &g, cudaStream_t s) {
  dim3 grid((g.n + BN - 1) / BN, (g.m + BM - 1) / BM, 1);
  for (uint64_t b0 = 0; b0 < g.batch_count; b0 += 65535) {
    GemmArgs gb = g;
    gb.batch_base = b0;
    grid.z = static_cast<unsigned>(g.batch_count - b0 < 65535 ? g.batch_count - b0 : 65535);
    launch_pdl(sgemm_kernel, grid, 256, 0, s, gb);
    int rc = launch_status("tl_gemm fp32");
    if (rc) return rc;
  }
  return TL_OK;
}

}  // namespace tl
