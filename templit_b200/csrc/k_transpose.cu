// Materialised axis swap (Runtime::transpose, src/my_metal/runtime.cpp:529-569;
// math.metal:566-584).  The reference decodes every output element through
// all dimensions and writes with a one-thread-per-element gather; here the
// host reduces the swap to one of two shapes:
//   * the innermost axis is not swapped: whole rows of L contiguous floats
//     move, so the kernel copies 128-bit vectors row by row;
//   * the innermost axis is swapped: x = [P, A, Q, B] -> out = [P, B, Q, A],
//     moved through 32x32 shared-memory tiles so both the read (along B) and
//     the write (along A) are coalesced.
#include "tl_common.cuh"

namespace tl {
namespace {

struct RowParams {
  int rank;                     // outer (row) dims of the output
  uint32_t oshape[TL_MAX_RANK];
  uint32_t istride[TL_MAX_RANK];  // input stride (in rows) of each output row dim
  uint32_t row_len;             // floats per row
};

template <int V>
__global__ void __launch_bounds__(256)
transpose_rows_kernel(const float *__restrict__ x, float *__restrict__ out,
                      RowParams p, uint64_t n_rows) {
  pdl_enter();
  const uint32_t per_row = p.row_len / V;
  const uint64_t total = n_rows * per_row;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       t < total; t += stride) {
    const uint64_t orow = t / per_row;
    const uint32_t col = static_cast<uint32_t>(t % per_row) * V;
    uint64_t rem = orow, irow = 0;
    for (int d = p.rank - 1; d >= 0; --d) {
      const uint64_t c = rem % p.oshape[d];
      rem /= p.oshape[d];
      irow += c * p.istride[d];
    }
    const float *src = x + irow * p.row_len + col;
    float *dst = out + orow * p.row_len + col;
    if constexpr (V == 4) *reinterpret_cast<float4 *>(dst) = *reinterpret_cast<const float4 *>(src);
    else *dst = *src;
  }
}

// x = [P, A, Q, B] -> out = [P, B, Q, A]; grid (ceil(B/32), ceil(A/32), P*Q).
__global__ void __launch_bounds__(256)
transpose_tile_kernel(const float *__restrict__ x, float *__restrict__ out,
                      uint32_t A, uint32_t Q, uint32_t B) {
  pdl_enter();
  __shared__ float tile[32][33];
  const uint32_t pq = blockIdx.z;
  const uint32_t p = pq / Q, q = pq % Q;
  const uint32_t b0 = blockIdx.x * 32, a0 = blockIdx.y * 32;
  const size_t xbase = static_cast<size_t>(p) * A * Q * B + static_cast<size_t>(q) * B;
  const size_t obase = static_cast<size_t>(p) * B * Q * A + static_cast<size_t>(q) * A;
  const size_t xrow = static_cast<size_t>(Q) * B;  // stride of A in x
  const size_t orow = static_cast<size_t>(Q) * A;  // stride of B in out
  const uint32_t tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (uint32_t i = ty; i < 32; i += 8) {
    const uint32_t a = a0 + i, b = b0 + tx;
    if (a < A && b < B) tile[i][tx] = x[xbase + a * xrow + b];
  }
  __syncthreads();
  for (uint32_t i = ty; i < 32; i += 8) {
    const uint32_t b = b0 + i, a = a0 + tx;
    if (a < A && b < B) out[obase + b * orow + a] = tile[tx][i];
  }
}

}  // namespace
}  // namespace tl

using namespace tl;

extern "C" int tl_transpose(const float *x, const uint32_t *shape, int rank,
                            int dim_a, int dim_b, float *out, void *stream) {
  if (rank < 2 || rank > TL_MAX_RANK)
    return fail(TL_ERR_INVALID, "transpose requires rank >= 2");
  if (dim_a < 0) dim_a += rank;
  if (dim_b < 0) dim_b += rank;
  if (dim_a < 0 || dim_a >= rank || dim_b < 0 || dim_b >= rank)
    return fail(TL_ERR_RANGE, "tensor dimension out of range");
  if (dim_a == dim_b) return fail(TL_ERR_INVALID, "transpose dimensions must be different");
  if (dim_a > dim_b) {
    const int t = dim_a;
    dim_a = dim_b;
    dim_b = t;
  }
  uint64_t n = 1;
  for (int i = 0; i < rank; ++i) n *= shape[i];
  if (n == 0) return TL_OK;
  if (!x || !out) return fail(TL_ERR_INVALID, "tl_transpose: null pointer");
  cudaStream_t s = as_stream(stream);
  if (shape[dim_a] == 1 || shape[dim_b] == 1)  // swapping a unit axis moves nothing
    return check_cuda(cudaMemcpyAsync(out, x, n * 4, cudaMemcpyDeviceToDevice, s),
                      "transpose copy");
  if (dim_b != rank - 1) {
    // rows of L = prod(shape[dim_b+1:]) floats move intact
    uint32_t L = 1;
    for (int i = dim_b + 1; i < rank; ++i) L *= shape[i];
    RowParams p{};
    p.rank = dim_b + 1;
    p.row_len = L;
    uint32_t in_shape_rows[TL_MAX_RANK];
    for (int i = 0; i <= dim_b; ++i) in_shape_rows[i] = shape[i];
    uint32_t istr[TL_MAX_RANK];
    uint64_t st = 1;
    for (int i = dim_b; i >= 0; --i) {
      istr[i] = static_cast<uint32_t>(st);
      st *= in_shape_rows[i];
    }
    for (int i = 0; i <= dim_b; ++i) {
      const int src = i == dim_a ? dim_b : (i == dim_b ? dim_a : i);
      p.oshape[i] = shape[src];
      p.istride[i] = istr[src];
    }
    const uint64_t rows = n / L;
    const bool vec = L % 4 == 0 && aligned16(x) && aligned16(out);
    if (vec)
      launch_pdl(transpose_rows_kernel<4>, grid_for(n / 4, 256), 256, 0, s, x, out, p, rows);
    else
      launch_pdl(transpose_rows_kernel<1>, grid_for(n, 256), 256, 0, s, x, out, p, rows);
    return launch_status("tl_transpose rows");
  }
  uint32_t P = 1, Q = 1;
  for (int i = 0; i < dim_a; ++i) P *= shape[i];
  for (int i = dim_a + 1; i < dim_b; ++i) Q *= shape[i];
  const uint32_t A = shape[dim_a], B = shape[dim_b];
  if (static_cast<uint64_t>(P) * Q > 65535u * 65535u)
    return fail(TL_ERR_RANGE, "tl_transpose: too many tiles");
  dim3 grid((B + 31) / 32, (A + 31) / 32, P * Q);
  if (grid.z > 65535u) return fail(TL_ERR_RANGE, "tl_transpose: batch too large");
  launch_pdl(transpose_tile_kernel, grid, 256, 0, s, x, out, A, Q, B);
  return launch_status("tl_transpose tiles");
}
