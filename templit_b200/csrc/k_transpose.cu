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

// Division by a loop-invariant 32-bit divisor as a multiply-high and a
// shift (Granlund and Montgomery, "Division by invariant integers using
// multiplication", 1994: s = ceil(log2 d), m = floor(2^32 (2^s - d) / d) + 1,
// n / d = (mulhi(n, m) + n) >> s for every 32-bit n).
struct FastDiv {
  uint32_t d, m, s;
  FastDiv() = default;
  explicit FastDiv(uint32_t d_) : d(d_), m(0), s(0) {
    while ((1ull << s) < d) ++s;
    m = static_cast<uint32_t>(((1ull << 32) * ((1ull << s) - d)) / d + 1);
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    return static_cast<uint32_t>((static_cast<uint64_t>(__umulhi(n, m)) + n) >> s);
  }
};

// Whole rows of L floats move: x = [P, A, Q, B, L] -> out = [P, B, Q, A, L].
struct RowParams {
  FastDiv A, Q, B, vecs;  // vecs: vectors per row
  uint32_t row_len;       // floats per row
};

// One vector per thread and grid-stride step: output row o = ((p B + b) Q +
// q) A + a reads input row ((p A + a) Q + q) B + b.  32-bit indexing (the
// host checks the sizes).
template <int V>
__global__ void __launch_bounds__(256)
transpose_rows_kernel(const float *__restrict__ x, float *__restrict__ out, RowParams p,
                      uint32_t total) {
  pdl_enter();
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += stride) {
    const uint32_t orow = p.vecs.div(t);
    const uint32_t col = (t - orow * p.vecs.d) * V;
    uint32_t r = orow;
    const uint32_t r1 = p.A.div(r), a = r - r1 * p.A.d;
    const uint32_t r2 = p.Q.div(r1), q = r1 - r2 * p.Q.d;
    const uint32_t pp = p.B.div(r2), b = r2 - pp * p.B.d;
    const uint32_t irow = ((pp * p.A.d + a) * p.Q.d + q) * p.B.d + b;
    const float *src = x + static_cast<size_t>(irow) * p.row_len + col;
    float *dst = out + static_cast<size_t>(orow) * p.row_len + col;
    if constexpr (V == 4) *reinterpret_cast<float4 *>(dst) = *reinterpret_cast<const float4 *>(src);
    else *dst = *src;
  }
}

// x = [P, A, Q, B] -> out = [P, B, Q, A] through 64 x 64 tiles in shared
// memory; grid (ceil(B/64), ceil(A/64), P*Q), 256 threads.  With A and B
// multiples of 4 and 16-byte aligned pointers (`vec`) both the loads (along
// B) and the stores (along A) move 128-bit vectors, four per thread, so a
// CTA keeps 16 KB in flight.
template <bool VEC>
__global__ void __launch_bounds__(256)
transpose_tile_kernel(const float *__restrict__ x, float *__restrict__ out,
                      uint32_t A, uint32_t Q, uint32_t B) {
  pdl_enter();
  __shared__ float tile[64][65];
  const uint32_t pq = blockIdx.z;
  const uint32_t p = pq / Q, q = pq % Q;
  const uint32_t b0 = blockIdx.x * 64, a0 = blockIdx.y * 64;
  const size_t xbase = static_cast<size_t>(p) * A * Q * B + static_cast<size_t>(q) * B;
  const size_t obase = static_cast<size_t>(p) * B * Q * A + static_cast<size_t>(q) * A;
  const size_t xrow = static_cast<size_t>(Q) * B;  // stride of A in x
  const size_t orow = static_cast<size_t>(Q) * A;  // stride of B in out
  const uint32_t t = threadIdx.x;
  if (VEC) {
    const uint32_t c4 = (t & 15) * 4, r = t >> 4;  // 16 vectors per 64-wide row
#pragma unroll
    for (uint32_t i = 0; i < 64; i += 16) {
      const uint32_t a = a0 + i + r, b = b0 + c4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (a < A && b < B) v = *reinterpret_cast<const float4 *>(x + xbase + a * xrow + b);
      tile[i + r][c4] = v.x;
      tile[i + r][c4 + 1] = v.y;
      tile[i + r][c4 + 2] = v.z;
      tile[i + r][c4 + 3] = v.w;
    }
    __syncthreads();
#pragma unroll
    for (uint32_t i = 0; i < 64; i += 16) {
      const uint32_t b = b0 + i + r, a = a0 + c4;
      if (a < A && b < B)
        *reinterpret_cast<float4 *>(out + obase + b * orow + a) =
            make_float4(tile[c4][i + r], tile[c4 + 1][i + r], tile[c4 + 2][i + r],
                        tile[c4 + 3][i + r]);
    }
  } else {
    const uint32_t tx = t & 63, ty = t >> 6;
    for (uint32_t i = ty; i < 64; i += 4) {
      const uint32_t a = a0 + i, b = b0 + tx;
      if (a < A && b < B) tile[i][tx] = x[xbase + a * xrow + b];
    }
    __syncthreads();
    for (uint32_t i = ty; i < 64; i += 4) {
      const uint32_t b = b0 + i, a = a0 + tx;
      if (a < A && b < B) out[obase + b * orow + a] = tile[tx][i];
    }
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
    uint64_t L = 1, P = 1, Q = 1;
    for (int i = dim_b + 1; i < rank; ++i) L *= shape[i];
    for (int i = 0; i < dim_a; ++i) P *= shape[i];
    for (int i = dim_a + 1; i < dim_b; ++i) Q *= shape[i];
    const bool vec = L % 4 == 0 && aligned16(x) && aligned16(out);
    const uint64_t total = vec ? n / 4 : n;
    if (n >= (1ull << 32)) return fail(TL_ERR_RANGE, "tl_transpose: tensor too large");
    RowParams p;
    p.A = FastDiv(shape[dim_a]);
    p.B = FastDiv(shape[dim_b]);
    p.Q = FastDiv(static_cast<uint32_t>(Q));
    p.vecs = FastDiv(static_cast<uint32_t>(vec ? L / 4 : L));
    p.row_len = static_cast<uint32_t>(L);
    (void)P;
    if (vec)
      launch_pdl(transpose_rows_kernel<4>, grid_for(total, 256), 256, 0, s, x, out, p,
                 static_cast<uint32_t>(total));
    else
      launch_pdl(transpose_rows_kernel<1>, grid_for(total, 256), 256, 0, s, x, out, p,
                 static_cast<uint32_t>(total));
    return launch_status("tl_transpose rows");
  }
  uint32_t P = 1, Q = 1;
  for (int i = 0; i < dim_a; ++i) P *= shape[i];
  for (int i = dim_a + 1; i < dim_b; ++i) Q *= shape[i];
  const uint32_t A = shape[dim_a], B = shape[dim_b];
  if (static_cast<uint64_t>(P) * Q > 65535u * 65535u)
    return fail(TL_ERR_RANGE, "tl_transpose: too many tiles");
  dim3 grid((B + 63) / 64, (A + 63) / 64, P * Q);
  if (grid.z > 65535u) return fail(TL_ERR_RANGE, "tl_transpose: batch too large");
  if (A % 4 == 0 && B % 4 == 0 && aligned16(x) && aligned16(out))
    launch_pdl(transpose_tile_kernel<true>, grid, 256, 0, s, x, out, A, Q, B);
  else
    launch_pdl(transpose_tile_kernel<false>, grid, 256, 0, s, x, out, A, Q, B);
  return launch_status("tl_transpose tiles");
}
