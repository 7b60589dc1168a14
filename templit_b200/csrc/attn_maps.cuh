// Tensor maps of attention operands: one [T, D] block per (batch, head) of a
// strided tensor, loaded as a K-major operand (rows of D, 128-byte swizzle),
// as an MN-major operand (32-wide column chunks, 32-byte-atom swizzle), or
// stored transposed ([D, T], the executor's K^T copy).
#pragma once

#include "attention_tc.h"
#include "tc_ptx.cuh"

#include <cuda.h>

namespace tl {
namespace attn_maps {

inline bool encode(CUtensorMap *map, const float *base, int rank, const cuuint64_t *dims,
                   const cuuint64_t *strides_bytes, const cuuint32_t *box,
                   CUtensorMapSwizzle swz) {
  EncodeTiledFn enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, static_cast<cuuint32_t>(rank),
             const_cast<float *>(base), dims, strides_bytes, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [T, D] head blocks as the 4-D tensor (D, T, H, B); box 32 columns x rows.
// Loaded once per 32 columns: K-major operand blocks [D / 32][rows][32].
inline bool rows(CUtensorMap *map, const HeadView &v, const AttnDims &d, uint32_t hd,
                 uint32_t box_rows) {
  const cuuint64_t dims[4] = {hd, d.T, d.H, d.B};
  const cuuint64_t st[3] = {v.ld * 4, v.sh * 4, v.sb * 4};
  const cuuint32_t box[4] = {32, box_rows, 1, 1};
  return encode(map, v.p, 4, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// [T, D] head blocks as (32, T, D / 32, H, B); box 32 x rows x D / 32: one
// load brings the MN-major operand layout [D / 32][rows][32].
inline bool rows_mn(CUtensorMap *map, const HeadView &v, const AttnDims &d, uint32_t hd,
                    uint32_t box_rows) {
  const cuuint64_t dims[5] = {32, d.T, hd / 32, d.H, d.B};
  const cuuint64_t st[4] = {v.ld * 4, 128, v.sh * 4, v.sb * 4};
  const cuuint32_t box[5] = {32, box_rows, hd / 32, 1, 1};
  return encode(map, v.p, 5, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
}

// Transposed [D, T] head blocks as (T, D, H, B); box 32 positions x D rows,
// 128-byte swizzle (a K-major operand over T) or 32-byte atoms (an MN-major
// operand over D).
inline bool trans(CUtensorMap *map, const HeadView &v, const AttnDims &d, uint32_t hd,
                  CUtensorMapSwizzle swz) {
  const cuuint64_t dims[4] = {d.T, hd, d.H, d.B};
  const cuuint64_t st[3] = {v.ld * 4, v.sh * 4, v.sb * 4};
  const cuuint32_t box[4] = {32, hd, 1, 1};
  return encode(map, v.p, 4, dims, st, box, swz);
}

}  // namespace attn_maps
}  // namespace tl
