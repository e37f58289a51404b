// Host-side TMA descriptors for [B, H, T, D] views (16-bit elements).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "kda_internal.h"

namespace kda {

inline PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 4-D map (D, T, H, B innermost first) with a [64 x 64] box and 128B swizzle:
// one box is a [64 tokens x 64 channels] tile.  Size-1 dimensions get a
// contiguous stride (their stride is never used to address memory).
inline bool make_tmap_bhtd(CUtensorMap *map, const View &v, int B, int H, int T, int D, bool bf16) {
  auto enc = tmap_encoder();
  if (enc == nullptr) return false;
  const uint64_t esz = 2;
  uint64_t st = (uint64_t)v.st * esz, sh = (uint64_t)v.sh * esz, sb = (uint64_t)v.sb * esz;
  if (T == 1 || st == 0) st = (uint64_t)D * esz;
  if (H == 1 || sh == 0) sh = st * (uint64_t)T;
  if (B == 1 || sb == 0) sb = sh * (uint64_t)H;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)T, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {st, sh, sb};
  cuuint32_t box[4] = {64, 64, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                   const_cast<void *>(v.data), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace kda
