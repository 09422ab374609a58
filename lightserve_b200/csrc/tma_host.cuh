// Host-side TMA tensor-map creation through the driver entry point (so the
// library links no libcuda and still loads on machines without a driver).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace lsb {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 4-D map over a [B, H, N, D] tensor with element strides {sb, sh, sn, 1}:
// dims (innermost first) D, N, H, B; box (box_d, box_rows, 1, 1); 128-byte
// swizzle; out-of-range rows read as zero.
inline int make_bhnd_map(CUtensorMap* map, const void* base, int dtype, int64_t B, int64_t H,
                         int64_t N, int64_t D, const int64_t* s, uint32_t box_d,
                         uint32_t box_rows) {
  EncodeTiledFn enc = get_encode_tiled();
  if (!enc) {
    set_error("cuTensorMapEncodeTiled unavailable (no CUDA driver?)");
    return LSB_ERR_CUDA;
  }
  const int esz = dtype_size(dtype);
  CUtensorMapDataType dt = dtype == LSB_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)N, (cuuint64_t)H, (cuuint64_t)B};
  // Strides of dims 1..3 in bytes. A size-1 dim's stride is irrelevant but
  // must still be a multiple of 16: substitute a dense one.
  int64_t sn = s[2], sh = s[1], sb = s[0];
  if (N == 1) sn = D;
  if (H == 1) sh = N * sn;
  if (B == 1) sb = H * sh;
  cuuint64_t strides[3] = {(cuuint64_t)(sn * esz), (cuuint64_t)(sh * esz), (cuuint64_t)(sb * esz)};
  cuuint32_t box[4] = {box_d, box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return LSB_ERR_CUDA;
  }
  return LSB_OK;
}

// True if a [B,H,N,D] tensor with these element strides can be described by
// make_bhnd_map: unit d-stride, 16-byte aligned base and strides.
inline bool tma_ok(const void* p, int64_t B, int64_t H, int64_t N, const int64_t* s, int esz) {
  if (!aligned16(p) || s[3] != 1) return false;
  if (N > 1 && (s[2] * esz) % 16 != 0) return false;
  if (H > 1 && (s[1] * esz) % 16 != 0) return false;
  if (B > 1 && (s[0] * esz) % 16 != 0) return false;
  if (N > 1 && s[2] <= 0) return false;
  return true;
}

}  // namespace lsb
