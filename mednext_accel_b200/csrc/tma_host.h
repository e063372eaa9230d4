// Host side of the TMA tensor maps: the driver's cuTensorMapEncodeTiled, found
// through the runtime's entry-point query (no link-time driver dependency), and
// encoders for contiguous 2-, 3- and 4-dimensional tensors.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace mednext {
namespace tma {

inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

template <typename T>
inline CUtensorMapDataType tma_dtype();
template <>
inline CUtensorMapDataType tma_dtype<__nv_bfloat16>() { return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; }
template <>
inline CUtensorMapDataType tma_dtype<__half>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT16; }
template <>
inline CUtensorMapDataType tma_dtype<float>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT32; }

// [d2][d1][d0] tensor, box (b0, b1, 1)
template <typename T>
inline bool encode3(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint32_t b0, uint32_t b1,
             CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {d0 * sizeof(T), d0 * d1 * sizeof(T)};
  const cuuint32_t box[3] = {b0, b1, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, tma_dtype<T>(), 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
template <typename T>
inline bool encode2(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint32_t b0, uint32_t b1,
             CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {d0, d1};
  const cuuint64_t strides[1] = {d0 * sizeof(T)};
  const cuuint32_t box[2] = {b0, b1};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, tma_dtype<T>(), 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [d3][d2][d1][d0] tensor, box (b0, b1, 1, 1), no swizzle: one plane tile of a
// volume per load (the depthwise kernels' halo tiles).  row_pitch: elements
// between consecutive d0-rows (0 = d0); columns past d0 read as zeros.
template <typename T>
inline bool encode4(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t d3, uint32_t b0,
                    uint32_t b1, uint64_t row_pitch = 0) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const uint64_t rp = row_pitch > 0 ? row_pitch : d0;
  const cuuint64_t dims[4] = {d0, d1, d2, d3};
  const cuuint64_t strides[3] = {rp * sizeof(T), rp * d1 * sizeof(T), rp * d1 * d2 * sizeof(T)};
  const cuuint32_t box[4] = {b0, b1, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(m, tma_dtype<T>(), 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The depthwise tensor-core operand: x [nc][d][h][w] viewed as
// (8 elements, h, d, w / 8 chunks, nc) with strides (2 B, w, h*w, 16 B, d*h*w), box
// (8, bh, bd, bc, 1): a copy lands as [chunk][plane][row] x 16 bytes.
template <typename T>
inline bool encode_dw_tc(CUtensorMap* m, const void* base, uint64_t w, uint64_t h, uint64_t d, uint64_t nc,
                         uint32_t bh, uint32_t bd, uint32_t bc) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const uint64_t e = 16 / sizeof(T);
  const cuuint64_t dims[5] = {e, h, d, w / e, nc};
  const cuuint64_t strides[4] = {w * sizeof(T), w * h * sizeof(T), 16, w * h * d * sizeof(T)};
  const cuuint32_t box[5] = {(cuuint32_t)e, bh, bd, bc, 1};
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return fn(m, tma_dtype<T>(), 5, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tma
}  // namespace mednext
