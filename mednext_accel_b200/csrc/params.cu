// mednext_cast_params: the fused block's fp32 parameters cast (and, for the
// input-grad GEMMs, transposed) to the compute type in one launch, instead of
// one small kernel per parameter and per use.
#include "plan.h"

namespace mednext {
namespace {

struct CastTable {
  mednext_cast_entry e[MEDNEXT_CAST_MAX_ENTRIES];
};

template <typename T>
__device__ __forceinline__ void store_as(void* dst, int64_t i, float v) {
  static_cast<T*>(dst)[i] = from_acc<T>(v);
}
__device__ __forceinline__ float round_via(float v, int via) {
  if (via == MEDNEXT_BFLOAT16) return __bfloat162float(__float2bfloat16_rn(v));
  if (via == MEDNEXT_FLOAT16) return __half2float(__float2half_rn(v));
  return v;
}

__device__ __forceinline__ void store_cast(const mednext_cast_entry& e, int i, float v) {
  switch (e.out_dtype) {
    case MEDNEXT_BFLOAT16: store_as<__nv_bfloat16>(e.dst, i, v); break;
    case MEDNEXT_FLOAT16: store_as<__half>(e.dst, i, v); break;
    default: static_cast<float*>(e.dst)[i] = round_via(v, e.via_dtype); break;
  }
}

// blockIdx.y selects the entry.  A plain entry is a flat, coalesced loop; a
// transposed one (dst = src^T, cols x rows) goes through 32 x 32 shared-memory
// tiles so that both the reads and the writes are coalesced.  Sizes are < 2^31.
constexpr int kCastTile = 32;
__global__ void __launch_bounds__(256) cast_params_kernel(CastTable t) {
  const mednext_cast_entry& e = t.e[blockIdx.y];
  const int rows = (int)e.rows, cols = (int)e.cols;
  if (!e.transpose) {
    const int n = rows * cols;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
      store_cast(e, i, __ldg(e.src + i));
    return;
  }
  __shared__ float tile[kCastTile][kCastTile + 1];
  const int tx = threadIdx.x & (kCastTile - 1), ty = threadIdx.x / kCastTile;  // 32 x 8
  const int trs = (rows + kCastTile - 1) / kCastTile, tcs = (cols + kCastTile - 1) / kCastTile;
  for (int tt = blockIdx.x; tt < trs * tcs; tt += gridDim.x) {
    const int r0 = (tt / tcs) * kCastTile, c0 = (tt % tcs) * kCastTile;
    for (int y = ty; y < kCastTile; y += blockDim.x / kCastTile)
      if (r0 + y < rows && c0 + tx < cols) tile[y][tx] = __ldg(e.src + (size_t)(r0 + y) * cols + c0 + tx);
    __syncthreads();
    // dst[c][r] = src[r][c]
    for (int y = ty; y < kCastTile; y += blockDim.x / kCastTile)
      if (c0 + y < cols && r0 + tx < rows) store_cast(e, (c0 + y) * rows + r0 + tx, tile[tx][y]);
    __syncthreads();
  }
}

}  // namespace
}  // namespace mednext

using namespace mednext;

int mednext_cast_params(const mednext_cast_entry* entries, int count, mednext_stream_t stream) {
  if (entries == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  if (count <= 0 || count > MEDNEXT_CAST_MAX_ENTRIES) return MEDNEXT_ERR_BAD_SHAPE;
  CastTable t{};
  int64_t most = 1;
  for (int i = 0; i < count; ++i) {
    const mednext_cast_entry& e = entries[i];
    if (e.src == nullptr || e.dst == nullptr) return MEDNEXT_ERR_NULL_POINTER;
    if (e.rows <= 0 || e.cols <= 0 || e.rows * e.cols >= ((int64_t)1 << 31)) return MEDNEXT_ERR_BAD_SHAPE;
    if (e.out_dtype != MEDNEXT_BFLOAT16 && e.out_dtype != MEDNEXT_FLOAT16 && e.out_dtype != MEDNEXT_FLOAT32)
      return MEDNEXT_ERR_BAD_DTYPE;
    if (e.via_dtype != MEDNEXT_FLOAT32 && e.via_dtype != MEDNEXT_BFLOAT16 && e.via_dtype != MEDNEXT_FLOAT16)
      return MEDNEXT_ERR_BAD_DTYPE;
    const size_t esz = e.out_dtype == MEDNEXT_FLOAT32 ? 4 : 2;
    if ((reinterpret_cast<uintptr_t>(e.src) & 3) || (reinterpret_cast<uintptr_t>(e.dst) % esz))
      return MEDNEXT_ERR_ALIGNMENT;
    t.e[i] = e;
    most = std::max(most, e.rows * e.cols);
  }
  // enough blocks for the largest entry at 256 elements per block (a transposed entry
  // needs a quarter of them: one 32 x 32 tile per block)
  const unsigned bx = (unsigned)std::min<int64_t>((most + 255) / 256, 1024);
  cast_params_kernel<<<dim3(bx, (unsigned)count), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(t);
  return record_launch();
}
