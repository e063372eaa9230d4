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

__global__ void __launch_bounds__(256) cast_params_kernel(CastTable t) {
  const mednext_cast_entry& e = t.e[blockIdx.y];
  const int64_t n = e.rows * e.cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    // i indexes the destination; a transposed destination is cols x rows
    int64_t src = i;
    if (e.transpose) {
      const int64_t r = i % e.rows, cidx = i / e.rows;
      src = r * e.cols + cidx;
    }
    const float v = __ldg(e.src + src);
    switch (e.out_dtype) {
      case MEDNEXT_BFLOAT16: store_as<__nv_bfloat16>(e.dst, i, v); break;
      case MEDNEXT_FLOAT16: store_as<__half>(e.dst, i, v); break;
      default: static_cast<float*>(e.dst)[i] = round_via(v, e.via_dtype); break;
    }
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
  const unsigned bx = (unsigned)std::min<int64_t>((most + 255) / 256, 1024);
  cast_params_kernel<<<dim3(bx, (unsigned)count), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(t);
  return record_launch();
}
