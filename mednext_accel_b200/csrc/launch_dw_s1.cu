// Template instantiation and launch of the depthwise kernels (stride 1) for every supported element type and kernel size.
#include "plan.h"

namespace mednext {

namespace {

template <typename T, int K>
int launch_s1_conv(const void* x, const void* wgt, const void* bias, const void* addend, void* y, GnPartial* st,
                   const S1Plan& p, int flip, cudaStream_t s) {
  constexpr int NH = K <= 3 ? 2 : 1;
  auto kern = dw_s1_conv_kernel<T, K, NH>;
  static size_t configured = 0;  // raise the opt-in limit once per instantiation
  if (p.smem > 48 * 1024 && p.smem > configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
    configured = p.smem;
  }
  kern<<<(unsigned)p.grid, p.threads, p.smem, s>>>(static_cast<const T*>(x), static_cast<const T*>(wgt),
                                                   static_cast<const T*>(bias), static_cast<const T*>(addend),
                                                   static_cast<T*>(y), st, p.g, flip);
  return record_launch();
}

template <typename T>
int finish_wgrad(const typename Elem<T>::Acc* part, void* dw, void* db, int N, int C, int tiles, int K3,
                 cudaStream_t s) {
  const int total = C * (K3 + 1);
  dw_wgrad_finish_kernel<T><<<(total + 127) / 128, 128, 0, s>>>(part, static_cast<T*>(dw), static_cast<T*>(db), N,
                                                                C, tiles, K3);
  return record_launch();
}

template <typename T, int K>
int launch_s1_wgrad(const void* x, const void* dy, void* dw, void* db, void* ws, const S1Plan& p, cudaStream_t s) {
  using Acc = typename Elem<T>::Acc;
  constexpr int NH = K <= 3 ? 2 : 1;
  Acc* part = static_cast<Acc*>(ws);
  if constexpr (K <= 3) {
    auto kern = dw_s1_wgrad_kernel<T, K, NH>;
    static size_t configured = 0;  // raise the opt-in limit once per instantiation
    if (p.smem > 48 * 1024 && p.smem > configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
    configured = p.smem;
  }
    kern<<<(unsigned)p.grid, p.threads, p.smem, s>>>(static_cast<const T*>(x), static_cast<const T*>(dy), part, p.g);
  } else {
    auto kern = dw_s1_wgrad_grouped_kernel<T, K, NH>;
    static size_t configured = 0;  // raise the opt-in limit once per instantiation
    if (p.smem > 48 * 1024 && p.smem > configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
    configured = p.smem;
  }
    kern<<<(unsigned)p.grid, p.threads, p.smem, s>>>(static_cast<const T*>(x), static_cast<const T*>(dy), part, p.g);
  }
  const int st = record_launch();
  if (st != MEDNEXT_OK) return st;
  return finish_wgrad<T>(part, dw, db, p.g.N, p.g.C, (int)s1_tiles(p), K * K * K, s);
}

}  // namespace

#define MEDNEXT_K_SWITCH(k, KC, ...)                         \
  switch (k) {                                               \
    case 1: { constexpr int KC = 1; __VA_ARGS__; } break;    \
    case 3: { constexpr int KC = 3; __VA_ARGS__; } break;    \
    case 5: { constexpr int KC = 5; __VA_ARGS__; } break;    \
    case 7: { constexpr int KC = 7; __VA_ARGS__; } break;    \
    default: return MEDNEXT_ERR_BAD_KERNEL;                  \
  }
#define MEDNEXT_T_SWITCH(dtype, TC, ...)                                     \
  switch (dtype) {                                                           \
    case MEDNEXT_FLOAT32: { using TC = float; __VA_ARGS__; } break;          \
    case MEDNEXT_BFLOAT16: { using TC = __nv_bfloat16; __VA_ARGS__; } break; \
    case MEDNEXT_FLOAT16: { using TC = __half; __VA_ARGS__; } break;         \
    case MEDNEXT_FLOAT64: { using TC = double; __VA_ARGS__; } break;         \
    default: return MEDNEXT_ERR_BAD_DTYPE;                                   \
  }

int dispatch_dw_s1_conv(int dtype, int k, const void* x, const void* w, const void* b, const void* addend, void* y,
                        GnPartial* stats, const S1Plan& p, int flip, cudaStream_t s) {
  int st = MEDNEXT_OK;
  MEDNEXT_T_SWITCH(dtype, T, MEDNEXT_K_SWITCH(k, KC, st = (launch_s1_conv<T, KC>(x, w, b, addend, y, stats, p, flip, s))));
  return st;
}
int dispatch_dw_s1_wgrad(int dtype, int k, const void* x, const void* dy, void* dw, void* db, void* ws,
                         const S1Plan& p, cudaStream_t s) {
  int st = MEDNEXT_OK;
  MEDNEXT_T_SWITCH(dtype, T, MEDNEXT_K_SWITCH(k, KC, st = (launch_s1_wgrad<T, KC>(x, dy, dw, db, ws, p, s))));
  return st;
}
MEDNEXT_DEFINE_ERROR_READER(read_clear_errors_dw)

}  // namespace mednext
