// Template instantiation and launch of the depthwise kernels (stride 2 and
// transpose) for every supported element type and kernel size.
#include "plan.h"

namespace mednext {

namespace {
template <typename T>
int finish_wgrad(const typename Elem<T>::Acc* part, void* dw, void* db, int N, int C, int tiles, int K3,
                 cudaStream_t s) {
  const int total = C * (K3 + 1);
  dw_wgrad_finish_kernel<T><<<(total + 127) / 128, 128, 0, s>>>(part, static_cast<T*>(dw), static_cast<T*>(db), N,
                                                                C, tiles, K3);
  return record_launch();
}

// One CTA per (sample, channel, plane): the grid must fit gridDim.x.
bool grid_ok(long long ctas) { return ctas > 0 && ctas < (1LL << 31); }

template <typename T, int K>
int launch_gather(const void* big, const void* w, const void* b, const void* addend, void* small, const DwS2Geom& g,
                  cudaStream_t s) {
  const long long ctas = (long long)g.N * g.C * g.Ds;
  if (!grid_ok(ctas)) return MEDNEXT_ERR_BAD_SHAPE;
  auto kern = addend != nullptr ? dw_s2_gather_kernel<T, K, true> : dw_s2_gather_kernel<T, K, false>;
  kern<<<(unsigned)ctas, kS2Warps * 32, 0, s>>>(static_cast<const T*>(big), static_cast<const T*>(w),
                                                static_cast<const T*>(b), static_cast<const T*>(addend),
                                                static_cast<T*>(small), g);
  return record_launch();
}
template <typename T, int K>
int launch_scatter(const void* small, const void* w, const void* b, const void* add_even, void* big,
                   const DwS2Geom& g, cudaStream_t s) {
  const long long ctas = (long long)g.N * g.C * ((g.Db + 1) / 2);
  if (!grid_ok(ctas)) return MEDNEXT_ERR_BAD_SHAPE;
  auto kern = add_even != nullptr ? dw_s2_scatter_kernel<T, K, true> : dw_s2_scatter_kernel<T, K, false>;
  kern<<<(unsigned)ctas, kS2Warps * 32, 0, s>>>(static_cast<const T*>(small), static_cast<const T*>(w),
                                                static_cast<const T*>(b), static_cast<const T*>(add_even),
                                                static_cast<T*>(big), g);
  return record_launch();
}
template <typename T>
int launch_upsample2_fill(const void* small, const float* bias, void* big, const DwS2Geom& g, cudaStream_t s) {
  const long long ctas = (long long)g.N * g.C * g.Db;
  if (!grid_ok(ctas)) return MEDNEXT_ERR_BAD_SHAPE;
  upsample2_fill_kernel<T><<<(unsigned)ctas, kS2Warps * 32, 0, s>>>(static_cast<const T*>(small), bias,
                                                                    static_cast<T*>(big), g);
  return record_launch();
}
template <typename T>
int launch_pad_front(const void* v, const void* addend, void* out, const DwS2Geom& g, bool unpad, cudaStream_t s) {
  const long long ctas = (long long)g.N * g.C * (unpad ? g.Db : g.Db + 1);
  if (!grid_ok(ctas)) return MEDNEXT_ERR_BAD_SHAPE;
  if (unpad)
    unpad_front_kernel<T><<<(unsigned)ctas, kS2Warps * 32, 0, s>>>(static_cast<const T*>(v), static_cast<T*>(out), g);
  else
    pad_front_add_kernel<T><<<(unsigned)ctas, kS2Warps * 32, 0, s>>>(static_cast<const T*>(v),
                                                                      static_cast<const T*>(addend),
                                                                      static_cast<T*>(out), g);
  return record_launch();
}
template <typename T, int K>
int launch_s2_wgrad(const void* big, const void* small, void* dw, void* db, void* ws, const DwS2Geom& g,
                    bool bias_from_big, cudaStream_t s) {
  using Acc = typename Elem<T>::Acc;
  const S2WPlan p = plan_s2w(g.N, g.C, g.Ds, K);
  Acc* part = static_cast<Acc*>(ws);
  const long long ctas = (long long)g.N * g.C * p.chunks;
  if (!grid_ok(ctas)) return MEDNEXT_ERR_BAD_SHAPE;
  const unsigned grid = (unsigned)ctas;
  dw_s2_wgrad_kernel<T, K><<<grid, p.threads, 0, s>>>(static_cast<const T*>(big), static_cast<const T*>(small), part,
                                                      g, p.chunk, p.chunks, bias_from_big ? 0 : 1);
  int st = record_launch();
  if (st != MEDNEXT_OK) return st;
  if (bias_from_big && db != nullptr) {
    const size_t bvol = (size_t)g.Db * g.Hb * g.Wb;
    chan_sum_into_partials_kernel<T><<<grid, 256, 0, s>>>(static_cast<const T*>(big), part, bvol, (size_t)g.bp, p.chunks,
                                                          K * K * K);
    st = record_launch();
    if (st != MEDNEXT_OK) return st;
  }
  return finish_wgrad<T>(part, dw, db, g.N, g.C, p.chunks, K * K * K, s);
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

int dispatch_dw_s2_gather(int dtype, int k, const void* big, const void* w, const void* b, const void* addend,
                          void* small, const DwS2Geom& g, cudaStream_t s) {
  int st = MEDNEXT_OK;
  MEDNEXT_T_SWITCH(dtype, T, MEDNEXT_K_SWITCH(k, KC, st = (launch_gather<T, KC>(big, w, b, addend, small, g, s))));
  return st;
}
int dispatch_dw_s2_scatter(int dtype, int k, const void* small, const void* w, const void* b, const void* add_even,
                           void* big, const DwS2Geom& g, cudaStream_t s) {
  int st = MEDNEXT_OK;
  MEDNEXT_T_SWITCH(dtype, T,
                   MEDNEXT_K_SWITCH(k, KC, st = (launch_scatter<T, KC>(small, w, b, add_even, big, g, s))));
  return st;
}
int dispatch_upsample2_fill(int dtype, const void* small, const float* bias, void* big, const DwS2Geom& g,
                            cudaStream_t s) {
  int st = MEDNEXT_OK;
  MEDNEXT_T_SWITCH(dtype, T, st = (launch_upsample2_fill<T>(small, bias, big, g, s)));
  return st;
}
int dispatch_pad_front(int dtype, const void* v, const void* addend, void* out, const DwS2Geom& g, bool unpad,
                       cudaStream_t s) {
  int st = MEDNEXT_OK;
  MEDNEXT_T_SWITCH(dtype, T, st = (launch_pad_front<T>(v, addend, out, g, unpad, s)));
  return st;
}
int dispatch_dw_s2_wgrad(int dtype, int k, const void* big, const void* small, void* dw, void* db, void* ws,
                         const DwS2Geom& g, bool bias_from_big, cudaStream_t s) {
  int st = MEDNEXT_OK;
  MEDNEXT_T_SWITCH(dtype, T,
                   MEDNEXT_K_SWITCH(k, KC, st = (launch_s2_wgrad<T, KC>(big, small, dw, db, ws, g, bias_from_big, s))));
  return st;
}

MEDNEXT_DEFINE_ERROR_READER(read_clear_errors_dw2)

}  // namespace mednext
