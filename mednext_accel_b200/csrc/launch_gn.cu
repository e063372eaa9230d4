// Template instantiation and launch of the GroupNorm kernels.
#include "plan.h"

namespace mednext {

#define MEDNEXT_T_SWITCH(dtype, TC, ...)                                     \
  switch (dtype) {                                                           \
    case MEDNEXT_FLOAT32: { using TC = float; __VA_ARGS__; } break;          \
    case MEDNEXT_BFLOAT16: { using TC = __nv_bfloat16; __VA_ARGS__; } break; \
    case MEDNEXT_FLOAT16: { using TC = __half; __VA_ARGS__; } break;         \
    case MEDNEXT_FLOAT64: { using TC = double; __VA_ARGS__; } break;         \
    default: return MEDNEXT_ERR_BAD_DTYPE;                                   \
  }
// (x type, second type in {x, float32}, gamma type in {float32, x})
#define MEDNEXT_GN_DISPATCH(xd, sd, gd, TXN, TSN, TGN, ...)                                             \
  MEDNEXT_T_SWITCH(xd, TXN, {                                                                             \
    if (sd != xd && sd != MEDNEXT_FLOAT32) return MEDNEXT_ERR_BAD_DTYPE;                                 \
    if (gd != xd && gd != MEDNEXT_FLOAT32) return MEDNEXT_ERR_BAD_DTYPE;                                 \
    if (sd == MEDNEXT_FLOAT32) {                                                                          \
      using TSN = float;                                                                                  \
      if (gd == MEDNEXT_FLOAT32) { using TGN = float; __VA_ARGS__; } else { using TGN = TXN; __VA_ARGS__; } \
    } else {                                                                                              \
      using TSN = TXN;                                                                                    \
      if (gd == MEDNEXT_FLOAT32) { using TGN = float; __VA_ARGS__; } else { using TGN = TXN; __VA_ARGS__; } \
    }                                                                                                     \
  })

int dispatch_gn_finalize(const GnPartial* part, int tiles, int nc, float eps, float* stats, cudaStream_t s) {
  gn_finalize_kernel<<<(unsigned)(((long long)nc * 32 + 127) / 128), 128, 0, s>>>(part, tiles, nc, eps, stats);
  return record_launch();
}

int dispatch_gn_stats(int dtype, const void* x, GnPartial* part, int64_t nc, int64_t vol, int64_t pitch, int chunks,
                      int row_pitch, int row_len, float eps, float* stats, cudaStream_t s) {
  int st = MEDNEXT_OK;
  MEDNEXT_T_SWITCH(dtype, T, {
    gn_stats_partial_kernel<T><<<(unsigned)(nc * chunks), 256, 0, s>>>(
        static_cast<const T*>(x), part, (size_t)vol, (size_t)pitch, chunks, row_pitch, row_len);
    st = record_launch();
  });
  if (st != MEDNEXT_OK) return st;
  return dispatch_gn_finalize(part, chunks, (int)nc, eps, stats, s);
}

int dispatch_gn_fwd(int x_dtype, int y_dtype, int g_dtype, const void* x, const float* stats, const void* gamma,
                    const void* beta, void* y, int C, int64_t nc, int64_t vol, cudaStream_t s) {
  const int chunks = gn_chunks(nc, vol);
  int st = MEDNEXT_OK;
  MEDNEXT_GN_DISPATCH(x_dtype, y_dtype, g_dtype, TX, TY, TG, {
    gn_fwd_kernel<TX, TY, TG><<<(unsigned)(nc * chunks), 256, 0, s>>>(
        static_cast<const TX*>(x), stats, static_cast<const TG*>(gamma), static_cast<const TG*>(beta),
        static_cast<TY*>(y), C, (size_t)vol, chunks);
    st = record_launch();
  });
  return st;
}

int dispatch_gn_bwd_partial(int x_dtype, int dz_dtype, const void* dz, const void* x, const float* stats,
                            GnBwdPartial* part, int64_t nc, int64_t vol, int chunks, cudaStream_t s) {
  int st = MEDNEXT_OK;
  MEDNEXT_GN_DISPATCH(x_dtype, dz_dtype, MEDNEXT_FLOAT32, TX, TD, TG, {
    gn_bwd_partial_kernel<TD, TX><<<(unsigned)(nc * chunks), 256, 0, s>>>(
        static_cast<const TD*>(dz), static_cast<const TX*>(x), stats, part, (size_t)vol, chunks);
    st = record_launch();
  });
  return st;
}

int dispatch_gn_bwd_apply(int x_dtype, int dz_dtype, int g_dtype, const void* dz, const void* x, const float* stats,
                          const void* gamma, const GnBwdPartial* part, int part_tiles, void* dx, float* dgamma,
                          float* dbeta, int N, int C, int64_t vol, int64_t pitch, cudaStream_t s) {
  const int64_t nc = (int64_t)N * C;
  const int chunks = gn_chunks(nc, vol);
  int st = MEDNEXT_OK;
  // one sample: the apply kernel adds the span sums and writes dgamma / dbeta itself
  const bool one = N == 1;
  int spans = 1;
  if (part_tiles > 1) {
    // fold in place; the workspace belongs to this call sequence
    spans = (part_tiles + kGnFoldSpan - 1) / kGnFoldSpan;
    gn_fold_partials_kernel<<<(unsigned)(nc * spans), 256, 0, s>>>(const_cast<GnBwdPartial*>(part), part_tiles);
    st = record_launch();
    if (st != MEDNEXT_OK) return st;
    if (spans > 1 && !one) {
      gn_fold_spans_kernel<<<(unsigned)((nc + 127) / 128), 128, 0, s>>>(const_cast<GnBwdPartial*>(part), part_tiles,
                                                                         (int)nc);
      st = record_launch();
      if (st != MEDNEXT_OK) return st;
      spans = 1;
    }
  }
  MEDNEXT_GN_DISPATCH(x_dtype, dz_dtype, g_dtype, TX, TD, TG, {
    gn_bwd_apply_kernel<TD, TX, TX, TG><<<(unsigned)(nc * chunks), 256, 0, s>>>(
        static_cast<const TD*>(dz), static_cast<const TX*>(x), stats, static_cast<const TG*>(gamma), part, part_tiles,
        spans, static_cast<TX*>(dx), C, (size_t)vol, (size_t)pitch, chunks, one ? dgamma : nullptr,
        one ? dbeta : nullptr);
    st = record_launch();
  });
  if (st != MEDNEXT_OK) return st;
  if (!one && (dgamma != nullptr || dbeta != nullptr)) {
    gn_param_grad_kernel<<<(C + 127) / 128, 128, 0, s>>>(part, part_tiles, N, C, dgamma, dbeta);
    st = record_launch();
  }
  return st;
}

MEDNEXT_DEFINE_ERROR_READER(read_clear_errors_gn)

}  // namespace mednext
