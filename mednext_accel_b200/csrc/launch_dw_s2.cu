// Template instantiation and launch of the depthwise kernels (stride 2 and
// transpose) for every supported element type and kernel size.
#include <type_traits>

#include "depthwise_s2_tma.cuh"
#include "plan.h"
#include "tma_host.h"

namespace mednext {

namespace {
// f32: write dW and dbias as fp32 (16-bit types only; the T-rounded values)
template <typename T>
int finish_wgrad(const typename Elem<T>::Acc* part, void* dw, void* db, int N, int C, int tiles, int K3, bool f32,
                 cudaStream_t s) {
  const int total = C * (K3 + 1);
  if constexpr (std::is_same<T, __nv_bfloat16>::value || std::is_same<T, __half>::value) {
    if (f32) {
      dw_wgrad_finish_kernel<T, float><<<(total + 127) / 128, 128, 0, s>>>(
          part, static_cast<float*>(dw), static_cast<float*>(db), N, C, tiles, K3);
      return record_launch();
    }
  } else {
    if (f32 && !std::is_same<T, float>::value) return MEDNEXT_ERR_BAD_DTYPE;
  }
  dw_wgrad_finish_kernel<T><<<(total + 127) / 128, 128, 0, s>>>(part, static_cast<T*>(dw), static_cast<T*>(db), N,
                                                                C, tiles, K3);
  return record_launch();
}

// One CTA per (sample, channel, plane): the grid must fit gridDim.x.
bool grid_ok(long long ctas) { return ctas > 0 && ctas < (1LL << 31); }

// Tiles of the TMA stride-2 kernels (k = 3, 16-bit types): 16-byte rows on both
// grids, the small grid's W a multiple of 8 and the big grid's rows 2 x small W
// elements apart, holding 2 x small W (down block) or 2 x small W - 1 (up block,
// one pad column) grid columns; (n, c) volumes packed.  Output planes are chunked
// to minimise (rounds of resident CTAs) x (input planes per CTA), with at most
// max_tiles tiles per (n, c).
bool s2pk_geom_ok(const DwS2Geom& g, const void* big, const void* small) {
  return g.bw == 2 * g.Ws && (g.Wb == g.bw || g.Wb == g.bw - 1) && g.Ws % 8 == 0 &&
         g.bp == (long long)g.Db * g.Hb * g.bw && (reinterpret_cast<uintptr_t>(big) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(small) & 15) == 0;
}
DwS2PkGeom s2pk_plan(const DwS2Geom& g, size_t (*smem_of)(const DwS2PkGeom&), long long max_tiles) {
  DwS2PkGeom pg{};
  pg.g = g;
  pg.TWo = std::min(64, g.Ws);
  pg.lw = pg.TWo / 8;
  pg.THo = std::min(std::min(kS2PkThreads / pg.lw, g.Hs), 127);
  pg.tilesW = (g.Ws + pg.TWo - 1) / pg.TWo;
  pg.tilesH = (g.Hs + pg.THo - 1) / pg.THo;
  const long long per_nc = (long long)pg.tilesW * pg.tilesH;
  const long long base = (long long)g.N * g.C * per_nc;
  pg.TDo = g.Ds;
  const size_t smem_one = smem_of(pg);
  const long long slots = 148 * std::max<long long>(1, std::min<long long>(2, (long long)(200 * 1024 / smem_one)));
  long long best_cost = -1;
  for (long long cand = 1; cand <= std::max(1, g.Ds / 2); ++cand) {
    const long long td = (g.Ds + cand - 1) / cand;
    const long long tiles_d = (g.Ds + td - 1) / td;
    if (per_nc * tiles_d > max_tiles) break;
    const long long cost = ((base * tiles_d + slots - 1) / slots) * (2 * td + 1);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      pg.TDo = (int)td;
    }
  }
  pg.tilesD = (g.Ds + pg.TDo - 1) / pg.TDo;
  return pg;
}
template <typename T>
size_t s2pk_gather_smem(const DwS2PkGeom& p) { return DwS2PkLayout<T>::smem(p); }
template <typename T>
size_t s2pk_wgrad_smem(const DwS2PkGeom& p) { return DwS2PkWLayout<T>::smem(p); }

template <typename T, int K>
int try_gather_pk(const void* big, const void* w, const void* b, const void* addend, void* small, const DwS2Geom& g,
                  cudaStream_t s) {
  if constexpr (K != 3 || !(std::is_same<T, __nv_bfloat16>::value || std::is_same<T, __half>::value)) {
    return -1;
  } else {
    if (!s2pk_geom_ok(g, big, small) || (reinterpret_cast<uintptr_t>(addend) & 15) != 0) return -1;
    using L = DwS2PkLayout<T>;
    const DwS2PkGeom pg = s2pk_plan(g, s2pk_gather_smem<T>, 1LL << 30);
    const long long ctas = (long long)g.N * g.C * pg.tilesW * pg.tilesH * pg.tilesD;
    if (!grid_ok(ctas)) return -1;
    CUtensorMap m;
    if (!tma::encode4<T>(&m, big, (uint64_t)g.Wb, (uint64_t)g.Hb, (uint64_t)g.Db, (uint64_t)g.N * g.C,
                         (uint32_t)L::pitch(pg.TWo), (uint32_t)L::rows(pg.THo), (uint64_t)g.bw))
      return -1;
    const size_t smem = L::smem(pg);
    const int threads = (pg.lw * pg.THo + 31) / 32 * 32;
    auto kern = addend != nullptr ? dw_s2_gather_pk_kernel<T, true> : dw_s2_gather_pk_kernel<T, false>;
    if (const int rc = ensure_smem(kern, smem)) return rc;
    kern<<<(unsigned)ctas, threads, smem, s>>>(m, static_cast<const T*>(w), static_cast<const T*>(b),
                                               static_cast<const T*>(addend), static_cast<T*>(small), pg);
    return record_launch();
  }
}

// Stride-2 weight grad on the same ring: partials per (n, c, tile), at most the
// Ds per (n, c) that the workspace holds, summed by dw_wgrad_finish_kernel.  The
// bias slot sums the small grid (the down block's dy) or, with bias_from_big
// (the up block, whose dy is the big grid), the big grid's planes as they pass.
template <typename T, int K>
int try_s2_wgrad_pk(const void* big, const void* small, void* dw, void* db, float* part, const DwS2Geom& g,
                    bool bias_from_big, bool f32, cudaStream_t s) {
  if constexpr (K != 3 || !(std::is_same<T, __nv_bfloat16>::value || std::is_same<T, __half>::value)) {
    return -1;
  } else {
    if (!s2pk_geom_ok(g, big, small)) return -1;
    using L = DwS2PkLayout<T>;
    const DwS2PkGeom pg = s2pk_plan(g, s2pk_wgrad_smem<T>, plan_s2w(g.N, g.C, g.Ds, K).chunks);
    const int tiles = pg.tilesW * pg.tilesH * pg.tilesD;
    if (tiles > plan_s2w(g.N, g.C, g.Ds, K).chunks) return -1;
    const long long ctas = (long long)g.N * g.C * tiles;
    if (!grid_ok(ctas)) return -1;
    CUtensorMap mx, mdy;
    const uint64_t nc = (uint64_t)g.N * g.C;
    if (!tma::encode4<T>(&mx, big, (uint64_t)g.Wb, (uint64_t)g.Hb, (uint64_t)g.Db, nc, (uint32_t)L::pitch(pg.TWo),
                         (uint32_t)L::rows(pg.THo), (uint64_t)g.bw))
      return -1;
    if (!tma::encode4<T>(&mdy, small, (uint64_t)g.Ws, (uint64_t)g.Hs, (uint64_t)g.Ds, nc, (uint32_t)pg.TWo,
                         (uint32_t)pg.THo))
      return -1;
    const size_t smem = DwS2PkWLayout<T>::smem(pg);
    const int threads = (pg.lw * pg.THo + 31) / 32 * 32;
    auto kern = bias_from_big ? dw_s2_wgrad_pk_kernel<T, true> : dw_s2_wgrad_pk_kernel<T, false>;
    if (const int rc = ensure_smem(kern, smem)) return rc;
    kern<<<(unsigned)ctas, threads, smem, s>>>(mx, mdy, part, pg);
    const int st = record_launch();
    if (st != MEDNEXT_OK) return st;
    return finish_wgrad<T>(part, dw, db, g.N, g.C, tiles, K * K * K, f32, s);
  }
}

template <typename T, int K>
int launch_gather(const void* big, const void* w, const void* b, const void* addend, void* small, const DwS2Geom& g,
                  cudaStream_t s) {
  const int pst = try_gather_pk<T, K>(big, w, b, addend, small, g, s);
  if (pst != -1) return pst;
  const long long ctas = (long long)g.N * g.C * g.Ds;
  if (!grid_ok(ctas)) return MEDNEXT_ERR_BAD_SHAPE;
  auto kern = addend != nullptr ? dw_s2_gather_kernel<T, K, true> : dw_s2_gather_kernel<T, K, false>;
  kern<<<(unsigned)ctas, kS2Warps * 32, 0, s>>>(static_cast<const T*>(big), static_cast<const T*>(w),
                                                static_cast<const T*>(b), static_cast<const T*>(addend),
                                                static_cast<T*>(small), g);
  return record_launch();
}
// Scatter (down-block input grad, up-block forward; k = 3, 16-bit types) on the
// TMA ring: the same grid conditions as the gather, plus a 16-byte aligned
// add_even.  Big plane pairs are chunked to minimise (rounds of resident CTAs) x
// (small planes per CTA).
// (Only meaningful where s2pk_geom_ok holds: the small W is a multiple of 8.)
DwS2ScGeom s2sc_plan(const DwS2Geom& g) {
  DwS2ScGeom pg{};
  pg.g = g;
  pg.TWs = std::max(8, std::min(64, g.Ws));
  pg.lw = pg.TWs / 8;
  pg.THs = std::min(std::min(kS2PkThreads / pg.lw, g.Hs), 255);
  pg.tilesW = (g.Ws + pg.TWs - 1) / pg.TWs;
  pg.tilesH = (g.Hs + pg.THs - 1) / pg.THs;
  const int QD = (g.Db + 1) / 2;
  const long long base = (long long)g.N * g.C * pg.tilesW * pg.tilesH;
  const long long slots = 148 * 2;
  long long best_cost = -1;
  pg.TDq = QD;
  for (long long cand = 1; cand <= std::max(1, QD / 2); ++cand) {
    const long long td = (QD + cand - 1) / cand;
    const long long tiles_d = (QD + td - 1) / td;
    const long long cost = ((base * tiles_d + slots - 1) / slots) * (td + 1);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      pg.TDq = (int)td;
    }
  }
  pg.tilesD = (QD + pg.TDq - 1) / pg.TDq;
  return pg;
}

template <typename T, int K>
bool scatter_pk_applies(const void* small, const void* add_even, const void* big, const DwS2Geom& g) {
  if constexpr (K != 3 || !(std::is_same<T, __nv_bfloat16>::value || std::is_same<T, __half>::value)) {
    return false;
  } else {
    if (!s2pk_geom_ok(g, big, small) || (reinterpret_cast<uintptr_t>(add_even) & 15) != 0) return false;
    const DwS2ScGeom pg = s2sc_plan(g);
    return grid_ok((long long)g.N * g.C * pg.tilesW * pg.tilesH * pg.tilesD);
  }
}

// stats: NULL, or GroupNorm partials, one per (n, c, tile) of s2sc_plan(g)
template <typename T, int K>
int try_scatter_pk(const void* small, const void* w, const void* b, const void* add_even, void* big,
                   GnPartial* stats, const DwS2Geom& g, cudaStream_t s) {
  if constexpr (K != 3 || !(std::is_same<T, __nv_bfloat16>::value || std::is_same<T, __half>::value)) {
    return -1;
  } else {
    if (!scatter_pk_applies<T, K>(small, add_even, big, g) || (stats != nullptr && add_even != nullptr)) return -1;
    using L = DwS2ScLayout<T>;
    const DwS2ScGeom pg = s2sc_plan(g);
    const long long ctas = (long long)g.N * g.C * pg.tilesW * pg.tilesH * pg.tilesD;
    CUtensorMap m;
    if (!tma::encode4<T>(&m, small, (uint64_t)g.Ws, (uint64_t)g.Hs, (uint64_t)g.Ds, (uint64_t)g.N * g.C,
                         (uint32_t)L::pitch(pg.TWs), (uint32_t)L::rows(pg.THs)))
      return -1;
    const size_t smem = L::smem(pg);
    const int threads = (pg.lw * pg.THs + 31) / 32 * 32;
    auto kern = stats != nullptr ? dw_s2_scatter_pk_kernel<T, false, true>
                : add_even != nullptr ? dw_s2_scatter_pk_kernel<T, true, false>
                                      : dw_s2_scatter_pk_kernel<T, false, false>;
    if (const int rc = ensure_smem(kern, smem)) return rc;
    kern<<<(unsigned)ctas, threads, smem, s>>>(m, static_cast<const T*>(w), static_cast<const T*>(b),
                                               static_cast<const T*>(add_even), static_cast<T*>(big), stats, pg);
    return record_launch();
  }
}

template <typename T, int K>
int launch_scatter(const void* small, const void* w, const void* b, const void* add_even, void* big,
                   const DwS2Geom& g, cudaStream_t s) {
  const int pst = try_scatter_pk<T, K>(small, w, b, add_even, big, nullptr, g, s);
  if (pst != -1) return pst;
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
                    bool bias_from_big, bool f32, cudaStream_t s) {
  using Acc = typename Elem<T>::Acc;
  const S2WPlan p = plan_s2w(g.N, g.C, g.Ds, K);
  Acc* part = static_cast<Acc*>(ws);
  if constexpr (std::is_same<Acc, float>::value) {
    const int pst = try_s2_wgrad_pk<T, K>(big, small, dw, db, part, g, bias_from_big, f32, s);
    if (pst != -1) return pst;
  }
  const long long ctas = (long long)g.N * g.C * p.chunks;
  if (!grid_ok(ctas)) return MEDNEXT_ERR_BAD_SHAPE;
  const unsigned grid = (unsigned)ctas;
  dw_s2_wgrad_kernel<T, K><<<grid, p.threads, 0, s>>>(static_cast<const T*>(big), static_cast<const T*>(small), part,
                                                      g, p.chunk, p.chunks, bias_from_big ? 0 : 1);
  int st = record_launch();
  if (st != MEDNEXT_OK) return st;
  if (bias_from_big && db != nullptr) {
    chan_sum_into_partials_kernel<T><<<grid, 256, 0, s>>>(static_cast<const T*>(big), part, (size_t)g.bp,
                                                          (size_t)g.bp, p.chunks, K * K * K, g.bw, g.Wb);
    st = record_launch();
    if (st != MEDNEXT_OK) return st;
  }
  return finish_wgrad<T>(part, dw, db, g.N, g.C, p.chunks, K * K * K, f32, s);
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
// The up block's forward with the GroupNorm statistics of its output: on the
// packed-FMA scatter, per-tile partials from the kernel itself (workspace: one
// GnPartial per (n, c, tile)); elsewhere the scatter, then the row-aware
// statistics pass (its own partials in the same workspace).
size_t dwT_fwd_stats_ws(int dtype, int k, const DwS2Geom& g) {
  const long long nc = (long long)g.N * g.C;
  const size_t gen = (size_t)nc * gn_chunks(nc, g.bp) * sizeof(GnPartial);
  if (k != 3 || !(dtype == MEDNEXT_BFLOAT16 || dtype == MEDNEXT_FLOAT16) || g.Ws % 8 != 0) return gen;
  const DwS2ScGeom pg = s2sc_plan(g);
  const size_t pk = (size_t)nc * pg.tilesW * pg.tilesH * pg.tilesD * sizeof(GnPartial);
  return std::max(gen, pk);
}

int dispatch_dwT_fwd_stats(int dtype, int k, const void* small, const void* w, const void* b, void* big,
                           GnPartial* part, float eps, float* stats, const DwS2Geom& g, cudaStream_t s) {
  if (k == 3 && (dtype == MEDNEXT_BFLOAT16 || dtype == MEDNEXT_FLOAT16)) {
    const int pst = dtype == MEDNEXT_BFLOAT16
                        ? try_scatter_pk<__nv_bfloat16, 3>(small, w, b, nullptr, big, part, g, s)
                        : try_scatter_pk<__half, 3>(small, w, b, nullptr, big, part, g, s);
    if (pst != -1) {
      if (pst != MEDNEXT_OK) return pst;
      const DwS2ScGeom pg = s2sc_plan(g);
      return dispatch_gn_finalize(part, pg.tilesW * pg.tilesH * pg.tilesD, g.N * g.C, eps, stats, s);
    }
  }
  const int st = dispatch_dw_s2_scatter(dtype, k, small, w, b, nullptr, big, g, s);
  if (st != MEDNEXT_OK) return st;
  const long long nc = (long long)g.N * g.C;
  return dispatch_gn_stats(dtype, big, part, nc, g.bp, g.bp, gn_chunks(nc, g.bp), g.bw, g.Wb, eps, stats, s);
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
                         const DwS2Geom& g, bool bias_from_big, bool out_f32, cudaStream_t s) {
  int st = MEDNEXT_OK;
  MEDNEXT_T_SWITCH(dtype, T,
                   MEDNEXT_K_SWITCH(k, KC, st = (launch_s2_wgrad<T, KC>(big, small, dw, db, ws, g, bias_from_big,
                                                                        out_f32, s))));
  return st;
}

MEDNEXT_DEFINE_ERROR_READER(read_clear_errors_dw2)

}  // namespace mednext
