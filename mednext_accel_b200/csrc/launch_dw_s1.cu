// Template instantiation and launch of the depthwise kernels (stride 1) for every supported element type and kernel size.
#include <type_traits>

#include "depthwise_s1_tma.cuh"
#include "plan.h"
#include "tma_host.h"

namespace mednext {

namespace {

// The TMA plane-ring kernels need rows of whole 16-byte chunks (W * sizeof(T) a
// multiple of 16), a 16-byte aligned base and a plane tile within the 256-element
// TMA box; fp64 and other shapes use the kernels of depthwise_s1.cuh.
template <typename T, int K>
bool s1_tma_ok(const void* base, const S1Plan& p) {
  if constexpr (std::is_same<T, double>::value) {
    return false;
  } else {
    const DwS1Geom& g = p.g;
    const int P = K / 2;
    return ((size_t)g.W * sizeof(T)) % 16 == 0 && (reinterpret_cast<uintptr_t>(base) & 15) == 0 &&
           p.threads <= kDwMaxComputeWarps * 32 && DwTile<T>::row_elems(g.TW, P) <= 256 && g.TH + 2 * P <= 256;
  }
}

template <typename T, int K>
int try_s1_conv_tma(const void* x, const void* wgt, const void* bias, const void* addend, void* y, GnPartial* st,
                    const S1Plan& p, int flip, cudaStream_t s) {
  if constexpr (std::is_same<T, double>::value) {
    return -1;
  } else {
    if (!s1_tma_ok<T, K>(x, p)) return -1;
    constexpr int NH = K <= 3 ? 2 : 1;
    using L = DwTmaLayout<T>;
    const DwS1Geom& g = p.g;
    CUtensorMap m;
    if (!tma::encode4<T>(&m, x, (uint64_t)g.W, (uint64_t)g.H, (uint64_t)g.D, (uint64_t)g.N * g.C,
                         (uint32_t)DwTile<T>::row_elems(g.TW, K / 2), (uint32_t)(g.TH + 2 * (K / 2))))
      return -1;
    const size_t smem = 128 + L::weights(K, sizeof(typename Elem<T>::Acc)) + kDwSlots * L::slot(g, K, false);
    auto kern = dw_s1_conv_tma_kernel<T, K, NH>;
    if (const int rc = ensure_smem(kern, smem)) return rc;
    kern<<<(unsigned)p.grid, p.threads + 32, smem, s>>>(m, static_cast<const T*>(wgt), static_cast<const T*>(bias),
                                                          static_cast<const T*>(addend), static_cast<T*>(y), st, p.g,
                                                          flip);
    return record_launch();
  }
}

template <typename T, bool STATS, bool ADD>
int launch_s1_conv_pk(const CUtensorMap& m, const void* wgt, const void* bias, const void* addend, void* y,
                      GnPartial* st, const S1Plan& p, int flip, cudaStream_t s) {
  const size_t smem = DwPkLayout<T>::smem(p.g);
  auto kern = dw_s1_conv_pk_kernel<T, STATS, ADD>;
  if (const int rc = ensure_smem(kern, smem)) return rc;
  kern<<<(unsigned)p.grid, p.threads, smem, s>>>(m, static_cast<const T*>(wgt), static_cast<const T*>(bias),
                                                   static_cast<const T*>(addend), static_cast<T*>(y), st, p.g, flip);
  return record_launch();
}

// k = 3 on 16-bit types with packed fp32 FMAs: one output row of 16 columns per
// thread, so the tile width must be a whole number of 16-column groups.
template <typename T, int K>
int try_s1_conv_pk(const void* x, const void* wgt, const void* bias, const void* addend, void* y, GnPartial* st,
                   const S1Plan& p, int flip, cudaStream_t s) {
  if constexpr (K != 3 || !(std::is_same<T, __nv_bfloat16>::value || std::is_same<T, __half>::value)) {
    return -1;
  } else {
    const DwS1Geom& g = p.g;
    if (!s1_tma_ok<T, K>(x, p) || g.LW < 2 || p.threads > kDwPkThreads) return -1;
    using L = DwPkLayout<T>;
    CUtensorMap m;
    if (L::pitch(g.TW) > 256 ||
        !tma::encode4<T>(&m, x, (uint64_t)g.W, (uint64_t)g.H, (uint64_t)g.D, (uint64_t)g.N * g.C,
                         (uint32_t)L::pitch(g.TW), (uint32_t)(g.TH + 2)))
      return -1;
    if (st != nullptr) {
      return addend != nullptr ? launch_s1_conv_pk<T, true, true>(m, wgt, bias, addend, y, st, p, flip, s)
                               : launch_s1_conv_pk<T, true, false>(m, wgt, bias, addend, y, st, p, flip, s);
    }
    return addend != nullptr ? launch_s1_conv_pk<T, false, true>(m, wgt, bias, addend, y, st, p, flip, s)
                             : launch_s1_conv_pk<T, false, false>(m, wgt, bias, addend, y, st, p, flip, s);
  }
}

// k = 5 / 7 on 16-bit types on the tensor cores (the plan decided: its GroupNorm
// partials follow the tensor-core tiling, so there is no fallback from here).
template <typename T, int K, bool STATS, bool ADD>
int launch_s1_conv_tc(const void* x, const void* wgt, const void* bias, const void* addend, void* y, GnPartial* st,
                      const S1Plan& p, int flip, cudaStream_t s) {
  const DwTcGeom& t = p.tc;
  CUtensorMap m;
  if (!tma::encode_dw_tc<T>(&m, x, (uint64_t)t.W, (uint64_t)t.H, (uint64_t)t.D, (uint64_t)t.N * t.C, (uint32_t)t.Hp,
                            (uint32_t)t.Dp, (uint32_t)t.chunks))
    return MEDNEXT_ERR_CUDA;
  const size_t smem = dw_tc_smem(t);
  auto kern = dw_s1_conv_tc_kernel<T, K, STATS, ADD>;
  if (const int rc = ensure_smem(kern, smem)) return rc;
  const long long ctas = (long long)t.N * t.C * t.tilesW * t.tilesH * t.tilesD;
  kern<<<(unsigned)ctas, kDwTcThreads, smem, s>>>(m, static_cast<const T*>(wgt), static_cast<const T*>(bias),
                                                   static_cast<const T*>(addend), static_cast<T*>(y), st, t, flip);
  return record_launch();
}

template <typename T, int K>
int launch_s1_conv(const void* x, const void* wgt, const void* bias, const void* addend, void* y, GnPartial* st,
                   const S1Plan& p, int flip, cudaStream_t s) {
  if constexpr ((K == 5 || K == 7) && (std::is_same<T, __nv_bfloat16>::value || std::is_same<T, __half>::value)) {
    if (p.use_tc) {
      if (st != nullptr)
        return addend != nullptr ? launch_s1_conv_tc<T, K, true, true>(x, wgt, bias, addend, y, st, p, flip, s)
                                 : launch_s1_conv_tc<T, K, true, false>(x, wgt, bias, addend, y, st, p, flip, s);
      return addend != nullptr ? launch_s1_conv_tc<T, K, false, true>(x, wgt, bias, addend, y, st, p, flip, s)
                               : launch_s1_conv_tc<T, K, false, false>(x, wgt, bias, addend, y, st, p, flip, s);
    }
  }
  const int pst = try_s1_conv_pk<T, K>(x, wgt, bias, addend, y, st, p, flip, s);
  if (pst != -1) return pst;
  const int tst = try_s1_conv_tma<T, K>(x, wgt, bias, addend, y, st, p, flip, s);
  if (tst != -1) return tst;
  constexpr int NH = K <= 3 ? 2 : 1;
  auto kern = dw_s1_conv_kernel<T, K, NH>;
  if (const int rc = ensure_smem(kern, p.smem)) return rc;
  kern<<<(unsigned)p.grid, p.threads, p.smem, s>>>(static_cast<const T*>(x), static_cast<const T*>(wgt),
                                                   static_cast<const T*>(bias), static_cast<const T*>(addend),
                                                   static_cast<T*>(y), st, p.g, flip);
  return record_launch();
}

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

template <typename T, int K>
int try_s1_wgrad_tma(const void* x, const void* dy, typename Elem<T>::Acc* part, const S1Plan& p, cudaStream_t s) {
  if constexpr (std::is_same<T, double>::value || K > 3) {
    return -1;
  } else {
    if (!s1_tma_ok<T, K>(x, p) || (reinterpret_cast<uintptr_t>(dy) & 15) != 0) return -1;
    constexpr int NH = K <= 3 ? 2 : 1;
    using L = DwTmaLayout<T>;
    const DwS1Geom& g = p.g;
    CUtensorMap mx, mdy;
    const uint64_t nc = (uint64_t)g.N * g.C;
    if (!tma::encode4<T>(&mx, x, (uint64_t)g.W, (uint64_t)g.H, (uint64_t)g.D, nc,
                         (uint32_t)DwTile<T>::row_elems(g.TW, K / 2), (uint32_t)(g.TH + 2 * (K / 2))))
      return -1;
    if (!tma::encode4<T>(&mdy, dy, (uint64_t)g.W, (uint64_t)g.H, (uint64_t)g.D, nc, (uint32_t)g.TW, (uint32_t)g.TH))
      return -1;
    const size_t smem = 128 + kDwSlots * L::slot(g, K, true);
    auto kern = dw_s1_wgrad_tma_kernel<T, K, NH>;
    if (const int rc = ensure_smem(kern, smem)) return rc;
    kern<<<(unsigned)p.grid, p.threads + 32, smem, s>>>(mx, mdy, part, p.g);
    return record_launch();
  }
}

// k >= 5 weight grad on the TMA plane ring (the taps split by kd across thread
// groups): 16-byte rows, tiles within the TMA box, at most 448 compute threads.
template <typename T, int K>
bool s1_wgrad_grouped_tma_ok(const void* x, const void* dy, const S1Plan& p) {
  if constexpr (std::is_same<T, double>::value || K < 5) {
    return false;
  } else {
    const DwS1Geom& g = p.g;
    return ((size_t)g.W * sizeof(T)) % 16 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(dy) & 15) == 0 && p.threads <= 448 && p.threads % (32 * K) == 0 &&
           DwTile<T>::row_elems(g.TW, K / 2) <= 256 && g.TH + 2 * (K / 2) <= 256;
  }
}

template <typename T, int K>
int try_s1_wgrad_grouped_tma(const void* x, const void* dy, typename Elem<T>::Acc* part, const S1Plan& p,
                             cudaStream_t s) {
  if constexpr (std::is_same<T, double>::value || K < 5) {
    return -1;
  } else {
    if (!s1_wgrad_grouped_tma_ok<T, K>(x, dy, p)) return -1;
    constexpr int NH = 1;
    using L = DwTmaLayout<T>;
    const DwS1Geom& g = p.g;
    CUtensorMap mx, mdy;
    const uint64_t nc = (uint64_t)g.N * g.C;
    if (!tma::encode4<T>(&mx, x, (uint64_t)g.W, (uint64_t)g.H, (uint64_t)g.D, nc,
                         (uint32_t)DwTile<T>::row_elems(g.TW, K / 2), (uint32_t)(g.TH + 2 * (K / 2))))
      return -1;
    if (!tma::encode4<T>(&mdy, dy, (uint64_t)g.W, (uint64_t)g.H, (uint64_t)g.D, nc, (uint32_t)g.TW, (uint32_t)g.TH))
      return -1;
    const size_t smem = 128 + (size_t)dw_gslots(K) * L::slot(g, K, true);
    auto kern = dw_s1_wgrad_grouped_tma_kernel<T, K, NH>;
    if (const int rc = ensure_smem(kern, smem)) return rc;
    kern<<<(unsigned)p.grid, p.threads + 32, smem, s>>>(mx, mdy, part, p.g);
    return record_launch();
  }
}

template <typename T, int K>
int launch_s1_wgrad(const void* x, const void* dy, void* dw, void* db, void* ws, const S1Plan& p, bool f32,
                    cudaStream_t s) {
  using Acc = typename Elem<T>::Acc;
  constexpr int NH = K <= 3 ? 2 : 1;
  Acc* part = static_cast<Acc*>(ws);
  const int gst = try_s1_wgrad_grouped_tma<T, K>(x, dy, part, p, s);
  if (gst == MEDNEXT_OK) return finish_wgrad<T>(part, dw, db, p.g.N, p.g.C, (int)s1_tiles(p), K * K * K, f32, s);
  if (gst != -1) return gst;
  const int tst = try_s1_wgrad_tma<T, K>(x, dy, part, p, s);
  if (tst == MEDNEXT_OK) return finish_wgrad<T>(part, dw, db, p.g.N, p.g.C, (int)s1_tiles(p), K * K * K, f32, s);
  if (tst != -1) return tst;
  if constexpr (K <= 3) {
    auto kern = dw_s1_wgrad_kernel<T, K, NH>;
    if (const int rc = ensure_smem(kern, p.smem)) return rc;
    kern<<<(unsigned)p.grid, p.threads, p.smem, s>>>(static_cast<const T*>(x), static_cast<const T*>(dy), part, p.g);
  } else {
    auto kern = dw_s1_wgrad_grouped_kernel<T, K, NH>;
    if (const int rc = ensure_smem(kern, p.smem)) return rc;
    kern<<<(unsigned)p.grid, p.threads, p.smem, s>>>(static_cast<const T*>(x), static_cast<const T*>(dy), part, p.g);
  }
  const int st = record_launch();
  if (st != MEDNEXT_OK) return st;
  return finish_wgrad<T>(part, dw, db, p.g.N, p.g.C, (int)s1_tiles(p), K * K * K, f32, s);
}

}  // namespace

#define MEDNEXT_K_SWITCH_HOST(k, KC, ...)                      \
  switch (k) {                                                 \
    case 1: { constexpr int KC = 1; __VA_ARGS__; } break;      \
    case 3: { constexpr int KC = 3; __VA_ARGS__; } break;      \
    case 5: { constexpr int KC = 5; __VA_ARGS__; } break;      \
    case 7: { constexpr int KC = 7; __VA_ARGS__; } break;      \
    default: return MEDNEXT_ERR_BAD_KERNEL;                    \
  }
#define MEDNEXT_DW_T_SWITCH_HOST(dtype, TC, ...)                              \
  switch (dtype) {                                                            \
    case MEDNEXT_FLOAT32: { using TC = float; __VA_ARGS__; } break;           \
    case MEDNEXT_BFLOAT16: { using TC = __nv_bfloat16; __VA_ARGS__; } break;  \
    case MEDNEXT_FLOAT16: { using TC = __half; __VA_ARGS__; } break;          \
    case MEDNEXT_FLOAT64: { using TC = double; __VA_ARGS__; } break;          \
    default: return MEDNEXT_ERR_BAD_DTYPE;                                    \
  }
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

// The kernel family and tiling the launches above choose for a stride-1 plan
// (operands assumed 16-byte aligned, as the entry points require):
// out = {family, tile W, tile H, tile D, tiles W, tiles H, tiles D, CTAs}.
int describe_dw_s1(int dtype, int k, const S1Plan& p, bool wgrad, int32_t* out) {
  const DwS1Geom& g = p.g;
  const void* aligned = reinterpret_cast<const void*>(uintptr_t{256});
  int family = MEDNEXT_DWPLAN_GENERIC;
  if (!wgrad && p.use_tc) {
    family = MEDNEXT_DWPLAN_TENSOR_CORES;
    const DwTcGeom& t = p.tc;
    const int32_t v[8] = {family, t.TW, t.Ht, t.Dt, t.tilesW, t.tilesH, t.tilesD,
                          (int32_t)((long long)t.N * t.C * t.tilesW * t.tilesH * t.tilesD)};
    for (int i = 0; i < 8; ++i) out[i] = v[i];
    return MEDNEXT_OK;
  }
  bool tma = false;
  MEDNEXT_DW_T_SWITCH_HOST(dtype, T, MEDNEXT_K_SWITCH_HOST(k, KC, tma = s1_tma_ok<T, KC>(aligned, p)));
  const bool sixteen = dtype == MEDNEXT_BFLOAT16 || dtype == MEDNEXT_FLOAT16;
  if (!wgrad) {
    if (k == 3 && sixteen && tma && g.LW >= 2 && p.threads <= kDwPkThreads &&
        DwPkLayout<__nv_bfloat16>::pitch(g.TW) <= 256)
      family = MEDNEXT_DWPLAN_PACKED_FMA;
    else if (tma)
      family = MEDNEXT_DWPLAN_TMA_RING;
  } else {
    bool gtma = false;
    MEDNEXT_DW_T_SWITCH_HOST(dtype, T, MEDNEXT_K_SWITCH_HOST(k, KC, gtma = s1_wgrad_grouped_tma_ok<T, KC>(aligned, aligned, p)));
    if (k <= 3 && tma) family = MEDNEXT_DWPLAN_TMA_RING;
    else if (k >= 5) family = gtma ? MEDNEXT_DWPLAN_GROUPED_TMA_RING : MEDNEXT_DWPLAN_GROUPED;
  }
  const int32_t v[8] = {family, g.TW, g.TH, g.TD, g.tilesW, g.tilesH, g.tilesD, (int32_t)p.grid};
  for (int i = 0; i < 8; ++i) out[i] = v[i];
  return MEDNEXT_OK;
}

int dispatch_dw_s1_conv(int dtype, int k, const void* x, const void* w, const void* b, const void* addend, void* y,
                        GnPartial* stats, const S1Plan& p, int flip, cudaStream_t s) {
  int st = MEDNEXT_OK;
  MEDNEXT_T_SWITCH(dtype, T, MEDNEXT_K_SWITCH(k, KC, st = (launch_s1_conv<T, KC>(x, w, b, addend, y, stats, p, flip, s))));
  return st;
}
int dispatch_dw_s1_wgrad(int dtype, int k, const void* x, const void* dy, void* dw, void* db, void* ws,
                         const S1Plan& p, bool out_f32, cudaStream_t s) {
  int st = MEDNEXT_OK;
  MEDNEXT_T_SWITCH(dtype, T, MEDNEXT_K_SWITCH(k, KC, st = (launch_s1_wgrad<T, KC>(x, dy, dw, db, ws, p, out_f32, s))));
  return st;
}
MEDNEXT_DEFINE_ERROR_READER(read_clear_errors_dw)

}  // namespace mednext
