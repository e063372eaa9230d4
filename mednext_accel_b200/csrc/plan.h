// Host-side tile planning and the per-family dispatch functions that
// launch_dw.cu, launch_gn.cu and launch_pw.cu define (one translation unit per
// kernel family so the library builds in parallel).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "../../include/mednext_b200.h"
#include "depthwise_s1.cuh"
#include "depthwise_s1_tc.cuh"
#include "depthwise_s2.cuh"
#include "groupnorm.cuh"
#include "pointwise.cuh"

namespace mednext {

constexpr int kTargetCtas = 148 * 4;  // 4 resident CTAs per SM on 148 SMs

inline size_t elem_size(int dtype) {
  switch (dtype) {
    case MEDNEXT_FLOAT32: return 4;
    case MEDNEXT_BFLOAT16: return 2;
    case MEDNEXT_FLOAT16: return 2;
    case MEDNEXT_FLOAT64: return 8;
    default: return 0;
  }
}
inline size_t acc_size(int dtype) { return dtype == MEDNEXT_FLOAT64 ? 8 : 4; }

// ------------------------------ stride-1 depthwise ------------------------------
struct S1Plan {
  DwS1Geom g;
  int threads;
  size_t smem;
  long long grid;
  bool use_tc;  // forward / input grad on the tensor cores (dw_s1_conv_tc_kernel), tiled by tc
  DwTcGeom tc;
};

// Tiles of the tensor-core k = 5 / 7 forward and input grad (16-bit types, W a
// multiple of 16).  Searched over the tile width (64, 32 or 16 columns, dividing
// W), 32-row tiles (Ht + K - 1 row slots per plane) and 1..4 blocks of 128 row
// slots (at most 256 TMEM columns), within 113 KB of shared memory so two CTAs
// share an SM.  Cost of a candidate: its tiles x (tensor-core operand bytes read
// from shared memory + 3 x the bytes its TMA copy loads); the smallest wins.
// tmem_cols = 0: not eligible.
inline DwTcGeom plan_dw_tc(int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k) {
  DwTcGeom best{};
  if ((k != 5 && k != 7) || w < 16 || w % 16 != 0 || d < 1 || h < 1) return best;
  double best_cost = -1.0;
  for (int tw = 64; tw >= 16; tw /= 2) {
    if (w % tw != 0) continue;
    for (int nb = 1; nb <= kDwTcMaxBlk; ++nb) {
      if (nb * tw > 256) continue;
      DwTcGeom t{};
      t.N = (int)n; t.C = (int)c; t.D = (int)d; t.H = (int)h; t.W = (int)w;
      t.K = k;
      t.TW = tw;
      t.chunks = tw / 8 + 2;
      t.Ht = (int)std::min<int64_t>(32, h);
      t.Hp = t.Ht + k - 1;
      const int dt_max = nb * 128 / t.Hp;
      if (dt_max < 1) continue;
      t.Dt = (int)std::min<int64_t>(dt_max, d);
      t.nblk = (t.Dt * t.Hp + 127) / 128;
      t.Dp = (t.nblk * 128 + (k - 1) * (t.Hp + 1) + t.Hp - 1) / t.Hp;
      if (t.Dp > 256 || dw_tc_smem(t) > 113 * 1024) continue;
      t.tilesW = (int)(w / tw);
      t.tilesH = (int)((h + t.Ht - 1) / t.Ht);
      t.tilesD = (int)((d + t.Dt - 1) / t.Dt);
      const double tiles = (double)n * c * t.tilesW * t.tilesH * t.tilesD;
      if (tiles >= 2147483648.0) continue;
      const double mma_bytes = (double)t.nblk * (tw / 16) * k * k * 2 * 4096;
      const double load_bytes = (double)dw_tc_x_bytes(t);
      const double cost = tiles * (mma_bytes + 3.0 * load_bytes);
      if (best_cost < 0.0 || cost < best_cost) {
        best_cost = cost;
        best = t;
      }
    }
  }
  if (best_cost < 0.0) return DwTcGeom{};
  uint32_t cols = 32;
  while (cols < (uint32_t)(best.nblk * best.TW)) cols *= 2;
  best.tmem_cols = cols;
  return best;
}

inline int nh_for(int k) { return k <= 3 ? 2 : 1; }

inline S1Plan plan_s1(int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k, size_t esz, bool wgrad) {
  S1Plan p{};
  DwS1Geom& g = p.g;
  g.N = (int)n; g.C = (int)c; g.D = (int)d; g.H = (int)h; g.W = (int)w;
  const int NH = nh_for(k);
  int lw = 1;
  while (lw * kDwNW < w && lw < 16) lw *= 2;
  g.LW = lw;
  g.TW = kDwNW * lw;
  const bool grouped = wgrad && k >= 5;
  const int rows_needed = (int)((h + NH - 1) / NH);
  int tr;
  if (grouped) {
    tr = std::max(1, std::min(64 / lw, rows_needed));
    const int G = ((lw * tr + 31) / 32) * 32;
    p.threads = G * k;
  } else {
    // the packed k = 3 forward / input grad on 16-bit types runs 4-warp tiles (4 CTAs per
    // SM): smaller units of work balance the SMs better than 8-warp tiles
    const bool packed = !wgrad && k == 3 && esz == 2 && lw >= 2;
    tr = std::max(1, std::min((packed ? 128 : 256) / lw, rows_needed));
    p.threads = ((lw * tr + 31) / 32) * 32;
  }
  g.TR = tr;
  g.TH = tr * NH;
  g.tilesW = (int)((w + g.TW - 1) / g.TW);
  g.tilesH = (int)((h + g.TH - 1) / g.TH);
  const long long base = (long long)n * c * g.tilesW * g.tilesH;
  const long long max_chunks = std::max(1LL, (long long)(d / 8));
  long long chunks;
  if (!grouped) {
    // Depth chunks that minimise the busiest SM's time: (CTAs it runs) x (planes each
    // streams, k - 1 of them halo, plus about 4 planes' worth of start-up: barriers,
    // the first load's latency, the statistics epilogue) / (its throughput).  An SM
    // runs at full rate with 16 resident warps and proportionally slower with fewer.
    // Residency: the packed k = 3 kernel on 16-bit types holds 16 warps per SM, the
    // other kernels about 12.
    // The weight-grad kernel (k <= 3) holds about 20 warps per SM (2 CTAs of 8 + 1).
    const bool packed = !wgrad && k == 3 && esz == 2 && lw >= 2;
    const int warps = (p.threads + 31) / 32 + (packed ? 0 : 1);
    const long long per_sm = std::max(1, (wgrad ? 20 : packed ? 16 : 12) / warps);
    double best_cost = -1.0;
    chunks = 1;
    for (long long cand = 1; cand <= max_chunks; ++cand) {
      const long long td = (d + cand - 1) / cand;
      const long long ctas = base * ((d + td - 1) / td);
      const long long on_sm = (ctas + 147) / 148;
      const double rate = std::min(1.0, (double)(std::min(on_sm, per_sm) * warps) / 16.0);
      const double cost = (double)on_sm * (double)(td + k - 1 + 4) / rate;
      if (best_cost < 0.0 || cost < best_cost) {
        best_cost = cost;
        chunks = cand;
      }
    }
  } else {
    chunks = std::max(1LL, std::min((kTargetCtas + base - 1) / base, max_chunks));
  }
  g.TD = (int)((d + chunks - 1) / chunks);
  g.tilesD = (int)((d + g.TD - 1) / g.TD);
  const int E = (int)(16 / esz);
  g.vec = (w % E) == 0 ? 1 : 0;
  const int P = k / 2;
  const int off = ((P + E - 1) / E) * E;
  const size_t rsw = (size_t)g.TW + 2 * off;
  const size_t tile = (size_t)(g.TH + 2 * P) * rsw * esz;
  const size_t acc = esz == 8 ? 8 : 4;
  p.smem = wgrad ? tile : (((size_t)k * k * k * acc + 15) / 16) * 16 + tile;
  p.grid = base * g.tilesD;
  if (!wgrad && (k == 5 || k == 7) && esz == 2) {
    p.tc = plan_dw_tc(n, c, d, h, w, k);
    p.use_tc = p.tc.tmem_cols != 0;
  }
  return p;
}
// GroupNorm partials per (n, c) that the forward of this plan writes
inline size_t s1_tiles(const S1Plan& p) {
  if (p.use_tc) return (size_t)p.tc.tilesW * p.tc.tilesH * p.tc.tilesD;
  return (size_t)p.g.tilesW * p.g.tilesH * p.g.tilesD;
}

// ------------------------------ stride-2 depthwise ------------------------------
constexpr int kS2Group = 64;
struct S2WPlan {
  int chunk, chunks, threads;
};
// One CTA per (sample, channel, small-grid plane): many short CTAs keep enough
// loads in flight; K thread groups (one per kd), 128 threads each for k <= 3.
inline S2WPlan plan_s2w(int64_t n, int64_t c, int64_t ds, int k) {
  (void)n;
  (void)c;
  S2WPlan p{};
  p.chunk = 1;
  p.chunks = (int)ds;
  p.threads = (k <= 3 ? 2 * kS2Group : kS2Group) * k;
  return p;
}
inline DwS2Geom s2_geom_down(int64_t n, int64_t c, int64_t d, int64_t h, int64_t w) {
  DwS2Geom g{};
  g.N = (int)n; g.C = (int)c;
  g.Db = (int)d; g.Hb = (int)h; g.Wb = (int)w;
  g.Ds = (int)((d + 1) / 2); g.Hs = (int)((h + 1) / 2); g.Ws = (int)((w + 1) / 2);
  g.bw = (int)w;
  g.bp = (long long)d * h * w;
  return g;
}
// row_pitch: elements between consecutive W-rows of the (2d-1, 2h-1, 2w-1) grid
// (0 = 2w-1, contiguous); the (n, c) volumes are (2d-1)(2h-1) row pitches apart
inline DwS2Geom s2_geom_up(int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int64_t row_pitch) {
  DwS2Geom g{};
  g.N = (int)n; g.C = (int)c;
  g.Ds = (int)d; g.Hs = (int)h; g.Ws = (int)w;
  g.Db = (int)(2 * d - 1); g.Hb = (int)(2 * h - 1); g.Wb = (int)(2 * w - 1);
  g.bw = row_pitch > 0 ? (int)row_pitch : g.Wb;
  g.bp = (long long)g.Db * g.Hb * g.bw;
  return g;
}

// ------------------------------ GroupNorm ------------------------------
inline int gn_chunks(int64_t nc, int64_t vol) {
  const long long want = std::max(1LL, (long long)kTargetCtas * 2 / std::max<int64_t>(1, nc));
  const long long maxc = std::max<long long>(1, vol / 2048);
  return (int)std::max(1LL, std::min(want, maxc));
}

// ------------------------------ pointwise ------------------------------
inline int pw_bn(int64_t cout) {
  if (cout >= 256) return 256;
  return (int)(((cout + 15) / 16) * 16);
}
// N tile of the forward / input-grad GEMM: up to 256 output channels.  Where the
// tiles would leave SMs idle (the deep levels: a few thousand voxels), GEMMs whose
// prologue is cheap take narrower N tiles, down to 32 channels, until about 128
// tiles exist; each N tile re-reads its A tile, which at these sizes comes from L2.
// A GELU prologue keeps the widest tile (each N tile would repeat the GELU work).
inline int pw_fwd_bn(int64_t n, int64_t cout, int64_t vox, int prologue) {
  int bn = pw_bn(cout);
  if (prologue == MEDNEXT_PRO_GELU) return bn;
  const int64_t mt = n * ((vox + 127) / 128);
  while (bn > 32 && mt * ((cout + bn - 1) / bn) < 128) bn = std::max(32, (bn / 2 + 15) / 16 * 16);
  return bn;
}
inline size_t pw_smem(int BN) { return 32768 + 2 * (size_t)BN * 128 + 1024; }
struct PwWPlan {
  int BN, mtiles, ntiles, splits;
  long long cps, total, per;
};
inline PwWPlan plan_pw_wgrad(int64_t n, int64_t cin, int64_t cout, int64_t vox) {
  PwWPlan p{};
  // one spare row past cin when it fits: the TMA kernel puts the bias grad there
  p.BN = cin < 256 ? pw_bn(cin + 1) : pw_bn(cin);
  p.mtiles = (int)((cout + kPwBM - 1) / kPwBM);
  p.ntiles = (int)((cin + p.BN - 1) / p.BN);
  p.cps = (vox + kPwBK - 1) / kPwBK;
  p.total = p.cps * n;
  // one split-K unit per SM for the persistent kernel (148 SMs)
  long long splits = std::max(1LL, (long long)148 / (p.mtiles * p.ntiles));
  splits = std::min(splits, p.total);
  p.per = (p.total + splits - 1) / splits;
  p.splits = (int)((p.total + p.per - 1) / p.per);
  return p;
}

// ------------------------------ dispatch (defined in launch_*.cu) ----------------
// Each returns a mednext_status and never allocates.
int describe_dw_s1(int dtype, int k, const S1Plan& p, bool wgrad, int32_t* out);
int dispatch_dw_s1_conv(int dtype, int k, const void* x, const void* w, const void* b, const void* addend, void* y,
                        GnPartial* stats, const S1Plan& p, int flip, cudaStream_t s);
int dispatch_dw_s1_wgrad(int dtype, int k, const void* x, const void* dy, void* dw, void* db, void* ws,
                         const S1Plan& p, bool out_f32, cudaStream_t s);
int dispatch_upsample2_fill(int dtype, const void* small, const float* bias, void* big, const DwS2Geom& g,
                            cudaStream_t s);
int dispatch_pad_front(int dtype, const void* v, const void* addend, void* out, const DwS2Geom& g, bool unpad,
                       cudaStream_t s);
int dispatch_dw_s2_gather(int dtype, int k, const void* big, const void* w, const void* b, const void* addend,
                          void* small,
                          const DwS2Geom& g, cudaStream_t s);
int dispatch_dw_s2_scatter(int dtype, int k, const void* small, const void* w, const void* b,
                           const void* add_even, void* big,
                           const DwS2Geom& g, cudaStream_t s);
int dispatch_dw_s2_wgrad(int dtype, int k, const void* big, const void* small, void* dw, void* db, void* ws,
                         const DwS2Geom& g, bool bias_from_big, bool out_f32, cudaStream_t s);
size_t dwT_fwd_stats_ws(int dtype, int k, const DwS2Geom& g);
int dispatch_dwT_fwd_stats(int dtype, int k, const void* small, const void* w, const void* b, void* big,
                           GnPartial* part, float eps, float* stats, const DwS2Geom& g, cudaStream_t s);
int dispatch_gn_finalize(const GnPartial* part, int tiles, int nc, float eps, float* stats, cudaStream_t s);
// rows of row_pitch elements of which the first row_len are statistics (equal: all)
int dispatch_gn_stats(int dtype, const void* x, GnPartial* part, int64_t nc, int64_t vol, int64_t pitch, int chunks,
                      int row_pitch, int row_len, float eps, float* stats, cudaStream_t s);
int dispatch_gn_fwd(int x_dtype, int y_dtype, int g_dtype, const void* x, const float* stats, const void* gamma,
                    const void* beta, void* y, int C, int64_t nc, int64_t vol, cudaStream_t s);
int dispatch_gn_bwd_partial(int x_dtype, int dz_dtype, const void* dz, const void* x, const float* stats,
                            GnBwdPartial* part, int64_t nc, int64_t vol, int chunks, cudaStream_t s);
int dispatch_gn_bwd_apply(int x_dtype, int dz_dtype, int g_dtype, const void* dz, const void* x, const float* stats,
                          const void* gamma, const GnBwdPartial* part, int part_tiles, void* dx, float* dgamma,
                          float* dbeta, int N, int C, int64_t vol, int64_t pitch, cudaStream_t s);
int dispatch_pw_fwd(int a_dtype, int y_dtype, int prologue, const PwFwdArgs& a, cudaStream_t s);
// Per-element-type forward instantiations (pw_fwd_*.cu).
int pw_fwd_bf16_bf16(int prologue, const PwFwdArgs& a, cudaStream_t s);
int pw_gelu_bwd_bf16(const PwFwdArgs& a, cudaStream_t s);
int pw_gn_bwd_bf16(const PwFwdArgs& a, cudaStream_t s);
int pw_mlp_fwd_bf16(const PwFwdArgs& a, cudaStream_t s);
// Forward GEMM that also writes g = GELU(y) to a.y2 (prologue none or GroupNorm, bias or
// none): MEDNEXT_OK when launched, -1 when the shape does not allow the TMA kernel.
int pw_fwd_gelu_out_bf16(int prologue, const PwFwdArgs& a, cudaStream_t s);
int pw_fused_grid(long long total_tiles);  // CTAs (= weight-grad splits) of pw_gelu_bwd_bf16
int dispatch_pw_wgrad_reduce(const float* part, const float* part_b, float* dw, float* dbias, int splits, int cout,
                             int cin, cudaStream_t s);
int pw_fwd_bf16_f32(int prologue, const PwFwdArgs& a, cudaStream_t s);
int pw_fwd_f16(int y_dtype, int prologue, const PwFwdArgs& a, cudaStream_t s);
int dispatch_pw_wgrad(int dtype, int prologue, const PwWgradArgs& a, int splits, cudaStream_t s);

// Read and clear the device error word of every translation unit.
int read_clear_errors_dw(int* code, cudaStream_t s);
int read_clear_errors_dw2(int* code, cudaStream_t s);
int read_clear_errors_gn(int* code, cudaStream_t s);
int read_clear_errors_pw(int* code, cudaStream_t s);
int read_clear_errors_pwf0(int* code, cudaStream_t s);
int read_clear_errors_pwf1(int* code, cudaStream_t s);
int read_clear_errors_pwf2(int* code, cudaStream_t s);
int read_clear_errors_loss(int* code, cudaStream_t s);

// Records the CUDA error of the last launch in a thread-local slot.
int record_launch();
int last_cuda_error();
// Records a CUDA runtime error for mednext_last_cuda_error() on this thread.
void note_cuda_error(cudaError_t e);

// Dynamic shared memory above 48 KB needs an opt-in per kernel and per device.
// Grants the opt-in for `smem` bytes on the current device (once per kernel,
// device and size; thread-safe).  Returns MEDNEXT_OK or MEDNEXT_ERR_CUDA.
int ensure_smem_fn(const void* fn, size_t smem);
template <typename K>
inline int ensure_smem(K* kern, size_t smem) {
  return smem <= 48 * 1024 ? 0 : ensure_smem_fn(reinterpret_cast<const void*>(kern), smem);
}

}  // namespace mednext

// Per-translation-unit reader of the device error word.
#define MEDNEXT_DEFINE_ERROR_READER(fn)                                                                  \
  int fn(int* code, cudaStream_t s) {                                                                     \
    int host = 0;                                                                                         \
    if (cudaMemcpyFromSymbolAsync(&host, g_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s) !=    \
            cudaSuccess ||                                                                                \
        cudaStreamSynchronize(s) != cudaSuccess)                                                          \
      return record_launch();                                                                             \
    const int zero = 0;                                                                                   \
    if (cudaMemcpyToSymbolAsync(g_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s) !=      \
            cudaSuccess ||                                                                                \
        cudaStreamSynchronize(s) != cudaSuccess)                                                          \
      return record_launch();                                                                             \
    if (*code == 0) *code = host;                                                                         \
    return MEDNEXT_OK;                                                                                    \
  }
