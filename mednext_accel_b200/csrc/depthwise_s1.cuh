// Depthwise Conv3d, stride 1, padding k/2: forward / input-grad and weight-grad
// kernels on CUDA cores.
//
// Work decomposition (all three kernels).  A CTA owns one (sample, channel)
// volume tile: TW columns (8 per thread), TH rows (NH per thread row) and a
// chunk of TD depth planes.  It streams the input planes of that chunk (plus
// the k-1 halo planes) through shared memory one plane at a time; each plane
// tile carries a zero-filled halo of k/2 rows and OFF columns, so the inner
// loops have no bounds checks.  A thread keeps a ring of k partial output
// planes (forward) or k input-grad planes (weight grad) in registers and
// consumes each shared-memory plane exactly once, so every input element is
// read from shared memory (NH + k - 1) / NH times per output plane instead of
// k^3 times as in a gather formulation (reference: ops/_triton/depthwise.py:
// 191-202 issues k^3 masked loads per output).
#pragma once

#include <type_traits>

#include "common.cuh"

namespace mednext {

constexpr int kDwNW = 8;  // outputs per thread along W

struct DwS1Geom {
  int N, C, D, H, W;
  int TW, LW;        // tile width (8*LW) and threads along W
  int TR, TH;        // thread rows and tile height (TR*NH)
  int TD;            // depth planes per CTA
  int tilesW, tilesH, tilesD;
  int vec;           // 1 when W is a multiple of the 16-byte element count
};

template <typename T>
struct DwTile {
  static constexpr int E = 16 / (int)sizeof(T);  // elements per 16-byte chunk
  // Left halo of the shared-memory row, rounded up to a whole chunk.
  static __host__ __device__ constexpr int off(int P) { return ((P + E - 1) / E) * E; }
  static __host__ __device__ constexpr int row_elems(int TW, int P) { return TW + 2 * off(P); }
};

// Cooperative load of one zero-padded input plane tile into shared memory:
// rows [h0-P, h0+TH+P), columns [w0-OFF, w0-OFF+RSW).
template <typename T, int P>
__device__ __forceinline__ void dw_load_plane(T* __restrict__ sp, const T* __restrict__ vol,
                                              int d_in, int h0, int w0, const DwS1Geom& g,
                                              int rows, int rsw) {
  constexpr int E = DwTile<T>::E;
  constexpr int OFF = DwTile<T>::off(P);
  const bool plane_ok = d_in >= 0 && d_in < g.D;
  const T* plane = vol + (size_t)(plane_ok ? d_in : 0) * g.H * g.W;
  if (g.vec) {
    const int cpr = rsw / E;  // chunks per row
    const int total = rows * cpr;
    uint4* s4 = reinterpret_cast<uint4*>(sp);
    for (int e = threadIdx.x; e < total; e += blockDim.x) {
      const int r = e / cpr;
      const int q = e - r * cpr;
      const int hh = h0 - P + r;
      const int ww = w0 - OFF + q * E;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (plane_ok && hh >= 0 && hh < g.H && ww >= 0 && ww < g.W) {
        v = __ldg(reinterpret_cast<const uint4*>(plane + (size_t)hh * g.W + ww));
      }
      s4[e] = v;
    }
  } else {
    const int total = rows * rsw;
    for (int e = threadIdx.x; e < total; e += blockDim.x) {
      const int r = e / rsw;
      const int q = e - r * rsw;
      const int hh = h0 - P + r;
      const int ww = w0 - OFF + q;
      T v = from_acc<T>(typename Elem<T>::Acc(0));
      if (plane_ok && hh >= 0 && hh < g.H && ww >= 0 && ww < g.W) v = plane[(size_t)hh * g.W + ww];
      sp[e] = v;
    }
  }
}

// Read the (8 + 2P)-wide input window of thread column `wt` from row `r` of a
// shared-memory plane tile: window[i] = input column w0 + 8*wt - P + i.
template <typename T, int P>
__device__ __forceinline__ void dw_read_window(const T* __restrict__ sp, int r, int rsw, int wt,
                                               typename Elem<T>::Acc* win) {
  using Acc = typename Elem<T>::Acc;
  constexpr int E = DwTile<T>::E;
  constexpr int OFF = DwTile<T>::off(P);
  constexpr int START = OFF - P;           // element index of window[0] relative to 8*wt
  constexpr int Q0 = START / E;            // first chunk
  constexpr int A = START - Q0 * E;        // offset inside that chunk
  constexpr int NCH = (A + kDwNW + 2 * P + E - 1) / E;
  const uint4* row = reinterpret_cast<const uint4*>(sp + (size_t)r * rsw) + (kDwNW / E) * wt + Q0;
  Acc buf[NCH * E];
#pragma unroll
  for (int q = 0; q < NCH; ++q) unpack16<T>(row[q], buf + q * E);
#pragma unroll
  for (int i = 0; i < kDwNW + 2 * P; ++i) win[i] = buf[A + i];
}

struct GnPartial {
  double count, mean, m2, pad;
};

// Chan et al. parallel merge of (count, mean, M2) triples.
template <typename A>
__device__ __forceinline__ void chan_merge(A& n, A& mean, A& m2, A nb, A meanb, A m2b) {
  const A tot = n + nb;
  if (nb == A(0)) return;
  if (n == A(0)) {
    n = nb;
    mean = meanb;
    m2 = m2b;
    return;
  }
  const A delta = meanb - mean;
  const A fb = nb / tot;
  mean = mean + delta * fb;
  m2 = m2 + m2b + delta * delta * n * fb;
  n = tot;
}

// Block-wide deterministic merge of per-thread statistics; thread 0 gets the result.
template <typename A>
__device__ void block_merge_stats(A& n, A& mean, A& m2, A* scratch /* 3 * 32 */) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const A nb = __shfl_down_sync(0xffffffffu, n, o);
    const A mb = __shfl_down_sync(0xffffffffu, mean, o);
    const A qb = __shfl_down_sync(0xffffffffu, m2, o);
    if (lane + o < 32) chan_merge(n, mean, m2, nb, mb, qb);
  }
  if (lane == 0) {
    scratch[3 * warp] = n;
    scratch[3 * warp + 1] = mean;
    scratch[3 * warp + 2] = m2;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int nw = blockDim.x >> 5;
    for (int w = 1; w < nw; ++w) chan_merge(n, mean, m2, scratch[3 * w], scratch[3 * w + 1], scratch[3 * w + 2]);
  }
}

// Load 8 consecutive values of one row (zeros past the edge) as Acc.
template <typename T>
__device__ __forceinline__ void dw_load_dy_patch(const T* __restrict__ plane, int oh, int ow0,
                                                 const DwS1Geom& g, bool vec,
                                                 typename Elem<T>::Acc* out) {
  using Acc = typename Elem<T>::Acc;
  constexpr int E = DwTile<T>::E;
  if (oh < g.H) {
    const T* src = plane + (size_t)oh * g.W + ow0;
    if (vec) {
#pragma unroll
      for (int q = 0; q < kDwNW / E; ++q)
        unpack16<T>(__ldg(reinterpret_cast<const uint4*>(src) + q), out + q * E);
      return;
    }
#pragma unroll
    for (int i = 0; i < kDwNW; ++i) out[i] = (ow0 + i < g.W) ? to_acc<T>(src[i]) : Acc(0);
    return;
  }
#pragma unroll
  for (int i = 0; i < kDwNW; ++i) out[i] = Acc(0);
}

// ----------------------------------------------------------------------------
// Forward (flip = 0) and input-grad (flip = 1, weights mirrored in all three
// axes) of the stride-1 same-padding depthwise convolution.
//   y[n,c,o] = bias[c] + sum_t x[n,c,o+t-P] * w[c,t]
// ----------------------------------------------------------------------------
template <typename T, int K, int NH>
__global__ void __launch_bounds__(256) dw_s1_conv_kernel(const T* __restrict__ x,
                                                         const T* __restrict__ wgt,
                                                         const T* __restrict__ bias,
                                                         const T* __restrict__ addend,
                                                         T* __restrict__ y,
                                                         GnPartial* __restrict__ stats,
                                                         DwS1Geom g, int flip) {
  using Acc = typename Elem<T>::Acc;
  constexpr int P = K / 2;
  constexpr int K3 = K * K * K;
  constexpr bool kWReg = (K <= 3);
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Acc* sw = reinterpret_cast<Acc*>(smem_raw);                                  // K^3 weights
  T* sp = reinterpret_cast<T*>(smem_raw + ((K3 * sizeof(Acc) + 15) / 16) * 16);  // plane tile

  int b = blockIdx.x;
  const int tw = b % g.tilesW;
  b /= g.tilesW;
  const int th = b % g.tilesH;
  b /= g.tilesH;
  const int td = b % g.tilesD;
  const int nc = b / g.tilesD;
  const int c = nc % g.C;
  const int w0 = tw * g.TW, h0 = th * g.TH, d0 = td * g.TD;
  const int rsw = DwTile<T>::row_elems(g.TW, P);
  const int rows = g.TH + 2 * P;
  const int wt = threadIdx.x % g.LW;
  const int tr = threadIdx.x / g.LW;
  const int hrow = tr * NH;  // first output row of this thread, relative to h0
  const bool active = tr < g.TR;

  for (int t = threadIdx.x; t < K3; t += blockDim.x) {
    const int src = flip ? (K3 - 1 - t) : t;
    sw[t] = to_acc<T>(wgt[(size_t)c * K3 + src]);
  }
  __syncthreads();
  Acc wr[kWReg ? K3 : 1];
  if constexpr (kWReg) {
#pragma unroll
    for (int t = 0; t < K3; ++t) wr[t] = sw[t];
  }
  const Acc bv = bias != nullptr ? to_acc<T>(bias[c]) : Acc(0);

  const size_t vol_elems = (size_t)g.D * g.H * g.W;
  const T* xv = x + (size_t)nc * vol_elems;
  T* yv = y + (size_t)nc * vol_elems;
  const int dcount = min(g.TD, g.D - d0);
  const int nsteps = dcount + K - 1;

  Acc acc[K][NH][kDwNW];
#pragma unroll
  for (int a = 0; a < K; ++a)
#pragma unroll
    for (int jh = 0; jh < NH; ++jh)
#pragma unroll
      for (int i = 0; i < kDwNW; ++i) acc[a][jh][i] = Acc(0);

  // shifted running sums for GroupNorm statistics
  Acc st_n = Acc(0), st_shift = Acc(0), st_s1 = Acc(0), st_s2 = Acc(0);

  const int ow0 = w0 + kDwNW * wt;
  const bool vec_store = g.vec && (ow0 + kDwNW <= g.W);

  for (int sb = 0; sb < nsteps; sb += K) {
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const int s = sb + j;
      if (s < nsteps) {
        __syncthreads();
        dw_load_plane<T, P>(sp, xv, d0 - P + s, h0, w0, g, rows, rsw);
        __syncthreads();
        // output plane s starts here: its slot is j
#pragma unroll
        for (int jh = 0; jh < NH; ++jh)
#pragma unroll
          for (int i = 0; i < kDwNW; ++i) acc[j][jh][i] = Acc(0);
        if (active) {
#pragma unroll
          for (int r = 0; r < NH + K - 1; ++r) {
            Acc win[kDwNW + 2 * P];
            dw_read_window<T, P>(sp, hrow + r, rsw, wt, win);
#pragma unroll
            for (int jh = 0; jh < NH; ++jh) {
              const int kh = r - jh;
              if (kh < 0 || kh >= K) continue;
#pragma unroll
              for (int kd = 0; kd < K; ++kd) {
                const int slot = (j - kd + K) % K;
#pragma unroll
                for (int kw = 0; kw < K; ++kw) {
                  const int ti = (kd * K + kh) * K + kw;
                  const Acc wv = kWReg ? wr[kWReg ? ti : 0] : sw[ti];
#pragma unroll
                  for (int i = 0; i < kDwNW; ++i) acc[slot][jh][i] = fma(win[i + kw], wv, acc[slot][jh][i]);
                }
              }
            }
          }
        }
        // output plane s-(K-1) is complete; its slot is (j+1) % K
        const int o = s - (K - 1);
        if (active && o >= 0) {
          const int slot = (j + 1) % K;
          const int od = d0 + o;
#pragma unroll
          for (int jh = 0; jh < NH; ++jh) {
            const int oh = h0 + hrow + jh;
            if (oh >= g.H) continue;
            Acc v[kDwNW];
#pragma unroll
            for (int i = 0; i < kDwNW; ++i) v[i] = acc[slot][jh][i] + bv;
            const size_t row_off = ((size_t)od * g.H + oh) * g.W + ow0;
            if (addend != nullptr) {
              Acc av[kDwNW];
              dw_load_dy_patch<T>(addend + (size_t)nc * vol_elems + (size_t)od * g.H * g.W, oh, ow0, g,
                                  vec_store, av);
#pragma unroll
              for (int i = 0; i < kDwNW; ++i) v[i] += av[i];
            }
            T* dst = yv + row_off;
            if (vec_store) {
              constexpr int E = DwTile<T>::E;
#pragma unroll
              for (int q = 0; q < kDwNW / E; ++q)
                reinterpret_cast<uint4*>(dst)[q] = pack16<T>(v + q * E);
            } else {
#pragma unroll
              for (int i = 0; i < kDwNW; ++i)
                if (ow0 + i < g.W) dst[i] = from_acc<T>(v[i]);
            }
            if (stats != nullptr) {
#pragma unroll
              for (int i = 0; i < kDwNW; ++i) {
                if (ow0 + i < g.W) {
                  const Acc r = to_acc<T>(from_acc<T>(v[i]));  // statistics of the stored value
                  if (st_n == Acc(0)) st_shift = r;
                  const Acc dlt = r - st_shift;
                  st_s1 += dlt;
                  st_s2 = fma(dlt, dlt, st_s2);
                  st_n += Acc(1);
                }
              }
            }
          }
        }
      }
    }
  }

  if (stats != nullptr) {
    __shared__ double red[3 * 32];
    double n = (double)st_n, mean = 0.0, m2 = 0.0;
    if (st_n > Acc(0)) {
      const double s1 = (double)st_s1, s2 = (double)st_s2;
      mean = (double)st_shift + s1 / n;
      m2 = fmax(s2 - s1 * s1 / n, 0.0);
    }
    __syncthreads();
    block_merge_stats(n, mean, m2, red);
    if (threadIdx.x == 0) {
      const int tiles = g.tilesW * g.tilesH * g.tilesD;
      const int tile = (td * g.tilesH + th) * g.tilesW + tw;
      GnPartial gp;
      gp.count = n;
      gp.mean = mean;
      gp.m2 = m2;
      gp.pad = 0.0;
      stats[(size_t)nc * tiles + tile] = gp;
    }
  }
}

// ----------------------------------------------------------------------------
// Weight grad, every tap in one thread (k = 1, 3):
//   dw[c,t] += sum_o x[n,c,o+t-P] * dy[n,c,o];  db[c] += sum_o dy[n,c,o]
// The thread keeps the last K dy planes of its 8*NH outputs in registers and
// pairs each new x plane with all of them.
// Partial sums per CTA go to part[(nc*tiles + tile)*(K^3+1) + tap].
// ----------------------------------------------------------------------------
template <typename A, int NV>
__device__ void block_sum_to_smem(A (&v)[NV], A* red /* [warps][NV] */) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
#pragma unroll
  for (int t = 0; t < NV; ++t) {
    A s = v[t];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    v[t] = s;
  }
  if (lane == 0) {
#pragma unroll
    for (int t = 0; t < NV; ++t) red[warp * NV + t] = v[t];
  }
}

template <typename T, int K, int NH>
__global__ void __launch_bounds__(256) dw_s1_wgrad_kernel(const T* __restrict__ x,
                                                          const T* __restrict__ dy,
                                                          typename Elem<T>::Acc* __restrict__ part,
                                                          DwS1Geom g) {
  using Acc = typename Elem<T>::Acc;
  constexpr int P = K / 2;
  constexpr int K3 = K * K * K;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* sp = reinterpret_cast<T*>(smem_raw);

  int b = blockIdx.x;
  const int tw = b % g.tilesW;
  b /= g.tilesW;
  const int th = b % g.tilesH;
  b /= g.tilesH;
  const int td = b % g.tilesD;
  const int nc = b / g.tilesD;
  const int w0 = tw * g.TW, h0 = th * g.TH, d0 = td * g.TD;
  const int rsw = DwTile<T>::row_elems(g.TW, P);
  const int rows = g.TH + 2 * P;
  const int wt = threadIdx.x % g.LW;
  const int tr = threadIdx.x / g.LW;
  const int hrow = tr * NH;
  const bool active = tr < g.TR;
  const int ow0 = w0 + kDwNW * wt;
  const bool vec = g.vec && (ow0 + kDwNW <= g.W);

  const size_t vol_elems = (size_t)g.D * g.H * g.W;
  const T* xv = x + (size_t)nc * vol_elems;
  const T* dyv = dy + (size_t)nc * vol_elems;
  const int dcount = min(g.TD, g.D - d0);
  const int nsteps = dcount + K - 1;

  Acc acc[K3 + 1];
#pragma unroll
  for (int t = 0; t <= K3; ++t) acc[t] = Acc(0);
  Acc dyr[K][NH][kDwNW];
#pragma unroll
  for (int a = 0; a < K; ++a)
#pragma unroll
    for (int jh = 0; jh < NH; ++jh)
#pragma unroll
      for (int i = 0; i < kDwNW; ++i) dyr[a][jh][i] = Acc(0);

  for (int sb = 0; sb < nsteps; sb += K) {
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const int s = sb + j;
      if (s < nsteps) {
        __syncthreads();
        dw_load_plane<T, P>(sp, xv, d0 - P + s, h0, w0, g, rows, rsw);
        // dy plane s (relative) into ring slot j
        if (active && s < dcount) {
          const T* plane = dyv + (size_t)(d0 + s) * g.H * g.W;
#pragma unroll
          for (int jh = 0; jh < NH; ++jh) dw_load_dy_patch<T>(plane, h0 + hrow + jh, ow0, g, vec, dyr[j][jh]);
#pragma unroll
          for (int jh = 0; jh < NH; ++jh)
#pragma unroll
            for (int i = 0; i < kDwNW; ++i) acc[K3] += dyr[j][jh][i];
        } else {
#pragma unroll
          for (int jh = 0; jh < NH; ++jh)
#pragma unroll
            for (int i = 0; i < kDwNW; ++i) dyr[j][jh][i] = Acc(0);
        }
        __syncthreads();
        if (active) {
#pragma unroll
          for (int r = 0; r < NH + K - 1; ++r) {
            Acc win[kDwNW + 2 * P];
            dw_read_window<T, P>(sp, hrow + r, rsw, wt, win);
#pragma unroll
            for (int jh = 0; jh < NH; ++jh) {
              const int kh = r - jh;
              if (kh < 0 || kh >= K) continue;
#pragma unroll
              for (int kd = 0; kd < K; ++kd) {
                const int slot = (j - kd + K) % K;
#pragma unroll
                for (int kw = 0; kw < K; ++kw) {
                  Acc sacc = acc[(kd * K + kh) * K + kw];
#pragma unroll
                  for (int i = 0; i < kDwNW; ++i) sacc = fma(win[i + kw], dyr[slot][jh][i], sacc);
                  acc[(kd * K + kh) * K + kw] = sacc;
                }
              }
            }
          }
        }
      }
    }
  }

  __shared__ Acc red[8 * (K3 + 1)];
  __syncthreads();
  block_sum_to_smem<Acc, K3 + 1>(acc, red);
  __syncthreads();
  const int nwarps = blockDim.x >> 5;
  const int tiles = g.tilesW * g.tilesH * g.tilesD;
  const int tile = (td * g.tilesH + th) * g.tilesW + tw;
  for (int t = threadIdx.x; t <= K3; t += blockDim.x) {
    Acc s = Acc(0);
    for (int w = 0; w < nwarps; ++w) s += red[w * (K3 + 1) + t];
    part[((size_t)nc * tiles + tile) * (K3 + 1) + t] = s;
  }
}

// ----------------------------------------------------------------------------
// Weight grad for k = 5, 7: the CTA's threads form K groups; group g owns the
// K*K taps with kd = g, so a thread holds K*K accumulators instead of K^3.
// All groups share the shared-memory x plane; group g pairs x plane d_in with
// dy plane d_in + P - g, read straight from global memory (L2-resident).
// ----------------------------------------------------------------------------
template <typename T, int K, int NH>
__global__ void __launch_bounds__(448) dw_s1_wgrad_grouped_kernel(
    const T* __restrict__ x, const T* __restrict__ dy, typename Elem<T>::Acc* __restrict__ part,
    DwS1Geom g) {
  using Acc = typename Elem<T>::Acc;
  constexpr int P = K / 2;
  constexpr int K2 = K * K;
  constexpr int K3 = K2 * K;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* sp = reinterpret_cast<T*>(smem_raw);

  int b = blockIdx.x;
  const int tw = b % g.tilesW;
  b /= g.tilesW;
  const int th = b % g.tilesH;
  b /= g.tilesH;
  const int td = b % g.tilesD;
  const int nc = b / g.tilesD;
  const int w0 = tw * g.TW, h0 = th * g.TH, d0 = td * g.TD;
  const int rsw = DwTile<T>::row_elems(g.TW, P);
  const int rows = g.TH + 2 * P;
  const int G = blockDim.x / K;  // threads per group: LW*TR rounded up to whole warps
  const int grp = threadIdx.x / G;
  const int lt = threadIdx.x - grp * G;
  const int wt = lt % g.LW;
  const int tr = lt / g.LW;
  const int hrow = tr * NH;
  const bool active = tr < g.TR;
  const int ow0 = w0 + kDwNW * wt;
  const bool vec = g.vec && (ow0 + kDwNW <= g.W);

  const size_t vol_elems = (size_t)g.D * g.H * g.W;
  const T* xv = x + (size_t)nc * vol_elems;
  const T* dyv = dy + (size_t)nc * vol_elems;
  const int dcount = min(g.TD, g.D - d0);
  const int nsteps = dcount + K - 1;

  Acc acc[K2 + 1];
#pragma unroll
  for (int t = 0; t <= K2; ++t) acc[t] = Acc(0);

  for (int s = 0; s < nsteps; ++s) {
    __syncthreads();
    dw_load_plane<T, P>(sp, xv, d0 - P + s, h0, w0, g, rows, rsw);
    // this group's dy plane: relative depth s - grp
    const int orel = s - grp;
    Acc dyp[NH][kDwNW];
    if (active && orel >= 0 && orel < dcount) {
      const T* plane = dyv + (size_t)(d0 + orel) * g.H * g.W;
#pragma unroll
      for (int jh = 0; jh < NH; ++jh) dw_load_dy_patch<T>(plane, h0 + hrow + jh, ow0, g, vec, dyp[jh]);
    } else {
#pragma unroll
      for (int jh = 0; jh < NH; ++jh)
#pragma unroll
        for (int i = 0; i < kDwNW; ++i) dyp[jh][i] = Acc(0);
    }
    if (grp == 0) {
#pragma unroll
      for (int jh = 0; jh < NH; ++jh)
#pragma unroll
        for (int i = 0; i < kDwNW; ++i) acc[K2] += dyp[jh][i];
    }
    __syncthreads();
    if (!active) continue;
#pragma unroll
    for (int r = 0; r < NH + K - 1; ++r) {
      Acc win[kDwNW + 2 * P];
      dw_read_window<T, P>(sp, hrow + r, rsw, wt, win);
#pragma unroll
      for (int jh = 0; jh < NH; ++jh) {
        const int kh = r - jh;
        if (kh < 0 || kh >= K) continue;
#pragma unroll
        for (int kw = 0; kw < K; ++kw) {
          Acc sacc = acc[kh * K + kw];
#pragma unroll
          for (int i = 0; i < kDwNW; ++i) sacc = fma(win[i + kw], dyp[jh][i], sacc);
          acc[kh * K + kw] = sacc;
        }
      }
    }
  }

  __shared__ Acc red[14 * (K2 + 1)];
  __syncthreads();
  block_sum_to_smem<Acc, K2 + 1>(acc, red);
  __syncthreads();
  const int wpg = G >> 5;  // warps per group
  const int tiles = g.tilesW * g.tilesH * g.tilesD;
  const int tile = (td * g.tilesH + th) * g.tilesW + tw;
  Acc* dst = part + ((size_t)nc * tiles + tile) * (K3 + 1);
  for (int e = threadIdx.x; e < K * (K2 + 1); e += blockDim.x) {
    const int gg = e / (K2 + 1);
    const int t = e - gg * (K2 + 1);
    if (t == K2 && gg != 0) continue;
    Acc s = Acc(0);
    for (int w = 0; w < wpg; ++w) s += red[(gg * wpg + w) * (K2 + 1) + t];
    if (t == K2) dst[K3] = s;
    else dst[gg * K2 + t] = s;
  }
}

// Deterministic second pass: dw[c,t] = sum over (n, tile) of the partials, in
// a fixed order; dbias[c] from tap index K^3.
template <typename T, typename O = T>
__global__ void dw_wgrad_finish_kernel(const typename Elem<T>::Acc* __restrict__ part,
                                       O* __restrict__ dw, O* __restrict__ db, int N, int C,
                                       int tiles, int K3) {
  using Acc = typename Elem<T>::Acc;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= C * (K3 + 1)) return;
  const int c = idx / (K3 + 1);
  const int t = idx - c * (K3 + 1);
  Acc s = Acc(0);
  for (int n = 0; n < N; ++n) {
    const Acc* p = part + ((size_t)(n * C + c) * tiles) * (K3 + 1) + t;
    for (int i = 0; i < tiles; ++i) s += p[(size_t)i * (K3 + 1)];
  }
  // O = float for 16-bit T: the T-rounded value, widened (what a T gradient cast to fp32 holds)
  const T v = from_acc<T>(s);
  O o;
  if constexpr (std::is_same<O, T>::value) {
    o = v;
  } else {
    o = static_cast<O>(to_acc<T>(v));
  }
  if (t < K3) dw[(size_t)c * K3 + t] = o;
  else if (db != nullptr) db[c] = o;
}

}  // namespace mednext
