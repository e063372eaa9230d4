// Depthwise Conv3d stride 2 (down block) and depthwise ConvTranspose3d stride 2
// (up block), both with padding k/2.  The two operators share three index
// patterns between a "big" grid and a "small" grid (small = ceil(big/2) for the
// down block, big = 2*small-1 for the up block):
//   gather : small[m] = sum_t big[2m - P + t] * w[t]          (down fwd, up dgrad)
//   scatter: big[i]   = sum_{t: i+P-t even} small[(i+P-t)/2] * w[t]
//                                                            (down dgrad, up fwd)
//   wgrad  : dw[t]    = sum_m big[2m - P + t] * small[m]     (down dW, up dW)
// Reference: ops/_triton/depthwise.py:206-268 (stride-2 dX), 86-156 (transpose dW).
#pragma once

#include "common.cuh"

namespace mednext {

struct DwS2Geom {
  int N, C;
  int Db, Hb, Wb;  // big grid
  int Ds, Hs, Ws;  // small grid
  long long bp;    // elements between consecutive (n, c) volumes of the big grid (>= Db*Hb*Wb)
};

// gather: one thread per small-grid output, consecutive threads along W.
template <typename T, int K>
__global__ void __launch_bounds__(256) dw_s2_gather_kernel(const T* __restrict__ big,
                                                           const T* __restrict__ wgt,
                                                           const T* __restrict__ bias,
                                                           T* __restrict__ small, DwS2Geom g) {
  using Acc = typename Elem<T>::Acc;
  constexpr int P = K / 2;
  constexpr int K3 = K * K * K;
  const size_t svol = (size_t)g.Ds * g.Hs * g.Ws;
  const size_t total = (size_t)g.N * g.C * svol;
  const size_t bvol = (size_t)g.Db * g.Hb * g.Wb;
  for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const size_t nc = idx / svol;
    size_t r = idx - nc * svol;
    const int ow = (int)(r % g.Ws);
    r /= g.Ws;
    const int oh = (int)(r % g.Hs);
    const int od = (int)(r / g.Hs);
    const int c = (int)(nc % g.C);
    const T* src = big + nc * (size_t)g.bp;
    const T* w = wgt + (size_t)c * K3;
    Acc acc = bias != nullptr ? to_acc<T>(bias[c]) : Acc(0);
#pragma unroll
    for (int kd = 0; kd < K; ++kd) {
      const int id = 2 * od - P + kd;
      if (id < 0 || id >= g.Db) continue;
#pragma unroll
      for (int kh = 0; kh < K; ++kh) {
        const int ih = 2 * oh - P + kh;
        if (ih < 0 || ih >= g.Hb) continue;
        const T* row = src + ((size_t)id * g.Hb + ih) * g.Wb;
#pragma unroll
        for (int kw = 0; kw < K; ++kw) {
          const int iw = 2 * ow - P + kw;
          if (iw < 0 || iw >= g.Wb) continue;
          acc = fma(to_acc<T>(__ldg(row + iw)), to_acc<T>(__ldg(w + (kd * K + kh) * K + kw)), acc);
        }
      }
    }
    small[idx] = from_acc<T>(acc);
  }
}

// scatter: one thread per big-grid output.  Per axis only taps with
// t = (i + P) mod 2 (mod 2) contribute, i.e. ceil(K/2) or floor(K/2) taps.
template <typename T, int K>
__global__ void __launch_bounds__(256) dw_s2_scatter_kernel(const T* __restrict__ small,
                                                            const T* __restrict__ wgt,
                                                            const T* __restrict__ bias,
                                                            T* __restrict__ big, DwS2Geom g) {
  using Acc = typename Elem<T>::Acc;
  constexpr int P = K / 2;
  constexpr int K3 = K * K * K;
  const size_t bvol = (size_t)g.Db * g.Hb * g.Wb;
  const size_t bp = (size_t)g.bp;
  const size_t total = (size_t)g.N * g.C * bp;
  const size_t svol = (size_t)g.Ds * g.Hs * g.Ws;
  for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const size_t nc = idx / bp;
    size_t r = idx - nc * bp;
    if (r >= bvol) {  // padding tail of a pitched row: keep it finite
      big[idx] = from_acc<T>(Acc(0));
      continue;
    }
    const int iw = (int)(r % g.Wb);
    r /= g.Wb;
    const int ih = (int)(r % g.Hb);
    const int id = (int)(r / g.Hb);
    const int c = (int)(nc % g.C);
    const T* src = small + nc * svol;
    const T* w = wgt + (size_t)c * K3;
    Acc acc = bias != nullptr ? to_acc<T>(bias[c]) : Acc(0);
    // first contributing tap per axis has the parity of (i + P)
    const int td0 = (id + P) & 1, th0 = (ih + P) & 1, tw0 = (iw + P) & 1;
    for (int kd = td0; kd < K; kd += 2) {
      const int md = (id + P - kd) >> 1;
      if (md < 0 || md >= g.Ds) continue;
      for (int kh = th0; kh < K; kh += 2) {
        const int mh = (ih + P - kh) >> 1;
        if (mh < 0 || mh >= g.Hs) continue;
        const T* row = src + ((size_t)md * g.Hs + mh) * g.Ws;
        for (int kw = tw0; kw < K; kw += 2) {
          const int mw = (iw + P - kw) >> 1;
          if (mw < 0 || mw >= g.Ws) continue;
          acc = fma(to_acc<T>(__ldg(row + mw)), to_acc<T>(__ldg(w + (kd * K + kh) * K + kw)), acc);
        }
      }
    }
    big[idx] = from_acc<T>(acc);
  }
}

// wgrad: the CTA's threads form K groups (group g owns the K*K taps with
// kd = g).  A CTA covers `chunk` consecutive small-grid positions of one
// (sample, channel); with `small_bias` it also sums the small grid (the down
// block's bias grad).  Partials: part[(nc*chunks + j)*(K^3+1) + tap].
template <typename T, int K>
__global__ void __launch_bounds__(448) dw_s2_wgrad_kernel(const T* __restrict__ big,
                                                          const T* __restrict__ small,
                                                          typename Elem<T>::Acc* __restrict__ part,
                                                          DwS2Geom g, int chunk, int chunks,
                                                          int small_bias) {
  using Acc = typename Elem<T>::Acc;
  constexpr int P = K / 2;
  constexpr int K2 = K * K;
  constexpr int K3 = K2 * K;
  const int G = blockDim.x / K;
  const int grp = threadIdx.x / G;
  const int lt = threadIdx.x - grp * G;
  const int j = blockIdx.x % chunks;
  const size_t nc = blockIdx.x / chunks;
  const size_t svol = (size_t)g.Ds * g.Hs * g.Ws;
  const size_t bvol = (size_t)g.Db * g.Hb * g.Wb;
  const T* bsrc = big + nc * (size_t)g.bp;
  const T* ssrc = small + nc * svol;
  const size_t beg = (size_t)j * chunk;
  const size_t end = min(beg + (size_t)chunk, svol);
  Acc acc[K2 + 1];
#pragma unroll
  for (int t = 0; t <= K2; ++t) acc[t] = Acc(0);
  const int kd = grp;
  for (size_t m = beg + lt; m < end; m += G) {
    size_t r = m;
    const int mw = (int)(r % g.Ws);
    r /= g.Ws;
    const int mh = (int)(r % g.Hs);
    const int md = (int)(r / g.Hs);
    const Acc sv = to_acc<T>(__ldg(ssrc + m));
    acc[K2] += sv;
    const int id = 2 * md - P + kd;
    if (id < 0 || id >= g.Db) continue;
#pragma unroll
    for (int kh = 0; kh < K; ++kh) {
      const int ih = 2 * mh - P + kh;
      if (ih < 0 || ih >= g.Hb) continue;
      const T* row = bsrc + ((size_t)id * g.Hb + ih) * g.Wb;
#pragma unroll
      for (int kw = 0; kw < K; ++kw) {
        const int iw = 2 * mw - P + kw;
        if (iw < 0 || iw >= g.Wb) continue;
        acc[kh * K + kw] = fma(to_acc<T>(__ldg(row + iw)), sv, acc[kh * K + kw]);
      }
    }
  }
  // reduce within each group (G is a multiple of 32)
  __shared__ Acc red[14 * (K2 + 1)];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
#pragma unroll
  for (int t = 0; t <= K2; ++t) {
    Acc s = acc[t];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp * (K2 + 1) + t] = s;
  }
  __syncthreads();
  const int wpg = G >> 5;
  Acc* dst = part + ((size_t)nc * chunks + j) * (K3 + 1);
  for (int e = threadIdx.x; e < K * (K2 + 1); e += blockDim.x) {
    const int gg = e / (K2 + 1);
    const int t = e - gg * (K2 + 1);
    Acc s = Acc(0);
    for (int w = 0; w < wpg; ++w) s += red[(gg * wpg + w) * (K2 + 1) + t];
    if (t < K2) dst[gg * K2 + t] = s;
    else if (gg == 0) dst[K3] = small_bias ? s : Acc(0);
  }
}

// Per-(sample, channel, chunk) sums of a tensor into slot K^3 of the wgrad
// partials (bias grad of the up block, whose dy is the big grid).
template <typename T>
__global__ void __launch_bounds__(256) chan_sum_into_partials_kernel(
    const T* __restrict__ src, typename Elem<T>::Acc* __restrict__ part, size_t vol, size_t pitch, int chunks,
    int K3) {
  using Acc = typename Elem<T>::Acc;
  const int j = blockIdx.x % chunks;
  const size_t nc = blockIdx.x / chunks;
  const size_t per = (vol + chunks - 1) / chunks;
  const size_t beg = (size_t)j * per;
  const size_t end = min(beg + per, vol);
  const T* p = src + nc * pitch;
  Acc s = Acc(0);
  for (size_t i = beg + threadIdx.x; i < end; i += blockDim.x) s += to_acc<T>(__ldg(p + i));
  __shared__ Acc red[8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    Acc t = Acc(0);
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    part[((size_t)nc * chunks + j) * (K3 + 1) + K3] = t;
  }
}

}  // namespace mednext
