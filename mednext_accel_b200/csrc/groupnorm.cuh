// GroupNorm with groups == channels (nn.GroupNorm(C, C), models/blocks.py:74 of
// the reference): per-(sample, channel) statistics over the spatial volume.
//   forward : z = (x - mean) * rstd * gamma + beta,  rstd = 1/sqrt(var + eps)
//   backward: dx = rstd * gamma * (dz - S1/V - xhat * S2/V),
//             S1 = sum dz, S2 = sum dz * xhat;  dgamma = sum_n S2, dbeta = sum_n S1
// Every reduction is two-pass with a fixed order, so results are bitwise
// reproducible from run to run.
#pragma once

#include <type_traits>

#include "common.cuh"
#include "depthwise_s1.cuh"  // GnPartial, chan_merge, block_merge_stats

namespace mednext {

struct GnBwdPartial {
  double s1, s2;
};

// Merge the per-tile (count, mean, M2) partials of each (n, c) in tile order.
// One warp per (n, c): lane l merges partials l, l + 32, ... in order, then a
// butterfly over the lanes; lane 0 writes.  The order is fixed (deterministic).
static __global__ void gn_finalize_kernel(const GnPartial* __restrict__ part, int tiles, int nc_total,
                                   float eps, float* __restrict__ stats) {
  const long long nc = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;  // 64-bit: no wrap at 2^27 warps
  const int lane = threadIdx.x & 31;
  if (nc >= nc_total) return;  // warp-uniform
  double n = 0.0, mean = 0.0, m2 = 0.0;
  const GnPartial* p = part + (size_t)nc * tiles;
  for (int t = lane; t < tiles; t += 32) chan_merge(n, mean, m2, p[t].count, p[t].mean, p[t].m2);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double nb = __shfl_xor_sync(0xffffffffu, n, o);
    const double mb = __shfl_xor_sync(0xffffffffu, mean, o);
    const double qb = __shfl_xor_sync(0xffffffffu, m2, o);
    chan_merge(n, mean, m2, nb, mb, qb);
  }
  if (lane != 0) return;
  const double var = n > 0.0 ? m2 / n : 0.0;  // biased variance, as GroupNorm uses
  stats[2 * nc] = (float)mean;
  stats[2 * nc + 1] = (float)(1.0 / sqrt(var + (double)eps));
}

template <typename T>
__device__ __forceinline__ bool vec_ok(const void* p, size_t vol) {
  constexpr int E = 16 / (int)sizeof(T);
  return (vol % E) == 0 && ((reinterpret_cast<uintptr_t>(p) & 15) == 0);
}

// Standalone statistics: per-thread shifted sums, block Chan merge, one
// partial per (n, c, chunk).  Each (n, c) volume starts `pitch` elements after
// the previous one and its first `vol` elements are read, as rows of
// `row_pitch` elements of which the first `row_len` are statistics (row_len =
// row_pitch: every element).
template <typename T>
__global__ void __launch_bounds__(256) gn_stats_partial_kernel(const T* __restrict__ x,
                                                               GnPartial* __restrict__ part,
                                                               size_t vol, size_t pitch, int chunks,
                                                               int row_pitch, int row_len) {
  using Acc = typename Elem<T>::Acc;
  const int j = blockIdx.x % chunks;
  const size_t nc = blockIdx.x / chunks;
  // chunks start on 8-element boundaries (16-byte vectors); trailing chunks may be empty
  const size_t per = ((vol + chunks - 1) / chunks + 7) / 8 * 8;
  const size_t beg = min((size_t)j * per, vol);
  const size_t end = min(beg + per, vol);
  const T* p = x + nc * pitch;
  const bool masked = row_len < row_pitch;
  Acc cnt = Acc(0), shift = Acc(0), s1 = Acc(0), s2 = Acc(0);
  auto add = [&](Acc v) {
    if (cnt == Acc(0)) shift = v;
    const Acc d = v - shift;
    s1 += d;
    s2 = fma(d, d, s2);
    cnt += Acc(1);
  };
  auto in_row = [&](size_t i) { return !masked || (int)(i % (size_t)row_pitch) < row_len; };
  constexpr int E = 16 / (int)sizeof(T);
  if (vec_ok<T>(x, pitch) && beg % E == 0 && (!masked || row_pitch % E == 0)) {
    // whole 16-byte chunks, then the (at most E-1) trailing elements
    const size_t vend = beg + (end - beg) / E * E;
    for (size_t i = beg + (size_t)threadIdx.x * E; i < vend; i += (size_t)blockDim.x * E) {
      Acc v[E];
      unpack16<T>(__ldg(reinterpret_cast<const uint4*>(p + i)), v);
      if (masked) {
        const int col = (int)(i % (size_t)row_pitch);
#pragma unroll
        for (int e = 0; e < E; ++e)
          if (col + e < row_len) add(v[e]);
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) add(v[e]);
      }
    }
    for (size_t i = vend + threadIdx.x; i < end; i += blockDim.x)
      if (in_row(i)) add(to_acc<T>(__ldg(p + i)));
  } else {
    for (size_t i = beg + threadIdx.x; i < end; i += blockDim.x)
      if (in_row(i)) add(to_acc<T>(__ldg(p + i)));
  }
  double n = (double)cnt, mean = 0.0, m2 = 0.0;
  if (cnt > Acc(0)) {
    mean = (double)shift + (double)s1 / n;
    m2 = fmax((double)s2 - (double)s1 * (double)s1 / n, 0.0);
  }
  __shared__ double red[3 * 32];
  block_merge_stats(n, mean, m2, red);
  if (threadIdx.x == 0) {
    GnPartial gp;
    gp.count = n;
    gp.mean = mean;
    gp.m2 = m2;
    gp.pad = 0.0;
    part[nc * chunks + j] = gp;
  }
}

template <typename G>
__device__ __forceinline__ float param_f(const G* p, int c) {
  return (float)to_acc<G>(p[c]);
}

// z = (x - mean) * rstd * gamma + beta
template <typename TX, typename TY, typename TG>
__global__ void __launch_bounds__(256) gn_fwd_kernel(const TX* __restrict__ x,
                                                     const float* __restrict__ stats,
                                                     const TG* __restrict__ gamma,
                                                     const TG* __restrict__ beta,
                                                     TY* __restrict__ y, int C, size_t vol,
                                                     int chunks) {
  const int j = blockIdx.x % chunks;
  const size_t nc = blockIdx.x / chunks;
  const int c = (int)(nc % C);
  const float mean = stats[2 * nc], rstd = stats[2 * nc + 1];
  const float a = rstd * (gamma != nullptr ? param_f(gamma, c) : 1.0f);
  const float bsh = (beta != nullptr ? param_f(beta, c) : 0.0f) - mean * a;
  const size_t per = (vol + chunks - 1) / chunks;
  const size_t beg = (size_t)j * per;
  const size_t end = min(beg + per, vol);
  const TX* src = x + nc * vol;
  TY* dst = y + nc * vol;
  for (size_t i = beg + threadIdx.x; i < end; i += blockDim.x) {
    const float v = (float)to_acc<TX>(src[i]);
    dst[i] = from_acc<TY>((typename Elem<TY>::Acc)fmaf(v, a, bsh));
  }
}

// Backward pass 1: S1 = sum dz, S2 = sum dz * xhat per (n, c, chunk).
template <typename TD, typename TX>
__global__ void __launch_bounds__(256) gn_bwd_partial_kernel(const TD* __restrict__ dz,
                                                             const TX* __restrict__ x,
                                                             const float* __restrict__ stats,
                                                             GnBwdPartial* __restrict__ part,
                                                             size_t vol, int chunks) {
  const int j = blockIdx.x % chunks;
  const size_t nc = blockIdx.x / chunks;
  const float mean = stats[2 * nc], rstd = stats[2 * nc + 1];
  const size_t per = (vol + chunks - 1) / chunks;
  const size_t beg = (size_t)j * per;
  const size_t end = min(beg + per, vol);
  const TD* g = dz + nc * vol;
  const TX* xs = x + nc * vol;
  float s1 = 0.f, s2 = 0.f;
  for (size_t i = beg + threadIdx.x; i < end; i += blockDim.x) {
    const float d = (float)to_acc<TD>(__ldg(g + i));
    const float xh = ((float)to_acc<TX>(__ldg(xs + i)) - mean) * rstd;
    s1 += d;
    s2 = fmaf(d, xh, s2);
  }
  __shared__ float red[2 * 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    s2 += __shfl_xor_sync(0xffffffffu, s2, o);
  }
  if ((threadIdx.x & 31) == 0) {
    red[2 * (threadIdx.x >> 5)] = s1;
    red[2 * (threadIdx.x >> 5) + 1] = s2;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double a = 0.0, b = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      a += red[2 * w];
      b += red[2 * w + 1];
    }
    GnBwdPartial gp;
    gp.s1 = a;
    gp.s2 = b;
    part[nc * chunks + j] = gp;
  }
}

// Fold the `tiles` partials of each (n, c) into slot 0 of its row, in place, in
// two passes with a fixed order: pass 1 has one CTA per span of kGnFoldSpan
// partials and writes the span's sum into the span's first slot; pass 2
// (gn_fold_spans_kernel) adds those slots into slot 0.  Within a CTA, thread t
// sums partials t, t+256, ... in order, then a fixed-shape tree.
constexpr int kGnFoldSpan = 4096;
static __global__ void __launch_bounds__(256) gn_fold_partials_kernel(GnBwdPartial* __restrict__ part, int tiles) {
  const int spans = (tiles + kGnFoldSpan - 1) / kGnFoldSpan;
  const size_t nc = blockIdx.x / spans;
  const int sp = (int)(blockIdx.x % spans);
  GnBwdPartial* p = part + nc * tiles + (size_t)sp * kGnFoldSpan;
  const int count = min(kGnFoldSpan, tiles - sp * kGnFoldSpan);
  double a = 0.0, b = 0.0;
  for (int t = threadIdx.x; t < count; t += blockDim.x) {
    a += p[t].s1;
    b += p[t].s2;
  }
  __shared__ double ra[256], rb[256];
  ra[threadIdx.x] = a;
  rb[threadIdx.x] = b;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if ((int)threadIdx.x < s) {
      ra[threadIdx.x] += ra[threadIdx.x + s];
      rb[threadIdx.x] += rb[threadIdx.x + s];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    GnBwdPartial gp;
    gp.s1 = ra[0];
    gp.s2 = rb[0];
    p[0] = gp;
  }
}
static __global__ void gn_fold_spans_kernel(GnBwdPartial* __restrict__ part, int tiles, int nc_total) {
  const int nc = blockIdx.x * blockDim.x + threadIdx.x;
  if (nc >= nc_total) return;
  GnBwdPartial* p = part + (size_t)nc * tiles;
  double a = p[0].s1, b = p[0].s2;
  for (int s = kGnFoldSpan; s < tiles; s += kGnFoldSpan) {
    a += p[s].s1;
    b += p[s].s2;
  }
  p[0].s1 = a;
  p[0].s2 = b;
}

// Backward pass 2: dx = rstd * gamma * (dz - S1/V - xhat * S2/V), with the
// folded sums of (n, c) at folded[nc * stride] and V = vol; all `pitch` elements
// of each (n, c) row are written (positions past the valid voxels of a pitched
// row get values without meaning).
// The sums of (n, c) are folded[nc * stride] plus, with spans > 1, the span sums
// at every kGnFoldSpan-th slot after it (added in order, as gn_fold_spans_kernel
// does).  dgamma / dbeta (one sample, N = 1): the chunk-0 CTA of each channel
// writes them, as gn_param_grad_kernel would.
template <typename TD, typename TX, typename TO, typename TG>
__global__ void __launch_bounds__(256) gn_bwd_apply_kernel(
    const TD* __restrict__ dz, const TX* __restrict__ x, const float* __restrict__ stats,
    const TG* __restrict__ gamma, const GnBwdPartial* __restrict__ folded, int stride, int spans,
    TO* __restrict__ dx, int C, size_t vol, size_t pitch, int chunks, float* __restrict__ dgamma,
    float* __restrict__ dbeta) {
  const int j = blockIdx.x % chunks;
  const size_t nc = blockIdx.x / chunks;
  const int c = (int)(nc % C);
  GnBwdPartial f = folded[nc * stride];
  for (int sp = 1; sp < spans; ++sp) {
    f.s1 += folded[nc * stride + (size_t)sp * kGnFoldSpan].s1;
    f.s2 += folded[nc * stride + (size_t)sp * kGnFoldSpan].s2;
  }
  if (j == 0 && threadIdx.x == 0) {
    if (dbeta != nullptr) dbeta[c] = (float)(0.0 + f.s1);
    if (dgamma != nullptr) dgamma[c] = (float)(0.0 + f.s2);
  }
  const float m1 = (float)(f.s1 / (double)vol);
  const float m2 = (float)(f.s2 / (double)vol);
  const float mean = stats[2 * nc], rstd = stats[2 * nc + 1];
  const float gr = rstd * (gamma != nullptr ? param_f(gamma, c) : 1.0f);
  // chunks start on 8-element boundaries (16-byte vectors); trailing chunks may be empty
  const size_t per = ((pitch + chunks - 1) / chunks + 7) / 8 * 8;
  const size_t beg = min((size_t)j * per, pitch);
  const size_t end = min(beg + per, pitch);
  const TD* g = dz + nc * pitch;
  const TX* xs = x + nc * pitch;
  TO* o = dx + nc * pitch;
  size_t i0 = beg;
  if constexpr (std::is_same<TD, TX>::value && std::is_same<TX, TO>::value && sizeof(TX) == 2) {
    constexpr int E = 8;
    if (vec_ok<TX>(dz, pitch) && vec_ok<TX>(x, pitch) && vec_ok<TX>(dx, pitch) && beg % E == 0) {
      const size_t vend = beg + (end - beg) / E * E;
      // four 16-byte vectors of each input in flight per thread: all loads first
      constexpr int U = 4;
      const size_t step = (size_t)blockDim.x * E;
      size_t i = beg + (size_t)threadIdx.x * E;
      for (; i + (U - 1) * step < vend; i += U * step) {
        uint4 qd[U], qx[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          qd[u] = __ldg(reinterpret_cast<const uint4*>(g + i + u * step));
          qx[u] = __ldg(reinterpret_cast<const uint4*>(xs + i + u * step));
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          float d[E], xv[E], r[E];
          unpack16<TD>(qd[u], d);
          unpack16<TX>(qx[u], xv);
#pragma unroll
          for (int e = 0; e < E; ++e) r[e] = gr * (d[e] - m1 - (xv[e] - mean) * rstd * m2);
          *reinterpret_cast<uint4*>(o + i + u * step) = pack16<TO>(r);
        }
      }
      for (; i < vend; i += step) {
        float d[E], xv[E], r[E];
        unpack16<TD>(__ldg(reinterpret_cast<const uint4*>(g + i)), d);
        unpack16<TX>(__ldg(reinterpret_cast<const uint4*>(xs + i)), xv);
#pragma unroll
        for (int e = 0; e < E; ++e) r[e] = gr * (d[e] - m1 - (xv[e] - mean) * rstd * m2);
        *reinterpret_cast<uint4*>(o + i) = pack16<TO>(r);
      }
      i0 = vend;
    }
  }
  for (size_t i = i0 + threadIdx.x; i < end; i += blockDim.x) {
    const float d = (float)to_acc<TD>(__ldg(g + i));
    const float xh = ((float)to_acc<TX>(__ldg(xs + i)) - mean) * rstd;
    o[i] = from_acc<TO>((typename Elem<TO>::Acc)(gr * (d - m1 - xh * m2)));
  }
}

// dgamma[c] = sum_n S2[n,c], dbeta[c] = sum_n S1[n,c] from the folded sums (fixed order).
static __global__ void gn_param_grad_kernel(const GnBwdPartial* __restrict__ folded, int stride, int N, int C,
                                            float* __restrict__ dgamma, float* __restrict__ dbeta) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  double a = 0.0, b = 0.0;
  for (int n = 0; n < N; ++n) {
    const GnBwdPartial f = folded[((size_t)n * C + c) * stride];
    a += f.s1;
    b += f.s2;
  }
  if (dbeta != nullptr) dbeta[c] = (float)a;
  if (dgamma != nullptr) dgamma[c] = (float)b;
}

}  // namespace mednext
