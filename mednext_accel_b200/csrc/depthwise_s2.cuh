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
  int bw;          // elements between consecutive W-rows of the big grid (>= Wb)
  long long bp;    // elements between consecutive (n, c) volumes of the big grid (Db*Hb*bw)
};

// Work decomposition of the three kernels: a CTA owns one (sample, channel) and
// one plane (gather, scatter) or a run of small-grid planes (wgrad); its warps
// take the rows of the plane in turn and the lanes run along W.  Index math is
// 32-bit per row, the per-channel weights are loaded once per CTA.
constexpr int kS2Warps = 8;

template <typename T, int K>
struct S2Weights {
  using Acc = typename Elem<T>::Acc;
  static constexpr int K3 = K * K * K;
  static constexpr bool kReg = K <= 3;  // registers for k <= 3, shared memory above
  Acc r[kReg ? K3 : 1];
  const Acc* s;
  __device__ __forceinline__ void load(const T* __restrict__ w, Acc* sm) {
    if constexpr (kReg) {
#pragma unroll
      for (int t = 0; t < K3; ++t) r[t] = to_acc<T>(__ldg(w + t));
    } else {
      for (int t = threadIdx.x; t < K3; t += blockDim.x) sm[t] = to_acc<T>(w[t]);
      __syncthreads();
      s = sm;
    }
  }
  __device__ __forceinline__ Acc operator[](int t) const {
    if constexpr (kReg) return r[t];
    else return s[t];
  }
};

// Clamped, unconditional load: out-of-range positions read a valid element and
// are multiplied by zero, so every load of an output's stencil can be in flight
// at once (range checks as branches would serialise the loads per tap row).
template <typename T>
__device__ __forceinline__ typename Elem<T>::Acc s2_ld(const T* __restrict__ p, int i, int n) {
  using Acc = typename Elem<T>::Acc;
  const int c = min(max(i, 0), n - 1);
  const Acc v = to_acc<T>(__ldg(p + c));
  return (i >= 0 && i < n) ? v : Acc(0);
}

// gather: CTA = (n, c, md) small-grid plane; one output per lane.  ADD: the
// addend operand is present (a template flag, so the plain gather keeps its own
// register allocation).
template <typename T, int K, bool ADD>
__global__ void __launch_bounds__(kS2Warps * 32) dw_s2_gather_kernel(const T* __restrict__ big,
                                                                     const T* __restrict__ wgt,
                                                                     const T* __restrict__ bias,
                                                                     const T* __restrict__ addend,
                                                                     T* __restrict__ small, DwS2Geom g) {
  using Acc = typename Elem<T>::Acc;
  constexpr int P = K / 2;
  constexpr int K3 = K * K * K;
  __shared__ Acc wsm[S2Weights<T, K>::kReg ? 1 : K3];
  const int md = (int)(blockIdx.x % (unsigned)g.Ds);
  const int nc = (int)(blockIdx.x / (unsigned)g.Ds);
  const int c = nc % g.C;
  S2Weights<T, K> w;
  w.load(wgt + (size_t)c * K3, wsm);
  const Acc b0 = bias != nullptr ? to_acc<T>(bias[c]) : Acc(0);
  const T* bsrc = big + (size_t)nc * (size_t)g.bp;
  T* dst = small + ((size_t)nc * g.Ds + md) * ((size_t)g.Hs * g.Ws);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int mh = warp; mh < g.Hs; mh += kS2Warps) {
    for (int mw = lane; mw < g.Ws; mw += 32) {
      Acc acc = b0;
#pragma unroll
      for (int kd = 0; kd < K; ++kd) {
        const int id = 2 * md - P + kd;
        const bool dok = id >= 0 && id < g.Db;
        const int idc = min(max(id, 0), g.Db - 1);
#pragma unroll
        for (int kh = 0; kh < K; ++kh) {
          const int ih = 2 * mh - P + kh;
          const bool ok = dok && ih >= 0 && ih < g.Hb;
          const int ihc = min(max(ih, 0), g.Hb - 1);
          const T* row = bsrc + ((size_t)idc * g.Hb + ihc) * g.bw;
#pragma unroll
          for (int kw = 0; kw < K; ++kw) {
            const Acc v = s2_ld<T>(row, 2 * mw - P + kw, g.Wb);
            acc = fma(ok ? v : Acc(0), w[(kd * K + kh) * K + kw], acc);
          }
        }
      }
      if constexpr (ADD) acc += to_acc<T>(addend[(((size_t)nc * g.Ds + md) * g.Hs + mh) * g.Ws + mw]);
      dst[(size_t)mh * g.Ws + mw] = from_acc<T>(acc);
    }
  }
}

// Parity blocks of the scatter.  Along an axis, big index i = 2q + e (e = 0, 1)
// receives small[m] through tap t = i + P - 2m; over both parities m runs over
// q + lo .. q + lo + R - 1, so a thread that owns the 2x2x2 outputs of block q
// reads R^3 small values and uses every tap once (K^3 FMAs for 8 outputs), with
// the tap of each (parity, window offset) pair known at compile time.
template <int K>
struct S2Block {
  static constexpr int P = K / 2;
  static constexpr int lo = -(P / 2);
  static constexpr int R = (1 + P) / 2 - lo + 1;
  // tap joining parity e to window offset a, or -1
  static constexpr int tap(int e, int a) { return (e + P - 2 * (lo + a) >= 0 && e + P - 2 * (lo + a) < K) ? e + P - 2 * (lo + a) : -1; }
};

// scatter: CTA = (n, c, qd) pair of big-grid planes 2qd, 2qd+1; warps take block
// rows, lanes run along W; each thread writes a 2x2x2 output block.  ADD:
// add_even (small-grid shaped) is added at the all-even output 2q.
template <typename T, int K, bool ADD>
__global__ void __launch_bounds__(kS2Warps * 32) dw_s2_scatter_kernel(const T* __restrict__ small,
                                                                      const T* __restrict__ wgt,
                                                                      const T* __restrict__ bias,
                                                                      const T* __restrict__ add_even,
                                                                      T* __restrict__ big, DwS2Geom g) {
  using Acc = typename Elem<T>::Acc;
  using B = S2Block<K>;
  constexpr int R = B::R;
  constexpr int K3 = K * K * K;
  __shared__ Acc wsm[S2Weights<T, K>::kReg ? 1 : K3];
  const int QD = (g.Db + 1) >> 1, QH = (g.Hb + 1) >> 1, QW = (g.Wb + 1) >> 1;
  const int qd = (int)(blockIdx.x % (unsigned)QD);
  const int nc = (int)(blockIdx.x / (unsigned)QD);
  const int c = nc % g.C;
  S2Weights<T, K> w;
  w.load(wgt + (size_t)c * K3, wsm);
  const Acc b0 = bias != nullptr ? to_acc<T>(bias[c]) : Acc(0);
  const T* src = small + (size_t)nc * ((size_t)g.Ds * g.Hs * g.Ws);
  T* bvol = big + (size_t)nc * (size_t)g.bp;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int qh = warp; qh < QH; qh += kS2Warps) {
    for (int qw = lane; qw < QW; qw += 32) {
      Acc sv[R][R][R];
#pragma unroll
      for (int ad = 0; ad < R; ++ad) {
        const int md = qd + B::lo + ad;
        const bool dok = md >= 0 && md < g.Ds;
        const int mdc = min(max(md, 0), g.Ds - 1);
#pragma unroll
        for (int ah = 0; ah < R; ++ah) {
          const int mh = qh + B::lo + ah;
          const bool ok = dok && mh >= 0 && mh < g.Hs;
          const int mhc = min(max(mh, 0), g.Hs - 1);
          const T* row = src + ((size_t)mdc * g.Hs + mhc) * g.Ws;
#pragma unroll
          for (int aw = 0; aw < R; ++aw) {
            const Acc v = s2_ld<T>(row, qw + B::lo + aw, g.Ws);
            sv[ad][ah][aw] = ok ? v : Acc(0);
          }
        }
      }
#pragma unroll
      for (int ed = 0; ed < 2; ++ed) {
        const int id = 2 * qd + ed;
#pragma unroll
        for (int eh = 0; eh < 2; ++eh) {
          const int ih = 2 * qh + eh;
          T* row = bvol + ((size_t)id * g.Hb + ih) * g.bw;
#pragma unroll
          for (int ew = 0; ew < 2; ++ew) {
            Acc acc = b0;
#pragma unroll
            for (int ad = 0; ad < R; ++ad) {
              const int td = B::tap(ed, ad);
              if (td < 0) continue;
#pragma unroll
              for (int ah = 0; ah < R; ++ah) {
                const int th = B::tap(eh, ah);
                if (th < 0) continue;
#pragma unroll
                for (int aw = 0; aw < R; ++aw) {
                  const int tw = B::tap(ew, aw);
                  if (tw < 0) continue;
                  acc = fma(sv[ad][ah][aw], w[(td * K + th) * K + tw], acc);
                }
              }
            }
            const int iw = 2 * qw + ew;
            if constexpr (ADD) {
              if (ed == 0 && eh == 0 && ew == 0)
                acc += to_acc<T>(add_even[(((size_t)nc * g.Ds + qd) * g.Hs + qh) * g.Ws + qw]);
            }
            if (id < g.Db && ih < g.Hb && iw < g.Wb) row[iw] = from_acc<T>(acc);
          }
        }
      }
    }
  }
  // pad columns [Wb, bw) of the CTA's rows: zeros
  if (g.bw > g.Wb) {
    const int pad = g.bw - g.Wb;
    for (int ed = 0; ed < 2; ++ed) {
      const int id = 2 * qd + ed;
      if (id >= g.Db) break;
      for (int e = threadIdx.x; e < g.Hb * pad; e += blockDim.x)
        bvol[((size_t)id * g.Hb + e / pad) * g.bw + g.Wb + e % pad] = from_acc<T>(Acc(0));
    }
  }
}

// Stride-2 expansion of a small grid onto the big grid of the up block:
// big[2m] = small[m] at the all-even positions, bias[c] (0 without bias) at the
// others, zeros in the pad columns [Wb, bw) of each row.  This is the layout of a ConvTranspose3d with a
// 1x1x1 kernel and stride 2 once its per-voxel product (small, bias included) is
// done.  CTA = (n, c, id) big-grid plane; warps take rows, lanes run along W.
template <typename T>
__global__ void __launch_bounds__(kS2Warps * 32) upsample2_fill_kernel(const T* __restrict__ small,
                                                                       const float* __restrict__ bias,
                                                                       T* __restrict__ big, DwS2Geom g) {
  const int id = (int)(blockIdx.x % (unsigned)g.Db);
  const int nc = (int)(blockIdx.x / (unsigned)g.Db);
  const T fill = from_acc<T>(bias != nullptr ? bias[nc % g.C] : 0.0f);
  const T* src = small + ((size_t)nc * g.Ds + (id >> 1)) * ((size_t)g.Hs * g.Ws);
  T* dst = big + (size_t)nc * (size_t)g.bp + (size_t)id * g.Hb * g.bw;
  const T zero = from_acc<T>(0.0f);
  if constexpr (sizeof(T) == 2) {
    // the up block's row-pitched grid (bw = 2 Ws, Ws a multiple of 4): one 16-byte
    // chunk of 8 big columns per thread; on an all-even row its even columns are
    // small[4j .. 4j+3] (one 8-byte load), every other element is the fill, and
    // the pad column gets zero
    if (g.bw == 2 * g.Ws && g.Ws % 4 == 0 && (reinterpret_cast<uintptr_t>(big) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(small) & 7) == 0) {
      const uint32_t f = (uint32_t)reinterpret_cast<const unsigned short&>(fill);
      const int cpr = g.bw / 8;
      for (int q = threadIdx.x; q < g.Hb * cpr; q += blockDim.x) {
        const int ih = q / cpr, j = q - ih * cpr;
        uint32_t o[4] = {f | (f << 16), f | (f << 16), f | (f << 16), f | (f << 16)};
        if (((id | ih) & 1) == 0) {
          const uint2 sv = __ldg(reinterpret_cast<const uint2*>(src + (size_t)(ih >> 1) * g.Ws + 4 * j));
          o[0] = (sv.x & 0xffffu) | (f << 16);
          o[1] = (sv.x >> 16) | (f << 16);
          o[2] = (sv.y & 0xffffu) | (f << 16);
          o[3] = (sv.y >> 16) | (f << 16);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (8 * j + e >= g.Wb) o[e >> 1] &= (e & 1) ? 0x0000ffffu : 0xffff0000u;
        reinterpret_cast<uint4*>(dst + (size_t)ih * g.bw)[j] = make_uint4(o[0], o[1], o[2], o[3]);
      }
      return;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int ih = warp; ih < g.Hb; ih += kS2Warps) {
    const bool even_row = ((id | ih) & 1) == 0;
    const T* srow = src + (size_t)(ih >> 1) * g.Ws;
    for (int iw = lane; iw < g.bw; iw += 32)
      dst[(size_t)ih * g.bw + iw] = iw >= g.Wb ? zero : (even_row && (iw & 1) == 0) ? srow[iw >> 1] : fill;
  }
}

// F.pad(v, (1, 0, 1, 0, 1, 0)) of the pitched grid v (Db, Hb, Wb), plus an
// optional addend of the padded shape (Db+1, Hb+1, Wb+1), in one pass:
//   out[nc, z, y, x] = (z, y, x > 0 ? v[nc, z-1, y-1, x-1] : 0) + addend[nc, z, y, x]
// with the sum rounded once, as torch's add of the two tensors does.  The up
// block's output (models/blocks.py:177-181) and the decoder's skip add
// (models/mednext_v1.py:205).  CTA = (n, c, output plane); warps take rows,
// lanes run along W.
template <typename T>
__global__ void __launch_bounds__(kS2Warps * 32) pad_front_add_kernel(const T* __restrict__ v,
                                                                      const T* __restrict__ addend,
                                                                      T* __restrict__ out, DwS2Geom g) {
  using Acc = typename Elem<T>::Acc;
  constexpr int E = 16 / (int)sizeof(T);  // elements per 16-byte chunk
  const int Dp = g.Db + 1, Hp = g.Hb + 1, Wp = g.Wb + 1;
  const int z = (int)(blockIdx.x % (unsigned)Dp);
  const int nc = (int)(blockIdx.x / (unsigned)Dp);
  const size_t plane = ((size_t)nc * Dp + z) * ((size_t)Hp * Wp);
  T* dst = out + plane;
  const T* add = addend != nullptr ? addend + plane : nullptr;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // padded rows of whole 16-byte chunks: one chunk of the output (and addend) per
  // lane step; the source row is shifted by one element, so it is read per element
  const bool vec = sizeof(T) <= 4 && Wp % E == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
                   (add == nullptr || (reinterpret_cast<uintptr_t>(addend) & 15) == 0);
  if (vec) {
    // the plane's 16-byte output chunks are spread over all the CTA's threads
    const int cpr = Wp / E;  // chunks per row
    for (int q = threadIdx.x; q < Hp * cpr; q += blockDim.x) {
      const int y = q / cpr, x0 = (q - y * cpr) * E;
      Acc a[E];
      if (add != nullptr) {
        unpack16<T>(*reinterpret_cast<const uint4*>(add + (size_t)y * Wp + x0), a);
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) a[e] = Acc(0);
      }
      if (z > 0 && y > 0) {
        const T* srow = v + (size_t)nc * (size_t)g.bp + ((size_t)(z - 1) * g.Hb + (y - 1)) * g.bw;
#pragma unroll
        for (int e = 0; e < E; ++e)
          if (x0 + e > 0) a[e] += to_acc<T>(srow[x0 + e - 1]);
      }
      *reinterpret_cast<uint4*>(dst + (size_t)y * Wp + x0) = pack16<T>(a);
    }
    return;
  }
  for (int y = warp; y < Hp; y += kS2Warps) {
    const bool row_in = z > 0 && y > 0;
    const T* srow = row_in ? v + (size_t)nc * (size_t)g.bp + ((size_t)(z - 1) * g.Hb + (y - 1)) * g.bw : nullptr;
    for (int x = lane; x < Wp; x += 32) {
      Acc a = (row_in && x > 0) ? to_acc<T>(srow[x - 1]) : Acc(0);
      if (add != nullptr) a += to_acc<T>(add[(size_t)y * Wp + x]);
      dst[(size_t)y * Wp + x] = from_acc<T>(a);
    }
  }
}

// The inverse: the interior (z, y, x >= 1) of a left-padded (Db+1, Hb+1, Wb+1)
// volume into the row-pitched grid, with zeros in the pad columns [Wb, bw).  The
// up block's output grad, repacked for its GEMMs.  CTA = (n, c, interior plane).
// When the padded rows are 16-byte chunks and bw = Wb + 1 (the up block's
// layout: a grid row and a padded row have the same length), output chunk j of a
// row is padded chunk j shifted left by one element, its last element taken from
// padded chunk j + 1 (or zero for the row's last chunk, the pad column): 16-byte
// loads and stores.
template <typename T>
__global__ void __launch_bounds__(kS2Warps * 32) unpad_front_kernel(const T* __restrict__ padded,
                                                                    T* __restrict__ v, DwS2Geom g) {
  const int Hp = g.Hb + 1, Wp = g.Wb + 1;
  const int z = (int)(blockIdx.x % (unsigned)g.Db);
  const int nc = (int)(blockIdx.x / (unsigned)g.Db);
  // padded row y+1 of plane z+1; output element x is its element x+1
  const T* src = padded + ((size_t)nc * (g.Db + 1) + (z + 1)) * ((size_t)Hp * Wp) + Wp;
  T* dst = v + (size_t)nc * (size_t)g.bp + (size_t)z * g.Hb * g.bw;
  constexpr int E = 16 / (int)sizeof(T);
  if constexpr (sizeof(T) == 2) {
    if (g.bw == Wp && Wp % E == 0 && (reinterpret_cast<uintptr_t>(padded) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(v) & 15) == 0) {
      const int cpr = Wp / E;
      for (int q = threadIdx.x; q < g.Hb * cpr; q += blockDim.x) {
        const int y = q / cpr, j = q - y * cpr;
        const T* srow = src + (size_t)y * Wp;
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(srow) + j);
        const uint32_t nx = j + 1 < cpr ? (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(srow) + (j + 1) * E) : 0u;
        uint4 o;
        o.x = __funnelshift_r(a.x, a.y, 16);
        o.y = __funnelshift_r(a.y, a.z, 16);
        o.z = __funnelshift_r(a.z, a.w, 16);
        o.w = __funnelshift_r(a.w, nx, 16);
        reinterpret_cast<uint4*>(dst + (size_t)y * g.bw)[j] = o;
      }
      return;
    }
  }
  const T zero = from_acc<T>(0.0f);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // lanes on consecutive elements: both the (shifted) reads and the writes coalesce
  for (int y = warp; y < g.Hb; y += kS2Warps)
    for (int x = lane; x < g.bw; x += 32) dst[(size_t)y * g.bw + x] = x < g.Wb ? src[(size_t)y * Wp + x + 1] : zero;
}

// wgrad: the CTA's threads form K groups (group g owns the K*K taps with kd = g,
// and its warps take the small-grid rows in turn).  A CTA covers `chunk`
// consecutive small-grid planes of one (sample, channel); with `small_bias` it
// also sums the small grid (the down block's bias grad).
// Partials: part[(nc*chunks + j)*(K^3+1) + tap].
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
  const int G = blockDim.x / K;  // threads per group, a multiple of 32
  const int grp = threadIdx.x / G;
  const int lt = threadIdx.x - grp * G;
  const int gwarp = lt >> 5, gwarps = G >> 5;
  const int lane = threadIdx.x & 31;
  const int j = (int)(blockIdx.x % (unsigned)chunks);
  const int nc = (int)(blockIdx.x / (unsigned)chunks);
  const size_t splane = (size_t)g.Hs * g.Ws;
  const T* bsrc = big + (size_t)nc * (size_t)g.bp;
  const T* ssrc = small + (size_t)nc * g.Ds * splane;
  const int md0 = j * chunk;
  const int md1 = min(md0 + chunk, g.Ds);
  Acc acc[K2 + 1];
#pragma unroll
  for (int t = 0; t <= K2; ++t) acc[t] = Acc(0);
  const int kd = grp;
  for (int md = md0; md < md1; ++md) {
    const int id = 2 * md - P + kd;
    const bool dok = id >= 0 && id < g.Db;
    const int idc = min(max(id, 0), g.Db - 1);
    for (int mh = gwarp; mh < g.Hs; mh += gwarps) {
      const T* srow = ssrc + (size_t)md * splane + (size_t)mh * g.Ws;
      for (int mw = lane; mw < g.Ws; mw += 32) {
        const Acc sv = to_acc<T>(__ldg(srow + mw));
        acc[K2] += sv;
        const Acc svd = dok ? sv : Acc(0);
#pragma unroll
        for (int kh = 0; kh < K; ++kh) {
          const int ih = 2 * mh - P + kh;
          const Acc svh = (ih >= 0 && ih < g.Hb) ? svd : Acc(0);
          const T* row = bsrc + ((size_t)idc * g.Hb + min(max(ih, 0), g.Hb - 1)) * g.bw;
#pragma unroll
          for (int kw = 0; kw < K; ++kw)
            acc[kh * K + kw] = fma(s2_ld<T>(row, 2 * mw - P + kw, g.Wb), svh, acc[kh * K + kw]);
        }
      }
    }
  }
  // reduce within each group (G is a multiple of 32)
  __shared__ Acc red[14 * (K2 + 1)];
  const int warp = threadIdx.x >> 5;
#pragma unroll
  for (int t = 0; t <= K2; ++t) {
    Acc s = acc[t];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp * (K2 + 1) + t] = s;
  }
  __syncthreads();
  Acc* dst = part + ((size_t)nc * chunks + j) * (K3 + 1);
  for (int e = threadIdx.x; e < K * (K2 + 1); e += blockDim.x) {
    const int gg = e / (K2 + 1);
    const int t = e - gg * (K2 + 1);
    Acc s = Acc(0);
    for (int w = 0; w < gwarps; ++w) s += red[(gg * gwarps + w) * (K2 + 1) + t];
    if (t < K2) dst[gg * K2 + t] = s;
    else if (gg == 0) dst[K3] = small_bias ? s : Acc(0);
  }
}

// Per-(sample, channel, chunk) sums of a tensor into slot K^3 of the wgrad
// partials (bias grad of the up block, whose dy is the big grid).  Volumes start
// every `pitch` elements and hold `vol` elements in rows of `row_pitch`, of which
// the first `row_len` are summed (row_len = row_pitch: all).  With a 16-byte
// aligned base, pitch and row pitch the chunks are read as 16-byte vectors.
template <typename T>
__global__ void __launch_bounds__(256) chan_sum_into_partials_kernel(
    const T* __restrict__ src, typename Elem<T>::Acc* __restrict__ part, size_t vol, size_t pitch, int chunks,
    int K3, int row_pitch, int row_len) {
  using Acc = typename Elem<T>::Acc;
  constexpr int E = 16 / (int)sizeof(T);
  const int j = (int)(blockIdx.x % (unsigned)chunks);
  const size_t nc = blockIdx.x / (unsigned)chunks;
  const T* p = src + nc * pitch;
  const bool masked = row_len < row_pitch;
  const bool vec = (reinterpret_cast<uintptr_t>(src) % 16 == 0) && (pitch % E == 0) && (row_pitch % E == 0);
  // chunk bounds on whole 16-byte vectors
  const size_t per = ((vol + chunks - 1) / chunks + E - 1) / E * E;
  const size_t beg = min((size_t)j * per, vol);
  const size_t end = min(beg + per, vol);
  Acc s = Acc(0);
  if (vec) {
    const size_t nv = (end - beg) / E;
    const uint4* pv = reinterpret_cast<const uint4*>(p + beg);
    for (size_t i = threadIdx.x; i < nv; i += blockDim.x) {
      Acc v[E];
      unpack16<T>(__ldg(pv + i), v);
      const int col = masked ? (int)((beg + i * E) % (size_t)row_pitch) : 0;
#pragma unroll
      for (int e = 0; e < E; ++e) s += (!masked || col + e < row_len) ? v[e] : Acc(0);
    }
    for (size_t i = beg + nv * E + threadIdx.x; i < end; i += blockDim.x)
      if (!masked || (int)(i % (size_t)row_pitch) < row_len) s += to_acc<T>(__ldg(p + i));
  } else {
    for (size_t i = beg + threadIdx.x; i < end; i += blockDim.x)
      if (!masked || (int)(i % (size_t)row_pitch) < row_len) s += to_acc<T>(__ldg(p + i));
  }
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
