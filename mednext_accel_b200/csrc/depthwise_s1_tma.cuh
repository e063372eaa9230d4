// Depthwise Conv3d, stride 1, padding k/2, with the input planes streamed by
// TMA through a shared-memory ring (sm_100a).
//
// Same work decomposition and per-plane arithmetic as depthwise_s1.cuh (a CTA
// owns one (sample, channel) TW x TH tile and a chunk of TD depth planes; each
// thread keeps a register ring of k partial output planes), but the plane tiles
// are not loaded by the compute threads between two CTA barriers.  One
// producer warp issues 4-D TMA tile loads (W, H, D, N*C) of the halo'd plane
// tiles into a ring of kDwSlots buffers; out-of-range rows, columns and planes
// arrive as zeros (TMA out-of-bounds fill), which is the convolution's zero
// padding.  Compute warps wait on the slot's mbarrier and release it per warp,
// so loads run ahead of the arithmetic and no CTA-wide barrier sits in the loop.
// All waits are bounded and warp-uniform (a warp leaves its loop as a whole);
// after an abort the producer waits for the fills it issued before the CTA exits.
#pragma once

#include <type_traits>

#include "depthwise_s1.cuh"

namespace mednext {

constexpr int kDwSlots = 4;            // plane ring depth
constexpr int kDwMaxComputeWarps = 8;  // 256 compute threads at most (+1 producer warp)

struct DwRing {
  uint64_t full[kDwSlots];
  uint64_t empty[kDwSlots];
  int abort;
};

// Shared-memory layout, from the first 128-byte boundary of the dynamic region
// (TMA destinations are 128-byte aligned): [K^3 weights as Acc, padded to 128 B]
// [kDwSlots slots].
// A slot holds the halo'd x plane tile (rows x rsw) and, for the weight grad,
// the dy plane tile (TH x TW) at the next 128-byte boundary: every TMA
// destination starts 128-byte aligned.
template <typename T>
struct DwTmaLayout {
  static __host__ __device__ size_t align128(size_t b) { return (b + 127) / 128 * 128; }
  static __host__ __device__ size_t weights(int K, size_t acc) { return align128((size_t)K * K * K * acc); }
  static __host__ __device__ size_t x_tile(const DwS1Geom& g, int K) {
    return (size_t)(g.TH + 2 * (K / 2)) * DwTile<T>::row_elems(g.TW, K / 2) * sizeof(T);
  }
  static __host__ __device__ size_t dy_tile(const DwS1Geom& g) { return (size_t)g.TH * g.TW * sizeof(T); }
  static __host__ __device__ size_t dy_offset(const DwS1Geom& g, int K) { return align128(x_tile(g, K)); }
  static __host__ __device__ size_t slot(const DwS1Geom& g, int K, bool with_dy) {
    return with_dy ? align128(dy_offset(g, K) + dy_tile(g)) : align128(x_tile(g, K));
  }
};

__device__ __forceinline__ void dw_ring_drain(DwRing& ring, int issued) {
  for (int q = issued > kDwSlots ? issued - kDwSlots : 0; q < issued; ++q)
    mbar_wait(&ring.full[q % kDwSlots], (uint32_t)((q / kDwSlots) & 1));
}

// ----------------------------------------------------------------------------
// Forward (flip = 0) and input grad (flip = 1).
// ----------------------------------------------------------------------------
template <typename T, int K, int NH>
__global__ void __launch_bounds__(kDwMaxComputeWarps * 32 + 32, 1)
    dw_s1_conv_tma_kernel(const __grid_constant__ CUtensorMap mX, const T* __restrict__ wgt,
                          const T* __restrict__ bias, const T* __restrict__ addend, T* __restrict__ y,
                          GnPartial* __restrict__ stats, DwS1Geom g, int flip) {
  using Acc = typename Elem<T>::Acc;
  using L = DwTmaLayout<T>;
  constexpr int P = K / 2;
  constexpr int K3 = K * K * K;
  constexpr int OFF = DwTile<T>::off(P);
  constexpr bool kWReg = (K <= 3);
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ DwRing ring;
  unsigned char* base = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  Acc* sw = reinterpret_cast<Acc*>(base);
  const size_t slot_bytes = L::slot(g, K, false);
  unsigned char* slots = base + L::weights(K, sizeof(Acc));
  const int compute_threads = (int)blockDim.x - 32;
  const bool producer = (int)threadIdx.x >= compute_threads;

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
  const int dcount = min(g.TD, g.D - d0);
  const int nsteps = dcount + K - 1;

  for (int t = threadIdx.x; t < K3; t += blockDim.x) {
    const int src = flip ? (K3 - 1 - t) : t;
    sw[t] = to_acc<T>(wgt[(size_t)c * K3 + src]);
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < kDwSlots; ++i) {
      mbar_init(&ring.full[i], 1);
      mbar_init(&ring.empty[i], (uint32_t)(compute_threads / 32));
    }
    ring.abort = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  volatile int* abort = &ring.abort;
  int issued = 0;

  // shifted running sums for GroupNorm statistics
  Acc st_n = Acc(0), st_shift = Acc(0), st_s1 = Acc(0), st_s2 = Acc(0);

  if (producer) {
    if ((threadIdx.x & 31) == 0) {
      tma_prefetch_map(&mX);
      const uint32_t bytes = (uint32_t)L::x_tile(g, K);
      for (int s = 0; s < nsteps && !*abort; ++s) {
        const int slot = s % kDwSlots, r = s / kDwSlots;
        if (r > 0 && !mbar_wait(&ring.empty[slot], (uint32_t)((r - 1) & 1))) {
          *abort = 1;
          break;
        }
        mbar_arrive_expect_tx(&ring.full[slot], bytes);
        tma_load_4d(slots + (size_t)slot * slot_bytes, &mX, &ring.full[slot], w0 - OFF, h0 - P, d0 - P + s, nc);
        ++issued;
      }
    }
  } else {
    const int lane = threadIdx.x & 31;
    const int wt = threadIdx.x % g.LW;
    const int tr = threadIdx.x / g.LW;
    const int hrow = tr * NH;  // first output row of this thread, relative to h0
    const bool active = tr < g.TR;
    Acc wr[kWReg ? K3 : 1];
    if constexpr (kWReg) {
#pragma unroll
      for (int t = 0; t < K3; ++t) wr[t] = sw[t];
    }
    const Acc bv = bias != nullptr ? to_acc<T>(bias[c]) : Acc(0);
    const size_t vol_elems = (size_t)g.D * g.H * g.W;
    T* yv = y + (size_t)nc * vol_elems;
    Acc acc[K][NH][kDwNW];
#pragma unroll
    for (int a = 0; a < K; ++a)
#pragma unroll
      for (int jh = 0; jh < NH; ++jh)
#pragma unroll
        for (int i = 0; i < kDwNW; ++i) acc[a][jh][i] = Acc(0);
    const int ow0 = w0 + kDwNW * wt;
    const bool vec_store = g.vec && (ow0 + kDwNW <= g.W);

    bool stop = false;  // warp-uniform: every lane leaves the loop at the same step
    for (int sb = 0; sb < nsteps && !stop; sb += K) {
#pragma unroll
      for (int j = 0; j < K; ++j) {
        const int s = sb + j;
        if (s < nsteps) {
          const int slot = s % kDwSlots;
          const bool ok = !*abort && mbar_wait(&ring.full[slot], (uint32_t)((s / kDwSlots) & 1));
          if (!__all_sync(0xffffffffu, ok)) {
            *abort = 1;
            stop = true;
            break;
          }
          const T* sp = reinterpret_cast<const T*>(slots + (size_t)slot * slot_bytes);
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
                  const int slotk = (j - kd + K) % K;
#pragma unroll
                  for (int kw = 0; kw < K; ++kw) {
                    const int ti = (kd * K + kh) * K + kw;
                    const Acc wv = kWReg ? wr[kWReg ? ti : 0] : sw[ti];
#pragma unroll
                    for (int i = 0; i < kDwNW; ++i) acc[slotk][jh][i] = fma(win[i + kw], wv, acc[slotk][jh][i]);
                  }
                }
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&ring.empty[slot]);
          // output plane s-(K-1) is complete; its slot is (j+1) % K
          const int o = s - (K - 1);
          if (active && o >= 0) {
            const int oslot = (j + 1) % K;
            const int od = d0 + o;
#pragma unroll
            for (int jh = 0; jh < NH; ++jh) {
              const int oh = h0 + hrow + jh;
              if (oh >= g.H) continue;
              Acc v[kDwNW];
#pragma unroll
              for (int i = 0; i < kDwNW; ++i) v[i] = acc[oslot][jh][i] + bv;
              const size_t row_off = ((size_t)od * g.H + oh) * g.W + ow0;
              if (addend != nullptr) {
                Acc av[kDwNW];
                dw_load_dy_patch<T>(addend + (size_t)nc * vol_elems + (size_t)od * g.H * g.W, oh, ow0, g, vec_store,
                                    av);
#pragma unroll
                for (int i = 0; i < kDwNW; ++i) v[i] += av[i];
              }
              T* dst = yv + row_off;
              if (vec_store) {
                constexpr int E = DwTile<T>::E;
#pragma unroll
                for (int q = 0; q < kDwNW / E; ++q) reinterpret_cast<uint4*>(dst)[q] = pack16<T>(v + q * E);
              } else {
#pragma unroll
                for (int i = 0; i < kDwNW; ++i)
                  if (ow0 + i < g.W) dst[i] = from_acc<T>(v[i]);
              }
              if (stats != nullptr) {
#pragma unroll
                for (int i = 0; i < kDwNW; ++i) {
                  if (ow0 + i < g.W) {
                    const Acc rv = to_acc<T>(from_acc<T>(v[i]));  // statistics of the stored value
                    if (st_n == Acc(0)) st_shift = rv;
                    const Acc dlt = rv - st_shift;
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
  }

  __syncthreads();
  if (*abort && producer && (threadIdx.x & 31) == 0) dw_ring_drain(ring, issued);
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
  if (*abort && threadIdx.x == 0) raise_device_error(kErrMbarTimeout);
}

// ----------------------------------------------------------------------------
// Forward (flip = 0) and input grad (flip = 1) for k = 3 on 16-bit types with
// the packed fp32 FMA of sm_100 (fma.rn.f32x2).  Same CTA tile and plane ring
// as dw_s1_conv_tma_kernel; each thread owns one output row of kDwPkCols = 16
// columns and holds its accumulators as column pairs (i, i + 8), so one packed
// FMA applies a tap to two outputs and the FMA instruction count halves.  Every
// output sums its taps in (kd, kh, kw) order from zero and adds the bias last,
// the order of dw_s1_conv_tma_kernel, so the two kernels give the same bits.
// Pairs are 64-bit values end to end (window, weights, accumulators), so the
// bf16 -> fp32 conversions write straight into the pair halves.  STATS
// (GroupNorm partial statistics of the stored output) and ADD (an addend
// tensor) are compile-time switches.
//
// No producer warp: thread 0 issues the first kDwSlots plane loads, and the
// warp that releases a slot last (a counter per slot) issues the slot's next
// load, so no thread polls for free slots.  Every warp computes; two CTAs of
// 8 warps fit an SM at up to 128 registers.
//
// Shared-memory reads are free of bank conflicts: the plane tile's rows are
// pitched to an odd number of 16-byte units (kDwPkPad extra columns in the TMA
// box), a quarter warp covers 4 threads x 2 rows, so the 8 lanes of every
// 16-byte load hit 8 different bank groups, and the two halo columns of a
// thread come from its neighbours by shuffle (tile edges from one broadcast
// load per row).
// ----------------------------------------------------------------------------
constexpr int kDwPkCols = 16;
constexpr int kDwPkPad = 8;
constexpr int kDwPkThreads = 256;  // 8 warps: 32 rows of a 128-wide tile

template <typename T>
struct DwPkLayout {
  static __host__ __device__ int pitch(int TW) { return DwTile<T>::row_elems(TW, 1) + kDwPkPad; }
  static __host__ __device__ size_t x_tile(const DwS1Geom& g) { return (size_t)(g.TH + 2) * pitch(g.TW) * sizeof(T); }
  static __host__ __device__ size_t slot(const DwS1Geom& g) { return DwTmaLayout<T>::align128(x_tile(g)); }
  static __host__ __device__ size_t weights() { return DwTmaLayout<T>::align128(27 * sizeof(uint64_t)); }
  static __host__ size_t smem(const DwS1Geom& g) { return 128 + weights() + kDwSlots * slot(g); }
};

struct DwPkRing {
  uint64_t full[kDwSlots];
  int released[kDwSlots];  // warp releases of the slot so far (nwarps per plane)
  int issued;              // plane loads issued so far
  int abort;
};

// fp32 bit patterns of the low / high 16-bit element of a packed word
template <typename T>
__device__ __forceinline__ uint32_t lo_bits(uint32_t w);
template <typename T>
__device__ __forceinline__ uint32_t hi_bits(uint32_t w);
template <>
__device__ __forceinline__ uint32_t lo_bits<__nv_bfloat16>(uint32_t w) {
  return w << 16;
}
template <>
__device__ __forceinline__ uint32_t hi_bits<__nv_bfloat16>(uint32_t w) {
  return w & 0xffff0000u;
}
template <>
__device__ __forceinline__ uint32_t lo_bits<__half>(uint32_t w) {
  return __float_as_uint(__half2float(__ushort_as_half((unsigned short)(w & 0xffffu))));
}
template <>
__device__ __forceinline__ uint32_t hi_bits<__half>(uint32_t w) {
  return __float_as_uint(__half2float(__ushort_as_half((unsigned short)(w >> 16))));
}

__device__ __forceinline__ uint64_t pk_pair(uint32_t lo, uint32_t hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo), "r"(hi));
  return d;
}
__device__ __forceinline__ void pk_split(uint64_t v, float& lo, float& hi) {
  uint32_t a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=r"(a), "=r"(b) : "l"(v));
  lo = __uint_as_float(a);
  hi = __uint_as_float(b);
}
// d = a * b + c on both fp32 halves, round to nearest even
__device__ __forceinline__ uint64_t pk_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// a + b on both fp32 halves, round to nearest even
__device__ __forceinline__ uint64_t pk_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// lane of the thread that owns (column group wt, tile row r) in its warp
__device__ __forceinline__ int dw_pk_lane(int wt, int r, int lw2) {
  return lw2 == 8 ? ((wt & 3) | ((wt & 4) << 1) | ((r & 1) << 2) | ((r & 2) << 3)) : ((r * lw2 + wt) & 31);
}

// p[m] = (x[m-1], x[m+7]) for the 18 inputs x[-1..16] around the thread's 16
// output columns.  rowp is the shared-memory row, col the thread's first column
// in it; x[-1] and x[16] come from the neighbouring lanes src_l / src_r, or from
// the row's halo columns at the tile edges.  Every lane of the warp takes part.
template <typename T>
__device__ __forceinline__ void dw_pk_window(const T* __restrict__ rowp, int col, int tw, bool left_edge,
                                             bool right_edge, int src_l, int src_r, uint64_t (&p)[10]) {
  constexpr int OFF = DwTile<T>::off(1);
  const uint4 c0 = *reinterpret_cast<const uint4*>(rowp + col);
  const uint4 c1 = *reinterpret_cast<const uint4*>(rowp + col + 8);
  const uint32_t from_l = __shfl_sync(0xffffffffu, c1.w, src_l);  // (x[14], x[15]) of the left neighbour
  const uint32_t from_r = __shfl_sync(0xffffffffu, c0.x, src_r);  // (x[0], x[1]) of the right neighbour
  const unsigned short* row16 = reinterpret_cast<const unsigned short*>(rowp);
  const uint32_t el = row16[OFF - 1], er = row16[OFF + tw];
  const uint32_t xl = left_edge ? el : (from_l >> 16);
  const uint32_t xr = right_edge ? er : (from_r & 0xffffu);
  const uint32_t a[4] = {c0.x, c0.y, c0.z, c0.w};  // x[0..7]
  const uint32_t b[4] = {c1.x, c1.y, c1.z, c1.w};  // x[8..15]
  p[0] = pk_pair(lo_bits<T>(xl), hi_bits<T>(a[3]));
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    p[2 * q + 1] = pk_pair(lo_bits<T>(a[q]), lo_bits<T>(b[q]));  // (x[2q], x[2q+8])
    p[2 * q + 2] = pk_pair(hi_bits<T>(a[q]), hi_bits<T>(b[q]));  // (x[2q+1], x[2q+9])
  }
  p[9] = pk_pair(lo_bits<T>(b[0]), lo_bits<T>(xr));
}

template <typename T, bool STATS, bool ADD>
__global__ void __launch_bounds__(kDwPkThreads, 2)
    dw_s1_conv_pk_kernel(const __grid_constant__ CUtensorMap mX, const T* __restrict__ wgt,
                         const T* __restrict__ bias, const T* __restrict__ addend, T* __restrict__ y,
                         GnPartial* __restrict__ stats, DwS1Geom g, int flip) {
  constexpr int K = 3;
  constexpr int K3 = 27;
  using L = DwPkLayout<T>;
  constexpr int OFF = DwTile<T>::off(1);
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ DwPkRing ring;
  unsigned char* base = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  uint64_t* sw = reinterpret_cast<uint64_t*>(base);
  const size_t slot_bytes = L::slot(g);
  unsigned char* slots = base + L::weights();
  const int nwarps = (int)blockDim.x >> 5;

  int b = blockIdx.x;
  const int tw = b % g.tilesW;
  b /= g.tilesW;
  const int th = b % g.tilesH;
  b /= g.tilesH;
  const int td = b % g.tilesD;
  const int nc = b / g.tilesD;
  const int c = nc % g.C;
  const int w0 = tw * g.TW, h0 = th * g.TH, d0 = td * g.TD;
  const int rsp = L::pitch(g.TW);
  const int dcount = min(g.TD, g.D - d0);
  const int nsteps = dcount + K - 1;
  const uint32_t tile_bytes = (uint32_t)L::x_tile(g);

  for (int t = threadIdx.x; t < K3; t += blockDim.x) {
    const uint32_t wv = __float_as_uint(to_acc<T>(wgt[(size_t)c * K3 + (flip ? K3 - 1 - t : t)]));
    sw[t] = pk_pair(wv, wv);
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < kDwSlots; ++i) {
      mbar_init(&ring.full[i], 1);
      ring.released[i] = 0;
    }
    ring.abort = 0;
    fence_mbarrier_init();
    tma_prefetch_map(&mX);
    const int first = min(nsteps, kDwSlots);
    for (int q = 0; q < first; ++q) {
      mbar_arrive_expect_tx(&ring.full[q], tile_bytes);
      tma_load_4d(slots + (size_t)q * slot_bytes, &mX, &ring.full[q], w0 - OFF, h0 - 1, d0 - 1 + q, nc);
    }
    ring.issued = first;
  }
  __syncthreads();
  volatile int* abort = &ring.abort;

  // shifted running sums for GroupNorm statistics, column pairs
  float st_n = 0.f, st_shift = 0.f;
  float2 st_s1 = make_float2(0.f, 0.f), st_s2 = make_float2(0.f, 0.f);

  const int lane = threadIdx.x & 31;
  const int lw2 = g.LW >> 1;
  int wt, row;
  if (lw2 == 8) {
    wt = (lane & 3) | ((lane >> 1) & 4);
    row = ((threadIdx.x >> 5) << 2) | ((lane >> 2) & 1) | ((lane >> 3) & 2);
  } else {
    wt = threadIdx.x % lw2;
    row = threadIdx.x / lw2;
  }
  const bool active = row < g.TH;
  const int oh = h0 + row;
  const int ow0 = w0 + kDwPkCols * wt;
  // W is a multiple of 8 on this path: each half of the 16 columns is in or out as a whole
  const bool store_row = active && oh < g.H && ow0 < g.W;
  const bool hi_ok = ow0 + 8 < g.W;
  const int src_l = dw_pk_lane(wt > 0 ? wt - 1 : wt, row, lw2);
  const int src_r = dw_pk_lane(wt < lw2 - 1 ? wt + 1 : wt, row, lw2);
  const bool left_edge = wt == 0, right_edge = wt == lw2 - 1;
  const uint32_t bvb = __float_as_uint(bias != nullptr ? to_acc<T>(bias[c]) : 0.f);
  // output row of this thread in plane 0 of its (n, c) volume; planes are plane_elems apart
  const size_t plane_elems = (size_t)g.H * g.W;
  const size_t out0 = (size_t)nc * g.D * plane_elems + (size_t)oh * g.W + ow0;
  // rows of lanes past the tile read row 0 (every lane joins the shuffles) and store nothing
  const int rbase = (active ? row : 0) * rsp;
  const int col = OFF + kDwPkCols * wt;
  uint64_t acc[K][8];
#pragma unroll
  for (int a = 0; a < K; ++a)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[a][i] = 0ull;

  // one ring step: plane s of the input enters, output plane s - (K - 1) leaves;
  // j = s % K names the accumulator slot at compile time.  False after an abort.
  auto step = [&](auto jc, const int s) -> bool {
    constexpr int j = decltype(jc)::value;
    const int slot = s % kDwSlots;
    const bool ok = !*abort && mbar_wait(&ring.full[slot], (uint32_t)((s / kDwSlots) & 1));
    if (!__all_sync(0xffffffffu, ok)) {
      *abort = 1;
      return false;
    }
    const T* sp = reinterpret_cast<const T*>(slots + (size_t)slot * slot_bytes) + rbase;
    // output plane s starts here: its slot is j
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[j][i] = 0ull;
#pragma unroll
    for (int kh = 0; kh < K; ++kh) {
      uint64_t p[10];
      dw_pk_window<T>(sp + kh * rsp, col, g.TW, left_edge, right_edge, src_l, src_r, p);
#pragma unroll
      for (int kd = 0; kd < K; ++kd) {
        const int slotk = (j - kd + K) % K;
#pragma unroll
        for (int kw = 0; kw < K; ++kw) {
          const uint64_t wv = sw[(kd * K + kh) * K + kw];
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[slotk][i] = pk_fma(p[i + kw], wv, acc[slotk][i]);
        }
      }
    }
    // release the slot; the warp that releases it last loads the slot's next plane
    __syncwarp();
    if (lane == 0) {
      int prev;
      asm volatile("atom.acq_rel.cta.shared::cta.add.s32 %0, [%1], 1;"
                   : "=r"(prev)
                   : "r"(smem_u32(&ring.released[slot]))
                   : "memory");
      // the count only grows: the slot's (s / kDwSlots)-th plane is released by nwarps arrivals
      if (prev == (s / kDwSlots + 1) * nwarps - 1) {
        const int q = s + kDwSlots;
        if (q < nsteps) {
          fence_async_smem();
          mbar_arrive_expect_tx(&ring.full[slot], tile_bytes);
          tma_load_4d(slots + (size_t)slot * slot_bytes, &mX, &ring.full[slot], w0 - OFF, h0 - 1, d0 - 1 + q,
                      nc);
          atomicAdd(&ring.issued, 1);
        }
      }
    }
    // output plane s-(K-1) is complete; its slot is (j+1) % K
    const int o = s - (K - 1);
    if (store_row && o >= 0) {
      const int oslot = (j + 1) % K;
      const size_t off = out0 + (size_t)(d0 + o) * plane_elems;
      const uint64_t bv2 = pk_pair(bvb, bvb);
      float lo[8], hi[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) pk_split(pk_add(acc[oslot][i], bv2), lo[i], hi[i]);
      if constexpr (ADD) {
        float al[8], ah[8];
        const uint4* ap = reinterpret_cast<const uint4*>(addend + off);
        unpack16<T>(__ldg(ap), al);
        unpack16<T>(hi_ok ? __ldg(ap + 1) : make_uint4(0, 0, 0, 0), ah);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          lo[i] += al[i];
          hi[i] += ah[i];
        }
      }
      const uint4 qlo = pack16<T>(lo), qhi = pack16<T>(hi);
      uint4* dst = reinterpret_cast<uint4*>(y + off);
      dst[0] = qlo;
      if (hi_ok) dst[1] = qhi;
      if constexpr (STATS) {
        // statistics of the stored values
        float rl[8], rh[8];
        unpack16<T>(qlo, rl);
        unpack16<T>(qhi, rh);
        if (st_n == 0.f) st_shift = rl[0];
        const float2 sh = make_float2(-st_shift, -st_shift);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float2 dv = __fadd2_rn(make_float2(rl[i], hi_ok ? rh[i] : st_shift), sh);
          st_s1 = __fadd2_rn(st_s1, dv);
          st_s2 = __ffma2_rn(dv, dv, st_s2);
        }
        st_n += hi_ok ? 16.f : 8.f;
      }
    }
    return true;
  };
  using J0 = std::integral_constant<int, 0>;
  using J1 = std::integral_constant<int, 1>;
  using J2 = std::integral_constant<int, 2>;
  // whole rounds of K steps, then the remainder; every lane of a warp leaves together
  int sb = 0;
  bool ok = true;
  for (; ok && sb + K <= nsteps; sb += K) ok = step(J0{}, sb) && step(J1{}, sb + 1) && step(J2{}, sb + 2);
  if (ok && sb < nsteps) ok = step(J0{}, sb);
  if (ok && sb + 1 < nsteps) step(J1{}, sb + 1);

  __syncthreads();
  // after an abort, wait (bounded) for the loads still in flight before the CTA exits
  if (*abort && threadIdx.x == 0) {
    const int issued = ring.issued;
    for (int q = issued > kDwSlots ? issued - kDwSlots : 0; q < issued; ++q)
      mbar_wait(&ring.full[q % kDwSlots], (uint32_t)((q / kDwSlots) & 1));
  }
  if constexpr (STATS) {
    __shared__ double red[3 * 32];
    double n = (double)st_n, mean = 0.0, m2 = 0.0;
    if (st_n > 0.f) {
      const double s1 = (double)st_s1.x + (double)st_s1.y, s2 = (double)st_s2.x + (double)st_s2.y;
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
  if (*abort && threadIdx.x == 0) raise_device_error(kErrMbarTimeout);
}

// Raw 16-bit window of thread column wt for the mixed-precision weight grads:
// window element m (input column w0 + 8 wt - P + m, m < 8 + 2P) is 16-bit
// element m + kMixH0<P> of xw.  rowb is the shared-memory row, whose element 0
// is input column w0 - 8 (16-bit types, P <= 3: the left halo is one chunk).
template <int P>
constexpr int kMixWL = (P + 1) / 2;  // words left (and right) of the thread's 4 words
template <int P>
constexpr int kMixH0 = 2 * kMixWL<P> - P;
template <int P>
__device__ __forceinline__ void dw_read_window_raw(const void* rowb, int wt, uint32_t (&xw)[4 + 2 * kMixWL<P>]) {
  constexpr int WL = kMixWL<P>;
  const uint32_t* rowp = reinterpret_cast<const uint32_t*>(rowb) + 4 * wt;
  const uint4 mid = *reinterpret_cast<const uint4*>(rowp + 4);
#pragma unroll
  for (int q = 0; q < WL; ++q) {
    xw[q] = rowp[4 - WL + q];
    xw[WL + 4 + q] = rowp[8 + q];
  }
  xw[WL] = mid.x;
  xw[WL + 1] = mid.y;
  xw[WL + 2] = mid.z;
  xw[WL + 3] = mid.w;
}

// ----------------------------------------------------------------------------
// Weight grad, every tap in one thread (k = 1, 3).  The ring slot carries the
// x plane tile and, after it, the dy plane tile of the same step.
// ----------------------------------------------------------------------------
template <typename T, int K, int NH>
__global__ void __launch_bounds__(kDwMaxComputeWarps * 32 + 32, 2)
    dw_s1_wgrad_tma_kernel(const __grid_constant__ CUtensorMap mX, const __grid_constant__ CUtensorMap mDY,
                           typename Elem<T>::Acc* __restrict__ part, DwS1Geom g) {
  using Acc = typename Elem<T>::Acc;
  using L = DwTmaLayout<T>;
  constexpr int P = K / 2;
  constexpr int K3 = K * K * K;
  constexpr int OFF = DwTile<T>::off(P);
  constexpr int E = DwTile<T>::E;
  // k = 3 on 16-bit types: mixed-precision FMAs straight from the packed elements
  constexpr bool kMixed =
      K == 3 && kDwNW == 8 && (std::is_same<T, __nv_bfloat16>::value || std::is_same<T, __half>::value);
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ DwRing ring;
  const size_t slot_bytes = L::slot(g, K, true);
  const size_t x_bytes = L::x_tile(g, K);
  const size_t dy_off = L::dy_offset(g, K);
  unsigned char* slots = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  const int compute_threads = (int)blockDim.x - 32;
  const bool producer = (int)threadIdx.x >= compute_threads;

  int b = blockIdx.x;
  const int tw = b % g.tilesW;
  b /= g.tilesW;
  const int th = b % g.tilesH;
  b /= g.tilesH;
  const int td = b % g.tilesD;
  const int nc = b / g.tilesD;
  const int w0 = tw * g.TW, h0 = th * g.TH, d0 = td * g.TD;
  const int rsw = DwTile<T>::row_elems(g.TW, P);
  const int dcount = min(g.TD, g.D - d0);
  const int nsteps = dcount + K - 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kDwSlots; ++i) {
      mbar_init(&ring.full[i], 1);
      mbar_init(&ring.empty[i], (uint32_t)(compute_threads / 32));
    }
    ring.abort = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  volatile int* abort = &ring.abort;
  int issued = 0;

  Acc acc[K3 + 1];
#pragma unroll
  for (int t = 0; t <= K3; ++t) acc[t] = Acc(0);

  if (producer) {
    if ((threadIdx.x & 31) == 0) {
      tma_prefetch_map(&mX);
      tma_prefetch_map(&mDY);
      for (int s = 0; s < nsteps && !*abort; ++s) {
        const int slot = s % kDwSlots, r = s / kDwSlots;
        if (r > 0 && !mbar_wait(&ring.empty[slot], (uint32_t)((r - 1) & 1))) {
          *abort = 1;
          break;
        }
        unsigned char* dst = slots + (size_t)slot * slot_bytes;
        const bool with_dy = s < dcount;
        mbar_arrive_expect_tx(&ring.full[slot], (uint32_t)(x_bytes + (with_dy ? L::dy_tile(g) : 0)));
        tma_load_4d(dst, &mX, &ring.full[slot], w0 - OFF, h0 - P, d0 - P + s, nc);
        if (with_dy) tma_load_4d(dst + dy_off, &mDY, &ring.full[slot], w0, h0, d0 + s, nc);
        ++issued;
      }
    }
  } else if constexpr (kMixed) {
    // 16-bit x and dy stay packed as loaded; every product is one mixed-precision
    // FMA (16-bit operands, fp32 accumulator), in the order of the branch below,
    // so the tap sums are bit-identical to it on the widened inputs.
    const int lane = threadIdx.x & 31;
    const int wt = threadIdx.x % g.LW;
    const int tr = threadIdx.x / g.LW;
    const int hrow = tr * NH;
    const bool active = tr < g.TR;
    uint32_t dyw[K][NH][kDwNW / 2];  // dy rows of the last K planes, two elements per word
#pragma unroll
    for (int a = 0; a < K; ++a)
#pragma unroll
      for (int jh = 0; jh < NH; ++jh)
#pragma unroll
        for (int i = 0; i < kDwNW / 2; ++i) dyw[a][jh][i] = 0u;

    bool stop = false;  // warp-uniform: every lane leaves the loop at the same step
    for (int sb = 0; sb < nsteps && !stop; sb += K) {
#pragma unroll
      for (int j = 0; j < K; ++j) {
        const int s = sb + j;
        if (s < nsteps) {
          const int slot = s % kDwSlots;
          const bool ok = !*abort && mbar_wait(&ring.full[slot], (uint32_t)((s / kDwSlots) & 1));
          if (!__all_sync(0xffffffffu, ok)) {
            *abort = 1;
            stop = true;
            break;
          }
          const unsigned char* base = slots + (size_t)slot * slot_bytes;
          const T* sp = reinterpret_cast<const T*>(base);
          if (active && s < dcount) {
            const T* dyt = reinterpret_cast<const T*>(base + dy_off);
#pragma unroll
            for (int jh = 0; jh < NH; ++jh) {
              const uint4 q = *reinterpret_cast<const uint4*>(dyt + (size_t)(hrow + jh) * g.TW + kDwNW * wt);
              dyw[j][jh][0] = q.x;
              dyw[j][jh][1] = q.y;
              dyw[j][jh][2] = q.z;
              dyw[j][jh][3] = q.w;
#pragma unroll
              for (int i = 0; i < kDwNW; ++i) acc[K3] = mix_fma<T>(half16(dyw[j][jh], i), one16<T>(), acc[K3]);
            }
          } else {
#pragma unroll
            for (int jh = 0; jh < NH; ++jh)
#pragma unroll
              for (int i = 0; i < kDwNW / 2; ++i) dyw[j][jh][i] = 0u;
          }
          if (active) {
#pragma unroll
            for (int r = 0; r < NH + K - 1; ++r) {
              uint32_t xw[4 + 2 * kMixWL<P>];
              dw_read_window_raw<P>(sp + (size_t)(hrow + r) * rsw, wt, xw);
#pragma unroll
              for (int jh = 0; jh < NH; ++jh) {
                const int kh = r - jh;
                if (kh < 0 || kh >= K) continue;
#pragma unroll
                for (int kd = 0; kd < K; ++kd) {
                  const int dslot = (j - kd + K) % K;
#pragma unroll
                  for (int kw = 0; kw < K; ++kw) {
                    float sacc = acc[(kd * K + kh) * K + kw];
#pragma unroll
                    for (int i = 0; i < kDwNW; ++i)
                      sacc = mix_fma<T>(half16(xw, i + kw + kMixH0<P>), half16(dyw[dslot][jh], i), sacc);
                    acc[(kd * K + kh) * K + kw] = sacc;
                  }
                }
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&ring.empty[slot]);
        }
      }
    }
  } else {
    const int lane = threadIdx.x & 31;
    const int wt = threadIdx.x % g.LW;
    const int tr = threadIdx.x / g.LW;
    const int hrow = tr * NH;
    const bool active = tr < g.TR;
    Acc dyr[K][NH][kDwNW];
#pragma unroll
    for (int a = 0; a < K; ++a)
#pragma unroll
      for (int jh = 0; jh < NH; ++jh)
#pragma unroll
        for (int i = 0; i < kDwNW; ++i) dyr[a][jh][i] = Acc(0);

    bool stop = false;  // warp-uniform: every lane leaves the loop at the same step
    for (int sb = 0; sb < nsteps && !stop; sb += K) {
#pragma unroll
      for (int j = 0; j < K; ++j) {
        const int s = sb + j;
        if (s < nsteps) {
          const int slot = s % kDwSlots;
          const bool ok = !*abort && mbar_wait(&ring.full[slot], (uint32_t)((s / kDwSlots) & 1));
          if (!__all_sync(0xffffffffu, ok)) {
            *abort = 1;
            stop = true;
            break;
          }
          const unsigned char* base = slots + (size_t)slot * slot_bytes;
          const T* sp = reinterpret_cast<const T*>(base);
          // dy plane s (relative) into ring slot j; zero beyond the chunk
          if (active && s < dcount) {
            const T* dyt = reinterpret_cast<const T*>(base + dy_off);
#pragma unroll
            for (int jh = 0; jh < NH; ++jh) {
              const uint4* rowp = reinterpret_cast<const uint4*>(dyt + (size_t)(hrow + jh) * g.TW + kDwNW * wt);
#pragma unroll
              for (int q = 0; q < kDwNW / E; ++q) unpack16<T>(rowp[q], dyr[j][jh] + q * E);
#pragma unroll
              for (int i = 0; i < kDwNW; ++i) acc[K3] += dyr[j][jh][i];
            }
          } else {
#pragma unroll
            for (int jh = 0; jh < NH; ++jh)
#pragma unroll
              for (int i = 0; i < kDwNW; ++i) dyr[j][jh][i] = Acc(0);
          }
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
                  const int dslot = (j - kd + K) % K;
#pragma unroll
                  for (int kw = 0; kw < K; ++kw) {
                    Acc sacc = acc[(kd * K + kh) * K + kw];
#pragma unroll
                    for (int i = 0; i < kDwNW; ++i) sacc = fma(win[i + kw], dyr[dslot][jh][i], sacc);
                    acc[(kd * K + kh) * K + kw] = sacc;
                  }
                }
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&ring.empty[slot]);
        }
      }
    }
  }

  __shared__ Acc red[(kDwMaxComputeWarps + 1) * (K3 + 1)];
  __syncthreads();
  if (*abort && producer && (threadIdx.x & 31) == 0) dw_ring_drain(ring, issued);
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
  if (*abort && threadIdx.x == 0) raise_device_error(kErrMbarTimeout);
}

// ----------------------------------------------------------------------------
// Weight grad for k = 5, 7 on a TMA plane ring.  The compute threads form K
// groups (group g owns the K*K taps with kd = g); a producer warp streams the x
// plane tile and the dy plane tile of each step into a ring of kDwGSlots(K)
// slots.  At step s group g pairs x plane d0 - P + s (slot s) with dy plane
// d0 + s - g (slot s - g, landed g steps earlier), so a slot is released by
// each group after its last use: group g's warps arrive on slot s - g's empty
// barrier at step s, and the producer refills a slot once every compute warp
// has arrived.  No block barrier inside the loop.
// ----------------------------------------------------------------------------
__host__ __device__ constexpr int dw_gslots(int K) { return K + 2; }
constexpr int kDwGMaxSlots = 9;

struct DwGRing {
  uint64_t full[kDwGMaxSlots];
  uint64_t empty[kDwGMaxSlots];
  int abort;
};

template <typename T, int K, int NH>
__global__ void __launch_bounds__(448 + 32, 1)
    dw_s1_wgrad_grouped_tma_kernel(const __grid_constant__ CUtensorMap mX, const __grid_constant__ CUtensorMap mDY,
                                   typename Elem<T>::Acc* __restrict__ part, DwS1Geom g) {
  using Acc = typename Elem<T>::Acc;
  using L = DwTmaLayout<T>;
  constexpr int P = K / 2;
  constexpr int K2 = K * K;
  constexpr int K3 = K2 * K;
  constexpr int OFF = DwTile<T>::off(P);
  constexpr int E = DwTile<T>::E;
  constexpr int S = dw_gslots(K);
  static_assert(S <= kDwGMaxSlots, "ring depth");
  // 16-bit types: mixed-precision FMAs straight from the packed elements
  constexpr bool kMixed = P <= 3 && kDwNW == 8 && DwTile<T>::off(P) == 8 &&
                          (std::is_same<T, __nv_bfloat16>::value || std::is_same<T, __half>::value);
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ DwGRing ring;
  const size_t slot_bytes = L::slot(g, K, true);
  const size_t x_bytes = L::x_tile(g, K);
  const size_t dy_off = L::dy_offset(g, K);
  unsigned char* slots = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  const int compute_threads = (int)blockDim.x - 32;
  const bool producer = (int)threadIdx.x >= compute_threads;

  int b = blockIdx.x;
  const int tw = b % g.tilesW;
  b /= g.tilesW;
  const int th = b % g.tilesH;
  b /= g.tilesH;
  const int td = b % g.tilesD;
  const int nc = b / g.tilesD;
  const int w0 = tw * g.TW, h0 = th * g.TH, d0 = td * g.TD;
  const int rsw = DwTile<T>::row_elems(g.TW, P);
  const int dcount = min(g.TD, g.D - d0);
  const int nsteps = dcount + K - 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&ring.full[i], 1);
      mbar_init(&ring.empty[i], (uint32_t)(compute_threads / 32));
    }
    ring.abort = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  volatile int* abort = &ring.abort;
  int issued = 0;

  Acc acc[K2 + 1];
#pragma unroll
  for (int t = 0; t <= K2; ++t) acc[t] = Acc(0);
  const int G = compute_threads / K;  // threads per group, whole warps
  const int grp = producer ? 0 : (int)threadIdx.x / G;

  if (producer) {
    if ((threadIdx.x & 31) == 0) {
      tma_prefetch_map(&mX);
      tma_prefetch_map(&mDY);
      for (int s = 0; s < nsteps && !*abort; ++s) {
        const int slot = s % S, r = s / S;
        if (r > 0 && !mbar_wait(&ring.empty[slot], (uint32_t)((r - 1) & 1))) {
          *abort = 1;
          break;
        }
        unsigned char* dst = slots + (size_t)slot * slot_bytes;
        const bool with_dy = s < dcount;
        mbar_arrive_expect_tx(&ring.full[slot], (uint32_t)(x_bytes + (with_dy ? L::dy_tile(g) : 0)));
        tma_load_4d(dst, &mX, &ring.full[slot], w0 - OFF, h0 - P, d0 - P + s, nc);
        if (with_dy) tma_load_4d(dst + dy_off, &mDY, &ring.full[slot], w0, h0, d0 + s, nc);
        ++issued;
      }
    }
  } else {
    const int lane = threadIdx.x & 31;
    const int lt = (int)threadIdx.x - grp * G;
    const int wt = lt % g.LW;
    const int tr = lt / g.LW;
    const int hrow = tr * NH;
    const bool active = tr < g.TR;
    for (int s = 0; s < nsteps; ++s) {
      const int slot = s % S;
      const bool ok = !*abort && mbar_wait(&ring.full[slot], (uint32_t)((s / S) & 1));
      if (!__all_sync(0xffffffffu, ok)) {
        *abort = 1;
        break;
      }
      const int orel = s - grp;  // this group's dy plane (relative), landed in slot orel % S
      if (orel >= 0) {
        if (active && orel < dcount) {
          const T* sp = reinterpret_cast<const T*>(slots + (size_t)slot * slot_bytes);
          const T* dyt = reinterpret_cast<const T*>(slots + (size_t)(orel % S) * slot_bytes + dy_off);
          if constexpr (kMixed) {
            // 16-bit operands straight from the packed elements (mixed-precision
            // FMAs; the products and their order as in the branch below)
            uint32_t dyw[NH][kDwNW / 2];
#pragma unroll
            for (int jh = 0; jh < NH; ++jh) {
              const uint4 q = *reinterpret_cast<const uint4*>(dyt + (size_t)(hrow + jh) * g.TW + kDwNW * wt);
              dyw[jh][0] = q.x;
              dyw[jh][1] = q.y;
              dyw[jh][2] = q.z;
              dyw[jh][3] = q.w;
              if (grp == 0) {
#pragma unroll
                for (int i = 0; i < kDwNW; ++i) acc[K2] = mix_fma<T>(half16(dyw[jh], i), one16<T>(), acc[K2]);
              }
            }
#pragma unroll
            for (int r = 0; r < NH + K - 1; ++r) {
              uint32_t xw[4 + 2 * kMixWL<P>];
              dw_read_window_raw<P>(sp + (size_t)(hrow + r) * rsw, wt, xw);
#pragma unroll
              for (int jh = 0; jh < NH; ++jh) {
                const int kh = r - jh;
                if (kh < 0 || kh >= K) continue;
#pragma unroll
                for (int kw = 0; kw < K; ++kw) {
                  float sacc = acc[kh * K + kw];
#pragma unroll
                  for (int i = 0; i < kDwNW; ++i)
                    sacc = mix_fma<T>(half16(xw, i + kw + kMixH0<P>), half16(dyw[jh], i), sacc);
                  acc[kh * K + kw] = sacc;
                }
              }
            }
          } else {
            Acc dyp[NH][kDwNW];
#pragma unroll
            for (int jh = 0; jh < NH; ++jh) {
              const uint4* rowp = reinterpret_cast<const uint4*>(dyt + (size_t)(hrow + jh) * g.TW + kDwNW * wt);
#pragma unroll
              for (int q = 0; q < kDwNW / E; ++q) unpack16<T>(rowp[q], dyp[jh] + q * E);
              if (grp == 0) {
#pragma unroll
                for (int i = 0; i < kDwNW; ++i) acc[K2] += dyp[jh][i];
              }
            }
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
        }
        // this group is done with slot orel (its x at step orel, its dy now)
        __syncwarp();
        if (lane == 0) mbar_arrive(&ring.empty[orel % S]);
      }
    }
  }

  __shared__ Acc red[15 * (K2 + 1)];
  __syncthreads();
  if (*abort && producer && (threadIdx.x & 31) == 0) {
    for (int q = issued > S ? issued - S : 0; q < issued; ++q)
      mbar_wait(&ring.full[q % S], (uint32_t)((q / S) & 1));
  }
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
    Acc sum = Acc(0);
    for (int w = 0; w < wpg; ++w) sum += red[(gg * wpg + w) * (K2 + 1) + t];
    if (t == K2) dst[K3] = sum;
    else dst[gg * K2 + t] = sum;
  }
  if (*abort && threadIdx.x == 0) raise_device_error(kErrMbarTimeout);
}

}  // namespace mednext
