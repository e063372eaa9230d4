// Stride-2 depthwise gather (the down block's forward, k = 3, 16-bit types)
// with the input planes streamed by TMA and packed fp32 FMAs (sm_100a).
//
//   small[m] = bias + sum_t big[2m - 1 + t] * w[t]    (t over the 3x3x3 taps)
//
// A CTA owns one (sample, channel) tile of TWo x THo outputs and a chunk of
// output planes.  The halo'd input plane tiles (2*THo + 1 rows, 2*TWo + 16
// columns starting at the 16-byte boundary 2*ow0 - 8) stream through the same
// kDwSlots ring as the stride-1 packed kernel, with no producer warp: thread 0
// issues the first loads and the warp that releases a slot last issues the
// slot's next load.  Out-of-range rows, columns and planes arrive as zeros,
// which is the convolution's zero padding.
//
// Each thread owns 8 outputs of one row and accumulates the pairs (i, i+4) with
// fma.rn.f32x2; the window pairs (x[m-1], x[m+7]) are the stride-1 packed
// kernel's.  Input plane s of a chunk feeds output plane s/2 with tap kd = 0
// (even s, which also finishes output s/2 - 1 with kd = 2) or output (s-1)/2
// with kd = 1 (odd s), so every output sums bias first, then its taps in
// (kd, kh, kw) order: the order of dw_s2_gather_kernel, whose results this
// kernel reproduces bit for bit.
#pragma once

#include <type_traits>

#include "depthwise_s1_tma.cuh"
#include "depthwise_s2.cuh"

namespace mednext {

constexpr int kS2PkThreads = 256;

struct DwS2PkGeom {
  DwS2Geom g;
  int TWo, THo, TDo;  // output tile (columns, rows, planes)
  int tilesW, tilesH, tilesD;
  int lw;             // threads along W (8 outputs each)
};

template <typename T>
struct DwS2PkLayout {
  static __host__ __device__ int pitch(int TWo) { return 2 * TWo + 16; }
  static __host__ __device__ int rows(int THo) { return 2 * THo + 1; }
  static __host__ __device__ size_t x_tile(const DwS2PkGeom& p) { return (size_t)rows(p.THo) * pitch(p.TWo) * sizeof(T); }
  static __host__ __device__ size_t slot(const DwS2PkGeom& p) { return DwTmaLayout<T>::align128(x_tile(p)); }
  static __host__ size_t smem(const DwS2PkGeom& p) { return 128 + kDwSlots * slot(p); }
};

// p[m] = (x[m-1], x[m+7]), m = 0..8, for the 17 inputs x[-1..15] of the thread's
// 8 outputs; rowp[col] is x[0].  x[-1] comes from the left neighbour's last
// input (lane src_l), or from the row's halo column at the tile edge.
template <typename T>
__device__ __forceinline__ void dw_s2pk_window(const T* __restrict__ rowp, int col, bool left_edge, int src_l,
                                               uint64_t (&p)[9]) {
  const uint4 c0 = *reinterpret_cast<const uint4*>(rowp + col);      // x[0..7]
  const uint4 c1 = *reinterpret_cast<const uint4*>(rowp + col + 8);  // x[8..15]
  const uint32_t from_l = __shfl_sync(0xffffffffu, c1.w, src_l);     // (x[14], x[15]) of the left neighbour
  const uint32_t el = reinterpret_cast<const unsigned short*>(rowp)[col - 1];
  const uint32_t xl = left_edge ? el : (from_l >> 16);
  const uint32_t a[4] = {c0.x, c0.y, c0.z, c0.w};
  const uint32_t b[4] = {c1.x, c1.y, c1.z, c1.w};
  p[0] = pk_pair(lo_bits<T>(xl), hi_bits<T>(a[3]));
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    p[2 * q + 1] = pk_pair(lo_bits<T>(a[q]), lo_bits<T>(b[q]));  // (x[2q], x[2q+8])
    p[2 * q + 2] = pk_pair(hi_bits<T>(a[q]), hi_bits<T>(b[q]));  // (x[2q+1], x[2q+9])
  }
}

// ADD: an addend of the output's shape is added last (the up block's input grad
// takes its residual branch's grad this way), one rounding per output.
template <typename T, bool ADD>
__global__ void __launch_bounds__(kS2PkThreads, 2)
    dw_s2_gather_pk_kernel(const __grid_constant__ CUtensorMap mX, const T* __restrict__ wgt,
                           const T* __restrict__ bias, const T* __restrict__ addend, T* __restrict__ small,
                           DwS2PkGeom pg) {
  constexpr int K = 3;
  constexpr int K3 = 27;
  using L = DwS2PkLayout<T>;
  const DwS2Geom& g = pg.g;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ DwPkRing ring;
  unsigned char* slots = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  const size_t slot_bytes = L::slot(pg);
  const uint32_t tile_bytes = (uint32_t)L::x_tile(pg);
  const int rsp = L::pitch(pg.TWo);
  const int nwarps = (int)blockDim.x >> 5;

  int bx = blockIdx.x;
  const int tw = bx % pg.tilesW;
  bx /= pg.tilesW;
  const int th = bx % pg.tilesH;
  bx /= pg.tilesH;
  const int td = bx % pg.tilesD;
  const int nc = bx / pg.tilesD;
  const int c = nc % g.C;
  const int ow0 = tw * pg.TWo, oh0 = th * pg.THo, md0 = td * pg.TDo;
  const int dcount = min(pg.TDo, g.Ds - md0);
  const int nsteps = 2 * dcount + 1;

  auto issue = [&](int q) {
    const int slot = q % kDwSlots;
    mbar_arrive_expect_tx(&ring.full[slot], tile_bytes);
    tma_load_4d(slots + (size_t)slot * slot_bytes, &mX, &ring.full[slot], 2 * ow0 - 8, 2 * oh0 - 1, 2 * md0 - 1 + q,
                nc);
  };
  if (threadIdx.x == 0) {
    for (int i = 0; i < kDwSlots; ++i) {
      mbar_init(&ring.full[i], 1);
      ring.released[i] = 0;
    }
    ring.abort = 0;
    fence_mbarrier_init();
    tma_prefetch_map(&mX);
    const int first = min(nsteps, kDwSlots);
    for (int q = 0; q < first; ++q) issue(q);
    ring.issued = first;
  }
  __syncthreads();
  volatile int* abort = &ring.abort;

  const int lane = threadIdx.x & 31;
  const int lw = pg.lw;
  const int wt = threadIdx.x % lw;
  const int r = threadIdx.x / lw;
  const bool active = r < pg.THo;
  const int oh = oh0 + r;
  const int ow = ow0 + 8 * wt;
  // Ws is a multiple of 8 on this path: a thread's 8 outputs are in or out as a whole
  const bool store_row = active && oh < g.Hs && ow < g.Ws;
  // a row of lw <= 8 threads lies within one warp: the left neighbour is lane - 1
  const int src_l = wt > 0 ? lane - 1 : lane;
  const bool left_edge = wt == 0;
  // lanes past the tile read row 0 (every lane joins the shuffles) and store nothing
  const int xbase = (active ? 2 * r : 0) * rsp;
  const int col = 8 + 16 * wt;
  uint64_t wp[K3];
#pragma unroll
  for (int t = 0; t < K3; ++t) {
    const uint32_t wv = __float_as_uint(to_acc<T>(__ldg(wgt + (size_t)c * K3 + t)));
    wp[t] = pk_pair(wv, wv);
  }
  const uint32_t bvb = __float_as_uint(bias != nullptr ? to_acc<T>(bias[c]) : 0.f);
  const uint64_t bv2 = pk_pair(bvb, bvb);
  const size_t plane = (size_t)g.Hs * g.Ws;
  T* out0 = small + ((size_t)nc * g.Ds) * plane + (size_t)oh * g.Ws + ow;
  const T* add0 = ADD ? addend + ((size_t)nc * g.Ds) * plane + (size_t)oh * g.Ws + ow : nullptr;

  uint64_t acc[2][4];
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[a][i] = 0ull;

  // step s (phase F = s % 4): input plane 2*md0 - 1 + s.  Even s = 2u finishes
  // output u - 1 (tap kd = 2, slot (u-1) % 2) and starts output u (bias, then
  // kd = 0, slot u % 2); odd s = 2u + 1 adds kd = 1 to output u.
  auto step = [&](auto fc, const int s) -> bool {
    constexpr int F = decltype(fc)::value;
    constexpr bool even = (F % 2) == 0;
    constexpr int cur = (F / 2) % 2;   // slot of output u = s / 2
    constexpr int prev = 1 - cur;      // slot of output u - 1
    const int slot = s % kDwSlots;
    const bool ok = !*abort && mbar_wait(&ring.full[slot], (uint32_t)((s / kDwSlots) & 1));
    if (!__all_sync(0xffffffffu, ok)) {
      *abort = 1;
      return false;
    }
    const int u = s >> 1;
    const bool finish = even && u >= 1;
    const bool start = even && u < dcount;
    if (start) {
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[cur][i] = bv2;
    }
    const T* xp = reinterpret_cast<const T*>(slots + (size_t)slot * slot_bytes) + xbase;
#pragma unroll
    for (int kh = 0; kh < K; ++kh) {
      uint64_t p[9];
      dw_s2pk_window<T>(xp + kh * rsp, col, left_edge, src_l, p);
#pragma unroll
      for (int kw = 0; kw < K; ++kw) {
        if constexpr (even) {
          if (finish) {
            const uint64_t w2 = wp[(2 * K + kh) * K + kw];
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[prev][i] = pk_fma(p[2 * i + kw], w2, acc[prev][i]);
          }
          if (start) {
            const uint64_t w0 = wp[(0 * K + kh) * K + kw];
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[cur][i] = pk_fma(p[2 * i + kw], w0, acc[cur][i]);
          }
        } else {
          const uint64_t w1 = wp[(1 * K + kh) * K + kw];
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[cur][i] = pk_fma(p[2 * i + kw], w1, acc[cur][i]);
        }
      }
    }
    // release the slot; the warp that releases it last loads the slot's next plane
    __syncwarp();
    if (lane == 0) {
      int prv;
      asm volatile("atom.acq_rel.cta.shared::cta.add.s32 %0, [%1], 1;"
                   : "=r"(prv)
                   : "r"(smem_u32(&ring.released[slot]))
                   : "memory");
      // the count only grows: the slot's (s / kDwSlots)-th plane is released by nwarps arrivals
      if (prv == (s / kDwSlots + 1) * nwarps - 1) {
        const int q = s + kDwSlots;
        if (q < nsteps) {
          fence_async_smem();
          issue(q);
          atomicAdd(&ring.issued, 1);
        }
      }
    }
    if (finish && store_row) {
      float lo[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) pk_split(acc[prev][i], lo[i], lo[i + 4]);
      if constexpr (ADD) {
        float av[8];
        unpack16<T>(__ldg(reinterpret_cast<const uint4*>(add0 + (size_t)(md0 + u - 1) * plane)), av);
#pragma unroll
        for (int e = 0; e < 8; ++e) lo[e] += av[e];
      }
      *reinterpret_cast<uint4*>(out0 + (size_t)(md0 + u - 1) * plane) = pack16<T>(lo);
    }
    return true;
  };
  using F0 = std::integral_constant<int, 0>;
  using F1 = std::integral_constant<int, 1>;
  using F2 = std::integral_constant<int, 2>;
  using F3 = std::integral_constant<int, 3>;
  // whole rounds of 4 steps, then the remainder; every lane of a warp leaves together
  int sb = 0;
  bool ok = true;
  for (; ok && sb + 4 <= nsteps; sb += 4)
    ok = step(F0{}, sb) && step(F1{}, sb + 1) && step(F2{}, sb + 2) && step(F3{}, sb + 3);
  if (ok && sb < nsteps) ok = step(F0{}, sb);
  if (ok && sb + 1 < nsteps) ok = step(F1{}, sb + 1);
  if (ok && sb + 2 < nsteps) step(F2{}, sb + 2);

  __syncthreads();
  // after an abort, wait (bounded) for the loads still in flight before the CTA exits
  if (*abort && threadIdx.x == 0) {
    const int issued = ring.issued;
    for (int q = issued > kDwSlots ? issued - kDwSlots : 0; q < issued; ++q)
      mbar_wait(&ring.full[q % kDwSlots], (uint32_t)((q / kDwSlots) & 1));
    raise_device_error(kErrMbarTimeout);
  }
}

// ----------------------------------------------------------------------------
// Stride-2 weight grad of the down block (k = 3, 16-bit types):
//   dw[t] = sum_m big[2m - 1 + t] * small[m],  dbias = sum_m small[m]
// Same tile, ring and input windows as dw_s2_gather_pk_kernel; a slot also holds
// the small-grid (dy) plane tile of output plane s/2 at even steps.  The thread's
// dy row (8 values as pairs (i, i+4)) stays in registers for the three steps that
// use it (kd = 0 at step 2u, kd = 1 at 2u + 1, kd = 2 at 2u + 2).  The 27 tap
// sums and the bias sum are per-thread pairs folded at the end in a fixed order;
// one partial per (sample, channel, tile), summed by dw_wgrad_finish_kernel.
// ----------------------------------------------------------------------------
template <typename T>
struct DwS2PkWLayout {
  static __host__ __device__ size_t dy_offset(const DwS2PkGeom& p) {
    return DwTmaLayout<T>::align128(DwS2PkLayout<T>::x_tile(p));
  }
  static __host__ __device__ size_t dy_tile(const DwS2PkGeom& p) { return (size_t)p.THo * p.TWo * sizeof(T); }
  static __host__ __device__ size_t slot(const DwS2PkGeom& p) { return DwTmaLayout<T>::align128(dy_offset(p) + dy_tile(p)); }
  static __host__ size_t smem(const DwS2PkGeom& p) { return 128 + kDwSlots * slot(p); }
};

// BIG_BIAS: the bias slot sums the big grid instead (the up block, whose dy is
// the big grid): each thread adds the 2 rows x 16 columns of the big planes that
// its outputs own (tile rows 1 + 2r, 2 + 2r; every plane but the chunk's first,
// which belongs to the previous chunk); zero-filled positions past the grid add
// nothing, so every grid voxel is summed once.
template <typename T, bool BIG_BIAS>
__global__ void __launch_bounds__(kS2PkThreads, 2)
    dw_s2_wgrad_pk_kernel(const __grid_constant__ CUtensorMap mX, const __grid_constant__ CUtensorMap mDY,
                          float* __restrict__ part, DwS2PkGeom pg) {
  constexpr int K = 3;
  constexpr int K3 = 27;
  using L = DwS2PkLayout<T>;
  using LW = DwS2PkWLayout<T>;
  const DwS2Geom& g = pg.g;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ DwPkRing ring;
  __shared__ float red[(kS2PkThreads / 32) * (K3 + 1)];
  unsigned char* slots = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  const size_t slot_bytes = LW::slot(pg);
  const size_t dy_off = LW::dy_offset(pg);
  const uint32_t x_bytes = (uint32_t)L::x_tile(pg);
  const uint32_t dy_bytes = (uint32_t)LW::dy_tile(pg);
  const int rsp = L::pitch(pg.TWo);
  const int nwarps = (int)blockDim.x >> 5;

  int bx = blockIdx.x;
  const int tw = bx % pg.tilesW;
  bx /= pg.tilesW;
  const int th = bx % pg.tilesH;
  bx /= pg.tilesH;
  const int td = bx % pg.tilesD;
  const int nc = bx / pg.tilesD;
  const int ow0 = tw * pg.TWo, oh0 = th * pg.THo, md0 = td * pg.TDo;
  const int dcount = min(pg.TDo, g.Ds - md0);
  const int nsteps = 2 * dcount + 1;

  // step q: the big plane 2*md0 - 1 + q and, at even q below 2*dcount, the small plane md0 + q/2
  auto issue = [&](int q) {
    const int slot = q % kDwSlots;
    unsigned char* dst = slots + (size_t)slot * slot_bytes;
    const bool with_dy = (q % 2) == 0 && q / 2 < dcount;
    mbar_arrive_expect_tx(&ring.full[slot], x_bytes + (with_dy ? dy_bytes : 0u));
    tma_load_4d(dst, &mX, &ring.full[slot], 2 * ow0 - 8, 2 * oh0 - 1, 2 * md0 - 1 + q, nc);
    if (with_dy) tma_load_4d(dst + dy_off, &mDY, &ring.full[slot], ow0, oh0, md0 + q / 2, nc);
  };
  if (threadIdx.x == 0) {
    for (int i = 0; i < kDwSlots; ++i) {
      mbar_init(&ring.full[i], 1);
      ring.released[i] = 0;
    }
    ring.abort = 0;
    fence_mbarrier_init();
    tma_prefetch_map(&mX);
    tma_prefetch_map(&mDY);
    const int first = min(nsteps, kDwSlots);
    for (int q = 0; q < first; ++q) issue(q);
    ring.issued = first;
  }
  __syncthreads();
  volatile int* abort = &ring.abort;

  const int lane = threadIdx.x & 31;
  const int lw = pg.lw;
  const int wt = threadIdx.x % lw;
  const int r = threadIdx.x / lw;
  const bool active = r < pg.THo;
  const int src_l = wt > 0 ? lane - 1 : lane;
  const bool left_edge = wt == 0;
  // lanes past the tile read row 0 (every lane joins the shuffles) with a zero dy
  const int xbase = (active ? 2 * r : 0) * rsp;
  const int col = 8 + 16 * wt;
  const int dybase = (active ? r : 0) * pg.TWo + 8 * wt;

  uint64_t acc[K3];
  uint64_t accb = 0ull;
  uint64_t dyp[2][4];
#pragma unroll
  for (int t = 0; t < K3; ++t) acc[t] = 0ull;
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int i = 0; i < 4; ++i) dyp[a][i] = 0ull;

  // step s (phase F = s % 4), u = s / 2: even s loads dy plane u into slot u % 2 and
  // adds kd = 0 (dy u) and kd = 2 (dy u - 1); odd s adds kd = 1 (dy u).
  auto step = [&](auto fc, const int s) -> bool {
    constexpr int F = decltype(fc)::value;
    constexpr bool even = (F % 2) == 0;
    constexpr int cur = (F / 2) % 2;
    constexpr int prev = 1 - cur;
    const int slot = s % kDwSlots;
    const bool ok = !*abort && mbar_wait(&ring.full[slot], (uint32_t)((s / kDwSlots) & 1));
    if (!__all_sync(0xffffffffu, ok)) {
      *abort = 1;
      return false;
    }
    const int u = s >> 1;
    const unsigned char* sb = slots + (size_t)slot * slot_bytes;
    if constexpr (even) {
      if (active && u < dcount) {
        const uint4 d = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(sb + dy_off) + dybase);
        dyp[cur][0] = pk_pair(lo_bits<T>(d.x), lo_bits<T>(d.z));
        dyp[cur][1] = pk_pair(hi_bits<T>(d.x), hi_bits<T>(d.z));
        dyp[cur][2] = pk_pair(lo_bits<T>(d.y), lo_bits<T>(d.w));
        dyp[cur][3] = pk_pair(hi_bits<T>(d.y), hi_bits<T>(d.w));
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) dyp[cur][i] = 0ull;
      }
      if constexpr (!BIG_BIAS) {
#pragma unroll
        for (int i = 0; i < 4; ++i) accb = pk_add(accb, dyp[cur][i]);
      }
    }
    const T* xp = reinterpret_cast<const T*>(sb) + xbase;
#pragma unroll
    for (int kh = 0; kh < K; ++kh) {
      uint64_t p[9];
      dw_s2pk_window<T>(xp + kh * rsp, col, left_edge, src_l, p);
      if constexpr (BIG_BIAS) {
        // p[1..8] hold the thread's own 16 columns of this row
        if (kh > 0 && s > 0 && active) {
#pragma unroll
          for (int m = 1; m <= 8; ++m) accb = pk_add(accb, p[m]);
        }
      }
#pragma unroll
      for (int kw = 0; kw < K; ++kw) {
        if constexpr (even) {
          uint64_t a0 = acc[(0 * K + kh) * K + kw], a2 = acc[(2 * K + kh) * K + kw];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            a0 = pk_fma(p[2 * i + kw], dyp[cur][i], a0);
            a2 = pk_fma(p[2 * i + kw], dyp[prev][i], a2);
          }
          acc[(0 * K + kh) * K + kw] = a0;
          acc[(2 * K + kh) * K + kw] = a2;
        } else {
          uint64_t a1 = acc[(1 * K + kh) * K + kw];
#pragma unroll
          for (int i = 0; i < 4; ++i) a1 = pk_fma(p[2 * i + kw], dyp[cur][i], a1);
          acc[(1 * K + kh) * K + kw] = a1;
        }
      }
    }
    // release the slot; the warp that releases it last loads the slot's next planes
    __syncwarp();
    if (lane == 0) {
      int prv;
      asm volatile("atom.acq_rel.cta.shared::cta.add.s32 %0, [%1], 1;"
                   : "=r"(prv)
                   : "r"(smem_u32(&ring.released[slot]))
                   : "memory");
      // the count only grows: the slot's (s / kDwSlots)-th planes are released by nwarps arrivals
      if (prv == (s / kDwSlots + 1) * nwarps - 1) {
        const int q = s + kDwSlots;
        if (q < nsteps) {
          fence_async_smem();
          issue(q);
          atomicAdd(&ring.issued, 1);
        }
      }
    }
    return true;
  };
  using F0 = std::integral_constant<int, 0>;
  using F1 = std::integral_constant<int, 1>;
  using F2 = std::integral_constant<int, 2>;
  using F3 = std::integral_constant<int, 3>;
  int sb = 0;
  bool ok = true;
  for (; ok && sb + 4 <= nsteps; sb += 4)
    ok = step(F0{}, sb) && step(F1{}, sb + 1) && step(F2{}, sb + 2) && step(F3{}, sb + 3);
  if (ok && sb < nsteps) ok = step(F0{}, sb);
  if (ok && sb + 1 < nsteps) ok = step(F1{}, sb + 1);
  if (ok && sb + 2 < nsteps) step(F2{}, sb + 2);

  __syncthreads();
  // after an abort, wait (bounded) for the loads still in flight before the CTA exits
  if (*abort && threadIdx.x == 0) {
    const int issued = ring.issued;
    for (int q = issued > kDwSlots ? issued - kDwSlots : 0; q < issued; ++q)
      mbar_wait(&ring.full[q % kDwSlots], (uint32_t)((q / kDwSlots) & 1));
    raise_device_error(kErrMbarTimeout);
  }
  float sums[K3 + 1];
#pragma unroll
  for (int t = 0; t < K3; ++t) {
    float lo, hi;
    pk_split(acc[t], lo, hi);
    sums[t] = lo + hi;
  }
  {
    float lo, hi;
    pk_split(accb, lo, hi);
    sums[K3] = lo + hi;
  }
  block_sum_to_smem<float, K3 + 1>(sums, red);
  __syncthreads();
  const int tiles = pg.tilesW * pg.tilesH * pg.tilesD;
  const int tile = (td * pg.tilesH + th) * pg.tilesW + tw;
  for (int t = threadIdx.x; t <= K3; t += blockDim.x) {
    float v = 0.f;
    for (int w = 0; w < nwarps; ++w) v += red[w * (K3 + 1) + t];
    part[((size_t)nc * tiles + tile) * (K3 + 1) + t] = v;
  }
}

// ----------------------------------------------------------------------------
// Stride-2 scatter of the down block's input grad (k = 3, 16-bit types):
//   big[2q + e] = bias + sum over a of small[q + a] * w[tap(e, a)]   (per axis;
//   e = 0: a = 0, tap 1; e = 1: a = 0, tap 2, then a = 1, tap 0)
// plus add_even at the all-even positions.  A CTA owns a tile of TWs x THs
// small-grid positions (2*TWs x 2*THs big outputs per plane) and a chunk of big
// plane pairs; the small plane tiles (THs + 1 rows, TWs + 8 columns) stream
// through the TMA ring.  Small plane q finishes big plane 2q (tap kd = 1), gives
// big plane 2q + 1 its first half (kd = 2) and big plane 2q - 1 its second half
// (kd = 0).  Each thread owns 8 small positions of one row, i.e. 16 big columns
// of 2 big rows, with pairs (i, i+4) of small positions; every output sums bias
// first, then its taps in (a_d, a_h, a_w) order and the addend last: the order
// of dw_s2_scatter_kernel, whose results this kernel reproduces bit for bit.
// ----------------------------------------------------------------------------
struct DwS2ScGeom {
  DwS2Geom g;
  int TWs, THs, TDq;  // small-grid tile (columns, rows) and big plane pairs per CTA
  int tilesW, tilesH, tilesD;
  int lw;             // threads along W (8 small columns each)
};

template <typename T>
struct DwS2ScLayout {
  static __host__ __device__ int pitch(int TWs) { return TWs + 8; }
  static __host__ __device__ int rows(int THs) { return THs + 1; }
  static __host__ __device__ size_t tile(const DwS2ScGeom& p) { return (size_t)rows(p.THs) * pitch(p.TWs) * sizeof(T); }
  static __host__ __device__ size_t slot(const DwS2ScGeom& p) { return DwTmaLayout<T>::align128(tile(p)); }
  static __host__ size_t smem(const DwS2ScGeom& p) { return 128 + kDwSlots * slot(p); }
};

// q[m] = (s[m], s[m+4]), m = 0..4, for the 9 small values s[0..8] of one row
// starting at the thread's first column; s[8] comes from the right neighbour
// (lane src_r), or from the tile's last column at the tile edge.
template <typename T>
__device__ __forceinline__ void dw_s2sc_window(const T* __restrict__ rowp, int col, int tws, bool right_edge,
                                               int src_r, uint64_t (&q)[5]) {
  const uint4 c = *reinterpret_cast<const uint4*>(rowp + col);     // s[0..7]
  const uint32_t from_r = __shfl_sync(0xffffffffu, c.x, src_r);    // (s[0], s[1]) of the right neighbour
  const uint32_t er = reinterpret_cast<const unsigned short*>(rowp)[tws];
  const uint32_t s8 = right_edge ? er : (from_r & 0xffffu);
  q[0] = pk_pair(lo_bits<T>(c.x), lo_bits<T>(c.z));
  q[1] = pk_pair(hi_bits<T>(c.x), hi_bits<T>(c.z));
  q[2] = pk_pair(lo_bits<T>(c.y), lo_bits<T>(c.w));
  q[3] = pk_pair(hi_bits<T>(c.y), hi_bits<T>(c.w));
  q[4] = pk_pair(lo_bits<T>(c.z), lo_bits<T>(s8));
}

// big-grid parity e and small offset a along one axis -> tap, or -1 (k = 3)
__host__ __device__ constexpr int s2sc_tap(int e, int a) { return e == 0 ? (a == 0 ? 1 : -1) : (a == 0 ? 2 : 0); }

// STATS: GroupNorm partial statistics (count, mean, M2) of the stored values of
// the grid columns, one per (n, c, tile) in `stats` (the up block's forward,
// whose output is normalised next).
template <typename T, bool ADD, bool STATS>
__global__ void __launch_bounds__(kS2PkThreads, 2)
    dw_s2_scatter_pk_kernel(const __grid_constant__ CUtensorMap mS, const T* __restrict__ wgt,
                            const T* __restrict__ bias, const T* __restrict__ add_even, T* __restrict__ big,
                            GnPartial* __restrict__ stats, DwS2ScGeom pg) {
  constexpr int K = 3;
  constexpr int K3 = 27;
  using L = DwS2ScLayout<T>;
  const DwS2Geom& g = pg.g;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ DwPkRing ring;
  unsigned char* slots = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  const size_t slot_bytes = L::slot(pg);
  const uint32_t tile_bytes = (uint32_t)L::tile(pg);
  const int rsp = L::pitch(pg.TWs);
  const int nwarps = (int)blockDim.x >> 5;

  int bx = blockIdx.x;
  const int tw = bx % pg.tilesW;
  bx /= pg.tilesW;
  const int th = bx % pg.tilesH;
  bx /= pg.tilesH;
  const int td = bx % pg.tilesD;
  const int nc = bx / pg.tilesD;
  const int c = nc % g.C;
  const int qw0 = tw * pg.TWs, qh0 = th * pg.THs, qd0 = td * pg.TDq;
  const int QD = (g.Db + 1) >> 1;
  const int dcount = min(pg.TDq, QD - qd0);
  const int nsteps = dcount + 1;

  auto issue = [&](int q) {
    const int slot = q % kDwSlots;
    mbar_arrive_expect_tx(&ring.full[slot], tile_bytes);
    tma_load_4d(slots + (size_t)slot * slot_bytes, &mS, &ring.full[slot], qw0, qh0, qd0 + q, nc);
  };
  if (threadIdx.x == 0) {
    for (int i = 0; i < kDwSlots; ++i) {
      mbar_init(&ring.full[i], 1);
      ring.released[i] = 0;
    }
    ring.abort = 0;
    fence_mbarrier_init();
    tma_prefetch_map(&mS);
    const int first = min(nsteps, kDwSlots);
    for (int q = 0; q < first; ++q) issue(q);
    ring.issued = first;
  }
  __syncthreads();
  volatile int* abort = &ring.abort;

  const int lane = threadIdx.x & 31;
  const int lw = pg.lw;
  const int wt = threadIdx.x % lw;
  const int r = threadIdx.x / lw;
  const bool active = r < pg.THs;
  const int qh = qh0 + r;
  const int qw = qw0 + 8 * wt;
  // Ws is a multiple of 8 and bw = 2 Ws on this path: a thread's 16 big columns lie in one row
  const bool cols_ok = active && qw < g.Ws;
  const bool row0_ok = cols_ok && 2 * qh < g.Hb, row1_ok = cols_ok && 2 * qh + 1 < g.Hb;
  // a row of lw <= 8 threads lies within one warp: the right neighbour is lane + 1
  const int src_r = wt < lw - 1 ? lane + 1 : lane;
  const bool right_edge = wt == lw - 1;
  // lanes past the tile read row 0 (every lane joins the shuffles) and store nothing
  const int sbase = (active ? r : 0) * rsp;
  const int col = 8 * wt;
  uint64_t wp[K3];
#pragma unroll
  for (int t = 0; t < K3; ++t) {
    const uint32_t wv = __float_as_uint(to_acc<T>(__ldg(wgt + (size_t)c * K3 + t)));
    wp[t] = pk_pair(wv, wv);
  }
  const uint32_t bvb = __float_as_uint(bias != nullptr ? to_acc<T>(bias[c]) : 0.f);
  const uint64_t bv2 = pk_pair(bvb, bvb);
  const size_t bplane = (size_t)g.Hb * g.bw;
  T* out0 = big + (size_t)nc * (size_t)g.bp + (size_t)(2 * qh) * g.bw + 2 * qw;
  // big columns of this thread past the grid's last (the pad columns of a row-pitched grid): zeros
  const int wvalid = g.Wb - 2 * qw;
  const T* add0 = ADD ? add_even + (size_t)nc * g.Ds * ((size_t)g.Hs * g.Ws) + (size_t)qh * g.Ws + qw : nullptr;

  // the odd big plane 2q + 1 between its two halves: [eh][ew][pair]
  uint64_t odd[2][2][4];
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int b2 = 0; b2 < 2; ++b2)
#pragma unroll
      for (int i = 0; i < 4; ++i) odd[a][b2][i] = 0ull;

  // acc[ew][i] += taps of plane tap td (and small offset a_d) for big row parity eh
  auto add_taps = [&](const int td, const int eh, uint64_t (&acc)[2][4], const uint64_t (&q0)[5],
                      const uint64_t (&q1)[5]) {
#pragma unroll
    for (int ah = 0; ah < 2; ++ah) {
      const int th2 = s2sc_tap(eh, ah);
      if (th2 < 0) continue;
#pragma unroll
      for (int ew = 0; ew < 2; ++ew) {
#pragma unroll
        for (int aw = 0; aw < 2; ++aw) {
          const int tw2 = s2sc_tap(ew, aw);
          if (tw2 < 0) continue;
          const uint64_t wv = wp[(td * K + th2) * K + tw2];
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[ew][i] = pk_fma(ah == 0 ? q0[i + aw] : q1[i + aw], wv, acc[ew][i]);
        }
      }
    }
  };
  // shifted sums of the stored values (STATS)
  float st_n = 0.f, st_shift = 0.f;
  float2 st_s1 = make_float2(0.f, 0.f), st_s2 = make_float2(0.f, 0.f);
  // 16 big columns of one row: column 2i + ew is pair (i % 4) of acc[ew], low half for i < 4
  auto store_row = [&](T* dst, const uint64_t (&acc)[2][4]) {
    float lo[8], hi[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      pk_split(acc[0][i], lo[2 * i], hi[2 * i]);
      pk_split(acc[1][i], lo[2 * i + 1], hi[2 * i + 1]);
    }
    if (wvalid < 16) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (e >= wvalid) lo[e] = 0.f;
        if (e + 8 >= wvalid) hi[e] = 0.f;
      }
    }
    const uint4 qlo = pack16<T>(lo), qhi = pack16<T>(hi);
    reinterpret_cast<uint4*>(dst)[0] = qlo;
    reinterpret_cast<uint4*>(dst)[1] = qhi;
    if constexpr (STATS) {
      float rl[8], rh[8];
      unpack16<T>(qlo, rl);
      unpack16<T>(qhi, rh);
      if (st_n == 0.f) st_shift = rl[0];
      const float2 sh = make_float2(-st_shift, -st_shift);
      // columns past the grid enter as the shift (a zero deviation) and are not counted
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float2 dv = __fadd2_rn(make_float2(e < wvalid ? rl[e] : st_shift, e + 8 < wvalid ? rh[e] : st_shift), sh);
        st_s1 = __fadd2_rn(st_s1, dv);
        st_s2 = __ffma2_rn(dv, dv, st_s2);
      }
      st_n += (float)min(16, wvalid);
    }
  };

  auto step = [&](const int s) -> bool {
    const int slot = s % kDwSlots;
    const bool ok = !*abort && mbar_wait(&ring.full[slot], (uint32_t)((s / kDwSlots) & 1));
    if (!__all_sync(0xffffffffu, ok)) {
      *abort = 1;
      return false;
    }
    const T* sp = reinterpret_cast<const T*>(slots + (size_t)slot * slot_bytes) + sbase;
    uint64_t q0[5], q1[5];
    dw_s2sc_window<T>(sp, col, pg.TWs, right_edge, src_r, q0);
    dw_s2sc_window<T>(sp + rsp, col, pg.TWs, right_edge, src_r, q1);
    const int qd = qd0 + s;  // small plane of this step
    // big plane 2qd - 1: its second half (a_d = 1, tap 0), then store
    if (s >= 1 && 2 * qd - 1 < g.Db) {
#pragma unroll
      for (int eh = 0; eh < 2; ++eh) {
        add_taps(0, eh, odd[eh], q0, q1);
        if (eh == 0 ? row0_ok : row1_ok) store_row(out0 + (size_t)(2 * qd - 1) * bplane + (size_t)eh * g.bw, odd[eh]);
      }
    }
    if (s < dcount) {
      // big plane 2qd (a_d = 0, tap 1): complete here
#pragma unroll
      for (int eh = 0; eh < 2; ++eh) {
        uint64_t acc[2][4];
#pragma unroll
        for (int ew = 0; ew < 2; ++ew)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[ew][i] = bv2;
        add_taps(1, eh, acc, q0, q1);
        if constexpr (ADD) {
          if (eh == 0 && cols_ok && qh < g.Hs) {
            float al[8];
            unpack16<T>(__ldg(reinterpret_cast<const uint4*>(add0 + (size_t)qd * ((size_t)g.Hs * g.Ws))), al);
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[0][i] = pk_add(acc[0][i], pk_pair(__float_as_uint(al[i]), __float_as_uint(al[i + 4])));
          }
        }
        if (2 * qd < g.Db && (eh == 0 ? row0_ok : row1_ok))
          store_row(out0 + (size_t)(2 * qd) * bplane + (size_t)eh * g.bw, acc);
      }
      // big plane 2qd + 1: bias and its first half (a_d = 0, tap 2)
#pragma unroll
      for (int eh = 0; eh < 2; ++eh) {
#pragma unroll
        for (int ew = 0; ew < 2; ++ew)
#pragma unroll
          for (int i = 0; i < 4; ++i) odd[eh][ew][i] = bv2;
        add_taps(2, eh, odd[eh], q0, q1);
      }
    }
    // release the slot; the warp that releases it last loads the slot's next plane
    __syncwarp();
    if (lane == 0) {
      int prv;
      asm volatile("atom.acq_rel.cta.shared::cta.add.s32 %0, [%1], 1;"
                   : "=r"(prv)
                   : "r"(smem_u32(&ring.released[slot]))
                   : "memory");
      // the count only grows: the slot's (s / kDwSlots)-th plane is released by nwarps arrivals
      if (prv == (s / kDwSlots + 1) * nwarps - 1) {
        const int q = s + kDwSlots;
        if (q < nsteps) {
          fence_async_smem();
          issue(q);
          atomicAdd(&ring.issued, 1);
        }
      }
    }
    return true;
  };
  for (int s = 0; s < nsteps; ++s)
    if (!step(s)) break;

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
      const int tiles = pg.tilesW * pg.tilesH * pg.tilesD;
      const int tile = (td * pg.tilesH + th) * pg.tilesW + tw;
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

}  // namespace mednext
