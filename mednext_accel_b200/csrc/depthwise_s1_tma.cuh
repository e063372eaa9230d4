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

}  // namespace mednext
