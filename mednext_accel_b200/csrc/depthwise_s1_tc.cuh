// Depthwise Conv3d, k = 5 and 7, stride 1, padding k/2, on the tensor cores
// (sm_100a, 16-bit types): the forward (with GroupNorm partial statistics) and
// the input grad (taps flipped, with the residual addend) of the MedNeXt block.
//
// Along W the convolution is a product with a banded (Toeplitz) matrix: for a
// tile of 16 output columns starting at w0 and the 32 input columns starting
// at w0 - 8,
//   y[row, w0 + n] += sum_k x[row + s(a, b), w0 - 8 + k] * T_ab[k, n],
//   T_ab[k, n] = w[a, b, c] where k = n + 8 - P + c (c = 0 .. K-1, P = K/2), else 0,
// one band matrix per (kd, kh) = (a, b) tap pair, and s(a, b) the row offset of
// that tap pair.  So each (a, b) is one tcgen05.mma of M = 128 rows, N = 16
// columns and K = 32 (two K = 16 steps), accumulated in TMEM in fp32.
//
// Cost model.  Every MMA reads its 4 KB A operand from shared memory for 2,048
// outputs, so an output costs K^2 x 2 x 32 B / 16 = 4 K^2 B of operand reads
// against K^3 FMAs on the FP32 pipes.  Shared memory (128 B/clk/SM) and the FMA
// pipes (128 lanes/clk/SM) then give 0.031 K^2 against 0.0078 K^3 clocks per
// output: the FMA form wins at k = 3 (36 B vs 27 FMAs, measured 165 vs 111 us at
// C32 128^3), this form at k = 5 (100 B vs 125 FMAs) and k = 7 (196 B vs 343).
//
// Rows.  A CTA loads, in one 5-D TMA copy, the input tile of Dp planes x Hp
// rows (Hp = Ht + K - 1, halo rows included) x (TW + 16) columns as 16-byte column
// chunks, laid out [chunk][plane][row] x 16 B: within one chunk the rows
// (plane, row) are consecutive 16-byte lines.  That is the no-swizzle K-major
// operand layout (8-row core matrices 128 B apart, the two K halves of a K = 16
// step one chunk apart), so the operand for tap pair (a, b) is the same tile
// shifted by s(a, b) = a * Hp + b rows: a descriptor start address 16 * s bytes
// further on.  An MMA block covers 128 consecutive row slots (plane, row) of
// the tile; output slot (od, oh) uses input slots (od + a, oh + b), and slots
// with oh >= Ht (the halo rows' positions) compute values that are discarded.
// Dp covers the largest shift past the last block: Dp * Hp >= nblk * 128 +
// (K - 1) * (Hp + 1).
//
// Roles: thread 0 issues the TMA copy; all threads write the K^2 band
// matrices; thread 32 issues the MMAs and commits one barrier per block; the
// four warps then read their 32 TMEM lanes (one output row each), add the bias
// and the addend, round once, store and accumulate statistics.  Every wait is
// bounded: on a timeout the CTA sets the device error word, waits (bounded) for
// its copy and MMAs, frees its TMEM and exits.
//
// Numerics: the products of 16-bit values are exact in fp32 and the tensor core
// sums them in fp32, so the result agrees with the fp32-FMA kernels to a few
// fp32 ulps before the final rounding (it is not their bit pattern).
#pragma once

#include "common.cuh"
#include "depthwise_s1.cuh"

namespace mednext {

constexpr int kDwTcThreads = 128;
constexpr int kDwTcMaxBlk = 4;
constexpr int kDwTcBandBytes = 1024;  // one band matrix: 16 (N) x 32 (K) 16-bit values

struct DwTcGeom {
  int N, C, D, H, W;
  int K;       // kernel size (5 or 7)
  int TW;      // output columns per tile: 16, 32 or 64
  int Ht, Hp;  // output rows per tile; row slots per plane (Ht + K - 1)
  int Dt, Dp;  // output planes per tile; planes loaded
  int nblk;    // 128-slot MMA blocks per tile
  int chunks;  // 16-byte input column chunks per row slot: TW / 8 + 2
  int tilesW, tilesH, tilesD;
  uint32_t tmem_cols;
};

__host__ __device__ inline uint32_t dw_tc_plane_bytes(const DwTcGeom& g) { return (uint32_t)g.Dp * g.Hp * 16u; }
__host__ __device__ inline size_t dw_tc_x_bytes(const DwTcGeom& g) { return (size_t)g.chunks * dw_tc_plane_bytes(g); }
__host__ inline size_t dw_tc_smem(const DwTcGeom& g) {
  return 128 + dw_tc_x_bytes(g) + (size_t)g.K * g.K * kDwTcBandBytes;
}

// Shared-memory matrix descriptor, no swizzle (K-major: 8-row x 16-byte core
// matrices; lbo = bytes between the two K halves, sbo = bytes between 8-row groups).
__device__ __forceinline__ uint64_t make_noswz_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
  return d;                // layout type 0: no swizzle
}

__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, %7}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

template <typename T, int K, bool STATS, bool ADD>
__global__ void __launch_bounds__(kDwTcThreads, 1)
    dw_s1_conv_tc_kernel(const __grid_constant__ CUtensorMap mX, const T* __restrict__ wgt, const T* __restrict__ bias,
                         const T* __restrict__ addend, T* __restrict__ y, GnPartial* __restrict__ stats, DwTcGeom g,
                         int flip) {
  constexpr int P = K / 2, K2 = K * K, K3 = K * K * K;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ uint64_t bar_load;
  __shared__ uint64_t bar_mma[kDwTcMaxBlk];
  __shared__ uint64_t bar_drain;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  __shared__ double red[3 * 32];
  unsigned char* xs = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  unsigned char* bs = xs + dw_tc_x_bytes(g);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t lbo = dw_tc_plane_bytes(g);

  int bx = blockIdx.x;
  const int tw = bx % g.tilesW;
  bx /= g.tilesW;
  const int th = bx % g.tilesH;
  bx /= g.tilesH;
  const int td = bx % g.tilesD;
  const int nc = bx / g.tilesD;
  const int c = nc % g.C;
  const int w0 = tw * g.TW, h0 = th * g.Ht, d0 = td * g.Dt;

  if (warp == 1) {
    tmem_alloc(&tmem_base, g.tmem_cols);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&bar_load, 1);
    for (int b = 0; b < kDwTcMaxBlk; ++b) mbar_init(&bar_mma[b], 1);
    mbar_init(&bar_drain, 1);
    abort_flag = 0;
    fence_mbarrier_init();
    mbar_arrive_expect_tx(&bar_load, (uint32_t)dw_tc_x_bytes(g));
    tma_load_5d(xs, &mX, &bar_load, 0, h0 - P, d0 - P, w0 / 8 - 1, nc);
  }
  // the K^2 band matrices, K-major without swizzle: (n, k) at (k / 8) * 256 + n * 16 + (k % 8) * 2
  for (int off = tid * 16; off < K2 * kDwTcBandBytes; off += kDwTcThreads * 16)
    *reinterpret_cast<uint4*>(bs + off) = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();
  for (int e = tid; e < K2 * 16 * K; e += kDwTcThreads) {
    const int ab = e / (16 * K), n = (e / K) % 16, cc = e % K;
    const int t = ab * K + cc;  // tap (a, b, cc) in (kd, kh, kw) order
    const T v = wgt[(size_t)c * K3 + (flip ? K3 - 1 - t : t)];
    const int k = n + 8 - P + cc;
    *reinterpret_cast<T*>(bs + ab * kDwTcBandBytes + (k >> 3) * 256 + n * 16 + (k & 7) * 2) = v;
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  volatile int* abort = &abort_flag;

  const int wtiles = g.TW / 16;
  if (tid == 32) {
    // ------------------------------------------------ MMA issuer
    const bool ok = mbar_wait(&bar_load, 0);
    if (!ok) {
      *abort = 1;
      for (int b = 0; b < g.nblk; ++b) mbar_arrive(&bar_mma[b]);
    } else {
      tc_fence_after();
      const uint32_t idesc = make_idesc_f16(128, 16, std::is_same<T, __nv_bfloat16>::value, false, false);
      const uint32_t xa = smem_u32(xs), ba = smem_u32(bs);
      for (int blk = 0; blk < g.nblk; ++blk) {
        for (int t = 0; t < wtiles; ++t) {
          const uint32_t d_tmem = tmem + (uint32_t)(blk * g.TW + t * 16);
          for (int ab = 0; ab < K2; ++ab) {
            const int s = (ab / K) * g.Hp + (ab % K);
#pragma unroll
            for (int ks = 0; ks < 2; ++ks) {
              const uint64_t ad = make_noswz_desc(xa + (uint32_t)(2 * t + 2 * ks) * lbo + (uint32_t)(blk * 128 + s) * 16u,
                                                  lbo, 128);
              const uint64_t bd = make_noswz_desc(ba + (uint32_t)ab * kDwTcBandBytes + (uint32_t)ks * 512u, 256, 128);
              mma_f16_ss(d_tmem, ad, bd, idesc, (ab > 0 || ks > 0) ? 1u : 0u);
            }
          }
        }
        mma_commit(&bar_mma[blk]);
      }
    }
  }
  __syncwarp();

  // ------------------------------------------------ epilogue: one TMEM lane (row slot) per thread
  const float bv = bias != nullptr ? to_acc<T>(bias[c]) : 0.f;
  float st_n = 0.f, st_shift = 0.f;
  float2 st_s1 = make_float2(0.f, 0.f), st_s2 = make_float2(0.f, 0.f);
  const size_t plane = (size_t)g.H * g.W;
  for (int blk = 0; blk < g.nblk; ++blk) {
    const bool okw = !*abort && mbar_wait(&bar_mma[blk], 0);
    if (!__all_sync(0xffffffffu, okw) || *abort) {
      *abort = 1;
      break;
    }
    tc_fence_after();
    const int slot = blk * 128 + warp * 32 + lane;
    const int od = slot / g.Hp, oh = slot - od * g.Hp;
    const int d = d0 + od, h = h0 + oh;
    const bool valid = oh < g.Ht && od < g.Dt && d < g.D && h < g.H;
    const size_t row = ((size_t)nc * g.D + d) * plane + (size_t)h * g.W + w0;
    for (int t = 0; t < wtiles; ++t) {
      uint32_t r[16];
      tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(blk * g.TW + t * 16), r);
      tmem_ld_wait();
      if (valid) {
        float lo[8], hi[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          lo[i] = __uint_as_float(r[i]) + bv;
          hi[i] = __uint_as_float(r[i + 8]) + bv;
        }
        if constexpr (ADD) {
          float al[8], ah[8];
          const uint4* ap = reinterpret_cast<const uint4*>(addend + row + t * 16);
          unpack16<T>(__ldg(ap), al);
          unpack16<T>(__ldg(ap + 1), ah);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            lo[i] += al[i];
            hi[i] += ah[i];
          }
        }
        const uint4 qlo = pack16<T>(lo), qhi = pack16<T>(hi);
        uint4* dst = reinterpret_cast<uint4*>(y + row + t * 16);
        dst[0] = qlo;
        dst[1] = qhi;
        if constexpr (STATS) {
          float rl[8], rh[8];
          unpack16<T>(qlo, rl);
          unpack16<T>(qhi, rh);
          if (st_n == 0.f) st_shift = rl[0];
          const float2 sh = make_float2(-st_shift, -st_shift);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float2 dv = __fadd2_rn(make_float2(rl[i], rh[i]), sh);
            st_s1 = __fadd2_rn(st_s1, dv);
            st_s2 = __ffma2_rn(dv, dv, st_s2);
          }
          st_n += 16.f;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*abort) {
    // the copy and the issuer's MMAs may still be in flight: wait (bounded) for
    // both before TMEM is freed and the CTA exits
    if (tid == 32) {
      if (mbar_wait(&bar_load, 0)) {
        mma_commit(&bar_drain);
        mbar_wait(&bar_drain, 0);
      }
    }
    if (tid == 0) raise_device_error(kErrMbarTimeout);
    __syncthreads();
  }
  if (warp == 1) tmem_dealloc(tmem, g.tmem_cols);
  if constexpr (STATS) {
    double n = (double)st_n, mean = 0.0, m2 = 0.0;
    if (st_n > 0.f) {
      const double s1 = (double)st_s1.x + (double)st_s1.y, s2 = (double)st_s2.x + (double)st_s2.y;
      mean = (double)st_shift + s1 / n;
      m2 = fmax(s2 - s1 * s1 / n, 0.0);
    }
    block_merge_stats(n, mean, m2, red);
    if (tid == 0) {
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

}  // namespace mednext
