// Persistent, warp-specialized tcgen05 pointwise GEMMs fed by TMA.
//
// Forward / input-grad (voxel-M): y[s, j, v] = epi( sum_k W[j, k] * pro(a[s, k, v]) )
//   warp 0      TMA producer: per (tile, k-stage) one 64x64 box per 64 voxels of A
//               (MN-major, 128B swizzle) and one 64xBN box of W (K-major, 128B
//               swizzle) into an S-stage ring; per tile the epilogue operands
//               (aux / residual tiles, no swizzle) into an E-stage ring.
//   warp 1      TMEM owner and MMA issuer (one lane): tcgen05.mma M=128 N=BN K=16,
//               accumulators double-buffered in TMEM so the epilogue of tile i
//               overlaps the MMAs of tile i+1.
//   warp 3      (prologue output requested) TMA-stores each transformed A stage to
//               pro_out and releases the stage once the store has read it.
//   warps 4-11  prologue (only when one is requested): GroupNorm apply or GELU on
//               the staged A tile, in place, then release it to the MMA.
//   epilogue    warps 12-19 with a prologue, warps 4-19 without: tcgen05.ld of
//               16-column accumulator chunks, bias / GELU' / residual / GroupNorm-
//               backward sums, staged in shared memory and written by TMA stores.
//               The epilogue flags are a template parameter, so the per-element
//               loop is straight-line code.
// Weight grad (voxel-K): producer, MMA, 4 prologue and 4 epilogue warps; the
// reduction runs over 64-voxel chunks of a split-K range, the prologue warps also
// accumulate the bias grad rows.
//
// All waits are bounded (common.cuh); a timed-out wait raises the device error
// word, sets the CTA abort flag and every role drains out.
#pragma once

#include <cuda.h>

#include "pointwise.cuh"

namespace mednext {

// forward kernel: warp 0 producer, warp 1 MMA, warps 4-11 prologue (when requested),
// the remaining warps up to 19 epilogue
constexpr int kFwdProWarp0 = 4;
constexpr int kFwdThreads = 640;
constexpr int kFwdProThreads = 256;
constexpr int kPwCW = 16;          // accumulator columns per epilogue chunk
constexpr int kEpiRuntime = -1;    // EPI template value: read the flags from the arguments
// EPI bit (internal, with GELU_GRAD or GN_BWD_STATS): the input-grad GEMM also
// computes the weight grad of the GEMM it differentiates.  The epilogue writes
// g = GELU(aux) (compress GEMM) or GroupNorm(aux) (expand GEMM) into a K-major
// shared-memory tile (rows = this GEMM's output channels, plus a row of ones),
// and the MMA warp accumulates D^T[row, k] += g[row, v] * a[k, v] over the CTA's
// tiles with the A tile (the incoming grad) still in the ring, so neither g nor a
// second read of the grad and aux reaches HBM.  The ones row of D^T is
// sum_v a[k, v], the bias grad.
constexpr int kEpiFusedWgrad = 16;
constexpr int kFwLag = 2;          // the weight-grad MMAs of tile i run after the input-grad MMAs of tile i+2
// EPI bit (internal, with PRO = GroupNorm and BIAS): the block's whole expansion,
// y = Wp @ GELU(We @ GroupNorm(t) + be) + bp (+ residual), in one kernel.  The
// first GEMM's epilogue writes u (saved for the backward) and GELU(u) into a
// shared-memory g tile, whose bytes are the MN-major A operand of the second GEMM
// (M = voxels, K = H); its resident weight Wp is the second B operand and its
// accumulators the second TMEM region.  The same epilogue group then adds bp and
// the residual and stores y.  u is never read back from HBM.
constexpr int kEpiMlp = 32;
constexpr int kFwGBytes = 32768;   // one g tile: two 64-voxel K-major boxes of 128 rows
// EPI bit (internal, fragment epilogue only): the epilogue also writes GELU of its
// output, g = GELU(y) with y rounded as stored, through the second output map (mY2):
// the expand GEMM hands the compress GEMM its activated input, so the compress GEMM
// needs no prologue and the compress weight grad can read g instead of recomputing it.
constexpr int kEpiGeluOut = 128;
// Warp roles after the producer / MMA / aux-producer / prologue-store warps 0-3:
// prologue warps 4 .. warp0 - 1 (8 of them, or 4 when the epilogue carries the
// GELU output and the prologue is the cheap GroupNorm apply), epilogue warps up to 19.
template <int PRO, int EPI>
struct FwdEpi {
  static constexpr bool gelu_out = EPI >= 0 && (EPI & kEpiGeluOut) != 0;
  static constexpr int warp0 = PRO == MEDNEXT_PRO_NONE ? 4 : (gelu_out ? 8 : 12);
  static constexpr int warps = kFwdThreads / 32 - warp0;
  static constexpr int threads = warps * 32;
  static constexpr int pro_threads = (warp0 - 4) * 32;
  // staging buffers per epilogue warp: y, and g with the GELU output, double-buffered
  static constexpr int stg_bufs = gelu_out ? 4 : 2;
};
constexpr int kMaxStages = 8;
// Prologue-output stores kept in flight by warp 3 (< ring stages, checked on the host).
#ifndef MEDNEXT_PRO_STORE_LAG
#define MEDNEXT_PRO_STORE_LAG 2
#endif
constexpr int kProStoreLag = MEDNEXT_PRO_STORE_LAG;
constexpr int kMaxEStages = 4;
constexpr int kMaxAcc = 4;  // TMEM accumulator buffers between the MMA and the epilogue

struct PwTmaCfg {
  int stages;       // A/B ring depth
  int estages;      // aux/residual ring depth
  int kstages;      // K stages per tile (forward) = ceil(cin / 64)
  int total_tiles;  // forward: S * ntiles * mtiles; wgrad: work units
  int aux_bytes;    // bytes of one aux tile (0 if unused)
  int res_bytes;    // bytes of one residual tile (0 if unused)
  int b_bytes;      // bytes of one W stage (BN * 128)
  int nacc;         // TMEM accumulator buffers (2 or 4)
  int tgroups;      // epilogue warp groups on alternate tiles (1 or 2)
  int a_rows;       // channel rows per A box: min(64, roundup16(cin)); the MMA reads no further
  int w_res;        // 1: the whole W operand (kstages boxes) is loaded once and stays in shared memory
  int tmem_cols;    // TMEM columns allocated (a power of two >= nacc x accumulator columns)
  int a_slot;       // bytes of one A stage: two boxes of a_rows x 128 B
  int ks2;          // MLP: K boxes of the resident second weight (ceil(H / 64)), else 0
  int b2_bytes;     // MLP: one box of the second weight, BN2 x 128 B
  int bn2;          // MLP: second GEMM's N (output channels rounded to 16)
  int d2_col;       // MLP: TMEM column of the second GEMM's two accumulators
  int d2_stride;    // MLP: TMEM columns between them (a power of two >= bn2)
  int pro_store;    // 1: warp 3 writes every transformed A stage to pro_out (tensor map mP)
};

struct PwTmaSmem {
  uint64_t full[kMaxStages];
  uint64_t ready[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t tfull[kMaxAcc];
  uint64_t tempty[kMaxAcc];
  uint64_t efull[kMaxEStages];
  uint64_t eempty[kMaxEStages];
  uint64_t drain;  // final tcgen05.commit: every MMA of the CTA has completed
  uint64_t wfull;  // resident W operand landed
  uint64_t gready[2];  // fused weight grad: g tile of epilogue group b written
  uint64_t gempty[2];  // fused weight grad: its MMAs have read g tile b (and the dy stage)
  uint64_t wdone;      // fused weight grad: every MMA into the weight-grad accumulator done
  uint64_t d2full[2];  // MLP: second-GEMM accumulator of epilogue group b complete
  uint64_t uready[2];  // MLP: u written into g tile b (the prologue warps then apply GELU in place)
  uint32_t tmem_base;
  int abort;
};

// Exit discipline: nothing asynchronous may still target the CTA's shared
// memory or TMEM when it exits.  On the normal path every fill and every MMA has
// been waited for by its consumer.  After an abort (a bounded wait gave up), the
// roles meet at a CTA barrier, then each producer waits, bounded, for the last
// fill of each ring slot it issued and the MMA issuer commits to `drain` and
// waits for it, before TMEM is freed.
__device__ __forceinline__ void drain_ring(uint64_t* full, int slots, long long issued) {
  for (long long q = issued > slots ? issued - slots : 0; q < issued; ++q)
    mbar_wait(&full[q % slots], (uint32_t)((q / slots) & 1));
}
__device__ __forceinline__ void drain_mma(uint64_t* drain) {
  mma_commit(drain);
  mbar_wait(drain, 0);
}

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (*abort) return false;
  if (!mbar_wait(bar, parity)) {
    *abort = 1;
    return false;
  }
  return true;
}

__host__ __device__ __forceinline__ uint32_t tmem_cols_for(int bn) {
  return bn <= 32 ? 32u : (bn <= 64 ? 64u : (bn <= 128 ? 128u : 256u));
}

// Column sums of a 32 (lanes) x 16 (v[]) block: five butterfly exchange steps
// that halve the columns each lane keeps, 16 shuffles in all.  On return lane L
// holds the sum over all 32 lanes of column (L >> 1); the order of the additions
// is fixed, so the result is deterministic.
__device__ __forceinline__ float warp_transpose_sum16(const float (&v)[16], int lane) {
  float w8[8], w4[4], w2[2];
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4, b1 = lane & 2;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    w8[i] = (b4 ? v[i + 8] : v[i]) + __shfl_xor_sync(0xffffffffu, b4 ? v[i] : v[i + 8], 16);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    w4[i] = (b3 ? w8[i + 4] : w8[i]) + __shfl_xor_sync(0xffffffffu, b3 ? w8[i] : w8[i + 4], 8);
#pragma unroll
  for (int i = 0; i < 2; ++i)
    w2[i] = (b2 ? w4[i + 2] : w4[i]) + __shfl_xor_sync(0xffffffffu, b2 ? w4[i] : w4[i + 2], 4);
  const float w1 = (b1 ? w2[1] : w2[0]) + __shfl_xor_sync(0xffffffffu, b1 ? w2[0] : w2[1], 2);
  return w1 + __shfl_xor_sync(0xffffffffu, w1, 1);
}

// ---------------------------------------------------------------- forward / dgrad
template <typename TA, typename TY, int PRO, int EPI>
__global__ void __launch_bounds__(kFwdThreads, 1)
    pw_tma_fwd_kernel(const __grid_constant__ CUtensorMap mA, const __grid_constant__ CUtensorMap mB,
                      const __grid_constant__ CUtensorMap mAux, const __grid_constant__ CUtensorMap mRes,
                      const __grid_constant__ CUtensorMap mY, const __grid_constant__ CUtensorMap mP,
                      const __grid_constant__ CUtensorMap mB2, const __grid_constant__ CUtensorMap mY2, PwFwdArgs p,
                      PwTmaCfg cfg) {
  extern __shared__ uint8_t smem_dyn[];
  __shared__ PwTmaSmem sh;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int BN = p.BN;
  const int S = cfg.stages, E = cfg.estages, KS = cfg.kstages;
  const bool has_aux = cfg.aux_bytes > 0, has_res = cfg.res_bytes > 0;

  const uint32_t base_u32 = smem_u32(smem_dyn);
  uint8_t* sbase = smem_dyn + (((base_u32 + 1023u) & ~1023u) - base_u32);
  // W: one box per ring stage, or (w_res) all KS boxes resident for the whole kernel
  const bool w_res = cfg.w_res != 0;
  uint8_t* ringA = sbase;                                 // S x a_slot
  // an A stage is two 64-voxel boxes of a_rows channel rows, a_slot = 256 * a_rows bytes
  const int AS = cfg.a_slot, AH = cfg.a_slot / 2;
  uint8_t* ringB = ringA + (size_t)S * AS;                // (w_res ? KS : S) x b_bytes
  uint8_t* ringB2 = ringB + (size_t)(w_res ? KS : S) * cfg.b_bytes;    // MLP: ks2 x b2_bytes (resident Wp)
  uint8_t* ringAux = ringB2 + (size_t)cfg.ks2 * cfg.b2_bytes;          // E x aux_bytes
  uint8_t* ringRes = ringAux + (size_t)E * cfg.aux_bytes; // E x res_bytes
  uint8_t* ringStg = ringRes + (size_t)E * cfg.res_bytes;  // epilogue warps x 2 x (16 x 32) TY
  constexpr int kStgBytes = 32 * kPwCW * (int)sizeof(TY);
  constexpr int kEpiWarp0 = FwdEpi<PRO, EPI>::warp0;
  constexpr int kEpiThreads = FwdEpi<PRO, EPI>::threads;
  constexpr int kProThreads = FwdEpi<PRO, EPI>::pro_threads > 0 ? FwdEpi<PRO, EPI>::pro_threads : kFwdProThreads;
  constexpr bool FW = EPI >= 0 && (EPI & kEpiFusedWgrad) != 0;
  constexpr bool FW_GELU = FW && (EPI & MEDNEXT_EPI_GELU_GRAD) != 0;      // g = GELU(aux)
  constexpr bool FW_GN = FW && (EPI & MEDNEXT_EPI_GN_BWD_STATS) != 0;     // g = GroupNorm(aux)
  static_assert(!(FW_GELU && FW_GN), "one fused weight-grad operand");
  constexpr bool MLP = EPI >= 0 && (EPI & kEpiMlp) != 0;
  static_assert(!(MLP && FW), "one fused second GEMM");
  constexpr bool GOUT = FwdEpi<PRO, EPI>::gelu_out;
  static_assert(!GOUT || (!MLP && !FW && sizeof(TY) == 2), "the GELU output rides on the plain fragment epilogue");
  // 16-bit outputs take the fragment epilogue (swizzled operand and staging tiles);
  // float32 outputs the one-voxel-per-lane epilogue (unswizzled tiles)
  constexpr bool kFrag = sizeof(TY) == 2;
  // fused weight grad: two g tiles (one per epilogue group) after the staging buffers
  uint8_t* gbuf = ringStg + (size_t)FwdEpi<PRO, EPI>::warps * FwdEpi<PRO, EPI>::stg_bufs * kStgBytes;
  gbuf += ((1024u - (smem_u32(gbuf) & 1023u)) & 1023u);

  const uint32_t ncols = tmem_cols_for(BN);
  if (warp == 1) {
    tmem_alloc(&sh.tmem_base, (uint32_t)cfg.tmem_cols);
    tmem_relinquish();
  }
  if constexpr (FW) {
    // rows past the H channels stay zero, row H holds ones (the bias grad)
    for (int off = tid * 16; off < 2 * kFwGBytes; off += kFwdThreads * 16)
      *reinterpret_cast<uint4*>(gbuf + off) = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();
    if (tid < 2 * 2 * 8) {
      const int b = tid >> 4, box = (tid >> 3) & 1, c = tid & 7;
      float one[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) one[k] = 1.0f;
      *reinterpret_cast<uint4*>(gbuf + b * kFwGBytes + box * 16384 + sw128_kmajor_off(p.cout, c)) = pack16<TA>(one);
    }
    fence_async_smem();
  }
  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&sh.full[i], 1);
      mbar_init(&sh.ready[i], kProThreads);
      // a stage is free again after its MMAs and, with a prologue output, its store
      mbar_init(&sh.empty[i], cfg.pro_store ? 2 : 1);
    }
    for (int i = 0; i < cfg.nacc; ++i) {
      mbar_init(&sh.tfull[i], 1);
      mbar_init(&sh.tempty[i], kEpiThreads / cfg.tgroups);
    }
    for (int i = 0; i < E; ++i) {
      mbar_init(&sh.efull[i], 1);
      mbar_init(&sh.eempty[i], kEpiThreads / cfg.tgroups);
    }
    mbar_init(&sh.drain, 1);
    mbar_init(&sh.wfull, 1);
    for (int b = 0; b < 2; ++b) {
      // the fused expansion's g tile is finished (GELU applied) by the prologue warps
      mbar_init(&sh.gready[b], MLP ? kProThreads : kEpiThreads / 2);
      mbar_init(&sh.gempty[b], 1);
      mbar_init(&sh.uready[b], kEpiThreads / 2);
    }
    mbar_init(&sh.wdone, 1);
    for (int b = 0; b < 2; ++b) mbar_init(&sh.d2full[b], 1);
    sh.abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&mA);
    tma_prefetch_map(&mB);
    if (has_aux) tma_prefetch_map(&mAux);
    if (has_res) tma_prefetch_map(&mRes);
    tma_prefetch_map(&mY);
    if (cfg.pro_store) tma_prefetch_map(&mP);
    if (cfg.ks2 > 0) {
      tma_prefetch_map(&mB2);
      tma_prefetch_map(&mY2);
    }
    if constexpr (GOUT) tma_prefetch_map(&mY2);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  volatile int* abort = &sh.abort;
  const int ntile_local = (cfg.total_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  long long a_issued = 0, aux_issued = 0;  // TMA fills issued by the two producers
  bool w_issued = false;

  auto decode = [&](int t, int& s, int& j0, long long& v0, int& mt) {
    mt = t % p.mtiles;
    const int rest = t / p.mtiles;
    j0 = (rest % p.ntiles) * BN;
    s = rest / p.ntiles;
    v0 = (long long)mt * kPwBM;
  };

  if (warp == 2) {
    // ------------------------------------------------ TMA producer of the epilogue operands
    if (lane == 0 && (has_aux || has_res)) {
      long long issued = 0;
      for (int i = 0; i < ntile_local && !*abort; ++i) {
        int s, j0, mt;
        long long v0;
        decode((int)blockIdx.x + i * (int)gridDim.x, s, j0, v0, mt);
        {
          const int e = i % E, re = i / E;
          if (re > 0 && !wait_or_abort(&sh.eempty[e], (re - 1) & 1, abort)) break;
          mbar_arrive_expect_tx(&sh.efull[e], (uint32_t)(cfg.aux_bytes + cfg.res_bytes));
          if (has_aux) {
            uint8_t* d = ringAux + (size_t)e * cfg.aux_bytes;
            tma_load_3d(d, &mAux, &sh.efull[e], (int)v0, j0, s);
            tma_load_3d(d + cfg.aux_bytes / 2, &mAux, &sh.efull[e], (int)v0 + 64, j0, s);
          }
          if (has_res) {
            uint8_t* d = ringRes + (size_t)e * cfg.res_bytes;
            tma_load_3d(d, &mRes, &sh.efull[e], (int)v0, j0, s);
            tma_load_3d(d + cfg.res_bytes / 2, &mRes, &sh.efull[e], (int)v0 + 64, j0, s);
          }
          ++issued;
        }
      }
      aux_issued = issued;
    }
  } else if (warp == 0) {
    // ------------------------------------------------ TMA producer of the A / W stages
    if (lane == 0) {
      if (w_res && ntile_local > 0) {
        // a single N tile (j0 = 0): every tile of the CTA multiplies by the same W
        mbar_arrive_expect_tx(&sh.wfull, (uint32_t)(KS * cfg.b_bytes + cfg.ks2 * cfg.b2_bytes));
        for (int kk = 0; kk < KS; ++kk)
          tma_load_2d(ringB + (size_t)kk * cfg.b_bytes, &mB, &sh.wfull, kk * kPwBK, 0);
        // MLP: the second GEMM's weight, resident too
        for (int k2 = 0; k2 < cfg.ks2; ++k2)
          tma_load_2d(ringB2 + (size_t)k2 * cfg.b2_bytes, &mB2, &sh.wfull, k2 * kPwBK, 0);
        w_issued = true;
      }
      const uint32_t stage_tx = (uint32_t)(2 * 128 * cfg.a_rows + (w_res ? 0 : cfg.b_bytes));
      long long issued = 0;
      for (int i = 0; i < ntile_local && !*abort; ++i) {
        int s, j0, mt;
        long long v0;
        decode((int)blockIdx.x + i * (int)gridDim.x, s, j0, v0, mt);
        for (int kk = 0; kk < KS; ++kk) {
          const int q = i * KS + kk;
          const int st = q % S, r = q / S;
          if (r > 0 && !wait_or_abort(&sh.empty[st], (r - 1) & 1, abort)) break;
          mbar_arrive_expect_tx(&sh.full[st], stage_tx);
          uint8_t* a = ringA + (size_t)st * AS;
          tma_load_3d(a, &mA, &sh.full[st], (int)v0, kk * kPwBK, s);
          tma_load_3d(a + AH, &mA, &sh.full[st], (int)v0 + 64, kk * kPwBK, s);
          if (!w_res) tma_load_2d(ringB + (size_t)st * cfg.b_bytes, &mB, &sh.full[st], kk * kPwBK, j0);
          ++issued;
        }
      }
      a_issued = issued;
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f16(kPwBM, BN, std::is_same<TA, __nv_bfloat16>::value, true, false);
      // fused weight grad: D^T[h, c] (M = 128 rows of g, N = cin columns of dy), both K-major
      const uint32_t widesc = make_idesc_f16(kPwBM, p.cin, std::is_same<TA, __nv_bfloat16>::value, false, false);
      const uint32_t wacc = tmem + (uint32_t)cfg.nacc * ncols;
      bool wfirst = true;
      // MLP: the second GEMM of tile w, y2[v, j] = sum_h g[h, v] * Wp[j, h]: A = the g tile of
      // epilogue group w & 1 (MN-major, the two 64-voxel boxes 16 KB apart), B = resident Wp
      const uint32_t idesc2 = make_idesc_f16(kPwBM, cfg.bn2, std::is_same<TA, __nv_bfloat16>::value, true, false);
      auto gemm2_tile = [&](int w) -> bool {
        const int gb = w & 1;
        if (!wait_or_abort(&sh.gready[gb], (uint32_t)((w >> 1) & 1), abort)) return false;
        tc_fence_after();
        const uint32_t g_addr = smem_u32(gbuf + gb * kFwGBytes);
        const uint32_t b2_addr = smem_u32(ringB2);
        const uint32_t d2 = tmem + (uint32_t)cfg.d2_col + (uint32_t)(gb * cfg.d2_stride);
        const int ksteps = p.cout / 16;  // K = H, a multiple of 16
        for (int ks = 0; ks < ksteps; ++ks) {
          const uint64_t ad = make_sw128_desc(g_addr + ks * 2048, 16384, 1024);
          const uint64_t bd = make_sw128_desc(b2_addr + (ks >> 2) * cfg.b2_bytes + (ks & 3) * 32, 16, 1024);
          mma_f16_ss(d2, ad, bd, idesc2, ks > 0 ? 1u : 0u);
        }
        mma_commit(&sh.gempty[gb]);
        mma_commit(&sh.d2full[gb]);
        return true;
      };
      // the weight-grad MMAs of tile w (KS == 1): g tile w & 1 times the dy stage of tile w,
      // then release both
      auto wgrad_tile = [&](int w) -> bool {
        const int gb = w & 1;
        if (!wait_or_abort(&sh.gready[gb], (uint32_t)((w >> 1) & 1), abort)) return false;
        tc_fence_after();
        const int st = w % S;
        const uint32_t g_addr = smem_u32(gbuf + gb * kFwGBytes);
        const uint32_t d_addr = smem_u32(ringA + (size_t)st * AS);
#pragma unroll
        for (int box = 0; box < 2; ++box) {
#pragma unroll
          for (int ks = 0; ks < kPwBK / 16; ++ks) {
            const uint64_t ad = make_sw128_desc(g_addr + box * 16384 + ks * 32, 16, 1024);
            const uint64_t bd = make_sw128_desc(d_addr + box * AH + ks * 32, 16, 1024);
            mma_f16_ss(wacc, ad, bd, widesc, wfirst ? 0u : 1u);
            wfirst = false;
          }
        }
        mma_commit(&sh.gempty[gb]);
        mma_commit(&sh.empty[st]);
        return true;
      };
      if (w_res && ntile_local > 0) wait_or_abort(&sh.wfull, 0, abort);
      bool ok = true;
      for (int i = 0; i < ntile_local && !*abort; ++i) {
        const int acc = i % cfg.nacc, ra = i / cfg.nacc;
        if (ra > 0 && !wait_or_abort(&sh.tempty[acc], (ra - 1) & 1, abort)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)acc * ncols;
        for (int kk = 0; kk < KS; ++kk) {
          const int q = i * KS + kk;
          const int st = q % S, r = q / S;
          uint64_t* bar = PRO != MEDNEXT_PRO_NONE ? &sh.ready[st] : &sh.full[st];
          if (!wait_or_abort(bar, r & 1, abort)) break;
          tc_fence_after();
          const uint32_t a_addr = smem_u32(ringA + (size_t)st * AS);
          const uint32_t b_addr = smem_u32(ringB + (size_t)(w_res ? kk : st) * cfg.b_bytes);
          const int ksteps = min(kPwBK, p.cin - kk * kPwBK + 15) / 16;
          for (int ks = 0; ks < ksteps; ++ks) {
            const uint64_t ad = make_sw128_desc(a_addr + ks * 2048, (uint32_t)AH, 1024);
            const uint64_t bd = make_sw128_desc(b_addr + ks * 32, 16, 1024);
            mma_f16_ss(d_tmem, ad, bd, idesc, (kk > 0 || ks > 0) ? 1u : 0u);
          }
          // fused weight grad: the stage is released after its weight-grad MMAs
          if constexpr (!FW) mma_commit(&sh.empty[st]);
        }
        mma_commit(&sh.tfull[acc]);
        if constexpr (FW) {
          if (i >= kFwLag && !wgrad_tile(i - kFwLag)) {
            ok = false;
            break;
          }
        }
        if constexpr (MLP) {
          if (i >= kFwLag && !gemm2_tile(i - kFwLag)) {
            ok = false;
            break;
          }
        }
      }
      if constexpr (FW) {
        for (int w = max(0, ntile_local - kFwLag); ok && !*abort && w < ntile_local; ++w) ok = wgrad_tile(w);
        if (ok && !*abort) mma_commit(&sh.wdone);
      }
      if constexpr (MLP) {
        for (int w = max(0, ntile_local - kFwLag); ok && !*abort && w < ntile_local; ++w) ok = gemm2_tile(w);
      }
    }
  } else if (warp == 3) {
    // ------------------------------------------------ prologue output store
    if constexpr (PRO != MEDNEXT_PRO_NONE) {
      if (cfg.pro_store && lane == 0) {
        long long q = 0;  // stages stored
        for (int i = 0; i < ntile_local && !*abort; ++i) {
          int s, j0, mt;
          long long v0;
          decode((int)blockIdx.x + i * (int)gridDim.x, s, j0, v0, mt);
          for (int kk = 0; kk < KS; ++kk) {
            const int st = (int)(q % S), r = (int)(q / S);
            if (!wait_or_abort(&sh.ready[st], r & 1, abort)) break;
            uint8_t* a = ringA + (size_t)st * AS;
            tma_store_3d(&mP, a, (int)v0, kk * kPwBK, s);
            tma_store_3d(&mP, a + AH, (int)v0 + 64, kk * kPwBK, s);
            bulk_commit();
            // kProStoreLag stores in flight; a stage is released once its store has read it
            bulk_wait_read<kProStoreLag>();
            if (q >= kProStoreLag) mbar_arrive(&sh.empty[(q - kProStoreLag) % S]);
            ++q;
          }
        }
        bulk_wait_read<0>();
        for (long long k = q > kProStoreLag ? q - kProStoreLag : 0; k < q; ++k) mbar_arrive(&sh.empty[k % S]);
        bulk_wait_all();
      }
    }
  } else if (warp >= kFwdProWarp0 && warp < kEpiWarp0) {
    // ------------------------------------------------ prologue transform (in place)
    if constexpr (PRO != MEDNEXT_PRO_NONE) {
      const int t = tid - kFwdProWarp0 * 32;  // 0 .. kProThreads - 1
      const int mch = t & 15;                 // 16 chunks of 8 voxels (two 64-voxel boxes)
      const int kr = t >> 4;                  // rows kr, kr + kRowStep, ... (the same swizzle row)
      constexpr int kRowStep = kProThreads / 16;
      // MLP: GELU in place over the u that epilogue group w & 1 wrote into its g tile (two
      // 64-voxel boxes of H rows, 16-byte chunks; elementwise, so the swizzle is irrelevant)
      auto gelu_tile = [&](int w) -> bool {
        const int gb = w & 1;
        if (!wait_or_abort(&sh.uready[gb], (uint32_t)((w >> 1) & 1), abort)) return false;
        uint8_t* gt = gbuf + gb * kFwGBytes;
        const int per_box = p.cout * 8;
        for (int item = t; item < 2 * per_box; item += kProThreads) {
          const int box = item / per_box, rem = item - box * per_box;
          uint4* chunk = reinterpret_cast<uint4*>(gt + box * 16384 + rem * 16);
          float v[8];
          unpack16<TA>(*chunk, v);
          pw_prologue<MEDNEXT_PRO_GELU>(v, 0.f, 0.f);
          *chunk = pack16<TA>(v);
        }
        fence_async_smem();
        mbar_arrive(&sh.gready[gb]);
        return true;
      };
      for (int i = 0; i < ntile_local && !*abort; ++i) {
        int s, j0, mt;
        long long v0;
        decode((int)blockIdx.x + i * (int)gridDim.x, s, j0, v0, mt);
        for (int kk = 0; kk < KS; ++kk) {
          const int q = i * KS + kk;
          const int st = q % S, r = q / S;
          if (!wait_or_abort(&sh.full[st], r & 1, abort)) break;
          uint8_t* a = ringA + (size_t)st * AS + (mch >> 3) * AH;
#pragma unroll
          for (int ii = 0; ii < kPwBK / kRowStep; ++ii) {
            const int kl = kr + kRowStep * ii;
            if (kl >= cfg.a_rows) break;  // rows the TMA box does not cover are never read
            const int k = kk * kPwBK + kl;
            uint4* chunk = reinterpret_cast<uint4*>(a + kl * 128 + ((((mch & 7) ^ (kl & 7))) << 4));
            float v[8];
            unpack16<TA>(*chunk, v);
            if constexpr (PRO == MEDNEXT_PRO_GROUPNORM) {
              float ca = 0.f, cb = 0.f;
              if (k < p.cin) {
                const float mean = __ldg(p.pro_stats + 2 * (s * p.cin + k));
                const float rstd = __ldg(p.pro_stats + 2 * (s * p.cin + k) + 1);
                ca = rstd * __ldg(p.pro_gamma + k);
                cb = __ldg(p.pro_beta + k) - mean * ca;
              }
              pw_prologue<PRO>(v, ca, cb);
            } else {
              pw_prologue<PRO>(v, 0.f, 0.f);
            }
            *chunk = pack16<TA>(v);
          }
          fence_async_smem();
          mbar_arrive(&sh.ready[st]);
        }
        if constexpr (MLP) {
          if (i >= kFwLag && !gelu_tile(i - kFwLag)) break;
        }
      }
      if constexpr (MLP) {
        for (int w = max(0, ntile_local - kFwLag); !*abort && w < ntile_local; ++w)
          if (!gelu_tile(w)) break;
      }
    }
  } else if (warp >= kEpiWarp0) {
    // ------------------------------------------------ epilogue
    // Two groups of epilogue warps take alternate tiles, so the latency chain of
    // one tile (TMEM load, staging, store issue) overlaps the next.  Within a
    // group, warp%4 selects the TMEM lane quarter (32 voxels) and the warps of
    // one quarter take turns over the 16-column chunks.  Every 32x16 result
    // block is staged in shared memory and written with one TMA bulk tensor
    // store (out-of-range rows and columns are clipped by the store).
    const int tgs = cfg.tgroups;
    const int kGroups = FwdEpi<PRO, EPI>::warps / 4 / tgs;
    const int ew = warp - kEpiWarp0;
    const int q4 = warp & 3;
    const int tg = (ew >> 2) % tgs;
    const int cg = (ew >> 2) / tgs;
    const int epi = EPI >= 0 ? EPI : p.epilogue;
    uint8_t* stg0 = ringStg + (size_t)ew * FwdEpi<PRO, EPI>::stg_bufs * kStgBytes;
    uint32_t nstored = 0;
    // fragment epilogue: lane L gives the row address of 8x8 matrix L / 8 = (x, vh) =
    // (L / 16, L / 8 % 2), row L % 8; t % 4 selects the thread's channel pair
    const int f_rr = lane & 7, f_x = (lane >> 4) & 1, f_vh = (lane >> 3) & 1, tq = lane & 3;
    for (int i = tg; i < ntile_local; i += tgs) {
      int s, j0, mt;
      long long v0;
      decode((int)blockIdx.x + i * (int)gridDim.x, s, j0, v0, mt);
      const int acc = i % cfg.nacc, ra = i / cfg.nacc;
      // warp-uniform waits: the warp issues tcgen05.ld and shuffles as a whole
      if (!__all_sync(0xffffffffu, wait_or_abort(&sh.tfull[acc], ra & 1, abort))) break;
      tc_fence_after();
      const int e = i % E, re = i / E;
      if ((has_aux || has_res) && !__all_sync(0xffffffffu, wait_or_abort(&sh.efull[e], re & 1, abort))) break;
      const int vl = q4 * 32 + lane;  // voxel within the tile
      const TA* auxt = reinterpret_cast<const TA*>(ringAux + (size_t)e * cfg.aux_bytes + (vl >> 6) * (cfg.aux_bytes / 2)) + (vl & 63);
      const TY* rest = reinterpret_cast<const TY*>(ringRes + (size_t)e * cfg.res_bytes + (vl >> 6) * (cfg.res_bytes / 2)) + (vl & 63);
      const uint32_t d_tmem = tmem + (uint32_t)acc * ncols + ((uint32_t)(q4 * 32) << 16);
      const uint32_t aux_u32 = smem_u32(ringAux + (size_t)e * cfg.aux_bytes);
      const uint32_t res_u32 = smem_u32(ringRes + (size_t)e * cfg.res_bytes);
      // fused weight grad: this group's g tile (voxel vl's column of box vl / 64), free
      // again once the weight-grad MMAs of the group's previous tile have read it
      // g-tile addresses of this lane's voxel in rows 8q + k (k < 8): the K-major
      // 128-byte swizzle XORs the 16-byte chunk index with k
      uint32_t gx[8];
      if constexpr ((FW || MLP) && !kFrag) {
        const uint32_t gcol = smem_u32(gbuf + tg * kFwGBytes + (vl >> 6) * 16384 + (vl & 7) * 2);
        const int gchunk = (vl & 63) >> 3;
#pragma unroll
        for (int k = 0; k < 8; ++k) gx[k] = gcol + (uint32_t)(k * 128 + ((gchunk ^ k) << 4));
      }
      if constexpr (FW || MLP) {
        if (i >= 2 && !__all_sync(0xffffffffu, wait_or_abort(&sh.gempty[tg], (uint32_t)(((i >> 1) - 1) & 1), abort)))
          break;
      }
      for (int c0 = kPwCW * cg; c0 < BN; c0 += kPwCW * kGroups) {
        if constexpr (kFrag) {
          // ---- fragment epilogue (16-bit outputs): thread t holds voxels t/4 (+8, +16,
          // +24) and channel pairs 8x + 2(t%4) of the chunk; auxiliary tiles come in and
          // the result goes out through 8x8 transposes (ldmatrix / stmatrix .trans) on
          // swizzled tiles, so every shared-memory access moves 16 bytes per lane.
          uint32_t r[16];
          tmem_ld_16x256b_x2(d_tmem + (uint32_t)c0, r);
          tmem_ld_16x256b_x2(d_tmem + (16u << 16) + (uint32_t)c0, r + 8);
          const int jr = c0 + 8 * f_x + f_rr;  // this lane's ldmatrix / stmatrix row (channel)
          uint32_t ax[8], rs[8];
          if (has_aux) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int vt = q4 * 32 + 16 * h + 8 * f_vh;
              ldsm_x4_trans(aux_u32 + (uint32_t)((vt >> 6) * (cfg.aux_bytes / 2) + jr * 128 +
                                                 ((((vt & 63) >> 3) ^ (jr & 7)) << 4)),
                            ax + 4 * h);
            }
          }
          if (epi & MEDNEXT_EPI_RESIDUAL) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int vt = q4 * 32 + 16 * h + 8 * f_vh;
              ldsm_x4_trans(res_u32 + (uint32_t)((vt >> 6) * (cfg.res_bytes / 2) + jr * 128 +
                                                 ((((vt & 63) >> 3) ^ (jr & 7)) << 4)),
                            rs + 4 * h);
            }
          }
          // per-channel constants of this thread's channels j0 + c0 + 8x + 2(t%4) + {0, 1}
          float2 bias2[2], mean2[2], rstd2[2], ca2[2], cb2[2];
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            const int jc = j0 + c0 + 8 * x + 2 * tq;
            const bool ok0 = jc < p.cout, ok1 = jc + 1 < p.cout;
            bias2[x] = make_float2(0.f, 0.f);
            mean2[x] = rstd2[x] = ca2[x] = cb2[x] = make_float2(0.f, 0.f);
            if (epi & MEDNEXT_EPI_BIAS)
              bias2[x] = make_float2(ok0 ? __ldg(p.bias + jc) : 0.f, ok1 ? __ldg(p.bias + jc + 1) : 0.f);
            if (epi & MEDNEXT_EPI_GN_BWD_STATS) {
              const float* st = p.epi_stats + 2 * ((size_t)s * p.cout + jc);
              mean2[x] = make_float2(ok0 ? __ldg(st) : 0.f, ok1 ? __ldg(st + 2) : 0.f);
              rstd2[x] = make_float2(ok0 ? __ldg(st + 1) : 0.f, ok1 ? __ldg(st + 3) : 0.f);
            }
            if constexpr (FW_GN) {
              // g = GroupNorm(aux) = aux * ca + cb, the weight-grad kernel's prologue coefficients
              if (ok0) {
                ca2[x].x = rstd2[x].x * __ldg(p.pro_gamma + jc);
                cb2[x].x = __ldg(p.pro_beta + jc) - mean2[x].x * ca2[x].x;
              }
              if (ok1) {
                ca2[x].y = rstd2[x].y * __ldg(p.pro_gamma + jc + 1);
                cb2[x].y = __ldg(p.pro_beta + jc + 1) - mean2[x].y * ca2[x].y;
              }
            }
          }
          // staging buffer: wait until the store issued two chunks ago has read it
          const uint32_t stg_u32 = smem_u32(stg0 + (nstored & 1) * kStgBytes);
          if (nstored >= 2 && lane == 0) bulk_wait_read<1>();
          __syncwarp();
          tmem_ld_wait();
          uint32_t out[8], gpk[8], gel[8];
          float2 st1[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
          float2 st2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
          for (int k = 0; k < 8; ++k) {  // pair k = (h, x, vh) = (k / 4, k / 2 % 2, k % 2)
            const int x = (k >> 1) & 1;
            float2 a = make_float2(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1]));
            if (epi & MEDNEXT_EPI_BIAS) a = make_float2(a.x + bias2[x].x, a.y + bias2[x].y);
            if (epi & (MEDNEXT_EPI_GELU_GRAD | MEDNEXT_EPI_RESIDUAL)) a = unpack2<TA>(pack2<TA>(a));
            float2 axv = make_float2(0.f, 0.f);
            if (has_aux) axv = unpack2<TA>(ax[k]);
            if constexpr (FW_GN)
              gpk[k] = pack2<TA>(make_float2(fmaf(axv.x, ca2[x].x, cb2[x].x), fmaf(axv.y, ca2[x].y, cb2[x].y)));
            if constexpr (FW_GELU) {
              float2 gv;
              const float2 g = gelu_grad2_and_gelu(axv, gv);
              gpk[k] = pack2<TA>(gv);
              a = make_float2(a.x * g.x, a.y * g.y);
            } else if (epi & MEDNEXT_EPI_GELU_GRAD) {
              const float2 g = gelu_grad2(axv);
              a = make_float2(a.x * g.x, a.y * g.y);
            }
            if (epi & MEDNEXT_EPI_RESIDUAL) {
              const float2 rv = unpack2<TY>(rs[k]);
              a = make_float2(a.x + rv.x, a.y + rv.y);
            }
            out[k] = pack2<TY>(a);
            if constexpr (MLP) gpk[k] = out[k];  // u as stored; GELU follows in place
            if constexpr (GOUT) gel[k] = pack2<TY>(gelu2(unpack2<TY>(out[k])));  // GELU of y as stored
            if (epi & MEDNEXT_EPI_GN_BWD_STATS) {
              // out-of-range voxels / channels hold exact zeros (zero-filled operands)
              const float2 d = unpack2<TY>(out[k]);
              st1[x] = make_float2(st1[x].x + d.x, st1[x].y + d.y);
              st2[x] = make_float2(st2[x].x + d.x * (axv.x - mean2[x].x), st2[x].y + d.y * (axv.y - mean2[x].y));
            }
          }
          {
            const int R = 8 * f_x + f_rr;  // staging row (channel of the chunk), 64-byte rows, 64-byte swizzle
#pragma unroll
            for (int h = 0; h < 2; ++h)
              stsm_x4_trans(stg_u32 + (uint32_t)(R * 64 + ((((2 * h + f_vh) ^ (R >> 1)) & 3) << 4)), out + 4 * h);
            if constexpr (GOUT) {
              const uint32_t stg_g = stg_u32 + 2 * kStgBytes;  // the g buffer of the same parity
#pragma unroll
              for (int h = 0; h < 2; ++h)
                stsm_x4_trans(stg_g + (uint32_t)(R * 64 + ((((2 * h + f_vh) ^ (R >> 1)) & 3) << 4)), gel + 4 * h);
            }
          }
          if constexpr (FW || MLP) {
            // g tile rows = this GEMM's output channels (rows past cout keep their zeros / ones)
            const uint32_t gt = smem_u32(gbuf + tg * kFwGBytes);
            if (c0 + kPwCW <= p.cout) {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int vt = q4 * 32 + 16 * h + 8 * f_vh;
                stsm_x4_trans(gt + (uint32_t)((vt >> 6) * 16384 + sw128_kmajor_off(jr, (vt & 63) >> 3)), gpk + 4 * h);
              }
            } else {
#pragma unroll
              for (int k = 0; k < 8; ++k) {
                const int h = k >> 2, x = (k >> 1) & 1, vh = k & 1;
                const int vt = q4 * 32 + 16 * h + 8 * vh + (lane >> 2);
#pragma unroll
                for (int e2 = 0; e2 < 2; ++e2) {
                  const int row = c0 + 8 * x + 2 * tq + e2;
                  if (row < p.cout)
                    st_shared_b16(gt + (uint32_t)((vt >> 6) * 16384 + sw128_kmajor_off(row, (vt & 63) >> 3) +
                                                  (vt & 7) * 2),
                                  (uint16_t)(gpk[k] >> (16 * e2)));
                }
              }
            }
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&mY, reinterpret_cast<void*>(stg0 + (nstored & 1) * kStgBytes), (int)v0 + q4 * 32, j0 + c0, s);
            if constexpr (GOUT)
              tma_store_3d(&mY2, reinterpret_cast<void*>(stg0 + (2 + (nstored & 1)) * kStgBytes), (int)v0 + q4 * 32,
                           j0 + c0, s);
            bulk_commit();
          }
          ++nstored;
          if (epi & MEDNEXT_EPI_GN_BWD_STATS) {
            // channel sums over the quarter's 32 voxels: the thread's four, then lanes
            // with the same t % 4 (xor 4, 8, 16); lanes 0-3 hold channels 8x + 2t + {0, 1}
#pragma unroll
            for (int x = 0; x < 2; ++x) {
#pragma unroll
              for (int o = 4; o < 32; o <<= 1) {
                st1[x].x += __shfl_xor_sync(0xffffffffu, st1[x].x, o);
                st1[x].y += __shfl_xor_sync(0xffffffffu, st1[x].y, o);
                st2[x].x += __shfl_xor_sync(0xffffffffu, st2[x].x, o);
                st2[x].y += __shfl_xor_sync(0xffffffffu, st2[x].y, o);
              }
              if (lane < 4) {
                const int col = j0 + c0 + 8 * x + 2 * lane;
                const size_t base = (((size_t)s * p.cout + col) * p.mtiles + mt) * 4 + q4;
                if (col < p.cout) {
                  GnBwdPartial gp;
                  gp.s1 = (double)st1[x].x;
                  gp.s2 = (double)(st2[x].x * rstd2[x].x);
                  p.gn_part[base] = gp;
                }
                if (col + 1 < p.cout) {
                  GnBwdPartial gp;
                  gp.s1 = (double)st1[x].y;
                  gp.s2 = (double)(st2[x].y * rstd2[x].y);
                  p.gn_part[base + (size_t)p.mtiles * 4] = gp;
                }
              }
            }
          }
        } else {
          uint32_t r[kPwCW];
          tmem_ld16(d_tmem + (uint32_t)c0, r);
          // per-column constants: lane l < 16 holds column c0 + l, broadcast with shuffles
          const int jc = j0 + c0 + lane;
          const bool jok = lane < kPwCW && jc < p.cout;
          const float bias_l = ((epi & MEDNEXT_EPI_BIAS) && jok) ? __ldg(p.bias + jc) : 0.f;
          float mean_l = 0.f, rstd_l = 0.f;
          if ((epi & MEDNEXT_EPI_GN_BWD_STATS) && jok) {
            mean_l = __ldg(p.epi_stats + 2 * (s * p.cout + jc));
            rstd_l = __ldg(p.epi_stats + 2 * (s * p.cout + jc) + 1);
          }
          // fused weight grad after a GroupNorm: g = GroupNorm(aux) = aux * ca + cb, with the
          // same coefficients (and rounding) as the weight-grad kernel's GroupNorm prologue
          float ca_l = 0.f, cb_l = 0.f;
          if constexpr (FW_GN) {
            if (jok) {
              ca_l = rstd_l * __ldg(p.pro_gamma + jc);
              cb_l = __ldg(p.pro_beta + jc) - mean_l * ca_l;
            }
          }
          // staging buffer: wait until the store issued two chunks ago has read it
          TY* stg = reinterpret_cast<TY*>(stg0 + (nstored & 1) * kStgBytes);
          if (nstored >= 2 && lane == 0) bulk_wait_read<1>();
          __syncwarp();
          tmem_ld_wait();
          float s1[kPwCW], s2[kPwCW];
          float gg[kPwCW];  // GELU'(aux) of the chunk's columns, in pairs
          // g row c0 + jj of this lane's voxel (rows past cout keep their zeros / ones)
          const bool gfull = c0 + kPwCW <= p.cout;
          auto gstore = [&](int jj, float v) {
            if (gfull || c0 + jj < p.cout) {
              const TA b = from_acc<TA>(v);
              st_shared_b16(gx[jj & 7] + (uint32_t)(((c0 >> 3) + (jj >> 3)) * 1024), *reinterpret_cast<const uint16_t*>(&b));
            }
          };
          if constexpr (FW_GELU) {
            // GELU(aux) as well, from the same Phi: into the g tile (channels past cout keep their zeros / ones)
  #pragma unroll
            for (int jj = 0; jj < kPwCW; jj += 2) {
              float2 gv;
              const float2 g = gelu_grad2_and_gelu(
                  make_float2(to_acc<TA>(auxt[(c0 + jj) * 64]), to_acc<TA>(auxt[(c0 + jj + 1) * 64])), gv);
              gg[jj] = g.x;
              gg[jj + 1] = g.y;
              gstore(jj, gv.x);
              gstore(jj + 1, gv.y);
            }
          } else if (epi & MEDNEXT_EPI_GELU_GRAD) {
  #pragma unroll
            for (int jj = 0; jj < kPwCW; jj += 2) {
              const float2 g = gelu_grad2(
                  make_float2(to_acc<TA>(auxt[(c0 + jj) * 64]), to_acc<TA>(auxt[(c0 + jj + 1) * 64])));
              gg[jj] = g.x;
              gg[jj + 1] = g.y;
            }
          }
  #pragma unroll
          for (int jj = 0; jj < kPwCW; ++jj) {
            const int jl = c0 + jj;
            float a = __uint_as_float(r[jj]);
            if (epi & MEDNEXT_EPI_BIAS) a += __shfl_sync(0xffffffffu, bias_l, jj);
            if (epi & (MEDNEXT_EPI_GELU_GRAD | MEDNEXT_EPI_RESIDUAL)) a = to_acc<TA>(from_acc<TA>(a));
            float ax = 0.f;
            if (epi & MEDNEXT_EPI_GN_BWD_STATS) ax = to_acc<TA>(auxt[jl * 64]);
            if constexpr (FW_GN)
              gstore(jj, fmaf(ax, __shfl_sync(0xffffffffu, ca_l, jj), __shfl_sync(0xffffffffu, cb_l, jj)));
            if (epi & MEDNEXT_EPI_GELU_GRAD) a *= gg[jj];
            if (epi & MEDNEXT_EPI_RESIDUAL) a += (float)to_acc<TY>(rest[jl * 64]);
            const TY o = from_acc<TY>((typename Elem<TY>::Acc)a);
            stg[jj * 32 + lane] = o;
            if constexpr (MLP) gstore(jj, (float)to_acc<TY>(o));  // u as stored; GELU follows in place
            if (epi & MEDNEXT_EPI_GN_BWD_STATS) {
              // out-of-range voxels / channels hold exact zeros (zero-filled operands)
              const float d = (float)to_acc<TY>(o);
              s1[jj] = d;
              s2[jj] = d * (ax - __shfl_sync(0xffffffffu, mean_l, jj));
            }
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&mY, stg, (int)v0 + q4 * 32, j0 + c0, s);
            bulk_commit();
          }
          ++nstored;
          if (epi & MEDNEXT_EPI_GN_BWD_STATS) {
            // column sums over the 32 voxels; lanes 2c and 2c+1 end up with column c
            const float t1 = warp_transpose_sum16(s1, lane);
            const float t2 = warp_transpose_sum16(s2, lane);
            const float rstd_c = __shfl_sync(0xffffffffu, rstd_l, lane >> 1);
            const int col = j0 + c0 + (lane >> 1);
            if ((lane & 1) == 0 && col < p.cout) {
              // one partial per (channel, tile, 32-voxel quarter): no cross-warp sync
              GnBwdPartial gp;
              gp.s1 = (double)t1;
              gp.s2 = (double)(t2 * rstd_c);
              p.gn_part[(((size_t)s * p.cout + col) * p.mtiles + mt) * 4 + q4] = gp;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&sh.tempty[acc]);
      if constexpr (FW) {
        // the group's g tile is complete: hand it to the MMA warp (async proxy)
        fence_async_smem();
        mbar_arrive(&sh.gready[tg]);
      }
      if constexpr (MLP) mbar_arrive(&sh.uready[tg]);  // u in the g tile: the prologue warps take over
      if constexpr (MLP) {
        // second GEMM of this tile: y2 = D2 + bias2 (+ residual), as the compress GEMM's epilogue
        if (!__all_sync(0xffffffffu, wait_or_abort(&sh.d2full[tg], (uint32_t)((i >> 1) & 1), abort))) break;
        tc_fence_after();
        const uint32_t d2_tmem = tmem + (uint32_t)cfg.d2_col + (uint32_t)(tg * cfg.d2_stride) + ((uint32_t)(q4 * 32) << 16);
        for (int c0 = kPwCW * cg; c0 < cfg.bn2; c0 += kPwCW * kGroups) {
          if constexpr (kFrag) {
            uint32_t r[16];
            tmem_ld_16x256b_x2(d2_tmem + (uint32_t)c0, r);
            tmem_ld_16x256b_x2(d2_tmem + (16u << 16) + (uint32_t)c0, r + 8);
            const int jr = c0 + 8 * f_x + f_rr;
            uint32_t rs[8];
            if (has_res) {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int vt = q4 * 32 + 16 * h + 8 * f_vh;
                ldsm_x4_trans(res_u32 + (uint32_t)((vt >> 6) * (cfg.res_bytes / 2) + jr * 128 +
                                                   ((((vt & 63) >> 3) ^ (jr & 7)) << 4)),
                              rs + 4 * h);
              }
            }
            float2 bias2[2];
#pragma unroll
            for (int x = 0; x < 2; ++x) {
              const int jc = c0 + 8 * x + 2 * tq;
              bias2[x] = make_float2(jc < p.cout2 ? __ldg(p.bias2 + jc) : 0.f,
                                     jc + 1 < p.cout2 ? __ldg(p.bias2 + jc + 1) : 0.f);
            }
            const uint32_t stg_u32 = smem_u32(stg0 + (nstored & 1) * kStgBytes);
            if (nstored >= 2 && lane == 0) bulk_wait_read<1>();
            __syncwarp();
            tmem_ld_wait();
            uint32_t out[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int x = (k >> 1) & 1;
              float2 a = make_float2(__uint_as_float(r[2 * k]) + bias2[x].x, __uint_as_float(r[2 * k + 1]) + bias2[x].y);
              if (has_res) {
                a = unpack2<TA>(pack2<TA>(a));
                const float2 rv = unpack2<TY>(rs[k]);
                a = make_float2(a.x + rv.x, a.y + rv.y);
              }
              out[k] = pack2<TY>(a);
            }
            const int R = 8 * f_x + f_rr;
#pragma unroll
            for (int h = 0; h < 2; ++h)
              stsm_x4_trans(stg_u32 + (uint32_t)(R * 64 + ((((2 * h + f_vh) ^ (R >> 1)) & 3) << 4)), out + 4 * h);
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_3d(&mY2, reinterpret_cast<void*>(stg0 + (nstored & 1) * kStgBytes), (int)v0 + q4 * 32, c0, s);
              bulk_commit();
            }
            ++nstored;
          } else {
            uint32_t r[kPwCW];
            tmem_ld16(d2_tmem + (uint32_t)c0, r);
            const int jc = c0 + lane;
            const float bias_l = (lane < kPwCW && jc < p.cout2) ? __ldg(p.bias2 + jc) : 0.f;
            TY* stg = reinterpret_cast<TY*>(stg0 + (nstored & 1) * kStgBytes);
            if (nstored >= 2 && lane == 0) bulk_wait_read<1>();
            __syncwarp();
            tmem_ld_wait();
  #pragma unroll
            for (int jj = 0; jj < kPwCW; ++jj) {
              float a = __uint_as_float(r[jj]) + __shfl_sync(0xffffffffu, bias_l, jj);
              if (has_res) a = to_acc<TA>(from_acc<TA>(a)) + (float)to_acc<TY>(rest[(c0 + jj) * 64]);
              stg[jj * 32 + lane] = from_acc<TY>((typename Elem<TY>::Acc)a);
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_3d(&mY2, stg, (int)v0 + q4 * 32, c0, s);
              bulk_commit();
            }
            ++nstored;
          }
        }
      }
      if (has_aux || has_res) mbar_arrive(&sh.eempty[e]);
    }
    if constexpr (FW) {
      // the CTA's weight-grad partial: D^T[h, c] from TMEM lane h, one split per CTA
      if (tg == 0 && cg == 0 && __all_sync(0xffffffffu, wait_or_abort(&sh.wdone, 0u, abort))) {
        tc_fence_after();
        const int h = q4 * 32 + lane;
        const uint32_t wt = tmem + (uint32_t)cfg.nacc * ncols + ((uint32_t)(q4 * 32) << 16);
        for (int c0 = 0; c0 < p.cin; c0 += kPwCW) {
          uint32_t r[kPwCW];
          tmem_ld16(wt + (uint32_t)c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int jj = 0; jj < kPwCW; ++jj) {
            const int c = c0 + jj;
            if (c >= p.cin) break;
            if (h < p.cout) p.w_part[((size_t)blockIdx.x * p.cin + c) * p.cout + h] = __uint_as_float(r[jj]);
            else if (h == p.cout) p.w_part_b[(size_t)blockIdx.x * p.cin + c] = __uint_as_float(r[jj]);
          }
        }
      }
    }
    if (lane == 0) bulk_wait_all();
  }
  __syncthreads();
  if (*abort && lane == 0) {
    if (warp == 0) {
      drain_ring(sh.full, S, a_issued);
      if (w_issued) mbar_wait(&sh.wfull, 0);
    }
    if (warp == 2) drain_ring(sh.efull, E, aux_issued);
    if (warp == 1) drain_mma(&sh.drain);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, (uint32_t)cfg.tmem_cols);
}

// ---------------------------------------------------------------- weight grad
// 512 threads: warp 0 TMA producer, warp 1 MMA issuer, warps 4-11 prologue,
// warps 12-15 epilogue.  D[j, k] = sum over the split's voxel chunks of
// g[j, v] * pro(a[k, v]): A = 128 rows of g, B = BN rows of a, both K-major.
//
// Bias grad: when the a rows fit in one N tile with a row to spare (ones_row >=
// 0), that row of every B stage holds 1.0, written once at start (the TMA box
// only covers the real a rows, so loads never overwrite it), and column
// ones_row of the accumulator is sum_v g[j, v] = dbias[j].  Otherwise the
// prologue warps sum the g rows.
constexpr int kWgThreads = 512;
constexpr int kWgProWarp0 = 4;
constexpr int kWgProThreads = 256;
constexpr int kWgEpiWarp0 = 12;
// epilogue staging after the ring: one 32 x 32 fp32 tile per epilogue warp (column
// c of row r at r * 32 + (c ^ r): conflict-free by rows and by columns), so that a
// warp turns its 32 rows x 32 columns of accumulator into 32 coalesced row stores
constexpr int kWgStgFloats = 32 * 32;
constexpr size_t kWgStgBytes = 4 * kWgStgFloats * sizeof(float);

struct PwTmaWgradCfg {
  int stages;
  int nch;       // 64-voxel chunks per ring stage (one TMA barrier phase covers all of them)
  int b_bytes;   // BN * 128: one B slot
  int units;     // mtiles * ntiles * splits
  int g_rows;    // rows of g per TMA box (min(128, cout))
  int a_rows;    // rows of a per TMA box
  int ones_row;  // B-tile row held at 1.0 for the bias grad, or -1
  int stage_epi; // the epilogue stores rows through the staging tiles after the ring
};

template <typename TA, int PRO>
__global__ void __launch_bounds__(kWgThreads, 1)
    pw_tma_wgrad_kernel(const __grid_constant__ CUtensorMap mG, const __grid_constant__ CUtensorMap mA,
                        PwWgradArgs p, PwTmaWgradCfg cfg) {
  extern __shared__ uint8_t smem_dyn[];
  __shared__ PwTmaSmem sh;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int BN = p.BN;
  const int S = cfg.stages;
  const bool ones = cfg.ones_row >= 0;
  // the prologue warps run for a GroupNorm / GELU prologue and for bias row sums
  const bool pro_on = PRO != MEDNEXT_PRO_NONE || !ones;
  const uint32_t base_u32 = smem_u32(smem_dyn);
  uint8_t* sbase = smem_dyn + (((base_u32 + 1023u) & ~1023u) - base_u32);
  // stage st holds chunk slots st*nch .. st*nch+nch-1: a stage of several chunks
  // amortises the per-phase cost of the TMA barrier hand-off
  const int NCH = cfg.nch;
  const int SL = S * NCH;                       // chunk slots
  uint8_t* ringA = sbase;                       // SL x 16 KB  (g rows)
  uint8_t* ringB = ringA + (size_t)SL * 16384;  // SL x b_bytes (a rows)
  const uint32_t chunk_tx = (uint32_t)(cfg.g_rows + cfg.a_rows) * 128u;

  // rows that TMA never writes stay zero; the bias row holds ones
  {
    const size_t ring_bytes = (size_t)SL * (16384 + cfg.b_bytes);
    for (size_t off = (size_t)tid * 16; off < ring_bytes; off += (size_t)kWgThreads * 16)
      *reinterpret_cast<uint4*>(sbase + off) = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();
    for (int t = tid; ones && t < SL * 8; t += kWgThreads) {
      const int sl = t >> 3, c = t & 7;
      float one[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) one[e] = 1.0f;
      *reinterpret_cast<uint4*>(ringB + (size_t)sl * cfg.b_bytes + sw128_kmajor_off(cfg.ones_row, c)) =
          pack16<TA>(one);
    }
    fence_async_smem();
  }

  const uint32_t ncols = tmem_cols_for(BN);
  if (warp == 1) {
    tmem_alloc(&sh.tmem_base, ncols);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&sh.full[i], 1);
      mbar_init(&sh.ready[i], kWgProThreads);
      mbar_init(&sh.empty[i], 1);
    }
    mbar_init(&sh.tfull[0], 1);
    mbar_init(&sh.tempty[0], 128);
    mbar_init(&sh.drain, 1);
    sh.abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&mG);
    tma_prefetch_map(&mA);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  volatile int* abort = &sh.abort;
  const int nunits = (cfg.units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  long long g_issued = 0;  // TMA fills issued by the producer

  auto unit_range = [&](int u, int& mt, int& nt, int& sp, long long& cb, long long& ce) {
    mt = u % p.mtiles;
    const int rest = u / p.mtiles;
    nt = rest % p.ntiles;
    sp = rest / p.ntiles;
    cb = (long long)sp * p.chunks_per_split;
    ce = min(cb + p.chunks_per_split, p.chunks_total);
  };

  if (warp == 0) {
    if (lane == 0) {
      long long q = 0;  // stages filled
      for (int i = 0; i < nunits && !*abort; ++i) {
        int mt, nt, sp;
        long long cb, ce;
        unit_range((int)blockIdx.x + i * (int)gridDim.x, mt, nt, sp, cb, ce);
        for (long long ch0 = cb; ch0 < ce; ch0 += NCH, ++q) {
          const int st = (int)(q % S);
          const long long r = q / S;
          if (r > 0 && !wait_or_abort(&sh.empty[st], (uint32_t)((r - 1) & 1), abort)) break;
          const int n = (int)min((long long)NCH, ce - ch0);
          mbar_arrive_expect_tx(&sh.full[st], chunk_tx * (uint32_t)n);
          for (int c = 0; c < n; ++c) {
            const long long ch = ch0 + c;
            const int s = (int)(ch / p.chunks_per_sample);
            const int v = (int)((ch - (long long)s * p.chunks_per_sample) * kPwBK);
            const int sl = st * NCH + c;
            tma_load_3d(ringA + (size_t)sl * 16384, &mG, &sh.full[st], v, mt * kPwBM, s);
            tma_load_3d(ringB + (size_t)sl * cfg.b_bytes, &mA, &sh.full[st], v, nt * BN, s);
          }
        }
      }
      g_issued = q;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f16(kPwBM, BN, std::is_same<TA, __nv_bfloat16>::value, false, false);
      long long q = 0;
      for (int i = 0; i < nunits && !*abort; ++i) {
        int mt, nt, sp;
        long long cb, ce;
        unit_range((int)blockIdx.x + i * (int)gridDim.x, mt, nt, sp, cb, ce);
        if (i > 0 && !wait_or_abort(&sh.tempty[0], (uint32_t)((i - 1) & 1), abort)) break;
        tc_fence_after();
        bool first = true;
        for (long long ch0 = cb; ch0 < ce; ch0 += NCH, ++q) {
          const int st = (int)(q % S);
          const long long r = q / S;
          if (!wait_or_abort(pro_on ? &sh.ready[st] : &sh.full[st], (uint32_t)(r & 1), abort)) break;
          tc_fence_after();
          const int n = (int)min((long long)NCH, ce - ch0);
          for (int c = 0; c < n; ++c) {
            const int sl = st * NCH + c;
            const uint32_t a_addr = smem_u32(ringA + (size_t)sl * 16384);
            const uint32_t b_addr = smem_u32(ringB + (size_t)sl * cfg.b_bytes);
#pragma unroll
            for (int ks = 0; ks < kPwBK / 16; ++ks) {
              const uint64_t ad = make_sw128_desc(a_addr + ks * 32, 16, 1024);
              const uint64_t bd = make_sw128_desc(b_addr + ks * 32, 16, 1024);
              mma_f16_ss(tmem, ad, bd, idesc, first ? 0u : 1u);
              first = false;
            }
          }
          mma_commit(&sh.empty[st]);
        }
        mma_commit(&sh.tfull[0]);
      }
    }
  } else if (warp >= kWgProWarp0 && warp < kWgEpiWarp0) {
    if (!pro_on) {
      // nothing to transform or sum: the MMA consumes the stages straight from TMA
    } else {
      // prologue on the a rows (in place) and, without a bias row, the g row sums
      const int t = tid - kWgProWarp0 * 32;  // 0..255
      long long q = 0;
      for (int i = 0; i < nunits && !*abort; ++i) {
        int mt, nt, sp;
        long long cb, ce;
        unit_range((int)blockIdx.x + i * (int)gridDim.x, mt, nt, sp, cb, ce);
        const bool rowsum = !ones && nt == 0 && t < kPwBM;
        float bsum = 0.f;  // row t of g (output channel mt*128 + t)
        for (long long ch0 = cb; ch0 < ce; ch0 += NCH, ++q) {
          const int st = (int)(q % S);
          const long long r = q / S;
          if (!wait_or_abort(&sh.full[st], (uint32_t)(r & 1), abort)) break;
          const int nc = (int)min((long long)NCH, ce - ch0);
          for (int c = 0; c < nc; ++c) {
            const int sl = st * NCH + c;
            const int s = (int)((ch0 + c) / p.chunks_per_sample);
            if (rowsum) {
              const uint8_t* row = ringA + (size_t)sl * 16384 + (t >> 3) * 1024 + (t & 7) * 128;
#pragma unroll
              for (int c16 = 0; c16 < 8; ++c16) {
                float v[8];
                unpack16<TA>(*reinterpret_cast<const uint4*>(row + c16 * 16), v);
#pragma unroll
                for (int e = 0; e < 8; ++e) bsum += v[e];
              }
            }
            if constexpr (PRO != MEDNEXT_PRO_NONE) {
              // a_rows x 8 chunks of 8 voxels; item -> (row, chunk), 4 rows per warp pass
              for (int item = t; item < cfg.a_rows * 8; item += kWgProThreads) {
                const int n = item >> 3, cq = item & 7;
                const int k = nt * BN + n;
                uint4* chunk = reinterpret_cast<uint4*>(ringB + (size_t)sl * cfg.b_bytes + sw128_kmajor_off(n, cq));
                float v[8];
                unpack16<TA>(*chunk, v);
                if constexpr (PRO == MEDNEXT_PRO_GROUPNORM) {
                  float ca = 0.f, cbb = 0.f;
                  if (k < p.cin) {
                    const float mean = __ldg(p.pro_stats + 2 * (s * p.cin + k));
                    const float rstd = __ldg(p.pro_stats + 2 * (s * p.cin + k) + 1);
                    ca = rstd * __ldg(p.pro_gamma + k);
                    cbb = __ldg(p.pro_beta + k) - mean * ca;
                  }
                  pw_prologue<PRO>(v, ca, cbb);
                } else {
                  pw_prologue<PRO>(v, 0.f, 0.f);
                }
                *chunk = pack16<TA>(v);
              }
            }
          }
          if constexpr (PRO != MEDNEXT_PRO_NONE) fence_async_smem();
          mbar_arrive(&sh.ready[st]);
        }
        if (rowsum) {
          const int j = mt * kPwBM + t;
          if (j < p.cout) p.part_b[(size_t)sp * p.cout + j] = bsum;
        }
      }
    }
  } else if (warp >= kWgEpiWarp0) {
    const int q4 = warp & 3;
    for (int i = 0; i < nunits; ++i) {
      int mt, nt, sp;
      long long cb, ce;
      unit_range((int)blockIdx.x + i * (int)gridDim.x, mt, nt, sp, cb, ce);
      const bool any = ce > cb;
      // the MMA warp commits tfull once per unit, with or without MMAs
      if (!__all_sync(0xffffffffu, wait_or_abort(&sh.tfull[0], (uint32_t)(i & 1), abort))) break;  // warp-uniform
      tc_fence_after();
      // lane = accumulator row j0 + lane.  With few chunks per unit (the deep
      // levels) the partial stores weigh: the staging tile turns each 32 x 32 block
      // into row stores, lane e writing column c0 + e of row j0 + jj, 32 lanes to one
      // 128-byte segment.  Otherwise each lane stores its own row (32 segments per
      // store, but once per several hundred chunks) and the ring keeps the space.
      const int j0 = mt * kPwBM + q4 * 32;
      if (!cfg.stage_epi) {
        const int j = j0 + lane;
        float bval = 0.f;
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t r[32];
          if (any) {
            tmem_ld32(tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)c0, r);
            tmem_ld_wait();
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) r[e] = 0u;
          }
          if (j < p.cout) {
            float* dst = p.part + ((size_t)sp * p.cout + j) * p.cin;
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const int k = nt * BN + c0 + e;
              if (c0 + e < BN && k < p.cin) dst[k] = __uint_as_float(r[e]);
              if (c0 + e == cfg.ones_row) bval = __uint_as_float(r[e]);
            }
          }
        }
        if (ones && j < p.cout) p.part_b[(size_t)sp * p.cout + j] = bval;
        tc_fence_before();
        mbar_arrive(&sh.tempty[0]);
        continue;
      }
      float* stg = reinterpret_cast<float*>(ringB + (size_t)SL * cfg.b_bytes) + q4 * kWgStgFloats;
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        if (any) {
          tmem_ld32(tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)c0, r);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) r[e] = 0u;
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) stg[lane * 32 + (e ^ lane)] = __uint_as_float(r[e]);
        __syncwarp();
        const int k = nt * BN + c0 + lane;
        const bool col_ok = c0 + lane < BN && k < p.cin;
        const bool bias_col = c0 + lane == cfg.ones_row;
        for (int jj = 0; jj < 32; ++jj) {
          const int j = j0 + jj;
          if (j >= p.cout) break;  // warp-uniform
          const float v = stg[jj * 32 + (lane ^ jj)];
          if (col_ok) p.part[((size_t)sp * p.cout + j) * p.cin + k] = v;
          if (bias_col) p.part_b[(size_t)sp * p.cout + j] = v;
        }
        __syncwarp();
      }
      tc_fence_before();
      mbar_arrive(&sh.tempty[0]);
    }
  }
  __syncthreads();
  if (*abort && lane == 0) {
    if (warp == 0) drain_ring(sh.full, S, g_issued);
    if (warp == 1) drain_mma(&sh.drain);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, ncols);
}

}  // namespace mednext
