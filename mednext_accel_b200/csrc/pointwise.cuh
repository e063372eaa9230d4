// Pointwise 1x1x1 convolutions of the MedNeXt block on the 5th-generation
// tensor cores (tcgen05.mma, fp32 accumulators in TMEM).
//
// NCDHW activations make the voxel axis contiguous, so:
//  * forward / input-grad GEMMs put voxels on M (128 per tile): the activation
//    operand is MN-major ([k][voxel] in memory), the weight operand K-major;
//  * weight-grad GEMMs reduce over voxels: both operands are K-major.
// Operands are staged into 128-byte-swizzled shared memory by the CTA's
// threads, which apply the fused prologue (GroupNorm apply or exact GELU) on
// the way; one thread issues the MMAs and commits them to an mbarrier; the
// accumulator tile is read back with tcgen05.ld for the fused epilogue
// (bias, residual add, GELU derivative, GroupNorm-backward partial sums).
// Reference: ops/adaptive.py:174-200 (per-sample addmm / F.conv3d) and the
// GroupNorm, GELU and residual of models/blocks.py:74-91.
#pragma once

#include <type_traits>

#include "common.cuh"
#include "groupnorm.cuh"

namespace mednext {

constexpr int kPwBM = 128;  // voxels (forward) or output channels (wgrad) per tile
constexpr int kPwBK = 64;   // K per pipeline stage: one 128-byte swizzle atom
constexpr int kPwThreads = 128;

struct PwFwdArgs {
  const void* a;      // [S, cin, vox]
  const void* wt;     // [cout, cin]
  void* y;            // [S, cout, vox]
  const float* pro_stats;  // [S*cin][2]
  const float* pro_gamma;
  const float* pro_beta;
  const float* bias;       // [cout]
  const void* residual;    // [S, cout, vox]
  const void* aux;         // [S, cout, vox]
  const float* epi_stats;  // [S*cout][2]
  GnBwdPartial* gn_part;   // [S*cout][mtiles]
  int S, cin, cout;
  long long vox;
  int BN, mtiles, ntiles;
  int epilogue;
  int vec_a;  // vox % 8 == 0 and aligned
  int vec_w;  // cin % 8 == 0 and aligned
  void* wpad;  // workspace for W with rows padded to a multiple of 8 (cin % 8 != 0), or null
  void* pro_out;  // [S, cin, vox] in a's dtype: pro(a) as the GEMM consumed it, or null
  float* w_part;    // fused compress weight grad: [splits][cin][cout] partials (splits = grid)
  float* w_part_b;  // [splits][cin] bias-grad partials
  // fused expansion (second GEMM): y2 = w2 @ GELU(y) + bias2 (+ residual, [S, cout2, vox])
  const void* w2;       // [cout2, cout] (K = cout contiguous)
  const float* bias2;   // [cout2]
  void* y2;             // [S, cout2, vox]
  int cout2;
};

// W [cout][cin] -> [cout][cin8] with zero columns: TMA needs 16-byte row strides.
template <typename T>
static __global__ void pw_pad_weight_kernel(const T* __restrict__ w, T* __restrict__ out, int cout, int cin, int cin8) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)cout * cin8) return;
  const int j = (int)(i / cin8), k = (int)(i - (long long)j * cin8);
  out[i] = k < cin ? w[(size_t)j * cin + k] : from_acc<T>(0.0f);
}

__device__ __forceinline__ uint32_t sw128_kmajor_off(int row, int chunk) {
  // 8-row x 128-byte atoms stacked along rows; 16-byte chunk index XOR row%8.
  return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}
__device__ __forceinline__ uint32_t sw128_mnmajor_off(int k, int mchunk) {
  // MN-major, 128 rows of M: atom (64 M x 8 k) = 1024 B; M atoms 1024 B apart
  // (LBO), K atoms 2048 B apart (SBO).  Row inside an atom = k%8.
  return (uint32_t)((k >> 3) * 2048 + (mchunk >> 3) * 1024 + (k & 7) * 128 +
                    (((mchunk & 7) ^ (k & 7)) << 4));
}

template <typename TA>
__device__ __forceinline__ uint4 pw_pack(const float* v) {
  return pack16<TA>(v);
}

// Apply the prologue to 8 values of input channel k (coefficients a*x+b for
// GroupNorm, erf-GELU for GELU).
template <int PRO>
__device__ __forceinline__ void pw_prologue(float* v, float ca, float cb) {
  if constexpr (PRO == MEDNEXT_PRO_GROUPNORM) {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = fmaf(v[i], ca, cb);
  } else if constexpr (PRO == MEDNEXT_PRO_GELU) {
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      const float2 g = gelu2(make_float2(v[i], v[i + 1]));
      v[i] = g.x;
      v[i + 1] = g.y;
    }
  }
}

// out = pro(a) elementwise over [S, cin, vox], with the same arithmetic as the
// GEMM prologue: the prologue output of the first-generation kernel.
template <typename TA, int PRO>
static __global__ void pw_prologue_out_kernel(const TA* __restrict__ a, TA* __restrict__ out,
                                              const float* __restrict__ stats, const float* __restrict__ gamma,
                                              const float* __restrict__ beta, int cin, long long vox,
                                              long long total) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    float v = to_acc<TA>(a[i]);
    if constexpr (PRO == MEDNEXT_PRO_GROUPNORM) {
      const long long row = i / vox;  // s * cin + k
      const int k = (int)(row % cin);
      const float ca = stats[2 * row + 1] * gamma[k];
      v = fmaf(v, ca, beta[k] - stats[2 * row] * ca);
    } else {
      v = gelu_f(v);
    }
    out[i] = from_acc<TA>(v);
  }
}

// Load 8 consecutive elements (zero beyond `limit`) as floats.
template <typename TA>
__device__ __forceinline__ void pw_load8(const TA* __restrict__ p, long long remaining, bool vec,
                                         float* v) {
  if (vec && remaining >= 8) {
    unpack16<TA>(__ldg(reinterpret_cast<const uint4*>(p)), v);
    return;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = (i < remaining) ? to_acc<TA>(p[i]) : 0.0f;
}

template <typename TA, typename TY, int PRO>
__global__ void __launch_bounds__(kPwThreads) pw_fwd_kernel(PwFwdArgs p) {
  extern __shared__ uint8_t smem_dyn[];
  __shared__ uint64_t mma_bar[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;
  __shared__ float coef[kPwBK][2];

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  // tile decode: voxel tile fastest so neighbouring CTAs share weight tiles
  int b = blockIdx.x;
  const int mt = b % p.mtiles;
  b /= p.mtiles;
  const int nt = b % p.ntiles;
  const int s = b / p.ntiles;
  const long long v0 = (long long)mt * kPwBM;
  const int j0 = nt * p.BN;
  const int BN = p.BN;

  // 1024-byte aligned stage buffers: A0 A1 (16 KB each), B0 B1 (BN*128 each)
  const uint32_t base_u32 = smem_u32(smem_dyn);
  const uint32_t pad = ((base_u32 + 1023u) & ~1023u) - base_u32;
  uint8_t* sbase = smem_dyn + pad;
  // stage buffer b: A at sbase + b*16 KB, B at sbase + 32 KB + b*BN*128
  auto stageA = [&](int bb) { return sbase + bb * 16384; };
  auto stageB = [&](int bb) { return sbase + 32768 + bb * BN * 128; };

  const uint32_t ncols = BN <= 32 ? 32u : (BN <= 64 ? 64u : (BN <= 128 ? 128u : 256u));
  if (warp == 0) {
    tmem_alloc(&tmem_base_sh, ncols);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&mma_bar[0], 1);
    mbar_init(&mma_bar[1], 1);
    fence_mbarrier_init();
    abort_sh = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  const TA* A = static_cast<const TA*>(p.a);
  const TA* W = static_cast<const TA*>(p.wt);
  const int nstage = (p.cin + kPwBK - 1) / kPwBK;
  const uint32_t idesc = make_idesc_f16(kPwBM, BN, std::is_same<TA, __nv_bfloat16>::value, true, false);

  for (int st = 0; st < nstage; ++st) {
    const int buf = st & 1;
    const int k0 = st * kPwBK;
    if (st >= 2 && !abort_sh) {
      if (!mbar_wait(&mma_bar[buf], ((st - 2) >> 1) & 1)) abort_sh = 1;
    }
    if constexpr (PRO == MEDNEXT_PRO_GROUPNORM) {
      if (tid < kPwBK) {
        const int k = k0 + tid;
        float ca = 0.f, cb = 0.f;
        if (k < p.cin) {
          const float mean = p.pro_stats[2 * (s * p.cin + k)];
          const float rstd = p.pro_stats[2 * (s * p.cin + k) + 1];
          ca = rstd * p.pro_gamma[k];
          cb = p.pro_beta[k] - mean * ca;
        }
        coef[tid][0] = ca;
        coef[tid][1] = cb;
      }
      __syncthreads();
    }
    // ---- A: 64 k-rows x 16 chunks of 8 voxels; thread owns k%8 = tid/16 ----
    {
      const int mch = tid & 15;
      const int kr = tid >> 4;
      const long long v = v0 + 8 * mch;
      const long long rem = p.vox - v;
      float vals[8][8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int k = k0 + kr + 8 * i;
        if (k < p.cin && rem > 0) {
          pw_load8<TA>(A + ((long long)s * p.cin + k) * p.vox + v, rem, p.vec_a != 0, vals[i]);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) vals[i][e] = 0.f;
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int kk = kr + 8 * i;
        const int k = k0 + kk;
        if (PRO != MEDNEXT_PRO_NONE && k < p.cin && rem > 0) {
          pw_prologue<PRO>(vals[i], PRO == MEDNEXT_PRO_GROUPNORM ? coef[kk][0] : 0.f,
                           PRO == MEDNEXT_PRO_GROUPNORM ? coef[kk][1] : 0.f);
          // voxels past the end must stay zero (GroupNorm shifts them)
          if (rem < 8) {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (e >= rem) vals[i][e] = 0.f;
          }
        }
        *reinterpret_cast<uint4*>(stageA(buf) + sw128_mnmajor_off(kk, mch)) = pw_pack<TA>(vals[i]);
      }
    }
    // ---- B: BN rows x 8 chunks of 8 k ----
    {
      const int q = tid & 7;
      for (int n = tid >> 3; n < BN; n += kPwThreads / 8) {
        const int j = j0 + n;
        const int k = k0 + 8 * q;
        float vals[8];
        if (j < p.cout && k < p.cin) {
          pw_load8<TA>(W + (long long)j * p.cin + k, p.cin - k, p.vec_w != 0, vals);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) vals[e] = 0.f;
        }
        *reinterpret_cast<uint4*>(stageB(buf) + sw128_kmajor_off(n, q)) = pw_pack<TA>(vals);
      }
    }
    fence_async_smem();
    __syncthreads();
    if (tid == 0 && !abort_sh) {
      tc_fence_after();
      const int ksteps = min(kPwBK, p.cin - k0 + 15) / 16;
      const uint32_t a_addr = smem_u32(stageA(buf));
      const uint32_t b_addr = smem_u32(stageB(buf));
      for (int ks = 0; ks < ksteps; ++ks) {
        const uint64_t ad = make_sw128_desc(a_addr + ks * 4096, 1024, 2048);
        const uint64_t bd = make_sw128_desc(b_addr + ks * 32, 16, 1024);
        mma_f16_ss(tmem, ad, bd, idesc, (st > 0 || ks > 0) ? 1u : 0u);
      }
      mma_commit(&mma_bar[buf]);
    }
  }
  // wait for the last commit (all earlier MMAs complete before it)
  {
    const int last = nstage - 1;
    // always, also after an abort: no MMA may still read shared memory or write TMEM at exit
    if (!mbar_wait(&mma_bar[last & 1], (last >> 1) & 1)) abort_sh = 1;
  }
  tc_fence_after();
  __syncthreads();

  if (!abort_sh) {
    // ---- epilogue: thread = voxel (TMEM lane), 32 output channels per load ----
    const long long v = v0 + warp * 32 + lane;
    const bool vok = v < p.vox;
    const TA* aux = static_cast<const TA*>(p.aux);
    const TY* res = static_cast<const TY*>(p.residual);
    TY* Y = static_cast<TY*>(p.y);
    const int epi = p.epilogue;
    for (int c0 = 0; c0 < BN; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, r);
      tmem_ld_wait();
      float gs1 = 0.f, gs2 = 0.f;
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const int j = j0 + c0 + jj;
        float acc = __uint_as_float(r[jj]);
        float s1 = 0.f, s2 = 0.f;
        if (j < p.cout && vok) {
          const long long off = ((long long)s * p.cout + j) * p.vox + v;
          if (epi & MEDNEXT_EPI_BIAS) acc += p.bias[j];
          // the convolution result is materialised in the activation dtype
          // before any elementwise step that follows it
          if (epi & (MEDNEXT_EPI_GELU_GRAD | MEDNEXT_EPI_RESIDUAL)) acc = to_acc<TA>(from_acc<TA>(acc));
          if (epi & MEDNEXT_EPI_GELU_GRAD) acc *= gelu_grad_f(to_acc<TA>(aux[off]));
          if (epi & MEDNEXT_EPI_RESIDUAL) acc += (float)to_acc<TY>(res[off]);
          const TY out = from_acc<TY>((typename Elem<TY>::Acc)acc);
          Y[off] = out;
          if (epi & MEDNEXT_EPI_GN_BWD_STATS) {
            const float d = (float)to_acc<TY>(out);
            const float mean = p.epi_stats[2 * (s * p.cout + j)];
            const float rstd = p.epi_stats[2 * (s * p.cout + j) + 1];
            const float xh = (to_acc<TA>(aux[off]) - mean) * rstd;
            s1 = d;
            s2 = d * xh;
          }
        }
        if (epi & MEDNEXT_EPI_GN_BWD_STATS) {
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            s1 += __shfl_xor_sync(0xffffffffu, s1, o);
            s2 += __shfl_xor_sync(0xffffffffu, s2, o);
          }
          if (lane == jj) {
            gs1 = s1;
            gs2 = s2;
          }
        }
      }
      if (epi & MEDNEXT_EPI_GN_BWD_STATS) {
        // lane jj holds the warp's sums for channel c0+jj: one partial per
        // (channel, tile, 32-voxel quarter), folded later in a fixed order
        const int j = j0 + c0 + lane;
        if (j < p.cout && c0 + lane < BN) {
          GnBwdPartial gp;
          gp.s1 = (double)gs1;
          gp.s2 = (double)gs2;
          p.gn_part[(((size_t)s * p.cout + j) * p.mtiles + mt) * 4 + warp] = gp;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, ncols);
}

// ----------------------------------------------------------------------------
// Weight grad:  dw[j, k] = sum_{s,v} g[s,j,v] * pro(a[s,k,v]),  dbias[j] = sum g
// M = output channel j (128 per tile), N = input channel k (BN per tile), the
// reduction runs over 64-voxel chunks; CTAs split the chunk list and write
// fp32 partial tiles that pw_wgrad_reduce_kernel folds in a fixed order.
// ----------------------------------------------------------------------------
struct PwWgradArgs {
  const void* g;   // [S, cout, vox]
  const void* a;   // [S, cin, vox]
  const float* pro_stats;
  const float* pro_gamma;
  const float* pro_beta;
  float* part;     // [splits][cout][cin]
  float* part_b;   // [splits][cout]
  float* dw;       // [cout][cin]
  float* dbias;    // [cout] or null
  int S, cin, cout;
  long long vox;
  int BN, mtiles, ntiles, splits;
  long long chunks_per_sample, chunks_total, chunks_per_split;
  int vec;
};

template <typename TA, int PRO>
__global__ void __launch_bounds__(kPwThreads) pw_wgrad_kernel(PwWgradArgs p) {
  extern __shared__ uint8_t smem_dyn[];
  __shared__ uint64_t mma_bar[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  int b = blockIdx.x;
  const int mt = b % p.mtiles;
  b /= p.mtiles;
  const int nt = b % p.ntiles;
  const int sp = b / p.ntiles;
  const int j0 = mt * kPwBM;
  const int k0 = nt * p.BN;
  const int BN = p.BN;

  const uint32_t base_u32 = smem_u32(smem_dyn);
  const uint32_t pad = ((base_u32 + 1023u) & ~1023u) - base_u32;
  uint8_t* sbase = smem_dyn + pad;
  // stage buffer b: A at sbase + b*16 KB, B at sbase + 32 KB + b*BN*128
  auto stageA = [&](int bb) { return sbase + bb * 16384; };
  auto stageB = [&](int bb) { return sbase + 32768 + bb * BN * 128; };

  const uint32_t ncols = BN <= 32 ? 32u : (BN <= 64 ? 64u : (BN <= 128 ? 128u : 256u));
  if (warp == 0) {
    tmem_alloc(&tmem_base_sh, ncols);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&mma_bar[0], 1);
    mbar_init(&mma_bar[1], 1);
    fence_mbarrier_init();
    abort_sh = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  const TA* G = static_cast<const TA*>(p.g);
  const TA* A = static_cast<const TA*>(p.a);
  const uint32_t idesc = make_idesc_f16(kPwBM, BN, std::is_same<TA, __nv_bfloat16>::value, false, false);
  const long long cbeg = (long long)sp * p.chunks_per_split;
  const long long cend = min(cbeg + p.chunks_per_split, p.chunks_total);
  const int q = tid & 7;
  float bsum[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) bsum[i] = 0.f;

  int st = 0;
  for (long long ch = cbeg; ch < cend; ++ch, ++st) {
    const int buf = st & 1;
    const int s = (int)(ch / p.chunks_per_sample);
    const long long vb = (ch - (long long)s * p.chunks_per_sample) * kPwBK;
    if (st >= 2 && !abort_sh) {
      if (!mbar_wait(&mma_bar[buf], ((st - 2) >> 1) & 1)) abort_sh = 1;
    }
    const long long v = vb + 8 * q;
    const long long rem = p.vox - v;
    // ---- A = g rows (output channels), 128 rows x 8 chunks ----
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int n = (tid >> 3) + 16 * i;
      const int j = j0 + n;
      float vals[8];
      if (j < p.cout && rem > 0) {
        pw_load8<TA>(G + ((long long)s * p.cout + j) * p.vox + v, rem, p.vec != 0, vals);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) vals[e] = 0.f;
      }
      const uint4 pk = pw_pack<TA>(vals);
      // bias grad from the values the MMA sees (already in the input dtype)
      float unp[8];
      unpack16<TA>(pk, unp);
#pragma unroll
      for (int e = 0; e < 8; ++e) bsum[i] += unp[e];
      *reinterpret_cast<uint4*>(stageA(buf) + sw128_kmajor_off(n, q)) = pk;
    }
    // ---- B = pro(a) rows (input channels), BN rows x 8 chunks ----
    for (int n = tid >> 3; n < BN; n += kPwThreads / 8) {
      const int k = k0 + n;
      float vals[8];
      if (k < p.cin && rem > 0) {
        pw_load8<TA>(A + ((long long)s * p.cin + k) * p.vox + v, rem, p.vec != 0, vals);
        if constexpr (PRO == MEDNEXT_PRO_GROUPNORM) {
          const float mean = p.pro_stats[2 * (s * p.cin + k)];
          const float rstd = p.pro_stats[2 * (s * p.cin + k) + 1];
          const float ca = rstd * p.pro_gamma[k];
          pw_prologue<PRO>(vals, ca, p.pro_beta[k] - mean * ca);
        } else if constexpr (PRO == MEDNEXT_PRO_GELU) {
          pw_prologue<PRO>(vals, 0.f, 0.f);
        }
        if (rem < 8) {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (e >= rem) vals[e] = 0.f;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) vals[e] = 0.f;
      }
      *reinterpret_cast<uint4*>(stageB(buf) + sw128_kmajor_off(n, q)) = pw_pack<TA>(vals);
    }
    fence_async_smem();
    __syncthreads();
    if (tid == 0 && !abort_sh) {
      tc_fence_after();
      const uint32_t a_addr = smem_u32(stageA(buf));
      const uint32_t b_addr = smem_u32(stageB(buf));
#pragma unroll
      for (int ks = 0; ks < kPwBK / 16; ++ks) {
        const uint64_t ad = make_sw128_desc(a_addr + ks * 32, 16, 1024);
        const uint64_t bd = make_sw128_desc(b_addr + ks * 32, 16, 1024);
        mma_f16_ss(tmem, ad, bd, idesc, (st > 0 || ks > 0) ? 1u : 0u);
      }
      mma_commit(&mma_bar[buf]);
    }
  }
  const bool any = st > 0;
  if (any) {
    const int last = st - 1;
    // always, also after an abort: no MMA may still read shared memory or write TMEM at exit
    if (!mbar_wait(&mma_bar[last & 1], (last >> 1) & 1)) abort_sh = 1;
  }
  tc_fence_after();
  __syncthreads();

  // bias partial: rows (tid>>3)+16i, fold the 8 threads sharing them (lanes q)
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float v = bsum[i];
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    bsum[i] = v;
  }
  if (nt == 0 && q == 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int j = j0 + (tid >> 3) + 16 * i;
      if (j < p.cout) p.part_b[(size_t)sp * p.cout + j] = bsum[i];
    }
  }
  if (!abort_sh) {
    const int j = j0 + warp * 32 + lane;  // TMEM lane = output channel
    for (int c0 = 0; c0 < BN; c0 += 32) {
      uint32_t r[32];
      if (any) {
        tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, r);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) r[e] = 0u;
      }
      if (j < p.cout) {
        float* dst = p.part + ((size_t)sp * p.cout + j) * p.cin;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int k = k0 + c0 + e;
          if (k < p.cin) dst[k] = __uint_as_float(r[e]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, ncols);
}

// dw[j,k] = sum_split part[split][j][k];  dbias[j] = sum_split part_b[split][j]
// A block of kPwRedThreads reduces kPwRedThreads / groups consecutive outputs (dw
// then dbias, one index space) with `groups` split groups: group g adds splits
// g, g + groups, ... in order (loads issued four at a time), then the group sums
// are added in group order.  The order is fixed, so the result is deterministic.
// Many splits and few outputs (level 0) take 8 groups; few splits one.
constexpr int kPwRedThreads = 256;
static __global__ void __launch_bounds__(kPwRedThreads)
    pw_wgrad_reduce_kernel(const float* __restrict__ part, const float* __restrict__ part_b, float* __restrict__ dw,
                           float* __restrict__ dbias, int splits, int cout, int cin, int groups) {
  __shared__ float acc[kPwRedThreads];
  const int per = kPwRedThreads / groups;  // outputs per block
  const int o = threadIdx.x % per, g = threadIdx.x / per;
  const long long nw = (long long)cout * cin;
  const long long idx = (long long)blockIdx.x * per + o;
  const float* src = nullptr;
  size_t stride = 0;
  if (idx < nw) {
    src = part + idx;
    stride = (size_t)nw;
  } else if (idx < nw + cout) {
    src = part_b + (idx - nw);
    stride = (size_t)cout;
  }
  float sum = 0.f;
  if (src != nullptr) {
    int i = g;
    for (; i + 3 * groups < splits; i += 4 * groups) {
      const float a0 = src[(size_t)i * stride], a1 = src[(size_t)(i + groups) * stride];
      const float a2 = src[(size_t)(i + 2 * groups) * stride], a3 = src[(size_t)(i + 3 * groups) * stride];
      sum += a0;
      sum += a1;
      sum += a2;
      sum += a3;
    }
    for (; i < splits; i += groups) sum += src[(size_t)i * stride];
  }
  if (groups > 1) {
    acc[threadIdx.x] = sum;
    __syncthreads();
    if (g != 0) return;
    for (int k = 1; k < groups; ++k) sum += acc[k * per + o];
  }
  if (idx < nw) dw[idx] = sum;
  else if (idx < nw + cout && dbias != nullptr) dbias[idx - nw] = sum;
}

}  // namespace mednext
