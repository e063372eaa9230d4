// MedNeXt v2 Global Response Norm on sm_100a (forward and backward).
//
//   norm[n,c] = ||x[n,c,:]||_2,  den[n] = sum_c norm[n,c] + eps,  r = norm / den
//   y  = x + gamma[c] * x * r + beta[c]
//   dx = dy * (1 + gamma[c] r) + (norm > 0 ? x / norm : 0) * dnorm[n,c]
//   dnorm[n,c] = (gamma[c] qx[n,c] - sum_j gamma[j] qx[n,j] r[n,j]) / den[n],  qx = sum_v dy x
//   dgamma[c] = sum_n qx[n,c] r[n,c],  dbeta[c] = sum_n sum_v dy[n,c,v]
// Reference: ops/grn.py:16-29 (formula), ops/_triton/grn.py:235-402 (the fused op's
// forward/backward split and its saved statistics norm and den).
//
// Every pass is HBM-bound: the forward reads x twice and writes y once, the
// backward reads dy and x twice and writes dx once.  Rows ([n, c] slices of
// `spatial` voxels) are cut into fixed work items of kItem voxels; a persistent
// grid walks the items round-robin, so the work is balanced whatever the number
// of rows, and each item's partial sum has a fixed slot, so the two-pass
// reductions are deterministic.  Rows whose start is 16-byte aligned are moved
// with 16-byte vector loads and stores.
#include "plan.h"

#include <math.h>

namespace mednext {
namespace {

constexpr int kGrnThreads = 256;
constexpr long long kItem = 16384;  // voxels per work item (a multiple of 8)

struct GrnGeom {
  long long rows;    // n * c
  long long vox;     // voxels per row
  long long splits;  // items per row
  int c;
  int vec;           // 1: every row is 16-byte aligned (vector path)
};

template <typename T>
__device__ __forceinline__ void load8(const T* p, float* v) {
  unpack16<T>(__ldg(reinterpret_cast<const uint4*>(p)), v);
}

// Sum over the CTA of one float per thread, fixed order: butterfly within each
// warp, then warp 0 adds the 8 warp sums in warp order.  Result valid in thread 0.
__device__ __forceinline__ float cta_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red[] may still be read by the previous call
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  if (threadIdx.x == 0)
    for (int w = 0; w < kGrnThreads / 32; ++w) s += red[w];
  return s;
}

// part[row * splits + item] = sum over the item's voxels of a*b (B != nullptr) or a*a;
// part2 (optional) = sum of a.
template <typename T, bool TWO>
__global__ void __launch_bounds__(kGrnThreads) grn_partial_kernel(const T* __restrict__ a, const T* __restrict__ b,
                                                                   float* __restrict__ part,
                                                                   float* __restrict__ part2, GrnGeom g) {
  __shared__ float red[kGrnThreads / 32];
  const long long items = g.rows * g.splits;
  for (long long it = blockIdx.x; it < items; it += gridDim.x) {
    const long long row = it / g.splits, sp = it - row * g.splits;
    const long long v0 = sp * kItem;
    const long long v1 = min(v0 + kItem, g.vox);
    const T* ar = a + row * g.vox;
    const T* br = b != nullptr ? b + row * g.vox : nullptr;
    float s1 = 0.f, s2 = 0.f;
    if (g.vec) {
      // v0 is a multiple of 8; the ragged end of the row is handled element-wise
      const long long vend = v0 + ((v1 - v0) & ~7LL);
      for (long long v = v0 + 8LL * threadIdx.x; v < vend; v += 8LL * kGrnThreads) {
        float x[8], y[8];
        load8<T>(ar + v, x);
        if (br != nullptr) load8<T>(br + v, y);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (br != nullptr) {
            s1 = fmaf(x[i], y[i], s1);
            if (TWO) s2 += x[i];
          } else {
            s1 = fmaf(x[i], x[i], s1);
          }
        }
      }
      for (long long v = vend + threadIdx.x; v < v1; v += kGrnThreads) {
        const float x = to_acc<T>(ar[v]);
        const float y = br != nullptr ? to_acc<T>(br[v]) : x;
        s1 = fmaf(x, y, s1);
        if (TWO) s2 += x;
      }
    } else {
      for (long long v = v0 + threadIdx.x; v < v1; v += kGrnThreads) {
        const float x = to_acc<T>(ar[v]);
        const float y = br != nullptr ? to_acc<T>(br[v]) : x;
        s1 = fmaf(x, y, s1);
        if (TWO) s2 += x;
      }
    }
    const float t1 = cta_sum(s1, red);
    float t2 = 0.f;
    if (TWO) t2 = cta_sum(s2, red);
    if (threadIdx.x == 0) {
      part[it] = t1;
      if (TWO) part2[it] = t2;
    }
  }
}

// One CTA per sample: norm[n,c] = sqrt(sum of the row's partials), den[n] = sum_c norm + eps.
__global__ void __launch_bounds__(kGrnThreads) grn_fwd_finish_kernel(const float* __restrict__ part,
                                                                      float* __restrict__ norm,
                                                                      float* __restrict__ den, GrnGeom g,
                                                                      float eps) {
  __shared__ float red[kGrnThreads / 32];
  const long long n = blockIdx.x;
  float local = 0.f;
  for (int c = threadIdx.x; c < g.c; c += kGrnThreads) {
    const float* p = part + (n * g.c + c) * g.splits;
    float s = 0.f;
    for (long long i = 0; i < g.splits; ++i) s += p[i];
    const float nv = __fsqrt_rn(s);
    norm[n * g.c + c] = nv;
    local += nv;
  }
  const float total = cta_sum(local, red);
  if (threadIdx.x == 0) den[n] = total + eps;
}

// y = x + x * (gamma r) + beta, r = norm / den (per row).
template <typename T>
__global__ void __launch_bounds__(kGrnThreads) grn_apply_kernel(const T* __restrict__ x, const float* __restrict__ gamma,
                                                                 const float* __restrict__ beta,
                                                                 const float* __restrict__ norm,
                                                                 const float* __restrict__ den, T* __restrict__ y,
                                                                 GrnGeom g) {
  const long long items = g.rows * g.splits;
  for (long long it = blockIdx.x; it < items; it += gridDim.x) {
    const long long row = it / g.splits, sp = it - row * g.splits;
    const long long n = row / g.c;
    const int c = (int)(row - n * g.c);
    const float a = gamma[c] * __fdiv_rn(norm[row], den[n]);
    const float b = beta[c];
    const long long v0 = sp * kItem, v1 = min(v0 + kItem, g.vox);
    const T* xr = x + row * g.vox;
    T* yr = y + row * g.vox;
    long long vend = v0;
    if (g.vec) {
      vend = v0 + ((v1 - v0) & ~7LL);
      for (long long v = v0 + 8LL * threadIdx.x; v < vend; v += 8LL * kGrnThreads) {
        float e[8];
        load8<T>(xr + v, e);
#pragma unroll
        for (int i = 0; i < 8; ++i) e[i] = fmaf(e[i], a, e[i]) + b;
        *reinterpret_cast<uint4*>(yr + v) = pack16<T>(e);
      }
    }
    for (long long v = vend + threadIdx.x; v < v1; v += kGrnThreads) {
      const float e = to_acc<T>(xr[v]);
      yr[v] = from_acc<T>(fmaf(e, a, e) + b);
    }
  }
}

// One CTA per sample: from the partials of sum(dy x) and sum(dy), the row
// gradient of the norm (gn), and per-sample dgamma / dbeta contributions.
__global__ void __launch_bounds__(kGrnThreads) grn_bwd_finish_kernel(
    const float* __restrict__ pqx, const float* __restrict__ pq, const float* __restrict__ gamma,
    const float* __restrict__ norm, const float* __restrict__ den, float* __restrict__ gn, float* __restrict__ bdg,
    float* __restrict__ bdb, GrnGeom g) {
  __shared__ float red[kGrnThreads / 32];
  __shared__ float coupled_s;
  const long long n = blockIdx.x;
  const float dn = den[n];
  float local = 0.f;
  for (int c = threadIdx.x; c < g.c; c += kGrnThreads) {
    const long long row = n * g.c + c;
    float qx = 0.f, q = 0.f;
    for (long long i = 0; i < g.splits; ++i) {
      qx += pqx[row * g.splits + i];
      q += pq[row * g.splits + i];
    }
    const float r = __fdiv_rn(norm[row], dn);
    const float h = gamma[c] * qx;
    gn[row] = h;  // finished below, once the coupling term is known
    bdg[row] = qx * r;
    bdb[row] = q;
    local = fmaf(h, r, local);
  }
  const float coupled = cta_sum(local, red);
  if (threadIdx.x == 0) coupled_s = coupled;
  __syncthreads();
  for (int c = threadIdx.x; c < g.c; c += kGrnThreads) {
    const long long row = n * g.c + c;
    gn[row] = __fdiv_rn(gn[row] - coupled_s, dn);
  }
}

// dgamma[c] = sum_n bdg[n,c], dbeta[c] = sum_n bdb[n,c], in sample order.
__global__ void grn_affine_grad_kernel(const float* __restrict__ bdg, const float* __restrict__ bdb,
                                       float* __restrict__ dgamma, float* __restrict__ dbeta, long long nsamples,
                                       int c) {
  const int ch = blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= c) return;
  float sg = 0.f, sb = 0.f;
  for (long long n = 0; n < nsamples; ++n) {
    sg += bdg[n * c + ch];
    sb += bdb[n * c + ch];
  }
  dgamma[ch] = sg;
  dbeta[ch] = sb;
}

// dx = dy (1 + gamma r) + x (gn / norm)  (the second term is zero where norm == 0).
template <typename T>
__global__ void __launch_bounds__(kGrnThreads) grn_bwd_apply_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                                     const float* __restrict__ gamma,
                                                                     const float* __restrict__ norm,
                                                                     const float* __restrict__ den,
                                                                     const float* __restrict__ gn, T* __restrict__ dx,
                                                                     GrnGeom g) {
  const long long items = g.rows * g.splits;
  for (long long it = blockIdx.x; it < items; it += gridDim.x) {
    const long long row = it / g.splits, sp = it - row * g.splits;
    const long long n = row / g.c;
    const int c = (int)(row - n * g.c);
    const float nv = norm[row];
    const float k1 = 1.0f + gamma[c] * __fdiv_rn(nv, den[n]);
    const float k2 = nv > 0.f ? __fdiv_rn(gn[row], nv) : 0.f;
    const long long v0 = sp * kItem, v1 = min(v0 + kItem, g.vox);
    const T* qr = dy + row * g.vox;
    const T* xr = x + row * g.vox;
    T* out = dx + row * g.vox;
    long long vend = v0;
    if (g.vec) {
      vend = v0 + ((v1 - v0) & ~7LL);
      for (long long v = v0 + 8LL * threadIdx.x; v < vend; v += 8LL * kGrnThreads) {
        float q[8], e[8];
        load8<T>(qr + v, q);
        load8<T>(xr + v, e);
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = fmaf(e[i], k2, q[i] * k1);
        *reinterpret_cast<uint4*>(out + v) = pack16<T>(q);
      }
    }
    for (long long v = vend + threadIdx.x; v < v1; v += kGrnThreads) {
      const float q = to_acc<T>(qr[v]), e = to_acc<T>(xr[v]);
      out[v] = from_acc<T>(fmaf(e, k2, q * k1));
    }
  }
}

bool grn_dtype_ok(int d) { return d == MEDNEXT_FLOAT32 || d == MEDNEXT_BFLOAT16 || d == MEDNEXT_FLOAT16; }

int grn_geom(int64_t n, int64_t c, int64_t spatial, int dtype, GrnGeom* g) {
  if (!grn_dtype_ok(dtype)) return MEDNEXT_ERR_BAD_DTYPE;
  if (n <= 0 || c <= 0 || spatial <= 0 || c >= ((int64_t)1 << 30) || n * c >= ((int64_t)1 << 40) ||
      spatial >= ((int64_t)1 << 40))
    return MEDNEXT_ERR_BAD_SHAPE;
  g->rows = n * c;
  g->vox = spatial;
  g->splits = (spatial + kItem - 1) / kItem;
  g->c = (int)c;
  g->vec = 0;
  return MEDNEXT_OK;
}

size_t grn_ws_bytes(const GrnGeom& g) {
  // backward: two partial arrays, gn, bdg, bdb; the forward uses the first array only
  return (size_t)(2 * g.rows * g.splits + 3 * g.rows) * sizeof(float);
}

int grn_grid(const GrnGeom& g) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long items = g.rows * g.splits;
  return (int)std::min<long long>(items, (long long)std::max(sms, 1) * (2048 / kGrnThreads));
}

template <typename T>
bool rows_aligned(const void* p, const GrnGeom& g) {
  const long long per = 16 / (long long)sizeof(T);
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0 && g.vox % per == 0;
}

template <typename T>
int grn_fwd_t(const void* x, const float* gamma, const float* beta, void* y, float* norm, float* den, float* ws,
              GrnGeom g, float eps, cudaStream_t s) {
  g.vec = sizeof(T) == 2 && rows_aligned<T>(x, g) && rows_aligned<T>(y, g);
  const int grid = grn_grid(g);
  grn_partial_kernel<T, false><<<grid, kGrnThreads, 0, s>>>(static_cast<const T*>(x), nullptr, ws, nullptr, g);
  int st = record_launch();
  if (st != MEDNEXT_OK) return st;
  grn_fwd_finish_kernel<<<(unsigned)(g.rows / g.c), kGrnThreads, 0, s>>>(ws, norm, den, g, eps);
  if ((st = record_launch()) != MEDNEXT_OK) return st;
  grn_apply_kernel<T><<<grid, kGrnThreads, 0, s>>>(static_cast<const T*>(x), gamma, beta, norm, den,
                                                   static_cast<T*>(y), g);
  return record_launch();
}

template <typename T>
int grn_bwd_t(const void* dy, const void* x, const float* gamma, const float* norm, const float* den, void* dx,
              float* dgamma, float* dbeta, float* ws, GrnGeom g, cudaStream_t s) {
  g.vec = sizeof(T) == 2 && rows_aligned<T>(x, g) && rows_aligned<T>(dy, g) && rows_aligned<T>(dx, g);
  const long long np = g.rows * g.splits;
  float* pqx = ws;
  float* pq = ws + np;
  float* gn = ws + 2 * np;
  float* bdg = gn + g.rows;
  float* bdb = bdg + g.rows;
  const int grid = grn_grid(g);
  const long long nsamples = g.rows / g.c;
  grn_partial_kernel<T, true><<<grid, kGrnThreads, 0, s>>>(static_cast<const T*>(dy), static_cast<const T*>(x), pqx,
                                                           pq, g);
  int st = record_launch();
  if (st != MEDNEXT_OK) return st;
  grn_bwd_finish_kernel<<<(unsigned)nsamples, kGrnThreads, 0, s>>>(pqx, pq, gamma, norm, den, gn, bdg, bdb, g);
  if ((st = record_launch()) != MEDNEXT_OK) return st;
  grn_affine_grad_kernel<<<(unsigned)((g.c + 255) / 256), 256, 0, s>>>(bdg, bdb, dgamma, dbeta, nsamples, g.c);
  if ((st = record_launch()) != MEDNEXT_OK) return st;
  grn_bwd_apply_kernel<T><<<grid, kGrnThreads, 0, s>>>(static_cast<const T*>(dy), static_cast<const T*>(x), gamma,
                                                       norm, den, gn, static_cast<T*>(dx), g);
  return record_launch();
}

}  // namespace
}  // namespace mednext

using namespace mednext;

size_t mednext_grn_workspace_size(int64_t n, int64_t c, int64_t spatial, int dtype) {
  GrnGeom g;
  if (grn_geom(n, c, spatial, dtype, &g) != MEDNEXT_OK) return 0;
  return grn_ws_bytes(g);
}

int mednext_grn_fwd(const void* x, const float* gamma, const float* beta, void* y, float* norm, float* denom,
                    void* workspace, size_t workspace_bytes, int64_t n, int64_t c, int64_t spatial, float eps,
                    int dtype, mednext_stream_t stream) {
  GrnGeom g;
  const int st = grn_geom(n, c, spatial, dtype, &g);
  if (st != MEDNEXT_OK) return st;
  if (!(eps > 0.f) || !isfinite(eps)) return MEDNEXT_ERR_BAD_VALUE;
  if (!x || !gamma || !beta || !y || !norm || !denom) return MEDNEXT_ERR_NULL_POINTER;
  if (!workspace || workspace_bytes < grn_ws_bytes(g)) return MEDNEXT_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 3) != 0) return MEDNEXT_ERR_ALIGNMENT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  float* ws = static_cast<float*>(workspace);
  switch (dtype) {
    case MEDNEXT_FLOAT32: return grn_fwd_t<float>(x, gamma, beta, y, norm, denom, ws, g, eps, s);
    case MEDNEXT_BFLOAT16: return grn_fwd_t<__nv_bfloat16>(x, gamma, beta, y, norm, denom, ws, g, eps, s);
    default: return grn_fwd_t<__half>(x, gamma, beta, y, norm, denom, ws, g, eps, s);
  }
}

int mednext_grn_bwd(const void* dy, const void* x, const float* gamma, const float* norm, const float* denom, void* dx,
                    float* dgamma, float* dbeta, void* workspace, size_t workspace_bytes, int64_t n, int64_t c,
                    int64_t spatial, int dtype, mednext_stream_t stream) {
  GrnGeom g;
  const int st = grn_geom(n, c, spatial, dtype, &g);
  if (st != MEDNEXT_OK) return st;
  if (!dy || !x || !gamma || !norm || !denom || !dx || !dgamma || !dbeta) return MEDNEXT_ERR_NULL_POINTER;
  if (!workspace || workspace_bytes < grn_ws_bytes(g)) return MEDNEXT_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 3) != 0) return MEDNEXT_ERR_ALIGNMENT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  float* ws = static_cast<float*>(workspace);
  switch (dtype) {
    case MEDNEXT_FLOAT32: return grn_bwd_t<float>(dy, x, gamma, norm, denom, dx, dgamma, dbeta, ws, g, s);
    case MEDNEXT_BFLOAT16: return grn_bwd_t<__nv_bfloat16>(dy, x, gamma, norm, denom, dx, dgamma, dbeta, ws, g, s);
    default: return grn_bwd_t<__half>(dy, x, gamma, norm, denom, dx, dgamma, dbeta, ws, g, s);
  }
}
