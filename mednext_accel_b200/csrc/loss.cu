// Mean cross-entropy over the class axis of [N, K, V] logits (F.cross_entropy with
// reduction="mean" and ignore_index), the deep-supervision loss of the training
// step (benchmarks/implementations.py:133-190 of the reference: five heads, three
// classes).  Forward: per-voxel log-sum-exp and target logit, fp32 arithmetic on
// the stored logits, deterministic block partials folded in a fixed order into
// out = {mean loss, number of counted targets}.  Backward: d logits = (softmax -
// onehot(target)) * grad / count, recomputed from the logits, in the logits' type.
#include "plan.h"

namespace mednext {
namespace {

constexpr int kCeThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kCeThreads) ce_partial_kernel(const T* __restrict__ logits,
                                                                const int64_t* __restrict__ target,
                                                                double* __restrict__ part, int K, long long V,
                                                                long long total, long long ignore_index) {
  double loss = 0.0, cnt = 0.0;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long n = i / V, v = i - n * V;
    const long long t = target[i];
    if (t == ignore_index) continue;
    if (t < 0 || t >= K) {
      raise_device_error(kErrBadTarget);
      continue;
    }
    const T* x = logits + (size_t)n * K * V + v;
    float m = -INFINITY;
    for (int k = 0; k < K; ++k) m = fmaxf(m, to_acc<T>(x[(size_t)k * V]));
    float se = 0.f;
    for (int k = 0; k < K; ++k) se += expf(to_acc<T>(x[(size_t)k * V]) - m);
    loss += (double)(logf(se) + m - to_acc<T>(x[(size_t)t * V]));
    cnt += 1.0;
  }
  __shared__ double sl[kCeThreads], sc[kCeThreads];
  sl[threadIdx.x] = loss;
  sc[threadIdx.x] = cnt;
  __syncthreads();
  for (int o = kCeThreads / 2; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) {
      sl[threadIdx.x] += sl[threadIdx.x + o];
      sc[threadIdx.x] += sc[threadIdx.x + o];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    part[2 * blockIdx.x] = sl[0];
    part[2 * blockIdx.x + 1] = sc[0];
  }
}

// out[0] = sum(loss) / count (NaN when nothing is counted, as torch), out[1] = count.
// One block: strided per-thread sums, then a tree, both in a fixed order.
__global__ void __launch_bounds__(kCeThreads) ce_finish_kernel(const double* __restrict__ part, int blocks,
                                                               float* __restrict__ out) {
  __shared__ double sl[kCeThreads], sc[kCeThreads];
  double l = 0.0, c = 0.0;
  for (int b = threadIdx.x; b < blocks; b += kCeThreads) {
    l += part[2 * b];
    c += part[2 * b + 1];
  }
  sl[threadIdx.x] = l;
  sc[threadIdx.x] = c;
  __syncthreads();
  for (int o = kCeThreads / 2; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) {
      sl[threadIdx.x] += sl[threadIdx.x + o];
      sc[threadIdx.x] += sc[threadIdx.x + o];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    out[0] = (float)(sl[0] / sc[0]);
    out[1] = (float)sc[0];
  }
}

template <typename T>
__global__ void __launch_bounds__(kCeThreads) ce_backward_kernel(const T* __restrict__ logits,
                                                                 const int64_t* __restrict__ target,
                                                                 const float* __restrict__ fwd_out,
                                                                 const float* __restrict__ grad_loss,
                                                                 T* __restrict__ grad, int K, long long V,
                                                                 long long total, long long ignore_index) {
  const float scale = grad_loss[0] / fwd_out[1];
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long n = i / V, v = i - n * V;
    const long long t = target[i];
    const T* x = logits + (size_t)n * K * V + v;
    T* g = grad + (size_t)n * K * V + v;
    if (t == ignore_index || t < 0 || t >= K) {
      for (int k = 0; k < K; ++k) g[(size_t)k * V] = from_acc<T>(0.0f);
      continue;
    }
    float m = -INFINITY;
    for (int k = 0; k < K; ++k) m = fmaxf(m, to_acc<T>(x[(size_t)k * V]));
    float se = 0.f;
    for (int k = 0; k < K; ++k) se += expf(to_acc<T>(x[(size_t)k * V]) - m);
    const float inv = 1.0f / se;
    for (int k = 0; k < K; ++k) {
      const float p = expf(to_acc<T>(x[(size_t)k * V]) - m) * inv;
      g[(size_t)k * V] = from_acc<T>((p - (k == t ? 1.0f : 0.0f)) * scale);
    }
  }
}

int ce_blocks(long long total) {
  return (int)std::max(1LL, std::min((total + kCeThreads - 1) / kCeThreads, 148LL * 8));
}

template <typename T>
int launch_ce_fwd(const void* logits, const int64_t* target, double* part, float* out, int K, long long V,
                  long long total, long long ignore_index, cudaStream_t s) {
  const int blocks = ce_blocks(total);
  ce_partial_kernel<T><<<blocks, kCeThreads, 0, s>>>(static_cast<const T*>(logits), target, part, K, V, total,
                                                     ignore_index);
  int st = record_launch();
  if (st != MEDNEXT_OK) return st;
  ce_finish_kernel<<<1, kCeThreads, 0, s>>>(part, blocks, out);
  return record_launch();
}

template <typename T>
int launch_ce_bwd(const void* logits, const int64_t* target, const float* out, const float* grad_loss, void* grad,
                  int K, long long V, long long total, long long ignore_index, cudaStream_t s) {
  ce_backward_kernel<T><<<ce_blocks(total), kCeThreads, 0, s>>>(static_cast<const T*>(logits), target, out,
                                                                grad_loss, static_cast<T*>(grad), K, V, total,
                                                                ignore_index);
  return record_launch();
}

bool ce_args_ok(int64_t n, int64_t k, int64_t v) { return n > 0 && k > 0 && k <= 1024 && v > 0 && n * v < (1LL << 40); }

}  // namespace

MEDNEXT_DEFINE_ERROR_READER(read_clear_errors_loss)

}  // namespace mednext

using namespace mednext;

size_t mednext_ce_workspace_size(int64_t n, int64_t k, int64_t v) {
  if (!ce_args_ok(n, k, v)) return 0;
  return (size_t)ce_blocks(n * v) * 2 * sizeof(double);
}

int mednext_ce_fwd(const void* logits, const int64_t* target, float* out, void* workspace, size_t workspace_bytes,
                   int64_t n, int64_t k, int64_t v, int64_t ignore_index, int dtype, mednext_stream_t stream) {
  if (!ce_args_ok(n, k, v)) return MEDNEXT_ERR_BAD_SHAPE;
  if (logits == nullptr || target == nullptr || out == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 7) ||
      workspace_bytes < mednext_ce_workspace_size(n, k, v))
    return MEDNEXT_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(target) & 7) || (reinterpret_cast<uintptr_t>(out) & 3)) return MEDNEXT_ERR_ALIGNMENT;
  double* part = static_cast<double*>(workspace);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case MEDNEXT_FLOAT32: return launch_ce_fwd<float>(logits, target, part, out, (int)k, v, n * v, ignore_index, s);
    case MEDNEXT_BFLOAT16:
      return launch_ce_fwd<__nv_bfloat16>(logits, target, part, out, (int)k, v, n * v, ignore_index, s);
    case MEDNEXT_FLOAT16: return launch_ce_fwd<__half>(logits, target, part, out, (int)k, v, n * v, ignore_index, s);
    default: return MEDNEXT_ERR_BAD_DTYPE;
  }
}

int mednext_ce_bwd(const void* logits, const int64_t* target, const float* fwd_out, const float* grad_loss,
                   void* grad, int64_t n, int64_t k, int64_t v, int64_t ignore_index, int dtype,
                   mednext_stream_t stream) {
  if (!ce_args_ok(n, k, v)) return MEDNEXT_ERR_BAD_SHAPE;
  if (logits == nullptr || target == nullptr || fwd_out == nullptr || grad_loss == nullptr || grad == nullptr)
    return MEDNEXT_ERR_NULL_POINTER;
  if ((reinterpret_cast<uintptr_t>(target) & 7)) return MEDNEXT_ERR_ALIGNMENT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case MEDNEXT_FLOAT32:
      return launch_ce_bwd<float>(logits, target, fwd_out, grad_loss, grad, (int)k, v, n * v, ignore_index, s);
    case MEDNEXT_BFLOAT16:
      return launch_ce_bwd<__nv_bfloat16>(logits, target, fwd_out, grad_loss, grad, (int)k, v, n * v, ignore_index,
                                          s);
    case MEDNEXT_FLOAT16:
      return launch_ce_bwd<__half>(logits, target, fwd_out, grad_loss, grad, (int)k, v, n * v, ignore_index, s);
    default: return MEDNEXT_ERR_BAD_DTYPE;
  }
}
