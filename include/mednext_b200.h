/*
 * mednext_b200.h — C ABI of the B200 (sm_100a) MedNeXt training operators.
 *
 * Every entry point takes plain device pointers, element counts and a CUDA
 * stream, launches its kernels asynchronously on that stream, and returns a
 * mednext_status code.  Nothing here allocates device memory: scratch space is
 * passed in by the caller (query its size with the matching *_workspace_size
 * function).  Tensors are contiguous NCDHW, exactly as the reference package
 * keeps them (mednext_accel/ops/adaptive.py:265 requires contiguous input).
 *
 * Reference interfaces replaced (paths inside the reference project
 * nanaHa1003/mednext-accel, src/mednext_accel/):
 *   mednext_dw_fwd        F.conv3d forward inside the custom op
 *                         depthwise_conv3d_odd_regular, ops/_triton/depthwise.py:549-563
 *   mednext_dw_dgrad      _depthwise_input_grad_kernel / depthwise_input_grad_regular,
 *                         ops/_triton/depthwise.py:159-203, 486-513
 *   mednext_dw_wgrad      _partial_dw_kernel + _finish_dw_kernel /
 *                         depthwise_weight_grad_regular, ops/_triton/depthwise.py:13-83, 445-483
 *                         (+ the native bias grad, ops/_triton/depthwise.py:613-633)
 *   mednext_dw_s2_fwd     F.conv3d stride 2 in depthwise_conv3d_stride2_regular,
 *                         ops/_triton/depthwise.py:654-666
 *   mednext_dw_s2_dgrad   _depthwise_stride2_input_grad_kernel /
 *                         depthwise_input_grad_stride2_regular, ops/_triton/depthwise.py:206-268, 516-546
 *   mednext_dw_s2_wgrad   native aten.convolution_backward dW of the stride-2 op,
 *                         ops/_triton/depthwise.py:698-713
 *   mednext_dwT_fwd       F.conv_transpose3d in depthwise_conv_transpose3d_odd_regular,
 *                         ops/_triton/depthwise.py:768-781
 *   mednext_dwT_dgrad     native aten.convolution_backward dX of the transpose op,
 *                         ops/_triton/depthwise.py:810-825
 *   mednext_dwT_wgrad     _partial_transpose_dw_kernel + _finish_dw_kernel /
 *                         depthwise_transpose_weight_grad_regular, ops/_triton/depthwise.py:86-156, 722-765
 *   mednext_gn_*          nn.GroupNorm(C, C) of MedNeXtBlock, models/blocks.py:74
 *   mednext_pw_*          AdaptivePointwise3d._gemm / F.conv3d 1x1x1, ops/adaptive.py:174-200,
 *                         with the GroupNorm apply, exact GELU (models/blocks.py:32-44) and the
 *                         residual add (models/blocks.py:89-90) fused into prologue/epilogue
 *   mednext_grn_*         the v2 Global Response Norm fused op mednext_accel::grn_forward /
 *                         grn_backward, ops/_triton/grn.py:235-402 (formula ops/grn.py:16-29)
 */
#ifndef MEDNEXT_B200_H
#define MEDNEXT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t; NULL means the legacy default stream. */
typedef struct CUstream_st* mednext_stream_t;

/* Element types.  Depthwise and GroupNorm kernels accept all four; the
 * tensor-core pointwise kernels accept BFLOAT16 and FLOAT16. */
enum mednext_dtype {
  MEDNEXT_FLOAT32 = 0,
  MEDNEXT_BFLOAT16 = 1,
  MEDNEXT_FLOAT16 = 2,
  MEDNEXT_FLOAT64 = 3
};

enum mednext_status {
  MEDNEXT_OK = 0,
  MEDNEXT_ERR_NULL_POINTER = 1, /* a required pointer is NULL */
  MEDNEXT_ERR_BAD_SHAPE = 2,    /* a size is non-positive, inconsistent or too large */
  MEDNEXT_ERR_BAD_KERNEL = 3,   /* kernel size is not one of 1, 3, 5, 7 */
  MEDNEXT_ERR_BAD_DTYPE = 4,    /* dtype not supported by this entry point */
  MEDNEXT_ERR_WORKSPACE = 5,    /* workspace missing or smaller than *_workspace_size */
  MEDNEXT_ERR_ALIGNMENT = 6,    /* a pointer is not aligned to its element size */
  MEDNEXT_ERR_CUDA = 7,         /* a CUDA launch failed (see mednext_last_cuda_error) */
  MEDNEXT_ERR_DEVICE = 8,       /* current device is not sm_100 */
  MEDNEXT_ERR_SCRATCH_LIMIT = 9, /* shape needs more than MEDNEXT_DW_WGRAD_NOALLOC_MAX_SCRATCH */
  MEDNEXT_ERR_UNSUPPORTED = 10,  /* a fused entry point does not cover this shape: run the parts */
  MEDNEXT_ERR_BAD_VALUE = 11     /* a scalar argument is out of range (e.g. eps not finite and > 0) */
};

/* Pointwise prologue applied to the activation operand while it is staged
 * into shared memory, and epilogue applied to the accumulator tile. */
enum mednext_pw_prologue {
  MEDNEXT_PRO_NONE = 0,
  MEDNEXT_PRO_GROUPNORM = 1, /* a <- (a - mean[n,k]) * rstd[n,k] * gamma[k] + beta[k] */
  MEDNEXT_PRO_GELU = 2       /* a <- gelu(a), exact erf form */
};
enum mednext_pw_epilogue {
  MEDNEXT_EPI_BIAS = 1,          /* y += bias[j] */
  MEDNEXT_EPI_RESIDUAL = 2,      /* y += residual[n, j, v] */
  MEDNEXT_EPI_GELU_GRAD = 4,     /* y *= gelu'(aux[n, j, v]) */
  MEDNEXT_EPI_GN_BWD_STATS = 8   /* also emit per-tile sums of y and y*xhat(aux) for GroupNorm backward */
};

int mednext_abi_version(void);
const char* mednext_status_string(int status);
/* Last CUDA runtime error seen by this library on the calling thread. */
int mednext_last_cuda_error(void);
/* Device-side error word: kernels with bounded waits set it instead of hanging.
 * Copies the word to *code and clears it (synchronous on the given stream). */
int mednext_device_error(int* code, mednext_stream_t stream);
/* Returns MEDNEXT_OK when the current device is sm_100 (B200). */
int mednext_check_device(void);
/* Number of kernels this library has launched in this process (all threads). */
uint64_t mednext_kernel_launches(void);

/* ---------------- depthwise Conv3d, stride 1, padding k/2 ----------------
 * x, y: [n, c, d, h, w]; weight: [c, 1, k, k, k]; bias: [c] or NULL.
 * If gn_stats is non-NULL the kernel also produces, for GroupNorm(c, c) on y,
 * the per-(n, c) mean and 1/sqrt(var + eps) as gn_stats[2*(n*c+i)+{0,1}];
 * that needs mednext_dw_fwd_workspace_size() bytes of workspace. */
size_t mednext_dw_fwd_workspace_size(int64_t n, int64_t c, int64_t d, int64_t h, int64_t w,
                                     int k, int dtype);
int mednext_dw_fwd(const void* x, const void* weight, const void* bias, void* y,
                   float* gn_stats, float gn_eps, void* workspace, size_t workspace_bytes,
                   int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k, int dtype,
                   mednext_stream_t stream);
/* dx = correlation of dy with the spatially flipped weight (same shapes as fwd),
 * plus addend (same shape, may be NULL) — the block's residual branch. */
int mednext_dw_dgrad(const void* dy, const void* weight, const void* addend, void* dx,
                     int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k, int dtype,
                     mednext_stream_t stream);
/* dweight[c,0,kd,kh,kw] = sum over n, positions of x(shifted) * dy; dbias = sum of dy
 * (dbias may be NULL).  Deterministic: fixed-order two-pass reduction. */
/* The kernel family and tiling that mednext_dw_fwd / mednext_dw_dgrad (wgrad = 0)
 * or mednext_dw_wgrad (wgrad = 1) choose for this shape (16-byte aligned
 * operands), with no launch: out[8] = {family, tile W, tile H, tile D, tiles along
 * W, H, D, CTAs}.  Families are the MEDNEXT_DWPLAN_* values.  No reference
 * counterpart: it replaces the reference's per-shape auto-tuning record
 * (optimization/*), which a fixed sm_100a table reports from here. */
enum {
  MEDNEXT_DWPLAN_GENERIC = 0,       /* per-output loads (fp64, unaligned rows) */
  MEDNEXT_DWPLAN_PACKED_FMA = 1,    /* k3, 16-bit: TMA plane ring, packed fp32 FMAs */
  MEDNEXT_DWPLAN_TENSOR_CORES = 2,  /* k5/k7, 16-bit: banded MMA, TMEM accumulators */
  MEDNEXT_DWPLAN_TMA_RING = 3,      /* TMA plane ring, scalar FMAs (16-bit weight grads: fp32 sums of 16-bit operands) */
  MEDNEXT_DWPLAN_GROUPED = 4,       /* weight grad k >= 5: taps split by kd across thread groups */
  MEDNEXT_DWPLAN_GROUPED_TMA_RING = 5  /* the same on a TMA plane ring with a producer warp */
};
int mednext_dw_plan(int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k, int dtype, int wgrad,
                    int32_t* out);
size_t mednext_dw_wgrad_workspace_size(int64_t n, int64_t c, int64_t d, int64_t h, int64_t w,
                                       int k, int dtype);
int mednext_dw_wgrad(const void* x, const void* dy, void* dweight, void* dbias, void* workspace,
                     size_t workspace_bytes, int64_t n, int64_t c, int64_t d, int64_t h,
                     int64_t w, int k, int dtype, mednext_stream_t stream);
/* The same weight grad with dweight / dbias written as fp32 (dtype bf16, fp16 or fp32):
 * the values mednext_dw_wgrad writes in dtype, widened, i.e. what casting its output to
 * fp32 gives (an autocast gradient reaching an fp32 parameter), without the cast. */
int mednext_dw_wgrad_f32out(const void* x, const void* dy, void* dweight, void* dbias,
                            void* workspace, size_t workspace_bytes, int64_t n, int64_t c,
                            int64_t d, int64_t h, int64_t w, int k, int dtype,
                            mednext_stream_t stream);

/* Same result as mednext_dw_wgrad, but the caller passes no workspace and the
 * call allocates no device memory.  No reference counterpart: the reference
 * lets torch allocate its partial-sum buffer inside the op.
 *
 * Who needs it: a host that cannot hand the library a workspace, e.g. a C or
 * FFI host that takes its whole device-memory budget at start-up and has no
 * allocator it can call per shape, or one that keeps cudaMalloc/cudaFree out
 * of its training loop because cudaFree synchronises the whole device.
 *
 * The partial sums live in one array compiled into the library, one copy per
 * device, of MEDNEXT_DW_WGRAD_NOALLOC_MAX_SCRATCH bytes (created when the
 * library's module is loaded on that device).  A shape whose
 * mednext_dw_wgrad_workspace_size() exceeds that returns
 * MEDNEXT_ERR_SCRATCH_LIMIT before anything is launched; use mednext_dw_wgrad
 * with a caller workspace for it.  16 MiB covers every MedNeXt stage up to
 * 2 x 64 x 160^3 at k = 7 (13.4 MiB).
 * Nothing in the array has to start at zero: each call writes every partial
 * sum before it reads it.
 * The first call on each device does one-time set-up with that device current
 * (it looks up the array's device address, which loads the library's module
 * on the device if needed); make that first call before any stream capture
 * begins.  The looked-up address is kept for the life of the process: after
 * cudaDeviceReset(), or any other teardown of the device's primary context,
 * the array may move, so a process that resets a device must not call this
 * entry point on that device again.
 * All calls on one device share the array: two calls that can run at the same
 * time (different streams with no ordering between them, or several host
 * threads) race on it and produce wrong gradients.  Calls issued in order on
 * one stream are safe. */
#define MEDNEXT_DW_WGRAD_NOALLOC_MAX_SCRATCH ((size_t)16 << 20)
int mednext_dw_wgrad_noalloc(const void* x, const void* dy, void* dweight, void* dbias,
                             int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k,
                             int dtype, mednext_stream_t stream);

/* ---------------- depthwise Conv3d, stride 2, padding k/2 (down block) ----
 * (d, h, w) are the INPUT sizes; the output is ((d+1)/2, (h+1)/2, (w+1)/2). */
int mednext_dw_s2_fwd(const void* x, const void* weight, const void* bias, void* y, int64_t n,
                      int64_t c, int64_t d, int64_t h, int64_t w, int k, int dtype,
                      mednext_stream_t stream);
/* addend_even: NULL, or a tensor of dy's shape added to dx at the all-even
 * positions 2m: the input grad of the down block's 1x1, stride-2 residual
 * convolution (models/blocks.py:128-136), which samples the input there. */
int mednext_dw_s2_dgrad(const void* dy, const void* weight, const void* addend_even, void* dx,
                        int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k, int dtype,
                        mednext_stream_t stream);
size_t mednext_dw_s2_wgrad_workspace_size(int64_t n, int64_t c, int64_t d, int64_t h, int64_t w,
                                          int k, int dtype);
int mednext_dw_s2_wgrad(const void* x, const void* dy, void* dweight, void* dbias,
                        void* workspace, size_t workspace_bytes, int64_t n, int64_t c, int64_t d,
                        int64_t h, int64_t w, int k, int dtype, mednext_stream_t stream);
/* mednext_dw_s2_wgrad with fp32 dweight / dbias (see mednext_dw_wgrad_f32out). */
int mednext_dw_s2_wgrad_f32out(const void* x, const void* dy, void* dweight, void* dbias,
                               void* workspace, size_t workspace_bytes, int64_t n, int64_t c,
                               int64_t d, int64_t h, int64_t w, int k, int dtype,
                               mednext_stream_t stream);

/* ------- depthwise ConvTranspose3d, stride 2, padding k/2 (up block) ------
 * (d, h, w) are the INPUT sizes; the output is (2d-1, 2h-1, 2w-1).
 * big_pitch: elements between consecutive W-rows of the (2d-1, 2h-1, 2w-1)
 * tensor (y in fwd, dy in dgrad/wgrad); 0 means 2w-1 (contiguous).  The (n, c)
 * volumes are then (2d-1)(2h-1)*big_pitch elements apart.  The fused up block
 * uses big_pitch = 2w (w a multiple of 4): every row starts 16-byte aligned, so
 * the depthwise kernels and the following 1x1 GEMMs reach the tensor by TMA, and
 * the GEMMs run over the pad column too.  fwd writes zeros into the pad columns;
 * dgrad and wgrad never read them. */
int mednext_dwT_fwd(const void* x, const void* weight, const void* bias, void* y, int64_t n,
                    int64_t c, int64_t d, int64_t h, int64_t w, int64_t big_pitch, int k, int dtype,
                    mednext_stream_t stream);
/* mednext_dwT_fwd plus the GroupNorm statistics of y over its grid voxels (pad
 * columns excluded): gn_stats = float [n*c][2] (mean, rstd with gn_eps), as
 * mednext_dw_fwd gives them for the regular block.  On the packed-FMA path the
 * kernel accumulates them while it stores y; elsewhere a second pass reads y.
 * The fused up block's transposed conv + GroupNorm statistics
 * (models/blocks.py:165-172 followed by the GroupNorm of blocks.py:74).
 * workspace: mednext_dwT_fwd_workspace_size bytes. */
size_t mednext_dwT_fwd_workspace_size(int64_t n, int64_t c, int64_t d, int64_t h, int64_t w,
                                      int64_t big_pitch, int k, int dtype);
int mednext_dwT_fwd_stats(const void* x, const void* weight, const void* bias, void* y,
                          float* gn_stats, float gn_eps, void* workspace, size_t workspace_bytes,
                          int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int64_t big_pitch,
                          int k, int dtype, mednext_stream_t stream);
/* addend: NULL, or a tensor of dx's shape added to dx: the input grad of the up
 * block's 1x1, stride-2 transposed residual convolution (models/blocks.py:173-182). */
int mednext_dwT_dgrad(const void* dy, const void* weight, const void* addend, void* dx, int64_t n,
                      int64_t c, int64_t d, int64_t h, int64_t w, int64_t big_pitch, int k,
                      int dtype, mednext_stream_t stream);
/* Stride-2 expansion onto the up block's (2d-1, 2h-1, 2w-1) grid (row pitch as
 * above): big[2m] = small[m] at the all-even positions, bias[c] (fp32, NULL = 0)
 * at all others, zeros in the pad columns.  With small = W x + bias from the pointwise
 * GEMM this is the output of the up block's ConvTranspose3d(1x1x1, stride 2)
 * residual branch (models/blocks.py:173-182). */
/* out [n, c, d+1, h+1, w+1] = F.pad(v, (1, 0, 1, 0, 1, 0)) + addend, one rounding;
 * v is the (d, h, w) grid with W-rows `pitch` elements apart (0 = w), (n, c)
 * volumes d*h*pitch apart; addend (out's shape,
 * may be NULL) in the same dtype.  Replaces the up block's output pad and the
 * decoder's skip add: models/blocks.py:177-181, models/mednext_v1.py:205. */
int mednext_pad_front_add(const void* v, const void* addend, void* out, int64_t n, int64_t c,
                          int64_t d, int64_t h, int64_t w, int64_t pitch, int dtype,
                          mednext_stream_t stream);
/* The inverse: v (the row-pitched (d, h, w) grid, as above) = the (z, y, x >= 1)
 * interior of padded [n, c, d+1, h+1, w+1], zeros in the pad columns.  The grad of the up block's padded output,
 * repacked for its GEMMs (the backward of models/blocks.py:178). */
int mednext_unpad_front(const void* padded, void* v, int64_t n, int64_t c, int64_t d, int64_t h,
                        int64_t w, int64_t pitch, int dtype, mednext_stream_t stream);
int mednext_upsample2_fill(const void* small, const float* bias, void* big, int64_t n, int64_t c,
                           int64_t d, int64_t h, int64_t w, int64_t big_pitch, int dtype,
                           mednext_stream_t stream);
size_t mednext_dwT_wgrad_workspace_size(int64_t n, int64_t c, int64_t d, int64_t h, int64_t w,
                                        int k, int dtype);
int mednext_dwT_wgrad(const void* x, const void* dy, void* dweight, void* dbias, void* workspace,
                      size_t workspace_bytes, int64_t n, int64_t c, int64_t d, int64_t h,
                      int64_t w, int64_t big_pitch, int k, int dtype, mednext_stream_t stream);
/* mednext_dwT_wgrad with fp32 dweight / dbias (see mednext_dw_wgrad_f32out). */
int mednext_dwT_wgrad_f32out(const void* x, const void* dy, void* dweight, void* dbias,
                             void* workspace, size_t workspace_bytes, int64_t n, int64_t c,
                             int64_t d, int64_t h, int64_t w, int64_t big_pitch, int k, int dtype,
                             mednext_stream_t stream);

/* ---------------- GroupNorm with groups == channels ----------------------
 * x: [n, c, spatial]; stats: float [n*c][2] = (mean, rstd).  gamma/beta: [c]
 * in gamma_dtype (FLOAT32 parameters in the reference model). */
size_t mednext_gn_stats_workspace_size(int64_t n, int64_t c, int64_t spatial);
/* pitch: elements between (n, c) rows (0 = spatial); only `spatial` are read. */
int mednext_gn_stats(const void* x, float* stats, void* workspace, size_t workspace_bytes,
                     int64_t n, int64_t c, int64_t spatial, int64_t pitch, float eps, int dtype,
                     mednext_stream_t stream);
/* Statistics of a row-pitched tensor: each (n, c) volume is `rows` rows of
 * row_pitch elements (0 = row_len), of which the first row_len are statistics;
 * volumes are rows*row_pitch elements apart.  The up block's transposed-conv
 * output with its pad column.  workspace: mednext_gn_stats_workspace_size(n, c,
 * rows * row_pitch) bytes.  No reference counterpart (the reference's tensors
 * are never pitched). */
int mednext_gn_stats_rows(const void* x, float* stats, void* workspace, size_t workspace_bytes,
                          int64_t n, int64_t c, int64_t rows, int64_t row_len, int64_t row_pitch,
                          float eps, int dtype, mednext_stream_t stream);
int mednext_gn_fwd(const void* x, const float* stats, const void* gamma, const void* beta,
                   void* y, int64_t n, int64_t c, int64_t spatial, int x_dtype, int y_dtype,
                   int gamma_dtype, mednext_stream_t stream);
/* dx from dy (grad of the GroupNorm output) and x; dgamma/dbeta (FLOAT32, may be
 * NULL) get the parameter grads.  Deterministic. */
size_t mednext_gn_bwd_workspace_size(int64_t n, int64_t c, int64_t spatial);
int mednext_gn_bwd(const void* dy, const void* x, const float* stats, const void* gamma,
                   void* dx, float* dgamma, float* dbeta, void* workspace,
                   size_t workspace_bytes, int64_t n, int64_t c, int64_t spatial, int dy_dtype,
                   int x_dtype, int dx_dtype, int gamma_dtype, mednext_stream_t stream);

/* ---------------- deep-supervision loss -------------------------------------
 * Mean cross-entropy over the class axis, F.cross_entropy(logits, target,
 * ignore_index=ignore_index) for the training step's heads
 * (benchmarks/implementations.py:133-190): logits [n, k, v] (FLOAT32, BFLOAT16 or
 * FLOAT16, computed in fp32), target INT64 [n, v].  fwd writes out[0] = mean loss,
 * out[1] = number of counted targets (FLOAT32, device); bwd writes grad (the
 * logits' shape and dtype) = (softmax - onehot) * grad_loss[0] / out[1], with
 * grad_loss a device FLOAT32 scalar.  A target outside [0, k) that is not
 * ignore_index is skipped and raises the device error word (0x300).
 * Deterministic. */
size_t mednext_ce_workspace_size(int64_t n, int64_t k, int64_t v);
int mednext_ce_fwd(const void* logits, const int64_t* target, float* out, void* workspace,
                   size_t workspace_bytes, int64_t n, int64_t k, int64_t v, int64_t ignore_index,
                   int dtype, mednext_stream_t stream);
int mednext_ce_bwd(const void* logits, const int64_t* target, const float* fwd_out,
                   const float* grad_loss, void* grad, int64_t n, int64_t k, int64_t v,
                   int64_t ignore_index, int dtype, mednext_stream_t stream);

/* ---------------- pointwise 1x1x1 convolution (tensor cores) -------------
 * Forward / input-grad form, one GEMM per sample with the voxel axis as M:
 *   y[s, j, v] = epi( sum_k wt[j, k] * pro(a[s, k, v]) )     j < cout, k < cin
 * a: [n, cin, vox]; wt: [cout, cin] (K contiguous); y: [n, cout, vox].
 * Prologue (enum mednext_pw_prologue) uses pro_stats [n*cin][2], pro_gamma,
 * pro_beta [cin] (FLOAT32).  Epilogue flags (mednext_pw_epilogue) use bias
 * [cout] (FLOAT32), residual [n, cout, vox] (y dtype), aux [n, cout, vox]
 * (a dtype).  GN_BWD_STATS additionally takes aux = the GroupNorm input,
 * epi_stats [n*cout][2] = its (mean, rstd), and writes per-(sample, channel,
 * voxel-tile) partial sums into the workspace; mednext_gn_bwd_from_partials
 * consumes them.  a, wt: BFLOAT16 or FLOAT16 (same type); y: a's type or FLOAT32. */
size_t mednext_pw_fwd_workspace_size(int64_t n, int64_t cin, int64_t cout, int64_t vox,
                                     int epilogue);
int mednext_pw_fwd(const void* a, const void* wt, void* y, int prologue, const float* pro_stats,
                   const float* pro_gamma, const float* pro_beta, int epilogue,
                   const float* bias, const void* residual, const void* aux,
                   const float* epi_stats, void* workspace, size_t workspace_bytes, int64_t n,
                   int64_t cin, int64_t cout, int64_t vox, int a_dtype, int y_dtype,
                   mednext_stream_t stream);
/* mednext_pw_fwd that also writes pro_out [n, cin, vox] (a's dtype) = pro(a), the
 * GEMM's transformed input, when prologue != NONE (pro_out NULL: same as
 * mednext_pw_fwd).  The compress GEMM of models/blocks.py:79-80
 * (project(activation(expand(x)))) keeps activation(expand(x)) this way, the
 * tensor PyTorch's autograd saves for project's weight grad.
 * pro_out must not alias a or y. */
int mednext_pw_fwd_pro_out(const void* a, const void* wt, void* y, int prologue,
                           const float* pro_stats, const float* pro_gamma,
                           const float* pro_beta, int epilogue, const float* bias,
                           const void* residual, const void* aux, const float* epi_stats,
                           void* pro_out, void* workspace, size_t workspace_bytes, int64_t n,
                           int64_t cin, int64_t cout, int64_t vox, int a_dtype, int y_dtype,
                           mednext_stream_t stream);
/* The forward GEMM of mednext_pw_fwd (bf16 only; prologue NONE or GROUPNORM; bias
 * or none) that also writes g = gelu(y) (exact erf form, of y as stored in bf16) to
 * g, an array of y's shape: the expand GEMM of the MedNeXt block hands the compress
 * GEMM its activated input this way, so that GEMM runs without a GELU prologue and
 * the compress weight grad reads g instead of recomputing it (models/blocks.py:75-77,
 * the expand -> GELU -> project chain).  y and g rows must start 16-byte aligned
 * (vox a multiple of 8).  Returns MEDNEXT_ERR_UNSUPPORTED for other dtypes, a GELU
 * prologue or other shapes (the caller then runs mednext_pw_fwd with a GELU
 * prologue on the next GEMM).  Workspace as mednext_pw_fwd_workspace_size(...,
 * bias ? MEDNEXT_EPI_BIAS : 0). */
int mednext_pw_fwd_gelu_out(const void* a, const void* wt, void* y, void* g, int prologue,
                            const float* pro_stats, const float* pro_gamma, const float* pro_beta,
                            const float* bias, void* workspace, size_t workspace_bytes, int64_t n,
                            int64_t cin, int64_t cout, int64_t vox, int dtype,
                            mednext_stream_t stream);
/* The block's expansion, fused (models/blocks.py:79-84 with the residual add of
 * 89-90): with z = GroupNorm(t) (stats [n*c][2], gamma, beta FLOAT32 [c]),
 *   u[s, h, v] = sum_k we[h, k] * z[s, k, v] + be[h]               (written: saved for backward)
 *   y[s, j, v] = sum_h wp[j, h] * GELU(u)[s, h, v] + bp[j] (+ residual[s, j, v])
 * in one kernel: GELU(u) stays in shared memory as the second GEMM's operand and u
 * is not read back.  t: [n, c, vox]; we: [h, c]; wp: [c2, h]; be [h], bp [c2] FLOAT32;
 * u: [n, h, vox]; y, residual (may be NULL): [n, c2, vox].  BFLOAT16 only; covers
 * c <= 64, h <= 128 (multiples of 8 and 16), c2 <= 256, vox % 8 == 0, and returns
 * MEDNEXT_ERR_UNSUPPORTED otherwise (the caller then runs two mednext_pw_fwd). */
int mednext_pw_mlp_fwd(const void* t, const float* stats, const float* gamma, const float* beta,
                       const void* we, const float* be, const void* wp, const float* bp,
                       const void* residual, void* u, void* y, int64_t n, int64_t c, int64_t h,
                       int64_t c2, int64_t vox, int dtype, mednext_stream_t stream);
/* Backward of the compress GEMM through the GELU, fused (models/blocks.py:80,
 * project(activation(u))), in one kernel plus a split reduction:
 *   du[s, h, v]  = (sum_c wpt[h, c] * dy[s, c, v]) * GELU'(u[s, h, v])
 *   dw[c, h]     = sum_{s, v} dy[s, c, v] * GELU(u[s, h, v]);  dbias[c] = sum dy
 * dy: [n, c, vox]; wpt: [h, c] (the compress weight transposed); u, du: [n, h, vox];
 * dw, dbias: FLOAT32.  GELU(u) is computed in the same pass as GELU'(u) and never
 * stored.  BFLOAT16 only.  workspace_size returns 0 for shapes the fused kernel
 * does not cover (c > 64, h > 127, ...); the call then returns
 * MEDNEXT_ERR_UNSUPPORTED and the caller runs mednext_pw_fwd + mednext_pw_wgrad.
 * Deterministic. */
size_t mednext_pw_gelu_bwd_workspace_size(int64_t n, int64_t c, int64_t h, int64_t vox, int dtype);
int mednext_pw_gelu_bwd(const void* dy, const void* wpt, const void* u, void* du, float* dw, float* dbias,
                        void* workspace, size_t workspace_bytes, int64_t n, int64_t c, int64_t h,
                        int64_t vox, int dtype, mednext_stream_t stream);
/* Backward of the expand GEMM after its GroupNorm, fused (models/blocks.py:79-84,
 * expand(norm(t))): one kernel computes
 *   dz[s, c, v] = sum_h wt[c, h] * du[s, h, v]   (wt = expand weight transposed, [c, h])
 * with the GroupNorm-backward partial sums of mednext_pw_fwd's
 * MEDNEXT_EPI_GN_BWD_STATS (aux = t, epi_stats = stats) at the start of the
 * workspace, for mednext_gn_bwd_from_partials, and
 *   dw[h, c] = sum_{s, v} du[s, h, v] * GroupNorm(t)[s, c, v];  dbias[h] = sum du
 * with GroupNorm(t) = t * rstd * gamma + (beta - mean * rstd * gamma) (gamma, beta
 * FLOAT32 [c]) computed in the same pass and never stored.  BFLOAT16 only.
 * workspace_size returns 0 when not covered (h > 64, c > 127, ...); the call then
 * returns MEDNEXT_ERR_UNSUPPORTED.  Deterministic. */
size_t mednext_pw_gn_bwd_fused_workspace_size(int64_t n, int64_t h, int64_t c, int64_t vox, int dtype);
int mednext_pw_gn_bwd_fused(const void* du, const void* wt, const void* t, const float* stats,
                            const float* gamma, const float* beta, void* dz, float* dw, float* dbias,
                            void* workspace, size_t workspace_bytes, int64_t n, int64_t h, int64_t c,
                            int64_t vox, int dtype, mednext_stream_t stream);
/* Weight-grad form, the voxel axis is the reduction:
 *   dw[j, k] = sum_{s, v} g[s, j, v] * pro(a[s, k, v]);  dbias[j] = sum g
 * dw, dbias: FLOAT32 (dbias may be NULL).  Deterministic split-K. */
size_t mednext_pw_wgrad_workspace_size(int64_t n, int64_t cin, int64_t cout, int64_t vox);
int mednext_pw_wgrad(const void* g, const void* a, float* dw, float* dbias, int prologue,
                     const float* pro_stats, const float* pro_gamma, const float* pro_beta,
                     void* workspace, size_t workspace_bytes, int64_t n, int64_t cin,
                     int64_t cout, int64_t vox, int dtype, mednext_stream_t stream);
/* GroupNorm backward driven by the partial sums that mednext_pw_fwd wrote with
 * MEDNEXT_EPI_GN_BWD_STATS (dz = that GEMM's output = grad of GroupNorm output).
 * vox: valid voxels per (n, c) row (the mean's divisor); pitch: row length the
 * GEMM ran over (its vox argument; 0 = vox).  dx is written over the whole pitch
 * (entries that are not valid voxels get values without meaning).  The partials
 * in pw_workspace are folded in place. */
int mednext_gn_bwd_from_partials(const void* dz, const void* x, const float* stats,
                                 const void* gamma, void* dx, float* dgamma, float* dbeta,
                                 void* pw_workspace, int64_t n, int64_t c, int64_t vox,
                                 int64_t pitch, int dz_dtype, int x_dtype, int dx_dtype,
                                 int gamma_dtype, mednext_stream_t stream);

/* ---------------- parameter casts of the fused block ----------------
 * No reference counterpart: under autocast the reference casts each fp32
 * parameter separately at every use.  One launch casts a table of fp32 tensors;
 * entry i reads src (rows x cols, fp32, 4-byte aligned) and writes dst:
 *   out_dtype BFLOAT16 / FLOAT16: the value rounded to that type;
 *   out_dtype FLOAT32: the value rounded to via_dtype (FLOAT32 = unchanged) and
 *     stored as fp32, e.g. a bias that autocast rounds before an fp32 epilogue;
 *   transpose != 0: dst is the cols x rows transpose.
 * At most MEDNEXT_CAST_MAX_ENTRIES entries of fewer than 2^31 elements each. */
#define MEDNEXT_CAST_MAX_ENTRIES 16
typedef struct {
  const float* src;
  void* dst;
  int64_t rows;
  int64_t cols;
  int out_dtype;
  int via_dtype;
  int transpose;
} mednext_cast_entry;
int mednext_cast_params(const mednext_cast_entry* entries, int count, mednext_stream_t stream);

/* ---------------- MedNeXt v2 Global Response Norm -------------------------
 * x [n, c, spatial] contiguous (NCDHW with spatial = D*H*W), dtype float32,
 * bfloat16 or float16; gamma, beta: [c] float32 (the (1, C, 1, 1, 1) parameters).
 *   norm[n,c] = ||x[n,c,:]||_2,  denom[n] = sum_c norm[n,c] + eps,
 *   y = x + gamma[c] * x * (norm[n,c] / denom[n]) + beta[c]   (fp32 math, one rounding)
 * norm ([n*c] float32) and denom ([n] float32) are outputs of the forward and
 * inputs of the backward.  Reductions run in a fixed order: deterministic.
 * Replaces the fused op mednext_accel::grn_forward / grn_backward
 * (ops/_triton/grn.py:235-290, 300-377), whose formula is ops/grn.py:16-29.
 * The workspace (float32 partial sums) is shared by the forward and backward:
 * mednext_grn_workspace_size() bytes, 4-byte aligned; 0 means invalid sizes. */
size_t mednext_grn_workspace_size(int64_t n, int64_t c, int64_t spatial, int dtype);
int mednext_grn_fwd(const void* x, const float* gamma, const float* beta, void* y, float* norm,
                    float* denom, void* workspace, size_t workspace_bytes, int64_t n, int64_t c,
                    int64_t spatial, float eps, int dtype, mednext_stream_t stream);
/* dx = dy (1 + gamma r) + (norm > 0 ? x / norm : 0) dnorm, with
 * dnorm[n,c] = (gamma[c] qx[n,c] - sum_j gamma[j] qx[n,j] r[n,j]) / denom[n],
 * qx = sum_v dy x, r = norm / denom; dgamma[c] = sum_n qx r, dbeta[c] = sum_n sum_v dy
 * ([c] float32 each, overwritten). */
int mednext_grn_bwd(const void* dy, const void* x, const float* gamma, const float* norm,
                    const float* denom, void* dx, float* dgamma, float* dbeta, void* workspace,
                    size_t workspace_bytes, int64_t n, int64_t c, int64_t spatial, int dtype,
                    mednext_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MEDNEXT_B200_H */
