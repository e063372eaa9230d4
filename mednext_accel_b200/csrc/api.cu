// C ABI of libmednext_b200.so: argument validation, tile planning and the
// calls into the per-family dispatchers.  Declarations, and the reference
// interface each entry point replaces, are in include/mednext_b200.h.
#include "plan.h"

#include <atomic>
#include <map>
#include <mutex>
#include <utility>

namespace mednext {
namespace {
thread_local int t_last_cuda_error = 0;
std::atomic<uint64_t> g_launches{0};
}  // namespace
int record_launch() {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    t_last_cuda_error = (int)e;
    return MEDNEXT_ERR_CUDA;
  }
  return MEDNEXT_OK;
}
int last_cuda_error() { return t_last_cuda_error; }
void note_cuda_error(cudaError_t e) { t_last_cuda_error = (int)e; }

int ensure_smem_fn(const void* fn, size_t smem) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    note_cuda_error(e);
    return MEDNEXT_ERR_CUDA;
  }
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> granted;  // largest size granted per (kernel, device)
  std::lock_guard<std::mutex> lock(mu);
  size_t& have = granted[{fn, dev}];
  if (smem <= have) return MEDNEXT_OK;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    note_cuda_error(e);
    return MEDNEXT_ERR_CUDA;
  }
  have = smem;
  return MEDNEXT_OK;
}
uint64_t launch_count() { return g_launches.load(std::memory_order_relaxed); }
}  // namespace mednext

using namespace mednext;

namespace {

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
bool aligned16(const void* p) { return aligned(p, 16); }
bool valid_k(int k) { return k == 1 || k == 3 || k == 5 || k == 7; }

// Index math inside the kernels uses 32-bit tile/plane counters and 64-bit
// element offsets; keep every axis and the (sample, channel) count in range.
int check_dw(int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k, int dtype) {
  if (elem_size(dtype) == 0) return MEDNEXT_ERR_BAD_DTYPE;
  if (!valid_k(k)) return MEDNEXT_ERR_BAD_KERNEL;
  const int64_t lim = (int64_t)1 << 30;
  if (n <= 0 || c <= 0 || d <= 0 || h <= 0 || w <= 0) return MEDNEXT_ERR_BAD_SHAPE;
  if (n >= lim || c >= lim || d >= lim || h >= lim || w >= lim || n * c >= lim || h * w >= lim)
    return MEDNEXT_ERR_BAD_SHAPE;
  return MEDNEXT_OK;
}
cudaStream_t as_stream(mednext_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

size_t s1_wgrad_ws(int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k, int dtype) {
  const S1Plan p = plan_s1(n, c, d, h, w, k, elem_size(dtype), true);
  return (size_t)n * c * s1_tiles(p) * ((size_t)k * k * k + 1) * acc_size(dtype);
}
size_t s2_wgrad_ws(int64_t n, int64_t c, int64_t ds, int k, int dtype) {
  const S2WPlan p = plan_s2w(n, c, ds, k);
  return (size_t)n * c * p.chunks * ((size_t)k * k * k + 1) * acc_size(dtype);
}
bool gn_shape_ok(int64_t n, int64_t c, int64_t spatial) {
  return n > 0 && c > 0 && spatial > 0 && n * c < ((int64_t)1 << 30) && spatial < ((int64_t)1 << 40);
}
bool pw_dtype_ok(int d) { return d == MEDNEXT_BFLOAT16 || d == MEDNEXT_FLOAT16; }
bool pw_shape_ok(int64_t n, int64_t cin, int64_t cout, int64_t vox) {
  return n > 0 && cin > 0 && cout > 0 && vox > 0 && n < (1 << 20) && cin < (1 << 16) && cout < (1 << 16) &&
         vox < ((int64_t)1 << 40);
}
size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
bool pitch_ok(int64_t pitch, int64_t vol) { return pitch == 0 || pitch >= vol; }
// a W-row pitch of rows `width` elements wide: 0 (contiguous) or at least width
bool row_pitch_ok(int64_t row_pitch, int64_t width) {
  return row_pitch == 0 || (row_pitch >= width && row_pitch < (1LL << 30));
}

}  // namespace

extern "C" {

int mednext_abi_version(void) { return 1; }

const char* mednext_status_string(int status) {
  switch (status) {
    case MEDNEXT_OK: return "ok";
    case MEDNEXT_ERR_NULL_POINTER: return "a required pointer is NULL";
    case MEDNEXT_ERR_BAD_SHAPE: return "invalid or inconsistent shape";
    case MEDNEXT_ERR_BAD_KERNEL: return "kernel_size must be 1, 3, 5 or 7";
    case MEDNEXT_ERR_BAD_DTYPE: return "unsupported dtype";
    case MEDNEXT_ERR_WORKSPACE: return "workspace missing or too small";
    case MEDNEXT_ERR_ALIGNMENT: return "pointer not aligned to its element size";
    case MEDNEXT_ERR_CUDA: return "CUDA launch failed";
    case MEDNEXT_ERR_DEVICE: return "current device is not sm_100";
    case MEDNEXT_ERR_SCRATCH_LIMIT:
      return "shape needs more scratch than the built-in array of the no-allocation entry point holds";
    case MEDNEXT_ERR_UNSUPPORTED: return "the fused entry point does not cover this shape; run its parts";
    case MEDNEXT_ERR_BAD_VALUE: return "a scalar argument is out of range";
    default: return "unknown status";
  }
}

int mednext_last_cuda_error(void) { return last_cuda_error(); }

int mednext_device_error(int* code, mednext_stream_t stream) {
  if (code == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  *code = 0;
  int st = read_clear_errors_dw(code, as_stream(stream));
  if (st == MEDNEXT_OK) st = read_clear_errors_dw2(code, as_stream(stream));
  if (st == MEDNEXT_OK) st = read_clear_errors_gn(code, as_stream(stream));
  if (st == MEDNEXT_OK) st = read_clear_errors_pw(code, as_stream(stream));
  if (st == MEDNEXT_OK) st = read_clear_errors_pwf0(code, as_stream(stream));
  if (st == MEDNEXT_OK) st = read_clear_errors_pwf1(code, as_stream(stream));
  if (st == MEDNEXT_OK) st = read_clear_errors_pwf2(code, as_stream(stream));
  if (st == MEDNEXT_OK) st = read_clear_errors_loss(code, as_stream(stream));
  return st;
}

uint64_t mednext_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

int mednext_check_device(void) {
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return record_launch();
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
    return record_launch();
  return (major == 10 && minor == 0) ? MEDNEXT_OK : MEDNEXT_ERR_DEVICE;
}

// ------------------------------ depthwise stride 1 ------------------------------
size_t mednext_dw_fwd_workspace_size(int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k, int dtype) {
  if (check_dw(n, c, d, h, w, k, dtype) != MEDNEXT_OK) return 0;
  const S1Plan p = plan_s1(n, c, d, h, w, k, elem_size(dtype), false);
  return (size_t)n * c * s1_tiles(p) * sizeof(GnPartial);
}

int mednext_dw_fwd(const void* x, const void* weight, const void* bias, void* y, float* gn_stats, float gn_eps,
                   void* workspace, size_t workspace_bytes, int64_t n, int64_t c, int64_t d, int64_t h, int64_t w,
                   int k, int dtype, mednext_stream_t stream) {
  int st = check_dw(n, c, d, h, w, k, dtype);
  if (st != MEDNEXT_OK) return st;
  if (x == nullptr || weight == nullptr || y == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  const size_t esz = elem_size(dtype);
  if (!aligned16(x) || !aligned16(y) || !aligned(weight, esz) || (bias && !aligned(bias, esz)))
    return MEDNEXT_ERR_ALIGNMENT;
  GnPartial* part = nullptr;
  if (gn_stats != nullptr) {
    if (workspace == nullptr || !aligned16(workspace) ||
        workspace_bytes < mednext_dw_fwd_workspace_size(n, c, d, h, w, k, dtype))
      return MEDNEXT_ERR_WORKSPACE;
    if (!aligned(gn_stats, 8)) return MEDNEXT_ERR_ALIGNMENT;
    part = static_cast<GnPartial*>(workspace);
  }
  const S1Plan p = plan_s1(n, c, d, h, w, k, esz, false);
  st = dispatch_dw_s1_conv(dtype, k, x, weight, bias, nullptr, y, part, p, 0, as_stream(stream));
  if (st != MEDNEXT_OK || gn_stats == nullptr) return st;
  return dispatch_gn_finalize(part, (int)s1_tiles(p), (int)(n * c), gn_eps, gn_stats, as_stream(stream));
}

int mednext_dw_dgrad(const void* dy, const void* weight, const void* addend, void* dx, int64_t n, int64_t c,
                     int64_t d, int64_t h, int64_t w, int k, int dtype, mednext_stream_t stream) {
  int st = check_dw(n, c, d, h, w, k, dtype);
  if (st != MEDNEXT_OK) return st;
  if (dy == nullptr || weight == nullptr || dx == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  const size_t esz = elem_size(dtype);
  if (!aligned16(dy) || !aligned16(dx) || !aligned(weight, esz) || (addend && !aligned16(addend)))
    return MEDNEXT_ERR_ALIGNMENT;
  const S1Plan p = plan_s1(n, c, d, h, w, k, esz, false);
  return dispatch_dw_s1_conv(dtype, k, dy, weight, nullptr, addend, dx, nullptr, p, 1, as_stream(stream));
}

int mednext_dw_plan(int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k, int dtype, int wgrad,
                    int32_t* out) {
  const int st = check_dw(n, c, d, h, w, k, dtype);
  if (st != MEDNEXT_OK) return st;
  if (out == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  const S1Plan p = plan_s1(n, c, d, h, w, k, elem_size(dtype), wgrad != 0);
  return describe_dw_s1(dtype, k, p, wgrad != 0, out);
}

size_t mednext_dw_wgrad_workspace_size(int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k, int dtype) {
  if (check_dw(n, c, d, h, w, k, dtype) != MEDNEXT_OK) return 0;
  return s1_wgrad_ws(n, c, d, h, w, k, dtype);
}

namespace {
// out_f32: dweight / dbias are fp32 (16-bit dtypes: the dtype-rounded sums, widened)
bool f32_out_ok(int dtype) { return dtype == MEDNEXT_BFLOAT16 || dtype == MEDNEXT_FLOAT16 || dtype == MEDNEXT_FLOAT32; }

int dw_wgrad_impl(const void* x, const void* dy, void* dweight, void* dbias, void* workspace, size_t workspace_bytes,
                  int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k, int dtype, bool out_f32,
                  mednext_stream_t stream) {
  int st = check_dw(n, c, d, h, w, k, dtype);
  if (st != MEDNEXT_OK) return st;
  if (out_f32 && !f32_out_ok(dtype)) return MEDNEXT_ERR_BAD_DTYPE;
  if (x == nullptr || dy == nullptr || dweight == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  const size_t esz = elem_size(dtype);
  const size_t osz = out_f32 ? 4 : esz;
  if (!aligned16(x) || !aligned16(dy) || !aligned(dweight, osz) || (dbias && !aligned(dbias, osz)))
    return MEDNEXT_ERR_ALIGNMENT;
  if (workspace == nullptr || !aligned16(workspace) || workspace_bytes < s1_wgrad_ws(n, c, d, h, w, k, dtype))
    return MEDNEXT_ERR_WORKSPACE;
  const S1Plan p = plan_s1(n, c, d, h, w, k, esz, true);
  return dispatch_dw_s1_wgrad(dtype, k, x, dy, dweight, dbias, workspace, p, out_f32, as_stream(stream));
}
}  // namespace

int mednext_dw_wgrad(const void* x, const void* dy, void* dweight, void* dbias, void* workspace,
                     size_t workspace_bytes, int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k, int dtype,
                     mednext_stream_t stream) {
  return dw_wgrad_impl(x, dy, dweight, dbias, workspace, workspace_bytes, n, c, d, h, w, k, dtype, false, stream);
}

int mednext_dw_wgrad_f32out(const void* x, const void* dy, void* dweight, void* dbias, void* workspace,
                            size_t workspace_bytes, int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k,
                            int dtype, mednext_stream_t stream) {
  return dw_wgrad_impl(x, dy, dweight, dbias, workspace, workspace_bytes, n, c, d, h, w, k, dtype, true, stream);
}

// ------------------------------ depthwise stride 2 ------------------------------
int mednext_dw_s2_fwd(const void* x, const void* weight, const void* bias, void* y, int64_t n, int64_t c, int64_t d,
                      int64_t h, int64_t w, int k, int dtype, mednext_stream_t stream) {
  int st = check_dw(n, c, d, h, w, k, dtype);
  if (st != MEDNEXT_OK) return st;
  if (x == nullptr || weight == nullptr || y == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  const size_t esz = elem_size(dtype);
  if (!aligned(x, esz) || !aligned(y, esz) || !aligned(weight, esz) || (bias && !aligned(bias, esz)))
    return MEDNEXT_ERR_ALIGNMENT;
  return dispatch_dw_s2_gather(dtype, k, x, weight, bias, nullptr, y, s2_geom_down(n, c, d, h, w),
                               as_stream(stream));
}

int mednext_dw_s2_dgrad(const void* dy, const void* weight, const void* addend_even, void* dx, int64_t n, int64_t c,
                        int64_t d, int64_t h, int64_t w, int k, int dtype, mednext_stream_t stream) {
  int st = check_dw(n, c, d, h, w, k, dtype);
  if (st != MEDNEXT_OK) return st;
  if (dy == nullptr || weight == nullptr || dx == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  const size_t esz = elem_size(dtype);
  if (!aligned(dy, esz) || !aligned(dx, esz) || !aligned(weight, esz) || (addend_even && !aligned(addend_even, esz)))
    return MEDNEXT_ERR_ALIGNMENT;
  return dispatch_dw_s2_scatter(dtype, k, dy, weight, nullptr, addend_even, dx, s2_geom_down(n, c, d, h, w),
                                as_stream(stream));
}

size_t mednext_dw_s2_wgrad_workspace_size(int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k, int dtype) {
  if (check_dw(n, c, d, h, w, k, dtype) != MEDNEXT_OK) return 0;
  const DwS2Geom g = s2_geom_down(n, c, d, h, w);
  return s2_wgrad_ws(n, c, g.Ds, k, dtype);
}

namespace {
int dw_s2_wgrad_impl(const void* x, const void* dy, void* dweight, void* dbias, void* workspace,
                     size_t workspace_bytes, int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k, int dtype,
                     bool out_f32, mednext_stream_t stream) {
  int st = check_dw(n, c, d, h, w, k, dtype);
  if (st != MEDNEXT_OK) return st;
  if (out_f32 && !f32_out_ok(dtype)) return MEDNEXT_ERR_BAD_DTYPE;
  if (x == nullptr || dy == nullptr || dweight == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  const size_t esz = elem_size(dtype);
  const size_t osz = out_f32 ? 4 : esz;
  if (!aligned(x, esz) || !aligned(dy, esz) || !aligned(dweight, osz) || (dbias && !aligned(dbias, osz)))
    return MEDNEXT_ERR_ALIGNMENT;
  if (workspace == nullptr || !aligned16(workspace) ||
      workspace_bytes < mednext_dw_s2_wgrad_workspace_size(n, c, d, h, w, k, dtype))
    return MEDNEXT_ERR_WORKSPACE;
  return dispatch_dw_s2_wgrad(dtype, k, x, dy, dweight, dbias, workspace, s2_geom_down(n, c, d, h, w), false,
                              out_f32, as_stream(stream));
}
}  // namespace

int mednext_dw_s2_wgrad(const void* x, const void* dy, void* dweight, void* dbias, void* workspace,
                        size_t workspace_bytes, int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k,
                        int dtype, mednext_stream_t stream) {
  return dw_s2_wgrad_impl(x, dy, dweight, dbias, workspace, workspace_bytes, n, c, d, h, w, k, dtype, false, stream);
}

int mednext_dw_s2_wgrad_f32out(const void* x, const void* dy, void* dweight, void* dbias, void* workspace,
                               size_t workspace_bytes, int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k,
                               int dtype, mednext_stream_t stream) {
  return dw_s2_wgrad_impl(x, dy, dweight, dbias, workspace, workspace_bytes, n, c, d, h, w, k, dtype, true, stream);
}

// ------------------------------ depthwise transpose ------------------------------
int mednext_dwT_fwd(const void* x, const void* weight, const void* bias, void* y, int64_t n, int64_t c, int64_t d,
                    int64_t h, int64_t w, int64_t big_pitch, int k, int dtype, mednext_stream_t stream) {
  int st = check_dw(n, c, d, h, w, k, dtype);
  if (st != MEDNEXT_OK) return st;
  if (!row_pitch_ok(big_pitch, 2 * w - 1)) return MEDNEXT_ERR_BAD_SHAPE;
  if (x == nullptr || weight == nullptr || y == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  const size_t esz = elem_size(dtype);
  if (!aligned(x, esz) || !aligned(y, esz) || !aligned(weight, esz) || (bias && !aligned(bias, esz)))
    return MEDNEXT_ERR_ALIGNMENT;
  return dispatch_dw_s2_scatter(dtype, k, x, weight, bias, nullptr, y, s2_geom_up(n, c, d, h, w, big_pitch),
                                as_stream(stream));
}

size_t mednext_dwT_fwd_workspace_size(int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int64_t big_pitch,
                                      int k, int dtype) {
  if (check_dw(n, c, d, h, w, k, dtype) != MEDNEXT_OK || !row_pitch_ok(big_pitch, 2 * w - 1)) return 0;
  const DwS2Geom g = s2_geom_up(n, c, d, h, w, big_pitch);
  if (!gn_shape_ok(n, c, g.bp)) return 0;
  return align_up(dwT_fwd_stats_ws(dtype, k, g), 256);
}

int mednext_dwT_fwd_stats(const void* x, const void* weight, const void* bias, void* y, float* gn_stats, float gn_eps,
                          void* workspace, size_t workspace_bytes, int64_t n, int64_t c, int64_t d, int64_t h,
                          int64_t w, int64_t big_pitch, int k, int dtype, mednext_stream_t stream) {
  int st = check_dw(n, c, d, h, w, k, dtype);
  if (st != MEDNEXT_OK) return st;
  if (!row_pitch_ok(big_pitch, 2 * w - 1)) return MEDNEXT_ERR_BAD_SHAPE;
  if (x == nullptr || weight == nullptr || y == nullptr || gn_stats == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  const size_t esz = elem_size(dtype);
  if (!aligned(x, esz) || !aligned(y, esz) || !aligned(weight, esz) || (bias && !aligned(bias, esz)) ||
      !aligned(gn_stats, 8))
    return MEDNEXT_ERR_ALIGNMENT;
  const size_t need = mednext_dwT_fwd_workspace_size(n, c, d, h, w, big_pitch, k, dtype);
  if (need == 0) return MEDNEXT_ERR_BAD_SHAPE;
  if (workspace == nullptr || !aligned16(workspace) || workspace_bytes < need) return MEDNEXT_ERR_WORKSPACE;
  return dispatch_dwT_fwd_stats(dtype, k, x, weight, bias, y, static_cast<GnPartial*>(workspace), gn_eps, gn_stats,
                                s2_geom_up(n, c, d, h, w, big_pitch), as_stream(stream));
}

int mednext_dwT_dgrad(const void* dy, const void* weight, const void* addend, void* dx, int64_t n, int64_t c,
                      int64_t d, int64_t h, int64_t w, int64_t big_pitch, int k, int dtype, mednext_stream_t stream) {
  int st = check_dw(n, c, d, h, w, k, dtype);
  if (st != MEDNEXT_OK) return st;
  if (!row_pitch_ok(big_pitch, 2 * w - 1)) return MEDNEXT_ERR_BAD_SHAPE;
  if (dy == nullptr || weight == nullptr || dx == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  const size_t esz = elem_size(dtype);
  if (!aligned(dy, esz) || !aligned(dx, esz) || !aligned(weight, esz) || (addend && !aligned(addend, esz)))
    return MEDNEXT_ERR_ALIGNMENT;
  return dispatch_dw_s2_gather(dtype, k, dy, weight, nullptr, addend, dx, s2_geom_up(n, c, d, h, w, big_pitch),
                               as_stream(stream));
}

int mednext_upsample2_fill(const void* small, const float* bias, void* big, int64_t n, int64_t c, int64_t d,
                           int64_t h, int64_t w, int64_t big_pitch, int dtype, mednext_stream_t stream) {
  int st = check_dw(n, c, d, h, w, 1, dtype);
  if (st != MEDNEXT_OK) return st;
  if (!row_pitch_ok(big_pitch, 2 * w - 1)) return MEDNEXT_ERR_BAD_SHAPE;
  if (small == nullptr || big == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  const size_t esz = elem_size(dtype);
  if (!aligned(small, esz) || !aligned(big, esz) || (bias && !aligned(bias, 4))) return MEDNEXT_ERR_ALIGNMENT;
  return dispatch_upsample2_fill(dtype, small, bias, big, s2_geom_up(n, c, d, h, w, big_pitch), as_stream(stream));
}

static DwS2Geom pad_geom(int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int64_t row_pitch) {
  DwS2Geom g{};
  g.N = (int)n; g.C = (int)c;
  g.Db = (int)d; g.Hb = (int)h; g.Wb = (int)w;
  g.bw = row_pitch > 0 ? (int)row_pitch : (int)w;
  g.bp = (long long)d * h * g.bw;
  return g;
}

int mednext_pad_front_add(const void* v, const void* addend, void* out, int64_t n, int64_t c, int64_t d, int64_t h,
                          int64_t w, int64_t pitch, int dtype, mednext_stream_t stream) {
  int st = check_dw(n, c, d + 1, h + 1, w + 1, 1, dtype);
  if (st != MEDNEXT_OK) return st;
  if (d < 1 || h < 1 || w < 1 || !row_pitch_ok(pitch, w)) return MEDNEXT_ERR_BAD_SHAPE;
  if (v == nullptr || out == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  const size_t esz = elem_size(dtype);
  if (!aligned(v, esz) || !aligned(out, esz) || (addend && !aligned(addend, esz))) return MEDNEXT_ERR_ALIGNMENT;
  return dispatch_pad_front(dtype, v, addend, out, pad_geom(n, c, d, h, w, pitch), false, as_stream(stream));
}

int mednext_unpad_front(const void* padded, void* v, int64_t n, int64_t c, int64_t d, int64_t h, int64_t w,
                        int64_t pitch, int dtype, mednext_stream_t stream) {
  int st = check_dw(n, c, d + 1, h + 1, w + 1, 1, dtype);
  if (st != MEDNEXT_OK) return st;
  if (d < 1 || h < 1 || w < 1 || !row_pitch_ok(pitch, w)) return MEDNEXT_ERR_BAD_SHAPE;
  if (padded == nullptr || v == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  const size_t esz = elem_size(dtype);
  if (!aligned(padded, esz) || !aligned(v, esz)) return MEDNEXT_ERR_ALIGNMENT;
  return dispatch_pad_front(dtype, padded, nullptr, v, pad_geom(n, c, d, h, w, pitch), true, as_stream(stream));
}

size_t mednext_dwT_wgrad_workspace_size(int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int k, int dtype) {
  if (check_dw(n, c, d, h, w, k, dtype) != MEDNEXT_OK) return 0;
  return s2_wgrad_ws(n, c, d, k, dtype);
}

namespace {
int dwT_wgrad_impl(const void* x, const void* dy, void* dweight, void* dbias, void* workspace, size_t workspace_bytes,
                   int64_t n, int64_t c, int64_t d, int64_t h, int64_t w, int64_t big_pitch, int k, int dtype,
                   bool out_f32, mednext_stream_t stream) {
  int st = check_dw(n, c, d, h, w, k, dtype);
  if (st != MEDNEXT_OK) return st;
  if (out_f32 && !f32_out_ok(dtype)) return MEDNEXT_ERR_BAD_DTYPE;
  if (!row_pitch_ok(big_pitch, 2 * w - 1)) return MEDNEXT_ERR_BAD_SHAPE;
  if (x == nullptr || dy == nullptr || dweight == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  const size_t esz = elem_size(dtype);
  const size_t osz = out_f32 ? 4 : esz;
  if (!aligned(x, esz) || !aligned(dy, esz) || !aligned(dweight, osz) || (dbias && !aligned(dbias, osz)))
    return MEDNEXT_ERR_ALIGNMENT;
  if (workspace == nullptr || !aligned16(workspace) ||
      workspace_bytes < mednext_dwT_wgrad_workspace_size(n, c, d, h, w, k, dtype))
    return MEDNEXT_ERR_WORKSPACE;
  // big grid = dy (2S-1), small grid = x (S); the bias grad sums dy (big)
  return dispatch_dw_s2_wgrad(dtype, k, dy, x, dweight, dbias, workspace, s2_geom_up(n, c, d, h, w, big_pitch),
                              true, out_f32, as_stream(stream));
}
}  // namespace

int mednext_dwT_wgrad(const void* x, const void* dy, void* dweight, void* dbias, void* workspace,
                      size_t workspace_bytes, int64_t n, int64_t c, int64_t d, int64_t h, int64_t w,
                      int64_t big_pitch, int k, int dtype, mednext_stream_t stream) {
  return dwT_wgrad_impl(x, dy, dweight, dbias, workspace, workspace_bytes, n, c, d, h, w, big_pitch, k, dtype, false,
                        stream);
}

int mednext_dwT_wgrad_f32out(const void* x, const void* dy, void* dweight, void* dbias, void* workspace,
                             size_t workspace_bytes, int64_t n, int64_t c, int64_t d, int64_t h, int64_t w,
                             int64_t big_pitch, int k, int dtype, mednext_stream_t stream) {
  return dwT_wgrad_impl(x, dy, dweight, dbias, workspace, workspace_bytes, n, c, d, h, w, big_pitch, k, dtype, true,
                        stream);
}

// ------------------------------ GroupNorm ------------------------------
size_t mednext_gn_stats_workspace_size(int64_t n, int64_t c, int64_t spatial) {
  if (!gn_shape_ok(n, c, spatial)) return 0;
  return (size_t)n * c * gn_chunks(n * c, spatial) * sizeof(GnPartial);
}

int mednext_gn_stats(const void* x, float* stats, void* workspace, size_t workspace_bytes, int64_t n, int64_t c,
                     int64_t spatial, int64_t pitch, float eps, int dtype, mednext_stream_t stream) {
  if (elem_size(dtype) == 0) return MEDNEXT_ERR_BAD_DTYPE;
  if (x == nullptr || stats == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  if (!gn_shape_ok(n, c, spatial)) return MEDNEXT_ERR_BAD_SHAPE;
  if (!aligned(x, elem_size(dtype)) || !aligned(stats, 8)) return MEDNEXT_ERR_ALIGNMENT;
  if (workspace == nullptr || !aligned16(workspace) || workspace_bytes < mednext_gn_stats_workspace_size(n, c, spatial))
    return MEDNEXT_ERR_WORKSPACE;
  if (!pitch_ok(pitch, spatial)) return MEDNEXT_ERR_BAD_SHAPE;
  return dispatch_gn_stats(dtype, x, static_cast<GnPartial*>(workspace), n * c, spatial, pitch > 0 ? pitch : spatial,
                           gn_chunks(n * c, spatial), 1, 1, eps, stats, as_stream(stream));
}

int mednext_gn_stats_rows(const void* x, float* stats, void* workspace, size_t workspace_bytes, int64_t n, int64_t c,
                          int64_t rows, int64_t row_len, int64_t row_pitch, float eps, int dtype,
                          mednext_stream_t stream) {
  if (elem_size(dtype) == 0) return MEDNEXT_ERR_BAD_DTYPE;
  if (x == nullptr || stats == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  if (rows < 1 || row_len < 1 || !row_pitch_ok(row_pitch, row_len)) return MEDNEXT_ERR_BAD_SHAPE;
  const int64_t rp = row_pitch > 0 ? row_pitch : row_len;
  const int64_t vol = rows * rp;
  if (!gn_shape_ok(n, c, vol)) return MEDNEXT_ERR_BAD_SHAPE;
  if (!aligned(x, elem_size(dtype)) || !aligned(stats, 8)) return MEDNEXT_ERR_ALIGNMENT;
  if (workspace == nullptr || !aligned16(workspace) || workspace_bytes < mednext_gn_stats_workspace_size(n, c, vol))
    return MEDNEXT_ERR_WORKSPACE;
  return dispatch_gn_stats(dtype, x, static_cast<GnPartial*>(workspace), n * c, vol, vol, gn_chunks(n * c, vol),
                           (int)rp, (int)row_len, eps, stats, as_stream(stream));
}

int mednext_gn_fwd(const void* x, const float* stats, const void* gamma, const void* beta, void* y, int64_t n,
                   int64_t c, int64_t spatial, int x_dtype, int y_dtype, int gamma_dtype, mednext_stream_t stream) {
  if (elem_size(x_dtype) == 0 || elem_size(y_dtype) == 0 || elem_size(gamma_dtype) == 0) return MEDNEXT_ERR_BAD_DTYPE;
  if (x == nullptr || stats == nullptr || y == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  if (!gn_shape_ok(n, c, spatial)) return MEDNEXT_ERR_BAD_SHAPE;
  if (!aligned(x, elem_size(x_dtype)) || !aligned(y, elem_size(y_dtype))) return MEDNEXT_ERR_ALIGNMENT;
  return dispatch_gn_fwd(x_dtype, y_dtype, gamma_dtype, x, stats, gamma, beta, y, (int)c, n * c, spatial,
                         as_stream(stream));
}

size_t mednext_gn_bwd_workspace_size(int64_t n, int64_t c, int64_t spatial) {
  if (!gn_shape_ok(n, c, spatial)) return 0;
  return (size_t)n * c * gn_chunks(n * c, spatial) * sizeof(GnBwdPartial);
}

int mednext_gn_bwd(const void* dy, const void* x, const float* stats, const void* gamma, void* dx, float* dgamma,
                   float* dbeta, void* workspace, size_t workspace_bytes, int64_t n, int64_t c, int64_t spatial,
                   int dy_dtype, int x_dtype, int dx_dtype, int gamma_dtype, mednext_stream_t stream) {
  if (elem_size(dy_dtype) == 0 || elem_size(x_dtype) == 0 || elem_size(gamma_dtype) == 0) return MEDNEXT_ERR_BAD_DTYPE;
  if (dx_dtype != x_dtype) return MEDNEXT_ERR_BAD_DTYPE;
  if (dy == nullptr || x == nullptr || stats == nullptr || dx == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  if (!gn_shape_ok(n, c, spatial)) return MEDNEXT_ERR_BAD_SHAPE;
  if (workspace == nullptr || !aligned16(workspace) || workspace_bytes < mednext_gn_bwd_workspace_size(n, c, spatial))
    return MEDNEXT_ERR_WORKSPACE;
  const int chunks = gn_chunks(n * c, spatial);
  GnBwdPartial* part = static_cast<GnBwdPartial*>(workspace);
  int st = dispatch_gn_bwd_partial(x_dtype, dy_dtype, dy, x, stats, part, n * c, spatial, chunks, as_stream(stream));
  if (st != MEDNEXT_OK) return st;
  return dispatch_gn_bwd_apply(x_dtype, dy_dtype, gamma_dtype, dy, x, stats, gamma, part, chunks, dx, dgamma, dbeta,
                               (int)n, (int)c, spatial, spatial, as_stream(stream));
}

int mednext_gn_bwd_from_partials(const void* dz, const void* x, const float* stats, const void* gamma, void* dx,
                                 float* dgamma, float* dbeta, void* pw_workspace, int64_t n, int64_t c,
                                 int64_t vox, int64_t pitch, int dz_dtype, int x_dtype, int dx_dtype,
                                 int gamma_dtype, mednext_stream_t stream) {
  if (elem_size(dz_dtype) == 0 || elem_size(x_dtype) == 0 || elem_size(gamma_dtype) == 0) return MEDNEXT_ERR_BAD_DTYPE;
  if (dx_dtype != x_dtype) return MEDNEXT_ERR_BAD_DTYPE;
  if (dz == nullptr || x == nullptr || stats == nullptr || dx == nullptr || pw_workspace == nullptr)
    return MEDNEXT_ERR_NULL_POINTER;
  if (!gn_shape_ok(n, c, vox)) return MEDNEXT_ERR_BAD_SHAPE;
  if (!pitch_ok(pitch, vox)) return MEDNEXT_ERR_BAD_SHAPE;
  const int64_t rows = pitch > 0 ? pitch : vox;
  // one partial per (sample, channel, 128-voxel tile, 32-voxel quarter) of the GEMM's rows
  const int parts = (int)((rows + kPwBM - 1) / kPwBM) * 4;
  return dispatch_gn_bwd_apply(x_dtype, dz_dtype, gamma_dtype, dz, x, stats, gamma,
                               static_cast<const GnBwdPartial*>(pw_workspace), parts, dx, dgamma, dbeta, (int)n,
                               (int)c, vox, rows, as_stream(stream));
}

// ------------------------------ pointwise ------------------------------
// GroupNorm-backward partials (with MEDNEXT_EPI_GN_BWD_STATS), then, when cin is
// not a multiple of 8, W padded to 8-element rows for the TMA kernels.
size_t pw_fwd_gn_bytes(int64_t n, int64_t cout, int64_t vox, int epilogue) {
  if (!(epilogue & MEDNEXT_EPI_GN_BWD_STATS)) return 0;
  const int64_t mtiles = (vox + kPwBM - 1) / kPwBM;
  return align_up((size_t)n * cout * mtiles * 4 * sizeof(GnBwdPartial), 256);
}
size_t pw_fwd_wpad_bytes(int64_t cin, int64_t cout) {
  return cin % 8 == 0 ? 0 : (size_t)cout * ((cin + 7) / 8 * 8) * 2;
}
size_t mednext_pw_fwd_workspace_size(int64_t n, int64_t cin, int64_t cout, int64_t vox, int epilogue) {
  if (!pw_shape_ok(n, cin, cout, vox)) return 0;
  return pw_fwd_gn_bytes(n, cout, vox, epilogue) + pw_fwd_wpad_bytes(cin, cout);
}

int mednext_pw_fwd(const void* a, const void* wt, void* y, int prologue, const float* pro_stats,
                   const float* pro_gamma, const float* pro_beta, int epilogue, const float* bias,
                   const void* residual, const void* aux, const float* epi_stats, void* workspace,
                   size_t workspace_bytes, int64_t n, int64_t cin, int64_t cout, int64_t vox, int a_dtype,
                   int y_dtype, mednext_stream_t stream) {
  return mednext_pw_fwd_pro_out(a, wt, y, prologue, pro_stats, pro_gamma, pro_beta, epilogue, bias, residual, aux,
                                epi_stats, nullptr, workspace, workspace_bytes, n, cin, cout, vox, a_dtype, y_dtype,
                                stream);
}

// Argument checks and the kernel arguments shared by the forward-GEMM entry points.
static int pw_fwd_setup(const void* a, const void* wt, void* y, int prologue, const float* pro_stats,
                        const float* pro_gamma, const float* pro_beta, int epilogue, const float* bias,
                        const void* residual, const void* aux, const float* epi_stats, void* pro_out,
                        void* workspace, size_t workspace_bytes, int64_t n, int64_t cin, int64_t cout,
                        int64_t vox, int a_dtype, int y_dtype, PwFwdArgs* out) {
  if (!pw_dtype_ok(a_dtype)) return MEDNEXT_ERR_BAD_DTYPE;
  if (y_dtype != a_dtype && y_dtype != MEDNEXT_FLOAT32) return MEDNEXT_ERR_BAD_DTYPE;
  if (!pw_shape_ok(n, cin, cout, vox)) return MEDNEXT_ERR_BAD_SHAPE;
  if (prologue < MEDNEXT_PRO_NONE || prologue > MEDNEXT_PRO_GELU) return MEDNEXT_ERR_BAD_SHAPE;
  if (epilogue & ~15) return MEDNEXT_ERR_BAD_SHAPE;
  if (a == nullptr || wt == nullptr || y == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  if (prologue == MEDNEXT_PRO_GROUPNORM && (pro_stats == nullptr || pro_gamma == nullptr || pro_beta == nullptr))
    return MEDNEXT_ERR_NULL_POINTER;
  if ((epilogue & MEDNEXT_EPI_BIAS) && bias == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  if ((epilogue & MEDNEXT_EPI_RESIDUAL) && residual == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  if ((epilogue & (MEDNEXT_EPI_GELU_GRAD | MEDNEXT_EPI_GN_BWD_STATS)) && aux == nullptr)
    return MEDNEXT_ERR_NULL_POINTER;
  if ((epilogue & MEDNEXT_EPI_GN_BWD_STATS) && epi_stats == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  const size_t ws_need = mednext_pw_fwd_workspace_size(n, cin, cout, vox, epilogue);
  if (ws_need > 0 && (workspace == nullptr || !aligned16(workspace) || workspace_bytes < ws_need))
    return MEDNEXT_ERR_WORKSPACE;
  const size_t asz = elem_size(a_dtype), ysz = elem_size(y_dtype);
  if (!aligned(a, asz) || !aligned(wt, asz) || !aligned(y, ysz) || (residual && !aligned(residual, ysz)) ||
      (aux && !aligned(aux, asz)) || (pro_out && !aligned(pro_out, asz)))
    return MEDNEXT_ERR_ALIGNMENT;
  if (prologue == MEDNEXT_PRO_NONE) pro_out = nullptr;  // nothing transformed: nothing to write
  PwFwdArgs& args = *out;
  args = PwFwdArgs{};
  args.a = a; args.wt = wt; args.y = y;
  args.pro_stats = pro_stats; args.pro_gamma = pro_gamma; args.pro_beta = pro_beta;
  args.bias = bias; args.residual = residual; args.aux = aux; args.epi_stats = epi_stats;
  args.pro_out = pro_out;
  args.gn_part = static_cast<GnBwdPartial*>(workspace);
  args.S = (int)n; args.cin = (int)cin; args.cout = (int)cout; args.vox = vox;
  args.BN = pw_fwd_bn(n, cout, vox, prologue);
  args.mtiles = (int)((vox + kPwBM - 1) / kPwBM);
  args.ntiles = (int)((cout + args.BN - 1) / args.BN);
  args.epilogue = epilogue;
  args.vec_a = (vox % 8 == 0) && aligned16(a);
  args.vec_w = (cin % 8 == 0) && aligned16(wt);
  args.wpad = pw_fwd_wpad_bytes(cin, cout) > 0 ? static_cast<char*>(workspace) + pw_fwd_gn_bytes(n, cout, vox, epilogue)
                                              : nullptr;
  if ((long long)args.S * args.ntiles * args.mtiles >= (1LL << 31)) return MEDNEXT_ERR_BAD_SHAPE;
  return MEDNEXT_OK;
}

int mednext_pw_fwd_pro_out(const void* a, const void* wt, void* y, int prologue, const float* pro_stats,
                           const float* pro_gamma, const float* pro_beta, int epilogue, const float* bias,
                           const void* residual, const void* aux, const float* epi_stats, void* pro_out,
                           void* workspace, size_t workspace_bytes, int64_t n, int64_t cin, int64_t cout,
                           int64_t vox, int a_dtype, int y_dtype, mednext_stream_t stream) {
  PwFwdArgs args;
  const int st = pw_fwd_setup(a, wt, y, prologue, pro_stats, pro_gamma, pro_beta, epilogue, bias, residual, aux,
                              epi_stats, pro_out, workspace, workspace_bytes, n, cin, cout, vox, a_dtype, y_dtype,
                              &args);
  if (st != MEDNEXT_OK) return st;
  return dispatch_pw_fwd(a_dtype, y_dtype, prologue, args, as_stream(stream));
}

int mednext_pw_fwd_gelu_out(const void* a, const void* wt, void* y, void* g, int prologue, const float* pro_stats,
                            const float* pro_gamma, const float* pro_beta, const float* bias, void* workspace,
                            size_t workspace_bytes, int64_t n, int64_t cin, int64_t cout, int64_t vox, int dtype,
                            mednext_stream_t stream) {
  if (g == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  if (!aligned(g, elem_size(dtype))) return MEDNEXT_ERR_ALIGNMENT;
  PwFwdArgs args;
  const int epilogue = bias != nullptr ? MEDNEXT_EPI_BIAS : 0;
  const int st = pw_fwd_setup(a, wt, y, prologue, pro_stats, pro_gamma, pro_beta, epilogue, bias, nullptr, nullptr,
                              nullptr, nullptr, workspace, workspace_bytes, n, cin, cout, vox, dtype, dtype, &args);
  if (st != MEDNEXT_OK) return st;
  if (dtype != MEDNEXT_BFLOAT16 || prologue == MEDNEXT_PRO_GELU || vox % 8 != 0) return MEDNEXT_ERR_UNSUPPORTED;
  args.y2 = g;
  const int rc = pw_fwd_gelu_out_bf16(prologue, args, as_stream(stream));
  return rc == -1 ? MEDNEXT_ERR_UNSUPPORTED : rc;
}

static bool pw_gelu_bwd_covered(int64_t n, int64_t c, int64_t h, int64_t vox, int dtype) {
  return dtype == MEDNEXT_BFLOAT16 && pw_shape_ok(n, c, h, vox) && c % 16 == 0 && c <= kPwBK && h + 1 <= kPwBM &&
         vox % 8 == 0;
}

size_t mednext_pw_gelu_bwd_workspace_size(int64_t n, int64_t c, int64_t h, int64_t vox, int dtype) {
  if (!pw_gelu_bwd_covered(n, c, h, vox, dtype)) return 0;
  const long long tiles = n * ((vox + kPwBM - 1) / kPwBM);
  const size_t splits = (size_t)pw_fused_grid(tiles);
  return align_up(splits * c * h * 4, 256) + splits * c * 4;
}

int mednext_pw_gelu_bwd(const void* dy, const void* wpt, const void* u, void* du, float* dw, float* dbias,
                        void* workspace, size_t workspace_bytes, int64_t n, int64_t c, int64_t h, int64_t vox,
                        int dtype, mednext_stream_t stream) {
  if (!pw_dtype_ok(dtype)) return MEDNEXT_ERR_BAD_DTYPE;
  if (!pw_shape_ok(n, c, h, vox)) return MEDNEXT_ERR_BAD_SHAPE;
  if (dy == nullptr || wpt == nullptr || u == nullptr || du == nullptr || dw == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  if (!pw_gelu_bwd_covered(n, c, h, vox, dtype)) return MEDNEXT_ERR_UNSUPPORTED;
  const size_t ws_need = mednext_pw_gelu_bwd_workspace_size(n, c, h, vox, dtype);
  if (workspace == nullptr || !aligned16(workspace) || workspace_bytes < ws_need) return MEDNEXT_ERR_WORKSPACE;
  if (!aligned16(dy) || !aligned16(wpt) || !aligned16(u) || !aligned16(du) || !aligned(dw, 4) ||
      (dbias && !aligned(dbias, 4)))
    return MEDNEXT_ERR_ALIGNMENT;
  PwFwdArgs args{};
  args.a = dy; args.wt = wpt; args.y = du; args.aux = u;
  args.S = (int)n; args.cin = (int)c; args.cout = (int)h; args.vox = vox;
  args.BN = pw_bn(h);
  args.mtiles = (int)((vox + kPwBM - 1) / kPwBM);
  args.ntiles = (int)((h + args.BN - 1) / args.BN);
  args.epilogue = MEDNEXT_EPI_GELU_GRAD;
  args.vec_a = 1; args.vec_w = (c % 8 == 0) ? 1 : 0;
  const int splits = pw_fused_grid((long long)args.S * args.mtiles);
  args.w_part = static_cast<float*>(workspace);
  args.w_part_b = reinterpret_cast<float*>(static_cast<char*>(workspace) + align_up((size_t)splits * c * h * 4, 256));
  const int st = pw_gelu_bwd_bf16(args, as_stream(stream));
  if (st == -1) return MEDNEXT_ERR_UNSUPPORTED;
  if (st != MEDNEXT_OK) return st;
  // dw[c][h] = sum over the CTAs' partials (cout = c rows, cin = h columns), dbias[c]
  return dispatch_pw_wgrad_reduce(args.w_part, args.w_part_b, dw, dbias, splits, (int)c, (int)h, as_stream(stream));
}

int mednext_pw_mlp_fwd(const void* t, const float* stats, const float* gamma, const float* beta, const void* we,
                       const float* be, const void* wp, const float* bp, const void* residual, void* u, void* y,
                       int64_t n, int64_t c, int64_t h, int64_t c2, int64_t vox, int dtype, mednext_stream_t stream) {
  if (!pw_dtype_ok(dtype)) return MEDNEXT_ERR_BAD_DTYPE;
  if (!pw_shape_ok(n, c, h, vox) || !pw_shape_ok(n, h, c2, vox)) return MEDNEXT_ERR_BAD_SHAPE;
  if (t == nullptr || stats == nullptr || gamma == nullptr || beta == nullptr || we == nullptr || be == nullptr ||
      wp == nullptr || bp == nullptr || u == nullptr || y == nullptr)
    return MEDNEXT_ERR_NULL_POINTER;
  if (dtype != MEDNEXT_BFLOAT16 || c % 8 != 0 || c > kPwBK || h % 16 != 0 || h > kPwBM || c2 % 8 != 0 || c2 > 256 ||
      vox % 8 != 0)
    return MEDNEXT_ERR_UNSUPPORTED;
  if (!aligned16(t) || !aligned16(we) || !aligned16(wp) || !aligned16(u) || !aligned16(y) ||
      (residual && !aligned16(residual)) || !aligned(stats, 4) || !aligned(gamma, 4) || !aligned(beta, 4) ||
      !aligned(be, 4) || !aligned(bp, 4))
    return MEDNEXT_ERR_ALIGNMENT;
  PwFwdArgs args{};
  args.a = t; args.wt = we; args.y = u;
  args.pro_stats = stats; args.pro_gamma = gamma; args.pro_beta = beta;
  args.bias = be; args.residual = residual;
  args.S = (int)n; args.cin = (int)c; args.cout = (int)h; args.vox = vox;
  args.BN = pw_bn(h);
  args.mtiles = (int)((vox + kPwBM - 1) / kPwBM);
  args.ntiles = (int)((h + args.BN - 1) / args.BN);
  args.epilogue = MEDNEXT_EPI_BIAS;
  args.vec_a = 1; args.vec_w = 1;
  args.w2 = wp; args.bias2 = bp; args.y2 = y; args.cout2 = (int)c2;
  const int st = pw_mlp_fwd_bf16(args, as_stream(stream));
  return st == -1 ? MEDNEXT_ERR_UNSUPPORTED : st;
}

// h = channels of du (the GEMM's K), c = channels of dz and t (its output)
static bool pw_gn_bwd_covered(int64_t n, int64_t h, int64_t c, int64_t vox, int dtype) {
  return dtype == MEDNEXT_BFLOAT16 && pw_shape_ok(n, h, c, vox) && h % 16 == 0 && h <= kPwBK && c + 1 <= kPwBM &&
         vox % 8 == 0;
}

size_t mednext_pw_gn_bwd_fused_workspace_size(int64_t n, int64_t h, int64_t c, int64_t vox, int dtype) {
  if (!pw_gn_bwd_covered(n, h, c, vox, dtype)) return 0;
  const long long tiles = n * ((vox + kPwBM - 1) / kPwBM);
  const size_t splits = (size_t)pw_fused_grid(tiles);
  return pw_fwd_gn_bytes(n, c, vox, MEDNEXT_EPI_GN_BWD_STATS) + align_up(splits * h * c * 4, 256) + splits * h * 4;
}

int mednext_pw_gn_bwd_fused(const void* du, const void* wt, const void* t, const float* stats, const float* gamma,
                            const float* beta, void* dz, float* dw, float* dbias, void* workspace,
                            size_t workspace_bytes, int64_t n, int64_t h, int64_t c, int64_t vox, int dtype,
                            mednext_stream_t stream) {
  if (!pw_dtype_ok(dtype)) return MEDNEXT_ERR_BAD_DTYPE;
  if (!pw_shape_ok(n, h, c, vox)) return MEDNEXT_ERR_BAD_SHAPE;
  if (du == nullptr || wt == nullptr || t == nullptr || stats == nullptr || gamma == nullptr || beta == nullptr ||
      dz == nullptr || dw == nullptr)
    return MEDNEXT_ERR_NULL_POINTER;
  if (!pw_gn_bwd_covered(n, h, c, vox, dtype)) return MEDNEXT_ERR_UNSUPPORTED;
  const size_t ws_need = mednext_pw_gn_bwd_fused_workspace_size(n, h, c, vox, dtype);
  if (workspace == nullptr || !aligned16(workspace) || workspace_bytes < ws_need) return MEDNEXT_ERR_WORKSPACE;
  if (!aligned16(du) || !aligned16(wt) || !aligned16(t) || !aligned16(dz) || !aligned(dw, 4) || !aligned(stats, 4) ||
      !aligned(gamma, 4) || !aligned(beta, 4) || (dbias && !aligned(dbias, 4)))
    return MEDNEXT_ERR_ALIGNMENT;
  PwFwdArgs args{};
  args.a = du; args.wt = wt; args.y = dz; args.aux = t; args.epi_stats = stats;
  args.pro_gamma = gamma; args.pro_beta = beta;  // the fused GroupNorm(t) coefficients
  args.gn_part = static_cast<GnBwdPartial*>(workspace);
  args.S = (int)n; args.cin = (int)h; args.cout = (int)c; args.vox = vox;
  args.BN = pw_bn(c);
  args.mtiles = (int)((vox + kPwBM - 1) / kPwBM);
  args.ntiles = (int)((c + args.BN - 1) / args.BN);
  args.epilogue = MEDNEXT_EPI_GN_BWD_STATS;
  args.vec_a = 1; args.vec_w = (h % 8 == 0) ? 1 : 0;
  const int splits = pw_fused_grid((long long)args.S * args.mtiles);
  char* wbase = static_cast<char*>(workspace) + pw_fwd_gn_bytes(n, c, vox, MEDNEXT_EPI_GN_BWD_STATS);
  args.w_part = reinterpret_cast<float*>(wbase);
  args.w_part_b = reinterpret_cast<float*>(wbase + align_up((size_t)splits * h * c * 4, 256));
  const int st = pw_gn_bwd_bf16(args, as_stream(stream));
  if (st == -1) return MEDNEXT_ERR_UNSUPPORTED;
  if (st != MEDNEXT_OK) return st;
  // dw[h][c] = sum over the CTAs' partials (h rows, c columns), dbias[h]
  return dispatch_pw_wgrad_reduce(args.w_part, args.w_part_b, dw, dbias, splits, (int)h, (int)c, as_stream(stream));
}

size_t mednext_pw_wgrad_workspace_size(int64_t n, int64_t cin, int64_t cout, int64_t vox) {
  if (!pw_shape_ok(n, cin, cout, vox)) return 0;
  const PwWPlan p = plan_pw_wgrad(n, cin, cout, vox);
  return align_up((size_t)p.splits * cout * cin * 4, 256) + (size_t)p.splits * cout * 4;
}

int mednext_pw_wgrad(const void* g, const void* a, float* dw, float* dbias, int prologue, const float* pro_stats,
                     const float* pro_gamma, const float* pro_beta, void* workspace, size_t workspace_bytes,
                     int64_t n, int64_t cin, int64_t cout, int64_t vox, int dtype, mednext_stream_t stream) {
  if (!pw_dtype_ok(dtype)) return MEDNEXT_ERR_BAD_DTYPE;
  if (!pw_shape_ok(n, cin, cout, vox)) return MEDNEXT_ERR_BAD_SHAPE;
  if (prologue < MEDNEXT_PRO_NONE || prologue > MEDNEXT_PRO_GELU) return MEDNEXT_ERR_BAD_SHAPE;
  if (g == nullptr || a == nullptr || dw == nullptr) return MEDNEXT_ERR_NULL_POINTER;
  if (prologue == MEDNEXT_PRO_GROUPNORM && (pro_stats == nullptr || pro_gamma == nullptr || pro_beta == nullptr))
    return MEDNEXT_ERR_NULL_POINTER;
  const size_t esz = elem_size(dtype);
  if (!aligned(g, esz) || !aligned(a, esz) || !aligned(dw, 4) || (dbias && !aligned(dbias, 4)))
    return MEDNEXT_ERR_ALIGNMENT;
  if (workspace == nullptr || !aligned16(workspace) ||
      workspace_bytes < mednext_pw_wgrad_workspace_size(n, cin, cout, vox))
    return MEDNEXT_ERR_WORKSPACE;
  const PwWPlan p = plan_pw_wgrad(n, cin, cout, vox);
  PwWgradArgs args{};
  args.g = g; args.a = a;
  args.pro_stats = pro_stats; args.pro_gamma = pro_gamma; args.pro_beta = pro_beta;
  args.part = static_cast<float*>(workspace);
  args.part_b = reinterpret_cast<float*>(static_cast<char*>(workspace) + align_up((size_t)p.splits * cout * cin * 4, 256));
  args.dw = dw; args.dbias = dbias;
  args.S = (int)n; args.cin = (int)cin; args.cout = (int)cout; args.vox = vox;
  args.BN = p.BN; args.mtiles = p.mtiles; args.ntiles = p.ntiles; args.splits = p.splits;
  args.chunks_per_sample = p.cps; args.chunks_total = p.total; args.chunks_per_split = p.per;
  args.vec = (vox % 8 == 0) && aligned16(g) && aligned16(a);
  return dispatch_pw_wgrad(dtype, prologue, args, p.splits, as_stream(stream));
}

}  // extern "C"
