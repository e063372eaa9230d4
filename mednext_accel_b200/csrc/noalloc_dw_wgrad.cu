// mednext_dw_wgrad_noalloc: the stride-1 depthwise weight gradient for hosts
// that cannot give the library a workspace (a host with a fixed device-memory
// budget taken at start-up, or one that keeps cudaMalloc/cudaFree, and the
// device-wide synchronisation of cudaFree, out of its training loop).
//
// The partial sums that mednext_dw_wgrad keeps in the caller's workspace live
// here in a file-scope device array instead, one copy per device.  The array
// never has to start at zero: the partial-sum kernels write every slot that the
// finishing kernel reads.  Every call on a device shares the one array, so
// calls that can overlap (unordered streams, several host threads) race.
#include <mutex>

#include "plan.h"

namespace mednext {
namespace {

constexpr size_t kScratchBytes = MEDNEXT_DW_WGRAD_NOALLOC_MAX_SCRATCH;
static_assert(kScratchBytes % 256 == 0, "scratch size must keep 256-byte granularity");

static __device__ __align__(256) unsigned char g_dw_wgrad_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the array on the current device, looked up once per device
// (the first lookup loads this library's module on that device if it is not
// loaded yet).
int scratch_on_current_device(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cudaGetLastError();
    note_cuda_error(e);
    return MEDNEXT_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) return MEDNEXT_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_dw_wgrad_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      note_cuda_error(e);
      return MEDNEXT_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return MEDNEXT_OK;
}

}  // namespace
}  // namespace mednext

using namespace mednext;

int mednext_dw_wgrad_noalloc(const void* x, const void* dy, void* dweight, void* dbias, int64_t n, int64_t c,
                             int64_t d, int64_t h, int64_t w, int k, int dtype, mednext_stream_t stream) {
  const size_t need = mednext_dw_wgrad_workspace_size(n, c, d, h, w, k, dtype);
  if (need == 0)  // invalid shape, kernel size or dtype: let the checked entry point say which
    return mednext_dw_wgrad(x, dy, dweight, dbias, nullptr, 0, n, c, d, h, w, k, dtype, stream);
  if (need > kScratchBytes) return MEDNEXT_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  const int st = scratch_on_current_device(&scratch);
  if (st != MEDNEXT_OK) return st;
  return mednext_dw_wgrad(x, dy, dweight, dbias, scratch, kScratchBytes, n, c, d, h, w, k, dtype, stream);
}
