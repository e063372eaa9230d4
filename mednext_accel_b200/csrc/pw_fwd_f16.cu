// Forward / input-grad pointwise GEMM instantiations: fp16 inputs, fp16 or fp32 output.
#include "pw_launch.cuh"

namespace mednext {

using namespace pwl;

int pw_fwd_f16(int y_dtype, int prologue, const PwFwdArgs& a, cudaStream_t s) {
  return y_dtype == MEDNEXT_FLOAT32 ? pw_fwd_pro<__half, float>(prologue, a, s)
                                    : pw_fwd_pro<__half, __half>(prologue, a, s);
}
MEDNEXT_DEFINE_ERROR_READER(read_clear_errors_pwf2)

}  // namespace mednext
