// Forward / input-grad pointwise GEMM instantiations: bf16 inputs, bf16 output.
#include "pw_launch.cuh"

namespace mednext {

using namespace pwl;

int pw_fwd_bf16_bf16(int prologue, const PwFwdArgs& a, cudaStream_t s) {
  return pw_fwd_pro<__nv_bfloat16, __nv_bfloat16>(prologue, a, s);
}
MEDNEXT_DEFINE_ERROR_READER(read_clear_errors_pwf0)

}  // namespace mednext
