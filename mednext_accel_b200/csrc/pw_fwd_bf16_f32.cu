// Forward / input-grad pointwise GEMM instantiations: bf16 inputs, fp32 output (residual add into an fp32 block input).
#include "pw_launch.cuh"

namespace mednext {

using namespace pwl;

int pw_fwd_bf16_f32(int prologue, const PwFwdArgs& a, cudaStream_t s) {
  return pw_fwd_pro<__nv_bfloat16, float>(prologue, a, s);
}
MEDNEXT_DEFINE_ERROR_READER(read_clear_errors_pwf1)

}  // namespace mednext
