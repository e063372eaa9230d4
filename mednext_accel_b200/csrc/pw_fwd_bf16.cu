// Forward / input-grad pointwise GEMM instantiations: bf16 inputs, bf16 output.
#include "pw_launch.cuh"

namespace mednext {

using namespace pwl;

int pw_fwd_bf16_bf16(int prologue, const PwFwdArgs& a, cudaStream_t s) {
  return pw_fwd_pro<__nv_bfloat16, __nv_bfloat16>(prologue, a, s);
}

// Compress input grad with the compress weight grad fused in (kEpiFusedWgrad):
// MEDNEXT_OK when launched, -1 when the shape or the shared-memory plan does not
// allow it (the caller then runs the two GEMMs separately).
int pw_gelu_bwd_bf16(const PwFwdArgs& a, cudaStream_t s) {
  return try_pw_fwd_tma<__nv_bfloat16, __nv_bfloat16, MEDNEXT_PRO_NONE, MEDNEXT_EPI_GELU_GRAD | kEpiFusedWgrad>(a, s);
}
// Expand input grad with the GroupNorm-backward sums and the expand weight grad fused in.
int pw_gn_bwd_bf16(const PwFwdArgs& a, cudaStream_t s) {
  return try_pw_fwd_tma<__nv_bfloat16, __nv_bfloat16, MEDNEXT_PRO_NONE, MEDNEXT_EPI_GN_BWD_STATS | kEpiFusedWgrad>(a,
                                                                                                             s);
}
// The block's whole expansion (GroupNorm prologue, expand GEMM + bias, GELU, compress
// GEMM + bias + residual) in one kernel.
int pw_mlp_fwd_bf16(const PwFwdArgs& a, cudaStream_t s) {
  return try_pw_fwd_tma<__nv_bfloat16, __nv_bfloat16, MEDNEXT_PRO_GROUPNORM, MEDNEXT_EPI_BIAS | kEpiMlp>(a, s);
}
int pw_fwd_gelu_out_bf16(int prologue, const PwFwdArgs& a, cudaStream_t s) {
  using T = __nv_bfloat16;
  const bool bias = (a.epilogue & MEDNEXT_EPI_BIAS) != 0;
  if (prologue == MEDNEXT_PRO_GROUPNORM)
    return bias ? try_pw_fwd_tma<T, T, MEDNEXT_PRO_GROUPNORM, MEDNEXT_EPI_BIAS | kEpiGeluOut>(a, s)
                : try_pw_fwd_tma<T, T, MEDNEXT_PRO_GROUPNORM, kEpiGeluOut>(a, s);
  return bias ? try_pw_fwd_tma<T, T, MEDNEXT_PRO_NONE, MEDNEXT_EPI_BIAS | kEpiGeluOut>(a, s)
              : try_pw_fwd_tma<T, T, MEDNEXT_PRO_NONE, kEpiGeluOut>(a, s);
}
int pw_fused_grid(long long total_tiles) { return (int)std::min<long long>(total_tiles, num_sms()); }
MEDNEXT_DEFINE_ERROR_READER(read_clear_errors_pwf0)

}  // namespace mednext
