// Template instantiation and launch of the tcgen05 pointwise kernels.
#include "plan.h"

namespace mednext {

namespace {
template <typename TA, typename TY, int PRO>
int launch_pw_fwd(const PwFwdArgs& a, cudaStream_t s) {
  auto kern = pw_fwd_kernel<TA, TY, PRO>;
  const size_t smem = pw_smem(a.BN);
  static size_t configured = 0;  // raise the opt-in limit once per instantiation
  if (smem > configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    configured = smem;
  }
  const long long grid = (long long)a.S * a.ntiles * a.mtiles;
  kern<<<(unsigned)grid, kPwThreads, smem, s>>>(a);
  return record_launch();
}
template <typename TA, int PRO>
int launch_pw_wgrad(const PwWgradArgs& a, cudaStream_t s) {
  auto kern = pw_wgrad_kernel<TA, PRO>;
  const size_t smem = pw_smem(a.BN);
  static size_t configured = 0;  // raise the opt-in limit once per instantiation
  if (smem > configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    configured = smem;
  }
  const long long grid = (long long)a.splits * a.ntiles * a.mtiles;
  kern<<<(unsigned)grid, kPwThreads, smem, s>>>(a);
  return record_launch();
}
template <typename TA, typename TY>
int pw_fwd_pro(int prologue, const PwFwdArgs& a, cudaStream_t s) {
  switch (prologue) {
    case MEDNEXT_PRO_NONE: return launch_pw_fwd<TA, TY, MEDNEXT_PRO_NONE>(a, s);
    case MEDNEXT_PRO_GROUPNORM: return launch_pw_fwd<TA, TY, MEDNEXT_PRO_GROUPNORM>(a, s);
    case MEDNEXT_PRO_GELU: return launch_pw_fwd<TA, TY, MEDNEXT_PRO_GELU>(a, s);
    default: return MEDNEXT_ERR_BAD_SHAPE;
  }
}
template <typename TA>
int pw_wgrad_pro(int prologue, const PwWgradArgs& a, cudaStream_t s) {
  switch (prologue) {
    case MEDNEXT_PRO_NONE: return launch_pw_wgrad<TA, MEDNEXT_PRO_NONE>(a, s);
    case MEDNEXT_PRO_GROUPNORM: return launch_pw_wgrad<TA, MEDNEXT_PRO_GROUPNORM>(a, s);
    case MEDNEXT_PRO_GELU: return launch_pw_wgrad<TA, MEDNEXT_PRO_GELU>(a, s);
    default: return MEDNEXT_ERR_BAD_SHAPE;
  }
}
}  // namespace

int dispatch_pw_fwd(int a_dtype, int y_dtype, int prologue, const PwFwdArgs& a, cudaStream_t s) {
  if (a_dtype == MEDNEXT_BFLOAT16) {
    return y_dtype == MEDNEXT_FLOAT32 ? pw_fwd_pro<__nv_bfloat16, float>(prologue, a, s)
                                      : pw_fwd_pro<__nv_bfloat16, __nv_bfloat16>(prologue, a, s);
  }
  if (a_dtype == MEDNEXT_FLOAT16) {
    return y_dtype == MEDNEXT_FLOAT32 ? pw_fwd_pro<__half, float>(prologue, a, s)
                                      : pw_fwd_pro<__half, __half>(prologue, a, s);
  }
  return MEDNEXT_ERR_BAD_DTYPE;
}

int dispatch_pw_wgrad(int dtype, int prologue, const PwWgradArgs& a, int splits, cudaStream_t s) {
  int st = MEDNEXT_ERR_BAD_DTYPE;
  if (dtype == MEDNEXT_BFLOAT16) st = pw_wgrad_pro<__nv_bfloat16>(prologue, a, s);
  if (dtype == MEDNEXT_FLOAT16) st = pw_wgrad_pro<__half>(prologue, a, s);
  if (st != MEDNEXT_OK) return st;
  const long long total = (long long)a.cout * a.cin + a.cout;
  pw_wgrad_reduce_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(a.part, a.part_b, a.dw, a.dbias, splits,
                                                                         a.cout, a.cin);
  return record_launch();
}

MEDNEXT_DEFINE_ERROR_READER(read_clear_errors_pw)

}  // namespace mednext
