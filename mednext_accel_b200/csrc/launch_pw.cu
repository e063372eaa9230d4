// Template instantiation and launch of the tcgen05 pointwise kernels.
//
// The persistent TMA kernels (pointwise_tma.cuh) run whenever every operand can
// be described by a TMA tensor map (16-byte aligned base and row strides, i.e.
// voxel count and channel counts multiples of 8 for 16-bit data); otherwise the
// first-generation kernels of pointwise.cuh stage the operands with threads.
#include "pw_launch.cuh"

namespace mednext {

using namespace pwl;

namespace {

// ------------------------------------------------------------------ wgrad (TMA)
template <typename TA, int PRO>
int try_pw_wgrad_tma(const PwWgradArgs& a, cudaStream_t s) {
  if (a.vox % 8 != 0 || !a16(a.g) || !a16(a.a)) return -1;
  PwTmaWgradCfg cfg{};
  // a bias row fits when all a rows sit in one N tile with a row to spare
  cfg.ones_row = (a.ntiles == 1 && a.cin < a.BN) ? a.cin : -1;
  cfg.g_rows = std::min(a.cout, kPwBM);
  cfg.a_rows = cfg.ones_row >= 0 ? a.cin : a.BN;
  CUtensorMap mG, mA;
  if (!encode3<TA>(&mG, a.g, (uint64_t)a.vox, (uint64_t)a.cout, (uint64_t)a.S, 64, (uint32_t)cfg.g_rows,
                   CU_TENSOR_MAP_SWIZZLE_128B))
    return -1;
  if (!encode3<TA>(&mA, a.a, (uint64_t)a.vox, (uint64_t)a.cin, (uint64_t)a.S, 64, (uint32_t)cfg.a_rows,
                   CU_TENSOR_MAP_SWIZZLE_128B))
    return -1;
  cfg.b_bytes = a.BN * 128;
  // two 64-voxel chunks per ring stage when four such stages fit: the hand-off
  // between the TMA producer and its consumers costs about the same per stage
  // whatever the stage holds, so larger stages stream faster
  const size_t per_chunk = 16384 + (size_t)cfg.b_bytes;
  cfg.nch = 4 * 2 * per_chunk <= kSmemBudget ? 2 : 1;
  const size_t per_stage = cfg.nch * per_chunk;
  // staged partial stores where a unit has few chunks (measured: level 2-4 weight
  // grads 10-20 % faster; at level 0-1 the larger L1 share is worth more): the ring,
  // the 1 KB alignment pad and the staging tiles within the 227 KB a CTA may hold
  // (2 KB left for the kernel's static shared memory)
  cfg.stage_epi = a.chunks_per_split < 16 ? 1 : 0;
  const size_t stg = cfg.stage_epi ? kWgStgBytes : 0;
  const size_t ring_budget = std::min<size_t>(kSmemBudget, 227 * 1024 - 1024 - stg - 2048);
  cfg.stages = (int)std::min<size_t>(kMaxStages, ring_budget / per_stage);
  if (cfg.stages < 2) return -1;
  cfg.units = a.mtiles * a.ntiles * a.splits;
  const size_t smem = 1024 + cfg.stages * per_stage + stg;
  auto kern = pw_tma_wgrad_kernel<TA, PRO>;
  if (const int rc = ensure_smem(kern, smem)) return rc;
  const int grid = std::min(cfg.units, num_sms());
  kern<<<grid, kWgThreads, smem, s>>>(mG, mA, a, cfg);
  return record_launch();
}

// ------------------------------------------------------------------ first-generation kernels
template <typename TA, int PRO>
int launch_pw_wgrad(const PwWgradArgs& a, cudaStream_t s) {
  const int st = try_pw_wgrad_tma<TA, PRO>(a, s);
  if (st != -1) return st;
  auto kern = pw_wgrad_kernel<TA, PRO>;
  const size_t smem = pw_smem(a.BN);
  if (const int rc = ensure_smem(kern, smem)) return rc;
  const long long grid = (long long)a.splits * a.ntiles * a.mtiles;
  kern<<<(unsigned)grid, kPwThreads, smem, s>>>(a);
  return record_launch();
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
  if (a_dtype == MEDNEXT_BFLOAT16)
    return y_dtype == MEDNEXT_FLOAT32 ? pw_fwd_bf16_f32(prologue, a, s) : pw_fwd_bf16_bf16(prologue, a, s);
  if (a_dtype == MEDNEXT_FLOAT16) return pw_fwd_f16(y_dtype, prologue, a, s);
  return MEDNEXT_ERR_BAD_DTYPE;
}

int dispatch_pw_wgrad(int dtype, int prologue, const PwWgradArgs& a, int splits, cudaStream_t s) {
  int st = MEDNEXT_ERR_BAD_DTYPE;
  if (dtype == MEDNEXT_BFLOAT16) st = pw_wgrad_pro<__nv_bfloat16>(prologue, a, s);
  if (dtype == MEDNEXT_FLOAT16) st = pw_wgrad_pro<__half>(prologue, a, s);
  if (st != MEDNEXT_OK) return st;
  return dispatch_pw_wgrad_reduce(a.part, a.part_b, a.dw, a.dbias, splits, a.cout, a.cin, s);
}

int dispatch_pw_wgrad_reduce(const float* part, const float* part_b, float* dw, float* dbias, int splits, int cout,
                             int cin, cudaStream_t s) {
  const long long total = (long long)cout * cin + cout;
  const int groups = splits >= 32 ? 8 : 1;
  const int per = kPwRedThreads / groups;
  pw_wgrad_reduce_kernel<<<(unsigned)((total + per - 1) / per), kPwRedThreads, 0, s>>>(part, part_b, dw, dbias,
                                                                                      splits, cout, cin, groups);
  return record_launch();
}

MEDNEXT_DEFINE_ERROR_READER(read_clear_errors_pw)

}  // namespace mednext
