// Host helpers shared by the pointwise launch units: TMA tensor-map encoding,
// shared-memory opt-in, and the forward-GEMM launcher templated on prologue and
// epilogue, instantiated per element type in pw_fwd_*.cu so that the library
// builds in parallel.
#pragma once

#include <cudaTypedefs.h>

#include <cstring>
#include <type_traits>

#include "plan.h"
#include "pointwise_tma.cuh"
#include "tma_host.h"

namespace mednext {
namespace pwl {

using namespace tma;

inline bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
constexpr size_t kSmemBudget = 220 * 1024;
constexpr size_t kWResidentBytes = 64 * 1024;  // largest W operand kept resident in the forward kernel
// SM count of the current device (queried per call: a process may drive
// several devices, and the runtime caches the attribute).
inline int num_sms() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      sms <= 0)
    return 148;
  return sms;
}

// ------------------------------------------------------------------ forward (TMA)
// Returns MEDNEXT_OK when launched, -1 when the shape is not TMA-describable.
template <typename TA, typename TY, int PRO, int EPI>
int try_pw_fwd_tma(const PwFwdArgs& a, cudaStream_t s) {
  if (a.vox % 8 != 0 || !a16(a.a) || !a16(a.wt)) return -1;
  // W rows must be whole 16-byte chunks for its tensor map: pad them in the workspace
  const void* wt = a.wt;
  int wk = a.cin;
  if (a.cin % 8 != 0) {
    if (a.wpad == nullptr || !a16(a.wpad)) return -1;
    wk = (a.cin + 7) / 8 * 8;
    const long long total = (long long)a.cout * wk;
    pw_pad_weight_kernel<TA><<<(unsigned)((total + 255) / 256), 256, 0, s>>>(
        static_cast<const TA*>(a.wt), static_cast<TA*>(a.wpad), a.cout, a.cin, wk);
    const int st = record_launch();
    if (st != MEDNEXT_OK) return st;
    wt = a.wpad;
  }
  constexpr bool MLP = EPI >= 0 && (EPI & kEpiMlp) != 0;
  const bool has_aux = (a.epilogue & (MEDNEXT_EPI_GELU_GRAD | MEDNEXT_EPI_GN_BWD_STATS)) != 0;
  // (the fused expansion's residual belongs to its second GEMM)
  const bool has_res = MLP ? a.residual != nullptr : (a.epilogue & MEDNEXT_EPI_RESIDUAL) != 0;
  const bool pro_store = PRO != MEDNEXT_PRO_NONE && a.pro_out != nullptr;
  if ((has_aux && !a16(a.aux)) || (has_res && !a16(a.residual))) return -1;
  if (!a16(a.y) || (pro_store && !a16(a.pro_out))) return -1;
  CUtensorMap mA, mB, mAux, mRes, mY, mP, mB2, mY2;
  memset(&mAux, 0, sizeof(mAux));
  memset(&mRes, 0, sizeof(mRes));
  memset(&mP, 0, sizeof(mP));
  memset(&mB2, 0, sizeof(mB2));
  memset(&mY2, 0, sizeof(mY2));
  // fused expansion: one K stage and one N tile in the first GEMM, H <= 128 rows of the g
  // tile, the second GEMM's N a legal MMA N
  const int bn2 = MLP ? (a.cout2 + 15) / 16 * 16 : 0;
  if (MLP && (a.cin > kPwBK || a.ntiles != 1 || a.cout % 16 != 0 || a.cout > kPwBM || bn2 < 16 || bn2 > 256 ||
              a.w2 == nullptr || a.y2 == nullptr || a.bias2 == nullptr || !a16(a.w2) || !a16(a.y2)))
    return -1;
  // 16-bit outputs: the fragment epilogue stages 32-voxel x 16-channel blocks with a
  // 64-byte swizzle and reads the aux / residual tiles with a 128-byte swizzle
  constexpr bool kFrag = sizeof(TY) == 2;
  const CUtensorMapSwizzle sw_out = kFrag ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE;
  const CUtensorMapSwizzle sw_opnd = kFrag ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE;
  if (!encode3<TY>(&mY, a.y, (uint64_t)a.vox, (uint64_t)a.cout, (uint64_t)a.S, 32, kPwCW, sw_out))
    return -1;
  const int a_rows = std::min(kPwBK, (a.cin + 15) / 16 * 16);
  if (!encode3<TA>(&mA, a.a, (uint64_t)a.vox, (uint64_t)a.cin, (uint64_t)a.S, 64, (uint32_t)a_rows,
                   CU_TENSOR_MAP_SWIZZLE_128B))
    return -1;
  // the prologue output leaves through the A stage's own (swizzled) layout
  if (pro_store && !encode3<TA>(&mP, a.pro_out, (uint64_t)a.vox, (uint64_t)a.cin, (uint64_t)a.S, 64,
                                (uint32_t)a_rows, CU_TENSOR_MAP_SWIZZLE_128B))
    return -1;
  if (!encode2<TA>(&mB, wt, (uint64_t)wk, (uint64_t)a.cout, kPwBK, (uint32_t)a.BN, CU_TENSOR_MAP_SWIZZLE_128B))
    return -1;
  if (has_aux && !encode3<TA>(&mAux, a.aux, (uint64_t)a.vox, (uint64_t)a.cout, (uint64_t)a.S, 64, (uint32_t)a.BN,
                              sw_opnd))
    return -1;
  const int res_rows = MLP ? a.cout2 : a.cout, res_bn = MLP ? bn2 : a.BN;
  if (has_res && !encode3<TY>(&mRes, a.residual, (uint64_t)a.vox, (uint64_t)res_rows, (uint64_t)a.S, 64,
                              (uint32_t)res_bn, sw_opnd))
    return -1;
  constexpr bool GOUT = FwdEpi<PRO, EPI>::gelu_out;
  if constexpr (GOUT) {
    // g = GELU(y): a second output of y's shape through the second output map
    if (!kFrag || a.y2 == nullptr || !a16(a.y2) ||
        !encode3<TY>(&mY2, a.y2, (uint64_t)a.vox, (uint64_t)a.cout, (uint64_t)a.S, 32, kPwCW, sw_out))
      return -1;
  }
  if (MLP) {
    if (!encode2<TA>(&mB2, a.w2, (uint64_t)a.cout, (uint64_t)a.cout2, kPwBK, (uint32_t)bn2, CU_TENSOR_MAP_SWIZZLE_128B))
      return -1;
    if (!encode3<TY>(&mY2, a.y2, (uint64_t)a.vox, (uint64_t)a.cout2, (uint64_t)a.S, 32, kPwCW, sw_out))
      return -1;
  }
  // fused compress weight grad (kEpiFusedWgrad): one K stage and one N tile, H + 1
  // rows of g within the 128-row MMA, the dy channels a legal MMA N
  constexpr bool FW = EPI >= 0 && (EPI & kEpiFusedWgrad) != 0;
  if (FW && (a.cin > kPwBK || a.ntiles != 1 || a.cout + 1 > kPwBM || a.cin % 16 != 0 || a.cin > 256 ||
             a.w_part == nullptr || a.w_part_b == nullptr))
    return -1;
  PwTmaCfg cfg{};
  cfg.a_rows = a_rows;
  cfg.pro_store = pro_store ? 1 : 0;
  cfg.kstages = (a.cin + kPwBK - 1) / kPwBK;
  cfg.total_tiles = a.S * a.ntiles * a.mtiles;
  cfg.b_bytes = a.BN * 128;
  // one N tile and a small W: load it once per CTA instead of once per ring stage
  cfg.w_res = (a.ntiles == 1 && (size_t)cfg.kstages * cfg.b_bytes <= kWResidentBytes) ? 1 : 0;
  const size_t w_bytes = cfg.w_res ? (size_t)cfg.kstages * cfg.b_bytes : 0;
  cfg.aux_bytes = has_aux ? a.BN * 64 * (int)sizeof(TA) * 2 : 0;
  cfg.res_bytes = has_res ? res_bn * 64 * (int)sizeof(TY) * 2 : 0;
  if (MLP && !cfg.w_res) return -1;
  cfg.ks2 = MLP ? (a.cout + kPwBK - 1) / kPwBK : 0;
  cfg.b2_bytes = MLP ? bn2 * 128 : 0;
  cfg.bn2 = bn2;
  const size_t w2_bytes = (size_t)cfg.ks2 * cfg.b2_bytes;
  cfg.a_slot = 2 * 128 * a_rows;  // a multiple of 4 KB: the boxes stay 1 KB aligned for the swizzle
  const size_t per_stage = (size_t)cfg.a_slot + (cfg.w_res ? 0 : (size_t)cfg.b_bytes);
  const size_t ebytes = (size_t)cfg.aux_bytes + cfg.res_bytes;
  // epilogue staging: 2 buffers per warp (4 with the GELU output)
  const size_t stg = (size_t)FwdEpi<PRO, EPI>::warps * FwdEpi<PRO, EPI>::stg_bufs * 32 * kPwCW * sizeof(TY);
  const size_t g_bytes = (FW || MLP) ? 1024 + 2 * (size_t)kFwGBytes : 0;       // two g tiles, 1 KB aligned
  const size_t budget = kSmemBudget - stg - w_bytes - g_bytes - w2_bytes;
  // Epilogue-operand ring: 4 or 2 stages while keeping at least 4 A/W stages,
  // else 1.  Two epilogue warp groups take alternate tiles only when every ring
  // slot then belongs to one group (an even ring, or none): a slot shared by two
  // groups would let one of them wait on a phase parity two fills ahead.
  cfg.estages = 1;
  if (ebytes > 0) {
    // (the fused weight grad and the fused expansion need the two groups, so they settle
    // for kFwLag + 1 A/W stages)
    const size_t min_a = (FW || MLP) ? kFwLag + 1 : 4;
    if (4 * ebytes + min_a * per_stage <= budget) cfg.estages = 4;
    else if (2 * ebytes + min_a * per_stage <= budget) cfg.estages = 2;
  }
  cfg.tgroups = (ebytes == 0 || cfg.estages % 2 == 0) ? 2 : 1;
  // an odd number of 4-warp epilogue groups (the GELU-output variant's 12 warps) stays one group
  if ((FwdEpi<PRO, EPI>::warps / 4) % 2 != 0) cfg.tgroups = 1;
  // the fused weight grad gives each of the two epilogue groups its own g tile
  if ((FW || MLP) && cfg.tgroups != 2) return -1;
  // extra TMEM: the fused weight grad's accumulator, or the fused expansion's two second-GEMM ones
  cfg.d2_stride = MLP ? (int)tmem_cols_for(bn2) : 0;
  const uint32_t wcols = FW ? tmem_cols_for(a.cin) : (MLP ? 2u * (uint32_t)cfg.d2_stride : 0u);
  cfg.nacc = (int)std::min<uint32_t>(kMaxAcc, (512u - wcols) / tmem_cols_for(a.BN));
  if (cfg.nacc < 1) return -1;
  {
    cfg.d2_col = cfg.nacc * (int)tmem_cols_for(a.BN);
    uint32_t cols = (uint32_t)cfg.nacc * tmem_cols_for(a.BN) + wcols, pow2 = 32;
    while (pow2 < cols) pow2 <<= 1;
    cfg.tmem_cols = (int)pow2;
  }
  const long long room = (long long)budget - (long long)cfg.estages * (long long)ebytes;
  cfg.stages = (int)std::min<long long>(kMaxStages, room / (long long)per_stage);
  // a stage of the fused weight grad is held until kFwLag tiles later
  if (cfg.stages < 2 || (pro_store && cfg.stages <= kProStoreLag) || ((FW || MLP) && cfg.stages <= kFwLag)) return -1;
  const size_t smem = 1024 + cfg.stages * per_stage + w_bytes + w2_bytes + cfg.estages * ebytes + stg + g_bytes;
  auto kern = pw_tma_fwd_kernel<TA, TY, PRO, EPI>;
  if (const int rc = ensure_smem(kern, smem)) return rc;
  const int grid = std::min(cfg.total_tiles, num_sms());
  kern<<<grid, kFwdThreads, smem, s>>>(mA, mB, mAux, mRes, mY, mP, mB2, mY2, a, cfg);
  return record_launch();
}

// ------------------------------------------------------------------ forward launch
template <typename TA, typename TY, int PRO, int EPI>
int launch_pw_fwd(const PwFwdArgs& a, cudaStream_t s) {
  const int st = try_pw_fwd_tma<TA, TY, PRO, EPI>(a, s);
  if (st != -1) return st;
  auto kern = pw_fwd_kernel<TA, TY, PRO>;
  const size_t smem = pw_smem(a.BN);
  if (const int rc = ensure_smem(kern, smem)) return rc;
  const long long grid = (long long)a.S * a.ntiles * a.mtiles;
  kern<<<(unsigned)grid, kPwThreads, smem, s>>>(a);
  int rc = record_launch();
  if (rc != MEDNEXT_OK || PRO == MEDNEXT_PRO_NONE || a.pro_out == nullptr) return rc;
  // the first-generation kernel keeps its transformed tiles private: write pro(a) separately
  const long long total = (long long)a.S * a.cin * a.vox;
  const unsigned blocks = (unsigned)std::min<long long>((total + 255) / 256, 148LL * 32);
  pw_prologue_out_kernel<TA, PRO><<<blocks, 256, 0, s>>>(static_cast<const TA*>(a.a), static_cast<TA*>(a.pro_out),
                                                         a.pro_stats, a.pro_gamma, a.pro_beta, a.cin, a.vox, total);
  return record_launch();
}
// Compile-time epilogue for the flag sets the MedNeXt block uses; any other set
// runs the same kernel with the flags read at run time.
template <typename TA, typename TY, int PRO>
int pw_fwd_epi(const PwFwdArgs& a, cudaStream_t s) {
  constexpr int B = MEDNEXT_EPI_BIAS, R = MEDNEXT_EPI_RESIDUAL, G = MEDNEXT_EPI_GELU_GRAD,
                N = MEDNEXT_EPI_GN_BWD_STATS;
  const int e = a.epilogue;
  if constexpr (std::is_same<TA, __nv_bfloat16>::value) {
    if constexpr (PRO == MEDNEXT_PRO_NONE) {
      if (e == 0) return launch_pw_fwd<TA, TY, PRO, 0>(a, s);
      if (e == B) return launch_pw_fwd<TA, TY, PRO, B>(a, s);
      if (e == G) return launch_pw_fwd<TA, TY, PRO, G>(a, s);
      if (e == N) return launch_pw_fwd<TA, TY, PRO, N>(a, s);
    } else if constexpr (PRO == MEDNEXT_PRO_GROUPNORM) {
      if (e == B) return launch_pw_fwd<TA, TY, PRO, B>(a, s);
    } else {
      if (e == B) return launch_pw_fwd<TA, TY, PRO, B>(a, s);
      if (e == (B | R)) return launch_pw_fwd<TA, TY, PRO, B | R>(a, s);
    }
  }
  return launch_pw_fwd<TA, TY, PRO, kEpiRuntime>(a, s);
}
template <typename TA, typename TY>
int pw_fwd_pro(int prologue, const PwFwdArgs& a, cudaStream_t s) {
  switch (prologue) {
    case MEDNEXT_PRO_NONE: return pw_fwd_epi<TA, TY, MEDNEXT_PRO_NONE>(a, s);
    case MEDNEXT_PRO_GROUPNORM: return pw_fwd_epi<TA, TY, MEDNEXT_PRO_GROUPNORM>(a, s);
    case MEDNEXT_PRO_GELU: return pw_fwd_epi<TA, TY, MEDNEXT_PRO_GELU>(a, s);
    default: return MEDNEXT_ERR_BAD_SHAPE;
  }
}

}  // namespace pwl
}  // namespace mednext
