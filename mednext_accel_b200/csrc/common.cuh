// Shared device helpers for the sm_100a MedNeXt kernels: element traits,
// 16-byte chunk unpacking, bounded mbarrier waits, the device error word and
// thin inline-PTX wrappers for tcgen05 (TMEM alloc / MMA / commit / ld).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mednext_b200.h"

namespace mednext {

// ----------------------------------------------------------------------------
// Element traits.  Acc is the accumulation type: fp64 inputs accumulate in
// fp64 (the reference does the same, ops/_triton/depthwise.py:190,299), all
// other inputs accumulate in fp32.
// ----------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  using Acc = float;
  static __device__ __forceinline__ float load(const float* p) { return *p; }
  static __device__ __forceinline__ float from(float v) { return v; }
  static __device__ __forceinline__ float to(float v) { return v; }
};
template <> struct Elem<double> {
  using Acc = double;
  static __device__ __forceinline__ double from(double v) { return v; }
  static __device__ __forceinline__ double to(double v) { return v; }
};
template <> struct Elem<__nv_bfloat16> {
  using Acc = float;
  static __device__ __forceinline__ float from(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 to(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Elem<__half> {
  using Acc = float;
  static __device__ __forceinline__ float from(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half to(float v) { return __float2half_rn(v); }
};

template <typename T>
__device__ __forceinline__ typename Elem<T>::Acc to_acc(T v) {
  return Elem<T>::from(v);
}
template <typename T, typename A>
__device__ __forceinline__ T from_acc(A v) {
  return Elem<T>::to(v);
}

// Unpack one 16-byte chunk holding 16/sizeof(T) elements into Acc values.
template <typename T>
__device__ __forceinline__ void unpack16(const uint4& q, typename Elem<T>::Acc* out);
template <>
__device__ __forceinline__ void unpack16<float>(const uint4& q, float* out) {
  out[0] = __uint_as_float(q.x);
  out[1] = __uint_as_float(q.y);
  out[2] = __uint_as_float(q.z);
  out[3] = __uint_as_float(q.w);
}
template <>
__device__ __forceinline__ void unpack16<double>(const uint4& q, double* out) {
  out[0] = __hiloint2double(q.y, q.x);
  out[1] = __hiloint2double(q.w, q.z);
}
template <>
__device__ __forceinline__ void unpack16<__nv_bfloat16>(const uint4& q, float* out) {
  // bf16 -> fp32 is exact: the bf16 bits become the top half of the fp32.
  const uint32_t v[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = __uint_as_float(v[i] << 16);
    out[2 * i + 1] = __uint_as_float(v[i] & 0xffff0000u);
  }
}
template <>
__device__ __forceinline__ void unpack16<__half>(const uint4& q, float* out) {
  const uint32_t v[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&v[i]);
    float2 f = __half22float2(h);
    out[2 * i] = f.x;
    out[2 * i + 1] = f.y;
  }
}

// Pack 16/sizeof(T) Acc values into one 16-byte chunk (round to nearest even).
template <typename T>
__device__ __forceinline__ uint4 pack16(const typename Elem<T>::Acc* in);
template <>
__device__ __forceinline__ uint4 pack16<float>(const float* in) {
  return make_uint4(__float_as_uint(in[0]), __float_as_uint(in[1]), __float_as_uint(in[2]),
                    __float_as_uint(in[3]));
}
template <>
__device__ __forceinline__ uint4 pack16<double>(const double* in) {
  return make_uint4(__double2loint(in[0]), __double2hiint(in[0]), __double2loint(in[1]),
                    __double2hiint(in[1]));
}
template <>
__device__ __forceinline__ uint4 pack16<__nv_bfloat16>(const float* in) {
  uint32_t v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 b = __floats2bfloat162_rn(in[2 * i], in[2 * i + 1]);
    v[i] = *reinterpret_cast<uint32_t*>(&b);
  }
  return make_uint4(v[0], v[1], v[2], v[3]);
}
template <>
__device__ __forceinline__ uint4 pack16<__half>(const float* in) {
  uint32_t v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = __floats2half2_rn(in[2 * i], in[2 * i + 1]);
    v[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(v[0], v[1], v[2], v[3]);
}

// ----------------------------------------------------------------------------
// Device error word.  Kernels never trap; a wait that exceeds its bound
// records a code here and the kernel returns.
// ----------------------------------------------------------------------------
enum DeviceError : int {
  kErrNone = 0,
  kErrMbarTimeout = 0x100,
  kErrTmemAlloc = 0x200,
  kErrBadTarget = 0x300,  // a class index outside [0, K) that is not ignore_index
};
// One word per translation unit (internal linkage); mednext_device_error()
// reads and clears all of them.
static __device__ int g_device_error = 0;

__device__ __forceinline__ void raise_device_error(int code) { atomicCAS(&g_device_error, 0, code); }

// ----------------------------------------------------------------------------
// mbarrier helpers (shared::cta).  Every wait is bounded.
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// (no memory clobber: the stores target a buffer this thread does not read; the
// asm-volatile fences and barriers that publish it keep their order)
__device__ __forceinline__ void st_shared_b16(uint32_t addr, uint16_t v) {
  asm volatile("st.shared.b16 [%0], %1;" ::"r"(addr), "h"(v));
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bound on one wait: far above any legitimate wait in these kernels (they
// wait microseconds for a copy or an MMA), far below anything that would
// look like a hung GPU.
constexpr uint64_t kMaxWaitNs = 250ull * 1000ull * 1000ull;

// Returns false (and records the error) when the bound is exceeded.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i) {
      if (mbar_try_wait(bar, parity)) return true;
    }
    if (global_timer_ns() - t0 > kMaxWaitNs) break;
  }
  raise_device_error(kErrMbarTimeout);
  return false;
}

// ----------------------------------------------------------------------------
// tcgen05 wrappers (PTX ISA 8.6+, sm_100a).
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Make generic-proxy shared-memory writes visible to the async proxy (MMA/TMA).
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16, issued by one thread.
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier once all previously issued MMAs of this thread finish.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns; thread i of the warp gets lane
// (warp%4)*32 + i.  Must be followed by tmem_ld_wait() before use.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 32 lanes x 16 consecutive 32-bit columns, same lane mapping as tmem_ld32.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// 16 lanes x 16 consecutive 32-bit columns in the MMA-fragment layout: thread t
// gets r[0..1] = (lane base + t/4, columns 2(t%4), 2(t%4)+1), r[2..3] = (lane
// base + 8 + t/4, the same columns), r[4..7] = the same at columns + 8.  The lane
// base must lie in the warp's own 32-lane quarter.  Followed by tmem_ld_wait().
__device__ __forceinline__ void tmem_ld_16x256b_x2(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(taddr));
}
// Four 8x8 16-bit matrices from shared memory, transposed: lanes 8m..8m+7 give
// the addresses of matrix m's eight 16-byte rows; thread t receives in q[m]
// (row 2(t%4), column t/4) in the low half and (row 2(t%4)+1, column t/4) in the high.
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t* q) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(q[0]), "=r"(q[1]), "=r"(q[2]), "=r"(q[3])
               : "r"(addr));
}
// The inverse: thread t's q[m] low/high halves land at (row 2(t%4) / 2(t%4)+1,
// column t/4) of matrix m, whose row addresses lanes 8m..8m+7 give.
__device__ __forceinline__ void stsm_x4_trans(uint32_t addr, const uint32_t* q) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(q[0]),
               "r"(q[1]), "r"(q[2]), "r"(q[3])
               : "memory");
}
// Two 16-bit values (low, high halves) <-> a float pair.
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t v);
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t v) {
  return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t v) {
  return __half22float2(*reinterpret_cast<const __half2*>(&v));
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(float2 v);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float2 v) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(v.x, v.y);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float2 v) {
  const __half2 h = __floats2half2_rn(v.x, v.y);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ----------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor) loads and stores, no multicast.
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N committed bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Shared-memory matrix descriptor for tcgen05.mma, SWIZZLE_128B layouts.
//   K-major: 8-row x 128-byte atoms; sbo = byte stride between 8-row groups.
//   MN-major: 64-element x 8-k atoms; lbo = byte stride between atoms along
//   M/N, sbo = byte stride between atoms along K.
// Bits: [0,14) addr>>4, [16,30) lbo>>4, [32,46) sbo>>4, [46,48) version=1,
// [61,64) layout (2 = SWIZZLE_128B).
__device__ __forceinline__ uint64_t make_sw128_desc(uint32_t smem_addr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
// Instruction descriptor, kind::f16 with fp32 accumulation.
//   ab_bf16: operands are bf16 (else fp16); a_mn / b_mn: operand is MN-major.
__host__ __device__ constexpr uint32_t make_idesc_f16(int M, int N, bool ab_bf16, bool a_mn,
                                                      bool b_mn) {
  return (1u << 4)                                     // D = f32
         | ((ab_bf16 ? 1u : 0u) << 7)                  // A format
         | ((ab_bf16 ? 1u : 0u) << 10)                 // B format
         | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// 2^x and 1/x by the PTX approximate instructions (relative error about 2^-22;
// denormal results flush to zero).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Mixed-precision FMA (sm_100): a * b + c with 16-bit a, b and an fp32 c, d.  The
// product of two 16-bit floats is exact in fp32, so the result is fmaf of the
// widened operands, with no widening instructions: the operands are halves of
// 32-bit registers.
template <typename T>
__device__ __forceinline__ float mix_fma(uint16_t a, uint16_t b, float c);
template <>
__device__ __forceinline__ float mix_fma<__nv_bfloat16>(uint16_t a, uint16_t b, float c) {
  float d;
  asm("fma.rn.f32.bf16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
  return d;
}
template <>
__device__ __forceinline__ float mix_fma<__half>(uint16_t a, uint16_t b, float c) {
  float d;
  asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
  return d;
}
// the 16-bit bit pattern of 1.0
template <typename T>
__device__ __forceinline__ uint16_t one16();
template <>
__device__ __forceinline__ uint16_t one16<__nv_bfloat16>() {
  return 0x3f80u;
}
template <>
__device__ __forceinline__ uint16_t one16<__half>() {
  return 0x3c00u;
}
// element i of an array of 32-bit words read as 16-bit elements (little endian:
// element 2q is the low half of word q)
template <int N>
__device__ __forceinline__ uint16_t half16(const uint32_t (&w)[N], int i) {
  return (i & 1) ? (uint16_t)(w[i >> 1] >> 16) : (uint16_t)(w[i >> 1] & 0xffffu);
}

// Exact (erf-form) GELU of F.gelu(approximate="none"): x * Phi(x), with
// Phi(x) = erfc(-x / sqrt 2) / 2.  erfc(z), z >= 0, by the Chebyshev fit of
// Numerical Recipes (Press et al., 2nd ed., sec. 6.2, "erfcc"):
//   t = 1 / (1 + z/2),  erfc(z) = t * exp(-z^2 + P(t)),  P a degree-9 polynomial,
// fractional error below 1.2e-7 for every z, so the negative tail keeps full
// relative accuracy.  One exp2 and one reciprocal per element.
__device__ __forceinline__ float gelu_f(float x) {
  const float z = fabsf(x) * 0.70710678118654752440f;
  const float t = rcp_approx(fmaf(0.5f, z, 1.0f));
  float p = fmaf(t, 0.17087277f, -0.82215223f);
  p = fmaf(t, p, 1.48851587f);
  p = fmaf(t, p, -1.13520398f);
  p = fmaf(t, p, 0.27886807f);
  p = fmaf(t, p, -0.18628806f);
  p = fmaf(t, p, 0.09678418f);
  p = fmaf(t, p, 0.37409196f);
  p = fmaf(t, p, 1.00002368f);
  p = fmaf(t, p, -1.26551223f);
  const float tail = 0.5f * t * ex2_approx(fmaf(-z, z, p) * 1.44269504088896340736f);  // Phi(-|x|)
  return x * (x >= 0.f ? 1.0f - tail : tail);
}
// d/dx of the exact GELU: Phi(x) + x * phi(x).  erfc by Abramowitz & Stegun,
// Handbook of Mathematical Functions (1964), eq. 7.1.26: for z >= 0,
//   t = 1 / (1 + 0.3275911 z),  erfc(z) = t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-z^2),
// absolute error at most 1.5e-7; exp(-z^2) = exp(-x^2 / 2) is shared with phi(x).
// The result is within 1e-7 absolute of the exact derivative (within 3e-4
// relative in the far negative tail, where x * phi(x) dominates).
__device__ __forceinline__ float gelu_grad_f(float x) {
  const float e = ex2_approx(x * x * -0.72134752044448170368f);  // exp(-x^2 / 2)
  const float z = fabsf(x) * 0.70710678118654752440f;
  const float t = rcp_approx(fmaf(0.3275911f, z, 1.0f));
  float p = fmaf(t, 1.061405429f, -1.453152027f);
  p = fmaf(t, p, 1.421413741f);
  p = fmaf(t, p, -0.284496736f);
  p = fmaf(t, p, 0.254829592f);
  const float tail = 0.5f * t * p * e;  // Phi(-|x|)
  return fmaf(x, 0.39894228040143267794f * e, x >= 0.f ? 1.0f - tail : tail);
}

// The same two functions on pairs with the packed fp32 instructions (FFMA2 /
// FMUL2 / FADD2): every lane rounds exactly as the scalar fmaf / mul / add, so
// the results are bit-identical to gelu_f / gelu_grad_f with half the FMA-pipe
// instructions.
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 abs2(float2 x) { return make_float2(fabsf(x.x), fabsf(x.y)); }
__device__ __forceinline__ float2 gelu2(float2 x) {
  const float2 z = __fmul2_rn(abs2(x), f2(0.70710678118654752440f));
  const float2 den = __ffma2_rn(f2(0.5f), z, f2(1.0f));
  const float2 t = make_float2(rcp_approx(den.x), rcp_approx(den.y));
  float2 p = __ffma2_rn(t, f2(0.17087277f), f2(-0.82215223f));
  p = __ffma2_rn(t, p, f2(1.48851587f));
  p = __ffma2_rn(t, p, f2(-1.13520398f));
  p = __ffma2_rn(t, p, f2(0.27886807f));
  p = __ffma2_rn(t, p, f2(-0.18628806f));
  p = __ffma2_rn(t, p, f2(0.09678418f));
  p = __ffma2_rn(t, p, f2(0.37409196f));
  p = __ffma2_rn(t, p, f2(1.00002368f));
  p = __ffma2_rn(t, p, f2(-1.26551223f));
  const float2 arg = __fmul2_rn(__ffma2_rn(make_float2(-z.x, -z.y), z, p), f2(1.44269504088896340736f));
  const float2 e = make_float2(ex2_approx(arg.x), ex2_approx(arg.y));
  const float2 tail = __fmul2_rn(__fmul2_rn(f2(0.5f), t), e);
  const float2 one_m = __fadd2_rn(f2(1.0f), make_float2(-tail.x, -tail.y));
  return __fmul2_rn(x, make_float2(x.x >= 0.f ? one_m.x : tail.x, x.y >= 0.f ? one_m.y : tail.y));
}
// gelu_grad2, also returning GELU(x) = x * Phi(x) from the same Phi (A&S 7.1.26;
// absolute error of Phi at most 7.5e-8).
__device__ __forceinline__ float2 gelu_grad2_and_gelu(float2 x, float2& gelu) {
  const float2 xx = __fmul2_rn(__fmul2_rn(x, x), f2(-0.72134752044448170368f));
  const float2 e = make_float2(ex2_approx(xx.x), ex2_approx(xx.y));
  const float2 z = __fmul2_rn(abs2(x), f2(0.70710678118654752440f));
  const float2 den = __ffma2_rn(f2(0.3275911f), z, f2(1.0f));
  const float2 t = make_float2(rcp_approx(den.x), rcp_approx(den.y));
  float2 p = __ffma2_rn(t, f2(1.061405429f), f2(-1.453152027f));
  p = __ffma2_rn(t, p, f2(1.421413741f));
  p = __ffma2_rn(t, p, f2(-0.284496736f));
  p = __ffma2_rn(t, p, f2(0.254829592f));
  const float2 tail = __fmul2_rn(__fmul2_rn(__fmul2_rn(f2(0.5f), t), p), e);
  const float2 one_m = __fadd2_rn(f2(1.0f), make_float2(-tail.x, -tail.y));
  const float2 cdf = make_float2(x.x >= 0.f ? one_m.x : tail.x, x.y >= 0.f ? one_m.y : tail.y);
  gelu = __fmul2_rn(x, cdf);
  return __ffma2_rn(x, __fmul2_rn(f2(0.39894228040143267794f), e), cdf);
}
__device__ __forceinline__ float2 gelu_grad2(float2 x) {
  const float2 xx = __fmul2_rn(__fmul2_rn(x, x), f2(-0.72134752044448170368f));
  const float2 e = make_float2(ex2_approx(xx.x), ex2_approx(xx.y));
  const float2 z = __fmul2_rn(abs2(x), f2(0.70710678118654752440f));
  const float2 den = __ffma2_rn(f2(0.3275911f), z, f2(1.0f));
  const float2 t = make_float2(rcp_approx(den.x), rcp_approx(den.y));
  float2 p = __ffma2_rn(t, f2(1.061405429f), f2(-1.453152027f));
  p = __ffma2_rn(t, p, f2(1.421413741f));
  p = __ffma2_rn(t, p, f2(-0.284496736f));
  p = __ffma2_rn(t, p, f2(0.254829592f));
  const float2 tail = __fmul2_rn(__fmul2_rn(__fmul2_rn(f2(0.5f), t), p), e);
  const float2 one_m = __fadd2_rn(f2(1.0f), make_float2(-tail.x, -tail.y));
  const float2 cdf = make_float2(x.x >= 0.f ? one_m.x : tail.x, x.y >= 0.f ? one_m.y : tail.y);
  return __ffma2_rn(x, __fmul2_rn(f2(0.39894228040143267794f), e), cdf);
}

}  // namespace mednext
