// Device-side building blocks shared by the prismaquant_b200 kernels.
//
// Numerics follow the reference's torch op chains exactly (paths relative to
// the prismaquant project):
//  * all divisions are IEEE round-to-nearest (__fdiv_rn), products that feed a
//    bf16 cast are __fmul_rn (never contracted into an FMA), bf16 casts are RNE;
//  * codebook RTN reproduces `torch.bucketize` + nearest-with-ties-to-lower on
//    a sorted signed codebook (format_registry.py:217-230) and the abs-codebook
//    variant with ties toward zero (export_native_compressed.py:118-136);
//  * E8M0 exponents use per-binade thresholds captured from torch's CPU
//    float32 log2 (pq_e8m0_tables.h).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "pq_e8m0_tables.h"

namespace pq {

constexpr unsigned FULL = 0xffffffffu;

// Device error word: set by a kernel whose bounded wait gave up; read and
// cleared from the host by pq_device_error().  (The library is one
// translation unit, pq_lib.cu, so this header is compiled exactly once.)
__device__ int g_pq_device_error = 0;

enum : int { ERR_MBAR_TIMEOUT = 1 };

__device__ __forceinline__ float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

__device__ __forceinline__ uint32_t bf16_bits(float x) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
// bf16 bits of a value that is already a bf16, NaN written as 0x7FC0 (torch's float -> bf16 NaN;
// the hardware conversion writes 0x7FFF)
__device__ __forceinline__ uint32_t bf16_bits_torch(float r) { return r != r ? 0x7FC0u : __float_as_uint(r) >> 16; }

__device__ __forceinline__ void unpack8(const uint4& v, float (&w)[8]) {
  w[0] = bf16lo(v.x); w[1] = bf16hi(v.x);
  w[2] = bf16lo(v.y); w[3] = bf16hi(v.y);
  w[4] = bf16lo(v.z); w[5] = bf16hi(v.z);
  w[6] = bf16lo(v.w); w[7] = bf16hi(v.w);
}

__device__ __forceinline__ float amax8(const float (&w)[8]) {
  float a = fabsf(w[0]);
#pragma unroll
  for (int i = 1; i < 8; ++i) a = fmaxf(a, fabsf(w[i]));
  return a;
}

// 2^e as float for e in [-127, 127] (2^-127 is the subnormal 0x00400000).
__device__ __forceinline__ float pow2i(int e) {
  return e >= -126 ? __uint_as_float((uint32_t)(e + 127) << 23) : __uint_as_float(0x00400000u);
}

// Nearest point of a sign-magnitude FP grid with MBITS mantissa bits and
// minimum normal exponent EMIN, for a magnitude a >= 0, saturated at maxv.
// An exact tie rounds the magnitude up iff tie_up.
//
// Grid spacing in a's binade is 2^(max(E, EMIN) - MBITS); a / spacing is an
// exact power-of-two scaling, its fraction is exact, so the tie test is exact.
template <int MBITS, int EMIN>
__device__ __forceinline__ float grid_round_abs(float a, bool tie_up, float maxv) {
  int e = (int)(__float_as_uint(a) >> 23) - 127;
  e = max(e, EMIN);
  e = min(e, 127 + MBITS - 1);                 // keep 2^-(e-MBITS) a normal float; a >= 2^(128-MBITS) saturates anyway
  const int sh = e - MBITS;                    // spacing exponent
  const float inv = __uint_as_float((uint32_t)(127 - sh) << 23);
  const float sp = pow2i(sh);
  const float q = __fmul_rn(a, inv);
  const float n = floorf(q);
  const float f = __fsub_rn(q, n);
  const bool up = (f > 0.5f) || (f == 0.5f && tie_up);
  const float r = __fmul_rn(__fadd_rn(n, up ? 1.0f : 0.0f), sp);
  return fminf(r, maxv);                       // also maps +inf (and NaN) to maxv
}

// Cost-path RTN on the signed codebook with ties to the LOWER value
// (format_registry.py:224-230): for x < 0 the lower value has the larger magnitude.
// The codebook holds only +0.0, so a negative x that rounds to zero gives +0.0
// (0 - r, not -r).
__device__ __forceinline__ float rtn_e2m1_cost(float x) {
  const float r = grid_round_abs<1, 0>(fabsf(x), x < 0.0f, 6.0f);
  return x < 0.0f ? __fsub_rn(0.0f, r) : r;
}
__device__ __forceinline__ float rtn_e4m3_cost(float x) {
  const float r = grid_round_abs<3, -6>(fabsf(x), x < 0.0f, 448.0f);
  return x < 0.0f ? __fsub_rn(0.0f, r) : r;
}

// Export-path NVFP4 code: |x| rounded on {0,.5,1,1.5,2,3,4,6} with ties toward
// zero, index 0..7, plus bit 3 = signbit(x) (export_native_compressed.py:118-136).
__device__ __forceinline__ uint32_t nvfp4_code(float x) {
  const float r = grid_round_abs<1, 0>(fabsf(x), false, 6.0f);
  const uint32_t u = __float_as_uint(r);
  // r in {0, .5} -> 0/1; r >= 1: index = 2*(E+1) + top mantissa bit
  const uint32_t idx = r >= 1.0f ? ((((u >> 23) - 126u) << 1) | ((u >> 22) & 1u)) : (r == 0.5f ? 1u : 0u);
  return idx | ((__float_as_uint(x) >> 31) << 3);
}

// torch.round(torch.log2(s)) for a normal float s > 0, clamped to [-127, 127]
// (format_registry.py:189-190).
__device__ __forceinline__ int e8m0_round(float s) {
  const uint32_t u = __float_as_uint(s);
  const int k = (int)(u >> 23) - 127;
  const int m = (int)(u & 0x7FFFFFu);
  // the thresholds of all binades lie in [PQ_ROUND_FIRST_MIN, PQ_ROUND_FIRST_MAX]: outside that
  // window the mantissa decides alone, and the per-lane indexed table read (which serializes
  // over the distinct binades of a warp) is skipped
  int e = m >= PQ_ROUND_FIRST_MAX ? k + 1 : k;
  if (m >= PQ_ROUND_FIRST_MIN && m < PQ_ROUND_FIRST_MAX) e = m >= PQ_ROUND_FIRST[k + 126] ? k + 1 : k;
  return max(-127, min(127, e));
}

// torch.ceil(torch.log2(s)).clamp(-127, 127) for s > 0 (possibly subnormal)
// (export_native_compressed.py:1153-1154).
__device__ __forceinline__ int e8m0_ceil(float s) {
  const uint32_t u = __float_as_uint(s);
  const int be = (int)(u >> 23);
  const int m = (int)(u & 0x7FFFFFu);
  if (be > 0) {
    const int k = be - 127;
    if (m <= PQ_CEIL_LAST_MIN) return k;                      // as e8m0_round: the table only
    if (m > PQ_CEIL_LAST_MAX) return min(127, k + 1);         // inside the thresholds' window
    return min(127, m <= PQ_CEIL_LAST[k + 127] ? k : k + 1);
  }
  if (m >= (1 << 22)) return (m - (1 << 22)) <= PQ_CEIL_LAST[0] ? -127 : -126;
  return -127;
}

// float -> float8_e4m3fn byte, round-to-nearest-even (torch `.to(float8_e4m3fn)`
// on values already clamped to +-448).
__device__ __forceinline__ uint32_t e4m3_byte(float x) {
  return (uint32_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  return (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3);
}

// ---------------------------------------------------------------------------
// Shared-memory staging: 1-D bulk async copies (TMA engine) + mbarriers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Global -> shared bulk copy; src/dst 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
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

// Bounded wait: gives up after `limit` polls (each poll is itself a
// hardware-suspended try_wait), records the error and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t limit = (1u << 24)) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  atomicExch(&g_pq_device_error, ERR_MBAR_TIMEOUT);
  return false;
}

// Iteration limit of the sweep kernels' stage waits (the waits for a work item's bulk copy).
// pq_set_wait_limit changes it so that a test can make those waits run out on purpose: the
// kernel then records ERR_MBAR_TIMEOUT, waits (with the fixed limit) for the copies it has
// issued, and returns, leaving the context usable.
constexpr uint32_t DEFAULT_WAIT_LIMIT = 1u << 24;
__device__ uint32_t g_pq_wait_limit = DEFAULT_WAIT_LIMIT;

__device__ __forceinline__ bool mbar_wait_stage(uint64_t* bar, uint32_t parity) {
  return mbar_wait_bounded(bar, parity, *(volatile uint32_t*)&g_pq_wait_limit);
}

// ---------------------------------------------------------------------------
// Reductions
// ---------------------------------------------------------------------------
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}
__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}
__device__ __forceinline__ uint32_t warp_max_u(uint32_t v) { return __reduce_max_sync(FULL, v); }

}  // namespace pq
