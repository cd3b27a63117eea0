// Output error of a quantized Linear on the tcgen05 tensor cores.
//
// measure_quant_cost.py:599-605, 630-635 computes, per Linear and format,
//   y_ref = bf16(X W^T),  y_q = bf16(X_hat W_hat^T)      (bf16 bmm, fp32 accumulate)
//   output_mse = mean(bf16(y_ref - y_q)^2),  ref_energy = mean(y_ref^2)
// This kernel computes both products for one 128x128 output tile per CTA with
// tcgen05.mma (BF16 x BF16 -> FP32) into two TMEM accumulators and reduces the
// error and the energy in the epilogue, so neither y_ref nor y_q is written.
//
//  * Operand tiles (128 rows x 64 K, bf16) are staged in shared memory in the
//    canonical K-major 128-byte-swizzle layout (8-row groups of 1024 B, the
//    16-byte chunk c of row r at chunk c ^ (r % 8)), by ordinary 16-byte loads;
//  * one thread issues the MMAs (4 x K=16 per operand pair and K step) and
//    commits them to an mbarrier; every wait is bounded and a timeout sets the
//    device error word and skips the remaining MMAs;
//  * TMEM: 256 columns per CTA (reference accumulator in [0,128), quantized in
//    [128,256)), allocated and freed by warp 0 on every path; at most two CTAs
//    per SM (96 KB of shared memory each), so the 512 columns always suffice.
#include "pq_common.cuh"
#include "pq_internal.h"

namespace pq {

constexpr int OE_M = 128, OE_N = 128, OE_K = 64, OE_THREADS = 128;
constexpr uint32_t OE_TMEM_COLS = 256;
constexpr int OE_TILE_BYTES = OE_M * OE_K * 2;            // 16 KB, A and B tiles alike (M == N)
constexpr int OE_SMEM_BYTES = 96 * 1024;                  // 1 KB alignment slack + 4 tiles + barrier, padded
                                                          // so that at most 2 CTAs share an SM

// Instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A and B bf16 (bits 7-9, 10-12 = 1),
// both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t OE_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(OE_N >> 3) << 17) |
                              ((uint32_t)(OE_M >> 4) << 24);

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Shared-memory matrix descriptor of a K-major, 128-byte-swizzled tile starting at `saddr`:
// start address >> 4 (bits 0-13), leading byte offset 16 B (>> 4 = 1, bits 16-29), stride byte
// offset 1024 B between 8-row groups (>> 4, bits 32-45), version 1 (bits 46-47), swizzle 128B
// (value 2, bits 61-63).
__device__ __forceinline__ uint64_t oe_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void oe_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, bool accumulate) {
  const uint32_t acc = accumulate ? 1u : 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
      :
      : "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(OE_IDESC), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__device__ __forceinline__ void oe_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void oe_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Rows [r0, r0 + 128) x K [k0, k0 + 64) of a row-major [nrows, K] bf16 matrix into a swizzled
// tile (zeros outside the matrix).  K % 8 == 0 and 16-byte-aligned rows (host-checked).
__device__ __forceinline__ void oe_stage(uint8_t* tile, const uint16_t* __restrict__ g, int64_t nrows, int64_t K,
                                         int64_t r0, int64_t k0, int tid) {
  for (int i = tid; i < OE_M * 8; i += OE_THREADS) {
    const int r = i >> 3, c = i & 7;
    const int64_t gr = r0 + r, gk = k0 + 8 * c;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (gr < nrows && gk < K) v = __ldg(reinterpret_cast<const uint4*>(g + gr * K + gk));
    *reinterpret_cast<uint4*>(tile + (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4)) = v;
  }
}

__global__ void __launch_bounds__(OE_THREADS, 1)
    outerr_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w, const uint16_t* __restrict__ xq,
                  const uint16_t* __restrict__ wq, int64_t rows, int64_t out, int64_t K, double* err_sum,
                  double* ref_energy, float* d_ref, float* d_q) {
  // batch entry blockIdx.z: its own X/X_hat [rows, K], W/W_hat [out, K], sums and fp32 outputs
  const int64_t bz = blockIdx.z;
  x += bz * rows * K;
  xq += bz * rows * K;
  w += bz * out * K;
  wq += bz * out * K;
  if (err_sum) err_sum += bz;
  if (ref_energy) ref_energy += bz;
  if (d_ref) d_ref += bz * rows * out;
  if (d_q) d_q += bz * rows * out;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // swizzle atoms are 1024-byte aligned: round the window up (1 KB of slack is allocated)
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint8_t* sA = smem;                          // X tile
  uint8_t* sB = smem + OE_TILE_BYTES;          // W tile
  uint8_t* sAq = smem + 2 * OE_TILE_BYTES;     // X_hat tile
  uint8_t* sBq = smem + 3 * OE_TILE_BYTES;     // W_hat tile
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 4 * OE_TILE_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  volatile int* failed = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t m0 = (int64_t)blockIdx.y * OE_M, n0 = (int64_t)blockIdx.x * OE_N;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(OE_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    *failed = 0;
    fence_mbar_init();
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  uint32_t phase = 0;
  const int64_t nk = (K + OE_K - 1) / OE_K;
  for (int64_t kb = 0; kb < nk; ++kb) {
    oe_stage(sA, x, rows, K, m0, kb * OE_K, tid);
    oe_stage(sB, w, out, K, n0, kb * OE_K, tid);
    oe_stage(sAq, xq, rows, K, m0, kb * OE_K, tid);
    oe_stage(sBq, wq, out, K, n0, kb * OE_K, tid);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic-proxy writes -> tensor core reads
    __syncthreads();
    if (tid == 0 && !*failed) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
      for (int kk = 0; kk < OE_K / 16; ++kk) {   // K = 16 per MMA: +32 bytes along the swizzled row
        const bool acc = kb > 0 || kk > 0;
        oe_mma(tmem, oe_desc(smem_addr(sA) + 32 * kk), oe_desc(smem_addr(sB) + 32 * kk), acc);
        oe_mma(tmem + 128, oe_desc(smem_addr(sAq) + 32 * kk), oe_desc(smem_addr(sBq) + 32 * kk), acc);
      }
      oe_commit(bar);
    }
    // the stage is rewritten next iteration: wait for the MMAs that read it
    if (!*failed && !mbar_wait_bounded(bar, phase)) *failed = 1;
    phase ^= 1;
    __syncthreads();
    if (*failed) break;
  }
  if (*failed && tid == 0) {
    // MMAs that may still be in flight read the stage and write TMEM: wait (bounded) before freeing
    (void)mbar_wait_bounded(bar, phase ^ 1u, 1u << 22);
  }
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

  if (!*failed) {
    // warp w reads TMEM lanes (= tile rows) 32w .. 32w + 31, 16 columns at a time
    const int64_t row = m0 + 32 * warp + lane;
    float es = 0.0f, rs = 0.0f;
    double esum = 0.0, rsum = 0.0;
    for (int j = 0; j < OE_N / 16; ++j) {
      float vr[16], vq[16];
      const uint32_t lane_base = tmem + ((uint32_t)(32 * warp) << 16) + 16 * j;
      oe_ld16(lane_base, vr);
      oe_ld16(lane_base + 128, vq);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float a = bf16_round(vr[e]), b = bf16_round(vq[e]);   // bf16 bmm outputs
        const float d = bf16_round(__fsub_rn(a, b));                 // bf16 subtraction
        es = __fadd_rn(es, __fmul_rn(d, d));
        rs = __fadd_rn(rs, __fmul_rn(a, a));
        const int64_t col = n0 + 16 * j + e;
        if (row < rows && col < out) {
          if (d_ref) d_ref[row * out + col] = vr[e];
          if (d_q) d_q[row * out + col] = vq[e];
        }
      }
      if ((j & 3) == 3) {   // fp32 partials of <= 64 squares
        esum += (double)es;
        rsum += (double)rs;
        es = rs = 0.0f;
      }
    }
    esum = warp_sum_d(esum + (double)es);
    rsum = warp_sum_d(rsum + (double)rs);
    if (lane == 0) {
      if (err_sum) atomicAdd(err_sum, esum);
      if (ref_energy) atomicAdd(ref_energy, rsum);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(OE_TMEM_COLS));
  }
}

cudaError_t launch_outerr(const uint16_t* x, const uint16_t* w, const uint16_t* xq, const uint16_t* wq, int64_t batch,
                          int64_t rows, int64_t out, int64_t K, double* err_sum, double* ref_energy, float* d_ref,
                          float* d_q, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(outerr_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, OE_SMEM_BYTES);
  if (e != cudaSuccess) return e;
  const dim3 grid((unsigned)((out + OE_N - 1) / OE_N), (unsigned)((rows + OE_M - 1) / OE_M), (unsigned)batch);
  outerr_kernel<<<grid, OE_THREADS, OE_SMEM_BYTES, stream>>>(x, w, xq, wq, rows, out, K, err_sum, ref_energy, d_ref,
                                                              d_q);
  return cudaGetLastError();
}

}  // namespace pq
