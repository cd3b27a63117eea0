// Output error of a quantized Linear on the tcgen05 tensor cores.
//
// measure_quant_cost.py:599-605, 630-635 computes, per chunk of same-shape Linears,
//   y_ref = bf16(X W^T)  once,  and per format  y_q = bf16(X_hat W_hat^T)
//   output_mse = mean(bf16(y_ref - y_q)^2),  ref_energy = mean(y_ref^2)
// with bf16 bmm's (fp32 accumulate).  Three kernel modes cover it:
//   OE_REF   X W^T          -> writes bf16 y_ref (optional), adds sum(y_ref^2)
//   OE_ERR   X_hat W_hat^T  -> reads bf16 y_ref, adds sum(bf16(y_ref - y_q)^2)
//   OE_DUAL  both products in one pass (two accumulators), adds both sums; y_ref never stored
//
// One CTA computes a 128 x BN output tile (BN = 256 for one product, 128 per product in
// OE_DUAL) of one batch entry:
//  * TMA (3-D tensor maps [batch, rows, k], 128-byte swizzle, zero fill past the edges) loads
//    64-wide K slices of the operands into an NSTAGE ring of shared-memory stages, in the
//    canonical K-major SW128 layout the MMA descriptors name;
//  * thread 0 produces (waits for a free stage, arms its full barrier, issues the loads);
//    thread 32 issues the MMAs (4 x K=16 per stage and product) and commits each stage back to
//    its empty barrier, then the whole tile to the accumulator barrier;
//  * all four warps then read the fp32 accumulators from TMEM (warp w owns lanes 32w..32w+31,
//    i.e. tile rows) and reduce the bf16 error / energy; sums go to fp64 atomics.
// Every wait is bounded: a timeout sets the device error word and the abort flag, the roles
// stop issuing, outstanding loads and MMAs are waited for (bounded) and TMEM is freed.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "pq_common.cuh"
#include "pq_internal.h"

namespace pq {

enum { OE_REF = 0, OE_ERR = 1, OE_DUAL = 2 };
constexpr int OE_BM = 128, OE_BK = 64, OE_THREADS = 128;
constexpr uint32_t OE_TMEM_COLS = 256;

template <int MODE, bool PAIR>
struct OeCfg {
  static constexpr bool DUAL = MODE == OE_DUAL;
  static_assert(!(DUAL && PAIR), "the dual-product mode runs on single CTAs");
  static constexpr int BN = DUAL ? 128 : 256;               // output columns per product
  static constexpr int MMA_M = PAIR ? 2 * OE_BM : OE_BM;    // rows of one MMA (a CTA pair: 256)
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;         // rows of the B tile this CTA holds
  static constexpr int A_BYTES = OE_BM * OE_BK * 2;         // 16 KB
  static constexpr int B_BYTES = B_ROWS * OE_BK * 2;        // 16 / 32 KB
  static constexpr int PAIR_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGE_BYTES = (DUAL ? 2 : 1) * PAIR_BYTES;   // 64 / 48 / 32 KB
  static constexpr int NSTAGE = DUAL ? 3 : (PAIR ? 6 : 4);
  static constexpr int SMEM = 1024 + NSTAGE * STAGE_BYTES + 256;    // align slack, stages, barriers
  // kind::f16 instruction descriptor: D f32 (bits 4-5 = 1), A and B bf16 (bits 7-9, 10-12 = 1),
  // both K-major (bits 15, 16 = 0), N >> 3 at bit 17, M >> 4 at bit 24.
  static constexpr uint32_t IDESC =
      (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(MMA_M >> 4) << 24);
};

// Stage ring of one launch: CTA pairs without K splits keep 3 stages (98 KB), so two CTAs share
// an SM and one's prologue and epilogue overlap the other's main loop; K-split launches keep 6
// (their fp32 partial tile, 128 KB, is staged in the ring) and so run one CTA per SM.
template <int MODE, bool PAIR, int S>
struct OeRing {
  using C = OeCfg<MODE, PAIR>;
  static constexpr int NSTAGE = (PAIR && S == 1) ? 3 : C::NSTAGE;
  static constexpr int SMEM = 1024 + NSTAGE * C::STAGE_BYTES + 256;
};

struct OeArgs {
  int64_t rows, out, k;
  double* err_sum;      // [batch] (ERR, DUAL)
  double* ref_sum;      // [batch] (REF, DUAL)
  uint16_t* y_ref;      // bf16 [batch, rows, out]: REF writes it (may be null), ERR reads it
  float* d_ref;         // DUAL: fp32 accumulators (may be null)
  float* d_q;
};

// Shared-memory matrix descriptor of a K-major, 128-byte-swizzled tile starting at `saddr`
// (1024-byte aligned atoms): start >> 4 (bits 0-13), leading byte offset 16 B (>> 4 = 1, bits
// 16-29), stride byte offset 1024 B between 8-row groups (>> 4, bits 32-45), version 1 (bits
// 46-47), layout SWIZZLE_128B (2, bits 61-63).  Advancing K by 16 bf16 adds 32 bytes to start.
__device__ __forceinline__ uint64_t oe_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void oe_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
      :
      : "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

// arrives on `bar` once every tcgen05 operation this thread issued before it has completed
__device__ __forceinline__ void oe_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---- CTA-pair forms (cta_group::2: one MMA of M = 256 over two SMs; each CTA holds its 128 rows
// of A, half of the B tile's rows, and its 128 rows of the accumulator in its own TMEM) ----
__device__ __forceinline__ void oe_mma_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n\t}\n"
      :
      : "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u),
        "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

// arrives on the barrier at `bar`'s offset in both CTAs of the pair once the MMAs issued so far
// have completed
__device__ __forceinline__ void oe_commit_pair(uint64_t* bar, uint16_t pair_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(pair_mask)
      : "memory");
}

__device__ __forceinline__ float4 oe_ld_dsmem_f4(uint32_t cluster_addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(cluster_addr)
               : "memory");
  return v;
}

// tile load into this CTA's shared memory whose completion is counted on the barrier at cluster
// address `bar_cluster` (the leader CTA's)
__device__ __forceinline__ void oe_tma_3d_pair(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                               uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
      "%4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar_cluster)
      : "memory");
}

__device__ __forceinline__ uint32_t oe_cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the variable at `saddr` (a shared::cta address) in CTA `rank`
__device__ __forceinline__ uint32_t oe_mapa(uint32_t saddr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
  return d;
}

__device__ __forceinline__ void oe_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void oe_tma_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
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

// 16 bf16 values of y_ref at [row, col0 .. col0+15] (zeros past `out`), as floats
__device__ __forceinline__ void oe_load_yref(const uint16_t* __restrict__ y, int64_t row_off, int64_t col0,
                                             int64_t out, bool vec, float (&a)[16]) {
  if (vec) {
    const uint4 u0 = __ldcs(reinterpret_cast<const uint4*>(y + row_off + col0));
    const uint4 u1 = __ldcs(reinterpret_cast<const uint4*>(y + row_off + col0 + 8));
    const uint32_t u[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      a[2 * i] = __uint_as_float(u[i] << 16);
      a[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      a[i] = col0 + i < out ? __uint_as_float((uint32_t)y[row_off + col0 + i] << 16) : 0.0f;
  }
}

// 16 values already rounded to bf16 (low 16 bits zero) into y_ref[row, col0 ..]
__device__ __forceinline__ void oe_store_yref(uint16_t* __restrict__ y, int64_t row_off, int64_t col0, int64_t out,
                                              bool vec, const float (&a)[16]) {
  if (vec) {
    uint32_t u[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) u[i] = (__float_as_uint(a[2 * i]) >> 16) | (__float_as_uint(a[2 * i + 1]) & 0xFFFF0000u);
    *reinterpret_cast<uint4*>(y + row_off + col0) = make_uint4(u[0], u[1], u[2], u[3]);
    *reinterpret_cast<uint4*>(y + row_off + col0 + 8) = make_uint4(u[4], u[5], u[6], u[7]);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (col0 + i < out) y[row_off + col0 + i] = (uint16_t)(__float_as_uint(a[i]) >> 16);
  }
}

// Bounded wait that also gives up as soon as another role has set the abort flag; a timeout
// records the device error (as mbar_wait_bounded does).
__device__ __forceinline__ bool oe_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  for (uint32_t i = 0; i < (1u << 24); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && *abort_flag) return false;
  }
  atomicExch(&g_pq_device_error, ERR_MBAR_TIMEOUT);
  return false;
}

// Epilogue arithmetic of one output value: `v` the fp32 accumulator, `a` the bf16 y_ref (ERR).
template <int MODE>
__device__ __forceinline__ float oe_value(float v, float a, float& es, float& rs) {
  if (MODE == OE_REF) {
    const float r = bf16_round(v);
    rs = __fadd_rn(rs, __fmul_rn(r, r));
    return r;
  }
  const float d = bf16_round(__fsub_rn(a, bf16_round(v)));   // bf16 y_ref - bf16 y_q
  es = __fadd_rn(es, __fmul_rn(d, d));
  return d;
}

// Grid: x = CTA (pairs of x for PAIR), y = output-column tile x S K-splits, z = batch entry.
// Cluster (PAIR ? 2 : 1, S, 1): cluster rank = pair rank + 2 * split.  With S > 1 each split runs
// its share of the K stages, stages its fp32 partial from TMEM in its own shared memory, and after
// a cluster barrier split t sums column slice t of the tile over all S partials (distributed
// shared memory, fixed order) and runs the epilogue on that slice.
template <int MODE, bool PAIR, int S>
__global__ void __launch_bounds__(OE_THREADS, 1)
    outerr_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                  const __grid_constant__ CUtensorMap taq, const __grid_constant__ CUtensorMap tbq, OeArgs p) {
  using C = OeCfg<MODE, PAIR>;
  constexpr int NSTAGE = OeRing<MODE, PAIR, S>::NSTAGE;
  static_assert(S == 1 || (PAIR && (S == 2 || S == 4)), "K splits run on CTA pairs, 2 or 4 of them");
  constexpr int SLICE = C::BN / S;               // epilogue columns per split
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);   // 1024-aligned atoms
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NSTAGE * C::STAGE_BYTES);
  uint64_t* empty = full + NSTAGE;
  uint64_t* acc_full = empty + NSTAGE;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* consumed = abort_flag + 1;   // stages the MMA thread has waited for

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bz = blockIdx.z;
  // PAIR: the two CTAs of a pair share one 256 x BN tile: pair rank r holds rows 128r.. of it and
  // B rows BN/2 * r ..; the pair's leader (even cluster rank) issues the MMAs.  M is the fastest
  // grid dimension, so the CTAs that read one W tile run together.
  const uint32_t crank = (PAIR || S > 1) ? oe_cluster_rank() : 0u;
  const uint32_t prank = PAIR ? (crank & 1u) : 0u;
  const uint32_t leader = crank & ~1u;
  const int split = (int)(blockIdx.y % S);
  const int m0 = PAIR ? (int)(blockIdx.x >> 1) * (2 * OE_BM) + (int)prank * OE_BM : (int)blockIdx.x * OE_BM;
  const int n0 = (int)(blockIdx.y / S) * C::BN;
  const int nb0 = n0 + (int)prank * C::B_ROWS;
  const int nk_all = (int)((p.k + OE_BK - 1) / OE_BK);
  const int kb0 = split * nk_all / S;
  const int nk = (split + 1) * nk_all / S - kb0;   // >= 1: the host keeps S <= nk_all

  if (warp == 0) {
    if (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(OE_TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(OE_TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  if (tid == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    *consumed = 0;
    fence_mbar_init();
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  if (PAIR || S > 1)
    oe_cluster_sync();   // every CTA's barriers exist before another signals them
  else
    __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const uint32_t peer_abort = PAIR ? oe_mapa(smem_u32((const void*)abort_flag), crank ^ 1u) : 0u;
  auto set_abort = [&]() {
    *abort_flag = 1;
    if (PAIR) asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer_abort), "r"(1u) : "memory");
  };

  // ERR: this thread's row of its epilogue columns of y_ref (SLICE bf16 = SLICE/8 x 16 B) is
  // fetched into registers now, so that the loads overlap the main loop instead of the epilogue
  const int64_t my_row = (int64_t)m0 + 32 * warp + lane;
  const bool row_ok = my_row < p.rows;
  const int64_t my_row_off = ((int64_t)bz * p.rows + my_row) * p.out;
  const int c0 = n0 + split * SLICE;               // first epilogue column
  const bool full_row = row_ok && (int64_t)c0 + SLICE <= p.out && (p.out & 7) == 0;
  uint4 ya[MODE == OE_ERR ? SLICE / 8 : 1];
  if (MODE == OE_ERR && full_row) {
    const uint4* src = reinterpret_cast<const uint4*>(p.y_ref + my_row_off + c0);
#pragma unroll
    for (int i = 0; i < SLICE / 8; ++i) ya[i] = __ldcs(src + i);
  }

  int produced = 0;
  if (tid == 0) {
    // ---- producer (each CTA loads its own operand rows) ----
    const uint32_t leader_full0 = PAIR ? oe_mapa(smem_u32(&full[0]), leader) : 0u;
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % NSTAGE, use = kb / NSTAGE;
      const int kc = (kb0 + kb) * OE_BK;
      if (use > 0 && !oe_wait(&empty[s], (uint32_t)((use - 1) & 1), abort_flag)) {
        set_abort();
        break;
      }
      if (*abort_flag) break;
      uint8_t* st = smem + s * C::STAGE_BYTES;
      if (PAIR) {
        // the leader's full barrier counts the bytes of both CTAs' loads
        if (prank == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(2 * C::STAGE_BYTES));
        const uint32_t fb = leader_full0 + 8u * (uint32_t)s;
        oe_tma_3d_pair(st, &ta, kc, m0, bz, fb);
        oe_tma_3d_pair(st + C::A_BYTES, &tb, kc, nb0, bz, fb);
      } else {
        mbar_arrive_expect_tx(&full[s], (uint32_t)C::STAGE_BYTES);
        oe_tma_3d(st, &ta, kc, m0, bz, &full[s]);
        oe_tma_3d(st + C::A_BYTES, &tb, kc, n0, bz, &full[s]);
        if (C::DUAL) {
          oe_tma_3d(st + C::PAIR_BYTES, &taq, kc, m0, bz, &full[s]);
          oe_tma_3d(st + C::PAIR_BYTES + C::A_BYTES, &tbq, kc, n0, bz, &full[s]);
        }
      }
      produced = kb + 1;
    }
  } else if (tid == 32 && prank == 0) {
    // ---- MMA issuer (the pair leader's) ----
    const uint16_t pair_mask = (uint16_t)(3u << leader);
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % NSTAGE, use = kb / NSTAGE;
      if (!oe_wait(&full[s], (uint32_t)(use & 1), abort_flag)) {
        set_abort();
        break;
      }
      *consumed = kb + 1;
      if (*abort_flag) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
#pragma unroll
      for (int kk = 0; kk < OE_BK / 16; ++kk) {
        const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
        if (PAIR) {
          oe_mma_pair(tmem, oe_desc(sa + 32 * kk), oe_desc(sa + C::A_BYTES + 32 * kk), C::IDESC, acc);
        } else {
          oe_mma(tmem, oe_desc(sa + 32 * kk), oe_desc(sa + C::A_BYTES + 32 * kk), C::IDESC, acc);
          if (C::DUAL)
            oe_mma(tmem + 128, oe_desc(sa + C::PAIR_BYTES + 32 * kk),
                   oe_desc(sa + C::PAIR_BYTES + C::A_BYTES + 32 * kk), C::IDESC, acc);
        }
      }
      // the stage is free (in both CTAs of a pair) once these MMAs have read it
      if (PAIR)
        oe_commit_pair(&empty[s], pair_mask);
      else
        oe_commit(&empty[s]);
    }
    // also the drain: arrives after every MMA issued above
    if (PAIR)
      oe_commit_pair(acc_full, pair_mask);
    else
      oe_commit(acc_full);
  }
  __syncwarp();

  // ---- epilogue: all four warps of each CTA, on its own TMEM rows ----
  if (!mbar_wait_bounded(acc_full, 0)) *abort_flag = 1;
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  __syncthreads();   // every thread sees the same abort flag
  const uint32_t tbase = tmem + ((uint32_t)(32 * warp) << 16);
  const int trow = 32 * warp + lane;               // row within the CTA's 128
  float es = 0.0f, rs = 0.0f;
  double esum = 0.0, rsum = 0.0;
  if (S > 1) {
    // stage this split's fp32 partial (128 rows x BN) into the now idle stage ring: row r at
    // r * 4 * BN bytes, 16-byte chunk c at chunk c ^ (r % 8) (conflict-free for thread = row)
    static_assert(S == 1 || OE_BM * C::BN * 4 <= NSTAGE * C::STAGE_BYTES, "partial tile fits the stage ring");
    if (!*abort_flag) {
      float* prow = reinterpret_cast<float*>(smem + (size_t)trow * 4 * C::BN);
#pragma unroll 1
      for (int j = 0; j < C::BN / 16; ++j) {
        float v[16];
        oe_ld16(tbase + 16 * j, v);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int c = 4 * j + q;
          *reinterpret_cast<float4*>(prow + 4 * (c ^ (trow & 7))) =
              make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
      }
    }
    // every TMEM read of this CTA is done and every partial staged before any partner reads
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    oe_cluster_sync();
    int any_abort = *abort_flag;
    if (!any_abort) {
      uint32_t part[S];
#pragma unroll
      for (int t = 0; t < S; ++t) part[t] = oe_mapa(smem_u32(smem + (size_t)trow * 4 * C::BN), prank + 2u * t);
      constexpr int NCH = SLICE / 4;               // 4-column chunks of this split's slice
      constexpr int CB = 4;                        // chunks whose S partials are loaded at once
      static_assert(NCH % CB == 0, "slice is a whole number of load batches");
#pragma unroll
      for (int cb = 0; cb < NCH; cb += CB) {
        float4 pv[CB][S];
#pragma unroll
        for (int q = 0; q < CB; ++q) {
          const uint32_t off = 16u * (uint32_t)((split * NCH + cb + q) ^ (trow & 7));
#pragma unroll
          for (int t = 0; t < S; ++t) pv[q][t] = oe_ld_dsmem_f4(part[t] + off);
        }
#pragma unroll
        for (int q = 0; q < CB; ++q) {
        const int cl = cb + q;
        float4 acc = pv[q][0];
#pragma unroll
        for (int t = 1; t < S; ++t) {   // fixed order: split 0, 1, ..
          acc.x = __fadd_rn(acc.x, pv[q][t].x);
          acc.y = __fadd_rn(acc.y, pv[q][t].y);
          acc.z = __fadd_rn(acc.z, pv[q][t].z);
          acc.w = __fadd_rn(acc.w, pv[q][t].w);
        }
        const float v4[4] = {acc.x, acc.y, acc.z, acc.w};
        const int64_t col0 = (int64_t)c0 + 4 * cl;
        float a4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (MODE == OE_ERR) {
          if (full_row) {
            const uint4 u = ya[cl >> 1];
            const uint32_t lo = (cl & 1) ? u.z : u.x, hi = (cl & 1) ? u.w : u.y;
            a4[0] = __uint_as_float(lo << 16);
            a4[1] = __uint_as_float(lo & 0xFFFF0000u);
            a4[2] = __uint_as_float(hi << 16);
            a4[3] = __uint_as_float(hi & 0xFFFF0000u);
          } else if (row_ok) {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              a4[e] = col0 + e < p.out ? __uint_as_float((uint32_t)p.y_ref[my_row_off + col0 + e] << 16) : 0.0f;
          }
        }
        float r4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) r4[e] = oe_value<MODE>(v4[e], a4[e], es, rs);
        if (MODE == OE_REF && p.y_ref && row_ok) {
          if (full_row) {
            const uint32_t lo = (__float_as_uint(r4[0]) >> 16) | (__float_as_uint(r4[1]) & 0xFFFF0000u);
            const uint32_t hi = (__float_as_uint(r4[2]) >> 16) | (__float_as_uint(r4[3]) & 0xFFFF0000u);
            *reinterpret_cast<uint2*>(p.y_ref + my_row_off + col0) = make_uint2(lo, hi);
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (col0 + e < p.out) p.y_ref[my_row_off + col0 + e] = (uint16_t)(__float_as_uint(r4[e]) >> 16);
          }
        }
        if ((cl & 15) == 15) {   // fp32 partials of <= 64 squares
          esum += (double)es;
          rsum += (double)rs;
          es = rs = 0.0f;
        }
        }
      }
    }
  } else if (!*abort_flag) {
    const int64_t row_off = my_row_off;
#pragma unroll
    for (int j = 0; j < C::BN / 16; ++j) {
      const int64_t col0 = (int64_t)n0 + 16 * j;
      const bool vec = row_ok && col0 + 16 <= p.out && (p.out & 7) == 0;
      float v[16];
      oe_ld16(tbase + 16 * j, v);
      if (MODE == OE_REF) {
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = oe_value<OE_REF>(v[e], 0.0f, es, rs);
        if (p.y_ref && row_ok) oe_store_yref(p.y_ref, row_off, col0, p.out, vec, v);
      } else if (MODE == OE_ERR) {
        float a[16];
        if (full_row) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 u = ya[2 * j + (i >> 1)];
            const uint32_t lo = (i & 1) ? u.z : u.x, hi = (i & 1) ? u.w : u.y;
            a[4 * i] = __uint_as_float(lo << 16);
            a[4 * i + 1] = __uint_as_float(lo & 0xFFFF0000u);
            a[4 * i + 2] = __uint_as_float(hi << 16);
            a[4 * i + 3] = __uint_as_float(hi & 0xFFFF0000u);
          }
        } else if (row_ok) {
          oe_load_yref(p.y_ref, row_off, col0, p.out, vec, a);
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) a[e] = 0.0f;
        }
#pragma unroll
        for (int e = 0; e < 16; ++e) (void)oe_value<OE_ERR>(v[e], a[e], es, rs);
      } else {
        float q[16];
        oe_ld16(tbase + 128 + 16 * j, q);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float a = bf16_round(v[e]);
          const float d = bf16_round(__fsub_rn(a, bf16_round(q[e])));
          es = __fadd_rn(es, __fmul_rn(d, d));
          rs = __fadd_rn(rs, __fmul_rn(a, a));
        }
        if (row_ok && (p.d_ref || p.d_q)) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            if (col0 + e < p.out) {
              if (p.d_ref) p.d_ref[row_off + col0 + e] = v[e];
              if (p.d_q) p.d_q[row_off + col0 + e] = q[e];
            }
          }
        }
      }
      if ((j & 3) == 3) {   // fp32 partials of <= 64 squares
        esum += (double)es;
        rsum += (double)rs;
        es = rs = 0.0f;
      }
    }
  }
  if (!*abort_flag) {
    esum = warp_sum_d(esum + (double)es);
    rsum = warp_sum_d(rsum + (double)rs);
    if (lane == 0) {
      if (MODE != OE_REF && p.err_sum) atomicAdd(p.err_sum + bz, esum);
      if (MODE != OE_ERR && p.ref_sum) atomicAdd(p.ref_sum + bz, rsum);
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (tid == 0 && prank == 0 && *abort_flag) {
    // loads armed but never waited for by the MMA thread still write shared memory (in a pair,
    // the leader's full barrier also counts the other CTA's loads of the same stage)
    for (int j = *consumed; j < produced; ++j)
      (void)mbar_wait_bounded(&full[j % NSTAGE], (uint32_t)((j / NSTAGE) & 1), 1u << 20);
  }
  if (PAIR || S > 1)
    oe_cluster_sync();   // no CTA frees the pair's TMEM or exits while a partner still reads it
  else
    __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(OE_TMEM_COLS));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(OE_TMEM_COLS));
  }
}

// ---------------------------------------------------------------------------
// Host side: tensor maps and launches
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 oe_encode_fn() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {   // thread-safe one-time initialisation
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
  }();
  return fn;
}

// bf16 [batch, rows, k] (k % 8 == 0, 16-byte aligned base), box 64 (k) x box_rows x 1, SW128
static bool oe_tmap(CUtensorMap* m, const uint16_t* base, int64_t batch, int64_t rows, int64_t k, uint32_t box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = oe_encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)k, (cuuint64_t)rows, (cuuint64_t)batch};
  const cuuint64_t strides[2] = {(cuuint64_t)k * 2, (cuuint64_t)rows * (cuuint64_t)k * 2};
  const cuuint32_t box[3] = {(cuuint32_t)OE_BK, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<uint16_t*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int MODE, bool PAIR, int S>
static cudaError_t oe_launch_s(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& taq,
                               const CUtensorMap& tbq, int64_t batch, int64_t mtiles, const OeArgs& args,
                               cudaStream_t stream) {
  using C = OeCfg<MODE, PAIR>;
  cudaError_t e =
      cudaFuncSetAttribute(outerr_kernel<MODE, PAIR, S>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           OeRing<MODE, PAIR, S>::SMEM);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)mtiles, (unsigned)(((args.out + C::BN - 1) / C::BN) * S), (unsigned)batch);
  cfg.blockDim = dim3(OE_THREADS, 1, 1);
  cfg.dynamicSmemBytes = OeRing<MODE, PAIR, S>::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = PAIR ? 2 : 1;
  attr[0].val.clusterDim.y = S;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, outerr_kernel<MODE, PAIR, S>, ta, tb, taq, tbq, args);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

// Clusters of outerr_kernel<MODE, true, S> (2 x S CTAs) the device holds at once (cached).
template <int MODE, int S>
static int oe_max_clusters() {
  static const int cached = [] {   // thread-safe one-time initialisation (one device model per process)
    int n = 0;
    if (cudaFuncSetAttribute(outerr_kernel<MODE, true, S>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             OeRing<MODE, true, S>::SMEM) ==
        cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2, S, 1);
      cfg.blockDim = dim3(OE_THREADS, 1, 1);
      cfg.dynamicSmemBytes = OeRing<MODE, true, S>::SMEM;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = S;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, outerr_kernel<MODE, true, S>, &cfg) != cudaSuccess) n = 0;
    }
    (void)cudaGetLastError();
    return n;
  }();
  return cached;
}

// K splits for a launch of `units` CTA pairs (one cluster each) over nk 64-wide K stages: the
// largest of 4, 2 that still fits every cluster on the device at once and gives every SM at most
// about one CTA, with at least two stages per split; 1 when the tiles alone fill the device.
template <int MODE>
static int oe_splits(int64_t units, int64_t nk) {
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t room = sms + sms / 8;
  if (nk >= 8 && 8 * units <= room && units <= oe_max_clusters<MODE, 4>()) return 4;
  if (nk >= 4 && 4 * units <= room && units <= oe_max_clusters<MODE, 2>()) return 2;
  return 1;
}

template <int MODE, bool PAIR>
static cudaError_t oe_launch(const uint16_t* a, const uint16_t* b, const uint16_t* aq, const uint16_t* bq,
                             int64_t batch, const OeArgs& args, cudaStream_t stream) {
  using C = OeCfg<MODE, PAIR>;
  CUtensorMap ta, tb, taq, tbq;
  if (!oe_tmap(&ta, a, batch, args.rows, args.k, OE_BM) || !oe_tmap(&tb, b, batch, args.out, args.k, C::B_ROWS))
    return cudaErrorInvalidValue;
  taq = ta;
  tbq = tb;
  if (C::DUAL && (!oe_tmap(&taq, aq, batch, args.rows, args.k, OE_BM) ||
                  !oe_tmap(&tbq, bq, batch, args.out, args.k, C::B_ROWS)))
    return cudaErrorInvalidValue;
  const int64_t mtiles = PAIR ? 2 * ((args.rows + 2 * OE_BM - 1) / (2 * OE_BM)) : (args.rows + OE_BM - 1) / OE_BM;
  if constexpr (!PAIR) {
    return oe_launch_s<MODE, false, 1>(ta, tb, taq, tbq, batch, mtiles, args, stream);
  } else {
    const int64_t units = (mtiles / 2) * ((args.out + C::BN - 1) / C::BN) * batch;
    switch (oe_splits<MODE>(units, (args.k + OE_BK - 1) / OE_BK)) {
      case 4: return oe_launch_s<MODE, true, 4>(ta, tb, taq, tbq, batch, mtiles, args, stream);
      case 2: return oe_launch_s<MODE, true, 2>(ta, tb, taq, tbq, batch, mtiles, args, stream);
      default: return oe_launch_s<MODE, true, 1>(ta, tb, taq, tbq, batch, mtiles, args, stream);
    }
  }
}

// ---------------------------------------------------------------------------
// Per-weight Fisher diagonal (sensitivity_probe.py:1114-1152): for one backward of one Linear,
//   grad_w = bf16(gy^T x)  (gy [T, M] output gradients, x [T, N] inputs, K = T tokens)
//   g2 = bf16(grad_w^2);  h[M, N] += g2 (fp32);  sums[0] += sum(g2);  sums[1] += sum(bf16(g2 * bf16(w^2)))
// on CTA pairs: both operands are M/N-contiguous, so they are loaded as they lie (64 x 64 TMA
// boxes, 128-byte swizzle) and described to the MMA as MN-major tiles; the epilogue reads the
// accumulators from TMEM and updates h in place (each h tile belongs to one CTA).
// ---------------------------------------------------------------------------
constexpr int GS_NSTAGE = 3;                          // 32 KB stages, two CTAs per SM
constexpr int GS_STAGE_BYTES = 2 * 16384;             // A (128 M x 64 K) + B (128 N x 64 K) per CTA
constexpr int GS_SMEM = 1024 + GS_NSTAGE * GS_STAGE_BYTES + 256;
// kind::f16: D f32, A and B bf16, both MN-major (bits 15, 16 = 1), N = 256, M = 256 (pair)
constexpr uint32_t GS_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (1u << 16) |
                              ((uint32_t)(256 >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);

struct GsArgs {
  int64_t m, n, t;      // grad_w is [m, n]; t tokens
  float* h;             // [m, n] fp32, updated in place
  const uint16_t* w;    // [m, n] bf16 weight (may be null: no w^2 sum)
  double* sums;         // [2]
};

// Shared-memory descriptor of an MN-major, 128-byte-swizzled tile: atoms of 8 K-rows x 128 bytes
// (64 M/N elements); the next 64 M/N elements 8192 bytes on (leading byte offset, >> 4 = 512), the
// next 8 K-rows 1024 bytes on (stride byte offset, >> 4 = 64); version 1, SWIZZLE_128B.
__device__ __forceinline__ uint64_t gs_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(8192 >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void gs_tma_2d_pair(void* dst, const CUtensorMap* map, int c0, int c1, uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar_cluster)
      : "memory");
}

__global__ void __launch_bounds__(OE_THREADS, 1)
    gradsq_kernel(const __grid_constant__ CUtensorMap tg, const __grid_constant__ CUtensorMap tx, GsArgs p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + GS_NSTAGE * GS_STAGE_BYTES);
  uint64_t* empty = full + GS_NSTAGE;
  uint64_t* acc_full = empty + GS_NSTAGE;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* consumed = abort_flag + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t crank = oe_cluster_rank();
  const uint32_t prank = crank & 1u;
  const uint32_t leader = crank & ~1u;
  const int m0 = (int)(blockIdx.x >> 1) * 256 + (int)prank * 128;   // this CTA's 128 rows of grad_w
  const int n0 = (int)blockIdx.y * 256;                              // the tile's 256 columns
  const int nb0 = n0 + (int)prank * 128;                             // this CTA's half of B
  const int nk = (int)((p.t + OE_BK - 1) / OE_BK);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(OE_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  if (tid == 0) {
    for (int s = 0; s < GS_NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    *consumed = 0;
    fence_mbar_init();
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  oe_cluster_sync();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const uint32_t peer_abort = oe_mapa(smem_u32((const void*)abort_flag), crank ^ 1u);
  auto set_abort = [&]() {
    *abort_flag = 1;
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer_abort), "r"(1u) : "memory");
  };

  int produced = 0;
  if (tid == 0) {
    // ---- producer: this CTA's A (gy, 128 rows of M) and half of B (x, 128 of N), 64 tokens a stage
    const uint32_t leader_full0 = oe_mapa(smem_u32(&full[0]), leader);
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % GS_NSTAGE, use = kb / GS_NSTAGE;
      if (use > 0 && !oe_wait(&empty[s], (uint32_t)((use - 1) & 1), abort_flag)) {
        set_abort();
        break;
      }
      if (*abort_flag) break;
      uint8_t* st = smem + s * GS_STAGE_BYTES;
      if (prank == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(2 * GS_STAGE_BYTES));
      const uint32_t fb = leader_full0 + 8u * (uint32_t)s;
      const int t0 = kb * OE_BK;
      gs_tma_2d_pair(st, &tg, m0, t0, fb);
      gs_tma_2d_pair(st + 8192, &tg, m0 + 64, t0, fb);
      gs_tma_2d_pair(st + 16384, &tx, nb0, t0, fb);
      gs_tma_2d_pair(st + 16384 + 8192, &tx, nb0 + 64, t0, fb);
      produced = kb + 1;
    }
  } else if (tid == 32 && prank == 0) {
    // ---- MMA issuer (the pair leader's): K = 16 tokens per MMA = two 8-row groups = 2048 bytes
    const uint16_t pair_mask = (uint16_t)(3u << leader);
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % GS_NSTAGE, use = kb / GS_NSTAGE;
      if (!oe_wait(&full[s], (uint32_t)(use & 1), abort_flag)) {
        set_abort();
        break;
      }
      *consumed = kb + 1;
      if (*abort_flag) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t sa = smem_u32(smem + s * GS_STAGE_BYTES);
#pragma unroll
      for (int kk = 0; kk < OE_BK / 16; ++kk)
        oe_mma_pair(tmem, gs_desc(sa + 2048 * kk), gs_desc(sa + 16384 + 2048 * kk), GS_IDESC,
                    (kb > 0 || kk > 0) ? 1u : 0u);
      oe_commit_pair(&empty[s], pair_mask);
    }
    oe_commit_pair(acc_full, pair_mask);
  }
  __syncwarp();

  // ---- epilogue: row m of grad_w per thread (TMEM lane), 256 columns, h updated in place
  if (!mbar_wait_bounded(acc_full, 0)) *abort_flag = 1;
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  __syncthreads();
  if (!*abort_flag) {
    const int64_t m = (int64_t)m0 + 32 * warp + lane;
    const bool row_ok = m < p.m;
    const uint32_t tbase = tmem + ((uint32_t)(32 * warp) << 16);
    float ts = 0.0f, ws = 0.0f;
    double tsum = 0.0, wsum = 0.0;
#pragma unroll 1
    for (int jb = 0; jb < 16; jb += 4) {   // 64 columns at a time: h and w loads issued first
      float4 hv[16];
      uint4 wv[8];
      const int64_t cb = (int64_t)n0 + 16 * jb;
      const bool vec = row_ok && cb + 64 <= p.n;
      if (vec) {
        const float4* hp = reinterpret_cast<const float4*>(p.h + m * p.n + cb);
#pragma unroll
        for (int i = 0; i < 16; ++i) hv[i] = hp[i];
        if (p.w) {
          const uint4* wp = reinterpret_cast<const uint4*>(p.w + m * p.n + cb);
#pragma unroll
          for (int i = 0; i < 8; ++i) wv[i] = __ldg(wp + i);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) wv[i] = make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        float v[16];
        oe_ld16(tbase + 16 * (jb + jj), v);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int64_t col = cb + 16 * jj + e;
          const float g = bf16_round(v[e]);                      // grad_w, bf16
          const float g2 = bf16_round(__fmul_rn(g, g));           // grad_w.pow(2), bf16
          float wf = 0.0f;
          if (vec) {
            const uint32_t u = (&wv[0].x)[(16 * jj + e) >> 1];
            wf = __uint_as_float(((16 * jj + e) & 1) ? (u & 0xFFFF0000u) : (u << 16));
            float* hc = &(&hv[0].x)[16 * jj + e];
            *hc = __fadd_rn(*hc, g2);
          } else if (row_ok && col < p.n) {
            if (p.w) wf = __uint_as_float((uint32_t)p.w[m * p.n + col] << 16);
            p.h[m * p.n + col] = __fadd_rn(p.h[m * p.n + col], g2);
          }
          ts = __fadd_rn(ts, g2);
          ws = __fadd_rn(ws, bf16_round(__fmul_rn(g2, bf16_round(__fmul_rn(wf, wf)))));
        }
        tsum += (double)ts;   // fp32 partials of 16 values
        wsum += (double)ws;
        ts = ws = 0.0f;
      }
      if (vec) {
        float4* hp = reinterpret_cast<float4*>(p.h + m * p.n + cb);
#pragma unroll
        for (int i = 0; i < 16; ++i) hp[i] = hv[i];
      }
    }
    tsum = warp_sum_d(tsum);
    wsum = warp_sum_d(wsum);
    if (lane == 0) {
      atomicAdd(p.sums, tsum);
      if (p.w) atomicAdd(p.sums + 1, wsum);
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (tid == 0 && prank == 0 && *abort_flag) {
    for (int j = *consumed; j < produced; ++j)
      (void)mbar_wait_bounded(&full[j % GS_NSTAGE], (uint32_t)((j / GS_NSTAGE) & 1), 1u << 20);
  }
  oe_cluster_sync();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(OE_TMEM_COLS));
  }
}

// bf16 [rows, cols] (cols % 8 == 0, 16-byte aligned base), box 64 (cols) x 64 (rows), SW128
static bool gs_tmap(CUtensorMap* map, const uint16_t* base, int64_t rows, int64_t cols) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = oe_encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {64, 64};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_gradsq(const uint16_t* gy, const uint16_t* x, const uint16_t* w, int64_t t, int64_t m, int64_t n,
                          float* h, double* sums, cudaStream_t stream) {
  CUtensorMap tg, tx;
  if (!gs_tmap(&tg, gy, t, m) || !gs_tmap(&tx, x, t, n)) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(gradsq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GS_SMEM);
  if (e != cudaSuccess) return e;
  const GsArgs args{m, n, t, h, w, sums};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * ((m + 255) / 256)), (unsigned)((n + 255) / 256), 1);
  cfg.blockDim = dim3(OE_THREADS, 1, 1);
  cfg.dynamicSmemBytes = GS_SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, gradsq_kernel, tg, tx, args);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_outerr(const uint16_t* x, const uint16_t* w, const uint16_t* xq, const uint16_t* wq, int64_t batch,
                          int64_t rows, int64_t out, int64_t K, double* err_sum, double* ref_energy, float* d_ref,
                          float* d_q, cudaStream_t stream) {
  const OeArgs a{rows, out, K, err_sum, ref_energy, nullptr, d_ref, d_q};
  return oe_launch<OE_DUAL, false>(x, w, xq, wq, batch, a, stream);
}

cudaError_t launch_outerr_ref(const uint16_t* x, const uint16_t* w, int64_t batch, int64_t rows, int64_t out,
                              int64_t K, uint16_t* y_ref, double* ref_energy, cudaStream_t stream) {
  const OeArgs a{rows, out, K, nullptr, ref_energy, y_ref, nullptr, nullptr};
  return oe_launch<OE_REF, true>(x, w, nullptr, nullptr, batch, a, stream);
}

cudaError_t launch_outerr_err(const uint16_t* xq, const uint16_t* wq, const uint16_t* y_ref, int64_t batch,
                              int64_t rows, int64_t out, int64_t K, double* err_sum, cudaStream_t stream) {
  const OeArgs a{rows, out, K, err_sum, nullptr, const_cast<uint16_t*>(y_ref), nullptr, nullptr};
  return oe_launch<OE_ERR, true>(xq, wq, nullptr, nullptr, batch, a, stream);
}

}  // namespace pq
