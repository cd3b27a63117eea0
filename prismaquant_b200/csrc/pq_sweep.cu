// Multi-format weight-error sweep and cost-path quantize->dequantize.
//
// Replaces, per (tensor, format), the reference chain
//   _batched_quantize -> err = (W - W_hat).float() -> err.pow(2).mean()
// (prismaquant/measure_quant_cost.py:452-491, 532-548, 627-632, 411-414) with
// ONE read of each bf16 weight for NVFP4, MXFP8 and FP8-per-channel together,
// and optionally the NVFP4 export codes in the same pass
// (prismaquant/export_native_compressed.py:1058-1102).
//
// Layout and schedule (staged kernel):
//  * a work item is `rows_per_item` consecutive rows of one tensor — one
//    contiguous chunk of <= STAGE_BYTES — so one 1-D bulk async copy (TMA
//    engine) moves it HBM -> shared memory, signalled on an mbarrier;
//  * a persistent CTA per SM walks its items round-robin through NSTAGE
//    shared-memory stages, the copies of the next items in flight while it
//    computes the current one;
//  * in the stage, thread t owns 8-element chunks c = t + k*blockDim (one
//    16-byte shared load each): NVFP4 16-groups are lane pairs, MXFP8
//    32-groups lane quads (shuffles); FP8-per-channel needs each row's amax
//    first, reduced into shared memory in a first pass over the stage.
#include "pq_common.cuh"
#include "pq_internal.h"

namespace pq {

struct ItemRef {
  int ti;
  int64_t r0;
  int64_t nr;
};

__device__ __forceinline__ ItemRef find_item(const SweepLaunch& L, int64_t item) {
  int lo = 0, hi = L.n - 1;
  while (lo < hi) {  // largest ti with prefix[ti] <= item
    const int mid = (lo + hi + 1) >> 1;
    if (L.item_prefix[mid] <= item) lo = mid; else hi = mid - 1;
  }
  const SweepDesc& d = L.t[lo];
  const int64_t local = item - L.item_prefix[lo];
  ItemRef r;
  r.ti = lo;
  r.r0 = local * d.rows_per_item;
  r.nr = min((int64_t)d.rows_per_item, d.rows - r.r0);
  return r;
}

// Per-format error of 8 elements sharing one scale.  Returns the fp32 sum of
// err^2 (each err is a bf16 value, so each square is exact in fp32) and, in
// QDQ mode, the bf16 reconstruction bits.
struct Chunk8 {
  float w[8];
};

__device__ __forceinline__ float nvfp4_cost8(const Chunk8& c, float a16, uint32_t (&rec)[8]) {
  const float s = __fdiv_rn(fmaxf(a16, 1e-8f), 6.0f);
  float part = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float x = __fdiv_rn(c.w[i], s);
    const float q = rtn_e2m1_cost(x);
    const float r = bf16_round(__fmul_rn(q, s));
    rec[i] = __float_as_uint(r) >> 16;
    const float e = bf16_round(__fsub_rn(c.w[i], r));
    part = fmaf(e, e, part);
  }
  return part;
}

__device__ __forceinline__ float mxfp8_cost8(const Chunk8& c, float a32, uint32_t (&rec)[8]) {
  const float s0 = __fdiv_rn(fmaxf(a32, 1e-8f), 448.0f);
  const int e = e8m0_round(s0);
  const float s = pow2i(e);
  const float inv = pow2i(-e);  // w * 2^-e == w / 2^e exactly (single rounding of the same value)
  float part = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float x = __fmul_rn(c.w[i], inv);
    const float q = rtn_e4m3_cost(x);
    const float r = bf16_round(__fmul_rn(q, s));
    rec[i] = __float_as_uint(r) >> 16;
    const float er = bf16_round(__fsub_rn(c.w[i], r));
    part = fmaf(er, er, part);
  }
  return part;
}

__device__ __forceinline__ float fp8ch_cost8(const Chunk8& c, float arow, uint32_t (&rec)[8]) {
  const float s = __fdiv_rn(fmaxf(arow, 1e-8f), 448.0f);
  float part = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float x = __fdiv_rn(c.w[i], s);
    const float q = rtn_e4m3_cost(x);
    const float r = bf16_round(__fmul_rn(q, s));
    rec[i] = __float_as_uint(r) >> 16;
    const float er = bf16_round(__fsub_rn(c.w[i], r));
    part = fmaf(er, er, part);
  }
  return part;
}

// NVFP4 export codes for 8 elements (8 nibbles, element 0 in the low nibble).
__device__ __forceinline__ uint32_t nvfp4_codes8(const Chunk8& c, float a16) {
  const float s = fmaxf(__fdiv_rn(fmaxf(a16, 1e-12f), 6.0f), 1e-12f);
  uint32_t out = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) out |= nvfp4_code(__fdiv_rn(c.w[i], s)) << (4 * i);
  return out;
}

__device__ __forceinline__ uint4 pack_rec8(const uint32_t (&rec)[8]) {
  return make_uint4(rec[0] | (rec[1] << 16), rec[2] | (rec[3] << 16), rec[4] | (rec[5] << 16),
                    rec[6] | (rec[7] << 16));
}

template <int MODE>
__global__ void __launch_bounds__(SWEEP_THREADS, 1) sweep_staged_kernel(const __grid_constant__ SweepLaunch L) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* stages = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NSTAGE * STAGE_BYTES);
  uint32_t* row_amax = reinterpret_cast<uint32_t*>(bars + NSTAGE + 1);
  double* red = reinterpret_cast<double*>(row_amax + MAX_ROWS_PER_ITEM);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + NSTAGE);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NWARPS = SWEEP_THREADS / 32;
  const int64_t n_items = L.item_prefix[L.n];
  const int64_t my_n = n_items > (int64_t)blockIdx.x ? (n_items - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;

  if (tid == 0) {
    for (int s = 0; s < NSTAGE; ++s) mbar_init(&bars[s], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  auto issue = [&](int64_t j) {
    const ItemRef it = find_item(L, (int64_t)blockIdx.x + j * gridDim.x);
    const SweepDesc& d = L.t[it.ti];
    const uint32_t bytes = (uint32_t)(it.nr * d.cols * 2);
    uint64_t* bar = &bars[j % NSTAGE];
    mbar_arrive_expect_tx(bar, bytes);
    bulk_g2s(stages + (j % NSTAGE) * STAGE_BYTES, d.w + it.r0 * d.cols, bytes, bar);
  };

  if (tid == 0)
    for (int64_t j = 0; j < NSTAGE && j < my_n; ++j) issue(j);

  int64_t j_abort = -1;
  for (int64_t j = 0; j < my_n; ++j) {
    const int s = (int)(j % NSTAGE);
    const uint32_t parity = (uint32_t)((j / NSTAGE) & 1);
    const ItemRef it = find_item(L, (int64_t)blockIdx.x + j * gridDim.x);
    const SweepDesc& d = L.t[it.ti];

    if (!mbar_wait_stage(&bars[s], parity)) *abort_flag = 1;
    __syncthreads();
    if (*abort_flag) {
      j_abort = j;
      break;
    }

    const uint4* st = reinterpret_cast<const uint4*>(stages + s * STAGE_BYTES);
    const int cpr = (int)(d.cols >> 3);
    const int nchunks = (int)it.nr * cpr;
    const uint32_t mask = MODE == MODE_QDQ ? (1u << L.qdq_fmt) : d.fmt_mask;
    const bool codes = MODE == MODE_SSE && d.nvfp4_codes != nullptr;

    if (mask & PQ_FMT_BIT(PQ_FMT_FP8_CHANNEL)) {
      for (int i = tid; i < it.nr; i += SWEEP_THREADS) row_amax[i] = 0u;
      __syncthreads();
      const bool warp_rows = (cpr & 31) == 0;  // every warp span lies inside one row
      const int iters = (nchunks + SWEEP_THREADS - 1) / SWEEP_THREADS;
      for (int k = 0; k < iters; ++k) {
        const int c = tid + k * SWEEP_THREADS;
        uint32_t a = 0u;
        if (c < nchunks) {
          Chunk8 ch;
          unpack8(st[c], ch.w);
          a = __float_as_uint(amax8(ch.w));
        }
        if (warp_rows) {
          a = warp_max_u(a);
          const int c0 = c - lane;
          if (lane == 0 && c0 < nchunks) atomicMax(&row_amax[c0 / cpr], a);
        } else if (c < nchunks) {
          atomicMax(&row_amax[c / cpr], a);
        }
      }
      __syncthreads();
    }

    double acc0 = 0.0, acc1 = 0.0, acc2 = 0.0;
    uint32_t tmax = 0u;
    const int64_t elem0 = it.r0 * d.cols;
    const int iters = (nchunks + SWEEP_THREADS - 1) / SWEEP_THREADS;
    for (int k = 0; k < iters; ++k) {
      const int c = tid + k * SWEEP_THREADS;
      const bool valid = c < nchunks;
      Chunk8 ch;
      unpack8(valid ? st[c] : make_uint4(0, 0, 0, 0), ch.w);
      const float a8 = amax8(ch.w);
      const float a16 = fmaxf(a8, __shfl_xor_sync(FULL, a8, 1));
      const float a32 = fmaxf(a16, __shfl_xor_sync(FULL, a16, 2));
      uint32_t rec[8];
      if (mask & PQ_FMT_BIT(PQ_FMT_NVFP4)) {
        const float p = nvfp4_cost8(ch, a16, rec);
        if (MODE == MODE_QDQ) {
          if (valid) *reinterpret_cast<uint4*>(d.out + elem0 + 8 * (int64_t)c) = pack_rec8(rec);
        } else if (valid) {
          acc0 += (double)p;
        }
      }
      if (mask & PQ_FMT_BIT(PQ_FMT_MXFP8)) {
        const float p = mxfp8_cost8(ch, a32, rec);
        if (MODE == MODE_QDQ) {
          if (valid) *reinterpret_cast<uint4*>(d.out + elem0 + 8 * (int64_t)c) = pack_rec8(rec);
        } else if (valid) {
          acc1 += (double)p;
        }
      }
      if (mask & PQ_FMT_BIT(PQ_FMT_FP8_CHANNEL)) {
        const float arow = valid ? __uint_as_float(row_amax[c / cpr]) : 0.0f;
        const float p = fp8ch_cost8(ch, arow, rec);
        if (MODE == MODE_QDQ) {
          if (valid) *reinterpret_cast<uint4*>(d.out + elem0 + 8 * (int64_t)c) = pack_rec8(rec);
        } else if (valid) {
          acc2 += (double)p;
        }
      }
      if (codes && valid) {
        const uint32_t cw = nvfp4_codes8(ch, a16);
        *reinterpret_cast<uint32_t*>(d.nvfp4_codes + (elem0 + 8 * (int64_t)c) / 2) = cw;
        if ((lane & 1) == 0) d.nvfp4_amax[(elem0 + 8 * (int64_t)c) / 16] = (uint16_t)(__float_as_uint(a16) >> 16);
        tmax = max(tmax, __float_as_uint(a16));
      }
    }

    if (MODE == MODE_SSE) {
      acc0 = warp_sum_d(acc0);
      acc1 = warp_sum_d(acc1);
      acc2 = warp_sum_d(acc2);
      if (codes) {
        tmax = warp_max_u(tmax);
        if (lane == 0) atomicMax(d.nvfp4_tmax, tmax);
      }
      if (lane == 0) {
        red[warp * 3 + 0] = acc0;
        red[warp * 3 + 1] = acc1;
        red[warp * 3 + 2] = acc2;
      }
      __syncthreads();
      if (warp == 0) {
#pragma unroll
        for (int f = 0; f < 3; ++f) {
          double v = lane < NWARPS ? red[lane * 3 + f] : 0.0;
          v = warp_sum_d(v);
          if (lane == 0 && (mask & (1u << f))) atomicAdd(d.sse + f, v);
        }
      }
    }
    __syncthreads();  // stage s and row_amax are free again
    if (tid == 0 && j + NSTAGE < my_n) {
      fence_proxy_async_smem();
      issue(j + NSTAGE);
    }
  }

  // On an aborted wait, drain the copies this CTA still has in flight
  // (bounded) before the shared memory goes away.
  if (j_abort >= 0 && tid == 0) {
    for (int64_t jj = j_abort; jj < j_abort + NSTAGE && jj < my_n; ++jj)
      (void)mbar_wait_bounded(&bars[jj % NSTAGE], (uint32_t)((jj / NSTAGE) & 1), 1u << 20);
  }
}

// ---------------------------------------------------------------------------
// Generic path: any shape (group = whole row when the row is shorter than the
// format's group; format_registry.py:208-212).  One warp per row, direct
// global loads.  Used for shapes the staged kernel does not take.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ldw(const uint16_t* p) { return __uint_as_float((uint32_t)__ldg(p) << 16); }

template <int MODE>
__global__ void __launch_bounds__(256) sweep_generic_kernel(const uint16_t* __restrict__ w, int64_t rows, int64_t cols,
                                                            uint32_t mask, double* sse, uint16_t* out) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  double acc[3] = {0.0, 0.0, 0.0};
  for (int64_t r = gw; r < rows; r += nw) {
    const uint16_t* row = w + r * cols;
    float ar = 0.0f;
    for (int64_t i = lane; i < cols; i += 32) ar = fmaxf(ar, fabsf(ldw(row + i)));
    ar = __uint_as_float(warp_max_u(__float_as_uint(ar)));
    for (int f = 0; f < 3; ++f) {
      if (!(mask & (1u << f))) continue;
      const int64_t g = f == PQ_FMT_NVFP4 ? (cols <= 16 ? cols : 16) : f == PQ_FMT_MXFP8 ? (cols <= 32 ? cols : 32) : cols;
      const int64_t ng = cols / g;
      const int64_t per_lane = f == PQ_FMT_FP8_CHANNEL ? 1 : 0;
      float part = 0.0f;
      if (per_lane) {
        const float s = __fdiv_rn(fmaxf(ar, 1e-8f), 448.0f);
        for (int64_t i = lane; i < cols; i += 32) {
          const float wi = ldw(row + i);
          const float r_ = bf16_round(__fmul_rn(rtn_e4m3_cost(__fdiv_rn(wi, s)), s));
          if (MODE == MODE_QDQ) out[r * cols + i] = (uint16_t)(__float_as_uint(r_) >> 16);
          const float e = bf16_round(__fsub_rn(wi, r_));
          part = fmaf(e, e, part);
        }
      } else {
        for (int64_t gi = lane; gi < ng; gi += 32) {
          const uint16_t* gp = row + gi * g;
          float a = 0.0f;
          for (int64_t i = 0; i < g; ++i) a = fmaxf(a, fabsf(ldw(gp + i)));
          float s, inv = 0.0f;
          bool mx = f == PQ_FMT_MXFP8;
          if (mx) {
            const int e = e8m0_round(__fdiv_rn(fmaxf(a, 1e-8f), 448.0f));
            s = pow2i(e);
            inv = pow2i(-e);
          } else {
            s = __fdiv_rn(fmaxf(a, 1e-8f), 6.0f);
          }
          for (int64_t i = 0; i < g; ++i) {
            const float wi = ldw(gp + i);
            const float q = mx ? rtn_e4m3_cost(__fmul_rn(wi, inv)) : rtn_e2m1_cost(__fdiv_rn(wi, s));
            const float r_ = bf16_round(__fmul_rn(q, s));
            if (MODE == MODE_QDQ) out[r * cols + gi * g + i] = (uint16_t)(__float_as_uint(r_) >> 16);
            const float e = bf16_round(__fsub_rn(wi, r_));
            part = fmaf(e, e, part);
          }
        }
      }
      acc[f] += (double)part;
    }
  }
  if (MODE == MODE_SSE) {
    for (int f = 0; f < 3; ++f) {
      if (!(mask & (1u << f))) continue;
      const double v = warp_sum_d(acc[f]);
      if (lane == 0) atomicAdd(sse + f, v);
    }
  }
}

// ---------------------------------------------------------------------------
// Host-side launchers (called from pq_capi.cu)
// ---------------------------------------------------------------------------
size_t sweep_smem_bytes() {
  return (size_t)NSTAGE * STAGE_BYTES + (NSTAGE + 1) * sizeof(uint64_t) + MAX_ROWS_PER_ITEM * sizeof(uint32_t) +
         (SWEEP_THREADS / 32) * 3 * sizeof(double);
}

cudaError_t launch_sweep_staged(const SweepLaunch& L, int mode, int grid, cudaStream_t stream) {
  const size_t smem = sweep_smem_bytes();
  cudaError_t e;
  if (mode == MODE_QDQ) {
    e = cudaFuncSetAttribute(sweep_staged_kernel<MODE_QDQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    sweep_staged_kernel<MODE_QDQ><<<grid, SWEEP_THREADS, smem, stream>>>(L);
  } else {
    e = cudaFuncSetAttribute(sweep_staged_kernel<MODE_SSE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    sweep_staged_kernel<MODE_SSE><<<grid, SWEEP_THREADS, smem, stream>>>(L);
  }
  return cudaGetLastError();
}

cudaError_t launch_sweep_generic(const uint16_t* w, int64_t rows, int64_t cols, uint32_t mask, double* sse,
                                 uint16_t* out, int mode, int num_sms, cudaStream_t stream) {
  const int64_t warps = rows;
  int64_t blocks = (warps * 32 + 255) / 256;
  blocks = blocks < (int64_t)num_sms * 8 ? blocks : (int64_t)num_sms * 8;
  if (blocks < 1) blocks = 1;
  if (mode == MODE_QDQ)
    sweep_generic_kernel<MODE_QDQ><<<(unsigned)blocks, 256, 0, stream>>>(w, rows, cols, mask, sse, out);
  else
    sweep_generic_kernel<MODE_SSE><<<(unsigned)blocks, 256, 0, stream>>>(w, rows, cols, mask, sse, out);
  return cudaGetLastError();
}

}  // namespace pq
