// Fisher-trace statistics as HBM-streaming reductions.
//
//  * sumsq_rows   — _GradNormCapture.backward (prismaquant/sensitivity_probe.py:451-482):
//                   scalar sum of g^2 (fp64) and the per-row [E, M] channel diagonal (fp32).
//  * rownorm2     — per-token ||x_t||^2 of a Linear's input, taken in the forward hook
//                   so the activation itself need not be kept for the backward.
//  * tokennorm_dot— sum_t ||x_t||^2 ||g_t||^2 in the backward hook: the per-token Fisher
//                   estimate that replaces grad_w = gy^T x; sum(grad_w^2)
//                   (prismaquant/sensitivity_probe.py:1115-1152), optionally over the
//                   tokens routed to one expert (token_idx).
//
// One warp per row; each lane reads 16-byte vectors (8 bf16), squares are
// summed in fp32 per 8 elements and in fp64 across them.
#include "pq_common.cuh"
#include "pq_internal.h"

namespace pq {

__device__ __forceinline__ float sq8(const uint4& v) {
  float w[8];
  unpack8(v, w);
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s = fmaf(w[i], w[i], s);
  return s;
}

// Sum of squares of one bf16 row, reduced over the warp (every lane gets it).
__device__ __forceinline__ double row_sumsq(const uint16_t* __restrict__ row, int64_t cols, int lane) {
  double acc = 0.0;
  if ((cols & 7) == 0 && (reinterpret_cast<uintptr_t>(row) & 15) == 0) {
    const uint4* rv = reinterpret_cast<const uint4*>(row);
    const int64_t n8 = cols >> 3;
    int64_t c = lane;
    for (; c + 32 < n8; c += 64) {  // two independent loads in flight per lane
      const uint4 a = __ldg(rv + c), b = __ldg(rv + c + 32);
      acc += (double)sq8(a) + (double)sq8(b);
    }
    for (; c < n8; c += 32) acc += (double)sq8(__ldg(rv + c));
  } else {
    float part = 0.0f;
    int cnt = 0;
    for (int64_t i = lane; i < cols; i += 32) {
      const float x = __uint_as_float((uint32_t)__ldg(row + i) << 16);
      part = fmaf(x, x, part);
      if (++cnt == 8) {
        acc += (double)part;
        part = 0.0f;
        cnt = 0;
      }
    }
    acc += (double)part;
  }
  return warp_sum_d(acc);
}

__global__ void __launch_bounds__(256) sumsq_rows_kernel(const uint16_t* __restrict__ g, int64_t rows, int64_t cols,
                                                         double* total, float* per_row) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  double acc = 0.0;
  for (int64_t r = gw; r < rows; r += nw) {
    const double v = row_sumsq(g + r * cols, cols, lane);
    if (lane == 0 && per_row != nullptr) per_row[r] += (float)v;
    acc += v;
  }
  __shared__ double red[8];
  if (lane == 0) red[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
    atomicAdd(total, t);
  }
}

// sumsq_rows with the per-weight [E, M, N] accumulator of _GradNormCapture
// (sensitivity_probe.py:486-503): h[i] += fp32(g[i])^2 in fp32 (each square is exact, each add
// one IEEE rounding, as the reference's `cur.add_(g.float().pow(2))`), in the same read of g.
__device__ __forceinline__ double row_sumsq_acc(const uint16_t* __restrict__ row, float* __restrict__ hrow,
                                                int64_t cols, int lane) {
  double acc = 0.0;
  if ((cols & 7) == 0 && (reinterpret_cast<uintptr_t>(row) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(hrow) & 15) == 0) {
    const uint4* rv = reinterpret_cast<const uint4*>(row);
    float4* hv = reinterpret_cast<float4*>(hrow);
    const int64_t n8 = cols >> 3;
    for (int64_t c = lane; c < n8; c += 32) {
      float w[8];
      unpack8(__ldg(rv + c), w);
      float4 h0 = hv[2 * c], h1 = hv[2 * c + 1];
      float s = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) s = fmaf(w[i], w[i], s);
      h0.x = __fadd_rn(h0.x, __fmul_rn(w[0], w[0])); h0.y = __fadd_rn(h0.y, __fmul_rn(w[1], w[1]));
      h0.z = __fadd_rn(h0.z, __fmul_rn(w[2], w[2])); h0.w = __fadd_rn(h0.w, __fmul_rn(w[3], w[3]));
      h1.x = __fadd_rn(h1.x, __fmul_rn(w[4], w[4])); h1.y = __fadd_rn(h1.y, __fmul_rn(w[5], w[5]));
      h1.z = __fadd_rn(h1.z, __fmul_rn(w[6], w[6])); h1.w = __fadd_rn(h1.w, __fmul_rn(w[7], w[7]));
      hv[2 * c] = h0;
      hv[2 * c + 1] = h1;
      acc += (double)s;
    }
  } else {
    float part = 0.0f;
    int cnt = 0;
    for (int64_t i = lane; i < cols; i += 32) {
      const float x = __uint_as_float((uint32_t)__ldg(row + i) << 16);
      const float x2 = __fmul_rn(x, x);
      hrow[i] = __fadd_rn(hrow[i], x2);
      part = __fadd_rn(part, x2);
      if (++cnt == 8) {
        acc += (double)part;
        part = 0.0f;
        cnt = 0;
      }
    }
    acc += (double)part;
  }
  return warp_sum_d(acc);
}

__global__ void __launch_bounds__(256) sumsq_rows_full_kernel(const uint16_t* __restrict__ g, int64_t rows,
                                                              int64_t cols, double* total, float* per_row,
                                                              float* __restrict__ h) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  double acc = 0.0;
  for (int64_t r = gw; r < rows; r += nw) {
    const double v = row_sumsq_acc(g + r * cols, h + r * cols, cols, lane);
    if (lane == 0 && per_row != nullptr) per_row[r] += (float)v;
    acc += v;
  }
  __shared__ double red[8];
  if (lane == 0) red[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
    atomicAdd(total, t);
  }
}

__global__ void __launch_bounds__(256) rownorm2_kernel(const uint16_t* __restrict__ x, int64_t T, int64_t d,
                                                       float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t t = gw; t < T; t += nw) {
    const double v = row_sumsq(x + t * d, d, lane);
    if (lane == 0) out[t] = (float)v;
  }
}

__global__ void __launch_bounds__(256) tokennorm_dot_kernel(const uint16_t* __restrict__ g, int64_t T, int64_t d,
                                                            const float* __restrict__ xnorm,
                                                            const int64_t* __restrict__ token_idx, double* acc) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  double a = 0.0;
  for (int64_t t = gw; t < T; t += nw) {
    const double gn = row_sumsq(g + t * d, d, lane);
    const int64_t src = token_idx != nullptr ? token_idx[t] : t;
    a += gn * (double)xnorm[src];
  }
  __shared__ double red[8];
  if (lane == 0) red[warp] = a;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += red[i];
    atomicAdd(acc, s);
    if (blockIdx.x == 0) atomicAdd(acc + 1, (double)T);
  }
}

// Routed experts in one launch: rows of g are the (token, expert) pairs of one packed projection,
// sorted by expert, row r belonging to expert seg[r]; acc[e] += (sum over e's rows of
// xnorm[tok(r)] * ||g_r||^2, row count).  Each warp takes a contiguous run of rows and flushes its
// running sums at every change of expert (fp64 atomics), so a run costs one atomic per expert it
// touches.  tok == NULL: row r's norm is xnorm[r] (inputs already in row order).
__global__ void __launch_bounds__(256) tokennorm_seg_kernel(const uint16_t* __restrict__ g, int64_t R, int64_t d,
                                                           const float* __restrict__ xnorm,
                                                           const int64_t* __restrict__ tok,
                                                           const int32_t* __restrict__ seg, double* acc) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t per = (R + nw - 1) / nw;
  const int64_t r0 = gw * per, r1 = min(R, r0 + per);
  double a = 0.0, cnt = 0.0;
  int cur = -1;
  for (int64_t r = r0; r < r1; ++r) {
    const int e = seg[r];
    if (e != cur) {
      if (cur >= 0 && lane == 0) {
        atomicAdd(acc + 2 * cur, a);
        atomicAdd(acc + 2 * cur + 1, cnt);
      }
      cur = e;
      a = cnt = 0.0;
    }
    const double gn = row_sumsq(g + r * d, d, lane);
    a += gn * (double)xnorm[tok != nullptr ? tok[r] : r];
    cnt += 1.0;
  }
  if (cur >= 0 && lane == 0) {
    atomicAdd(acc + 2 * cur, a);
    atomicAdd(acc + 2 * cur + 1, cnt);
  }
}

static inline int warp_grid(int64_t rows, int num_sms) {
  int64_t blocks = (rows + 7) / 8;
  const int64_t cap = (int64_t)num_sms * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

cudaError_t launch_sumsq_rows(const uint16_t* g, int64_t rows, int64_t cols, double* total, float* per_row,
                              int num_sms, cudaStream_t stream) {
  sumsq_rows_kernel<<<warp_grid(rows, num_sms), 256, 0, stream>>>(g, rows, cols, total, per_row);
  return cudaGetLastError();
}

cudaError_t launch_sumsq_rows_full(const uint16_t* g, int64_t rows, int64_t cols, double* total, float* per_row,
                                   float* h, int num_sms, cudaStream_t stream) {
  sumsq_rows_full_kernel<<<warp_grid(rows, num_sms), 256, 0, stream>>>(g, rows, cols, total, per_row, h);
  return cudaGetLastError();
}

cudaError_t launch_rownorm2(const uint16_t* x, int64_t T, int64_t d, float* out, int num_sms, cudaStream_t stream) {
  rownorm2_kernel<<<warp_grid(T, num_sms), 256, 0, stream>>>(x, T, d, out);
  return cudaGetLastError();
}

cudaError_t launch_tokennorm_dot(const uint16_t* g, int64_t T, int64_t d, const float* xnorm,
                                 const int64_t* token_idx, double* acc, int num_sms, cudaStream_t stream) {
  tokennorm_dot_kernel<<<warp_grid(T, num_sms), 256, 0, stream>>>(g, T, d, xnorm, token_idx, acc);
  return cudaGetLastError();
}

cudaError_t launch_tokennorm_seg(const uint16_t* g, int64_t R, int64_t d, const float* xnorm, const int64_t* tok,
                                 const int32_t* seg, double* acc, int num_sms, cudaStream_t stream) {
  int64_t blocks = (R + 8 * 8 - 1) / (8 * 8);   // about eight rows per warp
  const int64_t cap = (int64_t)num_sms * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  tokennorm_seg_kernel<<<(unsigned)blocks, 256, 0, stream>>>(g, R, d, xnorm, tok, seg, acc);
  return cudaGetLastError();
}

}  // namespace pq
