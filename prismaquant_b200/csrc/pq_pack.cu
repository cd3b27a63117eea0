// Export packing kernels: NVFP4 (codes + E4M3 block scales + fp32 global),
// MXFP8 (E4M3 values + E8M0 scales), FP8 per-channel (E4M3 values + fp32 row
// scales), in the compressed-tensors layouts the reference writes
// (prismaquant/export_native_compressed.py:1045-1226).
//
// All are HBM-streaming kernels: each warp instruction moves 512 contiguous
// bytes (one 16-byte vector per lane, 8 bf16 elements), groups are formed
// with lane shuffles, outputs are written with vector stores.
#include "pq_common.cuh"
#include "pq_fast.cuh"
#include "pq_internal.h"

namespace pq {

static inline int grid_for(int64_t warps_needed, int num_sms, int per_sm = 8, int threads = 256) {
  int64_t blocks = (warps_needed * 32 + threads - 1) / threads;
  const int64_t cap = (int64_t)num_sms * per_sm;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

// ---------------------------------------------------------------------------
// NVFP4 pass 1: codes, group amax (bf16), per-slice max group amax.
// Codes are independent of the global scale (export_native_compressed.py:1093-1096):
//   in_grid = w / max(max(amax,1e-12)/6, 1e-12), abs-codebook RTN, ties -> 0.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) nvfp4_codes_kernel(const uint16_t* __restrict__ w, int64_t n_chunks,
                                                          int64_t chunks_per_slice, uint8_t* __restrict__ codes,
                                                          uint16_t* __restrict__ amax, uint32_t* tmax) {
  const int lane = threadIdx.x & 31;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t cur_b = -1;
  uint32_t cur_max = 0u;
  for (int64_t c0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x - lane; c0 < n_chunks; c0 += stride) {
    const int64_t c = c0 + lane;
    const bool valid = c < n_chunks;
    float v[8];
    unpack8(valid ? __ldg(reinterpret_cast<const uint4*>(w) + c) : make_uint4(0, 0, 0, 0), v);
    const float a8 = amax8(v);
    const float a16 = fmaxf(a8, __shfl_xor_sync(FULL, a8, 1));
    if (valid) {
      const float s = fmaxf(__fdiv_rn(fmaxf(a16, 1e-12f), 6.0f), 1e-12f);
      uint32_t cw = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) cw |= nvfp4_code(__fdiv_rn(v[i], s)) << (4 * i);
      reinterpret_cast<uint32_t*>(codes)[c] = cw;
      if ((lane & 1) == 0) amax[c >> 1] = (uint16_t)(__float_as_uint(a16) >> 16);
    }
    // per-slice running max; flushed when the slice changes
    const int64_t b = valid ? c / chunks_per_slice : -1;
    const int64_t b0 = __shfl_sync(FULL, b, 0);
    const bool uniform = __all_sync(FULL, b == b0 || b < 0);
    if (uniform) {
      const uint32_t m = warp_max_u(valid ? __float_as_uint(a16) : 0u);
      if (lane == 0 && b0 >= 0) {
        if (b0 != cur_b) {
          if (cur_b >= 0) atomicMax(tmax + cur_b, cur_max);
          cur_b = b0;
          cur_max = 0u;
        }
        cur_max = max(cur_max, m);
      }
    } else if (valid) {
      atomicMax(tmax + b, __float_as_uint(a16));
    }
  }
  if (lane == 0 && cur_b >= 0) atomicMax(tmax + cur_b, cur_max);
}

cudaError_t launch_nvfp4_codes(const uint16_t* w, int64_t batch, int64_t rows, int64_t cols, uint8_t* codes,
                               uint16_t* amax, uint32_t* tmax, int num_sms, cudaStream_t stream) {
  const int64_t n_chunks = batch * rows * cols / 8;
  const int64_t cps = rows * cols / 8;
  nvfp4_codes_kernel<<<grid_for(n_chunks / 32 + 1, num_sms), 256, 0, stream>>>(w, n_chunks, cps, codes, amax,
                                                                                  tmax);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// NVFP4 pass 2: E4M3 block scales and the global divisor (1/global_real).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float nvfp4_global_from_tmax(uint32_t tmax_bits) {
  // compute_nvfp4_global_real: (max_g(max(amax,1e-12)/6) / 448).clamp_min(1e-12); the max of the
  // rounded quotients is the quotient of the max (round-to-nearest is monotone).
  const float sg = __fdiv_rn(fmaxf(__uint_as_float(tmax_bits), 1e-12f), 6.0f);
  return fmaxf(__fdiv_rn(sg, 448.0f), 1e-12f);
}

// compute_nvfp4_global_real (export_native_compressed.py:1045-1055) of `n_slices` consecutive
// slices of n_per bf16 values: one read of the weights.  Each block reduces its elements' bf16
// magnitude bits (two per 32-bit max) and adds its slices' maxima into tmax[] (float bits,
// atomic max; zeroed by the caller); the last block to finish turns every slice's maximum into
// its global_real.  The 16-groups need not be formed: the max over groups of max(amax, 1e-12) / 6
// is the same quotient of the slice's max (round-to-nearest is monotone).
__global__ void __launch_bounds__(256) nvfp4_global_kernel(const uint16_t* __restrict__ w, int64_t n_per, int n_slices,
                                                           uint32_t* tmax, unsigned int* done, float* global_real) {
  const int64_t total = n_per * n_slices;
  const int64_t n8 = total >> 3;   // the caller guarantees n_per % 8 == 0 and 16-byte alignment
  const uint4* v = reinterpret_cast<const uint4*>(w);
  __shared__ uint32_t s_max[MAX_SCALE_SLICES];
  for (int i = threadIdx.x; i < n_slices; i += blockDim.x) s_max[i] = 0u;
  __syncthreads();
  const int64_t per8 = n_per >> 3;
  int slice = -1;
  uint32_t m = 0u;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const int sl = (int)(i / per8);
    if (sl != slice) {
      if (slice >= 0) atomicMax(&s_max[slice], m);
      slice = sl;
      m = 0u;
    }
    const uint4 x = __ldg(v + i);
    const uint32_t a = bf16x2_maxabs(bf16x2_maxabs(x.x, x.y), bf16x2_maxabs(x.z, x.w));
    m = max(m, max(a & 0x7FFFu, (a >> 16) & 0x7FFFu));
  }
  if (slice >= 0) atomicMax(&s_max[slice], m);
  __syncthreads();
  for (int i = threadIdx.x; i < n_slices; i += blockDim.x)
    if (s_max[i]) atomicMax(&tmax[i], s_max[i] << 16);
  __threadfence();
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) last = atomicAdd(done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int i = threadIdx.x; i < n_slices; i += blockDim.x)
    global_real[i] = nvfp4_global_from_tmax(*(volatile uint32_t*)&tmax[i]);
}

cudaError_t launch_nvfp4_global(const uint16_t* w, int64_t n_per, int n_slices, uint32_t* scratch, float* global_real,
                                int num_sms, cudaStream_t stream) {
  cudaError_t e = cudaMemsetAsync(scratch, 0, (size_t)(n_slices + 1) * sizeof(uint32_t), stream);
  if (e != cudaSuccess) return e;
  const int64_t n8 = n_per * n_slices / 8;
  int64_t blocks = (n8 + 255) / 256;
  const int64_t cap = (int64_t)num_sms * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  nvfp4_global_kernel<<<(unsigned)blocks, 256, 0, stream>>>(w, n_per, n_slices, scratch,
                                                            reinterpret_cast<unsigned int*>(scratch + n_slices),
                                                            global_real);
  return cudaGetLastError();
}

// Block scale byte of one group: e4m3(clamp(RN(RN(max(amax, 1e-12) / 6) / glob), 0, 448)), RNE
// (export_native_compressed.py:1099-1102), by IEEE division.
__device__ __forceinline__ uint32_t nvfp4_scale_exact(uint32_t abits, float glob) {
  const float sg = __fdiv_rn(fmaxf(__uint_as_float(abits << 16), 1e-12f), 6.0f);
  return e4m3_byte(fminf(fmaxf(__fdiv_rn(sg, glob), 0.0f), 448.0f));
}

// RNE choice between adjacent E4M3 codes lo < hi (one byte) for the quotient a / s.
__device__ __forceinline__ uint32_t e4m3_rne_pick(float a, float s, uint32_t lo, uint32_t hi) {
  bool up, dn;
  mid_side(a, e4m3x2_to_f2_lo(lo), e4m3x2_to_f2_lo(hi), s, up, dn);
  return up ? hi : dn ? lo : ((lo & 1u) ? hi : lo);   // a tie goes to the even code
}

// Two groups at once (amax pair a2, low half first) without dividing: sg = a/6 by
// div_const (exact for every normal bf16 and the 1e-12 floor), then sg/glob is
// bracketed between RZ(sg * r_lo) and RZ(sg * r_hi) as in the fast sweep and both
// are converted with the hardware RNE E4M3 conversion (saturating at 448, as the
// clamp does).  Equal codes are the reference's code; where they differ (a
// quotient within ~2^-20 of an E4M3 midpoint) mid_side decides the side exactly.
__device__ __forceinline__ uint32_t nvfp4_scale_pair(uint32_t a2, float glob, uint64_t rlo2, uint64_t rhi2) {
  // div_const on the pair in float32x2 arithmetic (the same three roundings per element)
  const uint64_t a = f2_pack(fmaxf(__uint_as_float(a2 << 16), 1e-12f), fmaxf(__uint_as_float(a2 & 0xFFFF0000u), 1e-12f));
  const uint64_t rd2 = f2_pack(RCP6, RCP6), nd2 = f2_pack(-6.0f, -6.0f);
  const uint64_t q = f2_mul_rn(a, rd2);
  const uint64_t sg2 = f2_fma_rn(f2_fma_rn(q, nd2, a), rd2, q);
  float sg0, sg1;
  f2_unpack(sg2, sg0, sg1);
  const uint32_t lo = cvt_e4m3x2(f2_mul_rz(sg2, rlo2));
  const uint32_t hi = cvt_e4m3x2(f2_mul_rz(sg2, rhi2));
  if (lo == hi) return lo;
  uint32_t r = lo;
  if ((lo ^ hi) & 0x00FFu) r = (r & 0xFF00u) | e4m3_rne_pick(sg0, glob, lo & 0xFFu, hi & 0xFFu);
  if ((lo ^ hi) & 0xFF00u) r = (r & 0x00FFu) | (e4m3_rne_pick(sg1, glob, lo >> 8, hi >> 8) << 8);
  return r;
}

// One thread per 32 consecutive groups of the flattened (slice, group) space, so
// a huge slice (lm_head) spreads over the whole grid instead of one column of
// blocks.  Slice b covers flat groups [gprefix[b], gprefix[b+1]).
constexpr int SCALE_GROUPS_PER_THREAD = 32;

__global__ void __launch_bounds__(256) nvfp4_scales_kernel(const __grid_constant__ ScalesLaunch L) {
  __shared__ float s_nat[MAX_SCALE_SLICES];
  __shared__ float s_glob[MAX_SCALE_SLICES];
  __shared__ float s_rlo[MAX_SCALE_SLICES], s_rhi[MAX_SCALE_SLICES];
  if (L.override_ == nullptr)
    for (int c = threadIdx.x; c < L.n; c += blockDim.x) s_nat[c] = nvfp4_global_from_tmax(L.tmax[c]);
  __syncthreads();
  for (int b = threadIdx.x; b < L.n; b += blockDim.x) {
    float g;
    if (L.override_ != nullptr) {
      g = fmaxf(L.override_[b], 1e-12f);
    } else {
      g = s_nat[b];   // joint global of a fused-sibling group: the max of the members' globals
      if (L.group_of[b] >= 0)
        for (int c = 0; c < L.n; ++c)
          if (L.group_of[c] == L.group_of[b]) g = fmaxf(g, s_nat[c]);
    }
    s_glob[b] = g;
    // The bracket needs a normal reciprocal with room to spare; a slice whose global lies
    // outside [1e-30, 1e30] (only reachable through an override) is marked r_lo < 0 and
    // takes the division path.
    if (g >= 1.0e-30f && g <= 1.0e30f) {
      recip_bounds(g, s_rlo[b], s_rhi[b]);
    } else {
      s_rlo[b] = -1.0f;
      s_rhi[b] = -1.0f;
    }
    if (blockIdx.x == 0) L.global_div[b] = __frcp_rn(g);
  }
  __syncthreads();
  constexpr int G = SCALE_GROUPS_PER_THREAD;
  const int64_t total = L.gprefix[L.n];
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * G;
  int b = 0;
  for (int64_t g0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * G; g0 < total; g0 += stride) {
    while (b + 1 < L.n && L.gprefix[b + 1] <= g0) ++b;   // monotone per thread
    int bb = b;
    const int64_t local = g0 - L.gprefix[bb];
    const uint16_t* am = L.amax[bb];
    uint8_t* sc = L.scales[bb];
    if (g0 + G <= L.gprefix[bb + 1] && s_rlo[bb] > 0.0f && ((reinterpret_cast<uintptr_t>(am + local) & 15) == 0) &&
        ((reinterpret_cast<uintptr_t>(sc + local) & 15) == 0)) {
      const float glob0 = s_glob[bb];
      const uint64_t rlo2 = f2_pack(s_rlo[bb], s_rlo[bb]), rhi2 = f2_pack(s_rhi[bb], s_rhi[bb]);
      const uint4* src = reinterpret_cast<const uint4*>(am + local);
      uint4 a[G / 8];
#pragma unroll
      for (int i = 0; i < G / 8; ++i) a[i] = __ldg(src + i);   // all loads in flight before any arithmetic
#pragma unroll
      for (int h = 0; h < G / 16; ++h) {
        const uint32_t aw[8] = {a[2 * h].x, a[2 * h].y, a[2 * h].z, a[2 * h].w,
                                a[2 * h + 1].x, a[2 * h + 1].y, a[2 * h + 1].z, a[2 * h + 1].w};
        uint32_t out[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          out[k] = nvfp4_scale_pair(aw[2 * k], glob0, rlo2, rhi2) |
                   (nvfp4_scale_pair(aw[2 * k + 1], glob0, rlo2, rhi2) << 16);
        reinterpret_cast<uint4*>(sc + local)[h] = make_uint4(out[0], out[1], out[2], out[3]);
      }
    } else {
      for (int64_t g = g0; g < g0 + G && g < total; ++g) {
        while (bb + 1 < L.n && L.gprefix[bb + 1] <= g) ++bb;
        const int64_t lg = g - L.gprefix[bb];
        L.scales[bb][lg] = (uint8_t)nvfp4_scale_exact(L.amax[bb][lg], s_glob[bb]);
      }
    }
  }
}

cudaError_t launch_nvfp4_scales(const ScalesLaunch& L, int64_t max_groups, int num_sms, cudaStream_t stream) {
  (void)max_groups;
  const int64_t total = L.gprefix[L.n];
  int64_t blocks = (total / SCALE_GROUPS_PER_THREAD + 255) / 256;
  const int64_t cap = (int64_t)num_sms * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  nvfp4_scales_kernel<<<(unsigned)blocks, 256, 0, stream>>>(L);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// MXFP8 (export_native_compressed.py:1138-1162): lane quads form a 32-group.
// ---------------------------------------------------------------------------
// A warp takes MX_UNROLL x 32 consecutive 8-element chunks per pass and issues all its loads first
// (more bytes in flight per thread); four lanes form a 32-group.
constexpr int MX_UNROLL = 4;
__global__ void __launch_bounds__(256) mxfp8_pack_kernel(const uint16_t* __restrict__ w, int64_t n_chunks,
                                                         uint8_t* __restrict__ q, uint8_t* __restrict__ sc) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t base = gw * (32 * MX_UNROLL); base < n_chunks; base += nw * (32 * MX_UNROLL)) {
    uint4 u[MX_UNROLL];
#pragma unroll
    for (int j = 0; j < MX_UNROLL; ++j) {
      const int64_t c = base + 32 * j + lane;
      u[j] = c < n_chunks ? __ldg(reinterpret_cast<const uint4*>(w) + c) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < MX_UNROLL; ++j) {
      const int64_t c = base + 32 * j + lane;
      float v[8];
      unpack8(u[j], v);
      float a = amax8(v);
      a = fmaxf(a, __shfl_xor_sync(FULL, a, 1));
      a = fmaxf(a, __shfl_xor_sync(FULL, a, 2));
      if (c >= n_chunks) continue;
      const float s = __fdiv_rn(fmaxf(a, pow2i(-127)), 448.0f);  // amax.clamp_min(2^-127) / 448
      const int e = e8m0_ceil(s);
      const float inv = pow2i(-e);  // w / 2^e, exact
      uint32_t out[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        uint32_t word = 0;
#pragma unroll
        for (int i = 0; i < 4; i += 2) {
          const float x0 = fminf(fmaxf(__fmul_rn(v[4 * k + i], inv), -448.0f), 448.0f);
          const float x1 = fminf(fmaxf(__fmul_rn(v[4 * k + i + 1], inv), -448.0f), 448.0f);
          word |= e4m3x2(x0, x1) << (8 * i);
        }
        out[k] = word;
      }
      reinterpret_cast<uint2*>(q)[c] = make_uint2(out[0], out[1]);
      if ((lane & 3) == 0) sc[c >> 2] = (uint8_t)(e + 127);
    }
  }
}

cudaError_t launch_mxfp8_pack(const uint16_t* w, int64_t n_elems, uint8_t* q, uint8_t* sc, int num_sms,
                              cudaStream_t stream) {
  const int64_t n_chunks = n_elems / 8;
  mxfp8_pack_kernel<<<grid_for(n_chunks / (32 * MX_UNROLL) + 1, num_sms), 256, 0, stream>>>(w, n_chunks, q, sc);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// FP8 per-channel (export_native_compressed.py:1197-1226): warp per row, row
// amax then w / s (IEEE division), clamp, E4M3 RNE.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) fp8_channel_kernel(const uint16_t* __restrict__ w, int64_t rows, int64_t cols,
                                                          uint8_t* __restrict__ q, float* __restrict__ scale) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const bool vec = (cols & 7) == 0;
  for (int64_t r = gw; r < rows; r += nw) {
    const uint16_t* row = w + r * cols;
    float a = 0.0f;
    if (vec) {
      const uint4* rv = reinterpret_cast<const uint4*>(row);
      for (int64_t c = lane; c < cols / 8; c += 32) {
        float v[8];
        unpack8(__ldg(rv + c), v);
        a = fmaxf(a, amax8(v));
      }
    } else {
      for (int64_t i = lane; i < cols; i += 32) a = fmaxf(a, fabsf(__uint_as_float((uint32_t)__ldg(row + i) << 16)));
    }
    a = __uint_as_float(warp_max_u(__float_as_uint(a)));
    const float s = __fdiv_rn(fmaxf(a, pow2i(-127)), 448.0f);
    if (lane == 0) scale[r] = s;
    uint8_t* qrow = q + r * cols;
    if (vec) {
      const uint4* rv = reinterpret_cast<const uint4*>(row);
      for (int64_t c = lane; c < cols / 8; c += 32) {
        float v[8];
        unpack8(__ldg(rv + c), v);
        uint32_t out[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          uint32_t word = 0;
#pragma unroll
          for (int i = 0; i < 4; i += 2) {
            const float x0 = fminf(fmaxf(__fdiv_rn(v[4 * k + i], s), -448.0f), 448.0f);
            const float x1 = fminf(fmaxf(__fdiv_rn(v[4 * k + i + 1], s), -448.0f), 448.0f);
            word |= e4m3x2(x0, x1) << (8 * i);
          }
          out[k] = word;
        }
        reinterpret_cast<uint2*>(qrow)[c] = make_uint2(out[0], out[1]);
      }
    } else {
      for (int64_t i = lane; i < cols; i += 32) {
        const float x = __fdiv_rn(__uint_as_float((uint32_t)__ldg(row + i) << 16), s);
        qrow[i] = (uint8_t)e4m3_byte(fminf(fmaxf(x, -448.0f), 448.0f));
      }
    }
  }
}

cudaError_t launch_fp8_channel_pack(const uint16_t* w, int64_t rows, int64_t cols, uint8_t* q, float* scale,
                                    int num_sms, cudaStream_t stream) {
  fp8_channel_kernel<<<grid_for(rows, num_sms), 256, 0, stream>>>(w, rows, cols, q, scale);
  return cudaGetLastError();
}

}  // namespace pq
