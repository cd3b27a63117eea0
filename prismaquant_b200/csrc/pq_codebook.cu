// Exact cost-path quantize-dequantize for the rest of the format registry
// (MXFP4, MXFP6 E3M2/E2M3, MXFP8/FP8 E5M2, NVFP3, the symmetric INT formats,
// and E4M3 with real per-128 scales), first-principles arithmetic:
//
//  * codebook formats follow _rtn_fp_codebook (format_registry.py:194-233):
//    scale = max(amax, 1e-8) / cmax (E8M0-snapped for the MX family),
//    x = fl(w / scale), x placed in the sorted signed codebook as
//    torch.bucketize does (first entry >= x), the neighbour chosen only when
//    strictly closer in float32 (ties to the lower value), W_hat = bf16(q * scale);
//  * integer formats follow _rtn_uniform_int, symmetric (format_registry.py:147-172):
//    scale = max(amax, 1e-8) / (2^(b-1) - 1), q = round_half_even(w / scale)
//    clamped to [-2^(b-1), 2^(b-1) - 1], W_hat = bf16(q * scale).
//
// The codebooks are generated from the same definitions as the reference's
// (format_registry.py:237-300): FP6 and FP3 have no subnormals, and the E5M2
// codebook keeps exponent 31 as finite values (largest magnitude 114688).
// These formats are not on the fused hot path; one warp per row is plenty.
// The same kernel (which can also describe NVFP4, MXFP8 and FP8 per channel)
// computes the H-weighted error sum behind predicted_dloss.
#include <type_traits>
#include "pq_common.cuh"
#include "pq_internal.h"

namespace pq {

enum CodebookId { CB_E2M1 = 0, CB_E3M2, CB_E2M3, CB_E2M0, CB_E4M3, CB_E5M2 };

struct XFmt {
  bool is_int;
  int cb;      // codebook (is_int == false)
  int bits;    // integer width (is_int == true)
  int group;   // 0: one group per row
  bool mx;     // E8M0-snapped scale
};

__host__ __device__ inline bool xfmt_known(int fmt) { return fmt >= PQ_FMT_MXFP4 && fmt < PQ_NUM_FMTS_ALL; }
// Formats this kernel can score (the fused-sweep ones too, for the weighted sum).
__host__ __device__ inline bool xfmt_scorable(int fmt) {
  return fmt == PQ_FMT_NVFP4 || fmt == PQ_FMT_MXFP8 || fmt == PQ_FMT_FP8_CHANNEL || xfmt_known(fmt);
}

// format_registry.py:391-533 and measure_quant_cost.py:516-548 (FP8_SOURCE's batched form)
__host__ __device__ inline XFmt xfmt_of(int fmt) {
  switch (fmt) {
    case PQ_FMT_NVFP4: return {false, CB_E2M1, 0, 16, false};
    case PQ_FMT_MXFP8: return {false, CB_E4M3, 0, 32, true};
    case PQ_FMT_FP8_CHANNEL: return {false, CB_E4M3, 0, 0, false};
    case PQ_FMT_MXFP4: return {false, CB_E2M1, 0, 32, true};
    case PQ_FMT_MXFP6_E3M2: return {false, CB_E3M2, 0, 32, true};
    case PQ_FMT_MXFP6_E2M3: return {false, CB_E2M3, 0, 32, true};
    case PQ_FMT_MXFP8_E5M2: return {false, CB_E5M2, 0, 32, true};
    case PQ_FMT_FP8_E5M2: return {false, CB_E5M2, 0, 0, false};
    case PQ_FMT_NVFP3: return {false, CB_E2M0, 0, 16, false};
    case PQ_FMT_INT3: return {true, 0, 3, 16, false};
    case PQ_FMT_INT2: return {true, 0, 2, 16, false};
    case PQ_FMT_INT8_CHANNEL: return {true, 0, 8, 0, false};
    case PQ_FMT_INT4_G128: return {true, 0, 4, 128, false};
    default: return {false, CB_E4M3, 0, 128, false};   // PQ_FMT_FP8_E4M3_G128
  }
}

// Ascending non-negative magnitudes of a codebook (mags[0] = 0); returns their count.
__device__ int codebook_magnitudes(int cb, float* mags) {
  int n = 0;
  mags[n++] = 0.0f;
  switch (cb) {
    case CB_E2M1: {
      const float v[7] = {0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
      for (int i = 0; i < 7; ++i) mags[n++] = v[i];
      break;
    }
    case CB_E3M2:   // (1 + m/4) 2^(e-3), e = 0..7
      for (int e = 0; e < 8; ++e)
        for (int m = 0; m < 4; ++m) mags[n++] = ldexpf(1.0f + 0.25f * m, e - 3);
      break;
    case CB_E2M3:   // (1 + m/8) 2^(e-1), e = 0..3
      for (int e = 0; e < 4; ++e)
        for (int m = 0; m < 8; ++m) mags[n++] = ldexpf(1.0f + 0.125f * m, e - 1);
      break;
    case CB_E2M0:   // 2^(e-2), e = 0..3
      for (int e = 0; e < 4; ++e) mags[n++] = ldexpf(1.0f, e - 2);
      break;
    case CB_E4M3:   // subnormals m/8 2^-6, then (1 + m/8) 2^(e-7) up to 448
      for (int m = 1; m < 8; ++m) mags[n++] = ldexpf(0.125f * m, -6);
      for (int e = 1; e < 16; ++e)
        for (int m = 0; m < 8; ++m) {
          const float v = ldexpf(1.0f + 0.125f * m, e - 7);
          if (v <= 448.0f) mags[n++] = v;
        }
      break;
    default:        // CB_E5M2: subnormals m/4 2^-14, then (1 + m/4) 2^(e-15), e = 1..31
      for (int m = 1; m < 4; ++m) mags[n++] = ldexpf(0.25f * m, -14);
      for (int e = 1; e < 32; ++e)
        for (int m = 0; m < 4; ++m) mags[n++] = ldexpf(1.0f + 0.25f * m, e - 15);
      break;
  }
  return n;
}

constexpr int XCB_MAX = 256;   // signed codebook entries (E5M2: 255)

// Reconstruction of one element.  cb / ncb: sorted signed codebook.
__device__ __forceinline__ float xfmt_rec(const XFmt& f, const float* cb, int ncb, float w, float scale) {
  const float x = __fdiv_rn(w, scale);
  float q;
  if (f.is_int) {
    const float lv = (float)((1 << (f.bits - 1)) - 1);
    q = fminf(fmaxf(rintf(x), -lv - 1.0f), lv);
  } else {
    int lo = 0, hi = ncb;   // first entry >= x (torch.bucketize, right=False)
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (cb[mid] < x) lo = mid + 1; else hi = mid;
    }
    const float a = cb[max(lo - 1, 0)], b = cb[min(lo, ncb - 1)];
    q = fabsf(__fsub_rn(b, x)) < fabsf(__fsub_rn(x, a)) ? b : a;
  }
  return bf16_round(__fmul_rn(q, scale));
}

__device__ __forceinline__ float xfmt_scale(const XFmt& f, float cmax, float amax) {
  const float a = fmaxf(amax, 1e-8f);
  if (f.is_int) return __fdiv_rn(a, (float)((1 << (f.bits - 1)) - 1));
  const float s = __fdiv_rn(a, cmax);
  return f.mx ? pow2i(e8m0_round(s)) : s;   // s >= 1e-8 / 114688: normal, never clamped
}

// h_mode: 0 unweighted, 1 one weight per element ([rows, cols]), 2 one weight per row.
template <int MODE>
__global__ void __launch_bounds__(256) xfmt_kernel(const uint16_t* __restrict__ w, int64_t rows, int64_t cols,
                                                   int fmt, double* sse, uint16_t* out, const float* __restrict__ h,
                                                   int h_mode) {
  __shared__ float cb[XCB_MAX];
  __shared__ float mags[XCB_MAX / 2 + 1];
  __shared__ int s_ncb;
  __shared__ float s_cmax;
  const XFmt f = xfmt_of(fmt);
  if (threadIdx.x == 0) {
    int ncb = 0;
    float cmax = 0.0f;
    if (!f.is_int) {
      const int nm = codebook_magnitudes(f.cb, mags);
      for (int k = nm - 1; k >= 1; --k) cb[ncb++] = -mags[k];
      for (int k = 0; k < nm; ++k) cb[ncb++] = mags[k];
      cmax = mags[nm - 1];
    }
    s_ncb = ncb;
    s_cmax = cmax;
  }
  __syncthreads();
  const int ncb = s_ncb;
  const float cmax = s_cmax;

  const int lane = threadIdx.x & 31;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t g = (f.group > 0 && f.group < cols) ? f.group : cols;
  double acc = 0.0;
  float part = 0.0f;
  int nsq = 0;
  auto emit = [&](int64_t idx, float wi, float r) {
    if (MODE == MODE_QDQ) out[idx] = (uint16_t)(__float_as_uint(r) >> 16);
    const float e = bf16_round(__fsub_rn(wi, r));
    const float e2 = __fmul_rn(e, e);   // the reference squares in fp32, then weights
    part = h_mode == 0 ? __fadd_rn(part, e2)
                       : fmaf(h_mode == 1 ? __ldg(h + idx) : __ldg(h + idx / cols), e2, part);
    if (++nsq == 64) {   // fp32 partials hold <= 64 exact squares
      acc += (double)part;
      part = 0.0f;
      nsq = 0;
    }
  };
  for (int64_t r = gw; r < rows; r += nw) {
    const uint16_t* row = w + r * cols;
    if (g == cols) {   // one group per row: the warp reduces the row maximum
      float ar = 0.0f;
      for (int64_t i = lane; i < cols; i += 32) ar = fmaxf(ar, fabsf(bf16lo((uint32_t)row[i])));
      ar = __uint_as_float(warp_max_u(__float_as_uint(ar)));
      const float scale = xfmt_scale(f, cmax, ar);
      for (int64_t i = lane; i < cols; i += 32) {
        const float wi = bf16lo((uint32_t)row[i]);
        emit(r * cols + i, wi, xfmt_rec(f, cb, ncb, wi, scale));
      }
    } else {           // lanes take whole groups
      for (int64_t gi = lane; gi < cols / g; gi += 32) {
        const uint16_t* gp = row + gi * g;
        float a = 0.0f;
        for (int64_t i = 0; i < g; ++i) a = fmaxf(a, fabsf(bf16lo((uint32_t)gp[i])));
        const float scale = xfmt_scale(f, cmax, a);
        for (int64_t i = 0; i < g; ++i) {
          const float wi = bf16lo((uint32_t)gp[i]);
          emit(r * cols + gi * g + i, wi, xfmt_rec(f, cb, ncb, wi, scale));
        }
      }
    }
  }
  if (MODE == MODE_SSE) {
    const double v = warp_sum_d(acc + (double)part);
    if (lane == 0 && v != 0.0) atomicAdd(sse, v);
  }
}

// ---------------------------------------------------------------------------
// Coalesced kernel for rows of a multiple of 8 elements (16-byte aligned): each lane takes 8
// consecutive elements with one 16-byte load; the lanes of a 16/32/128-group reduce its maximum
// with shuffles (row-wise formats: the warp, over the row).  The rounding is closed-form:
// the codebook RTN above (bucketize, then the strictly closer neighbour) is the nearest codebook
// value with ties to the lower signed value, saturated at the largest magnitude, because the
// reference's two float32 differences are exact wherever they can decide (adjacent entries are
// within a factor of two, Sterbenz), so grid_round_abs gives the same point.  The FP6 / FP3
// codebooks have no subnormals: below their smallest normal 2^EMIN they hold only 0, with the
// tie at 2^(EMIN-1).  MX scales are powers of two, so w / scale is the exact product
// w * 2^-e.
// ---------------------------------------------------------------------------
enum XKind { XK_E2M1 = 0, XK_E3M2, XK_E2M3, XK_E2M0, XK_E4M3, XK_E5M2, XK_INT };

template <int KIND> struct XK;
template <> struct XK<XK_E2M1> { static constexpr int M = 1, EMIN = 0; static constexpr bool SUB = true; static constexpr float MAXV = 6.0f; };
template <> struct XK<XK_E3M2> { static constexpr int M = 2, EMIN = -3; static constexpr bool SUB = false; static constexpr float MAXV = 28.0f; };
template <> struct XK<XK_E2M3> { static constexpr int M = 3, EMIN = -1; static constexpr bool SUB = false; static constexpr float MAXV = 7.5f; };
template <> struct XK<XK_E2M0> { static constexpr int M = 0, EMIN = -2; static constexpr bool SUB = false; static constexpr float MAXV = 2.0f; };
template <> struct XK<XK_E4M3> { static constexpr int M = 3, EMIN = -6; static constexpr bool SUB = true; static constexpr float MAXV = 448.0f; };
template <> struct XK<XK_E5M2> { static constexpr int M = 2, EMIN = -14; static constexpr bool SUB = true; static constexpr float MAXV = 114688.0f; };

__host__ __device__ inline int xkind_of(const XFmt& f) {
  if (f.is_int) return XK_INT;
  switch (f.cb) {
    case CB_E2M1: return XK_E2M1;
    case CB_E3M2: return XK_E3M2;
    case CB_E2M3: return XK_E2M3;
    case CB_E2M0: return XK_E2M0;
    case CB_E4M3: return XK_E4M3;
    default: return XK_E5M2;
  }
}

// Cost-path RTN of x on the format's grid (codebook: ties to the lower value, +0.0 for a
// negative x that rounds to zero; integer: round half even, then clamp).
template <int KIND>
__device__ __forceinline__ float xk_round(float x, int bits) {
  if constexpr (KIND == XK_INT) {
    const float lv = (float)((1 << (bits - 1)) - 1);
    return fminf(fmaxf(rintf(x), -lv - 1.0f), lv);
  } else {
    using K = XK<KIND>;
    const float a = fabsf(x);
    const bool neg = x < 0.0f;
    float r = grid_round_abs<K::M, K::EMIN>(a, neg, K::MAXV);
    if constexpr (!K::SUB) {
      const float lo = K::EMIN >= 0 ? (float)(1 << K::EMIN) : 1.0f / (float)(1 << -K::EMIN);
      const float half = 0.5f * lo;
      const float rs = (a > half || (a == half && neg)) ? lo : 0.0f;
      r = a < lo ? rs : r;
    }
    return neg ? __fsub_rn(0.0f, r) : r;
  }
}

// MX reconstruction of 8 elements without the generic rounding, for a group scale 2^es with
// |es| <= 100 and no NaN among the 8 (w holds their bf16 bits, wv their values):
//  - |w| >= 2^(EMIN+es) (the format's normal range): the grid point is w rounded to M mantissa
//    bits, ties to the lower signed value (up in magnitude for a negative w), saturated at
//    MAXV 2^es — integer arithmetic on the bf16 magnitudes, two per word (a magnitude plus the
//    rounding increment stays below 0x10000, so no carry crosses into the other half);
//  - |w| < 2^(EMIN+es): t = |w| + 2^(EMIN+es) lies in the binade of 2^(EMIN+es), and t rounded
//    to MS mantissa bits (MS = M with subnormals, 0 without: then only 0 and 2^EMIN) minus
//    2^(EMIN+es) is the grid point.  The sum is exact wherever it can reach a rounding
//    boundary (|w| >= 2^(EMIN+es-4) there); a smaller |w| rounds to 0 either way.
// Every grid point times 2^es is a bf16, so this is bf16(q 2^es) of the generic rule, with +0 for
// a negative w that rounds to zero.
template <int KIND>
__device__ __forceinline__ void mx_rec8(const uint4& u, const float (&wv)[8], int es, float (&rec)[8]) {
  using K = XK<KIND>;
  constexpr int MS = K::SUB ? K::M : 0;
  constexpr uint32_t DROP = 7 - K::M;
  constexpr uint32_t HALF = ((1u << (DROP - 1)) - 1u) * 0x00010001u;
  constexpr uint32_t MASK = ((0xFFFFu >> DROP) << DROP) * 0x00010001u;
  constexpr uint32_t HALF32 = (1u << (22 - MS)) - 1u;
  constexpr uint32_t MASK32 = ~((1u << (23 - MS)) - 1u);
  const float cw = pow2i(K::EMIN + es);
  const uint32_t satb = (__float_as_uint(K::MAXV) >> 16) + ((uint32_t)es << 7);
  const uint32_t sat2 = (satb & 0xFFFFu) * 0x00010001u;
  const uint32_t words[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t v = words[p];
    const uint32_t neg = (v >> 15) & 0x00010001u;
    const uint32_t m = __vminu2(((v & 0x7FFF7FFFu) + HALF + neg) & MASK, sat2);
    const float big[2] = {__uint_as_float(m << 16), __uint_as_float(m & 0xFFFF0000u)};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = 2 * p + h;
      const float a = fabsf(wv[i]);
      const uint32_t ng = (v >> (15 + 16 * h)) & 1u;
      const float t = __fadd_rn(a, cw);
      const float small = __fsub_rn(__uint_as_float((__float_as_uint(t) + HALF32 + ng) & MASK32), cw);
      const float mag = a < cw ? small : big[h];
      rec[i] = ng ? __fsub_rn(0.0f, mag) : mag;
    }
  }
}

// NaN among 8 bf16 values: a magnitude above 0x7F80 in some half
__device__ __forceinline__ bool has_nan8(const uint4& u) {
  const uint32_t t = (((u.x & 0x7FFF7FFFu) + 0x007F007Fu) | ((u.y & 0x7FFF7FFFu) + 0x007F007Fu) |
                      ((u.z & 0x7FFF7FFFu) + 0x007F007Fu) | ((u.w & 0x7FFF7FFFu) + 0x007F007Fu));
  return (t & 0x80008000u) != 0u;
}

template <int MODE, int KIND>
__global__ void __launch_bounds__(256) xfmt2_kernel(const uint16_t* __restrict__ w, int64_t rows, int64_t cols,
                                                    int fmt, double* sse, uint16_t* out,
                                                    const float* __restrict__ h, int h_mode) {
  const XFmt f = xfmt_of(fmt);
  const float cmax = KIND == XK_INT ? 0.0f : XK<(KIND == XK_INT ? XK_E2M1 : KIND)>::MAXV;
  const int lane = threadIdx.x & 31;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const bool grouped = f.group > 0 && f.group < cols;
  constexpr bool MXK = KIND != XK_INT && KIND != XK_E2M0;   // kinds some MX format uses
  double acc = 0.0;

  // scale of a group with maximum a, and the factor x = w * inv or w / scale
  auto scale_of = [&](float a, float& inv) {
    const float s = xfmt_scale(f, cmax, a);
    inv = (!f.is_int && f.mx) ? __frcp_rn(s) : 0.0f;   // exact: s is a power of two
    return s;
  };
  // 8 elements at flat index idx (row r): reconstruction, error, optional W_hat store
  // fast: MX group in range, reconstructions by mx_rec8, whose errors w - rec are bf16 already
  auto do8 = [&](const uint4& u, const float (&wv)[8], int64_t idx, int64_t r, float scale, float inv,
                 auto fast) {
    constexpr bool FAST = decltype(fast)::value;
    float hv[8];
    if (h_mode == 1) {
      const float4 h0 = __ldg(reinterpret_cast<const float4*>(h + idx));
      const float4 h1 = __ldg(reinterpret_cast<const float4*>(h + idx + 4));
      hv[0] = h0.x; hv[1] = h0.y; hv[2] = h0.z; hv[3] = h0.w;
      hv[4] = h1.x; hv[5] = h1.y; hv[6] = h1.z; hv[7] = h1.w;
    } else {
      const float hr = h_mode == 2 ? __ldg(h + r) : 1.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) hv[i] = hr;
    }
    float part = 0.0f;
    uint32_t o[4];
    float recv[8];
    if constexpr (FAST && KIND != XK_INT) {
      mx_rec8<(KIND == XK_INT ? XK_E2M1 : KIND)>(u, wv, (int)(__float_as_uint(scale) >> 23) - 127, recv);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float x = inv != 0.0f ? __fmul_rn(wv[i], inv) : __fdiv_rn(wv[i], scale);
        recv[i] = bf16_round(__fmul_rn(xk_round<KIND>(x, f.bits), scale));
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float rec = recv[i];
      const float e = FAST ? __fsub_rn(wv[i], rec) : bf16_round(__fsub_rn(wv[i], rec));
      const float e2 = __fmul_rn(e, e);   // the reference squares in fp32, then weights
      part = h_mode == 0 ? __fadd_rn(part, e2) : fmaf(hv[i], e2, part);
      if (MODE == MODE_QDQ) {
        const uint32_t b = __float_as_uint(rec) >> 16;
        o[i >> 1] = (i & 1) ? (o[i >> 1] | (b << 16)) : b;
      }
    }
    if (MODE == MODE_QDQ) *reinterpret_cast<uint4*>(out + idx) = make_uint4(o[0], o[1], o[2], o[3]);
    acc += (double)part;   // fp32 partials of 8 exact squares
  };

  if (grouped) {
    // warps take 256-element chunks of rows; a group (16/32/128 | 256) lies in one chunk
    const int64_t cpr = (cols + 255) / 256;
    const int gl = (int)(f.group >> 3);   // lanes per group: 2, 4 or 16
    for (int64_t c = gw; c < rows * cpr; c += nw) {
      const int64_t r = c / cpr;
      const int64_t col = (c - r * cpr) * 256 + lane * 8;
      const bool valid = col < cols;      // cols % group == 0: a group is all valid or all not
      uint4 u = make_uint4(0, 0, 0, 0);
      if (valid) u = __ldg(reinterpret_cast<const uint4*>(w + r * cols + col));
      float wv[8];
      unpack8(u, wv);
      float a = amax8(wv);
      for (int o = 1; o < gl; o <<= 1) a = fmaxf(a, __shfl_xor_sync(FULL, a, o));
      float inv;
      const float scale = scale_of(a, inv);
      if (valid) {
        // an MX group in range with no NaN among the lane's 8 takes the integer reconstruction
        if (MXK && f.mx && scale >= 0x1p-100f && scale <= 0x1p100f && !has_nan8(u))
          do8(u, wv, r * cols + col, r, scale, inv, std::true_type{});
        else
          do8(u, wv, r * cols + col, r, scale, inv, std::false_type{});
      }
    }
  } else {
    // one scale per row: the warp reduces the row maximum, then scores the row
    for (int64_t r = gw; r < rows; r += nw) {
      const uint16_t* row = w + r * cols;
      float a = 0.0f;
      for (int64_t col = lane * 8; col < cols; col += 256) {
        float wv[8];
        unpack8(__ldg(reinterpret_cast<const uint4*>(row + col)), wv);
        a = fmaxf(a, amax8(wv));
      }
      a = __uint_as_float(warp_max_u(__float_as_uint(a)));
      float inv;
      const float scale = scale_of(a, inv);
      for (int64_t col = lane * 8; col < cols; col += 256) {
        float wv[8];
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(row + col));
        unpack8(u, wv);
        do8(u, wv, r * cols + col, r, scale, inv, std::false_type{});
      }
    }
  }
  if (MODE == MODE_SSE) {
    const double v = warp_sum_d(acc);
    if (lane == 0 && v != 0.0) atomicAdd(sse, v);
  }
}

template <int MODE>
static void launch_xfmt2_mode(int kind, unsigned blocks, const uint16_t* w, int64_t rows, int64_t cols, int fmt,
                              double* sse, uint16_t* out, const float* h, int h_mode, cudaStream_t stream) {
  switch (kind) {
#define PQ_XK_CASE(K) \
    case K: xfmt2_kernel<MODE, K><<<blocks, 256, 0, stream>>>(w, rows, cols, fmt, sse, out, h, h_mode); break;
    PQ_XK_CASE(XK_E2M1)
    PQ_XK_CASE(XK_E3M2)
    PQ_XK_CASE(XK_E2M3)
    PQ_XK_CASE(XK_E2M0)
    PQ_XK_CASE(XK_E4M3)
    PQ_XK_CASE(XK_E5M2)
    default: xfmt2_kernel<MODE, XK_INT><<<blocks, 256, 0, stream>>>(w, rows, cols, fmt, sse, out, h, h_mode); break;
#undef PQ_XK_CASE
  }
}

// Group length the format uses for rows of `cols`, or 0 if the row does not split into groups
// (the reference's reshape raises, format_registry.py:208-212 / :151-154).
int64_t xfmt_group(int fmt, int64_t cols) {
  const XFmt f = xfmt_of(fmt);
  if (f.group > 0 && f.group < cols) return cols % f.group ? 0 : f.group;
  return cols;
}

cudaError_t launch_xfmt(const uint16_t* w, int64_t rows, int64_t cols, int fmt, double* sse, uint16_t* out,
                        int mode, int num_sms, cudaStream_t stream, const float* h, int h_mode) {
  const auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (cols % 8 == 0 && al16(w) && (mode != MODE_QDQ || al16(out)) && (h_mode != 1 || al16(h))) {
    const XFmt f = xfmt_of(fmt);
    const int64_t work = (f.group > 0 && f.group < cols) ? rows * ((cols + 255) / 256) : rows;   // warp tasks
    int64_t blocks2 = (work + 7) / 8;
    if (blocks2 > (int64_t)num_sms * 8) blocks2 = (int64_t)num_sms * 8;
    if (blocks2 < 1) blocks2 = 1;
    if (mode == MODE_QDQ)
      launch_xfmt2_mode<MODE_QDQ>(xkind_of(f), (unsigned)blocks2, w, rows, cols, fmt, sse, out, h, h_mode, stream);
    else
      launch_xfmt2_mode<MODE_SSE>(xkind_of(f), (unsigned)blocks2, w, rows, cols, fmt, sse, out, h, h_mode, stream);
    return cudaGetLastError();
  }
  int64_t blocks = (rows * 32 + 255) / 256;
  if (blocks > (int64_t)num_sms * 8) blocks = (int64_t)num_sms * 8;
  if (blocks < 1) blocks = 1;
  if (mode == MODE_QDQ)
    xfmt_kernel<MODE_QDQ><<<(unsigned)blocks, 256, 0, stream>>>(w, rows, cols, fmt, sse, out, h, h_mode);
  else
    xfmt_kernel<MODE_SSE><<<(unsigned)blocks, 256, 0, stream>>>(w, rows, cols, fmt, sse, out, h, h_mode);
  return cudaGetLastError();
}

}  // namespace pq
