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
#include "pq_fast.cuh"
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
    q = x != x ? x : fminf(fmaxf(rintf(x), -lv - 1.0f), lv);   // torch.clamp keeps a NaN
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
    if (MODE == MODE_QDQ) out[idx] = (uint16_t)bf16_bits_torch(r);
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
    return x != x ? x : fminf(fmaxf(rintf(x), -lv - 1.0f), lv);   // torch.clamp keeps a NaN
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

// Squared error of 8 elements of an MX group (one 16-byte word of bf16 pairs) with scale 2^es,
// |es| <= 100, no NaN among them, on packed bf16 pairs (cost path only: at a tie both grid
// neighbours are equally far, so the tie rule does not change the squared error):
//  - |w| >= 2^(EMIN+es): the magnitude rounded to M mantissa bits on the bit pattern (half up; a
//    finite bf16 half never carries into its sign bit or the other half), saturated at
//    MAXV 2^es by a packed magnitude min;
//  - |w| <= 2^(EMIN+es): w rounded on the grid of step 2^(EMIN+es-MS) (MS = M with subnormals,
//    0 without, where the grid below 2^EMIN is {0, 2^EMIN}) by adding and subtracting
//    C = 1.5 x 2^(step + 7) in bf16 arithmetic: w + C stays in C's binade, whose spacing is the
//    step, and the subtraction is exact;
//  - the range test is a packed subtraction 0x8000 + bits(2^(EMIN+es)) - |w| per half, whose bit
//    15 is set iff |w| <= 2^(EMIN+es) (no borrow crosses halves), spread over the half by a
//    sign-replicating byte permute.
// The error w - q is exact in bf16 (q is w rounded within its binade, or the saturation value
// one binade below a larger w, or a grid point within 2^(EMIN+es) of a subnormal-range w), so
// its square is exact in fp32.  Returns the fp32 sum of the 8 squares.
template <int KIND>
__device__ __forceinline__ float mx_sse8(const uint4& u, int es) {
  using K = XK<KIND>;
  constexpr int MS = K::SUB ? K::M : 0;
  constexpr uint32_t DROP = 7 - K::M;
  constexpr uint32_t HALFUP = (1u << (DROP - 1)) * 0x00010001u;
  constexpr uint32_t MASK = ((0xFFFFu >> DROP) << DROP) * 0x00010001u;
  const uint32_t sat2 = ((__float_as_uint(K::MAXV) >> 16) + ((uint32_t)es << 7)) * 0x00010001u;
  const uint32_t lo = (uint32_t)(K::EMIN + es + 127) << 7;                       // bits of 2^(EMIN+es)
  const uint32_t thr2 = (0x8000u + lo) * 0x00010001u;
  const uint32_t c2 = ((((uint32_t)(K::EMIN + es - MS + 7 + 127)) << 7) | 0x40u) * 0x00010001u;   // 1.5 x 2^(step+7)
  const uint32_t words[4] = {u.x, u.y, u.z, u.w};
  float acc = 0.0f;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t v = words[p];
    const uint32_t qn = bf16x2_minabs((v + HALFUP) & MASK, sat2);
    const uint32_t qs = bf16x2_sub(bf16x2_add(v, c2), c2);
    const uint32_t m = prmt_sign_halves(thr2 - (v & 0x7FFF7FFFu));   // 0xFFFF where |w| <= 2^(EMIN+es)
    acc = sq2_acc(bf16x2_sub(v, (qs & m) | (qn & ~m)), acc);
  }
  return acc;
}

// W_hat of 8 elements of an MX group (one 16-byte word of bf16 pairs) with scale 2^es, |es| <= 90,
// no NaN among them, as four bf16 pairs: the grid points of mx_rec8 with the reference's tie rule
// (ties to the lower signed value, +0 for a negative w that rounds to zero), two per step:
//  - |w| >= 2^(EMIN+es): the magnitude rounded to M mantissa bits on the bit pattern with the
//    sign-dependent tie increment of mx_rec8, saturated at MAXV 2^es by a packed unsigned min,
//    the sign put back;
//  - |w| <= 2^(EMIN+es): w - eps rounded to a multiple of step = 2^(EMIN+es-MS) by adding and
//    subtracting c = 1.5 x 2^(step+23) in float32 pairs, eps = step x 2^-11.  Where w can reach
//    a half-step, w and eps are multiples of step x 2^-11 below 8 step, so w - eps is exact; a
//    bf16 w that is not a tie lies at least step x 2^-8 from the half-step, so it stays on its
//    side, and a tie moves to the lower neighbour; a zero result is c - c = +0.  |es| <= 90
//    keeps c and eps normal float32 numbers;
//  - the range mask is mx_sse8's packed subtraction (both sides agree at |w| = 2^(EMIN+es)).
template <int KIND>
__device__ __forceinline__ void mx_qdq8(const uint4& u, int es, uint32_t (&o)[4]) {
  using K = XK<KIND>;
  constexpr int MS = K::SUB ? K::M : 0;
  constexpr uint32_t DROP = 7 - K::M;
  constexpr uint32_t HALF = ((1u << (DROP - 1)) - 1u) * 0x00010001u;
  constexpr uint32_t MASK = ((0xFFFFu >> DROP) << DROP) * 0x00010001u;
  const uint32_t sat2 = ((__float_as_uint(K::MAXV) >> 16) + ((uint32_t)es << 7)) * 0x00010001u;
  const uint32_t thr2 = (0x8000u + ((uint32_t)(K::EMIN + es + 127) << 7)) * 0x00010001u;
  const int sexp = K::EMIN + es - MS;
  const float c = __uint_as_float(((uint32_t)(sexp + 23 + 127) << 23) | 0x400000u);
  const float eps = __uint_as_float((uint32_t)(sexp - 11 + 127) << 23);
  const uint64_t c2 = f2_pack(c, c), nc2 = f2_pack(-c, -c), neps2 = f2_pack(-eps, -eps);
  const uint32_t words[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t v = words[p];
    const uint32_t neg = (v >> 15) & 0x00010001u;
    const uint32_t qn = __vminu2(((v & 0x7FFF7FFFu) + HALF + neg) & MASK, sat2) | (v & 0x80008000u);
    const uint64_t t = f2_add_rn(f2_add_rn(f2_add_rn(f2_from_bf16x2(v), neps2), c2), nc2);
    const uint32_t qs = f2_to_bf16x2(t);
    const uint32_t m = prmt_sign_halves(thr2 - (v & 0x7FFF7FFFu));   // 0xFFFF where |w| <= 2^(EMIN+es)
    o[p] = (qs & m) | (qn & ~m);
  }
}

// NVFP3 (the E2M0 codebook {0, 1/4, 1/2, 1, 2} with a real scale per 16 elements;
// format_registry.py:264-272, 505-514) without division.  s = fl32(a / 2) with
// a = max(amax, 1e-8) is a / 2 exactly, so the nearest codebook point of fl32(w / s) is decided by
// comparing |w| with the midpoints times s: a/16, 3a/16, 3a/8 and 3a/4.  For a bf16 a
// (amax >= 1e-8) the quotient 2w/a is either exactly such a midpoint or at least 2^-13 (relative)
// away from it, so fl32 rounding never moves it across or onto one, and the exact comparisons are
// the reference's.  On bf16 bit patterns, |w| > t is
// bits(|w|) > bits(RD(t)), and |w| >= t is bits(|w|) + 1 > bits(t) when t is a bf16, else
// bits(|w|) > bits(RD(t)); a/16 is always a bf16, the three 3a thresholds are together or not.
// Ties go to the lower signed value: up in magnitude (>=) for a negative w, down (>) for a
// positive one.  The level gives |W_hat| = 0, a/8, a/4, a/2 or a (bf16 values); the error
// |w| - |W_hat| has the reference's square.  Used by fp3sse_kernel (squared error) and by
// xfmt2_kernel (W_hat) for groups whose maximum is at least 1e-8 and below 2^126 (so that 3a
// is finite).
constexpr uint32_t BF16_1EM8_CEIL = 0x322Cu;   // the smallest bf16 magnitude >= 1e-8f
constexpr uint32_t FP3_FAST_CEIL = 0x7E80u;    // group maxima below 2^126 keep 3a finite

struct Fp3Group {
  uint32_t k[4];   // 0x7FFF - bits(RD(threshold k)) per half: bit 15 of mag' + k[i] is mag' > RD
  uint32_t ex;     // 0x00010001 where the 3a thresholds are bf16 values, else 0
  uint32_t r[4];   // |W_hat| bits per half at levels 1..4: a/8, a/4, a/2, a
};

__device__ __forceinline__ Fp3Group fp3_group(uint32_t ab) {   // ab: bits of amax, 1e-8 <= amax < 2^126
  const uint32_t t3 = __float_as_uint(__uint_as_float(ab << 16) * 3.0f);   // 3a, exact in float32
  const uint32_t rd3 = t3 >> 16;
  Fp3Group g;
  g.k[0] = (0x7FFFu - (ab - 4u * 0x80u)) * 0x00010001u;
  g.k[1] = (0x7FFFu - (rd3 - 4u * 0x80u)) * 0x00010001u;
  g.k[2] = (0x7FFFu - (rd3 - 3u * 0x80u)) * 0x00010001u;
  g.k[3] = (0x7FFFu - (rd3 - 2u * 0x80u)) * 0x00010001u;
  g.ex = (t3 & 0xFFFFu) == 0u ? 0x00010001u : 0u;
#pragma unroll
  for (int j = 0; j < 4; ++j) g.r[j] = (ab - (uint32_t)(3 - j) * 0x80u) * 0x00010001u;
  return g;
}

// W_hat bits of the two halves of a bf16 pair word: magnitudes, or with w's sign (+0 at level 0)
template <bool SIGNED>
__device__ __forceinline__ uint32_t fp3_rec2(uint32_t v, const Fp3Group& g) {
  const uint32_t mag = v & 0x7FFF7FFFu;
  const uint32_t neg = (v >> 15) & 0x00010001u;
  const uint32_t m0 = prmt_sign_halves(mag + neg + g.k[0]);
  const uint32_t mge = mag + (neg & g.ex);
  const uint32_t m1 = prmt_sign_halves(mge + g.k[1]);
  const uint32_t m2 = prmt_sign_halves(mge + g.k[2]);
  const uint32_t m3 = prmt_sign_halves(mge + g.k[3]);
  uint32_t r = (g.r[1] & m1) | (g.r[0] & ~m1);
  r = (g.r[2] & m2) | (r & ~m2);
  r = (g.r[3] & m3) | (r & ~m3);
  return SIGNED ? (r | (v & 0x80008000u)) & m0 : r & m0;
}

// FP8_E5M2 (format_registry.py:291-300, 466-473: one real scale per row, s = fl32(a / 114688),
// a codebook with exponent 31 kept finite, so up to 1.75 x 2^16) without division, two elements
// per step.  The quotient's half x/2 = w / (2s) is bracketed between RZ(w r_lo / 2) and
// RZ(w r_hi / 2) with the widened reciprocal bounds of the fast sweep (pq_fast.cuh), and both are
// converted by the hardware E5M2 conversion (round to nearest even, saturating at 57344).  Where
// the two codes agree, no codebook midpoint lies strictly between the brackets, fl32(w / s) lies
// strictly inside them, so the reference's nearest point (ties to the lower value) of fl32(w / s)
// is that code times 2: above 2^-13 the hardware grid of x/2, doubled, is the reference's grid of
// x (the 2^16 binade included), and saturation agrees.  With a row maximum of at least 1e-8 the
// lower bracket alone decides (e5m2_word<true>); below it, a word with a pair whose codes differ
// (an element within 2^-20 of a midpoint, exact ties among them) is redone by the exact rule, and
// in both a word with a nonzero |w| at or below RU(s 2^-12) (x/2 in the hardware's subnormal
// range, where the grids part) or a NaN is.  W_hat = bf16(fl32((x/2 code) (2s))), the error bf16(w - W_hat); a w of zero
// gives W_hat +0 as the reference's codebook zero does.
struct E5m2Row {
  uint64_t rlo2, rhi2, s2;   // r_lo / 2, r_hi / 2 and 2s, in both halves of a float32 pair
  uint32_t tiny2;            // 0x8000 + bits(RU(s 2^-12)) per half
};

__device__ __forceinline__ E5m2Row e5m2_row(float s) {   // s: a positive normal scale
  float rl, rh;
  recip_bounds(s, rl, rh);
  E5m2Row q;
  q.rlo2 = f2_pack(0.5f * rl, 0.5f * rl);
  q.rhi2 = f2_pack(0.5f * rh, 0.5f * rh);
  q.s2 = f2_pack(2.0f * s, 2.0f * s);
  q.tiny2 = (0x8000u + (__float_as_uint(s * 0x1p-12f) >> 16) + 1u) * 0x00010001u;
  return q;
}

// 8 elements: W_hat words and the fp32 sum of the 8 exact squares; false if the word needs the
// exact rule.  LOWER: convert the lower bracket min(RZ(w r_lo / 2), RZ(w r_hi / 2)) alone, which
// is the reference's point of fl32(w / s) for every element above the tiny bound, exact ties
// included, when the row maximum is a bf16 of at least 1e-8 (tests/test_fast_rules.py checks it
// for every bf16 w under every maximum of four binades and each of rcp.approx's results); only
// tiny elements then need the exact rule.
template <bool LOWER>
__device__ __forceinline__ bool e5m2_word(const uint4& u, const E5m2Row& q, uint32_t (&o)[4], float& part) {
  const uint32_t v[4] = {u.x, u.y, u.z, u.w};
  uint32_t bad = 0u;
  float acc = 0.0f;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint64_t w2 = f2_from_bf16x2(v[p]);
    uint32_t cl;
    if constexpr (LOWER) {
      cl = cvt_e5m2x2(f2_min(f2_mul_rz(w2, q.rlo2), f2_mul_rz(w2, q.rhi2)));
    } else {
      cl = cvt_e5m2x2(f2_mul_rz(w2, q.rlo2));
      bad |= cl ^ cvt_e5m2x2(f2_mul_rz(w2, q.rhi2));   // the two codes differ
    }
    const uint32_t mag = v[p] & 0x7FFF7FFFu;
    bad |= (q.tiny2 - mag) & (mag + 0x7FFF7FFFu) & 0x80008000u;   // 0 < |w| <= RU(s 2^-12)
    const uint32_t rec = f2_to_bf16x2(f2_mul_rn(f16x2_to_f2(__byte_perm(cl, 0u, 0x1404u)), q.s2));
    o[p] = rec & (prmt_sign_halves(mag + 0x7FFF7FFFu) | 0x7FFF7FFFu);   // -0 -> +0 where w = +-0
    acc = sq2_acc(bf16x2_sub(v[p], rec), acc);
  }
  part = acc;
  return bad == 0u;
}

// E4M3 with a real scale per group (FP8_E4M3_G128, the batched form of FP8_SOURCE;
// measure_quant_cost.py:516-548 with format_registry.py:194-233): the codebook is the hardware
// E4M3 grid up to 448, so the bracket of the fast sweep decides each pair: RZ(w r_lo) and
// RZ(w r_hi) hold fl32(w / s) strictly between them, and where their hardware conversions (round
// to nearest even, saturating at 448) agree no midpoint lies between them, so the code is the
// reference's nearest point of fl32(w / s) whatever its tie rule.  A word with a pair that
// disagrees (exact ties among them) or a NaN takes the exact rule.  W_hat = bf16(fl32(q s)), +0
// where q is zero, as the reference's codebook zero gives.
__device__ __forceinline__ bool e4m3g_word(const uint4& u, uint64_t lo2, uint64_t hi2, uint64_t s2, uint32_t (&o)[4],
                                           float& part) {
  const uint32_t v[4] = {u.x, u.y, u.z, u.w};
  uint32_t dx = 0u;
  float acc = 0.0f;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint64_t w2 = f2_from_bf16x2(v[p]);
    const uint32_t cl = cvt_e4m3x2(f2_mul_rz(w2, lo2));
    dx |= cl ^ cvt_e4m3x2(f2_mul_rz(w2, hi2));
    const uint32_t rec = f2_to_bf16x2(f2_mul_rn(e4m3x2_to_f2(cl), s2));
    o[p] = rec & (prmt_sign_halves((rec & 0x7FFF7FFFu) + 0x7FFF7FFFu) | 0x7FFF7FFFu);   // -0 -> +0
    acc = sq2_acc(bf16x2_sub(v[p], rec), acc);
  }
  part = acc;
  return dx == 0u;
}

// The same groups outside the flagged family of the fast sweep's FP8 rows (row_tab in
// pq_sweep_fast.cu): with 1e-8 <= a < 2^60 and not (|a - 448 s| >= 160 ulp(s) and s's significand
// below 1.5), the conversion of the lower bracket min(RZ(w r_lo), RZ(w r_hi)) is the reference's
// code, exact ties included (tests/test_fast_rules.py checks the rule for every pair of bf16
// values), so no word needs the exact rule.
__device__ __forceinline__ void e4m3g_lower_word(const uint4& u, uint64_t lo2, uint64_t hi2, uint64_t s2,
                                                 uint32_t (&o)[4], float& part) {
  const uint32_t v[4] = {u.x, u.y, u.z, u.w};
  float acc = 0.0f;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint64_t w2 = f2_from_bf16x2(v[p]);
    const uint32_t c = cvt_e4m3x2(f2_min(f2_mul_rz(w2, lo2), f2_mul_rz(w2, hi2)));
    const uint32_t rec = f2_to_bf16x2(f2_mul_rn(e4m3x2_to_f2(c), s2));
    o[p] = rec & (prmt_sign_halves((rec & 0x7FFF7FFFu) + 0x7FFF7FFFu) | 0x7FFF7FFFu);   // -0 -> +0
    acc = sq2_acc(bf16x2_sub(v[p], rec), acc);
  }
  part = acc;
}

// Row-wise symmetric integer formats (INT8_W8A16, and any integer format whose group is a whole
// row; format_registry.py:147-172: s = fl32(max(a, 1e-8) / L), q = round half even (fl32(w / s))
// clamped to [-L-1, L], W_hat = bf16(q s)) without division per element: the reciprocal bracket
// of intsse_kernel, RN(w RN(r (1 -+ 2^-19))) with r = rcp.approx(s), each rounded half even to
// an integer by adding and subtracting 1.5 x 2^23 in float32 pairs.  Where the two integers agree
// no half-integer lies between the products, which hold fl32(w / s) strictly between them, so
// that integer is the reference's (|w| <= a keeps it within [-L, L]).  W_hat takes w's sign, as
// torch.round gives -0.0 for a negative w that rounds to zero.  A word with a pair that
// disagrees (an exact tie among them) or a NaN takes the exact rule.
struct IntRow {
  uint64_t lo2, hi2, s2;   // the two bracket reciprocals and s, in both halves of a float32 pair
};

__device__ __forceinline__ IntRow int_row(float s) {   // s: a positive normal scale
  const float r = rcp_approx(s);
  const float lo = __fmul_rn(r, 1.0f - 0x1p-19f), hi = __fmul_rn(r, 1.0f + 0x1p-19f);
  return {f2_pack(lo, lo), f2_pack(hi, hi), f2_pack(s, s)};
}

// 8 elements: W_hat words and the fp32 sum of the 8 exact squares; false if the word needs the
// exact rule
__device__ __forceinline__ bool int_word(const uint4& u, const IntRow& q, uint32_t (&o)[4], float& part) {
  const uint64_t m2 = f2_pack(12582912.0f, 12582912.0f), nm2 = f2_pack(-12582912.0f, -12582912.0f);   // 1.5 x 2^23
  const uint32_t v[4] = {u.x, u.y, u.z, u.w};
  bool split = false;
  float acc = 0.0f;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint64_t w2 = f2_from_bf16x2(v[p]);
    const uint64_t ql = f2_add_rn(f2_add_rn(f2_mul_rn(w2, q.lo2), m2), nm2);
    const uint64_t qh = f2_add_rn(f2_add_rn(f2_mul_rn(w2, q.hi2), m2), nm2);
    split = split || ql != qh;
    const uint32_t rec = f2_to_bf16x2(f2_mul_rn(ql, q.s2));
    o[p] = rec | (v[p] & 0x80008000u);   // q = 0 keeps w's sign; q != 0 has it already
    acc = sq2_acc(bf16x2_sub(v[p], rec), acc);
  }
  part = acc;
  return !split;
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
        const uint32_t b = FAST ? __float_as_uint(rec) >> 16 : bf16_bits_torch(rec);   // NaN: 0 x inf
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
        if (MXK && f.mx && scale >= 0x1p-100f && scale <= 0x1p100f && !has_nan8(u)) {
          const int es = (int)(__float_as_uint(scale) >> 23) - 127;
          if (MODE == MODE_SSE && h_mode == 0)
            acc += (double)mx_sse8<(KIND == XK_INT ? XK_E2M1 : KIND)>(u, es);
          else if (MODE == MODE_QDQ && es >= -90 && es <= 90) {
            uint32_t o[4];
            mx_qdq8<(KIND == XK_INT ? XK_E2M1 : KIND)>(u, es, o);
            *reinterpret_cast<uint4*>(out + r * cols + col) = make_uint4(o[0], o[1], o[2], o[3]);
          } else
            do8(u, wv, r * cols + col, r, scale, inv, std::true_type{});
        } else if (KIND == XK_E4M3 && !f.mx && h_mode == 0 && a >= 1e-8f && a < F8_EXACT_ROW_AMAX &&
                   !has_nan8(u)) {
          // E4M3 with real group scales (FP8_E4M3_G128): the lower-bracket rule, or the bracket of
          // e4m3g_word in groups of the flagged family
          float rl, rh;
          recip_bounds(scale, rl, rh);
          const uint32_t sb = __float_as_uint(scale);
          const float ulp = __uint_as_float((sb & 0x7F800000u) - (23u << 23));
          const bool flagged = fabsf(__fmaf_rn(-448.0f, scale, a)) >= 160.0f * ulp && (sb & 0x7FFFFFu) < 0x400000u;
          const uint64_t lo2 = f2_pack(rl, rl), hi2 = f2_pack(rh, rh), s2 = f2_pack(scale, scale);
          uint32_t o[4];
          float part;
          bool fast = true;
          if (flagged) fast = e4m3g_word(u, lo2, hi2, s2, o, part);
          else e4m3g_lower_word(u, lo2, hi2, s2, o, part);
          if (fast) {
            if (MODE == MODE_QDQ)
              *reinterpret_cast<uint4*>(out + r * cols + col) = make_uint4(o[0], o[1], o[2], o[3]);
            else
              acc += (double)part;
          } else {
            do8(u, wv, r * cols + col, r, scale, inv, std::false_type{});
          }
        } else if (KIND == XK_E2M0 && MODE == MODE_QDQ && (__float_as_uint(a) >> 16) >= BF16_1EM8_CEIL &&
                   (__float_as_uint(a) >> 16) < FP3_FAST_CEIL && !has_nan8(u)) {
          // NVFP3 with a group maximum in [1e-8, 2^126): the comparisons of fp3sse_kernel
          const Fp3Group g3 = fp3_group(__float_as_uint(a) >> 16);
          const uint4 o = make_uint4(fp3_rec2<true>(u.x, g3), fp3_rec2<true>(u.y, g3), fp3_rec2<true>(u.z, g3),
                                     fp3_rec2<true>(u.w, g3));
          *reinterpret_cast<uint4*>(out + r * cols + col) = o;
        } else
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
      if constexpr (KIND == XK_E5M2 || KIND == XK_INT) {
        // FP8_E5M2 (e5m2_word) and the integer formats (int_word) by their brackets where the
        // scale is a normal number, unweighted
        if (!f.mx && h_mode == 0 && scale >= 0x1p-126f && scale <= 0x1p120f) {
          E5m2Row qe{};
          IntRow qi{};
          if constexpr (KIND == XK_E5M2) qe = e5m2_row(scale); else qi = int_row(scale);
          for (int64_t col = lane * 8; col < cols; col += 256) {
            const uint4 u = __ldg(reinterpret_cast<const uint4*>(row + col));
            uint32_t o[4];
            float part;
            bool fast;
            if constexpr (KIND == XK_E5M2)
              fast = !has_nan8(u) && (a >= 1e-8f ? e5m2_word<true>(u, qe, o, part) : e5m2_word<false>(u, qe, o, part));
            else fast = !has_nan8(u) && int_word(u, qi, o, part);
            if (fast) {
              if (MODE == MODE_QDQ)
                *reinterpret_cast<uint4*>(out + r * cols + col) = make_uint4(o[0], o[1], o[2], o[3]);
              else
                acc += (double)part;
            } else {   // rare: a near-midpoint element, a tiny one or a NaN
              float wv[8];
              unpack8(u, wv);
              do8(u, wv, r * cols + col, r, scale, inv, std::false_type{});
            }
          }
          continue;
        }
      }
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

// ---------------------------------------------------------------------------
// Squared error of the MX formats (E8M0 scale per 32 elements) from one read of the weights,
// unweighted (the cost path's weight_mse), any set of the five MX kinds in one launch.  Rows are
// a multiple of 32 elements, so the tensor is one flat run of 32-element groups: a lane takes
// 16-byte words (8 elements) and the four lanes of a group reduce its maximum magnitude with two
// shuffles.  The group exponent, round(log2(max(amax, 1e-8) / cmax)) (format_registry.py:175-191),
// has a closed form in the bits of the bf16 maximum: with E its unbiased exponent and m its 7
// mantissa bits, e = E + C + (m >= T) for amax >= 1e-8 and a constant below it, per format
// (tests/test_fast_rules.py checks C, T and the constant against the torch-derived rule for every
// bf16 value).  Groups with e <= 100 and a finite maximum take mx_sse8; the others (an infinity or
// NaN in the group, or a scale above 2^100) the generic per-element rule.

// closed-form group exponent of each MX kind
template <int KIND> struct MXE;
template <> struct MXE<XK_E2M1> { static constexpr int C = -3, T = 8, FLOOR = -29; };
template <> struct MXE<XK_E3M2> { static constexpr int C = -5, T = 31, FLOOR = -31; };
template <> struct MXE<XK_E2M3> { static constexpr int C = -3, T = 42, FLOOR = -29; };
template <> struct MXE<XK_E4M3> { static constexpr int C = -9, T = 31, FLOOR = -35; };
template <> struct MXE<XK_E5M2> { static constexpr int C = -17, T = 31, FLOOR = -43; };

template <int KIND>
__device__ __forceinline__ int mx_exp_closed(uint32_t ab) {   // ab: finite max |w| bits
  using X = MXE<KIND>;
  return ab < BF16_1EM8_CEIL ? X::FLOOR : (int)(ab >> 7) - 127 + X::C + ((ab & 0x7Fu) >= (uint32_t)X::T ? 1 : 0);
}

// The generic rule for 8 elements of a group with scale 2^e (what xfmt2_kernel does for them).
template <int KIND>
__device__ __forceinline__ float mx_sse8_generic(const uint4& u, int e) {
  const float scale = pow2i(e);
  const float inv = __frcp_rn(scale);
  float wv[8];
  unpack8(u, wv);
  float part = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float x = __fmul_rn(wv[i], inv);
    const float rec = bf16_round(__fmul_rn(xk_round<KIND>(x, 0), scale));
    const float er = bf16_round(__fsub_rn(wv[i], rec));
    part = __fadd_rn(part, __fmul_rn(er, er));
  }
  return part;
}

// max |w| bits over 8 bf16 values (integer max of the magnitude patterns: NaN above infinity
// above every finite value, which it orders as float comparisons do)
__device__ __forceinline__ uint32_t amax_bits8(const uint4& u) {
  uint32_t t;
  asm("{\n\t.reg .b32 a, b;\n\t"
      "max.u16x2 a, %1, %2;\n\tmax.u16x2 b, %3, %4;\n\tmax.u16x2 %0, a, b;\n\t}"
      : "=r"(t)
      : "r"(u.x & 0x7FFF7FFFu), "r"(u.y & 0x7FFF7FFFu), "r"(u.z & 0x7FFF7FFFu), "r"(u.w & 0x7FFF7FFFu));
  return max(t & 0xFFFFu, t >> 16);
}

// kinds present in a kind mask, in a fixed order; bit k = kind XK_E2M1 + k ... see mx_kind_bit
__host__ __device__ constexpr int mx_kind_bit(int kind) {
  return kind == XK_E2M1 ? 0 : kind == XK_E3M2 ? 1 : kind == XK_E2M3 ? 2 : kind == XK_E4M3 ? 3 : 4;
}
constexpr int MX_KIND_OF_BIT[5] = {XK_E2M1, XK_E3M2, XK_E2M3, XK_E4M3, XK_E5M2};

struct MxSseLaunch {
  double* sse[5];   // per kind bit: the format's fp64 sum (added to), null if absent
};

// one format of the set: its partial for this word, added to the fp32 accumulator
template <uint32_t KM, int BIT>
__device__ __forceinline__ void mx_word(const uint4& u, uint32_t ab, bool finite, float (&acc)[5]) {
  if constexpr ((KM >> BIT) & 1u) {
    constexpr int K = MX_KIND_OF_BIT[BIT];
    const int e = finite ? mx_exp_closed<K>(ab) : 127;   // an infinity's group: log2 clamped at 127
    acc[BIT] += (finite && e <= 100) ? mx_sse8<K>(u, e) : mx_sse8_generic<K>(u, e);
  }
}

constexpr int MXSSE_UNROLL = 4;   // 16-byte words per lane in flight per pass

template <uint32_t KM>
__global__ void __launch_bounds__(256) mxsse_kernel(const uint4* __restrict__ w, int64_t nwords,
                                                    const __grid_constant__ MxSseLaunch L) {
  const int lane = threadIdx.x & 31;
  const int64_t warp_first = (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * (32 * MXSSE_UNROLL);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * MXSSE_UNROLL;
  double acc[5] = {0.0, 0.0, 0.0, 0.0, 0.0};
  // warp-uniform loop: a pass covers 32 x MXSSE_UNROLL consecutive words; a 4-word group is all
  // inside the tensor or all past its end (nwords is a multiple of 4), and words past the end
  // are zeros, which add nothing
  for (int64_t base = warp_first; base < nwords; base += stride) {
    uint4 u[MXSSE_UNROLL];
#pragma unroll
    for (int k = 0; k < MXSSE_UNROLL; ++k) {
      const int64_t j = base + 32 * k + lane;
      u[k] = j < nwords ? __ldg(w + j) : make_uint4(0u, 0u, 0u, 0u);
    }
    float part[5] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f};   // <= 32 exact squares each
#pragma unroll
    for (int k = 0; k < MXSSE_UNROLL; ++k) {
      uint32_t ab = amax_bits8(u[k]);
      ab = max(ab, (uint32_t)__shfl_xor_sync(FULL, ab, 1));
      ab = max(ab, (uint32_t)__shfl_xor_sync(FULL, ab, 2));
      const bool finite = ab < 0x7F80u;
      mx_word<KM, 0>(u[k], ab, finite, part);
      mx_word<KM, 1>(u[k], ab, finite, part);
      mx_word<KM, 2>(u[k], ab, finite, part);
      mx_word<KM, 3>(u[k], ab, finite, part);
      mx_word<KM, 4>(u[k], ab, finite, part);
    }
#pragma unroll
    for (int f = 0; f < 5; ++f)
      if ((KM >> f) & 1u) acc[f] += (double)part[f];
  }
#pragma unroll
  for (int f = 0; f < 5; ++f) {
    if (!((KM >> f) & 1u)) continue;
    const double v = warp_sum_d(acc[f]);
    if (lane == 0 && v != 0.0) atomicAdd(L.sse[f], v);
  }
}

// MX kind of a format, false if it is not an MX format of this kernel
__host__ __device__ inline bool mx_kind_of(int fmt, int& kind) {
  switch (fmt) {
    case PQ_FMT_MXFP4: kind = XK_E2M1; return true;
    case PQ_FMT_MXFP6_E3M2: kind = XK_E3M2; return true;
    case PQ_FMT_MXFP6_E2M3: kind = XK_E2M3; return true;
    case PQ_FMT_MXFP8: kind = XK_E4M3; return true;
    case PQ_FMT_MXFP8_E5M2: kind = XK_E5M2; return true;
    default: return false;
  }
}

// The one-read path applies: the format is an MX format of mxsse_kernel, rows are a whole number
// of 32-element groups, and the weights start on a 16-byte boundary.
bool mxsse_ok(const uint16_t* w, int64_t cols, int fmt) {
  int kind;
  return mx_kind_of(fmt, kind) && cols % 32 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0;
}

// fmts: distinct MX formats, each mxsse_ok; sse[f] receives format f's sum
cudaError_t launch_mxsse(const uint16_t* w, int64_t rows, int64_t cols, const int* fmts, int nf,
                         double* const* sse, int num_sms, cudaStream_t stream) {
  MxSseLaunch L{};
  uint32_t km = 0;
  for (int f = 0; f < nf; ++f) {
    int kind = 0;
    mx_kind_of(fmts[f], kind);
    const int bit = mx_kind_bit(kind);
    km |= 1u << bit;
    L.sse[bit] = sse[f];
  }
  const int64_t nwords = rows * cols / 8;
  int64_t blocks = (nwords + 256 * MXSSE_UNROLL - 1) / (256 * MXSSE_UNROLL);
  if (blocks > (int64_t)num_sms * 8) blocks = (int64_t)num_sms * 8;
  if (blocks < 1) blocks = 1;
  const uint4* w4 = reinterpret_cast<const uint4*>(w);
  switch (km) {
#define PQ_MX_CASE(M) \
    case M: mxsse_kernel<M><<<(unsigned)blocks, 256, 0, stream>>>(w4, nwords, L); break;
    PQ_MX_CASE(1) PQ_MX_CASE(2) PQ_MX_CASE(3) PQ_MX_CASE(4) PQ_MX_CASE(5) PQ_MX_CASE(6) PQ_MX_CASE(7)
    PQ_MX_CASE(8) PQ_MX_CASE(9) PQ_MX_CASE(10) PQ_MX_CASE(11) PQ_MX_CASE(12) PQ_MX_CASE(13) PQ_MX_CASE(14)
    PQ_MX_CASE(15) PQ_MX_CASE(16) PQ_MX_CASE(17) PQ_MX_CASE(18) PQ_MX_CASE(19) PQ_MX_CASE(20) PQ_MX_CASE(21)
    PQ_MX_CASE(22) PQ_MX_CASE(23) PQ_MX_CASE(24) PQ_MX_CASE(25) PQ_MX_CASE(26) PQ_MX_CASE(27) PQ_MX_CASE(28)
    PQ_MX_CASE(29) PQ_MX_CASE(30) PQ_MX_CASE(31)
#undef PQ_MX_CASE
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}
// ---------------------------------------------------------------------------
// Squared error of the grouped symmetric integer formats (INT2 / INT3 in groups of 16, INT4 in
// groups of 128; format_registry.py:147-172): s = fl32(max(amax, 1e-8) / L), q = round half even
// (fl32(w / s)) clamped to [-L-1, L], W_hat = bf16(q s).  The integer comes from a reciprocal
// bracket, two products per pair of elements (int_sse_word); words where the bracket straddles a
// half-integer (every exact tie among them) are redone by IEEE division, about 1e-4 of bf16 data.
// Rows are a multiple of the group, so the tensor is one flat run of groups; LANES = group / 8
// lanes reduce a group's maximum.  Groups with an infinity or NaN take IEEE division throughout
// (int_err_sq, which alone takes the product p = RN(w r) when p lies further than 2^-19 |M| from
// the nearest midpoint M = floor(p) + 1/2).
template <int L>
__device__ __forceinline__ float int_err_sq(float w, float s, float r, bool exact) {
  const float p = __fmul_rn(w, r);
  const float mid = floorf(p) + 0.5f;
  float x = p;
  if (exact || fabsf(p - mid) <= fabsf(mid) * 0x1p-19f) x = __fdiv_rn(w, s);   // rare
  const float q = x != x ? x : fminf(fmaxf(rintf(x), (float)(-L - 1)), (float)L);   // torch.clamp keeps a NaN
  const float e = bf16_round(__fsub_rn(w, bf16_round(__fmul_rn(q, s))));
  return __fmul_rn(e, e);   // the reference squares in fp32
}

// The 8 elements of one 16-byte word in float32 pairs: the two bracket products p_lo = RN(w r_lo)
// and p_hi = RN(w r_hi), r_lo / r_hi RN(1/s) (1 -+ 2^-19) rounded, hold fl32(w / s) strictly
// between them; each is rounded half even to an integer by adding and subtracting 1.5 x 2^23.
// Where the two integers agree no half-integer lies between the products (one exactly on a
// half-integer rounds toward the other side's integer or to the same one), so that integer is
// the reference's; it is never outside [-L, L] here (|w| <= amax).  A word with a pair that
// disagrees (an exact tie among them) is redone by IEEE division.  Returns the fp32 sum of the
// 8 exact squares.
template <int L>
__device__ __forceinline__ float int_sse_word(const uint4& u, float s, float r_lo, float r_hi) {
  const uint64_t lo2 = f2_pack(r_lo, r_lo), hi2 = f2_pack(r_hi, r_hi), s2 = f2_pack(s, s);
  const uint64_t m2 = f2_pack(12582912.0f, 12582912.0f), nm2 = f2_pack(-12582912.0f, -12582912.0f);   // 1.5 x 2^23
  const uint32_t v[4] = {u.x, u.y, u.z, u.w};
  float acc = 0.0f;
  bool split = false;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint64_t w2 = f2_from_bf16x2(v[p]);
    const uint64_t ql = f2_add_rn(f2_add_rn(f2_mul_rn(w2, lo2), m2), nm2);
    const uint64_t qh = f2_add_rn(f2_add_rn(f2_mul_rn(w2, hi2), m2), nm2);
    split = split || ql != qh;
    acc = sq2_acc(bf16x2_sub(v[p], f2_to_bf16x2(f2_mul_rn(ql, s2))), acc);
  }
  if (split) {   // rare
    const float r = __frcp_rn(s);
    float wv[8];
    unpack8(u, wv);
    acc = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc = __fadd_rn(acc, int_err_sq<L>(wv[i], s, r, true));
  }
  return acc;
}

template <int L, int LANES>
__global__ void __launch_bounds__(256) intsse_kernel(const uint4* __restrict__ w, int64_t nwords, double* sse) {
  static_assert(L == 1 || L == 3 || L == 7, "div_const is checked for these divisors");
  const int lane = threadIdx.x & 31;
  const int64_t warp_first = (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * (32 * MXSSE_UNROLL);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * MXSSE_UNROLL;
  double acc = 0.0;
  for (int64_t base = warp_first; base < nwords; base += stride) {   // warp-uniform
    uint4 u[MXSSE_UNROLL];
#pragma unroll
    for (int k = 0; k < MXSSE_UNROLL; ++k) {
      const int64_t j = base + 32 * k + lane;
      u[k] = j < nwords ? __ldg(w + j) : make_uint4(0u, 0u, 0u, 0u);
    }
    float part = 0.0f;
#pragma unroll
    for (int k = 0; k < MXSSE_UNROLL; ++k) {
      uint32_t ab = amax_bits8(u[k]);
#pragma unroll
      for (int o = 1; o < LANES; o <<= 1) ab = max(ab, (uint32_t)__shfl_xor_sync(FULL, ab, o));
      const bool finite = ab < 0x7F80u;
      const float am = fmaxf(__uint_as_float(ab << 16), 1e-8f);
      if (finite) {
        // s = RN(am / L) (div_const is IEEE division for every normal bf16 and the floor); the
        // bracket tolerates a reciprocal within one ulp
        const float s = L == 1 ? am : div_const(am, (float)L, L == 3 ? RCP3 : RCP7);
        const float r = rcp_approx(s);
        part += int_sse_word<L>(u[k], s, __fmul_rn(r, 1.0f - 0x1p-19f), __fmul_rn(r, 1.0f + 0x1p-19f));
      } else {   // an infinity or NaN in the group
        const float s = __fdiv_rn(am, (float)L);
        float wv[8];
        unpack8(u[k], wv);
#pragma unroll
        for (int i = 0; i < 8; ++i) part = __fadd_rn(part, int_err_sq<L>(wv[i], s, 0.0f, true));
      }
    }
    acc += (double)part;   // fp32 partials of 32 exact squares
  }
  const double v = warp_sum_d(acc);
  if (lane == 0 && v != 0.0) atomicAdd(sse, v);
}

// levels L and group length of a grouped integer format of intsse_kernel (0 if it is not one)
__host__ __device__ inline int int_group_of(int fmt, int& L) {
  switch (fmt) {
    case PQ_FMT_INT2: L = 1; return 16;
    case PQ_FMT_INT3: L = 3; return 16;
    case PQ_FMT_INT4_G128: L = 7; return 128;
    default: return 0;
  }
}

bool intsse_ok(const uint16_t* w, int64_t cols, int fmt) {
  int L;
  const int g = int_group_of(fmt, L);
  return g > 0 && cols > g && cols % g == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0;
}

cudaError_t launch_intsse(const uint16_t* w, int64_t rows, int64_t cols, int fmt, double* sse, int num_sms,
                          cudaStream_t stream) {
  int L = 0;
  int_group_of(fmt, L);
  const int64_t nwords = rows * cols / 8;
  int64_t blocks = (nwords + 256 * MXSSE_UNROLL - 1) / (256 * MXSSE_UNROLL);
  if (blocks > (int64_t)num_sms * 8) blocks = (int64_t)num_sms * 8;
  if (blocks < 1) blocks = 1;
  const uint4* w4 = reinterpret_cast<const uint4*>(w);
  switch (fmt) {
    case PQ_FMT_INT2: intsse_kernel<1, 2><<<(unsigned)blocks, 256, 0, stream>>>(w4, nwords, sse); break;
    case PQ_FMT_INT3: intsse_kernel<3, 2><<<(unsigned)blocks, 256, 0, stream>>>(w4, nwords, sse); break;
    default: intsse_kernel<7, 16><<<(unsigned)blocks, 256, 0, stream>>>(w4, nwords, sse); break;
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Squared error of NVFP3 from one read, flat over the tensor's groups like intsse_kernel, with the
// comparisons of fp3_group / fp3_rec2.  Groups whose maximum is below 1e-8 (all zeros excepted,
// which add nothing), at least 2^126 or not finite take the per-element rule.

__device__ __forceinline__ float fp3_sse8(const uint4& u, const Fp3Group& g) {
  const uint32_t v[4] = {u.x, u.y, u.z, u.w};
  float acc = 0.0f;
#pragma unroll
  for (int p = 0; p < 4; ++p) acc = sq2_acc(bf16x2_sub(v[p] & 0x7FFF7FFFu, fp3_rec2<false>(v[p], g)), acc);
  return acc;
}

// the per-element rule for 8 elements of a group with maximum bits ab (xfmt2_kernel's arithmetic)
__device__ __forceinline__ float fp3_sse8_generic(const uint4& u, uint32_t ab) {
  const float s = __fdiv_rn(fmaxf(__uint_as_float(ab << 16), 1e-8f), 2.0f);
  float wv[8];
  unpack8(u, wv);
  float part = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float rec = bf16_round(__fmul_rn(xk_round<XK_E2M0>(__fdiv_rn(wv[i], s), 0), s));
    const float e = bf16_round(__fsub_rn(wv[i], rec));
    part = __fadd_rn(part, __fmul_rn(e, e));
  }
  return part;
}

__global__ void __launch_bounds__(256) fp3sse_kernel(const uint4* __restrict__ w, int64_t nwords, double* sse) {
  const int lane = threadIdx.x & 31;
  const int64_t warp_first = (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * (32 * MXSSE_UNROLL);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * MXSSE_UNROLL;
  double acc = 0.0;
  for (int64_t base = warp_first; base < nwords; base += stride) {   // warp-uniform
    uint4 u[MXSSE_UNROLL];
#pragma unroll
    for (int k = 0; k < MXSSE_UNROLL; ++k) {
      const int64_t j = base + 32 * k + lane;
      u[k] = j < nwords ? __ldg(w + j) : make_uint4(0u, 0u, 0u, 0u);
    }
    float part = 0.0f;
#pragma unroll
    for (int k = 0; k < MXSSE_UNROLL; ++k) {
      uint32_t ab = amax_bits8(u[k]);
      ab = max(ab, (uint32_t)__shfl_xor_sync(FULL, ab, 1));   // the two lanes of a 16-element group
      if (ab >= BF16_1EM8_CEIL && ab < FP3_FAST_CEIL)
        part += fp3_sse8(u[k], fp3_group(ab));
      else if (ab != 0u)   // rare: a maximum below 1e-8 or at least 2^126, an infinity or a NaN
        part += fp3_sse8_generic(u[k], ab);
    }
    acc += (double)part;   // fp32 partials of 32 exact squares
  }
  const double v = warp_sum_d(acc);
  if (lane == 0 && v != 0.0) atomicAdd(sse, v);
}

bool fp3sse_ok(const uint16_t* w, int64_t cols, int fmt) {
  return fmt == PQ_FMT_NVFP3 && cols % 16 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0;
}

cudaError_t launch_fp3sse(const uint16_t* w, int64_t rows, int64_t cols, double* sse, int num_sms,
                          cudaStream_t stream) {
  const int64_t nwords = rows * cols / 8;
  int64_t blocks = (nwords + 256 * MXSSE_UNROLL - 1) / (256 * MXSSE_UNROLL);
  if (blocks > (int64_t)num_sms * 8) blocks = (int64_t)num_sms * 8;
  if (blocks < 1) blocks = 1;
  fp3sse_kernel<<<(unsigned)blocks, 256, 0, stream>>>(reinterpret_cast<const uint4*>(w), nwords, sse);
  return cudaGetLastError();
}

}  // namespace pq
