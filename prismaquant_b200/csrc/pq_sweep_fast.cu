// Fast multi-format sweep (SSE mode): same work items, staging and outputs as
// sweep_staged_kernel<MODE_SSE>, with the per-element arithmetic rebuilt on
// packed sm_100a instructions (pq_fast.cuh):
//
//  * a thread owns a 16-element NVFP4 group ("unit", two 16-byte shared
//    loads); MXFP8 32-groups are lane pairs (one shuffle);
//  * NVFP4 cost: the code of fma(w, r, -2^-18) with r = rcp.approx(s), one
//    hardware conversion per pair.  w and the group max a have 8-bit
//    significands, so w / (a / 6) is either exactly an E2M1 midpoint or at
//    least ~2^-11 (relative) away from every midpoint; at an exact midpoint
//    the reference's fl32(w / s) IS the midpoint (a / 6 is exact unless the
//    midpoint is 0.75, and there the scale's rounding moves the quotient by
//    at most half an ulp of 0.75), so its nearest-with-ties-to-lower code is
//    "the code below", which the absolute bias toward -inf gives.  The NVFP4
//    export code (ties toward zero) is the code of RZ(w r_lo), r_lo just
//    below 1/s.  Both rules are checked against the reference rule on every
//    pair of bf16 values (tests/test_fast_rules.py);
//  * FP8 per channel: the code of min(RZ(w r_lo), RZ(w r_hi)), the bracket
//    product below the quotient, the same tie rule.  It is exact except in
//    rows where |a - 448 s| = 3 * 64 ulp(s) and s's significand is below 1.5
//    (and rows whose max is below the 1e-8 floor): there the quotient of an
//    exact tie can round off the midpoint.  Those rows also convert both
//    brackets; a unit with a pair whose brackets differ is queued and
//    resolved exactly at the end of the item (division-free, mid_side);
//  * then exact f16 decode -> f32x2 product with the scale -> bf16x2
//    reconstruction -> bf16x2 error -> mixed-precision square-accumulate;
//  * MXFP8 (power-of-two scale): the E4M3 rounding is an integer rounding of
//    the bf16 bit pattern, two elements per 32-bit operation (low 4 mantissa
//    bits), saturated at 448 * 2^e by a packed magnitude min; its exponent is
//    a closed form of the group amax bits (e = E - 136 + (mantissa >= 31)),
//    checked over every bf16 amax.  Only the squared error is needed, and at a
//    tie both neighbours are 8 ulp away (also when the upper one saturates), so
//    the magnitude is rounded half-up whatever the reference's tie rule;
//  * a unit or row outside the fast path's range is done by the exact path
//    (IEEE division, the reference's tie rules).
#include "pq_fast.cuh"
#include "pq_internal.h"

namespace pq {

constexpr int FAST_THREADS = SWEEP_THREADS;

// FP8 per-channel rows whose max |w| reaches this are done entirely by the
// exact path (a provisional fp32 square could overflow).
constexpr float F8_EXACT_ROW_AMAX = 1.152921504606846976e18f;  // 2^60

struct RowParam {
  float s, r_lo, r_hi, amax;
  bool flag;   // the lower-bracket rule may differ from the reference here: resolve exactly
};

// FP8 per-channel row scale from the row's max |w| (bf16 bits): s = max(amax, 1e-8) / 448
// (div_const is exact for every normal bf16 value and for the 1e-8 floor).  flag: the row's max
// is below the floor (s is not amax / 448), or d = amax - 448 s (exact as one FMA: a multiple of
// 64 ulp(s) of at most 3 of them) is 3 x 64 ulp(s) and s's significand is below 1.5, the only
// rows where an exact midpoint's fl32 quotient can round off the midpoint.
__device__ __forceinline__ RowParam row_param(uint32_t ra_bits) {
  RowParam p;
  p.amax = __uint_as_float(ra_bits << 16);
  p.s = div_const(fmaxf(p.amax, 1e-8f), 448.0f, RCP448);
  recip_bounds(p.s, p.r_lo, p.r_hi);
  const uint32_t sb = __float_as_uint(p.s);
  const float ulp = __uint_as_float((sb & 0x7F800000u) - (23u << 23));
  const float d = __fmaf_rn(-448.0f, p.s, p.amax);
  p.flag = p.amax < 1e-8f || (fabsf(d) >= 160.0f * ulp && (sb & 0x7FFFFFu) < 0x400000u);
  return p;
}

// Loads unit u (16 bf16) from the stage into v[0..7]; lanes of a quarter-warp
// alternate which 16-byte half they read first so the 128-bit loads are
// bank-conflict free.  Returns true if the halves were swapped.
__device__ __forceinline__ bool load_unit(const uint4* st, int u, bool valid, int lane, uint32_t (&v)[8]) {
  const bool sw = (lane >> 2) & 1;
  uint4 a = make_uint4(0, 0, 0, 0), b = a;
  if (valid) {
    a = st[2 * u + (sw ? 1 : 0)];
    b = st[2 * u + (sw ? 0 : 1)];
  }
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  return sw;
}

// bf16 magnitude max / min over the 16 elements, as 16-bit patterns.
__device__ __forceinline__ void unit_absmax_min(const uint32_t (&v)[8], uint32_t& amax_bits, uint32_t& amin_bits) {
  uint32_t m01 = bf16x2_maxabs(v[0], v[1]), m23 = bf16x2_maxabs(v[2], v[3]);
  uint32_t m45 = bf16x2_maxabs(v[4], v[5]), m67 = bf16x2_maxabs(v[6], v[7]);
  uint32_t m = bf16x2_maxabs(bf16x2_maxabs(m01, m23), bf16x2_maxabs(m45, m67));
  m = bf16x2_maxabs(m, (m >> 16) | (m << 16));
  amax_bits = m & 0x7FFFu;
  uint32_t n01 = bf16x2_minabs(v[0], v[1]), n23 = bf16x2_minabs(v[2], v[3]);
  uint32_t n45 = bf16x2_minabs(v[4], v[5]), n67 = bf16x2_minabs(v[6], v[7]);
  uint32_t n = bf16x2_minabs(bf16x2_minabs(n01, n23), bf16x2_minabs(n45, n67));
  n = bf16x2_minabs(n, (n >> 16) | (n << 16));
  amin_bits = n & 0x7FFFu;
}

__device__ __forceinline__ uint32_t unit_absmax(const uint32_t (&v)[8]) {
  uint32_t m01 = bf16x2_maxabs(v[0], v[1]), m23 = bf16x2_maxabs(v[2], v[3]);
  uint32_t m45 = bf16x2_maxabs(v[4], v[5]), m67 = bf16x2_maxabs(v[6], v[7]);
  uint32_t m = bf16x2_maxabs(bf16x2_maxabs(m01, m23), bf16x2_maxabs(m45, m67));
  m = bf16x2_maxabs(m, (m >> 16) | (m << 16));
  return m & 0x7FFFu;
}

__device__ __forceinline__ void unit_to_chunks(const uint32_t (&v)[8], Chunk8& c0, Chunk8& c1) {
  unpack8(make_uint4(v[0], v[1], v[2], v[3]), c0.w);
  unpack8(make_uint4(v[4], v[5], v[6], v[7]), c1.w);
}

constexpr int FAST_QCAP = 64;            // queued FP8 units per warp
// NVFP4 cost products are biased by this (absolute, in units of the scaled value |w / s| <= 6):
// below 2^-13 x 0.25, the smallest distance of a non-midpoint quotient from a midpoint, and
// above the products' own error at a midpoint (tests/test_fast_rules.py checks every bf16 pair)
constexpr float NV_COST_BIAS = 3.814697265625e-06f;   // 2^-18
constexpr int FAST_MAX_ROWS = FAST_MAX_ROWS_PER_ITEM;

__device__ __forceinline__ float sq_exact_err(float w, float r) {
  const float e = bf16_round(__fsub_rn(w, r));
  return e * e;
}

// A unit whose amax is below the reference's 1e-8 scale floor, or so large
// that a provisional fp32 square could overflow, is done entirely by the
// exact path (main loop contributes nothing for it).
__device__ __forceinline__ bool exact_unit(float a16) { return a16 < 1e-8f || a16 >= 1.152921504606846976e18f; }

// NVFP4 bracket of one pair: low / high conversion codes (one byte each).
__device__ __forceinline__ void nv_bracket(uint64_t w2, uint64_t rlo2, uint64_t rhi2, uint32_t& cl, uint32_t& ch) {
  cl = cvt_e2m1x2(f2_mul_rz(w2, rlo2));
  ch = cvt_e2m1x2(f2_mul_rz(w2, rhi2));
}
// bf16 pair with each -0.0 replaced by +0.0: the cost codebook holds only +0.0, so a value that
// rounds to zero reconstructs as +0.0 whatever its sign.
__device__ __forceinline__ uint32_t bf16x2_plus_zero(uint32_t r) {
  const uint32_t nz = ((r & 0x7FFF7FFFu) + 0x7FFF7FFFu) & 0x80008000u;   // bit 15 / 31 set iff |half| != 0
  return r & (nz | 0x7FFF7FFFu);
}
__device__ __forceinline__ uint32_t nv_pair_rec(uint32_t cl, uint64_t s2) {
  return bf16x2_plus_zero(f2_to_bf16x2(f2_mul_rn(e2m1x2_to_f2(cl), s2)));
}
__device__ __forceinline__ uint32_t f8_pair_rec(uint32_t cl, uint64_t s2) {
  return bf16x2_plus_zero(f2_to_bf16x2(f2_mul_rn(e4m3x2_to_f2(cl), s2)));
}
// W_hat words of unit u (16 elements = 8 bf16 pairs) from the pairs as load_unit ordered them
// (swapped 16-byte halves when sw).
__device__ __forceinline__ void store_unit_words(uint32_t* out_words, int u, bool sw, const uint32_t (&r)[8]) {
  uint4* o = reinterpret_cast<uint4*>(out_words + 8 * (int64_t)u);
  const uint4 lo = make_uint4(r[0], r[1], r[2], r[3]), hi = make_uint4(r[4], r[5], r[6], r[7]);
  o[0] = sw ? hi : lo;
  o[1] = sw ? lo : hi;
}

__device__ __forceinline__ float nv_pair_sq(uint32_t v, uint32_t cl, uint64_t s2) {
  const uint32_t rec = f2_to_bf16x2(f2_mul_rn(e2m1x2_to_f2(cl), s2));
  return sq2_acc(bf16x2_sub(v, rec), 0.0f);
}
__device__ __forceinline__ float f8_pair_sq(uint32_t v, uint32_t cl, uint64_t s2) {
  const uint32_t rec = f2_to_bf16x2(f2_mul_rn(e4m3x2_to_f2(cl), s2));
  return sq2_acc(bf16x2_sub(v, rec), 0.0f);
}

// Weighted sums (predicted_dloss, measure_quant_cost.py:638-640: sum(H * err^2) with err the
// bf16 difference): H of the item's elements, one value per element or one per row.
struct HRef {
  const float* el;    // per element, from the item's first element (null: per row)
  const float* row;   // per row, from the item's first row
  int upr;
  uint32_t rdiv;
  // H of element k (0..15, element order) of unit u
  __device__ __forceinline__ float at(int u, int k) const {
    return el ? __ldg(el + 16 * (int64_t)u + k)
              : __ldg(row + (upr == 1 ? u : (int)__umulhi((uint32_t)u, rdiv)));
  }
};

// acc + h_lo e_lo^2 + h_hi e_hi^2 for a bf16 error pair (exact squares)
__device__ __forceinline__ float wsq2_acc(uint32_t e, float hlo, float hhi, float acc) {
  const float lo = __uint_as_float(e << 16), hi = __uint_as_float(e & 0xFFFF0000u);
  acc = __fmaf_rn(hlo, __fmul_rn(lo, lo), acc);
  return __fmaf_rn(hhi, __fmul_rn(hi, hi), acc);
}
__device__ __forceinline__ float nv_pair_wsq(uint32_t v, uint32_t cl, uint64_t s2, float h0, float h1) {
  const uint32_t rec = f2_to_bf16x2(f2_mul_rn(e2m1x2_to_f2(cl), s2));
  return wsq2_acc(bf16x2_sub(v, rec), h0, h1, 0.0f);
}
__device__ __forceinline__ float f8_pair_wsq(uint32_t v, uint32_t cl, uint64_t s2, float h0, float h1) {
  const uint32_t rec = f2_to_bf16x2(f2_mul_rn(e4m3x2_to_f2(cl), s2));
  return wsq2_acc(bf16x2_sub(v, rec), h0, h1, 0.0f);
}

// FP8 pair (16-bit code pair, low byte = low element), cost rule.
__device__ __forceinline__ uint32_t f8_resolve_pair(uint32_t vp, uint32_t cl, uint32_t ch, float s) {
  float ql0, ql1, qh0, qh1;
  f2_unpack(e4m3x2_to_f2(cl), ql0, ql1);
  f2_unpack(e4m3x2_to_f2(ch), qh0, qh1);
  const float w0 = bf16lo(vp), w1 = bf16hi(vp);
  const uint32_t d = cl ^ ch;
  uint32_t cx = cl;
  if (d & 0x00FFu) {
    bool up, dn;
    mid_side(fabsf(w0), ql0, qh0, s, up, dn);
    if (up || (!dn && w0 < 0.0f)) cx = (cx & 0xFF00u) | (ch & 0x00FFu);
  }
  if (d & 0xFF00u) {
    bool up, dn;
    mid_side(fabsf(w1), ql1, qh1, s, up, dn);
    if (up || (!dn && w1 < 0.0f)) cx = (cx & 0x00FFu) | (ch & 0xFF00u);
  }
  return cx;
}

// Units outside the fast path's range (amax below the 1e-8 scale floor, or
// large enough for an fp32 square to overflow): every element by IEEE
// division and the exact tie rules.  The main loop contributed nothing.
// H (weighted sums): the unit's weights, u its index; null for plain sums.
__device__ __noinline__ double nv_exact_unit(const uint32_t* vw, float a16, uint8_t* cu, bool cost, uint32_t* ou,
                                            const HRef* H = nullptr, int u = 0) {
  const float s = __fdiv_rn(fmaxf(a16, 1e-8f), 6.0f);
  const float se = fmaxf(__fdiv_rn(fmaxf(a16, 1e-12f), 6.0f), 1e-12f);   // export scale
  double delta = 0.0;
  for (int p = 0; p < 8; ++p) {
    const uint32_t vp = vw[p];
    const float w0 = bf16lo(vp), w1 = bf16hi(vp);
    if (cost || ou) {
      const float r0 = bf16_round(__fmul_rn(rtn_e2m1_cost(__fdiv_rn(w0, s)), s));
      const float r1 = bf16_round(__fmul_rn(rtn_e2m1_cost(__fdiv_rn(w1, s)), s));
      if (cost && H) {
        delta += (double)__fmaf_rn(H->at(u, 2 * p), sq_exact_err(w0, r0),
                                   __fmul_rn(H->at(u, 2 * p + 1), sq_exact_err(w1, r1)));
      } else if (cost) {
        delta += (double)(sq_exact_err(w0, r0) + sq_exact_err(w1, r1));
      }
      if (ou) ou[p] = (__float_as_uint(r0) >> 16) | (__float_as_uint(r1) & 0xFFFF0000u);
    }
    if (cu) cu[p] = (uint8_t)(nvfp4_code(__fdiv_rn(w0, se)) | (nvfp4_code(__fdiv_rn(w1, se)) << 4));
  }
  return delta;
}

__device__ __noinline__ double f8_exact_unit(const uint32_t* vw, float s, uint32_t* ou, const HRef* H = nullptr,
                                            int u = 0) {
  double delta = 0.0;
  for (int p = 0; p < 8; ++p) {
    const uint32_t vp = vw[p];
    const float w0 = bf16lo(vp), w1 = bf16hi(vp);
    const float r0 = bf16_round(__fmul_rn(rtn_e4m3_cost(__fdiv_rn(w0, s)), s));
    const float r1 = bf16_round(__fmul_rn(rtn_e4m3_cost(__fdiv_rn(w1, s)), s));
    if (H)
      delta += (double)__fmaf_rn(H->at(u, 2 * p), sq_exact_err(w0, r0),
                                 __fmul_rn(H->at(u, 2 * p + 1), sq_exact_err(w1, r1)));
    else
      delta += (double)(sq_exact_err(w0, r0) + sq_exact_err(w1, r1));
    if (ou) ou[p] = (__float_as_uint(r0) >> 16) | (__float_as_uint(r1) & 0xFFFF0000u);
  }
  return delta;
}

constexpr int FAST_TASK_CAP = 8 * 32;   // uncertain pairs of one 32-unit batch

// Inclusive warp prefix sum.
__device__ __forceinline__ int warp_incl_scan(int x, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(FULL, x, o);
    if (lane >= o) x += y;
  }
  return x;
}

// Warp-cooperative resolution of queued FP8 units (entry = unit index), in batches of 32 units:
// each lane finds its unit's pairs whose two bracket codes differ, a prefix sum packs them into
// the warp's task list, and the whole warp resolves the list, so a batch costs one round per 32
// pairs instead of one per pair of its busiest lane.  Each resolved pair adds its exact squared
// errors minus those of the main loop's provisional code (the lower bracket's) and, in W_hat
// launches, rewrites its reconstruction.
// Task word: pair (bits 0-2) | unit (3-14).
template <bool HW = false>
__device__ __forceinline__ double f8_fixup_body(const uint32_t* q0, int c0, const uint32_t* q1, int c1, const uint4* st,
                                               int lane, const uint32_t* ramax, int upr, uint32_t rdiv,
                                               uint32_t* tasks, int64_t elem0, uint32_t* outw, HRef H = HRef{}) {
  const int cnt = c0 + c1;
  double delta = 0.0;
  const uint32_t* words = reinterpret_cast<const uint32_t*>(st);
  for (int base = 0; base < cnt; base += 32) {   // warp-uniform
    const int i = base + lane;
    uint32_t pm = 0;
    int u = 0;
    if (i < cnt) {
      u = (int)(i < c0 ? q0[i] : q1[i - c0]);
      const RowParam rp = row_param(ramax[upr == 1 ? u : (int)__umulhi((uint32_t)u, rdiv)]);
      if (rp.amax >= F8_EXACT_ROW_AMAX) {
        delta += f8_exact_unit(words + 8 * u, rp.s, outw ? outw + (elem0 + 16 * (int64_t)u) / 2 : nullptr,
                               HW ? &H : nullptr, u);
      } else {
        const uint4 a = st[2 * u], b = st[2 * u + 1];
        const uint32_t v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        const uint64_t rlo2 = f2_pack(rp.r_lo, rp.r_lo), rhi2 = f2_pack(rp.r_hi, rp.r_hi);
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const uint64_t w2 = f2_from_bf16x2(v[p]);
          pm |= (cvt_e4m3x2(f2_mul_rz(w2, rlo2)) != cvt_e4m3x2(f2_mul_rz(w2, rhi2)) ? 1u : 0u) << p;
        }
      }
    }
    const int n = __popc(pm);
    const int incl = warp_incl_scan(n, lane);
    const int tot = __shfl_sync(FULL, incl, 31);
    int off = incl - n;
    for (uint32_t m = pm; m; m &= m - 1) tasks[off++] = (uint32_t)(__ffs(m) - 1) | ((uint32_t)u << 3);
    __syncwarp();
    float dl = 0.0f;
    for (int t = lane; t < tot; t += 32) {
      const uint32_t task = tasks[t];
      const int p = (int)(task & 7u), uu = (int)(task >> 3);
      const RowParam rp = row_param(ramax[upr == 1 ? uu : (int)__umulhi((uint32_t)uu, rdiv)]);
      const uint64_t rlo2 = f2_pack(rp.r_lo, rp.r_lo), rhi2 = f2_pack(rp.r_hi, rp.r_hi), s2 = f2_pack(rp.s, rp.s);
      const uint32_t vp = words[8 * uu + p];
      const uint64_t w2 = f2_from_bf16x2(vp);
      const uint64_t lo = f2_mul_rz(w2, rlo2), hi = f2_mul_rz(w2, rhi2);
      const uint32_t cl = cvt_e4m3x2(lo), ch = cvt_e4m3x2(hi);
      const uint32_t cp = cvt_e4m3x2(f2_min(lo, hi));   // the main loop's code
      const uint32_t cx = f8_resolve_pair(vp, cl, ch, rp.s);
      if (HW && cx != cp) {
        const float h0 = H.at(uu, 2 * p), h1 = H.at(uu, 2 * p + 1);
        dl += f8_pair_wsq(vp, cx, s2, h0, h1) - f8_pair_wsq(vp, cp, s2, h0, h1);
      } else if (cx != cp) {
        dl += f8_pair_sq(vp, cx, s2) - f8_pair_sq(vp, cp, s2);
      }
      if (outw && cx != cp) outw[(elem0 + 16 * (int64_t)uu) / 2 + p] = f8_pair_rec(cx, s2);
    }
    delta += (double)dl;
    __syncwarp();
  }
  return delta;
}

// Out-of-line copy for the rare early flush inside the per-unit loop (the loop body stays small);
// the end-of-item resolution inlines the body.
template <bool HW>
__device__ __noinline__ double f8_fixup(const uint32_t* q, int cnt, const uint4* st, int lane, const uint32_t* ramax,
                                        int upr, uint32_t rdiv, uint32_t* tasks, int64_t elem0, uint32_t* outw,
                                        HRef H) {
  return f8_fixup_body<HW>(q, cnt, q, 0, st, lane, ramax, upr, rdiv, tasks, elem0, outw, H);
}

// Tensor index of item `item`, scanning forward from the previous one (items
// of a CTA are visited in increasing order, so this is O(1) amortised).
__device__ __forceinline__ ItemRef next_item(const SweepLaunch& L, int64_t item, int& ti) {
  while (ti + 1 < L.n && L.item_prefix[ti + 1] <= item) ++ti;
  const SweepDesc& d = L.t[ti];
  const int64_t local = item - L.item_prefix[ti];
  ItemRef r;
  r.ti = ti;
  r.r0 = local * d.rows_per_item;
  r.nr = min((int64_t)d.rows_per_item, d.rows - r.r0);
  return r;
}

// Per-thread state of one work item.
struct ItemCtx {
  const uint4* st;
  int nunits, upr;
  uint32_t rdiv;
  uint8_t* codes_it;     // codes of the item's first element
  uint16_t* amax_it;     // group amax of the item's first group
  uint32_t* ramax;       // per-row max |w| (bf16 bits) of this item's rows
  uint32_t* tasks;       // the warp's fix-up task list
  int64_t elem0;
  // W_hat launches: each format's W_hat of the tensor as bf16 pairs, one slice per format present,
  // in format order (NVFP4, MXFP8, FP8 per channel); null otherwise
  uint32_t* outw;        // NVFP4
  uint32_t* outw_mx;     // MXFP8
  uint32_t* outw_f8;     // FP8 per channel
  uint32_t* outw_copy;   // the weight itself (copy_slice launches), after the format slices
  HRef h;                // weighted launches: the item's H
};

// H of unit u's 16 elements in load_unit's order (16-byte halves swapped when sw)
__device__ __forceinline__ void load_unit_h(const HRef& H, int u, bool sw, float (&h)[16]) {
  if (H.el) {
    const float4* p = reinterpret_cast<const float4*>(H.el + 16 * (int64_t)u);
    const float4 a = __ldg(p + (sw ? 2 : 0)), b = __ldg(p + (sw ? 3 : 1));
    const float4 c = __ldg(p + (sw ? 0 : 2)), d = __ldg(p + (sw ? 1 : 3));
    h[0] = a.x; h[1] = a.y; h[2] = a.z; h[3] = a.w; h[4] = b.x; h[5] = b.y; h[6] = b.z; h[7] = b.w;
    h[8] = c.x; h[9] = c.y; h[10] = c.z; h[11] = c.w; h[12] = d.x; h[13] = d.y; h[14] = d.z; h[15] = d.w;
  } else {
    const float x = H.at(u, 0);
#pragma unroll
    for (int i = 0; i < 16; ++i) h[i] = x;
  }
}

struct Accum {
  float nv, mx, f8;
  double dnv, dmx, df8;
  uint32_t tmax;
  int cnt_f8;
};

__device__ __forceinline__ int row_of(const ItemCtx& c, int u) {
  return c.upr == 1 ? u : (int)__umulhi((uint32_t)u, c.rdiv);   // exact for u < 4096 (host-checked)
}

// Pass A over one unit: NVFP4 cost and export codes, MXFP8 cost, and (when the
// FP8 format is on) the unit's contribution to its row maximum.
// HW: sums weighted by H (per element or per row).  OSSE (with OUT): the error sums as well.
template <bool NV, bool MX, bool F8, bool CODES, bool OUT, bool HW, bool OSSE>
__device__ __forceinline__ void unit_pass_a(const ItemCtx& c, int u, int lane, bool warp_rows, Accum& A) {
  const bool valid = u < c.nunits;
  const int uc = valid ? u : c.nunits - 1;
  uint32_t v[8];
  const bool sw = load_unit(c.st, uc, true, lane, v);
  if (OUT && c.outw_copy && valid) store_unit_words(c.outw_copy + c.elem0 / 2, uc, sw, v);
  float hv[16];
  if (HW && (NV || MX)) load_unit_h(c.h, uc, sw, hv);
  uint32_t a16b, amin = 0;
  if (MX) unit_absmax_min(v, a16b, amin); else a16b = unit_absmax(v);
  const float a16 = __uint_as_float(a16b << 16);

  if (NV || CODES) {
    const bool ex = exact_unit(a16);
    const float snv = div_const(fmaxf(a16, 1e-8f), 6.0f, RCP6);
    const float r = rcp_approx(snv);
    const float rlo = __fmul_rz(r, 1.0f - 9.5367431640625e-07f);   // 1 - 2^-20
    const uint64_t r2 = f2_pack(r, r), rlo2 = f2_pack(rlo, rlo), s2 = f2_pack(snv, snv);
    const uint64_t nb2 = f2_pack(-NV_COST_BIAS, -NV_COST_BIAS);
    uint32_t cw[2], q[8];
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {   // four pairs per conversion block
      float cc[8], l[8];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const uint64_t w2 = f2_from_bf16x2(v[4 * hf + p]);
        if (NV) f2_unpack(f2_fma_rn(w2, r2, nb2), cc[2 * p], cc[2 * p + 1]);
        if (CODES) f2_unpack(f2_mul_rz(w2, rlo2), l[2 * p], l[2 * p + 1]);
      }
      if (NV) nv_cost4(cc, *reinterpret_cast<uint32_t(*)[4]>(q + 4 * hf));
      if (CODES) cw[hf] = nv_export4(l);
    }
    if (NV) {
      float pe = 0.0f, po = 0.0f;   // two accumulation chains
      uint32_t recw[8];
#pragma unroll
      for (int p = 0; p < 8; ++p) {
        const uint32_t rec = f2_to_bf16x2(f2_mul_rn(f16x2_to_f2(q[p]), s2));
        if (OUT) recw[p] = bf16x2_plus_zero(rec);
        if (OUT && !OSSE) continue;
        if (HW && (p & 1)) po = wsq2_acc(bf16x2_sub(v[p], rec), hv[2 * p], hv[2 * p + 1], po);
        else if (HW) pe = wsq2_acc(bf16x2_sub(v[p], rec), hv[2 * p], hv[2 * p + 1], pe);
        else if (p & 1) po = sq2_acc(bf16x2_sub(v[p], rec), po);
        else pe = sq2_acc(bf16x2_sub(v[p], rec), pe);
      }
      if (OUT) {   // exact-path units are rewritten below
        if (valid) store_unit_words(c.outw + c.elem0 / 2, uc, sw, recw);
      }
      if (!OUT || OSSE) A.nv += (valid && !ex) ? pe + po : 0.0f;
    }
    if (CODES) {   // lanes past the end re-store the last unit's identical bytes
      reinterpret_cast<uint2*>(c.codes_it)[uc] = sw ? make_uint2(cw[1], cw[0]) : make_uint2(cw[0], cw[1]);
      c.amax_it[uc] = (uint16_t)a16b;
      A.tmax = max(A.tmax, a16b);
    }
    if (ex && valid) {   // rare: amax below the 1e-8 floor or near fp32 overflow; overwrites the unit
      A.dnv += nv_exact_unit(reinterpret_cast<const uint32_t*>(c.st) + 8 * uc, a16,
                             CODES ? c.codes_it + 8 * (int64_t)uc : nullptr, NV && (!OUT || OSSE),
                             (OUT && NV) ? c.outw + c.elem0 / 2 + 8 * (int64_t)uc : nullptr, HW ? &c.h : nullptr, uc);
    }
  }

  if (MX) {
    const uint32_t a32b = max(a16b, (uint32_t)__shfl_xor_sync(FULL, a16b, 1));
    const float a32 = __uint_as_float(a32b << 16);
    const int ea = (int)(a32b >> 7), ma = (int)(a32b & 0x7F);
    const int e = a32 < 1e-8f ? -35 : ea - 136 + (ma >= 31 ? 1 : 0);
    const uint32_t m448 = ((uint32_t)(e + 135) << 7) | 0x60u;   // bf16 bits of 448 * 2^e
    const uint32_t m448x2 = m448 | (m448 << 16);
    const bool ok = amin >= ((uint32_t)(e + 121) << 7);          // every |w| >= 2^(e-6): E4M3 normal range
    float pe = 0.0f, po = 0.0f;
    uint32_t recw[8];
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      // the magnitude rounded to 3 mantissa bits (a finite bf16 half never carries into its sign
      // bit or the next half).  The cost needs only the nearest value: a tie's two neighbours
      // are equally far, so half-up will do.  W_hat needs the reference's tie rule, to the lower
      // value: toward zero for w > 0, away from zero for w < 0.
      const uint32_t rq = OUT ? ((v[p] + 0x00070007u + ((v[p] >> 15) & 0x00010001u)) & 0xFFF0FFF0u)
                              : ((v[p] + 0x00080008u) & 0xFFF0FFF0u);
      const uint32_t q = bf16x2_minabs(rq, m448x2);                   // saturate |q| at 448 * 2^e
      if (OUT) recw[p] = bf16x2_plus_zero(q);
      if (OUT && !OSSE) continue;
      if (HW && (p & 1)) po = wsq2_acc(bf16x2_sub(v[p], q), hv[2 * p], hv[2 * p + 1], po);
      else if (HW) pe = wsq2_acc(bf16x2_sub(v[p], q), hv[2 * p], hv[2 * p + 1], pe);
      else if (p & 1) po = sq2_acc(bf16x2_sub(v[p], q), po);
      else pe = sq2_acc(bf16x2_sub(v[p], q), pe);
    }
    float part = pe + po;
    if (!ok && valid) {
      Chunk8 c0, c1;
      unit_to_chunks(v, c0, c1);
      uint32_t rec[8];
      if (OUT || HW) {
        const float p0 = mxfp8_cost8(c0, a32, rec);
#pragma unroll
        for (int i = 0; i < 4; ++i) recw[i] = rec[2 * i] | (rec[2 * i + 1] << 16);
        const float p1 = mxfp8_cost8(c1, a32, rec);
#pragma unroll
        for (int i = 0; i < 4; ++i) recw[4 + i] = rec[2 * i] | (rec[2 * i + 1] << 16);
        if (OSSE) part = p0 + p1;
        if (HW) {
          part = 0.0f;
#pragma unroll
          for (int p = 0; p < 8; ++p) part = wsq2_acc(bf16x2_sub(v[p], recw[p]), hv[2 * p], hv[2 * p + 1], part);
        }
      } else {
        part = mxfp8_cost8(c0, a32, rec) + mxfp8_cost8(c1, a32, rec);
      }
    }
    if (OUT) {
      if (valid) store_unit_words(c.outw_mx + c.elem0 / 2, uc, sw, recw);
    }
    if (!OUT || OSSE) A.mx += valid ? part : 0.0f;
  }

  if (F8) {   // row maxima for pass B
    const int row = row_of(c, uc);
    if (warp_rows) {   // the warp's 32 units lie in one row, all valid or all past the end
      const uint32_t m = warp_max_u(a16b);
      if (lane == 0 && u - lane < c.nunits) atomicMax(&c.ramax[row], m);
    } else if (valid) {
      atomicMax(&c.ramax[row], a16b);
    }
  }
}

// Pass B over one unit: FP8 per-channel cost with the completed row maximum.  The code is the
// lower bracket's; in flagged rows (row_param) both brackets are converted too, and a unit with a
// pair whose brackets differ is queued for the exact resolution.
template <bool OUT, bool HW, bool OSSE>
__device__ __forceinline__ void unit_pass_b(const ItemCtx& c, int u, int lane, uint32_t lanemask_lt, uint32_t* q_f8,
                                            Accum& A) {
  const bool valid = u < c.nunits;
  const int uc = valid ? u : c.nunits - 1;
  uint32_t v[8];
  const bool sw = load_unit(c.st, uc, true, lane, v);
  float hv[16];
  if (HW) load_unit_h(c.h, uc, sw, hv);
  const RowParam rp = row_param(c.ramax[row_of(c, uc)]);
  const uint64_t rlo2 = f2_pack(rp.r_lo, rp.r_lo), rhi2 = f2_pack(rp.r_hi, rp.r_hi), s2 = f2_pack(rp.s, rp.s);
  const bool exf = rp.amax >= F8_EXACT_ROW_AMAX;
  uint32_t ux = 0;
  float pe = 0.0f, po = 0.0f;
  uint32_t recw[8];
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {   // four pairs per conversion block
    float l[8], h[8], x[8];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint64_t w2 = f2_from_bf16x2(v[4 * hf + p]);
      f2_unpack(f2_mul_rz(w2, rlo2), l[2 * p], l[2 * p + 1]);
      f2_unpack(f2_mul_rz(w2, rhi2), h[2 * p], h[2 * p + 1]);
      x[2 * p] = fminf(l[2 * p], h[2 * p]);
      x[2 * p + 1] = fminf(l[2 * p + 1], h[2 * p + 1]);
    }
    uint32_t q[4];
    f8_codes_q4(x, q);
    if (rp.flag) {   // which pairs lie on a midpoint's bracket
      uint32_t dx, qq[4];
      f8_codes4(l, h, dx, qq);
      ux |= dx;
    }
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint32_t rec = f2_to_bf16x2(f2_mul_rn(f16x2_to_f2(q[p]), s2));
      const int pp = 4 * hf + p;
      if (OUT) recw[pp] = bf16x2_plus_zero(rec);
      if (OUT && !OSSE) continue;
      if (HW && (p & 1)) po = wsq2_acc(bf16x2_sub(v[pp], rec), hv[2 * pp], hv[2 * pp + 1], po);
      else if (HW) pe = wsq2_acc(bf16x2_sub(v[pp], rec), hv[2 * pp], hv[2 * pp + 1], pe);
      else if (p & 1) po = sq2_acc(bf16x2_sub(v[pp], rec), po);
      else pe = sq2_acc(bf16x2_sub(v[pp], rec), pe);
    }
  }
  if (OUT) {   // the queued pairs and exact-path rows are rewritten by the fix-ups
    if (valid) store_unit_words(c.outw_f8 + c.elem0 / 2, uc, sw, recw);
  }
  if (!OUT || OSSE) A.f8 += (valid && !exf) ? pe + po : 0.0f;
  const bool need = valid && (ux != 0 || exf);
  const uint32_t bal = __ballot_sync(FULL, need);
  if (bal) {
    if (need) q_f8[A.cnt_f8 + __popc(bal & lanemask_lt)] = (uint32_t)u;
    A.cnt_f8 += __popc(bal);
    if (A.cnt_f8 > FAST_QCAP - 32) {
      __syncwarp();
      A.df8 += f8_fixup<HW>(q_f8, A.cnt_f8, c.st, lane, c.ramax, c.upr, c.rdiv, c.tasks, c.elem0, c.outw_f8, c.h);
      __syncwarp();
      A.cnt_f8 = 0;
    }
  }
}

__device__ __forceinline__ void fold(float& f, double& d) {
  d += (double)f;
  f = 0.0f;
}

template <bool NV, bool MX, bool F8, bool CODES, bool OUT, bool HW, bool OSSE>
__global__ void __launch_bounds__(FAST_THREADS, 1) sweep_fast_kernel(const __grid_constant__ SweepLaunch L) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int NWARPS = FAST_THREADS / 32;
  uint8_t* stages = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + FAST_NSTAGE * FAST_STAGE_BYTES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + FAST_NSTAGE);
  uint32_t* ramax_buf = reinterpret_cast<uint32_t*>(bars + FAST_NSTAGE + 1);   // [2][FAST_MAX_ROWS]
  double* red = reinterpret_cast<double*>(ramax_buf + 2 * FAST_MAX_ROWS);
  uint32_t* qbase = reinterpret_cast<uint32_t*>(red + NWARPS * 3);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t* q_f8 = qbase + warp * FAST_QCAP;
  uint32_t* tasks = qbase + NWARPS * FAST_QCAP + warp * FAST_TASK_CAP;
  const uint32_t lanemask_lt = (1u << lane) - 1u;
  const int64_t n_items = L.item_prefix[L.n];
  const int64_t my_n = n_items > (int64_t)blockIdx.x ? (n_items - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;

  for (int i = tid; i < 2 * FAST_MAX_ROWS; i += FAST_THREADS) ramax_buf[i] = 0u;
  if (tid == 0) {
    for (int s = 0; s < FAST_NSTAGE; ++s) mbar_init(&bars[s], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  int ti_issue = 0;
  auto issue = [&](int64_t j) {
    const ItemRef it = next_item(L, (int64_t)blockIdx.x + j * gridDim.x, ti_issue);
    const SweepDesc& d = L.t[it.ti];
    const uint32_t bytes = (uint32_t)(it.nr * d.cols * 2);
    uint64_t* bar = &bars[j % FAST_NSTAGE];
    mbar_arrive_expect_tx(bar, bytes);
    bulk_g2s(stages + (j % FAST_NSTAGE) * FAST_STAGE_BYTES, d.w + it.r0 * d.cols, bytes, bar);
  };
  if (tid == 0)
    for (int64_t j = 0; j < FAST_NSTAGE && j < my_n; ++j) issue(j);

  Accum A;
  A.nv = A.mx = A.f8 = 0.0f;
  A.dnv = A.dmx = A.df8 = 0.0;
  A.tmax = 0u;
  A.cnt_f8 = 0;
  int cur_t = -1, ti_proc = 0;
  auto flush_tensor = [&](int t) {   // CTA-uniform call
    const SweepDesc& d = L.t[t];
    fold(A.nv, A.dnv);
    fold(A.mx, A.dmx);
    fold(A.f8, A.df8);
    const double a0 = warp_sum_d(A.dnv), a1 = warp_sum_d(A.dmx), a2 = warp_sum_d(A.df8);
    if (CODES) {
      const uint32_t m = warp_max_u(A.tmax);
      if (lane == 0) atomicMax(d.nvfp4_tmax, m << 16);
    }
    if (lane == 0) {
      red[warp * 3 + 0] = a0;
      red[warp * 3 + 1] = a1;
      red[warp * 3 + 2] = a2;
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
      for (int f = 0; f < 3; ++f) {
        double x = lane < NWARPS ? red[lane * 3 + f] : 0.0;
        x = warp_sum_d(x);
        if ((!OUT || OSSE) && lane == 0 && (d.fmt_mask & (1u << f))) atomicAdd(d.sse + f, x);
      }
    }
    __syncthreads();
    A.dnv = A.dmx = A.df8 = 0.0;
    A.tmax = 0u;
  };

  int64_t j_abort = -1;
  for (int64_t j = 0; j < my_n; ++j) {
    const int s = (int)(j % FAST_NSTAGE);
    const uint32_t parity = (uint32_t)((j / FAST_NSTAGE) & 1);
    const ItemRef it = next_item(L, (int64_t)blockIdx.x + j * gridDim.x, ti_proc);
    if (it.ti != cur_t) {
      if (cur_t >= 0) flush_tensor(cur_t);
      cur_t = it.ti;
    }
    const SweepDesc& d = L.t[it.ti];
    if (!mbar_wait_stage(&bars[s], parity)) {
      *abort_flag = 1;
      j_abort = j;
    }

    ItemCtx c;
    c.st = reinterpret_cast<const uint4*>(stages + s * FAST_STAGE_BYTES);
    c.upr = (int)(d.cols >> 4);
    c.nunits = (int)it.nr * c.upr;
    c.rdiv = 0xFFFFFFFFu / (uint32_t)c.upr + 1u;
    c.elem0 = it.r0 * d.cols;
    c.codes_it = CODES ? d.nvfp4_codes + c.elem0 / 2 : nullptr;
    c.amax_it = CODES ? d.nvfp4_amax + c.elem0 / 16 : nullptr;
    c.ramax = ramax_buf + (j & 1) * FAST_MAX_ROWS;
    c.tasks = tasks;
    c.h.el = (HW && !d.h_per_row) ? d.h + c.elem0 : nullptr;
    c.h.row = (HW && d.h_per_row) ? d.h + it.r0 : nullptr;
    c.h.upr = c.upr;
    c.h.rdiv = c.rdiv;
    {
      const int64_t slot = (L.out_slice > 0 ? L.out_slice : d.rows * d.cols) / 2;   // words between slices
      uint32_t* base = OUT ? reinterpret_cast<uint32_t*>(d.out) : nullptr;
      c.outw = (OUT && NV) ? base : nullptr;
      c.outw_mx = (OUT && MX) ? base + (NV ? slot : 0) : nullptr;
      c.outw_f8 = (OUT && F8) ? base + ((NV ? 1 : 0) + (MX ? 1 : 0)) * slot : nullptr;
      c.outw_copy = (OUT && L.copy_slice) ? base + ((NV ? 1 : 0) + (MX ? 1 : 0) + (F8 ? 1 : 0)) * slot : nullptr;
    }
    const int iters = (c.nunits + FAST_THREADS - 1) / FAST_THREADS;
    const bool warp_rows = (c.upr & 31) == 0;

    if (NV || MX || CODES || F8) {
#pragma unroll 1
      for (int k = 0; k < iters; ++k) {   // not unrolled: the body stays small enough for the instruction cache
        unit_pass_a<NV, MX, F8, CODES, OUT, HW, OSSE>(c, tid + k * FAST_THREADS, lane, warp_rows, A);
        if ((k & 3) == 3) {   // fp32 partials hold <= 64 squares
          fold(A.nv, A.dnv);
          fold(A.mx, A.dmx);
        }
      }
      fold(A.nv, A.dnv);
      fold(A.mx, A.dmx);
    }
    if (F8) {
      __syncthreads();   // row maxima complete; a failed wait is visible to every thread
      if (*abort_flag) {
        if (j_abort < 0) j_abort = j;
        break;
      }
      uint32_t* next = ramax_buf + ((j + 1) & 1) * FAST_MAX_ROWS;   // last read by item j-1
      for (int i = tid; i < FAST_MAX_ROWS; i += FAST_THREADS) next[i] = 0u;
#pragma unroll 1
      for (int k = 0; k < iters; ++k) {
        unit_pass_b<OUT, HW, OSSE>(c, tid + k * FAST_THREADS, lane, lanemask_lt, q_f8, A);
        if ((k & 3) == 3) fold(A.f8, A.df8);
      }
      fold(A.f8, A.df8);
    }
    __syncwarp();
    if (F8 && A.cnt_f8)   // the warp's own queued FP8 units (flagged rows, exact-path rows)
      A.df8 += f8_fixup_body<HW>(q_f8, A.cnt_f8, q_f8, 0, c.st, lane, c.ramax, c.upr, c.rdiv, c.tasks, c.elem0,
                                 c.outw_f8, c.h);
    A.cnt_f8 = 0;
    __syncthreads();   // stage s and the queues are free again
    if (*abort_flag) {
      if (j_abort < 0) j_abort = j;
      break;
    }
    if (tid == 0 && j + FAST_NSTAGE < my_n) {
      fence_proxy_async_smem();
      issue(j + FAST_NSTAGE);
    }
  }
  if (cur_t >= 0 && j_abort < 0) flush_tensor(cur_t);
  if (j_abort >= 0 && tid == 0) {
    for (int64_t jj = j_abort; jj < j_abort + FAST_NSTAGE && jj < my_n; ++jj)
      (void)mbar_wait_bounded(&bars[jj % FAST_NSTAGE], (uint32_t)((jj / FAST_NSTAGE) & 1), 1u << 20);
  }
}

size_t sweep_fast_smem_bytes() {
  return (size_t)FAST_NSTAGE * FAST_STAGE_BYTES + (FAST_NSTAGE + 1) * sizeof(uint64_t) +
         2 * FAST_MAX_ROWS * sizeof(uint32_t) + (FAST_THREADS / 32) * 3 * sizeof(double) +
         (FAST_THREADS / 32) * (FAST_QCAP + FAST_TASK_CAP) * sizeof(uint32_t);
}

template <bool NV, bool MX, bool F8, bool CODES, bool OUT = false, bool HW = false, bool OSSE = false>
static cudaError_t launch_fast_t(const SweepLaunch& L, int grid, cudaStream_t stream) {
  const size_t smem = sweep_fast_smem_bytes();
  cudaError_t e = cudaFuncSetAttribute(sweep_fast_kernel<NV, MX, F8, CODES, OUT, HW, OSSE>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  sweep_fast_kernel<NV, MX, F8, CODES, OUT, HW, OSSE><<<grid, FAST_THREADS, smem, stream>>>(L);
  return cudaGetLastError();
}

// All descriptors of L share the flag set `key` (format mask bits 0-2, bit 3 = NVFP4 codes, bit 4 =
// W_hat of each format in the mask into each descriptor's `out`, one slice per format in format
// order, no error sums; bit 5 = error sums weighted by each descriptor's `h`; bit 6 with bit 4 =
// W_hat and the plain error sums together).
cudaError_t launch_sweep_fast(const SweepLaunch& L, int grid, uint32_t key, cudaStream_t stream) {
  switch (key & 127u) {
    case 80 | 1: return launch_fast_t<true, false, false, false, true, false, true>(L, grid, stream);
    case 80 | 2: return launch_fast_t<false, true, false, false, true, false, true>(L, grid, stream);
    case 80 | 3: return launch_fast_t<true, true, false, false, true, false, true>(L, grid, stream);
    case 80 | 4: return launch_fast_t<false, false, true, false, true, false, true>(L, grid, stream);
    case 80 | 5: return launch_fast_t<true, false, true, false, true, false, true>(L, grid, stream);
    case 80 | 6: return launch_fast_t<false, true, true, false, true, false, true>(L, grid, stream);
    case 80 | 7: return launch_fast_t<true, true, true, false, true, false, true>(L, grid, stream);
    case 32 | 1: return launch_fast_t<true, false, false, false, false, true>(L, grid, stream);
    case 32 | 2: return launch_fast_t<false, true, false, false, false, true>(L, grid, stream);
    case 32 | 3: return launch_fast_t<true, true, false, false, false, true>(L, grid, stream);
    case 32 | 4: return launch_fast_t<false, false, true, false, false, true>(L, grid, stream);
    case 32 | 5: return launch_fast_t<true, false, true, false, false, true>(L, grid, stream);
    case 32 | 6: return launch_fast_t<false, true, true, false, false, true>(L, grid, stream);
    case 32 | 7: return launch_fast_t<true, true, true, false, false, true>(L, grid, stream);
    case 16 | 1: return launch_fast_t<true, false, false, false, true>(L, grid, stream);
    case 16 | 2: return launch_fast_t<false, true, false, false, true>(L, grid, stream);
    case 16 | 3: return launch_fast_t<true, true, false, false, true>(L, grid, stream);
    case 16 | 4: return launch_fast_t<false, false, true, false, true>(L, grid, stream);
    case 16 | 5: return launch_fast_t<true, false, true, false, true>(L, grid, stream);
    case 16 | 6: return launch_fast_t<false, true, true, false, true>(L, grid, stream);
    case 16 | 7: return launch_fast_t<true, true, true, false, true>(L, grid, stream);
#define PQ_CASE(K) \
  case K: return launch_fast_t<(K & 1) != 0, (K & 2) != 0, (K & 4) != 0, (K & 8) != 0>(L, grid, stream);
    PQ_CASE(1) PQ_CASE(2) PQ_CASE(3) PQ_CASE(4) PQ_CASE(5) PQ_CASE(6) PQ_CASE(7)
    PQ_CASE(8) PQ_CASE(9) PQ_CASE(10) PQ_CASE(11) PQ_CASE(12) PQ_CASE(13) PQ_CASE(14) PQ_CASE(15)
#undef PQ_CASE
    default: return cudaSuccess;
  }
}

}  // namespace pq
