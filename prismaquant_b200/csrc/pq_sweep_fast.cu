// Fast multi-format sweep (SSE mode): same work items, staging and outputs as
// sweep_staged_kernel<MODE_SSE>, with the per-element arithmetic rebuilt on
// packed sm_100a instructions (pq_fast.cuh):
//
//  * a thread owns a 16-element NVFP4 group ("unit", two 16-byte shared
//    loads); MXFP8 32-groups are lane pairs (one shuffle);
//  * NVFP4 cost: the code of fma(w, r, -2^-18) with r = rcp.approx(s), one
//    hardware conversion per pair.  w and the group max a have 8-bit
//    significands, so w / (a / 6) is either exactly an E2M1 midpoint or at
//    least ~2^-13 (relative) away from every midpoint; at an exact midpoint
//    the reference's fl32(w / s) IS the midpoint (a / 6 is exact unless the
//    midpoint is 0.75, and there the scale's rounding moves the quotient by
//    at most half an ulp of 0.75), so its nearest-with-ties-to-lower code is
//    "the code below", which the absolute bias toward -inf gives.  The NVFP4
//    export code (ties toward zero) is the code of RZ(w r_lo), r_lo just
//    below 1/s.  Both rules are checked against the reference rule on every
//    pair of bf16 values (tests/test_fast_rules.py);
//  * FP8 per channel: the code of min(RZ(w r_lo), RZ(w r_hi)), the bracket
//    product below the quotient, the same tie rule.  It is exact except in
//    rows where d = a - 448 s is 3 x 64 ulp(s) and s's significand is below
//    1.5: there the exact ties (448 w / a exactly a midpoint; with 7 not
//    dividing a's significand every such midpoint has significand 21/16, or
//    is 7 x 2^-10) have fl32 quotients off the midpoint when the significand
//    is below 1.125 (or, for 7 x 2^-10, below 1.5), and round up when d > 0,
//    down when d < 0.  Units of those rows convert both brackets too and
//    pick the reference's code per element in registers (f8_flag_select);
//    rows below the 1e-8 floor or near fp32 overflow take the exact path;
//  * the item is read twice from shared memory: a pre-pass takes every
//    unit's group maximum and minimum (kept in shared memory) and the row
//    maxima, one table per item holds each row's FP8 scale, reciprocal
//    brackets and flags, and then ONE pass per unit computes every format
//    from one unpack of its values;
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
//    (IEEE division, the reference's tie rules).  Every format's fast
//    arithmetic runs for every unit, and the rare units (exact path, MXFP8
//    values in the E4M3 subnormal range, flagged FP8 rows) are redone behind
//    one branch per unit (slow_unit), so the common path carries no other
//    divergent branch.
#include "pq_fast.cuh"
#include "pq_internal.h"

namespace pq {

constexpr int FAST_THREADS = SWEEP_THREADS;

// FP8 per-channel rows whose max |w| reaches this are done entirely by the
// exact path (a provisional fp32 square could overflow).
constexpr float F8_EXACT_ROW_AMAX = 1.152921504606846976e18f;  // 2^60

// One row's FP8 per-channel parameters (shared-memory table, one entry per row of the item).
struct RowTab {
  float s, r_lo, r_hi;
  uint32_t info;   // bit 0: exact-path row; 1: f7; 2: f21; 3: d > 0; bits 16-31: subnormal threshold
};
enum : uint32_t { RT_EXACT = 1u, RT_F7 = 2u, RT_F21 = 4u, RT_UP = 8u };

// FP8 per-channel row scale from the row's max |w| (bf16 bits): s = max(amax, 1e-8) / 448
// (div_const is exact for every normal bf16 value and for the 1e-8 floor), its reciprocal
// brackets, and where the lower-bracket rule needs help:
//  * exact-path rows: the max is below the floor (s is not amax / 448) or near fp32 overflow;
//  * d = amax - 448 s is exact as one FMA (a multiple of 64 ulp(s), at most 3 of them).  With
//    |d| = 3 x 64 ulp(s), an exact tie's fl32 quotient leaves the midpoint (up when d > 0, down
//    when d < 0) when s's significand is below 1.125 (f21: every tie of the row) or below 1.5
//    for the subnormal midpoint 7 x 2^-10 (f7); elsewhere it is a tie;
//  * the subnormal threshold: bf16 bits just above 2^-6 s; a unit whose smallest |w| is at or
//    above it cannot hold a subnormal tie.
__device__ __forceinline__ RowTab row_tab(uint32_t ra_bits) {
  RowTab t;
  const float amax = __uint_as_float(ra_bits << 16);
  t.s = div_const(fmaxf(amax, 1e-8f), 448.0f, RCP448);
  recip_bounds(t.s, t.r_lo, t.r_hi);
  const uint32_t sb = __float_as_uint(t.s);
  const float ulp = __uint_as_float((sb & 0x7F800000u) - (23u << 23));
  const float d = __fmaf_rn(-448.0f, t.s, amax);
  const bool j3 = fabsf(d) >= 160.0f * ulp;
  const uint32_t sig = sb & 0x7FFFFFu;
  uint32_t info = 0u;
  if (amax < 1e-8f || amax >= F8_EXACT_ROW_AMAX) info |= RT_EXACT;
  if (j3 && sig < 0x400000u) info |= RT_F7;
  if (j3 && sig < 0x100000u) info |= RT_F21;
  if (d > 0.0f) info |= RT_UP;
  const uint32_t thr = (__float_as_uint(__fmul_rn(t.s, 0.015625f)) >> 16) + 1u;   // 2^-6 s, rounded up
  t.info = info | (min(thr, 0x7F80u) << 16);
  return t;
}

// Loads unit u (16 bf16) from the stage into v[0..7], its two 16-byte halves in order.  (Lanes
// of a quarter-warp are 32 bytes apart, so the 128-bit loads meet a 2-way bank conflict, which
// the shared-memory pipe absorbs; swapping the halves of every other lane to avoid it cost
// selects on the ALU pipe, the one that binds: 0.6 % slower.)  Returns false: the halves were not
// swapped (the stores that mirror the load take this flag).
__device__ __forceinline__ bool load_unit(const uint4* st, int u, bool valid, int lane, uint32_t (&v)[8]) {
  (void)lane;
  uint4 a = make_uint4(0, 0, 0, 0), b = a;
  if (valid) {
    a = st[2 * u];
    b = st[2 * u + 1];
  }
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  return false;
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
  uint32_t* ab;          // per unit: group max |w| bits | group min |w| bits << 16 (pre-pass)
  const RowTab* rowtab;  // per row of the item: FP8 per-channel parameters
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
};

__device__ __forceinline__ int row_of(const ItemCtx& c, int u) {
  return c.upr == 1 ? u : (int)__umulhi((uint32_t)u, c.rdiv);   // exact for u < 4096 (host-checked)
}

// Pre-pass over one unit: its group max and min |w| into the item's table, and (with FP8 per
// channel, when a warp's 32 units lie in one row) the warp's share of the row maximum.  Items
// whose rows are not a multiple of 32 units take their row maxima from the table afterwards
// (build_row_table) instead of one shared-memory atomic per lane.
template <bool MINS, bool F8>
__device__ __forceinline__ void unit_prepass(const ItemCtx& c, int u, int lane, bool warp_rows) {
  const bool valid = u < c.nunits;
  const int uc = valid ? u : c.nunits - 1;
  uint32_t v[8];
  (void)load_unit(c.st, uc, true, lane, v);   // the order of the values does not matter here
  uint32_t a16b, amin = 0;
  if (MINS) unit_absmax_min(v, a16b, amin); else a16b = unit_absmax(v);
  if (valid) c.ab[uc] = a16b | (amin << 16);
  if (F8 && warp_rows) {   // the warp's 32 units lie in one row, all valid or all past the end
    const uint32_t m = warp_max_u(a16b);
    if (lane == 0 && u - lane < c.nunits) atomicMax(&c.ramax[row_of(c, uc)], m);
  }
}

// The FP8 per-channel row table of the item: warp w takes rows w, w + NWARPS, ...; each row's
// maximum is a warp max over its units' group maxima in the unit table, and lane k computes the
// table entry of the warp's k-th row, so the entries of one warp are computed side by side.  Not
// inlined: the main pass keeps its register allocation.
template <int NWARPS>
__device__ __noinline__ void build_row_table(const uint32_t* ab, int nr, int upr, int warp, int lane,
                                                RowTab* rowtab) {
  uint32_t mine = 0u;
  int myrow = -1, k = 0;
#pragma unroll 1
  for (int row = warp; row < nr; row += NWARPS, ++k) {   // at most FAST_MAX_ROWS / NWARPS < 32 rows
    const uint32_t* r = ab + (int64_t)row * upr;
    uint32_t m = 0u;
    for (int i = lane; i < upr; i += 32) m = max(m, r[i] & 0x7FFFu);
    m = warp_max_u(m);   // every lane arrives here
    if (lane == k) {
      mine = m;
      myrow = row;
    }
  }
  if (myrow >= 0) rowtab[myrow] = row_tab(mine);
}

// The rare per-unit work, all behind one branch of the main pass: NVFP4 units outside the fast
// range (nv_exact_unit), MXFP8 units with a value in the E4M3 subnormal range of their scale,
// FP8 per-channel rows outside the fast range (f8_exact_unit) and units of flagged FP8 rows
// (the reference's code per element from both brackets).  The main pass left nothing of these
// in the accumulators.  W_hat words (OUT) of each format handled here are stored here.
struct SlowSums {
  double nv, mx, f8;
};
// Everything is passed by value: the caller's state stays in registers on the common path.
template <bool NV, bool MX, bool F8, bool CODES, bool OUT, bool HW, bool OSSE>
__device__ __noinline__ SlowSums slow_unit(const ItemCtx c, int uc, int lane, uint32_t which, float a16, float a32,
                                           const RowTab rt) {
  SlowSums A{0.0, 0.0, 0.0};
  const uint32_t* vw = reinterpret_cast<const uint32_t*>(c.st) + 8 * uc;
  uint32_t v[8];
  const bool sw = load_unit(c.st, uc, true, lane, v);
  float hv[16];
  if (HW && (which & 6u)) load_unit_h(c.h, uc, sw, hv);
  if ((NV || CODES) && (which & 1u))
    A.nv += nv_exact_unit(vw, a16, CODES ? c.codes_it + 8 * (int64_t)uc : nullptr, NV && (!OUT || OSSE),
                           (OUT && NV) ? c.outw + c.elem0 / 2 + 8 * (int64_t)uc : nullptr, HW ? &c.h : nullptr, uc);
  if (MX && (which & 2u)) {
    Chunk8 c0, c1;
    unit_to_chunks(v, c0, c1);
    uint32_t rec[8], recw[8];
    const float p0 = mxfp8_cost8(c0, a32, rec);
#pragma unroll
    for (int i = 0; i < 4; ++i) recw[i] = rec[2 * i] | (rec[2 * i + 1] << 16);
    const float p1 = mxfp8_cost8(c1, a32, rec);
#pragma unroll
    for (int i = 0; i < 4; ++i) recw[4 + i] = rec[2 * i] | (rec[2 * i + 1] << 16);
    float part = p0 + p1;
    if (HW) {
      part = 0.0f;
#pragma unroll
      for (int p = 0; p < 8; ++p) part = wsq2_acc(bf16x2_sub(v[p], recw[p]), hv[2 * p], hv[2 * p + 1], part);
    }
    if (OUT) {
#pragma unroll
      for (int p = 0; p < 8; ++p) recw[p] = bf16x2_plus_zero(recw[p]);
      store_unit_words(c.outw_mx + c.elem0 / 2, uc, sw, recw);
    }
    if (!OUT || OSSE) A.mx += (double)part;
  }
  if (F8 && (which & 4u)) {
    if (rt.info & RT_EXACT) {
      A.f8 += f8_exact_unit(vw, rt.s, OUT ? c.outw_f8 + c.elem0 / 2 + 8 * (int64_t)uc : nullptr,
                            HW ? &c.h : nullptr, uc);
      return A;
    }
    const uint64_t rlo2 = f2_pack(rt.r_lo, rt.r_lo), rhi2 = f2_pack(rt.r_hi, rt.r_hi), s2 = f2_pack(rt.s, rt.s);
    const uint32_t all_mask = (rt.info & RT_F21) ? 0xFFFFFFFFu : 0u;
    const uint32_t up_mask = (rt.info & RT_UP) ? 0xFFFFFFFFu : 0u;
    float part = 0.0f;
    uint32_t recw[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {   // two pairs per 32-bit code word
      float l[4], h[4], x[4];
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const uint64_t w2 = f2_from_bf16x2(v[2 * k + p]);
        f2_unpack(f2_mul_rz(w2, rlo2), l[2 * p], l[2 * p + 1]);
        f2_unpack(f2_mul_rz(w2, rhi2), h[2 * p], h[2 * p + 1]);
        x[2 * p] = fminf(l[2 * p], h[2 * p]);
        x[2 * p + 1] = fminf(l[2 * p + 1], h[2 * p + 1]);
      }
      const uint32_t cl = f8_codes2(l[0], l[1], l[2], l[3]);
      const uint32_t ch = f8_codes2(h[0], h[1], h[2], h[3]);
      const uint32_t cm = f8_codes2(x[0], x[1], x[2], x[3]);
      uint32_t q[2];
      f8_decode2(f8_flag_select(cl, ch, cm, all_mask, up_mask), q[0], q[1]);
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const int pp = 2 * k + p;
        const uint32_t rec = f2_to_bf16x2(f2_mul_rn(f16x2_to_f2(q[p]), s2));
        if (OUT) recw[pp] = bf16x2_plus_zero(rec);
        if (OUT && !OSSE) continue;
        if (HW) part = wsq2_acc(bf16x2_sub(v[pp], rec), hv[2 * pp], hv[2 * pp + 1], part);
        else part = sq2_acc(bf16x2_sub(v[pp], rec), part);
      }
    }
    if (OUT) store_unit_words(c.outw_f8 + c.elem0 / 2, uc, sw, recw);
    if (!OUT || OSSE) A.f8 += (double)part;
  }
  return A;
}

// The one pass over a unit: NVFP4 cost and export codes, MXFP8 cost and FP8 per-channel cost from
// one load and one unpack of its 16 values, with the group extrema of the pre-pass and the row
// table.  HW: sums weighted by H (per element or per row).  OSSE (with OUT): the error sums too.
// Every format's fast arithmetic runs for every unit; units the fast rules do not cover are left
// out of the sums here (their W_hat words are stored by slow_unit after these) and redone by
// slow_unit behind a single branch.
template <bool NV, bool MX, bool F8, bool CODES, bool OUT, bool HW, bool OSSE>
__device__ __forceinline__ void unit_main(const ItemCtx& c, int u, int lane, Accum& A) {
  const bool valid = u < c.nunits;
  const int uc = valid ? u : c.nunits - 1;
  uint32_t v[8];
  const bool sw = load_unit(c.st, uc, true, lane, v);
  if (OUT && c.outw_copy && valid) store_unit_words(c.outw_copy + c.elem0 / 2, uc, sw, v);
  float hv[16];
  if (HW) load_unit_h(c.h, uc, sw, hv);
  const uint32_t ab = c.ab[uc];
  const uint32_t a16b = ab & 0xFFFFu, amin = ab >> 16;
  const float a16 = __uint_as_float(a16b << 16);
  uint64_t w2[8];
  if (NV || CODES || F8) {
#pragma unroll
    for (int p = 0; p < 8; ++p) w2[p] = f2_from_bf16x2(v[p]);
  }
  uint32_t which = 0u;   // bit 0: NVFP4 exact unit, 1: MXFP8 exact unit, 2: FP8 exact row or flagged unit

  if (NV || CODES) {
    const bool ex = exact_unit(a16);
    which |= ex ? 1u : 0u;
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
        if (NV) f2_unpack(f2_fma_rn(w2[4 * hf + p], r2, nb2), cc[2 * p], cc[2 * p + 1]);
        if (CODES) f2_unpack(f2_mul_rz(w2[4 * hf + p], rlo2), l[2 * p], l[2 * p + 1]);
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
      if (OUT) {   // exact-path units are rewritten by slow_unit
        if (valid) store_unit_words(c.outw + c.elem0 / 2, uc, sw, recw);
      }
      if (!OUT || OSSE) A.nv += (valid && !ex) ? pe + po : 0.0f;
    }
    if (CODES) {   // lanes past the end re-store the last unit's identical bytes
      reinterpret_cast<uint2*>(c.codes_it)[uc] = sw ? make_uint2(cw[1], cw[0]) : make_uint2(cw[0], cw[1]);
      c.amax_it[uc] = (uint16_t)a16b;
      A.tmax = max(A.tmax, a16b);
    }
  }

  float a32 = 0.0f;
  if (MX) {
    const uint32_t a32b = max(a16b, (uint32_t)__shfl_xor_sync(FULL, a16b, 1));
    a32 = __uint_as_float(a32b << 16);
    const int ea = (int)(a32b >> 7), ma = (int)(a32b & 0x7F);
    const int e = a32 < 1e-8f ? -35 : ea - 136 + (ma >= 31 ? 1 : 0);
    const uint32_t m448 = ((uint32_t)(e + 135) << 7) | 0x60u;   // bf16 bits of 448 * 2^e
    const uint32_t m448x2 = m448 | (m448 << 16);
    const bool ok = amin >= ((uint32_t)(e + 121) << 7);          // every |w| >= 2^(e-6): E4M3 normal range
    which |= ok ? 0u : 2u;
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
    if (OUT) {   // units with subnormal-range values are rewritten by slow_unit
      if (valid) store_unit_words(c.outw_mx + c.elem0 / 2, uc, sw, recw);
    }
    if (!OUT || OSSE) A.mx += (valid && ok) ? pe + po : 0.0f;
  }

  RowTab rt{0.0f, 0.0f, 0.0f, 0u};
  if (F8) {
    rt = c.rowtab[row_of(c, uc)];
    // ties may leave their midpoint: every tie in f21 rows, the subnormal midpoint's in f7 rows (only
    // a unit holding a |w| below 2^-6 s can have one); exact-path rows are redone entirely
    const bool other = (rt.info & (RT_EXACT | RT_F21)) || ((rt.info & RT_F7) && amin < (rt.info >> 16));
    which |= other ? 4u : 0u;
    const uint64_t rlo2 = f2_pack(rt.r_lo, rt.r_lo), rhi2 = f2_pack(rt.r_hi, rt.r_hi), s2 = f2_pack(rt.s, rt.s);
    float pe = 0.0f, po = 0.0f;
    uint32_t recw[8];
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {   // four pairs per conversion block
      float x[8];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        float l0, l1, h0, h1;
        f2_unpack(f2_mul_rz(w2[4 * hf + p], rlo2), l0, l1);
        f2_unpack(f2_mul_rz(w2[4 * hf + p], rhi2), h0, h1);
        x[2 * p] = fminf(l0, h0);
        x[2 * p + 1] = fminf(l1, h1);
      }
      uint32_t q[4];
      f8_codes_q4(x, q);
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
    if (OUT) {   // exact rows and flagged units are rewritten by slow_unit
      if (valid) store_unit_words(c.outw_f8 + c.elem0 / 2, uc, sw, recw);
    }
    if (!OUT || OSSE) A.f8 += (valid && !other) ? pe + po : 0.0f;
  }

  if (valid && which) {
    const SlowSums d = slow_unit<NV, MX, F8, CODES, OUT, HW, OSSE>(c, uc, lane, which, a16, a32, rt);
    A.dnv += d.nv;
    A.dmx += d.mx;
    A.df8 += d.f8;
  }
}

__device__ __forceinline__ void fold(float& f, double& d) {
  d += (double)f;
  f = 0.0f;
}

constexpr int FAST_MAX_UNITS = FAST_STAGE_BYTES / 32;   // 16-element units per item

template <bool NV, bool MX, bool F8, bool CODES, bool OUT, bool HW, bool OSSE>
__global__ void __launch_bounds__(FAST_THREADS, 1) sweep_fast_kernel(const __grid_constant__ SweepLaunch L) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int NWARPS = FAST_THREADS / 32;
  uint8_t* stages = smem;
  RowTab* rowtab = reinterpret_cast<RowTab*>(smem + FAST_NSTAGE * FAST_STAGE_BYTES);   // [FAST_MAX_ROWS]
  uint32_t* ab = reinterpret_cast<uint32_t*>(rowtab + FAST_MAX_ROWS);                   // [FAST_MAX_UNITS]
  uint32_t* ramax = ab + FAST_MAX_UNITS;                                                // [FAST_MAX_ROWS]
  double* red = reinterpret_cast<double*>(ramax + FAST_MAX_ROWS);                       // [NWARPS][3]
  uint64_t* bars = reinterpret_cast<uint64_t*>(red + NWARPS * 3);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + FAST_NSTAGE);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t n_items = L.item_prefix[L.n];
  const int64_t my_n = n_items > (int64_t)blockIdx.x ? (n_items - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;

  for (int i = tid; i < FAST_MAX_ROWS; i += FAST_THREADS) ramax[i] = 0u;
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
    c.ramax = ramax;
    c.ab = ab;
    c.rowtab = rowtab;
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

    // pre-pass: group extrema of every unit (a thread reads back only its own units) and row maxima
#pragma unroll 1
    for (int k = 0; k < iters; ++k) unit_prepass<MX || F8, F8>(c, tid + k * FAST_THREADS, lane, warp_rows);
    if (F8) {
      __syncthreads();   // row maxima complete; a failed wait is visible to every thread
      if (*abort_flag) {
        if (j_abort < 0) j_abort = j;
        break;
      }
      if (warp_rows) {
        for (int i = tid; i < (int)it.nr; i += FAST_THREADS) {
          rowtab[i] = row_tab(ramax[i]);
          ramax[i] = 0u;   // ready for the next item's pre-pass
        }
      } else {
        build_row_table<NWARPS>(c.ab, (int)it.nr, c.upr, warp, lane, rowtab);
      }
      __syncthreads();   // row table complete
    }
    // not unrolled: the body stays small enough for the instruction cache.  The fp32 partials
    // hold <= 64 squares (four units); the fold sits in the outer loop, so it runs once per four
    // units instead of as predicated instructions in every iteration
#pragma unroll 1
    for (int k0 = 0; k0 < iters; k0 += 4) {
      const int k1 = min(k0 + 4, iters);
#pragma unroll 1
      for (int k = k0; k < k1; ++k) unit_main<NV, MX, F8, CODES, OUT, HW, OSSE>(c, tid + k * FAST_THREADS, lane, A);
      fold(A.nv, A.dnv);
      fold(A.mx, A.dmx);
      fold(A.f8, A.df8);
    }
    __syncthreads();   // stage s, the unit table and the row table are free again
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
  return (size_t)FAST_NSTAGE * FAST_STAGE_BYTES + FAST_MAX_ROWS * sizeof(RowTab) +
         (FAST_MAX_UNITS + FAST_MAX_ROWS) * sizeof(uint32_t) + (FAST_THREADS / 32) * 3 * sizeof(double) +
         (FAST_NSTAGE + 1) * sizeof(uint64_t);
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
