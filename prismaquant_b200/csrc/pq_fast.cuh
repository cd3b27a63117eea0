// Packed-arithmetic building blocks of the fast sweep path (sm_100a PTX).
//
// The fast path never computes w / s.  For a group scale s it brackets the
// exact quotient between two round-toward-zero products with widened
// reciprocal bounds, L = RZ(w * r_lo) and H = RZ(w * r_hi), and converts both
// with the hardware round-to-nearest FP4 / FP8 conversions.  If the two codes
// agree, every real number in [L, H] — the exact w / s and its float32
// rounding included — rounds to that code and no codebook midpoint lies in
// [L, H]; so it is also the reference's nearest-with-ties-to-lower (cost) and
// nearest-with-ties-toward-zero (export) code.  If they differ the element is
// within ~2^-20 (relative) of a midpoint and the unit is redone with IEEE
// division and the exact tie rules (pq_common.cuh).
//
// Bracket proof sketch: r = rcp.approx(s) is within 1 ulp of 1/s (PTX ISA
// bound); r_lo = RZ(r (1 - 2^-20)) < (1 - 2^-21)/s and r_hi = RZ(r (1 + 2^-20))
// > (1 + 2^-21)/s, hence |L| < |w/s| (1 - 2^-21) and |H| > |w/s| (1 + 2^-22).
// A float32 quotient equal to a midpoint m has |w/s| within m (1 +- 2^-24),
// so |L| < m < |H| strictly and the two conversions differ.
#pragma once
#include "pq_common.cuh"

namespace pq {

__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
// bf16 pair {lo, hi} (one 32-bit word) -> float32 pair
// (each half as v * 1 + (-0), one mixed-precision FMA: exact, keeps -0, and
// runs on the FMA pipe instead of the integer shift/mask units)
__device__ __forceinline__ uint64_t f2_from_bf16x2(uint32_t v) {
  float lo, hi;
  asm("{\n\t.reg .b16 a, b, one;\n\tmov.b32 {a, b}, %2;\n\tmov.b16 one, 0x3F80;\n\t"
      "fma.rn.f32.bf16 %0, a, one, 0f80000000;\n\tfma.rn.f32.bf16 %1, b, one, 0f80000000;\n\t}"
      : "=f"(lo), "=f"(hi) : "r"(v));
  return f2_pack(lo, hi);
}
__device__ __forceinline__ uint64_t f2_mul_rz(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rz.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul_rn(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ uint64_t f2_add_rn(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_fma_rn(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// per-element minimum of two float32 pairs
__device__ __forceinline__ uint64_t f2_min(uint64_t a, uint64_t b) {
  float a0, a1, b0, b1;
  f2_unpack(a, a0, a1);
  f2_unpack(b, b0, b1);
  return f2_pack(fminf(a0, b0), fminf(a1, b1));
}

// FP4 E2M1 pair, round-to-nearest-even, saturating at 6: low nibble = lo.
__device__ __forceinline__ uint32_t cvt_e2m1x2(uint64_t x) {
  float lo, hi;
  f2_unpack(x, lo, hi);
  uint16_t r;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u16.u8 %0, t;\n\t}" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
// FP8 E4M3 pair, round-to-nearest-even, saturating at 448: low byte = lo.
__device__ __forceinline__ uint32_t cvt_e4m3x2(uint64_t x) {
  float lo, hi;
  f2_unpack(x, lo, hi);
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
// FP8 E5M2 pair, round-to-nearest-even, saturating at 57344: low byte = lo.
__device__ __forceinline__ uint32_t cvt_e5m2x2(uint64_t x) {
  float lo, hi;
  f2_unpack(x, lo, hi);
  uint16_t r;
  asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
// Code pair -> float32 pair (exact: both formats embed in f16).
__device__ __forceinline__ uint64_t e2m1x2_to_f2(uint32_t c) {
  uint32_t h;
  asm("{\n\t.reg .b8 t;\n\tcvt.u8.u16 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}" : "=r"(h) : "h"((uint16_t)c));
  float lo, hi;
  asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\tcvt.f32.f16 %0, a;\n\tcvt.f32.f16 %1, b;\n\t}"
      : "=f"(lo), "=f"(hi) : "r"(h));
  return f2_pack(lo, hi);
}
__device__ __forceinline__ uint64_t e4m3x2_to_f2(uint32_t c) {
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"((uint16_t)c));
  float lo, hi;
  asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\tcvt.f32.f16 %0, a;\n\tcvt.f32.f16 %1, b;\n\t}"
      : "=f"(lo), "=f"(hi) : "r"(h));
  return f2_pack(lo, hi);
}
// f16 pair (one 32-bit word) -> float32 pair (exact).
__device__ __forceinline__ uint64_t f16x2_to_f2(uint32_t h) {
  float lo, hi;
  asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\tcvt.f32.f16 %0, a;\n\tcvt.f32.f16 %1, b;\n\t}"
      : "=f"(lo), "=f"(hi) : "r"(h));
  return f2_pack(lo, hi);
}

// Four NVFP4 pairs at once, codes kept in byte registers: l[2p], l[2p+1] are
// the low-bracket products of pair p, h[] the high ones.  cw gets the four
// low-bracket code bytes (pair p in byte p), dx = cw ^ the high-bracket
// bytes, q[p] the f16 pair of pair p's low-bracket code.
__device__ __forceinline__ void nv_codes4(const float (&l)[8], const float (&h)[8], uint32_t& cw, uint32_t& dx,
                                          uint32_t (&q)[4]) {
  asm("{\n\t.reg .b8 c0, c1, c2, c3, d0, d1, d2, d3;\n\t.reg .b32 t;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 c0, %7, %6;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 c1, %9, %8;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 c2, %11, %10;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 c3, %13, %12;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 d0, %15, %14;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 d1, %17, %16;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 d2, %19, %18;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 d3, %21, %20;\n\t"
      "mov.b32 %0, {c0, c1, c2, c3};\n\t"
      "mov.b32 t, {d0, d1, d2, d3};\n\t"
      "xor.b32 %1, %0, t;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, c0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, c1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %4, c2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %5, c3;\n\t}"
      : "=r"(cw), "=r"(dx), "=r"(q[0]), "=r"(q[1]), "=r"(q[2]), "=r"(q[3])
      : "f"(l[0]), "f"(l[1]), "f"(l[2]), "f"(l[3]), "f"(l[4]), "f"(l[5]), "f"(l[6]), "f"(l[7]),
        "f"(h[0]), "f"(h[1]), "f"(h[2]), "f"(h[3]), "f"(h[4]), "f"(h[5]), "f"(h[6]), "f"(h[7]));
}

// Four NVFP4 pairs of biased cost products c (pair p = c[2p], c[2p+1]): q[p] the f16 pair of the
// pair's E2M1 codes.
__device__ __forceinline__ void nv_cost4(const float (&c)[8], uint32_t (&q)[4]) {
  asm("{\n\t.reg .b8 c0, c1, c2, c3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 c0, %5, %4;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 c1, %7, %6;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 c2, %9, %8;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 c3, %11, %10;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, c0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, c1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, c2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, c3;\n\t}"
      : "=r"(q[0]), "=r"(q[1]), "=r"(q[2]), "=r"(q[3])
      : "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]), "f"(c[4]), "f"(c[5]), "f"(c[6]), "f"(c[7]));
}

// Four NVFP4 pairs of export products l: the four code bytes (pair p in byte p).
__device__ __forceinline__ uint32_t nv_export4(const float (&l)[8]) {
  uint32_t cw;
  asm("{\n\t.reg .b8 c0, c1, c2, c3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 c0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 c1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 c2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 c3, %8, %7;\n\t"
      "mov.b32 %0, {c0, c1, c2, c3};\n\t}"
      : "=r"(cw)
      : "f"(l[0]), "f"(l[1]), "f"(l[2]), "f"(l[3]), "f"(l[4]), "f"(l[5]), "f"(l[6]), "f"(l[7]));
  return cw;
}

// Four FP8 (E4M3) pairs of products x: q[p] the f16 pair of pair p's codes.
__device__ __forceinline__ void f8_codes_q4(const float (&x)[8], uint32_t (&q)[4]) {
  asm("{\n\t.reg .b16 c0, c1, c2, c3;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 c0, %5, %4;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 c1, %7, %6;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 c2, %9, %8;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 c3, %11, %10;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, c0;\n\t"
      "cvt.rn.f16x2.e4m3x2 %1, c1;\n\t"
      "cvt.rn.f16x2.e4m3x2 %2, c2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %3, c3;\n\t}"
      : "=r"(q[0]), "=r"(q[1]), "=r"(q[2]), "=r"(q[3])
      : "f"(x[0]), "f"(x[1]), "f"(x[2]), "f"(x[3]), "f"(x[4]), "f"(x[5]), "f"(x[6]), "f"(x[7]));
}

// Four FP8 (E4M3) pairs at once: dx is nonzero iff some pair's bracket codes
// differ, q[p] the f16 pair of pair p's low-bracket code.
__device__ __forceinline__ void f8_codes4(const float (&l)[8], const float (&h)[8], uint32_t& dx, uint32_t (&q)[4]) {
  asm("{\n\t.reg .b16 c0, c1, c2, c3, d0, d1, d2, d3;\n\t.reg .b32 t0, t1, u0, u1;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 c0, %6, %5;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 c1, %8, %7;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 c2, %10, %9;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 c3, %12, %11;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 d0, %14, %13;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 d1, %16, %15;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 d2, %18, %17;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 d3, %20, %19;\n\t"
      "mov.b32 t0, {c0, c1};\n\t"
      "mov.b32 t1, {c2, c3};\n\t"
      "mov.b32 u0, {d0, d1};\n\t"
      "mov.b32 u1, {d2, d3};\n\t"
      "xor.b32 t0, t0, u0;\n\t"
      "xor.b32 t1, t1, u1;\n\t"
      "or.b32 %0, t0, t1;\n\t"
      "cvt.rn.f16x2.e4m3x2 %1, c0;\n\t"
      "cvt.rn.f16x2.e4m3x2 %2, c1;\n\t"
      "cvt.rn.f16x2.e4m3x2 %3, c2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %4, c3;\n\t}"
      : "=r"(dx), "=r"(q[0]), "=r"(q[1]), "=r"(q[2]), "=r"(q[3])
      : "f"(l[0]), "f"(l[1]), "f"(l[2]), "f"(l[3]), "f"(l[4]), "f"(l[5]), "f"(l[6]), "f"(l[7]),
        "f"(h[0]), "f"(h[1]), "f"(h[2]), "f"(h[3]), "f"(h[4]), "f"(h[5]), "f"(h[6]), "f"(h[7]));
}

// E4M3 codes of two pairs (x0, x1) and (x2, x3): pair 0 in the low 16 bits, low byte = x0.
__device__ __forceinline__ uint32_t f8_codes2(float x0, float x1, float x2, float x3) {
  uint32_t r;
  asm("{\n\t.reg .b16 a, b;\n\tcvt.rn.satfinite.e4m3x2.f32 a, %2, %1;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 b, %4, %3;\n\tmov.b32 %0, {a, b};\n\t}"
      : "=r"(r) : "f"(x0), "f"(x1), "f"(x2), "f"(x3));
  return r;
}
// f16 pairs of the two code pairs packed as f8_codes2 packs them.
__device__ __forceinline__ void f8_decode2(uint32_t c, uint32_t& q0, uint32_t& q1) {
  asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\tcvt.rn.f16x2.e4m3x2 %0, a;\n\t"
      "cvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
      : "=r"(q0), "=r"(q1) : "r"(c));
}

// The reference's E4M3 codes of four elements of a flagged FP8 row (bytes of a word), from the
// codes of the lower bracket (cl), the upper bracket (ch) and the lower-bracket rule (cm).  An
// element whose two bracket codes differ is an exact tie; it takes the code on the side the
// reference's fl32 quotient falls (the upper code when `up_mask` is all ones, the lower one
// otherwise) when `all_mask` is all ones (every tie of the row leaves its midpoint) or when its
// lower code is subnormal (only the subnormal midpoint's ties do); every other element keeps cm.
// Byte-wise tests without carries between bytes: a byte y <= 0x7F is nonzero iff bit 7 of
// (y + 0x7F) | y is set.
__device__ __forceinline__ uint32_t f8_flag_select(uint32_t cl, uint32_t ch, uint32_t cm, uint32_t all_mask,
                                                   uint32_t up_mask) {
  const uint32_t e = cl & 0x78787878u;                     // exponent fields
  const uint32_t nze = (e + 0x7F7F7F7Fu) | e;              // bit 7: normal lower code
  const uint32_t u = cl ^ ch;                              // same signs, so bytes <= 0x7F
  const uint32_t nzu = (u + 0x7F7F7F7Fu) | u;              // bit 7: the bracket codes differ
  const uint32_t sel = nzu & (all_mask | ~nze) & 0x80808080u;
  const uint32_t m = (sel >> 7) * 0xFFu;
  const uint32_t alt = (ch & up_mask) | (cl & ~up_mask);
  return (cm & ~m) | (alt & m);
}

// One E4M3 code byte -> float32 (exact).
__device__ __forceinline__ float e4m3x2_to_f2_lo(uint32_t c) {
  float lo, hi;
  f2_unpack(e4m3x2_to_f2(c & 0xFFu), lo, hi);
  return lo;
}
// float32 pair -> bf16 pair, RNE (low half = lo).
__device__ __forceinline__ uint32_t f2_to_bf16x2(uint64_t x) {
  float lo, hi;
  f2_unpack(x, lo, hi);
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// Each 16-bit half set to all ones where its bit 15 is set, else zero: PTX prmt in its generic
// mode, where a selector nibble with bit 3 set replicates the sign bit of the chosen byte
// (bytes 1 and 3 here).  (CUDA's __byte_perm reads only the low 3 bits of each nibble.)
__device__ __forceinline__ uint32_t prmt_sign_halves(uint32_t x) {
  uint32_t d;
  asm("prmt.b32 %0, %1, 0, 0xBB99;" : "=r"(d) : "r"(x));
  return d;
}
__device__ __forceinline__ uint32_t bf16x2_add(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// max(|a|, |b|) per half (sign = sign(a) ^ sign(b)); on magnitudes it is the magnitude max.
__device__ __forceinline__ uint32_t bf16x2_maxabs(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf16x2_minabs(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("min.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// acc += lo^2 + hi^2 of a bf16 pair (exact bf16 products, fp32 accumulate).
__device__ __forceinline__ float sq2_acc(uint32_t e, float acc) {
  asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %1;\n\tfma.rn.f32.bf16 %0, a, a, %0;\n\tfma.rn.f32.bf16 %0, b, b, %0;\n\t}"
      : "+f"(acc) : "r"(e));
  return acc;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

constexpr float RCP6 = 0.16666667163372039794921875f;   // RN(1/6)
constexpr float RCP448 = 0x1.24924ap-9f;                // RN(1/448)
constexpr float RCP3 = 0x1.555556p-2f;                  // RN(1/3)
constexpr float RCP7 = 0x1.24924ap-3f;                  // RN(1/7)

// RN(a / d) for a normal bf16 value a and d in {3, 6, 7, 448}, with rd = RN(1/d):
// product plus one remainder correction (Markstein); checked exhaustively
// against IEEE division over all normal bf16 inputs and the floors 1e-8 and 1e-12
// (tests/test_fast_rules.py).
__device__ __forceinline__ float div_const(float a, float d, float rd) {
  const float q = __fmul_rn(a, rd);
  const float r = __fmaf_rn(-q, d, a);
  return __fmaf_rn(r, rd, q);
}

// Exact side of an uncertain quotient a / s (a, s > 0 float32).  The bracket
// codes of a / s are the neighbours qlo < qhi (magnitudes) with midpoint m
// between them, and |a / s - m| <= 2^-19 m, so r = a - m s is exact as one
// FMA: m has at most 5 significant bits and s 24, so r is an integer multiple
// of the finer of ulp(a) and ulp(m) ulp(s), and |r| <= 2^-19 a is below 2^11
// of those units.  The reference rounds q = fl(a / s) and compares it with m
// (m has a short mantissa, so it is an even float32):
//   q > m  <=>  a / s > m + ulp(m) / 2   <=>  r > s ulp(m) / 2        (up)
//   q < m  <=>  a / s < m - ulp-(m) / 2  <=>  r < -s ulp-(m) / 2      (dn)
// and q == m otherwise (a tie); ulp-(m) is the spacing below m, half of
// ulp(m) when m is a power of two.  s ulp(m) / 2 is a power-of-two multiple
// of s, exact and normal for every scale the fast paths accept.
__device__ __forceinline__ void mid_side(float a, float qlo, float qhi, float s, bool& up, bool& dn) {
  const float m = 0.5f * (fabsf(qlo) + fabsf(qhi));
  const uint32_t mb = __float_as_uint(m);
  const float t = __fmul_rn(s, __uint_as_float((mb & 0x7F800000u) - (24u << 23)));
  const float tdn = (mb & 0x7FFFFFu) ? t : 0.5f * t;
  const float r = __fmaf_rn(-m, s, a);
  up = r > t;
  dn = r < -tdn;
}

// Widened reciprocal bounds of a positive normal scale s (see header comment).
__device__ __forceinline__ void recip_bounds(float s, float& r_lo, float& r_hi) {
  const float r = rcp_approx(s);
  r_lo = __fmul_rz(r, 1.0f - 9.5367431640625e-07f);   // 1 - 2^-20
  r_hi = __fmul_rz(r, 1.0f + 9.5367431640625e-07f);   // 1 + 2^-20
}

}  // namespace pq
