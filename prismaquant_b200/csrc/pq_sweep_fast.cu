// Fast multi-format sweep (SSE mode): same work items, staging and outputs as
// sweep_staged_kernel<MODE_SSE>, with the per-element arithmetic rebuilt on
// packed sm_100a instructions (pq_fast.cuh):
//
//  * a thread owns a 16-element NVFP4 group ("unit", two 16-byte shared
//    loads); MXFP8 32-groups are lane pairs (one shuffle);
//  * NVFP4 / FP8-per-channel: bracketed quotient -> hardware FP4 / FP8
//    conversion -> exact f16 decode -> f32x2 product with the scale -> bf16x2
//    reconstruction -> bf16x2 error -> mixed-precision square-accumulate;
//  * MXFP8 (power-of-two scale): the E4M3 rounding is an integer rounding of
//    the bf16 bit pattern, two elements per 32-bit operation (low 4 mantissa
//    bits, ties to the lower value), saturated at 448 * 2^e by a packed
//    magnitude min; its exponent is a closed form of the group amax bits
//    (e = E - 136 + (mantissa >= 31)), checked over every bf16 amax;
//  * a unit whose bracket is ambiguous (or that has values outside the fast
//    path's range) recomputes that format exactly, as the first-principles
//    kernel does.
// The fused NVFP4 export codes are the FP4 conversion codes of the bracket.
#include "pq_fast.cuh"
#include "pq_internal.h"

namespace pq {

constexpr int FAST_THREADS = SWEEP_THREADS;
constexpr float RCP6 = 0.16666667163372039794921875f;        // RN(1/6)

struct RowParam {
  float s, r_lo, r_hi, amax;
};

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

constexpr int FAST_QCAP = 64;            // queued uncertain units per warp and format
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
__device__ __forceinline__ float nv_pair_sq(uint32_t v, uint32_t cl, uint64_t s2) {
  const uint32_t rec = f2_to_bf16x2(f2_mul_rn(e2m1x2_to_f2(cl), s2));
  return sq2_acc(bf16x2_sub(v, rec), 0.0f);
}
__device__ __forceinline__ float f8_pair_sq(uint32_t v, uint32_t cl, uint64_t s2) {
  const uint32_t rec = f2_to_bf16x2(f2_mul_rn(e4m3x2_to_f2(cl), s2));
  return sq2_acc(bf16x2_sub(v, rec), 0.0f);
}

// Warp-cooperative resolution of queued units (entry = unit index).  For each
// uncertain pair (bracket codes differ) or every pair of an exact unit, adds
// exact squared errors minus the main loop's provisional ones and rewrites
// the export code bytes.
__device__ double nv_fixup(const uint32_t* q, int cnt, const uint4* st, int lane, int64_t elem0, uint8_t* codes,
                         bool cost) {
  double delta = 0.0;
  for (int i = lane; i < cnt; i += 32) {
    const int u = (int)q[i];
    const uint4 a = st[2 * u], b = st[2 * u + 1];
    const uint32_t v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    const float a16 = __uint_as_float(unit_absmax(v) << 16);
    const bool ex = exact_unit(a16);
    const float s = __fdiv_rn(fmaxf(a16, 1e-8f), 6.0f);
    float rlo, rhi;
    recip_bounds(s, rlo, rhi);
    const uint64_t rlo2 = f2_pack(rlo, rlo), rhi2 = f2_pack(rhi, rhi), s2 = f2_pack(s, s);
    const float se = fmaxf(__fdiv_rn(fmaxf(a16, 1e-12f), 6.0f), 1e-12f);   // export scale
    uint32_t pm = ex ? 0xFFu : 0u;
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      uint32_t cl, ch;
      nv_bracket(f2_from_bf16x2(v[p]), rlo2, rhi2, cl, ch);
      pm |= (cl != ch ? 1u : 0u) << p;
    }
    const uint32_t* vw = reinterpret_cast<const uint32_t*>(st) + 8 * u;
    for (; pm; pm &= pm - 1) {
      const int p = __ffs(pm) - 1;
      const uint32_t vp = vw[p];
      const float w0 = bf16lo(vp), w1 = bf16hi(vp);
      const float r0 = bf16_round(__fmul_rn(rtn_e2m1_cost(__fdiv_rn(w0, s)), s));
      const float r1 = bf16_round(__fmul_rn(rtn_e2m1_cost(__fdiv_rn(w1, s)), s));
      if (cost) {
        delta += (double)(sq_exact_err(w0, r0) + sq_exact_err(w1, r1));
        if (!ex) delta -= (double)nv_pair_sq(vp, cvt_e2m1x2(f2_mul_rz(f2_from_bf16x2(vp), rlo2)), s2);
      }
      if (codes) {
        const uint32_t c = nvfp4_code(__fdiv_rn(w0, se)) | (nvfp4_code(__fdiv_rn(w1, se)) << 4);
        codes[(elem0 + 16 * (int64_t)u + 2 * p) / 2] = (uint8_t)c;
      }
    }
  }
  return delta;
}

__device__ double f8_fixup(const uint32_t* q, int cnt, const uint4* st, int lane, const RowParam* rowp, int upr,
                           uint32_t rdiv) {
  double delta = 0.0;
  for (int i = lane; i < cnt; i += 32) {
    const int u = (int)q[i];
    const uint4 a = st[2 * u], b = st[2 * u + 1];
    const uint32_t v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    const bool ex = __uint_as_float(unit_absmax(v) << 16) >= 1.152921504606846976e18f;   // overflow guard
    const RowParam rp = rowp[upr == 1 ? u : (int)__umulhi((uint32_t)u, rdiv)];
    const uint64_t rlo2 = f2_pack(rp.r_lo, rp.r_lo), rhi2 = f2_pack(rp.r_hi, rp.r_hi), s2 = f2_pack(rp.s, rp.s);
    uint32_t pm = ex ? 0xFFu : 0u;
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      const uint64_t w2 = f2_from_bf16x2(v[p]);
      pm |= (cvt_e4m3x2(f2_mul_rz(w2, rlo2)) != cvt_e4m3x2(f2_mul_rz(w2, rhi2)) ? 1u : 0u) << p;
    }
    const uint32_t* vw = reinterpret_cast<const uint32_t*>(st) + 8 * u;
    for (; pm; pm &= pm - 1) {
      const int p = __ffs(pm) - 1;
      const uint32_t vp = vw[p];
      const float w0 = bf16lo(vp), w1 = bf16hi(vp);
      const float r0 = bf16_round(__fmul_rn(rtn_e4m3_cost(__fdiv_rn(w0, rp.s)), rp.s));
      const float r1 = bf16_round(__fmul_rn(rtn_e4m3_cost(__fdiv_rn(w1, rp.s)), rp.s));
      delta += (double)(sq_exact_err(w0, r0) + sq_exact_err(w1, r1));
      if (!ex) delta -= (double)f8_pair_sq(vp, cvt_e4m3x2(f2_mul_rz(f2_from_bf16x2(vp), rlo2)), s2);
    }
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
  const RowParam* rowp;
  int64_t elem0;
};

struct Accum {
  float nv, mx, f8;
  double dnv, dmx, df8;
  uint32_t tmax;
  int cnt_nv, cnt_f8;
};

template <bool NV, bool MX, bool F8, bool CODES>
__device__ __forceinline__ void process_unit(const ItemCtx& c, int u, int lane, uint32_t lanemask_lt,
                                             uint32_t* q_nv, uint32_t* q_f8, Accum& A) {
  const bool valid = u < c.nunits;
  const int uc = valid ? u : c.nunits - 1;
  uint32_t v[8];
  const bool sw = load_unit(c.st, uc, true, lane, v);
  uint32_t a16b, amin = 0;
  if (MX) unit_absmax_min(v, a16b, amin); else a16b = unit_absmax(v);
  const float a16 = __uint_as_float(a16b << 16);
  uint64_t w2[8];
  if (NV || CODES || F8) {
#pragma unroll
    for (int p = 0; p < 8; ++p) w2[p] = f2_from_bf16x2(v[p]);
  }

  if (NV || CODES) {
    const bool ex = exact_unit(a16);
    const float snv = div_const(fmaxf(a16, 1e-8f), 6.0f, RCP6);
    float rlo, rhi;
    recip_bounds(snv, rlo, rhi);
    const uint64_t rlo2 = f2_pack(rlo, rlo), rhi2 = f2_pack(rhi, rhi), s2 = f2_pack(snv, snv);
    uint32_t ux = 0, cc[8];
    float part = 0.0f;
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      uint32_t ch;
      nv_bracket(w2[p], rlo2, rhi2, cc[p], ch);
      ux |= cc[p] ^ ch;
      if (NV) {
        const uint32_t rec = f2_to_bf16x2(f2_mul_rn(e2m1x2_to_f2(cc[p]), s2));
        part = sq2_acc(bf16x2_sub(v[p], rec), part);
      }
    }
    if (NV) A.nv += (valid && !ex) ? part : 0.0f;
    if (CODES) {   // lanes past the end re-store the last unit's identical bytes
      const uint32_t cw0 = __byte_perm(__byte_perm(cc[0], cc[1], 0x0040), __byte_perm(cc[2], cc[3], 0x0040), 0x5410);
      const uint32_t cw1 = __byte_perm(__byte_perm(cc[4], cc[5], 0x0040), __byte_perm(cc[6], cc[7], 0x0040), 0x5410);
      reinterpret_cast<uint2*>(c.codes_it)[uc] = sw ? make_uint2(cw1, cw0) : make_uint2(cw0, cw1);
      c.amax_it[uc] = (uint16_t)a16b;
      A.tmax = max(A.tmax, a16b);
    }
    const bool need = valid && (ux != 0 || ex);
    const uint32_t bal = __ballot_sync(FULL, need);
    if (bal) {
      if (need) q_nv[A.cnt_nv + __popc(bal & lanemask_lt)] = (uint32_t)u;
      A.cnt_nv += __popc(bal);
      if (A.cnt_nv > FAST_QCAP - 32) {   // flush early only when the next unit could overflow
        __syncwarp();
        A.dnv += nv_fixup(q_nv, A.cnt_nv, c.st, lane, c.elem0, CODES ? c.codes_it - c.elem0 / 2 : nullptr, NV);
        __syncwarp();
        A.cnt_nv = 0;
      }
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
    float part = 0.0f;
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      const uint32_t neg = (v[p] >> 15) & 0x00010001u;
      const uint32_t rq = (v[p] + 0x00070007u + neg) & 0xFFF0FFF0u;   // ties to the lower value
      const uint32_t q = bf16x2_minabs(rq, m448x2);                   // saturate |q| at 448 * 2^e
      part = sq2_acc(bf16x2_sub(v[p], q), part);
    }
    if (!ok && valid) {
      Chunk8 c0, c1;
      unit_to_chunks(v, c0, c1);
      uint32_t rec[8];
      part = mxfp8_cost8(c0, a32, rec) + mxfp8_cost8(c1, a32, rec);
    }
    A.mx += valid ? part : 0.0f;
  }

  if (F8) {
    const RowParam rp = c.rowp[c.upr == 1 ? uc : (int)__umulhi((uint32_t)uc, c.rdiv)];
    const uint64_t rlo2 = f2_pack(rp.r_lo, rp.r_lo), rhi2 = f2_pack(rp.r_hi, rp.r_hi), s2 = f2_pack(rp.s, rp.s);
    const bool exf = a16 >= 1.152921504606846976e18f;
    uint32_t ux = 0;
    float part = 0.0f;
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      const uint32_t cl = cvt_e4m3x2(f2_mul_rz(w2[p], rlo2));
      const uint32_t ch = cvt_e4m3x2(f2_mul_rz(w2[p], rhi2));
      ux |= cl ^ ch;
      const uint32_t rec = f2_to_bf16x2(f2_mul_rn(e4m3x2_to_f2(cl), s2));
      part = sq2_acc(bf16x2_sub(v[p], rec), part);
    }
    A.f8 += (valid && !exf) ? part : 0.0f;
    const bool need = valid && (ux != 0 || exf);
    const uint32_t bal = __ballot_sync(FULL, need);
    if (bal) {
      if (need) q_f8[A.cnt_f8 + __popc(bal & lanemask_lt)] = (uint32_t)u;
      A.cnt_f8 += __popc(bal);
      if (A.cnt_f8 > FAST_QCAP - 32) {
        __syncwarp();
        A.df8 += f8_fixup(q_f8, A.cnt_f8, c.st, lane, c.rowp, c.upr, c.rdiv);
        __syncwarp();
        A.cnt_f8 = 0;
      }
    }
  }
}

template <bool NV, bool MX, bool F8, bool CODES>
__global__ void __launch_bounds__(FAST_THREADS, 1) sweep_fast_kernel(const __grid_constant__ SweepLaunch L) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int NWARPS = FAST_THREADS / 32;
  uint8_t* stages = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NSTAGE * STAGE_BYTES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + NSTAGE);
  RowParam* rowp = reinterpret_cast<RowParam*>(bars + NSTAGE + 2);
  double* red = reinterpret_cast<double*>(rowp + FAST_MAX_ROWS);
  uint32_t* qbase = reinterpret_cast<uint32_t*>(red + NWARPS * 3);
  auto row_amax = [&](int i) -> uint32_t* { return reinterpret_cast<uint32_t*>(&rowp[i].amax); };

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t* q_nv = qbase + warp * (2 * FAST_QCAP);
  uint32_t* q_f8 = q_nv + FAST_QCAP;
  const uint32_t lanemask_lt = (1u << lane) - 1u;
  const int64_t n_items = L.item_prefix[L.n];
  const int64_t my_n = n_items > (int64_t)blockIdx.x ? (n_items - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;

  for (int i = tid; i < FAST_MAX_ROWS; i += FAST_THREADS) *row_amax(i) = 0u;
  if (tid == 0) {
    for (int s = 0; s < NSTAGE; ++s) mbar_init(&bars[s], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  int ti_issue = 0;
  auto issue = [&](int64_t j) {
    const ItemRef it = next_item(L, (int64_t)blockIdx.x + j * gridDim.x, ti_issue);
    const SweepDesc& d = L.t[it.ti];
    const uint32_t bytes = (uint32_t)(it.nr * d.cols * 2);
    uint64_t* bar = &bars[j % NSTAGE];
    mbar_arrive_expect_tx(bar, bytes);
    bulk_g2s(stages + (j % NSTAGE) * STAGE_BYTES, d.w + it.r0 * d.cols, bytes, bar);
  };
  if (tid == 0)
    for (int64_t j = 0; j < NSTAGE && j < my_n; ++j) issue(j);

  Accum A;
  A.nv = A.mx = A.f8 = 0.0f;
  A.dnv = A.dmx = A.df8 = 0.0;
  A.tmax = 0u;
  int cur_t = -1, ti_proc = 0;
  auto flush_tensor = [&](int t) {   // CTA-uniform call
    const SweepDesc& d = L.t[t];
    A.dnv += (double)A.nv;
    A.dmx += (double)A.mx;
    A.df8 += (double)A.f8;
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
        if (lane == 0 && (d.fmt_mask & (1u << f))) atomicAdd(d.sse + f, x);
      }
    }
    __syncthreads();
    A.nv = A.mx = A.f8 = 0.0f;
    A.dnv = A.dmx = A.df8 = 0.0;
    A.tmax = 0u;
  };

  int64_t j_abort = -1;
  for (int64_t j = 0; j < my_n; ++j) {
    const int s = (int)(j % NSTAGE);
    const uint32_t parity = (uint32_t)((j / NSTAGE) & 1);
    const ItemRef it = next_item(L, (int64_t)blockIdx.x + j * gridDim.x, ti_proc);
    if (it.ti != cur_t) {
      if (cur_t >= 0) flush_tensor(cur_t);
      cur_t = it.ti;
    }
    const SweepDesc& d = L.t[it.ti];
    if (!mbar_wait_bounded(&bars[s], parity)) {
      *abort_flag = 1;
      j_abort = j;
    }

    ItemCtx c;
    c.st = reinterpret_cast<const uint4*>(stages + s * STAGE_BYTES);
    c.upr = (int)(d.cols >> 4);
    c.nunits = (int)it.nr * c.upr;
    c.rdiv = 0xFFFFFFFFu / (uint32_t)c.upr + 1u;   // u / upr = umulhi(u, rdiv), exact for u < 4096 (host-checked)
    c.elem0 = it.r0 * d.cols;
    c.codes_it = CODES ? d.nvfp4_codes + c.elem0 / 2 : nullptr;
    c.amax_it = CODES ? d.nvfp4_amax + c.elem0 / 16 : nullptr;
    c.rowp = rowp;
    const int iters = (c.nunits + FAST_THREADS - 1) / FAST_THREADS;

    if (F8) {
      __syncthreads();   // a failed wait is visible to every thread before the stage is read
      if (*abort_flag) {
        if (j_abort < 0) j_abort = j;
        break;
      }
      const bool warp_rows = (c.upr & 31) == 0;
      for (int k = 0; k < iters; ++k) {
        const int u = tid + k * FAST_THREADS;
        uint32_t v[8];
        load_unit(c.st, min(u, c.nunits - 1), true, lane, v);
        uint32_t a = unit_absmax(v);
        const int row = c.upr == 1 ? u : (int)__umulhi((uint32_t)u, c.rdiv);
        if (warp_rows) {
          a = warp_max_u(a);
          if (lane == 0 && u - lane < c.nunits) atomicMax(row_amax(row), a);
        } else if (u < c.nunits) {
          atomicMax(row_amax(row), a);
        }
      }
      __syncthreads();
      for (int i = tid; i < it.nr; i += FAST_THREADS) {
        const float ar = __uint_as_float(*row_amax(i) << 16);
        const float sr = __fdiv_rn(fmaxf(ar, 1e-8f), 448.0f);
        RowParam p;
        p.s = sr;
        p.amax = ar;
        recip_bounds(sr, p.r_lo, p.r_hi);
        rowp[i] = p;
      }
      __syncthreads();
    }

    A.cnt_nv = A.cnt_f8 = 0;
    for (int k = 0; k < iters; k += 4) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        if (k + kk < iters) process_unit<NV, MX, F8, CODES>(c, tid + (k + kk) * FAST_THREADS, lane, lanemask_lt, q_nv, q_f8, A);
      A.dnv += (double)A.nv;   // fold fp32 partials (<= 64 squares each) into fp64
      A.dmx += (double)A.mx;
      A.df8 += (double)A.f8;
      A.nv = A.mx = A.f8 = 0.0f;
    }
    __syncwarp();
    if ((NV || CODES) && A.cnt_nv)
      A.dnv += nv_fixup(q_nv, A.cnt_nv, c.st, lane, c.elem0, CODES ? d.nvfp4_codes : nullptr, NV);
    if (F8 && A.cnt_f8) A.df8 += f8_fixup(q_f8, A.cnt_f8, c.st, lane, rowp, c.upr, c.rdiv);
    if (F8)
      for (int i = tid; i < it.nr; i += FAST_THREADS) *row_amax(i) = 0u;   // ready for the next item
    __syncthreads();   // stage s, row parameters and queues are free again
    if (*abort_flag) {
      if (j_abort < 0) j_abort = j;
      break;
    }
    if (tid == 0 && j + NSTAGE < my_n) {
      fence_proxy_async_smem();
      issue(j + NSTAGE);
    }
  }
  if (cur_t >= 0 && j_abort < 0) flush_tensor(cur_t);
  if (j_abort >= 0 && tid == 0) {
    for (int64_t jj = j_abort; jj < j_abort + NSTAGE && jj < my_n; ++jj)
      (void)mbar_wait_bounded(&bars[jj % NSTAGE], (uint32_t)((jj / NSTAGE) & 1), 1u << 20);
  }
}

size_t sweep_fast_smem_bytes() {
  return (size_t)NSTAGE * STAGE_BYTES + (NSTAGE + 2) * sizeof(uint64_t) + FAST_MAX_ROWS * sizeof(RowParam) +
         (FAST_THREADS / 32) * 3 * sizeof(double) + (FAST_THREADS / 32) * 2 * FAST_QCAP * sizeof(uint32_t);
}

template <bool NV, bool MX, bool F8, bool CODES>
static cudaError_t launch_fast_t(const SweepLaunch& L, int grid, cudaStream_t stream) {
  const size_t smem = sweep_fast_smem_bytes();
  cudaError_t e = cudaFuncSetAttribute(sweep_fast_kernel<NV, MX, F8, CODES>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  sweep_fast_kernel<NV, MX, F8, CODES><<<grid, FAST_THREADS, smem, stream>>>(L);
  return cudaGetLastError();
}

// All descriptors of L share the flag set `key` (format mask bits 0-2, bit 3 = NVFP4 codes).
cudaError_t launch_sweep_fast(const SweepLaunch& L, int grid, uint32_t key, cudaStream_t stream) {
  switch (key & 15u) {
#define PQ_CASE(K) \
  case K: return launch_fast_t<(K & 1) != 0, (K & 2) != 0, (K & 4) != 0, (K & 8) != 0>(L, grid, stream);
    PQ_CASE(1) PQ_CASE(2) PQ_CASE(3) PQ_CASE(4) PQ_CASE(5) PQ_CASE(6) PQ_CASE(7)
    PQ_CASE(8) PQ_CASE(9) PQ_CASE(10) PQ_CASE(11) PQ_CASE(12) PQ_CASE(13) PQ_CASE(14) PQ_CASE(15)
#undef PQ_CASE
    default: return cudaSuccess;
  }
}

}  // namespace pq
