"""The fast sweep's division-free rounding rules against the reference's rule, on EVERY pair of
bf16 values (group / row maximum a in [1, 2), every bf16 w with |w| <= a) — the ratios and
roundings are the same in every binade of a inside the fast path's range [1e-8, 2^60).

Reference (format_registry.py:194-233): x = fl32(w / s) with s = fl32(a / d) (d = 6 for NVFP4,
448 for FP8 per channel), nearest point of the signed codebook with ties to the LOWER value; the
NVFP4 export (export_native_compressed.py:114-136) takes the abs codebook with ties toward zero.

Kernel rules, with r = rcp.approx(s) (within one ulp of 1/s: every r in {RN(1/s), its two
neighbours} is tried), r_lo = RZ(r (1 - 2^-20)), r_hi = RZ(r (1 + 2^-20)) and the hardware
conversions (round to nearest, ties to even, saturating):
  * NVFP4 cost:    cvt_e2m1(fma(w, r, -2^-18))     (an absolute bias toward -inf)
  * NVFP4 export:  cvt_e2m1(RZ(w r_lo))
  * FP8 cost:      cvt_e4m3(min(RZ(w r_lo), RZ(w r_hi)))   (the lower of the two brackets)
Why they hold: w and a have 8-bit significands, so w / (a / d) is either exactly a codebook
midpoint m or at least ~2^-13 (relative) away from every midpoint, while the products are within
2^-19 of it.  At an exact midpoint the reference's fl32(w / s) is m itself (a tie) whenever
a / d is exact or m's significand is short enough; then "ties to lower" is "the bracket below".
For NVFP4 that covers every case.  For FP8 per channel it leaves one family: rows where
|a - 448 s| = 3 * 64 ulp(s) and s's significand is below 1.5, at midpoints with significand 21/16
or 7/16; the kernel's row flags and per-element selection (f8_flag_select) for those rows are
emulated here too, and the whole rule must then agree with the reference on every pair."""
import numpy as np

F32 = np.float32


def _bf16_in(lo, hi):
    b = np.arange(1 << 15, dtype=np.uint32)
    with np.errstate(invalid="ignore"):
        f = (b << 16).view(np.float32).astype(np.float64)
    f = f[np.isfinite(f)]
    return f[(f >= lo) & (f < hi)]


def _rz32(v):
    f = v.astype(F32).astype(np.float64)
    return np.where(np.abs(f) > np.abs(v), np.nextafter(f.astype(F32), F32(0)).astype(np.float64), f)


def _rne(p, mags, even, maxv):
    a = np.abs(p)
    i = np.clip(np.searchsorted(mags, a), 1, len(mags) - 1)
    lo, hi = i - 1, i
    mid = (mags[lo] + mags[hi]) / 2
    pick = np.where(a < mid, lo, np.where(a > mid, hi, np.where(even[lo], lo, hi)))
    pick = np.where(a >= maxv, len(mags) - 1, pick)
    return np.where(np.signbit(p), -1.0, 1.0) * mags[pick]


def _ties_lower(x, mags):
    cb = np.concatenate([-mags[::-1], mags[1:]])
    i = np.clip(np.searchsorted(cb, x), 1, len(cb) - 1)
    lo, hi = cb[i - 1], cb[i]
    return np.where(np.abs(hi - x) < np.abs(x - lo), hi, lo)


def _ties_zero(x, mags):
    a = np.abs(x)
    i = np.clip(np.searchsorted(mags, a), 1, len(mags) - 1)
    lo, hi = mags[i - 1], mags[i]
    m = np.where(np.abs(hi - a) < np.abs(a - lo), hi, lo)
    return np.where(x < 0, -1.0, 1.0) * np.minimum(m, mags[-1])


def _reciprocals(s):
    r0 = F32(1) / s
    for r in (np.nextafter(r0, F32(0)), r0, np.nextafter(r0, F32(10))):
        r = np.float64(r)
        yield r, np.float64(_rz32(np.array([r * (1 - 2.0 ** -20)]))[0]), \
            np.float64(_rz32(np.array([r * (1 + 2.0 ** -20)]))[0])


E2M1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6], dtype=np.float64)
E2M1_EVEN = np.arange(8) % 2 == 0


def _e4m3():
    vals = sorted({k * 2.0 ** -9 for k in range(8)} | {(1 + m / 8) * 2.0 ** (e - 7) for e in range(1, 16)
                                                      for m in range(8)})
    mags = np.array([v for v in vals if v <= 448], dtype=np.float64)
    man = np.array([round(v / 2.0 ** -9) if v < 2.0 ** -6 else round((v / 2.0 ** np.floor(np.log2(v)) - 1) * 8)
                    for v in mags])
    return mags, man % 2 == 0


def test_nvfp4_cost_and_export_rules_are_exact_for_every_bf16_pair():
    ws = _bf16_in(0, 2.01)
    ws = np.concatenate([ws, -ws])
    bad = n = 0
    for a in _bf16_in(1, 2):
        w = ws[np.abs(ws) <= a]
        s = F32(a) / F32(6)
        x = (w.astype(F32) / s).astype(np.float64)
        want_cost, want_exp = _ties_lower(x, E2M1), _ties_zero(x, E2M1)
        for r, r_lo, _ in _reciprocals(s):
            p = (w * r - 2.0 ** -18).astype(F32).astype(np.float64)       # fma, one rounding
            bad += np.count_nonzero(_rne(p, E2M1, E2M1_EVEN, 6.0) != want_cost)
            bad += np.count_nonzero(_rne(_rz32(w * r_lo), E2M1, E2M1_EVEN, 6.0) != want_exp)
            n += 2 * w.size
    assert n > 10_000_000 and bad == 0


def fp8_row_flag(a: float) -> bool:
    """The kernel's per-row flag (rows whose near-midpoint pairs it resolves exactly): with
    s = fl32(a / 448), d = a - 448 s (exact as one FMA: a multiple of 64 ulp(s), at most 3 of them)
    and s's significand: |d| >= 160 ulp(s) (i.e. 3 x 64) and significand < 1.5."""
    s = F32(a) / F32(448)
    d = np.float64(a) - 448.0 * np.float64(s)
    u = np.float64(np.spacing(s))
    sig_bits = int(np.array([s], dtype=F32).view(np.uint32)[0]) & 0x7FFFFF
    return abs(d) >= 160 * u and sig_bits < 0x400000


def test_fp8_channel_lower_bracket_rule_exact_outside_flagged_rows():
    mags, even = _e4m3()
    ws = _bf16_in(0, 2.01)
    ws = np.concatenate([ws, -ws])
    n = 0
    flagged_with_misses = 0
    for a in _bf16_in(1, 2):
        w = ws[np.abs(ws) <= a]
        s = F32(a) / F32(448)
        x = (w.astype(F32) / s).astype(np.float64)
        want = _ties_lower(x, mags)
        miss = 0
        for _, r_lo, r_hi in _reciprocals(s):
            got = _rne(np.minimum(_rz32(w * r_lo), _rz32(w * r_hi)), mags, even, 448.0)
            miss += np.count_nonzero(got != want)
            n += w.size
        if miss:
            assert fp8_row_flag(a), (a, miss)
            flagged_with_misses += 1
    assert n > 10_000_000
    assert flagged_with_misses > 0      # the flagged family exists: the exact resolution is needed


def _e4m3_code(v, mags):
    """E4M3 code byte of an exactly representable value (sign bit 7, magnitude index as
    exponent/mantissa fields)."""
    i = np.searchsorted(mags, np.abs(v))
    e = np.where(i < 8, 0, (i - 8) // 8 + 1)
    m = np.where(i < 8, i, (i - 8) % 8)
    return (np.where(np.signbit(v), 0x80, 0) | (e << 3) | m).astype(np.int64)


def test_fp8_channel_full_kernel_rule_exact_for_every_bf16_pair():
    """The lower-bracket code, replaced in flagged rows by the flag selection, equals the
    reference's code for every bf16 pair (row flags as row_tab computes them)."""
    mags, even = _e4m3()
    ws = _bf16_in(0, 2.01)
    ws = np.concatenate([ws, -ws])
    bad = n = 0
    for a in _bf16_in(1, 2):
        w = ws[np.abs(ws) <= a]
        s = F32(a) / F32(448)
        x = (w.astype(F32) / s).astype(np.float64)
        want = _ties_lower(x, mags)
        d = np.float64(a) - 448.0 * np.float64(s)
        ulp = np.float64(np.spacing(s))
        sig = int(np.array([s], dtype=F32).view(np.uint32)[0]) & 0x7FFFFF
        j3 = abs(d) >= 160 * ulp
        f7, f21, up = j3 and sig < 0x400000, j3 and sig < 0x100000, d > 0
        for _, r_lo, r_hi in _reciprocals(s):
            lo, hi = _rz32(w * r_lo), _rz32(w * r_hi)
            cm = _rne(np.minimum(lo, hi), mags, even, 448.0)
            got = cm
            if f7:   # flagged row: the kernel's per-element selection (f8_flag_select)
                cl, ch = _rne(lo, mags, even, 448.0), _rne(hi, mags, even, 448.0)
                bl = _e4m3_code(cl, mags)
                subnormal = (bl & 0x78) == 0
                sel = (cl != ch) & (f21 | subnormal)
                got = np.where(sel, ch if up else cl, cm)
            bad += np.count_nonzero(got != want)
            n += w.size
    assert n > 10_000_000 and bad == 0


# MX formats of the codebook kernel's packed squared-error path (mx_sse8): kind -> (M, EMIN,
# subnormals, MAXV), as in the codebook kernel's table of kinds
MX_KINDS = {"E2M1": (1, 0, True, 6.0), "E3M2": (2, -3, False, 28.0), "E2M3": (3, -1, False, 7.5),
            "E4M3": (3, -6, True, 448.0), "E5M2": (2, -14, True, 114688.0)}


def _mx_grid(M, EMIN, sub, maxv):
    """Non-negative grid points of the format (the reference's codebook magnitudes)."""
    pts = {0.0}
    e = EMIN
    while True:
        for k in range(1 << M):
            v = (1 + k / (1 << M)) * 2.0 ** e
            if v <= maxv:
                pts.add(v)
        if 2.0 ** e > maxv:
            break
        e += 1
    if sub:
        pts |= {k / (1 << M) * 2.0 ** EMIN for k in range(1 << M)}
    return np.array(sorted(pts))


def _mx_sse8_emulated(bits, es, M, EMIN, sub, maxv):
    """The packed path's grid point for each bf16 pattern (int arithmetic as the kernel does it;
    the bf16 add/subtract of C as its exact value: w rounded to the step, ties to the even
    multiple)."""
    MS = M if sub else 0
    drop = 7 - M
    mag = bits.astype(np.int64) & 0x7FFF
    sign = np.where(bits & 0x8000, -1.0, 1.0)
    qn_mag = (mag + (1 << (drop - 1))) & ((0xFFFF >> drop) << drop)
    sat = (int(np.array([maxv], dtype=np.float32).view(np.uint32)[0]) >> 16) + (es << 7)
    qn_mag = np.minimum(qn_mag, sat)
    qn = sign * ((qn_mag << 16).astype(np.uint32).view(np.float32).astype(np.float64))
    w = ((bits.astype(np.uint32) << 16).view(np.float32)).astype(np.float64)
    step = 2.0 ** (EMIN + es - MS)
    qs = np.round(w / step) * step                                   # numpy rounds half to even
    lo = (EMIN + es + 127) << 7
    d = 0x8000 + lo - mag                    # one half of the packed subtraction: never negative,
    assert (d > 0).all()                     # so no borrow reaches the other half
    return w, np.where(d & 0x8000, qs, qn)   # bit 15 (spread over the half by the byte permute)


def test_mx_packed_cost_rounding_matches_the_codebook_rule():
    """mx_sse8's grid point gives the reference's squared error for every finite bf16 w, every
    MX kind the codebook kernel serves, at scales 2^es across its fast range (|es| <= 100)."""
    b = np.arange(1 << 16, dtype=np.uint32)
    with np.errstate(invalid="ignore"):
        f = (b << 16).view(np.float32)
    bits = b[np.isfinite(f)].astype(np.uint16)
    for name, (M, EMIN, sub, maxv) in MX_KINDS.items():
        grid = _mx_grid(M, EMIN, sub, maxv)
        for es in (-100, -40, -7, -1, 0, 3, 20, 100):
            w, q = _mx_sse8_emulated(bits, es, M, EMIN, sub, maxv)
            x = np.abs(w) / 2.0 ** es
            i = np.clip(np.searchsorted(grid, x), 1, len(grid) - 1)
            lo_, hi_ = grid[i - 1], grid[i]
            ref = np.where(hi_ - x < x - lo_, hi_, lo_)          # nearest, ties to the lower magnitude
            ref = np.where(x >= grid[-1], grid[-1], ref) * 2.0 ** es
            ok = np.abs(np.abs(w - q) - np.abs(np.abs(w) - ref)) == 0
            assert ok.all(), (name, es, w[~ok][:5], q[~ok][:5], ref[~ok][:5])


def test_mx_group_exponent_closed_form_matches_the_torch_rule():
    """mxsse_kernel's closed form e = E + C + (m >= T) (FLOOR below 1e-8) against
    round(log2(max(max(amax, 1e-8) / cmax, 2^-127))) with the torch-derived thresholds, for every
    finite bf16 amax and each MX kind; the constants are read from the kernel source."""
    import re
    from pathlib import Path
    from oracle import pq_oracle as O
    src = (Path(__file__).resolve().parent.parent / "prismaquant_b200" / "csrc" / "pq_codebook.cu").read_text()
    consts = {k: tuple(int(x) for x in v) for k, *v in
              re.findall(r"struct MXE<XK_(\w+)> \{ static constexpr int C = (-?\d+), T = (\d+), FLOOR = (-?\d+); \}", src)}
    ceil_1em8 = int(re.search(r"BF16_1EM8_CEIL = 0x([0-9A-Fa-f]+)u", src).group(1), 16)
    assert set(consts) == set(MX_KINDS)
    assert (np.array([ceil_1em8 << 16], dtype=np.uint32).view(F32)[0] >= F32(1e-8) >
            np.array([(ceil_1em8 - 1) << 16], dtype=np.uint32).view(F32)[0])
    b = np.arange(0x7F80, dtype=np.uint32)               # every finite bf16 magnitude
    a = (b << 16).view(F32)
    for kind, (C, T, FLOOR) in consts.items():
        cmax = F32(MX_KINDS[kind][3])
        s = np.maximum((np.maximum(a, F32(1e-8)) / cmax).astype(F32), F32(2.0 ** -127))
        want = O.e8m0().round_log2(s)
        got = np.where(b < ceil_1em8, FLOOR, (b >> 7).astype(np.int64) - 127 + C + ((b & 0x7F) >= T))
        assert np.array_equal(got, want), kind


def _rn32(x):
    """Round a Fraction to the nearest float32, ties to even (exactly)."""
    from fractions import Fraction as Fr
    if x == 0:
        return F32(0)
    f = F32(float(x))
    cands = [np.nextafter(f, F32(-np.inf)), f, np.nextafter(f, F32(np.inf))]
    return min(cands, key=lambda c: (abs(Fr(float(c)) - x), int(np.array([c], F32).view(np.uint32)[0]) & 1))


def test_div_const_is_ieee_division_for_every_bf16_value():
    """div_const (q = RN(a rd), r = fma(-q, d, a), RN(q + r rd) with rd = RN(1/d)) equals IEEE
    division for every normal bf16 a and the 1e-8 / 1e-12 floors, for the divisors the kernels
    use it with: 6 (NVFP4 group scale), 448 (FP8 row scale), 3 and 7 (INT3 / INT4 group scales)."""
    from fractions import Fraction as Fr
    b = np.arange(0x0080, 0x7F80, dtype=np.uint32)
    vals = list((b << 16).view(F32)) + [F32(1e-8), F32(1e-12)]
    for d in (3, 6, 7, 448):
        rd = _rn32(Fr(1, d))
        for a in vals:
            q = F32(a) * rd
            r = _rn32(Fr(float(a)) - Fr(float(q)) * d)
            got = _rn32(Fr(float(r)) * Fr(float(rd)) + Fr(float(q)))
            assert got == _rn32(Fr(float(a)) / d), (d, a)


def _mx_qdq8_emulated(bits, es, M, EMIN, sub, maxv):
    """mx_qdq8's output bf16 pattern for each bf16 pattern: the integer half as the kernel does it,
    the float32 pair arithmetic (w - eps + c - c, round to nearest even) in numpy float32."""
    MS = M if sub else 0
    drop = 7 - M
    b = bits.astype(np.int64)
    mag = b & 0x7FFF
    neg = (b >> 15) & 1
    sat = (int(np.array([maxv], dtype=F32).view(np.uint32)[0]) >> 16) + (es << 7)
    qn = np.minimum((mag + ((1 << (drop - 1)) - 1) + neg) & ((0xFFFF >> drop) << drop), sat) | (b & 0x8000)
    sexp = EMIN + es - MS
    c = np.array([((sexp + 23 + 127) << 23) | 0x400000], dtype=np.uint32).view(F32)[0]
    eps = np.array([(sexp - 11 + 127) << 23], dtype=np.uint32).view(F32)[0]
    w = (bits.astype(np.uint32) << 16).view(F32)
    t = ((w + (-eps)) + c) + (-c)                 # numpy float32 arithmetic rounds to nearest even
    tb = t.view(np.uint32)
    qs = (tb >> 16).astype(np.int64)
    d = 0x8000 + ((EMIN + es + 127) << 7) - mag
    small = (d & 0x8000) != 0
    assert ((tb[small] & 0xFFFF) == 0).all()      # every selected result is a bf16: the cvt is exact
    return np.where(small, qs, qn)


def test_mx_packed_w_hat_rounding_matches_the_codebook_rule():
    """mx_qdq8 (the MX W_hat of the codebook kernel's grouped fast path) gives the reference's
    bf16 pattern for every finite bf16 w, every MX kind, at scales 2^es across its range
    (|es| <= 90): the nearest grid point with ties to the lower signed value, saturated at MAXV,
    +0 for a negative w that rounds to zero."""
    b = np.arange(1 << 16, dtype=np.uint32)
    with np.errstate(invalid="ignore"):
        f = (b << 16).view(F32)
    bits = b[np.isfinite(f)].astype(np.uint16)
    w = ((bits.astype(np.uint32) << 16).view(F32)).astype(np.float64)
    for name, (M, EMIN, sub, maxv) in MX_KINDS.items():
        grid = _mx_grid(M, EMIN, sub, maxv)
        for es in (-90, -40, -7, -1, 0, 3, 20, 90):
            got = _mx_qdq8_emulated(bits, es, M, EMIN, sub, maxv)
            x = w / 2.0 ** es
            near = np.abs(x) <= 1.5 * maxv            # beyond, float64 distances could tie falsely
            ref = np.where(np.abs(x) >= maxv, np.sign(x) * maxv, _ties_lower(np.where(near, x, 0.0), grid))
            ref = ref * 2.0 ** es + 0.0                # + 0.0: a negative w that rounds to zero gives +0
            want = (ref.astype(F32).view(np.uint32) >> 16).astype(np.int64)
            assert (ref.astype(F32).astype(np.float64) == ref).all()
            ok = got == want
            assert ok.all(), (name, es, bits[~ok][:5], got[~ok][:5], want[~ok][:5])


def _fp3_err_sq_kernel(wbits, abits):
    """fp3_rec2 / fp3_sse8 of the codebook kernel, emulated on the bit patterns: the squared
    bf16 error of each w in a group whose maximum has bits abits."""
    from oracle import pq_oracle as O
    ab = int(abits)
    t3 = int(np.array([np.float32((np.uint32(ab) << 16).view(F32) * F32(3.0))], F32).view(np.uint32)[0])
    rd3, ex = t3 >> 16, int((t3 & 0xFFFF) == 0)
    thr = [ab - 4 * 0x80, rd3 - 4 * 0x80, rd3 - 3 * 0x80, rd3 - 2 * 0x80]
    w = wbits.astype(np.int64)
    mag, neg = w & 0x7FFF, (w >> 15) & 1
    lvl = np.zeros(w.shape, np.int64)
    for k, t in enumerate(thr):
        mk = mag + (neg if k == 0 else neg * ex)
        lvl += ((mk + 0x7FFF - t) >> 15) & 1
    rec = np.where(lvl == 0, 0, ab - (4 - lvl) * 0x80)
    f = lambda b: (b.astype(np.uint32) << 16).view(F32).astype(np.float64)
    d = f(mag) - f(rec)
    assert (d.astype(F32).astype(np.float64) == d).all()   # exact in float32: one rounding, to bf16
    e = O.bf16_round(d.astype(F32))
    w_hat = np.where(lvl == 0, 0, rec | (neg << 15))        # signed W_hat bits, +0 at level 0
    return w_hat, (e.astype(F32) * e.astype(F32)).astype(F32)


def _fp3_err_sq_reference(wbits, abits):
    """format_registry.py:194-233 for NVFP3: s = fl32(a / 2), x = fl32(w / s), bucketize into the
    signed E2M0 codebook, the upper neighbour only when strictly closer in float32,
    W_hat = bf16(q s), error bf16(w - W_hat), squared in float32."""
    from oracle import pq_oracle as O
    cb = np.array([-2, -1, -0.5, -0.25, 0, 0.25, 0.5, 1, 2], F32)
    a = (np.uint32(abits) << 16).view(F32)
    s = F32(a) / F32(2.0)
    w = (wbits.astype(np.uint32) << 16).view(F32)
    x = (w / s).astype(F32)
    i = np.searchsorted(cb, x, side="left")
    lo, hi = cb[np.maximum(i - 1, 0)], cb[np.minimum(i, cb.size - 1)]
    q = np.where(np.abs(hi - x) < np.abs(x - lo), hi, lo)
    rec = O.bf16_round((q * s).astype(F32))
    e = O.bf16_round((w - rec).astype(F32))
    return O.f32_to_bf16_bits(rec).astype(np.int64), (e * e).astype(F32)


def test_nvfp3_threshold_rule_matches_the_codebook_rule():
    """fp3sse_kernel's comparisons on bf16 bit patterns give the reference's W_hat and squared
    error for every finite bf16 w with |w| <= a and every group maximum a in [1, 2), and for
    maxima in the binades of 1e-8, 2^-60, 2^100 and 2^125 (the thresholds move with a's
    exponent; from 2^126 up, where 3a would overflow, the kernel takes the per-element rule).  The
    squared error alone cannot see the tie rule (a tie of fl32(w / s) is an exact tie here, both
    neighbours equally far), so W_hat is compared too."""
    b = np.arange(1 << 16, dtype=np.uint32)
    with np.errstate(invalid="ignore"):
        fin = b[np.isfinite((b << 16).view(F32))]
    import re
    from pathlib import Path
    src = (Path(__file__).resolve().parent.parent / "prismaquant_b200" / "csrc" / "pq_codebook.cu").read_text()
    lo = int(re.search(r"BF16_1EM8_CEIL = 0x([0-9A-Fa-f]+)u", src).group(1), 16)
    hi = int(re.search(r"FP3_FAST_CEIL = 0x([0-9A-Fa-f]+)u", src).group(1), 16)
    assert hi == 0x7E80                                    # 2^126: 3a stays finite below it
    binades = [0x3F80, 0x3200, 0x2180, 0x7180, 0x7E00]   # 1, 2^-27 (holds 1e-8), 2^-60, 2^100, 2^125
    for base in binades:
        for ab in range(base, base + 0x80):
            if ab < lo or ab >= hi:                        # the per-element path
                continue
            wb = fin[(fin & 0x7FFF) <= ab].astype(np.uint16)
            with np.errstate(over="ignore"):               # squares of errors near 2^100
                got, want = _fp3_err_sq_kernel(wb, ab), _fp3_err_sq_reference(wb, ab)
            for g, r in zip(got, want):
                bad = g != r
                assert not bad.any(), (hex(ab), wb[bad][:5], g[bad][:5], r[bad][:5])


def _e5m2_standard_mags():
    """Non-negative values of the hardware E5M2 format (finite, up to 57344), ascending."""
    m = [k / 4 * 2.0 ** -14 for k in range(4)]
    m += [(1 + k / 4) * 2.0 ** (e - 15) for e in range(1, 31) for k in range(4)]
    return np.array(m)


def test_fp8_e5m2_bracket_rule_matches_the_codebook_rule():
    """e5m2_word of the codebook kernel: for a row maximum a (every bf16 a in [1, 2), and binades
    of 2^-27 (from 1e-8 up), 2^39 and 2^97) and every finite bf16 w with |w| <= a, with r any of
    RN(1/s) and its two neighbours (rcp.approx is within one ulp), the hardware conversions (round
    to nearest even, saturating) of RZ(w r_lo / 2) and RZ(w r_hi / 2), where they agree and the
    word is not flagged tiny, give the reference's W_hat bf16(q s) (nearest codebook point of
    fl32(w / s), ties to the lower value, codebook exponent 31 finite); and the conversion of the
    lower of the two alone gives it for every element that is not tiny (e5m2_word<true>, row
    maxima of at least 1e-8)."""
    from oracle import pq_oracle as O
    mags = _e5m2_standard_mags()
    even = (np.arange(mags.size) % 2) == 0
    cb = O.CODEBOOKS["fp8_e5m2"].astype(np.float64)
    b = np.arange(1 << 16, dtype=np.uint32)
    with np.errstate(invalid="ignore"):
        fin = b[np.isfinite((b << 16).view(F32))]
    checked = fast = 0
    for base in (0x3F80, 0x3200, 0x53 << 8, 0x7000):
        for ab in range(base, base + 0x80, 3 if base != 0x3F80 else 1):
            if ab < 0x322C:                                # below 1e-8: agree-or-exact only
                continue
            a = (np.uint32(ab) << 16).view(F32)
            s = F32(max(a, F32(1e-8)) / F32(114688.0))
            wb = fin[(fin & 0x7FFF) <= ab]
            w = (wb << 16).view(F32)
            x = (w / s).astype(F32).astype(np.float64)
            ref = _ties_lower(x, cb[cb >= 0])
            ref = np.where(np.abs(x) >= 114688.0, np.sign(x) * 114688.0, ref)
            want = O.f32_to_bf16_bits((ref * np.float64(s)).astype(F32))
            want = np.where(want == 0x8000, 0, want)
            tiny_t = ((int(np.array([s * F32(2.0 ** -12)], F32).view(np.uint32)[0]) >> 16) + 1)
            mag = wb & 0x7FFF
            tiny = (mag > 0) & (mag <= tiny_t)
            r0 = F32(1.0) / s
            for r in (np.nextafter(r0, F32(0)), r0, np.nextafter(r0, F32(np.inf))):
                r_lo = _rz32(np.array([np.float64(r) * (1 - 2.0 ** -20)]))[0] * 0.5
                r_hi = _rz32(np.array([np.float64(r) * (1 + 2.0 ** -20)]))[0] * 0.5
                cl = _rne(_rz32(w.astype(np.float64) * r_lo), mags, even, 57344.0)
                ch = _rne(_rz32(w.astype(np.float64) * r_hi), mags, even, 57344.0)
                ok = (cl == ch) & ~tiny
                rec = O.f32_to_bf16_bits((cl * np.float64(F32(2.0) * s)).astype(F32))   # fl32(code x 2s)
                got = np.where(rec == 0x8000, 0, rec)
                bad = ok & (got != want)
                assert not bad.any(), (hex(ab), wb[bad][:5], got[bad][:5], want[bad][:5])
                # e5m2_word<true> (row maximum >= 1e-8): the lower bracket alone, every non-tiny w
                cm = _rne(np.minimum(_rz32(w.astype(np.float64) * r_lo), _rz32(w.astype(np.float64) * r_hi)),
                          mags, even, 57344.0)
                low = O.f32_to_bf16_bits((cm * np.float64(F32(2.0) * s)).astype(F32))
                low = np.where(low == 0x8000, 0, low)
                bad = ~tiny & (mag > 0) & (low != want)
                assert not bad.any(), ("lower", hex(ab), wb[bad][:5], low[bad][:5], want[bad][:5])
                checked += int((mag > tiny_t).sum())
                fast += int((ok & (mag > tiny_t)).sum())
    assert fast > 0.99 * checked                       # beside tiny elements, the exact rule is rare


def test_integer_row_bracket_matches_the_reference_rule():
    """int_word of the codebook kernel's row path: for L = 127 (INT8_W8A16) and L = 1, 3, 7, row
    maxima a across [1, 2) and two more binades, every finite bf16 w with |w| <= a, and r any of
    RN(1/s) and its two neighbours, the products RN(w RN(r (1 -+ 2^-19))) rounded half even, where
    they agree, give the reference's W_hat: bf16(q s), q = round half even of fl32(w / s),
    -0 for a negative w that rounds to zero (format_registry.py:147-172)."""
    from oracle import pq_oracle as O
    b = np.arange(1 << 16, dtype=np.uint32)
    with np.errstate(invalid="ignore"):
        fin = b[np.isfinite((b << 16).view(F32))]
    checked = fast = 0
    for L in (127, 1, 3, 7):
        for base in (0x3F80, 0x2F00, 0x5500):
            for ab in range(base, base + 0x80, 1 if (L == 127 and base == 0x3F80) else 9):
                a = (np.uint32(ab) << 16).view(F32)
                s = F32(max(a, F32(1e-8)) / F32(L))
                wb = fin[(fin & 0x7FFF) <= ab]
                w = (wb << 16).view(F32)
                q_ref = np.clip(np.rint((w / s).astype(F32)), -L - 1, L).astype(F32)
                want = O.f32_to_bf16_bits((q_ref * s).astype(F32))
                r0 = F32(1.0) / s
                for r in (np.nextafter(r0, F32(0)), r0, np.nextafter(r0, F32(np.inf))):
                    lo, hi = F32(r * F32(1 - 2.0 ** -19)), F32(r * F32(1 + 2.0 ** -19))
                    m = F32(1.5 * 2.0 ** 23)                           # the kernel's magic add: half
                    ql = ((w * lo).astype(F32) + m) - m                # even, and +0 for a small w < 0
                    qh = ((w * hi).astype(F32) + m) - m
                    ok = ql == qh
                    rec = O.f32_to_bf16_bits((ql * s).astype(F32)).astype(np.uint32) | (wb & 0x8000)
                    bad = ok & (rec != want)
                    assert not bad.any(), (L, hex(ab), wb[bad][:5], rec[bad][:5], want[bad][:5])
                    big = (wb & 0x7FFF) > ab - 0x600                   # within 2^-12 of the maximum
                    checked += int(big.sum())
                    fast += int((ok & big).sum())
    assert fast > 0.99 * checked                                       # the exact rule is rare


def test_fp8_e4m3_group_bracket_matches_the_codebook_rule():
    """e4m3g_word (FP8_E4M3_G128 on the codebook kernel): for group maxima a across [1, 2) and two
    more binades, every finite bf16 w with |w| <= a, and r any of RN(1/s) and its two neighbours,
    the hardware conversions of RZ(w r_lo) and RZ(w r_hi), where they agree, give the reference's
    W_hat bf16(q s) (nearest E4M3 point of fl32(w / s), ties to the lower value, +0 for zero);
    outside the flagged family (fp8_row_flag) the lower bracket's conversion gives it for every
    w (e4m3g_lower_word)."""
    from oracle import pq_oracle as O
    cb = O.CODEBOOKS["fp8_e4m3"].astype(np.float64)
    mags = cb[cb >= 0]
    even = (np.arange(mags.size) % 2) == 0
    b = np.arange(1 << 16, dtype=np.uint32)
    with np.errstate(invalid="ignore"):
        fin = b[np.isfinite((b << 16).view(F32))]
    checked = fast = 0
    for base in (0x3F80, 0x3080, 0x5300):
        for ab in range(base, base + 0x80, 1 if base == 0x3F80 else 5):
            a = (np.uint32(ab) << 16).view(F32)
            s = F32(max(a, F32(1e-8)) / F32(448.0))
            wb = fin[(fin & 0x7FFF) <= ab]
            w = (wb << 16).view(F32)
            x = (w / s).astype(F32).astype(np.float64)
            ref = np.where(np.abs(x) >= 448.0, np.sign(x) * 448.0, _ties_lower(x, mags))
            want = O.f32_to_bf16_bits((ref * np.float64(s)).astype(F32))
            want = np.where(want == 0x8000, 0, want)
            r0 = F32(1.0) / s
            for r in (np.nextafter(r0, F32(0)), r0, np.nextafter(r0, F32(np.inf))):
                r_lo = _rz32(np.array([np.float64(r) * (1 - 2.0 ** -20)]))[0]
                r_hi = _rz32(np.array([np.float64(r) * (1 + 2.0 ** -20)]))[0]
                cl = _rne(_rz32(w.astype(np.float64) * r_lo), mags, even, 448.0)
                ch = _rne(_rz32(w.astype(np.float64) * r_hi), mags, even, 448.0)
                ok = cl == ch
                rec = O.f32_to_bf16_bits((cl * np.float64(s)).astype(F32))
                got = np.where(rec == 0x8000, 0, rec)                    # -0 -> +0
                bad = ok & (got != want)
                assert not bad.any(), (hex(ab), wb[bad][:5], got[bad][:5], want[bad][:5])
                if not fp8_row_flag(a):                                  # e4m3g_lower_word: every w
                    cm = _rne(np.minimum(_rz32(w.astype(np.float64) * r_lo),
                                         _rz32(w.astype(np.float64) * r_hi)), mags, even, 448.0)
                    low = O.f32_to_bf16_bits((cm * np.float64(s)).astype(F32))
                    low = np.where(low == 0x8000, 0, low)
                    assert (low == want).all(), (hex(ab), wb[low != want][:5])
                big = (wb & 0x7FFF) > ab - 0x600
                checked += int(big.sum())
                fast += int((ok & big).sum())
    assert fast > 0.99 * checked
