"""CPU oracle for the quantization-cost hot path — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference algorithms that the CUDA
kernels in `prismaquant_b200` replace.  It exists to check those kernels:
only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg
may import it, and never as the thing measured or shipped.

Every function cites the reference code it follows (paths relative to the
prismaquant project).  Arithmetic follows the reference's torch op chain
step by step in float32 (numpy float32 ops are IEEE round-to-nearest-even,
as torch's CPU kernels are), so results are bit-identical, not just close:

* cost path  — prismaquant/format_registry.py:175-233 (`_snap_scale_e8m0`,
  `_rtn_fp_codebook`), prismaquant/measure_quant_cost.py:452-548
  (`_batched_codebook_rtn`, `_batched_quantize`) and the MSE at
  prismaquant/measure_quant_cost.py:304-305,631-632.
* export path — prismaquant/export_native_compressed.py:80-136,226-233
  (`FLOAT_TO_E2M1`, `_round_to_codebook`, `pack_fp4_indices`),
  :1045-1129 (NVFP4), :1135-1194 (MXFP8), :1197-1226 (FP8 dynamic),
  :2051-2099 (fused-sibling joint global).
* Fisher      — prismaquant/sensitivity_probe.py:451-504
  (`_GradNormCapture.backward`) and the per-token estimator that replaces
  the GEMM-then-square of :1115-1152.

torch.log2 is not correctly rounded everywhere, and the E8M0 exponents
depend on its exact float32 output.  `E8M0Thresholds` recovers, per binade,
the mantissa at which `ceil(log2(x))` / `round(log2(x))` steps up, by
bisection over torch's own CPU log2 (monotone in every binade: checked
exhaustively when the CUDA tables are generated).
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass

import numpy as np

F32 = np.float32

# ---------------------------------------------------------------------------
# bf16 / fp8 bit helpers
# ---------------------------------------------------------------------------


def bf16_bits_to_f32(u16: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32 values (exact)."""
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(F32)


def f32_to_bf16_bits(f: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits with round-to-nearest-even, NaN -> 0x7FC0.

    Same rounding as torch's c10::BFloat16 conversion (the `.to(bfloat16)`
    at prismaquant/format_registry.py:233).
    """
    f = np.ascontiguousarray(f, dtype=F32)
    u = f.view(np.uint32)
    bias = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    out = ((u + bias) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        out = out.copy()
        out[nan] = 0x7FC0
    return out


def bf16_round(f: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 value, returned as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(f))


def f32_to_e4m3fn_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> float8_e4m3fn bit pattern, round-to-nearest-even.

    OCP FP8 E4M3 (bias 7, no infinities, 0x7F/0xFF = NaN, max 448,
    subnormals m/8 * 2^-6).  Inputs with |x| >= 480 map to NaN like torch's
    `.to(torch.float8_e4m3fn)`; every export call site clamps to +-448
    first, so that branch never fires on the hot path.
    """
    x = np.ascontiguousarray(x, dtype=F32)
    sign = np.signbit(x).astype(np.uint8) << np.uint8(7)
    a = np.abs(x).astype(np.float64)  # exact
    out = np.zeros(x.shape, dtype=np.uint8)
    sub = a < 2.0 ** -6
    # subnormals: grid 2^-9, RNE via rint (half-to-even).  m == 8 becomes
    # the smallest normal (code 0x08), which is the right bit pattern.
    out[sub] = np.rint(a[sub] * 512.0).astype(np.uint8)
    nrm = ~sub
    if nrm.any():
        an = a[nrm]
        mant, exp = np.frexp(an)          # an = mant * 2^exp, mant in [0.5, 1)
        e = exp - 1                       # an = (2*mant) * 2^e, 2*mant in [1, 2)
        m = np.rint((2.0 * mant - 1.0) * 8.0)   # RNE on the 3-bit mantissa
        carry = m >= 8.0
        e = np.where(carry, e + 1, e)
        m = np.where(carry, 0.0, m)
        code = ((e + 7).astype(np.int64) << 3) | m.astype(np.int64)
        big = (an >= 480.0) | np.isnan(an) | (code > 0x7E)
        code = np.where(big, 0x7F, code)
        out[nrm] = code.astype(np.uint8)
    nan = np.isnan(x)
    out[nan] = 0x7F
    return out | sign


def e4m3fn_bits_to_f32(b: np.ndarray) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint8)
    s = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = (b & 7).astype(np.float64)
    v = np.where(e == 0, m / 8.0 * 2.0 ** -6, (1.0 + m / 8.0) * np.exp2(e.astype(np.float64) - 7.0))
    v = np.where((b & 0x7F) == 0x7F, np.nan, v)
    return (s * v).astype(F32)


# ---------------------------------------------------------------------------
# E8M0 exponents (torch float32 log2 + ceil / round)
# ---------------------------------------------------------------------------


class E8M0Thresholds:
    """Per-binade mantissa thresholds reproducing torch's CPU
    `ceil(log2(s))` (export, export_native_compressed.py:1153-1154) and
    `round(log2(s))` (cost path, format_registry.py:189-190).

    For a positive float32 s = 2^k * (1 + m/2^23) (k in [-126, 127]) and for
    the subnormal binade [2^-127, 2^-126) (k = -127, m counted from 2^22):
      ceil(log2 s)  == k   iff m <= ceil_last[k]  (else k + 1)
      round(log2 s) == k+1 iff m >= round_first[k] (else k)
    Thresholds are found by bisection over torch.log2 itself.
    """

    def __init__(self):
        import torch

        ks = np.arange(-126, 128, dtype=np.int64)
        nk = ks.size

        def vals(k, m):
            bits = ((k + 127) << 23) | m
            return torch.from_numpy(bits.astype(np.uint32).view(F32).copy())

        def first_true(pred):
            # smallest m in [0, 2^23] with pred(k, m) true (pred monotone in m)
            lo = np.zeros(nk, dtype=np.int64)
            hi = np.full(nk, 1 << 23, dtype=np.int64)
            while np.any(lo < hi):
                mid = (lo + hi) // 2
                midc = np.minimum(mid, (1 << 23) - 1)
                t = pred(ks, midc) & (mid < (1 << 23))
                hi = np.where(t & (lo < hi), mid, hi)
                lo = np.where((~t) & (lo < hi), mid + 1, lo)
            return lo

        def ceil_up(k, m):
            r = torch.ceil(torch.log2(vals(k, m))).numpy().astype(np.int64)
            return r > k

        def round_up(k, m):
            r = torch.round(torch.log2(vals(k, m))).numpy().astype(np.int64)
            return r > k

        self.ceil_last = {int(k): int(v) - 1 for k, v in zip(ks, first_true(ceil_up))}
        self.round_first = {int(k): int(v) for k, v in zip(ks, first_true(round_up))}
        # subnormal binade [2^-127, 2^-126): m runs over [2^22, 2^23)
        sub = np.arange(1 << 22, 1 << 23, dtype=np.uint32)
        c = torch.ceil(torch.log2(torch.from_numpy(sub.view(F32).copy()))).numpy()
        self.ceil_last[-127] = int(np.count_nonzero(c <= -127)) - 1

    def _split(self, s: np.ndarray):
        s = np.asarray(s, dtype=F32)
        u = s.view(np.uint32).astype(np.int64)
        e = (u >> 23) & 0xFF
        m = u & 0x7FFFFF
        k = e - 127
        return k, m, e

    def ceil_log2(self, s: np.ndarray) -> np.ndarray:
        """torch.ceil(torch.log2(s)).clamp(-127, 127) for s > 0 (float32)."""
        k, m, e = self._split(s)
        out = np.empty(k.shape, dtype=np.int64)
        nrm = e > 0
        tab = np.array([self.ceil_last[int(i)] for i in range(-126, 128)], dtype=np.int64)
        kk = k[nrm]
        out[nrm] = np.where(m[nrm] <= tab[kk + 126], kk, kk + 1)
        subn = ~nrm
        ms = m[subn]
        hi_band = ms >= (1 << 22)
        r = np.full(ms.shape, -127, dtype=np.int64)
        r[hi_band] = np.where(ms[hi_band] - (1 << 22) <= self.ceil_last[-127], -127, -126)
        out[subn] = r
        return np.clip(out, -127, 127)

    def round_log2(self, s: np.ndarray) -> np.ndarray:
        """torch.round(torch.log2(max(s, 2^-127))).clamp(-127, 127), s normal or +inf (a group
        holding an infinity: log2 is inf, clamped to 127)."""
        k, m, e = self._split(s)
        if np.any(e == 0):
            raise ValueError("cost-path MX scale is never subnormal (amax >= 1e-8)")
        if np.any(np.isnan(s)):
            raise ValueError("NaN scale: the reference's group is NaN throughout")
        tab = np.array([self.round_first[int(i)] for i in range(-126, 128)], dtype=np.int64)
        kc = np.minimum(k, 127)
        out = np.where(np.isinf(s), 127, np.where(m >= tab[kc + 126], kc + 1, kc))
        return np.clip(out, -127, 127)


_E8M0: E8M0Thresholds | None = None


def e8m0() -> E8M0Thresholds:
    global _E8M0
    if _E8M0 is None:
        _E8M0 = E8M0Thresholds()
    return _E8M0


# ---------------------------------------------------------------------------
# Codebooks (format_registry.py:237-241, 275-288)
# ---------------------------------------------------------------------------


def e2m1_codebook() -> np.ndarray:
    vals = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    return np.array(sorted(set([0.0] + vals[1:] + [-v for v in vals[1:]])), dtype=F32)


def e4m3_codebook() -> np.ndarray:
    codes = {0.0}
    for exp in range(16):
        for m in range(8):
            val = (m / 8) * 2.0 ** -6 if exp == 0 else (1 + m / 8) * 2.0 ** (exp - 7)
            codes.add(val)
            codes.add(-val)
    return np.array(sorted(c for c in codes if abs(c) <= 448.0), dtype=F32)


def e3m2_codebook() -> np.ndarray:
    """format_registry.py:244-251: (1 + m/4) 2^(exp-3), exp 0..7, m 0..3 (no subnormals), and 0."""
    codes = {0.0}
    for exp in range(8):
        for m in range(4):
            v = (1 + m / 4) * 2.0 ** (exp - 3)
            codes.update((v, -v))
    return np.array(sorted(codes), dtype=F32)


def e2m3_codebook() -> np.ndarray:
    """format_registry.py:254-261: (1 + m/8) 2^(exp-1), exp 0..3, m 0..7 (no subnormals), and 0."""
    codes = {0.0}
    for exp in range(4):
        for m in range(8):
            v = (1 + m / 8) * 2.0 ** (exp - 1)
            codes.update((v, -v))
    return np.array(sorted(codes), dtype=F32)


def e2m0_codebook() -> np.ndarray:
    """format_registry.py:264-272: 2^(exp-2), exp 0..3, and 0: {0, +-.25, +-.5, +-1, +-2}."""
    codes = {0.0}
    for exp in range(4):
        v = 2.0 ** (exp - 2)
        codes.update((v, -v))
    return np.array(sorted(codes), dtype=F32)


def e5m2_codebook() -> np.ndarray:
    """format_registry.py:291-300: subnormals (m/4) 2^-14 and (1 + m/4) 2^(exp-15) for exp 1..31.
    Exponent 31 is kept as finite values, so the largest magnitude is 1.75 * 2^16 = 114688."""
    codes = {0.0}
    for exp in range(32):
        for m in range(4):
            v = (m / 4) * 2.0 ** -14 if exp == 0 else (1 + m / 4) * 2.0 ** (exp - 15)
            codes.update((v, -v))
    return np.array(sorted(codes), dtype=F32)


CODEBOOKS = {"fp4_e2m1": e2m1_codebook(), "fp8_e4m3": e4m3_codebook(), "fp6_e3m2": e3m2_codebook(),
             "fp6_e2m3": e2m3_codebook(), "fp3_e2m0": e2m0_codebook(), "fp8_e5m2": e5m2_codebook()}

# (codebook, group_size, mx_scale) for the formats on the hot path,
# format_registry.py:368-376 (NVFP4), :418-426 (MXFP8), :457-465 (FP8_E4M3).
COST_FORMATS = {
    "NVFP4": ("fp4_e2m1", 16, False),
    "NVFP4A16": ("fp4_e2m1", 16, False),
    "MXFP8": ("fp8_e4m3", 32, True),
    "MXFP8_E4M3": ("fp8_e4m3", 32, True),
    "MXFP8A16": ("fp8_e4m3", 32, True),
    "FP8_E4M3": ("fp8_e4m3", 0, False),
    # the rest of the registry: format_registry.py:391-398 (MXFP4), :400-416 (MXFP6), :436-443
    # (MXFP8_E5M2), :466-473 (FP8_E5M2), :505-514 (NVFP3)
    "MXFP4": ("fp4_e2m1", 32, True),
    "MXFP6_E3M2": ("fp6_e3m2", 32, True),
    "MXFP6_E2M3": ("fp6_e2m3", 32, True),
    "MXFP8_E5M2": ("fp8_e5m2", 32, True),
    "FP8_E5M2": ("fp8_e5m2", 0, False),
    "NVFP3": ("fp3_e2m0", 16, False),
}

# Symmetric uniform-integer formats (bits, group_size): format_registry.py:483-500 (INT3, INT2),
# :516-533 (INT8_W8A16 per channel, INT4_W4A16_g128).
INT_FORMATS = {"INT3": (3, 16), "INT2": (2, 16), "INT8_W8A16": (8, 0), "INT4_W4A16_g128": (4, 128)}
FORMAT_ALIASES = {"NVINT2": "INT2", "NVINT3": "INT3"}
IDENTITY_FORMATS = ("BF16", "FP8_SOURCE")   # quantize_dequantize = clone (format_registry.py:536-576)

# ---------------------------------------------------------------------------
# Cost path: RTN quantize-dequantize + MSE_W
# ---------------------------------------------------------------------------


def _grouped(w32: np.ndarray, group_size: int) -> np.ndarray:
    """format_registry.py:207-212: [rows, in] -> [rows, in/g, g] (or one group per row)."""
    in_f = w32.shape[-1]
    w2 = w32.reshape(-1, in_f)
    if group_size > 0 and group_size < in_f:
        if in_f % group_size:
            raise ValueError(f"cannot reshape row of {in_f} into groups of {group_size}")
        return w2.reshape(w2.shape[0], in_f // group_size, group_size)
    return w2.reshape(w2.shape[0], 1, in_f)


def cost_qdq_f32(w_bits: np.ndarray, fmt: str) -> np.ndarray:
    """Cost-path quantize->dequantize of a bf16 tensor (bit patterns),
    returning the bf16-rounded reconstruction as float32 (format_registry.py:194-233).
    """
    fmt = FORMAT_ALIASES.get(fmt, fmt)
    if fmt in IDENTITY_FORMATS:
        return bf16_bits_to_f32(w_bits)
    if fmt in INT_FORMATS:
        return int_qdq_f32(w_bits, *INT_FORMATS[fmt])
    cb_name, group_size, mx = COST_FORMATS[fmt]
    return codebook_qdq_f32(w_bits, cb_name, group_size, mx)


def codebook_qdq_f32(w_bits: np.ndarray, cb_name: str, group_size: int, mx: bool) -> np.ndarray:
    """_rtn_fp_codebook (format_registry.py:194-233) for one codebook, group size and scale mode."""
    cb = CODEBOOKS[cb_name]
    cmax = F32(np.abs(cb).max())
    w32 = bf16_bits_to_f32(w_bits)
    shape = w32.shape
    w2 = _grouped(w32, group_size)
    amax = np.maximum(np.abs(w2).max(axis=-1, keepdims=True), F32(1e-8))
    scale = (amax / cmax).astype(F32)
    if mx:
        sc = np.maximum(scale, F32(2.0 ** -127))
        scale = np.ldexp(F32(1.0), e8m0().round_log2(sc)).astype(F32)
    x = (w2 / scale).astype(F32)
    idx = np.searchsorted(cb, x, side="left")        # torch.bucketize(right=False)
    lo = cb[np.clip(idx - 1, 0, None)]
    hi = cb[np.clip(idx, None, cb.size - 1)]
    choose_hi = np.abs(hi - x) < np.abs(x - lo)      # ties -> lo
    q = np.where(choose_hi, hi, lo).astype(F32)
    rec = (q * scale).astype(F32)
    return bf16_round(rec).reshape(shape)


# measure_quant_cost._batched_quantize (measure_quant_cost.py:516-548) dispatches on the element
# dtype, not on the format's own quantize_dequantize: codebook families (E2M1, E3M2, E2M3, E4M3,
# E5M2) take the format's group size and E8M0 snapping for family "mx", integer families the
# format's bits and group, bfloat16 a clone, anything else (fp3_e2m0 = NVFP3) raises.  So
# FP8_SOURCE (E4M3, group 128, family "fp") is an E4M3 RTN with real g128 scales there, although
# its per-Linear quantize_dequantize is a clone.
# fmt -> (element dtype, family, weight bits, group size), format_registry.py:368-576
REGISTRY_DTYPES = {
    "NVFP4": ("fp4_e2m1", "nv", 4, 16), "NVFP4A16": ("fp4_e2m1", "nv", 4, 16),
    "MXFP4": ("fp4_e2m1", "mx", 4, 32), "MXFP6_E3M2": ("fp6_e3m2", "mx", 6, 32),
    "MXFP6_E2M3": ("fp6_e2m3", "mx", 6, 32), "MXFP8": ("fp8_e4m3", "mx", 8, 32),
    "MXFP8_E4M3": ("fp8_e4m3", "mx", 8, 32), "MXFP8_E5M2": ("fp8_e5m2", "mx", 8, 32),
    "MXFP8A16": ("fp8_e4m3", "mx", 8, 32), "FP8_E4M3": ("fp8_e4m3", "fp", 8, 0),
    "FP8_E5M2": ("fp8_e5m2", "fp", 8, 0), "INT3": ("int3", "nv", 3, 16), "INT2": ("int2", "nv", 2, 16),
    "NVFP3": ("fp3_e2m0", "nv", 3, 16), "INT8_W8A16": ("int8", "int", 8, 0),
    "INT4_W4A16_g128": ("int4", "int", 4, 128), "BF16": ("bfloat16", "fp", 16, 0),
    "FP8_SOURCE": ("fp8_e4m3", "fp", 8, 128),
}
_BATCHED_CODEBOOKS = ("fp4_e2m1", "fp6_e3m2", "fp6_e2m3", "fp8_e4m3", "fp8_e5m2")


def batched_qdq_f32(w_bits: np.ndarray, fmt: str) -> np.ndarray:
    """measure_quant_cost._batched_quantize on a stacked [N, out, in] (or 2-D) bf16 tensor."""
    elt, fam, bits, group = REGISTRY_DTYPES[FORMAT_ALIASES.get(fmt, fmt)]
    if elt in _BATCHED_CODEBOOKS:
        return codebook_qdq_f32(w_bits, elt, group, fam == "mx")
    if elt.startswith("int"):
        return int_qdq_f32(w_bits, bits, group)
    if elt == "bfloat16":
        return bf16_bits_to_f32(w_bits)
    raise ValueError(f"Unknown weight_element_dtype {elt!r} for batched RTN")


def int_qdq_f32(w_bits: np.ndarray, bits: int, group_size: int) -> np.ndarray:
    """_rtn_uniform_int, symmetric (format_registry.py:147-172): scale = max(amax, 1e-8) / (2^(b-1) - 1),
    q = round_half_even(w / scale) clamped to [-2^(b-1), 2^(b-1) - 1], W_hat = bf16(q * scale)."""
    w32 = bf16_bits_to_f32(w_bits)
    shape = w32.shape
    w2 = _grouped(w32, group_size)
    levels = (1 << (bits - 1)) - 1
    amax = np.maximum(np.abs(w2).max(axis=-1, keepdims=True), F32(1e-8))
    scale = (amax / F32(levels)).astype(F32)
    q = np.clip(np.rint((w2 / scale).astype(F32)), -levels - 1, levels).astype(F32)
    return bf16_round((q * scale).astype(F32)).reshape(shape)


def cost_err_bf16(w_bits: np.ndarray, fmt: str) -> np.ndarray:
    """err = (W - W_hat) in bf16 arithmetic (measure_quant_cost.py:631), as float32."""
    w = bf16_bits_to_f32(w_bits)
    return bf16_round((w - cost_qdq_f32(w_bits, fmt)).astype(F32))


FLT_MAX = float(np.finfo(np.float32).max)


def cost_sse(w_bits: np.ndarray, fmt: str) -> float:
    """Sum of err^2: the square is taken in float32 like `err.float().pow(2)`
    (so |err| > 1.8e19 gives inf), the sum in float64; a sum above FLT_MAX is
    inf, as torch's float32 sum would be."""
    e = cost_err_bf16(w_bits, fmt).ravel()
    with np.errstate(over="ignore"):
        sq = (e * e).astype(F32)
    s = float(sq.astype(np.float64).sum())
    return s if s <= FLT_MAX else float("inf")


def cost_mse(w_bits: np.ndarray, fmt: str) -> float:
    """weight_mse = err.pow(2).mean() (measure_quant_cost.py:304-305)."""
    return cost_sse(w_bits, fmt) / max(np.asarray(w_bits).size, 1)


# ---------------------------------------------------------------------------
# Export path
# ---------------------------------------------------------------------------
FLOAT_TO_E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=F32)
NVFP4_MAX = F32(6.0)
FP8_E4M3_MAX = F32(448.0)


def round_to_codebook(values: np.ndarray) -> np.ndarray:
    """export_native_compressed.py:118-136: abs bucketize, ties toward 0, sign bit from signbit."""
    v = np.asarray(values, dtype=F32)
    cb = FLOAT_TO_E2M1
    a = np.abs(v)
    idx = np.searchsorted(cb, a, side="left")
    lo_i = np.clip(idx - 1, 0, cb.size - 1)
    hi_i = np.clip(idx, None, cb.size - 1)
    pick_hi = np.abs(cb[hi_i] - a) < np.abs(a - cb[lo_i])
    abs_idx = np.where(pick_hi, hi_i, lo_i).astype(np.int64)
    return abs_idx + (np.signbit(v).astype(np.int64) << 3)


def pack_fp4_indices(idx: np.ndarray) -> np.ndarray:
    """export_native_compressed.py:226-233: byte = code[2j] | code[2j+1] << 4."""
    idx = np.asarray(idx, dtype=np.int64)
    if idx.shape[-1] % 2:
        raise ValueError("nvfp4 pack requires an even last dim")
    pairs = idx.reshape(*idx.shape[:-1], idx.shape[-1] // 2, 2)
    return (pairs[..., 0] | (pairs[..., 1] << 4)).astype(np.uint8)


def _nvfp4_group_scale(w32: np.ndarray, group_size: int = 16):
    *lead, cols = w32.shape
    if cols % group_size:
        raise ValueError(f"NVFP4 group_size={group_size} ∤ {cols}")
    g = w32.reshape(*lead, cols // group_size, group_size)
    max_abs = np.maximum(np.abs(g).max(axis=-1), F32(1e-12))
    s_g = (max_abs / NVFP4_MAX).astype(F32)
    return g, s_g


def nvfp4_global_real(w32: np.ndarray, group_size: int = 16) -> F32:
    """compute_nvfp4_global_real (export_native_compressed.py:1045-1055)."""
    _, s_g = _nvfp4_group_scale(np.asarray(w32, dtype=F32), group_size)
    return F32(max(F32(s_g.max() / FP8_E4M3_MAX), F32(1e-12)))


def nvfp4_pack(w32: np.ndarray, global_real_override=None, group_size: int = 16):
    """quantize_dequantize_nvfp4 (export_native_compressed.py:1058-1102).

    Returns (weight_packed u8 [rows, cols/2], weight_scale e4m3 bits u8
    [rows, cols/16], weight_global_scale f32 [1]).
    """
    w32 = np.asarray(w32, dtype=F32)
    rows, cols = w32.shape
    g, s_g = _nvfp4_group_scale(w32, group_size)
    if global_real_override is not None:
        glob = F32(max(F32(global_real_override), F32(1e-12)))
    else:
        glob = F32(max(F32(s_g.max() / FP8_E4M3_MAX), F32(1e-12)))
    fp8_real = np.clip((s_g / glob).astype(F32), F32(0), FP8_E4M3_MAX)
    in_grid = (g / np.maximum(s_g, F32(1e-12))[..., None]).astype(F32)
    codes = round_to_codebook(in_grid).reshape(rows, cols)
    return (pack_fp4_indices(codes), f32_to_e4m3fn_bits(fp8_real),
            np.array([F32(1.0) / glob], dtype=F32))


def nvfp4_pack_packed(p32: np.ndarray, group_size: int = 16):
    """quantize_dequantize_nvfp4_packed (export_native_compressed.py:1105-1129): per-expert global."""
    p32 = np.asarray(p32, dtype=F32)
    E, M, N = p32.shape
    g, s_g = _nvfp4_group_scale(p32, group_size)
    glob = np.maximum((s_g.reshape(E, -1).max(axis=-1) / FP8_E4M3_MAX).astype(F32), F32(1e-12))
    fp8_real = np.clip((s_g / glob[:, None, None]).astype(F32), F32(0), FP8_E4M3_MAX)
    in_grid = (g / np.maximum(s_g, F32(1e-12))[..., None]).astype(F32)
    codes = round_to_codebook(in_grid).reshape(E, M, N)
    return (pack_fp4_indices(codes), f32_to_e4m3fn_bits(fp8_real),
            (F32(1.0) / glob).astype(F32))


def joint_global_real(tensors) -> F32:
    """Fused-sibling joint global = max of natural globals
    (export_native_compressed.py:2090-2098, :1671-1683)."""
    return F32(max(nvfp4_global_real(t) for t in tensors))


def _mxfp8_grouped(grouped: np.ndarray):
    """_mxfp8_quantize_grouped (export_native_compressed.py:1138-1162)."""
    s = (np.maximum(np.abs(grouped).max(axis=-1), F32(2.0 ** -127)) / FP8_E4M3_MAX).astype(F32)
    e = e8m0().ceil_log2(s)
    s_g = np.ldexp(F32(1.0), e).astype(F32)
    q = (grouped / np.maximum(s_g, F32(2.0 ** -127))[..., None]).astype(F32)
    q = np.clip(q, -FP8_E4M3_MAX, FP8_E4M3_MAX)
    return f32_to_e4m3fn_bits(q), np.clip(e + 127, 0, 255).astype(np.uint8)


def mxfp8_pack(w32: np.ndarray, group_size: int = 32):
    """quantize_dequantize_mxfp8[_packed] (export_native_compressed.py:1165-1194)."""
    w32 = np.asarray(w32, dtype=F32)
    *lead, cols = w32.shape
    if cols % group_size:
        raise ValueError(f"MXFP8 group_size={group_size} ∤ {cols}")
    q, sc = _mxfp8_grouped(w32.reshape(*lead, cols // group_size, group_size))
    return q.reshape(w32.shape), sc


def fp8_dynamic_pack(w32: np.ndarray):
    """quantize_dequantize_fp8_dynamic[_packed] (export_native_compressed.py:1197-1226)."""
    w32 = np.asarray(w32, dtype=F32)
    s = (np.maximum(np.abs(w32).max(axis=-1, keepdims=True), F32(2.0 ** -127)) / FP8_E4M3_MAX).astype(F32)
    q = np.clip((w32 / s).astype(F32), -FP8_E4M3_MAX, FP8_E4M3_MAX)
    return f32_to_e4m3fn_bits(q), s


# ---------------------------------------------------------------------------
# Fisher statistics
# ---------------------------------------------------------------------------


def sumsq_rows(g_bits: np.ndarray):
    """_GradNormCapture.backward (sensitivity_probe.py:451-482): scalar sum of
    g^2 and the per-row (per expert, per output channel) sum over the last dim."""
    g = bf16_bits_to_f32(g_bits).astype(np.float64)
    per_row = (g * g).sum(axis=-1)
    return float(per_row.sum()), per_row


def rownorm2(x_bits: np.ndarray) -> np.ndarray:
    """Per-token squared L2 norm of a [T, d] bf16 activation, float64."""
    x = bf16_bits_to_f32(x_bits).astype(np.float64)
    return (x * x).sum(axis=-1)


def tokennorm_trace(x_bits: np.ndarray, g_bits: np.ndarray, token_idx=None) -> float:
    """Per-token Fisher trace estimate sum_t ||x_t||^2 ||g_t||^2.

    Equals the reference's ||gy^T x||_F^2 (sensitivity_probe.py:1125-1139)
    when a single token flows through the backward; for T tokens it is the
    per-token (diagonal-in-t) empirical Fisher.  `token_idx` selects the
    rows of x routed to an expert (HF Qwen3MoeExperts.forward `token_idx`),
    with g given only for those routed rows.
    """
    xn = rownorm2(x_bits)
    if token_idx is not None:
        xn = xn[np.asarray(token_idx, dtype=np.int64)]
    gn = rownorm2(g_bits)
    return float(np.dot(xn, gn))


def ref_grad_w_trace(x_bits: np.ndarray, g_bits: np.ndarray) -> float:
    """The reference estimator ||gy^T x||_F^2 (sensitivity_probe.py:1125-1139), in float64."""
    x = bf16_bits_to_f32(x_bits).astype(np.float64)
    g = bf16_bits_to_f32(g_bits).astype(np.float64)
    gw = g.T @ x
    return float((gw * gw).sum())


# ---------------------------------------------------------------------------
# Synthetic inputs (seeded, reproducible on any x86 host with this numpy)
# ---------------------------------------------------------------------------


def synthetic_weight_bits(shape, seed: int, std: float = 0.02, outlier_frac: float = 0.0,
                          outlier_mult: float = 20.0) -> np.ndarray:
    """N(0, std^2) bf16 weight as uint16 bit patterns; optional random
    outliers scaled by `outlier_mult` (the single-Linear sweep's 0.1 % x20)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    n = int(np.prod(shape))
    w = rng.standard_normal(n, dtype=np.float32) * F32(std)
    if outlier_frac > 0:
        k = int(n * outlier_frac)
        idx = rng.permutation(n)[:k]
        w[idx] = w[idx] * F32(outlier_mult)
    return f32_to_bf16_bits(w).reshape(shape)


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()
