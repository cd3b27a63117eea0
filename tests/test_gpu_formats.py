"""The rest of the format registry on the GPU (exact codebook / integer kernel):
MXFP4, MXFP6 E3M2/E2M3, MXFP8/FP8 E5M2, NVFP3, INT2/INT3, INT8_W8A16,
INT4_W4A16_g128 and FP8_SOURCE, against the reference's outputs (golden
fixtures) and the oracle.  Bar: bit-exact W_hat, MSE_W within 1e-5."""
import numpy as np
import pytest
import torch

from oracle import pq_oracle as O
from prismaquant_b200 import format_registry as fr
from prismaquant_b200 import measure_quant_cost as mqc
from tests._helpers import bits_of, to_cuda_bf16

pytestmark = pytest.mark.gpu

EXT_FMTS = ["MXFP4", "MXFP6_E3M2", "MXFP6_E2M3", "MXFP8_E5M2", "FP8_E5M2", "NVFP3", "INT3", "INT2",
            "INT8_W8A16", "INT4_W4A16_g128", "FP8_SOURCE"]
CASES = ["rand_64x128", "rand_33x256", "ties_4x32", "zeros_3x64", "wide_range_8x96", "row1_1x4096",
         "cols16_5x16", "cols48_7x48", "cols8_4x8", "packed_4x32x64", "packed_3x16x96", "bf16mix_128x32"]


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("fmt", EXT_FMTS)
def test_qdq_matches_reference(golden, case, fmt):
    """2-D inputs through the spec's quantize_dequantize, packed 3-D ones through _batched_quantize,
    as the fixtures were made."""
    bits = golden[f"{case}/input"]
    key = f"{case}/cost/{fmt}"
    w = to_cuda_bf16(bits)
    spec = fr.get_format(fmt)
    run = (lambda: mqc._batched_quantize(spec, w)) if bits.ndim == 3 else (lambda: spec.quantize_dequantize(w))
    if f"{key}/error" in golden:
        with pytest.raises(ValueError):
            run()
        return
    np.testing.assert_array_equal(bits_of(run()), golden[f"{key}/qdq"])


def _all_bf16_rows(cols):
    allv = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    fin = allv[np.isfinite(O.bf16_bits_to_f32(allv))]
    fin = np.random.default_rng(cols).permutation(fin)
    return fin[: (fin.size // cols) * cols].reshape(-1, cols)


@pytest.mark.parametrize("fmt", EXT_FMTS + ["FP8_E4M3_G128"])
@pytest.mark.parametrize("cols", [32, 256])
def test_qdq_every_bf16_value_matches_oracle(fmt, cols):
    """Every finite bf16 value, randomly grouped, through the kernel and the oracle."""
    from prismaquant_b200 import _lib
    bits = _all_bf16_rows(cols)
    got = bits_of(_lib.cost_qdq(to_cuda_bf16(bits), fmt)) if fmt != "FP8_SOURCE" else \
        bits_of(fr.get_format(fmt).quantize_dequantize(to_cuda_bf16(bits)))
    if fmt == "FP8_E4M3_G128":
        want = O.f32_to_bf16_bits(O.codebook_qdq_f32(bits, "fp8_e4m3", 128, False))
    else:
        want = O.f32_to_bf16_bits(O.cost_qdq_f32(bits, fmt))
    bad = np.nonzero(got != want)
    assert bad[0].size == 0, (fmt, got[bad][:5], want[bad][:5], bits[bad][:5])


def _oracle_mse(bits, fmt, per_linear):
    rec = O.cost_qdq_f32(bits, fmt) if per_linear else O.batched_qdq_f32(bits, fmt)
    err = O.bf16_round((O.bf16_bits_to_f32(bits) - rec).astype(np.float32))
    with np.errstate(over="ignore"):
        sq = (err * err).astype(np.float32).astype(np.float64)
    return float(sq.sum()) / bits.size


@pytest.mark.parametrize("per_linear", [False, True])
def test_sweep_weight_mse_matches_oracle(per_linear):
    """MSE_W of every registry format over Linears and packed experts, in the batched path's
    semantics (NVFP3 an error, FP8_SOURCE an E4M3 g128 RTN) and in the per-Linear ones."""
    shapes = {"a.q_proj": (96, 256), "b.o_proj": (40, 512), "c.experts.gate_up_proj": (4, 32, 384),
              "d.small": (6, 48)}
    bits = {n: O.synthetic_weight_bits(s, seed=31 + i, outlier_frac=0.01) for i, (n, s) in enumerate(shapes.items())}
    specs = [fr.get_format(f) for f in sorted(fr.REGISTRY)]
    res = mqc.sweep_weight_mse({n: to_cuda_bf16(b) for n, b in bits.items()}, specs, per_linear=per_linear)
    for n, b in bits.items():
        for s in specs:
            got = res[n][s.name]
            try:
                want = _oracle_mse(b, s.name, per_linear)
            except ValueError as e:
                assert isinstance(got, dict) and "error" in got, (n, s.name, got)
                if "Unknown weight_element_dtype" in str(e):
                    assert got["error"] == str(e)
                continue
            assert not isinstance(got, dict), (n, s.name, got)
            assert got == pytest.approx(want, rel=1e-5, abs=1e-30), (n, s.name)


def test_activation_quantizers():
    """MX / FP8-E5M2 formats quantize activations with the same RTN as weights; the integer and
    NVFP3 formats leave them alone; FP8_SOURCE clones (format_registry.py:391-576)."""
    x = to_cuda_bf16(O.synthetic_weight_bits((64, 256), seed=3, std=1.0))
    for f in ("MXFP4", "MXFP6_E3M2", "MXFP6_E2M3", "MXFP8_E5M2", "FP8_E5M2"):
        s = fr.get_format(f)
        assert torch.equal(s.activation_quantize_dequantize(x), s.quantize_dequantize(x))
    for f in ("INT3", "INT2", "NVFP3", "INT8_W8A16", "INT4_W4A16_g128"):
        assert fr.get_format(f).activation_quantize_dequantize(x) is x
    y = fr.get_format("FP8_SOURCE").activation_quantize_dequantize(x)
    assert torch.equal(y, x) and y is not x


def test_shape_errors_raise():
    w = torch.zeros(4, 40, dtype=torch.bfloat16, device="cuda")
    for f in ("MXFP4", "INT3", "NVFP3"):
        with pytest.raises(ValueError):
            fr.get_format(f).quantize_dequantize(w)
    res = mqc.sweep_weight_mse({"w": w}, [fr.get_format("INT3"), fr.get_format("FP8_E5M2")])
    assert "error" in res["w"]["INT3"] and res["w"]["FP8_E5M2"] == 0.0


@pytest.mark.parametrize("fmt", ["FP8_E5M2", "INT8_W8A16", "FP8_E4M3"])
@pytest.mark.parametrize("cols", [12, 20, 36])
def test_rows_off_the_16_byte_grid_match_oracle(fmt, cols):
    """Row-wise formats on rows that are not a multiple of 8 elements take the scalar kernel;
    W_hat must still match the oracle bit for bit."""
    from prismaquant_b200 import _lib
    bits = O.synthetic_weight_bits((33, cols), seed=cols, outlier_frac=0.02)
    if fmt == "FP8_E4M3":   # the exact codebook path scores it for the weighted sum
        h = torch.ones(33 * cols, dtype=torch.float32, device="cuda")
        out = torch.zeros((), dtype=torch.float64, device="cuda")
        _lib.weighted_sse(to_cuda_bf16(bits), fmt, h, out)
        err = O.bf16_round((O.bf16_bits_to_f32(bits) - O.cost_qdq_f32(bits, fmt)).astype(np.float32))
        assert out.item() == pytest.approx(float((err * err).astype(np.float32).astype(np.float64).sum()), rel=1e-5)
        return
    got = bits_of(_lib.cost_qdq(to_cuda_bf16(bits), fmt))
    np.testing.assert_array_equal(got, O.f32_to_bf16_bits(O.cost_qdq_f32(bits, fmt)))


@pytest.mark.parametrize("fmt", EXT_FMTS[:-1] + ["FP8_E4M3_G128"])
def test_misaligned_view_takes_the_scalar_kernel_with_equal_results(fmt):
    """A contiguous view 2 bytes off a 16-byte boundary cannot use 16-byte loads; both kernels
    must give the same W_hat and the same error sum."""
    from prismaquant_b200 import _lib
    bits = O.synthetic_weight_bits((64, 256), seed=5, outlier_frac=0.01)
    w = to_cuda_bf16(bits)
    buf = torch.empty(w.numel() + 1, dtype=torch.bfloat16, device="cuda")
    buf[1:].copy_(w.reshape(-1))
    wm = buf[1:].view(64, 256)
    assert wm.data_ptr() % 16 != 0 and wm.is_contiguous()
    a = bits_of(_lib.cost_qdq(w, fmt))
    b = bits_of(_lib.cost_qdq(wm, fmt))
    np.testing.assert_array_equal(a, b)
    s1 = torch.zeros((), dtype=torch.float64, device="cuda")
    s2 = torch.zeros((), dtype=torch.float64, device="cuda")
    _lib.format_sse(w, fmt, s1)
    _lib.format_sse(wm, fmt, s2)
    assert s1.item() == pytest.approx(s2.item(), rel=1e-6)   # fp32 partials of 8 vs 64 squares


MX_EXT = ["MXFP4", "MXFP6_E3M2", "MXFP6_E2M3", "MXFP8_E5M2"]


def _oracle_sse(bits, fmt):
    err = O.bf16_round((O.bf16_bits_to_f32(bits) - O.cost_qdq_f32(bits, fmt)).astype(np.float32))
    with np.errstate(over="ignore", invalid="ignore"):
        return float((err * err).astype(np.float32).astype(np.float64).sum())


def _special_rows(kind):
    """Rows of 32-element groups that leave the packed path: tiny scales (group exponents below
    -100, whose squares underflow), all-zero groups (the 1e-8 floor) and bf16 subnormals beside
    ordinary groups ("tiny"); a group with an exponent above 100, whose squared error overflows
    fp32 as the reference's does ("huge"); an infinity in a group, whose error is inf - inf
    ("inf")."""
    rng = np.random.default_rng(7)
    f = O.bf16_bits_to_f32(O.synthetic_weight_bits((16, 64), seed=9, outlier_frac=0.0)).astype(np.float32)
    f[1, 32:] *= np.float32(2.0 ** -110)
    f[2, :32] = 0.0
    f[5, :] = rng.standard_normal(64).astype(np.float32) * np.float32(2.0 ** -126)
    if kind == "huge":
        f[0, :32] *= np.float32(2.0 ** 120)
    if kind == "inf":
        f[3, 5] = np.inf
    return O.f32_to_bf16_bits(f)


@pytest.mark.parametrize("kind", ["tiny", "huge", "inf"])
def test_mx_multi_format_sse_special_groups(kind):
    """Groups outside the packed path's range, subnormals, overflowing squares and infinities: the
    oracle's sums, inf and NaN included (the MX formats from one read, the rest one by one)."""
    import warnings
    from prismaquant_b200 import _lib
    bits = _special_rows(kind)
    fmts = MX_EXT + ["INT3", "BF16", "FP8_E5M2", "NVFP3"]
    out = torch.zeros(len(fmts), dtype=torch.float64, device="cuda")
    _lib.format_sse_multi(to_cuda_bf16(bits), fmts, out)
    got = out.cpu().numpy()
    for i, fmt in enumerate(fmts):
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            want = 0.0 if fmt == "BF16" else _oracle_sse(bits, fmt)
        if np.isnan(want):
            assert np.isnan(got[i]), (fmt, got[i])
        elif np.isinf(want):
            assert got[i] == want, (fmt, got[i])
        else:
            assert got[i] == pytest.approx(want, rel=1e-5, abs=1e-30), fmt


def test_mx_multi_format_sse_rejects_before_running():
    """A format that cannot group the rows fails the whole call and adds nothing."""
    from prismaquant_b200 import _lib
    w = to_cuda_bf16(O.synthetic_weight_bits((4, 40), seed=2))
    out = torch.zeros(2, dtype=torch.float64, device="cuda")
    with pytest.raises(ValueError):
        _lib.format_sse_multi(w, ["FP8_E5M2", "MXFP4"], out)
    assert (out == 0).all()


def test_mx_multi_format_sse_repeated_and_mixed_formats():
    """A repeated MX format is scored on its own, a non-MX one by the codebook kernel; every entry
    equals the oracle's sum for its format."""
    from prismaquant_b200 import _lib
    bits = O.synthetic_weight_bits((64, 96), seed=4, outlier_frac=0.01)
    w = to_cuda_bf16(bits)
    fmts = ["MXFP4", "MXFP4", "MXFP6_E2M3", "NVFP3", "MXFP8_E5M2", "MXFP6_E3M2"]
    out = torch.zeros(len(fmts), dtype=torch.float64, device="cuda")
    _lib.format_sse_multi(w, fmts, out)
    for i, f in enumerate(fmts):
        assert out[i].item() == pytest.approx(_oracle_sse(bits, f), rel=1e-5, abs=1e-30), f


INT_GROUPED = ["INT2", "INT3", "INT4_W4A16_g128"]


def _int_tie_rows():
    """Rows whose quotients w / s sit exactly on half-integers (round half even decides) next to
    rows with inexact scales: each group's maximum is L (s = 1) or L x 2^k with odd multiples of
    s / 2 around it, and groups with maximum 1 (s = fl32(1 / L))."""
    rng = np.random.default_rng(3)
    rows = []
    for L in (1, 3, 7):
        for k in (-3, 0, 5):
            half = (rng.integers(-L, L, size=256) + 0.5) * 2.0 ** k   # |x| <= L - 1/2: ties
            half[::16] = L * 2.0 ** k        # the group maximum
            rows.append(half)
        rows.append(rng.uniform(-1, 1, size=256))
    f = np.clip(np.array(rows, dtype=np.float32), -1e30, 1e30)
    return O.f32_to_bf16_bits(f)


@pytest.mark.parametrize("fmt", INT_GROUPED)
@pytest.mark.parametrize("case", ["every_bf16", "ties"])
def test_int_grouped_sse_matches_oracle(fmt, case):
    """The grouped integer formats' squared error (product with exact fallback near midpoints)
    against the oracle, and against the codebook kernel's IEEE division (the weighted sum with
    unit weights)."""
    from prismaquant_b200 import _lib
    bits = _all_bf16_rows(256) if case == "every_bf16" else _int_tie_rows()
    w = to_cuda_bf16(bits)
    got = torch.zeros((), dtype=torch.float64, device="cuda")
    _lib.format_sse(w, fmt, got)
    ref = torch.zeros((), dtype=torch.float64, device="cuda")
    _lib.weighted_sse(w, fmt, torch.ones(bits.size, dtype=torch.float32, device="cuda"), ref)
    want = _oracle_sse(bits, fmt)
    assert got.item() == pytest.approx(want, rel=1e-5, abs=1e-30), fmt
    # fp32 partials of 32 squares here, of 8 there: the sums agree to fp32 rounding
    assert got.item() == pytest.approx(ref.item(), rel=1e-6, abs=1e-30), fmt


@pytest.mark.parametrize("fmt", MX_EXT)
def test_mx_w_hat_across_the_group_exponent_range(fmt):
    """W_hat of 32-element groups whose scales run from 2^-110 to 2^112 (the packed pair path
    serves group exponents within +-90, the per-element path the rest), with ties to the lower
    value planted in every group, the special rows (tiny, huge, an infinity) beside them:
    bit-exact against the oracle."""
    from prismaquant_b200 import _lib
    rng = np.random.default_rng(11)
    shifts = np.arange(-110, 114, 2)
    f = rng.standard_normal((shifts.size, 32)).astype(np.float32)
    f[:, :8] = np.array([0.25, -0.25, 0.75, -0.75, 1.25, -1.25, 3.5, -3.5], np.float32)   # grid midpoints
    f[:, 8] = 6.0                                                   # the group's maximum
    f = f * np.float32(2.0) ** shifts[:, None].astype(np.float32)
    bits = np.concatenate([O.f32_to_bf16_bits(f).reshape(-1, 64)] +
                          [_special_rows(k) for k in ("tiny", "huge", "inf")])
    got = bits_of(_lib.cost_qdq(to_cuda_bf16(bits), fmt))
    with np.errstate(all="ignore"):
        want = O.f32_to_bf16_bits(O.cost_qdq_f32(bits, fmt))
    bad = np.nonzero(got != want)
    assert bad[0].size == 0, (fmt, got[bad][:5], want[bad][:5], bits[bad][:5])


def _moderate_bf16_rows(cols):
    """Every bf16 value of magnitude below 2^60 (squares stay finite), randomly grouped."""
    allv = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    keep = allv[(allv & 0x7FFF) < 0x5D80]
    keep = np.random.default_rng(cols + 1).permutation(keep)
    return keep[: (keep.size // cols) * cols].reshape(-1, cols)


def _nvfp3_threshold_rows():
    """16-element groups around NVFP3's decision points: group maxima a with 3a a bf16 (exact ties
    possible) and not, each group holding a, the bf16 values next to a/16, 3a/16, 3a/8 and 3a/4
    (on them where they are bf16 values) with both signs; beside them all-zero groups and groups
    whose maximum is below 1e-8."""
    groups = []
    for a0 in (1.0, 1.25, 1.5, 1.0078125, 1.3359375, 1.9921875):
        for k in (-20, 0, 7):
            a = np.float32(a0 * 2.0 ** k)
            near = []
            for t in (a / 16, 3 * np.float64(a) / 16, 3 * np.float64(a) / 8, 3 * np.float64(a) / 4):
                b = int(O.f32_to_bf16_bits(np.array([t], np.float32))[0])   # nearest bf16, its neighbours
                near += [b, b + 1, b - 1]
            vals = O.bf16_bits_to_f32(np.array(near, np.uint16))
            for sign in (1, -1):
                g = np.zeros(16, np.float32)
                g[0] = a
                g[1:1 + vals.size] = sign * vals[:15]
                groups.append(g)
    groups.append(np.linspace(-9e-9, 9e-9, 16).astype(np.float32))
    while len(groups) % 4:
        groups.append(np.zeros(16, np.float32))
    return O.f32_to_bf16_bits(np.concatenate(groups).reshape(-1, 64))


@pytest.mark.parametrize("case", ["every_bf16", "moderate_bf16", "thresholds", "tiny", "huge", "inf"])
def test_nvfp3_sse_and_w_hat_match_oracle(case):
    """NVFP3's squared error (fp3sse_kernel) and W_hat (the codebook kernel's comparison path)
    against the oracle, the error sum also against the codebook kernel's division rule (the
    weighted sum with unit weights)."""
    import warnings
    from prismaquant_b200 import _lib
    bits = {"every_bf16": lambda: _all_bf16_rows(256), "moderate_bf16": lambda: _moderate_bf16_rows(256),
            "thresholds": _nvfp3_threshold_rows}.get(case, lambda: _special_rows(case))()
    w = to_cuda_bf16(bits)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        want_sse = _oracle_sse(bits, "NVFP3")
        want_hat = O.f32_to_bf16_bits(O.cost_qdq_f32(bits, "NVFP3"))
    got = torch.zeros((), dtype=torch.float64, device="cuda")
    _lib.format_sse(w, "NVFP3", got)
    ref = torch.zeros((), dtype=torch.float64, device="cuda")
    _lib.weighted_sse(w, "NVFP3", torch.ones(bits.size, dtype=torch.float32, device="cuda"), ref)
    if np.isnan(want_sse) or np.isinf(want_sse):
        assert got.item() == want_sse or (np.isnan(want_sse) and np.isnan(got.item())), (got.item(), want_sse)
    else:
        assert got.item() == pytest.approx(want_sse, rel=1e-5, abs=1e-30)
        assert got.item() == pytest.approx(ref.item(), rel=1e-6, abs=1e-30)
    hat = bits_of(_lib.cost_qdq(w, "NVFP3"))
    bad = np.nonzero(hat != want_hat)
    assert bad[0].size == 0, (hat[bad][:5], want_hat[bad][:5], bits[bad][:5])


def _e5m2_rows():
    """Rows for FP8_E5M2's bracket path: maxima with significand 1.75 (s a power of two, so w / s
    is exact and every codebook midpoint among the elements is an exact tie), others with inexact
    scales; elements on and next to midpoints, +-0, values far below the maximum (the exact rule)
    and values near it (saturation)."""
    rng = np.random.default_rng(5)
    rows = []
    for amax in (1.75, 1.75 * 2.0 ** -9, 1.0078125, 1.5, 1.75 * 2.0 ** 20):
        s = np.float64(np.float32(np.float32(amax) / np.float32(114688.0)))
        for _ in range(3):
            k = rng.integers(-14, 16, size=256)
            mid = (1 + (2 * rng.integers(0, 4, size=256) + 1) / 8) * 2.0 ** k * s      # midpoints x s
            row = np.where(rng.random(256) < 0.5, mid, rng.standard_normal(256) * amax / 3)
            row = np.clip(row, -amax, amax) * np.where(rng.random(256) < 0.5, -1, 1)
            row[:4] = [amax, -amax, 0.0, -0.0]
            row[4:8] = np.array([2.0 ** -40, -2.0 ** -40, 2.0 ** -20, 1e-30]) * amax
            row[8] = 0.97 * amax
            rows.append(row)
    return O.f32_to_bf16_bits(np.array(rows, np.float32))


def test_fp8_e5m2_bracket_path_matches_oracle():
    """FP8_E5M2's W_hat (bit-exact) and squared error (rel 1e-5) against the oracle on rows with
    exact ties, zeros of both signs and elements on the exact rule, the error also against the
    codebook kernel's per-element rule (the weighted sum with unit weights)."""
    from prismaquant_b200 import _lib
    bits = _e5m2_rows()
    w = to_cuda_bf16(bits)
    hat = bits_of(_lib.cost_qdq(w, "FP8_E5M2"))
    want = O.f32_to_bf16_bits(O.cost_qdq_f32(bits, "FP8_E5M2"))
    bad = np.nonzero(hat != want)
    assert bad[0].size == 0, (hat[bad][:5], want[bad][:5], bits[bad][:5])
    got = torch.zeros((), dtype=torch.float64, device="cuda")
    _lib.format_sse(w, "FP8_E5M2", got)
    ref = torch.zeros((), dtype=torch.float64, device="cuda")
    _lib.weighted_sse(w, "FP8_E5M2", torch.ones(bits.size, dtype=torch.float32, device="cuda"), ref)
    assert got.item() == pytest.approx(_oracle_sse(bits, "FP8_E5M2"), rel=1e-5, abs=1e-30)
    assert got.item() == pytest.approx(ref.item(), rel=1e-6, abs=1e-30)


@pytest.mark.parametrize("kind", ["tiny", "huge", "inf"])
@pytest.mark.parametrize("fmt", EXT_FMTS[:-1] + ["FP8_E4M3_G128"])
def test_w_hat_of_special_groups_matches_oracle(fmt, kind):
    """W_hat of groups with tiny scales, bf16 subnormals, all zeros, overflowing scales and an
    infinity, for every format of the codebook kernel: bit-exact against the oracle (a NaN
    reconstruction, 0 x an infinite scale, is written 0x7FC0 as torch writes it)."""
    import warnings
    from prismaquant_b200 import _lib
    bits = _special_rows(kind).reshape(8, 128)
    got = bits_of(_lib.cost_qdq(to_cuda_bf16(bits), fmt))
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        if fmt == "FP8_E4M3_G128":
            want = O.f32_to_bf16_bits(O.codebook_qdq_f32(bits, "fp8_e4m3", 128, False))
        else:
            want = O.f32_to_bf16_bits(O.cost_qdq_f32(bits, fmt))
    bad = np.nonzero(got != want)
    assert bad[0].size == 0, (fmt, got[bad][:5], want[bad][:5], bits[bad][:5])


def _int8_tie_rows():
    """Rows for the integer row path: maxima 127 x 2^k (s = 2^k, so elements at half-integer
    multiples of s are exact ties) beside rows with inexact scales, negative values that round
    to zero, and +-0."""
    rng = np.random.default_rng(8)
    rows = []
    for k in (-9, 0, 6):
        half = (rng.integers(-127, 127, size=512) + 0.5) * 2.0 ** k
        half[0] = 127 * 2.0 ** k
        half[1:5] = np.array([-0.3, -0.5, 0.5, -0.0]) * 2.0 ** k
        rows.append(half)
        rows.append(rng.standard_normal(512) * 2.0 ** k)
    return O.f32_to_bf16_bits(np.array(rows, dtype=np.float32))


@pytest.mark.parametrize("fmt,cols", [("INT8_W8A16", 512), ("INT3", 16), ("INT4_W4A16_g128", 128)])
def test_integer_row_path_matches_oracle(fmt, cols):
    """The row path's integer bracket (INT8_W8A16, and INT3 / INT4 rows one group long): W_hat
    bit-exact and the squared error within 1e-5 of the oracle, on exact ties, values that round
    to -0 and ordinary rows; the error also against the per-element rule (unit weights)."""
    from prismaquant_b200 import _lib
    bits = _int8_tie_rows().reshape(-1, cols)
    w = to_cuda_bf16(bits)
    hat = bits_of(_lib.cost_qdq(w, fmt))
    want = O.f32_to_bf16_bits(O.cost_qdq_f32(bits, fmt))
    bad = np.nonzero(hat != want)
    assert bad[0].size == 0, (fmt, hat[bad][:5], want[bad][:5], bits[bad][:5])
    got = torch.zeros((), dtype=torch.float64, device="cuda")
    _lib.format_sse(w, fmt, got)
    ref = torch.zeros((), dtype=torch.float64, device="cuda")
    _lib.weighted_sse(w, fmt, torch.ones(bits.size, dtype=torch.float32, device="cuda"), ref)
    assert got.item() == pytest.approx(_oracle_sse(bits, fmt), rel=1e-5, abs=1e-30)
    assert got.item() == pytest.approx(ref.item(), rel=1e-6, abs=1e-30)


def test_fp8_e4m3_g128_bracket_path_matches_oracle():
    """FP8_E4M3_G128 (real scale per 128 elements) on the codebook kernel's bracket: groups whose
    maxima have significands that are multiples of 7 (exact scales, so E4M3 midpoints among the
    quotients are exact ties, taken by the exact rule), signed zeros and values that round to
    zero; W_hat bit-exact, squared error within 1e-5 of the oracle and 1e-6 of the per-element
    rule (unit weights)."""
    from prismaquant_b200 import _lib
    rng = np.random.default_rng(14)
    b = np.arange(1 << 15, dtype=np.uint32)
    mags = b[b < 0x7F80]
    groups = []
    for sig in (1.75, 1.3125, 1.09375, 1.0, 1.5390625):
        for k in (-20, 0, 11):
            a_bits = int(O.f32_to_bf16_bits(np.array([sig * 2.0 ** k], np.float32))[0])
            pool = mags[mags <= a_bits]
            g = rng.choice(pool[pool > a_bits - 0x500], size=127).astype(np.uint32)
            g |= rng.integers(0, 2, size=127).astype(np.uint32) << 15
            g[:3] = [0, 0x8000, 0x8000 | (a_bits - 0x500)]
            groups.append(np.concatenate([[a_bits], g]).astype(np.uint16))
    bits = np.array(groups).reshape(-1, 384)                     # three groups a row
    w = to_cuda_bf16(bits)
    hat = bits_of(_lib.cost_qdq(w, "FP8_E4M3_G128"))
    want = O.f32_to_bf16_bits(O.codebook_qdq_f32(bits, "fp8_e4m3", 128, False))
    bad = np.nonzero(hat != want)
    assert bad[0].size == 0, (hat[bad][:5], want[bad][:5], bits[bad][:5])
    err = O.bf16_round((O.bf16_bits_to_f32(bits) - O.codebook_qdq_f32(bits, "fp8_e4m3", 128, False)).astype(np.float32))
    got = torch.zeros((), dtype=torch.float64, device="cuda")
    _lib.format_sse(w, "FP8_E4M3_G128", got)
    ref = torch.zeros((), dtype=torch.float64, device="cuda")
    _lib.weighted_sse(w, "FP8_E4M3_G128", torch.ones(bits.size, dtype=torch.float32, device="cuda"), ref)
    assert got.item() == pytest.approx(float((err * err).astype(np.float32).astype(np.float64).sum()), rel=1e-5)
    assert got.item() == pytest.approx(ref.item(), rel=1e-6)
