"""Cost path on the GPU vs the reference (golden fixtures) and the oracle.

Bar: quantize-dequantize reconstructions bit-exact; MSE_W within 1e-5
relative (fp64 accumulation of fp32 squares vs the reference's fp32 mean)."""
import numpy as np
import pytest
import torch

from oracle import pq_oracle as O
from prismaquant_b200 import format_registry as fr
from prismaquant_b200 import measure_quant_cost as mqc
from tests._helpers import assert_rel, bits_of, to_cuda_bf16

pytestmark = pytest.mark.gpu

CASES = ["rand_64x128", "rand_33x256", "ties_4x32", "zeros_3x64", "wide_range_8x96",
         "row1_1x4096", "cols16_5x16", "cols48_7x48", "cols8_4x8", "packed_4x32x64", "packed_3x16x96"]
FMTS = ["NVFP4", "MXFP8", "FP8_E4M3", "BF16"]


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("fmt", FMTS)
def test_qdq_matches_reference(golden, case, fmt):
    bits = golden[f"{case}/input"]
    w = to_cuda_bf16(bits)
    spec = fr.get_format(fmt)
    key = f"{case}/cost/{fmt}"
    if f"{key}/error" in golden:
        with pytest.raises(ValueError):
            spec.quantize_dequantize(w)
        return
    out = spec.quantize_dequantize(w) if w.dim() == 2 else mqc._batched_quantize(spec, w)
    np.testing.assert_array_equal(bits_of(out), golden[f"{key}/qdq"])


@pytest.mark.parametrize("case", CASES)
def test_fused_sweep_matches_reference(golden, case):
    w = to_cuda_bf16(golden[f"{case}/input"])
    specs = [fr.get_format(f) for f in FMTS]
    res = mqc.sweep_weight_mse({"t": w}, specs)["t"]
    for f in FMTS:
        key = f"{case}/cost/{f}"
        if f"{key}/error" in golden:
            assert isinstance(res[f], dict) and "error" in res[f]
        else:
            assert_rel(res[f], float(golden[f"{key}/mse"][0]), 1e-5, f"{case} {f}")


@pytest.mark.parametrize("shape,seed", [((512, 4096), 1), ((96, 14336), 2), ((4, 128, 768), 3),
                                        ((1000, 1536), 4), ((3, 2048), 5), ((77, 48), 6), ((13, 24), 7)])
def test_sweep_and_qdq_vs_oracle(shape, seed):
    bits = O.synthetic_weight_bits(shape, seed=seed, outlier_frac=0.002)
    w = to_cuda_bf16(bits)
    specs = [fr.get_format(f) for f in FMTS]
    res = mqc.sweep_weight_mse({"t": w}, specs)["t"]
    for f in FMTS:
        try:
            ref_q = O.f32_to_bf16_bits(O.cost_qdq_f32(bits, f))
        except ValueError:
            assert isinstance(res[f], dict)
            continue
        q = mqc._batched_quantize(fr.get_format(f), w)
        np.testing.assert_array_equal(bits_of(q), ref_q, err_msg=f)
        assert_rel(res[f], O.cost_mse(bits, f), 1e-5, f)


def test_many_tensors_one_launch():
    """Hundreds of tensors of mixed shapes in one sweep call (several launches
    of the descriptor table) give the per-tensor oracle values."""
    rng = np.random.default_rng(0)
    shapes = [(int(rng.integers(1, 40)), int(rng.choice([16, 32, 64, 128, 256, 4096]))) for _ in range(400)]
    bits = [O.synthetic_weight_bits(s, seed=100 + i) for i, s in enumerate(shapes)]
    specs = [fr.get_format(f) for f in ("NVFP4", "MXFP8", "FP8_E4M3")]
    res = mqc.sweep_weight_mse({str(i): to_cuda_bf16(b) for i, b in enumerate(bits)}, specs)
    for i, b in enumerate(bits):
        for s in specs:
            assert_rel(res[str(i)][s.name], O.cost_mse(b, s.name), 1e-5, f"{i} {s.name} {shapes[i]}")


def test_all_bf16_values_rtn():
    """Every finite bf16 value, in rows whose amax fixes exact power-of-two
    scales, goes through every format's rounding (ties, subnormals, saturation)."""
    allv = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    f = O.bf16_bits_to_f32(allv)
    vals = allv[np.isfinite(f) & (np.abs(f) < 1e30)]
    vals = vals[: (vals.size // 256) * 256].reshape(-1, 256)
    for fmt in ("NVFP4", "MXFP8", "FP8_E4M3"):
        q = fr.get_format(fmt).quantize_dequantize(to_cuda_bf16(vals))
        np.testing.assert_array_equal(bits_of(q), O.f32_to_bf16_bits(O.cost_qdq_f32(vals, fmt)), err_msg=fmt)


def test_linear4096_digest(full_digests):
    """Full single-Linear sweep (4096x4096, 0.1 % x20 outliers, seed 0) against
    the reference's own outputs (SHA-256 of W_hat) and MSE_W."""
    d = full_digests["linear4096"]
    bits = O.synthetic_weight_bits((4096, 4096), seed=0, outlier_frac=0.001)
    assert O.digest(bits) == d["input"], "synthetic generator differs on this host"
    w = to_cuda_bf16(bits)
    specs = [fr.get_format(f) for f in FMTS]
    res = mqc.sweep_weight_mse({"w": w}, specs)["w"]
    for f in FMTS:
        assert O.digest(bits_of(fr.get_format(f).quantize_dequantize(w))) == d[f"qdq/{f}"], f
        assert_rel(res[f], d[f"mse/{f}"], 1e-5, f)


def test_fast_sweep_per_row_exact():
    """The fast sweep path (bracketed quotients, packed conversions, SWAR MX
    rounding) against the oracle with every finite bf16 value, one 32-element
    row per tensor so that a single mis-rounded element shows (rel 2e-6 is
    the fp32-partial-sum noise of 32 exact squares)."""
    allv = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    f = O.bf16_bits_to_f32(allv)
    vals = allv[np.isfinite(f) & (np.abs(f) < 1e30)]
    rng = np.random.default_rng(1)
    vals = rng.permutation(vals)
    rows = vals[: (vals.size // 32) * 32].reshape(-1, 32)
    # scale rows into realistic ranges: each row keeps its bf16 patterns but rows with huge spread are common
    specs = [fr.get_format(f) for f in ("NVFP4", "MXFP8", "FP8_E4M3")]
    named = {str(i): to_cuda_bf16(r.reshape(1, 32)) for i, r in enumerate(rows)}
    res = mqc.sweep_weight_mse(named, specs)
    bad = []
    for i, r in enumerate(rows):
        b = r.reshape(1, 32)
        for s in specs:
            ref = O.cost_mse(b, s.name)
            got = res[str(i)][s.name]
            if not (got == ref or abs(got - ref) <= 2e-6 * max(abs(ref), 1e-38)):
                bad.append((i, s.name, got, ref))
    assert not bad, bad[:10]


def test_fast_sweep_gaussian_rows_exact():
    """Same per-row check on realistic N(0, 0.02^2) rows with outliers, many tensors."""
    bits = O.synthetic_weight_bits((3000, 32), seed=77, outlier_frac=0.01)
    specs = [fr.get_format(f) for f in ("NVFP4", "MXFP8", "FP8_E4M3")]
    res = mqc.sweep_weight_mse({str(i): to_cuda_bf16(bits[i:i + 1]) for i in range(bits.shape[0])}, specs)
    for i in range(bits.shape[0]):
        for s in specs:
            assert_rel(res[str(i)][s.name], O.cost_mse(bits[i:i + 1], s.name), 2e-6, f"row {i} {s.name}")


def _tie_rows(n_rows, seed):
    """32-element rows seeded with the values where the fast path's bracket is ambiguous:
    NVFP4 near-ties m * fl(amax/6) for every E2M1 midpoint m, FP8 near-ties m * fl(row_max/448) for
    E4M3 midpoints, MXFP8 bit patterns whose low 4 mantissa bits are 1000, both signs, plus
    subnormal and signed-zero elements."""
    rng = np.random.default_rng(seed)
    e2m1_mid = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=np.float32)
    e4m3 = O.e4m3_codebook()
    e4m3 = np.unique(np.abs(e4m3[np.isfinite(e4m3)]))
    e4m3_mid = ((e4m3[:-1] + e4m3[1:]) / 2).astype(np.float32)
    rows = []
    for _ in range(n_rows):
        amax_bits = np.uint16(rng.integers(0x3C00, 0x4100))          # row/group max in [2^-7, 8)
        amax = O.bf16_bits_to_f32(np.array([amax_bits]))[0]
        s_nv = np.float32(amax / np.float32(6))
        s_f8 = np.float32(amax / np.float32(448))
        cand = np.concatenate([e2m1_mid * s_nv, rng.choice(e4m3_mid, 16) * s_f8]).astype(np.float32)
        cb = O.f32_to_bf16_bits(cand)
        cb = np.concatenate([cb, cb + 1, cb - 1]).astype(np.uint16)   # the near-tie value and neighbours
        picks = rng.choice(cb, 27)
        mx_tie = ((rng.integers(0x3800, 0x3F00, 3) & 0xFFF0) | 0x8).astype(np.uint16)
        extra = np.array([0x0001, 0x8000], dtype=np.uint16)          # a subnormal and -0.0
        r = np.concatenate([picks, mx_tie, extra])
        r = r ^ (rng.integers(0, 2, r.size).astype(np.uint16) << 15)  # random signs
        r[rng.integers(0, 16)] = amax_bits                            # each 16-group has a known max
        r[16 + rng.integers(0, 16)] = amax_bits
        rows.append(r[:32])
    return np.stack(rows).astype(np.uint16)


def test_fast_sweep_tie_rows_exact():
    """Rows built from near-tie values: per-row MSE of every format (rel 2e-6, the fp32 partial-sum
    noise) and the fused NVFP4 export bytes (bit-exact) against the oracle."""
    from prismaquant_b200 import export_native_compressed as enc
    from tests._helpers import u8_of
    rows = _tie_rows(600, seed=5)
    specs = [fr.get_format(f) for f in ("NVFP4", "MXFP8", "FP8_E4M3")]
    named = {str(i): to_cuda_bf16(r.reshape(1, 32)) for i, r in enumerate(rows)}
    costs, outs = enc.sweep_and_export(named, specs)
    bad = []
    for i, r in enumerate(rows):
        b = r.reshape(1, 32)
        for s in specs:
            ref = O.cost_mse(b, s.name)
            got = costs[str(i)][s.name]
            if not (got == ref or abs(got - ref) <= 2e-6 * max(abs(ref), 1e-38)):
                bad.append((i, s.name, got, ref))
        p, sc, g = O.nvfp4_pack(O.bf16_bits_to_f32(b))
        if not (np.array_equal(u8_of(outs[str(i)][0]), p) and np.array_equal(u8_of(outs[str(i)][1]), sc)):
            bad.append((i, "export"))
    assert not bad, bad[:10]


@pytest.mark.parametrize("fmt", ["NVFP4", "MXFP8", "FP8_E4M3"])
def test_qdq_tie_rows_exact(fmt):
    """W_hat of rows built from near-tie values (the fast kernel's uncertain pairs, rewritten by
    its fix-ups) and of rows with out-of-range maxima (its exact path), bit-exact with the oracle."""
    rows = _tie_rows(600, seed=7)
    tiny = (O.synthetic_weight_bits((8, 32), seed=9) & np.uint16(0x807F)) | np.uint16(0x0100)   # |w| ~ 1e-37
    bits = np.concatenate([rows, tiny]).astype(np.uint16)
    q = fr.get_format(fmt).quantize_dequantize(to_cuda_bf16(bits))
    np.testing.assert_array_equal(bits_of(q), O.f32_to_bf16_bits(O.cost_qdq_f32(bits, fmt)), err_msg=fmt)


@pytest.mark.parametrize("fmts", [("NVFP4", "MXFP8", "FP8_E4M3"), ("NVFP4", "FP8_E4M3"), ("MXFP8", "FP8_E4M3"),
                                  ("NVFP4", "MXFP8")])
@pytest.mark.parametrize("shape", [(512, 4096), (4, 128, 768), (600, 32), (7, 48)])
def test_fused_w_hat_equals_single_format(fmts, shape):
    """W_hat of several formats from one read (one slice per format) equals each format's own W_hat
    and the oracle, including the near-tie rows that the fix-ups rewrite; odd shapes take the
    per-format path."""
    from prismaquant_b200 import _lib
    bits = _tie_rows(600, seed=11)[:, :32] if shape == (600, 32) else \
        O.synthetic_weight_bits(shape, seed=sum(shape), outlier_frac=0.002)
    w = to_cuda_bf16(bits)
    if "MXFP8" in fmts and shape[-1] % 32 and shape[-1] > 32:   # MXFP8 cannot group the row
        with pytest.raises(ValueError):
            _lib.cost_qdq_fused(w, fmts)
        return
    got = _lib.cost_qdq_fused(w, fmts)
    for f in fmts:
        try:
            want = O.f32_to_bf16_bits(O.cost_qdq_f32(bits, f))
        except ValueError:   # MXFP8 cannot group 48 columns
            continue
        np.testing.assert_array_equal(bits_of(got[f]), want, err_msg=f)
        np.testing.assert_array_equal(bits_of(got[f]), bits_of(_lib.cost_qdq(w, f)), err_msg=f)


def _stacked_case(name):
    if name == "ties_2x600x32":
        return _tie_rows(1200, seed=13).reshape(2, 600, 32)
    if name == "exact_units_3x64x64":   # tiny groups, an FP8 row at 2^64, ordinary rows
        b = O.synthetic_weight_bits((3, 64, 64), seed=14)
        b[0, :8] = (b[0, :8] & np.uint16(0x807F)) | np.uint16(0x0100)
        b[1, 5, 9] = np.uint16(0x5F80)
        return b
    shape = {"dense_3x512x4096": (3, 512, 4096), "rows_of_96_4x128x96": (4, 128, 96),
             "narrow_2x10x8": (2, 10, 8), "odd_1x7x48": (1, 7, 48)}[name]
    return O.synthetic_weight_bits(shape, seed=sum(shape), outlier_frac=0.002)


@pytest.mark.parametrize("case", ["dense_3x512x4096", "ties_2x600x32", "exact_units_3x64x64", "rows_of_96_4x128x96",
                                  "narrow_2x10x8", "odd_1x7x48"])
@pytest.mark.parametrize("fmts", [("NVFP4", "MXFP8", "FP8_E4M3"), ("NVFP4", "FP8_E4M3"), ("MXFP8",)])
def test_fused_w_hat_with_sums(case, fmts):
    """pq_cost_qdq_fused_sse: the W_hat slices of a stacked weight equal each format's own W_hat bit
    for bit, and each W[b]'s sums equal pq_sweep_sse of W[b] (same arithmetic; only the fp64
    atomics may add in another order) and the oracle (1e-5); rows the one-read kernel does not
    take go through the per-format path; MXFP8 on rows it cannot group raises."""
    from prismaquant_b200 import _lib
    bits = _stacked_case(case)
    w = to_cuda_bf16(bits)
    batch, cols = bits.shape[0], bits.shape[-1]
    if "MXFP8" in fmts and cols > 32 and cols % 32:
        with pytest.raises(ValueError):
            _lib.cost_qdq_fused_sse(w, fmts)
        return
    hats, sse = _lib.cost_qdq_fused_sse(w, fmts)
    mask = sum(1 << _lib.FMT_IDS[f] for f in fmts)
    ref = _lib.sweep_sse([w[b] for b in range(batch)], [mask] * batch).cpu().numpy()
    got = sse.cpu().numpy()
    for f in fmts:
        np.testing.assert_array_equal(bits_of(hats[f]), bits_of(_lib.cost_qdq(w, f)), err_msg=f"{case} {f}")
        col = _lib.FMT_IDS[f]
        for b in range(batch):
            assert got[b, col] == pytest.approx(ref[b, col], rel=1e-12, abs=1e-30), (case, f, b)
            rec = O.cost_qdq_f32(bits[b], f)
            err = O.bf16_round((O.bf16_bits_to_f32(bits[b]) - rec).astype(np.float32))
            with np.errstate(over="ignore"):
                want = float((err * err).astype(np.float32).astype(np.float64).sum())
            assert got[b, col] == pytest.approx(want, rel=1e-5, abs=1e-30), (case, f, b)
    for f in _lib.FUSED_FMTS:
        if f not in fmts:
            assert (got[:, _lib.FMT_IDS[f]] == 0).all(), f


@pytest.mark.parametrize("shape", [(3, 512, 4096), (4, 128, 96), (2, 10, 8)])
def test_fused_w_hat_with_sums_from_separate_weights(shape):
    """pq_cost_qdq_fused_sse_list: weights in separate allocations give the stacked entry point's
    W_hat slices bit for bit, their stacked copy equals torch.stack, and the sums agree (only the
    fp64 atomics may add in another order); rows the one-read kernel does not take are stacked
    first and go through the stacked entry point."""
    from prismaquant_b200 import _lib
    bits = O.synthetic_weight_bits(shape, seed=sum(shape) + 1, outlier_frac=0.002)
    ws = [to_cuda_bf16(bits[b].copy()) for b in range(shape[0])]   # one allocation each
    fmts = _lib.FUSED_FMTS
    hats, W, sse = _lib.cost_qdq_fused_sse_list(ws, fmts)
    stacked = torch.stack(ws)
    assert torch.equal(W, stacked)
    want_hats, want_sse = _lib.cost_qdq_fused_sse(stacked, fmts)
    for f in fmts:
        np.testing.assert_array_equal(bits_of(hats[f]), bits_of(want_hats[f]), err_msg=f"{shape} {f}")
    np.testing.assert_allclose(sse.cpu().numpy(), want_sse.cpu().numpy(), rtol=1e-12, atol=1e-30)
