"""The oracle is pinned against the reference's own outputs (golden fixtures
produced by tests/golden/make_golden.py) before any kernel is compared to it."""
import numpy as np
import pytest

from oracle import pq_oracle as O

CASES = ["rand_64x128", "rand_33x256", "ties_4x32", "zeros_3x64", "wide_range_8x96",
         "row1_1x4096", "cols16_5x16", "cols48_7x48", "cols8_4x8", "packed_4x32x64",
         "packed_3x16x96", "bf16mix_128x32"]
COST_FMTS = ["NVFP4", "MXFP8", "FP8_E4M3", "BF16"]
EXT_FMTS = ["MXFP4", "MXFP6_E3M2", "MXFP6_E2M3", "MXFP8_E5M2", "FP8_E5M2", "NVFP3", "INT3", "INT2",
            "INT8_W8A16", "INT4_W4A16_g128", "FP8_SOURCE"]


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("fmt", COST_FMTS + EXT_FMTS)
def test_cost_path_matches_reference(golden, case, fmt):
    bits = golden[f"{case}/input"]
    key = f"{case}/cost/{fmt}"
    # the fixtures ran quantize_dequantize on 2-D inputs and _batched_quantize on packed 3-D ones
    qdq = O.batched_qdq_f32 if bits.ndim == 3 else O.cost_qdq_f32
    if f"{key}/error" in golden:
        with pytest.raises(ValueError):
            qdq(bits, fmt)
        return
    rec = qdq(bits, fmt)
    np.testing.assert_array_equal(O.f32_to_bf16_bits(rec), golden[f"{key}/qdq"])
    ref_mse = float(golden[f"{key}/mse"][0])
    w = O.bf16_bits_to_f32(bits)
    err = O.bf16_round((w - rec).astype(np.float32))
    with np.errstate(over="ignore"):
        sq = (err * err).astype(np.float32).astype(np.float64)
    mse = float(sq.sum()) / max(bits.size, 1)
    if bits.ndim == 2:
        assert mse == pytest.approx(O.cost_mse(bits, fmt), rel=1e-12, abs=1e-300)
    assert mse == pytest.approx(ref_mse, rel=1e-5, abs=1e-30)


@pytest.mark.parametrize("case", [c for c in CASES if not c.startswith("packed")])
def test_export_2d_matches_reference(golden, case):
    w = O.bf16_bits_to_f32(golden[f"{case}/input"])
    if f"{case}/nvfp4/packed" in golden:
        p, s, g = O.nvfp4_pack(w)
        np.testing.assert_array_equal(p, golden[f"{case}/nvfp4/packed"])
        np.testing.assert_array_equal(s, golden[f"{case}/nvfp4/scale"])
        np.testing.assert_array_equal(g, golden[f"{case}/nvfp4/global"])
        assert O.nvfp4_global_real(w) == golden[f"{case}/nvfp4/global_real"][0]
        ov = golden[f"{case}/nvfp4_ovr/override"][0]
        p, s, g = O.nvfp4_pack(w, global_real_override=ov)
        np.testing.assert_array_equal(p, golden[f"{case}/nvfp4_ovr/packed"])
        np.testing.assert_array_equal(s, golden[f"{case}/nvfp4_ovr/scale"])
        np.testing.assert_array_equal(g, golden[f"{case}/nvfp4_ovr/global"])
    if f"{case}/mxfp8/weight" in golden:
        q, sc = O.mxfp8_pack(w)
        np.testing.assert_array_equal(q, golden[f"{case}/mxfp8/weight"])
        np.testing.assert_array_equal(sc, golden[f"{case}/mxfp8/scale"])
    q, sc = O.fp8_dynamic_pack(w)
    np.testing.assert_array_equal(q, golden[f"{case}/fp8dyn/weight"])
    np.testing.assert_array_equal(sc, golden[f"{case}/fp8dyn/scale"])


@pytest.mark.parametrize("case", ["packed_4x32x64", "packed_3x16x96"])
def test_export_packed_matches_reference(golden, case):
    w = O.bf16_bits_to_f32(golden[f"{case}/input"])
    p, s, g = O.nvfp4_pack_packed(w)
    np.testing.assert_array_equal(p, golden[f"{case}/nvfp4p/packed"])
    np.testing.assert_array_equal(s, golden[f"{case}/nvfp4p/scale"])
    np.testing.assert_array_equal(g, golden[f"{case}/nvfp4p/global"])
    q, sc = O.mxfp8_pack(w)
    np.testing.assert_array_equal(q, golden[f"{case}/mxfp8p/weight"])
    np.testing.assert_array_equal(sc, golden[f"{case}/mxfp8p/scale"])
    np.testing.assert_array_equal(q, golden[f"{case}/grouped_mxfp8/weight"])
    q, sc = O.fp8_dynamic_pack(w)
    np.testing.assert_array_equal(q, golden[f"{case}/fp8dynp/weight"])
    np.testing.assert_array_equal(sc, golden[f"{case}/fp8dynp/scale"])


@pytest.mark.parametrize("case", ["packed_4x32x64", "packed_3x16x96"])
def test_gradnorm_capture_matches_reference(golden, case):
    total, per_row = O.sumsq_rows(golden[f"{case}/input"])
    assert total == pytest.approx(float(golden[f"{case}/gradnorm/scalar"][0]), rel=1e-6)
    np.testing.assert_allclose(per_row, golden[f"{case}/gradnorm/channel"], rtol=1e-6)


@pytest.mark.parametrize("lin", ["0", "1"])
def test_per_token_estimator_bridges_reference_at_one_token(golden, lin):
    x = golden[f"bridge/{lin}/x"].astype(np.float64)
    g = golden[f"bridge/{lin}/gy"].astype(np.float64)
    per_token = float(((x * x).sum(-1) * (g * g).sum(-1)).sum())
    assert per_token == pytest.approx(float(golden[f"bridge/{lin}/h_trace_raw"][0]), rel=1e-5)
    assert int(golden[f"bridge/{lin}/n_tokens_seen"][0]) == x.shape[0]


def test_known_answers(golden):
    # reference tests: _round_to_codebook([0, .5, 1, 6, -6]) == [0, 1, 2, 7, 15]; 0x21 nibble order
    assert O.round_to_codebook(np.array([0.0, 0.5, 1.0, 6.0, -6.0], np.float32)).tolist() == [0, 1, 2, 7, 15]
    assert O.pack_fp4_indices(np.array([[1, 2, 3, 4]])).tolist() == [[0x21, 0x43]]
    np.testing.assert_array_equal(O.round_to_codebook(golden["ka/round_to_codebook/in"]),
                                  golden["ka/round_to_codebook/out"])
    np.testing.assert_array_equal(O.pack_fp4_indices(np.array([[1, 2, 3, 4]])), golden["ka/pack/out"])
    c = golden["ka/cost_e2m1/in"]
    got = O.cost_qdq_f32(O.f32_to_bf16_bits(c), "NVFP4")
    # (the reference call ran in fp32; all these values are bf16-exact)
    np.testing.assert_array_equal(got[:, :12], golden["ka/cost_e2m1/out"][:, :12])


def test_e4m3_conversion_matches_torch():
    import torch
    allbf = O.bf16_bits_to_f32(np.arange(1 << 16, dtype=np.uint32).astype(np.uint16))
    rng = np.random.default_rng(0)
    rnd = (rng.standard_normal(1 << 20) * np.exp2(rng.integers(-14, 9, 1 << 20))).astype(np.float32)
    grid = np.array([O.e4m3fn_bits_to_f32(np.array([b], np.uint8))[0] for b in range(0x7F)], np.float32)
    mids = ((grid[1:].astype(np.float64) + grid[:-1]) / 2).astype(np.float32)
    near = np.concatenate([np.nextafter(mids, np.inf), mids, np.nextafter(mids, -np.inf)])
    x = np.concatenate([allbf, rnd, near, -near])
    x = x[np.isfinite(x) & (np.abs(x) <= 448)]
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(O.f32_to_e4m3fn_bits(x), ref)


def test_e8m0_thresholds_match_torch_log2():
    import torch
    t = O.e8m0()
    ks = np.arange(-126, 128)
    for table, op in ((t.ceil_last, torch.ceil), (t.round_first, torch.round)):
        for k in ks:
            m0 = table[int(k)]
            m = np.clip(np.arange(m0 - 40, m0 + 41), 0, (1 << 23) - 1).astype(np.int64)
            x = (((k + 127) << 23) | m).astype(np.uint32).view(np.float32)
            r = op(torch.log2(torch.from_numpy(x.copy()))).numpy().astype(np.int64)
            if op is torch.ceil:
                np.testing.assert_array_equal(t.ceil_log2(x), np.clip(r, -127, 127))
            else:
                np.testing.assert_array_equal(t.round_log2(x), np.clip(r, -127, 127))


def test_full_linear_digest_oracle(full_digests):
    """The oracle reproduces the reference on the full 4096x4096 single-Linear sweep."""
    d = full_digests["linear4096"]
    w = O.synthetic_weight_bits((4096, 4096), seed=0, outlier_frac=0.001)
    assert O.digest(w) == d["input"], "synthetic generator differs on this host"
    for fmt in ("NVFP4", "MXFP8", "FP8_E4M3", "BF16"):
        assert O.digest(O.f32_to_bf16_bits(O.cost_qdq_f32(w, fmt))) == d[f"qdq/{fmt}"], fmt
        assert O.cost_mse(w, fmt) == pytest.approx(d[f"mse/{fmt}"], rel=1e-5, abs=1e-30)
    wf = O.bf16_bits_to_f32(w)
    assert O.digest(*O.nvfp4_pack(wf)) == d["nvfp4"]
    assert O.digest(*O.mxfp8_pack(wf)) == d["mxfp8"]
    assert O.digest(*O.fp8_dynamic_pack(wf)) == d["fp8dyn"]


def test_extended_codebooks_match_reference_definitions():
    """Codebook sizes and extremes as the reference defines them (format_registry.py:237-300):
    FP6 and FP3 have no subnormals, and E5M2 keeps exponent 31 as finite values."""
    sizes = {k: (v.size, float(v.max()), float(v[v > 0].min())) for k, v in O.CODEBOOKS.items()}
    assert sizes["fp6_e3m2"] == (65, 28.0, 0.125)
    assert sizes["fp6_e2m3"] == (65, 7.5, 0.5)
    assert sizes["fp3_e2m0"] == (9, 2.0, 0.25)
    assert sizes["fp8_e5m2"] == (255, 114688.0, 2.0 ** -16)
    assert O.FORMAT_ALIASES == {"NVINT2": "INT2", "NVINT3": "INT3"}
