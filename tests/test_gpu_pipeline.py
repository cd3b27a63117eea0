"""The cost-table entry points end to end on the GPU, against the reference's own tables
(tests/golden/cost_pipeline.json, made by running the reference's measure_batched_gpu,
measure_unbatched and _measure_packed_experts on the same toy model): every registry format,
with per-weight and per-channel Fisher diagonals (predicted_dloss) and the error entries.

weight_mse and predicted_dloss come from the bit-exact quantizers and must match within 1e-5.
output_mse compares bf16 bmm results computed on different devices (CPU for the fixture, cuBLAS
here), whose bf16 roundings differ, so it is held to the same order of magnitude only."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import pq_oracle as O
from prismaquant_b200 import format_registry as fr
from prismaquant_b200 import measure_quant_cost as mqc
from tests._helpers import to_cuda_bf16
from tests.golden.pipeline_model import run_cost_pipeline

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "cost_pipeline.json"


@pytest.fixture(scope="module")
def pipeline():
    return run_cost_pipeline(mqc, fr, "cuda"), json.loads(GOLDEN.read_text())


@pytest.mark.parametrize("entry", ["batched", "unbatched", "packed"])
def test_cost_tables_match_reference(pipeline, entry):
    got, want = pipeline[0][entry], pipeline[1][entry]
    assert set(got) == set(want)
    for name in want:
        assert set(got[name]) == set(want[name]), name
        for fmt, w in want[name].items():
            g = got[name][fmt]
            if "error" in w:
                assert "error" in g, (entry, name, fmt, g)
                continue
            assert "error" not in g, (entry, name, fmt, g)
            for k in ("weight_mse", "predicted_dloss"):
                assert g[k] == pytest.approx(w[k], rel=1e-5, abs=1e-30), (entry, name, fmt, k)
            for k in ("output_mse", "rel_output_mse"):
                if w[k] == 0.0:
                    assert g[k] == 0.0, (entry, name, fmt, k)
                else:
                    assert 0.2 < g[k] / w[k] < 5.0, (entry, name, fmt, k, g[k], w[k])


def _oracle_weighted(bits, fmt, h, per_row, batched):
    rec = O.batched_qdq_f32(bits, fmt) if batched else O.cost_qdq_f32(bits, fmt)
    w = O.bf16_bits_to_f32(bits)
    err = O.bf16_round((w - rec).astype(np.float32)).reshape(-1, bits.shape[-1])
    sq = (err * err).astype(np.float32).astype(np.float64)
    hh = np.asarray(h, dtype=np.float64)
    return float((sq.sum(axis=1) * hh.reshape(-1)).sum() if per_row else (sq * hh.reshape(sq.shape)).sum())


@pytest.mark.parametrize("fmt", ["NVFP4", "MXFP8", "FP8_E4M3", "MXFP4", "MXFP6_E2M3", "FP8_E5M2", "NVFP3", "INT3",
                                 "INT4_W4A16_g128", "FP8_E4M3_G128"])
@pytest.mark.parametrize("per_row", [False, True])
def test_weighted_sse_matches_oracle(fmt, per_row):
    """pq_weighted_sse: sum(h * err^2) with h per element or per row, against the oracle (1e-5)."""
    from prismaquant_b200 import _lib
    bits = O.synthetic_weight_bits((96, 256), seed=17, outlier_frac=0.01)
    rng = np.random.default_rng(3)
    h = rng.random(96 if per_row else (96, 256), dtype=np.float32) * np.float32(4.0)
    out = torch.zeros((), dtype=torch.float64, device="cuda")
    _lib.weighted_sse(to_cuda_bf16(bits), fmt, torch.from_numpy(h).cuda(), out, per_row=per_row)
    if fmt == "FP8_E4M3_G128":
        rec = O.codebook_qdq_f32(bits, "fp8_e4m3", 128, False)
        err = O.bf16_round((O.bf16_bits_to_f32(bits) - rec).astype(np.float32))
        sq = (err * err).astype(np.float32).astype(np.float64)
        want = float((sq.sum(axis=1) * h).sum() if per_row else (sq * h).sum())
    else:
        want = _oracle_weighted(bits, fmt, h, per_row, batched=False)
    assert out.item() == pytest.approx(want, rel=1e-5)


def _fused_cases():
    from tests.test_gpu_cost import _tie_rows
    ties = _tie_rows(800, seed=21)                                            # fix-ups of every format
    tiny = (O.synthetic_weight_bits((8, 32), seed=5) & np.uint16(0x807F)) | np.uint16(0x0100)   # amax < 1e-8
    huge = O.synthetic_weight_bits((4, 32), seed=6)
    huge[:, 3] = np.uint16(0x5F80)                                           # 2^64: exact units and FP8 rows
    return {
        "ties_tiny_huge_836x32": np.concatenate([ties, tiny, huge]).astype(np.uint16),
        "dense_300x4096": O.synthetic_weight_bits((300, 4096), seed=8, outlier_frac=0.002),
        "rows_of_96_2x700x96": O.synthetic_weight_bits((2, 700, 96), seed=9),   # several rows per warp
        "odd_cols_40x48": O.synthetic_weight_bits((40, 48), seed=10),          # no MXFP8 grouping
        "narrow_12x8": O.synthetic_weight_bits((12, 8), seed=11),              # rows under one group
    }


@pytest.mark.parametrize("case", list(_fused_cases()))
@pytest.mark.parametrize("fmts", [("NVFP4", "MXFP8", "FP8_E4M3"), ("NVFP4", "FP8_E4M3"), ("MXFP8",), ("FP8_E4M3",)])
@pytest.mark.parametrize("per_row", [False, True])
def test_weighted_sse_fused_matches_oracle(case, fmts, per_row):
    """pq_weighted_sse_fused: every format's sum(h * err^2) from one read of W and h, against the
    oracle (1e-5) and against pq_weighted_sse of the format alone (fp32 partial regrouping only);
    shapes the one-read kernel does not take go format by format; MXFP8 on rows it cannot group
    raises."""
    from prismaquant_b200 import _lib
    bits = _fused_cases()[case]
    rows, cols = bits.size // bits.shape[-1], bits.shape[-1]
    rng = np.random.default_rng(rows + cols)
    h = rng.random(rows if per_row else (rows, cols), dtype=np.float32) * np.float32(4.0)
    w, hc = to_cuda_bf16(bits), torch.from_numpy(h).cuda()
    if "MXFP8" in fmts and cols > 32 and cols % 32:
        with pytest.raises(ValueError):
            _lib.weighted_sse_fused(w, fmts, hc, per_row=per_row)
        return
    got = _lib.weighted_sse_fused(w, fmts, hc, per_row=per_row).cpu().numpy()
    for f in _lib.FUSED_FMTS:
        v = got[_lib.FMT_IDS[f]]
        if f not in fmts:
            assert v == 0.0, f
            continue
        want = _oracle_weighted(bits.reshape(rows, cols), f, h, per_row, batched=False)
        assert v == pytest.approx(want, rel=1e-5, abs=1e-30), (case, f)
        one = torch.zeros((), dtype=torch.float64, device="cuda")
        _lib.weighted_sse(w, f, hc, one, per_row=per_row)
        assert v == pytest.approx(one.item(), rel=1e-6, abs=1e-30), (case, f)


def test_weighted_sse_fused_rejects_other_formats():
    from prismaquant_b200 import _lib
    w = to_cuda_bf16(O.synthetic_weight_bits((4, 64), seed=1))
    h = torch.ones(4, 64, device="cuda")
    for fmts in [("MXFP4",), ("NVFP4", "BF16"), ()]:
        with pytest.raises(ValueError):
            _lib.weighted_sse_fused(w, fmts, h)
    with pytest.raises(ValueError):
        _lib.weighted_sse_fused(w, ("NVFP4",), torch.ones(5, device="cuda"), per_row=True)


@pytest.mark.parametrize("shape", [(5, 300, 256), (3, 64, 96), (2, 10, 8)])
@pytest.mark.parametrize("per_row", [False, True])
def test_weighted_sse_fused_batch_matches_single(shape, per_row):
    """pq_weighted_sse_fused_batch: one launch over a stacked weight gives each w[b] the sums of
    pq_weighted_sse_fused(w[b], h[b]) (the same arithmetic: only the fp64 atomics may add in another
    order); rows the one-read kernel does not take go tensor by tensor."""
    from prismaquant_b200 import _lib
    bits = O.synthetic_weight_bits(shape, seed=sum(shape), outlier_frac=0.002)
    rng = np.random.default_rng(7)
    b, rows, cols = shape
    h = rng.random((b, rows) if per_row else shape, dtype=np.float32) * np.float32(4.0)
    w, hc = to_cuda_bf16(bits), torch.from_numpy(h).cuda()
    fmts = ("NVFP4", "FP8_E4M3") if cols % 32 and cols > 32 else _lib.FUSED_FMTS
    got = _lib.weighted_sse_fused_batch(w, fmts, hc, per_row=per_row).cpu().numpy()
    for i in range(b):
        one = _lib.weighted_sse_fused(w[i], fmts, hc[i], per_row=per_row).cpu().numpy()
        np.testing.assert_allclose(got[i], one, rtol=1e-12, atol=1e-30, err_msg=f"{shape} {i}")


def test_batched_gpu_takes_list_entry_with_plain_cuda_device(monkeypatch):
    """measure_batched_gpu(..., "cuda", bf16): callers name the device "cuda" (no index); the
    weights live on cuda:<current>, and the chunk must still take the one-read list entry point
    (pq_cost_qdq_fused_sse_list) instead of stacking in torch first."""
    from prismaquant_b200 import _lib
    from tests.golden.pipeline_model import PIPE_LINEARS, Index, build_pipeline_model, pipeline_inputs, to_t
    calls = []
    orig = _lib.cost_qdq_fused_sse_list

    def counted(*a, **kw):
        calls.append(1)
        return orig(*a, **kw)

    monkeypatch.setattr(_lib, "cost_qdq_fused_sse_list", counted)
    ws, acts, _ = pipeline_inputs()
    model = build_pipeline_model(ws, device="cuda")
    act = Index({n: to_t(a) for n, a in acts.items()})
    specs = [fr.get_format(n) for n in ("NVFP4", "MXFP8", "FP8_E4M3", "BF16")]
    got = mqc.measure_batched_gpu(model, act, set(PIPE_LINEARS), specs, "cuda", torch.bfloat16, chunk_size=2)
    assert calls, "the list entry point was not reached with device='cuda'"
    ref = mqc.measure_batched_gpu(model, act, set(PIPE_LINEARS), specs, torch.device("cuda", 0), torch.bfloat16,
                                  chunk_size=2)
    for name in got:
        for fmt in got[name]:
            assert got[name][fmt]["weight_mse"] == ref[name][fmt]["weight_mse"]
