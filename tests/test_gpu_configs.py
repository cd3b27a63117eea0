"""Full-shape parity for the benchmark's model configurations against the reference's own run
(tests/golden/config_digests.json, made by tests/golden/make_golden.py `configs`):

  * one Llama-8B decoder layer (q/k/v/o [4096|1024|1024|4096, 4096], gate/up [14336, 4096],
    down [4096, 14336]) plus lm_head rows 0-4095: the fused sweep + NVFP4 export in one pass
    (joint globals for q/k/v and gate/up), MSE_W of every cost format at 1e-5, the W_hat, NVFP4,
    MXFP8 and FP8 bytes bit-exact (SHA-256);
  * one Qwen3-30B-A3B-like MoE layer (gate_up_proj [128, 1536, 2048], down_proj [128, 2048,
    768]): _measure_packed_experts' cost table at 1e-5, the batched W_hat and the per-expert
    NVFP4 export bit-exact.

Weights are N(0, 0.02^2) from the oracle's seeded generator, one seed per tensor name."""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import pq_oracle as O
from prismaquant_b200 import export_native_compressed as enc
from prismaquant_b200 import format_registry as fr
from prismaquant_b200 import measure_quant_cost as mqc
from tests._helpers import assert_rel, bits_of, to_cuda_bf16, u8_of

pytestmark = pytest.mark.gpu

FIX = Path(__file__).resolve().parent / "golden" / "config_digests.json"
FMTS = ("NVFP4", "MXFP8", "FP8_E4M3", "BF16")


def name_seed(name: str) -> int:
    return int.from_bytes(hashlib.sha256(name.encode()).digest()[:6], "little")


@pytest.fixture(scope="module")
def fix():
    return json.loads(FIX.read_text())


def _f32(t):
    return t.detach().contiguous().cpu().float().numpy()


def test_llama8b_layer_sweep_and_export(fix):
    dg = fix["llama8b_layer"]
    ws = {}
    for name, d in dg.items():
        bits = O.synthetic_weight_bits(tuple(d["shape"]), seed=name_seed(name))
        assert O.digest(bits) == d["input"], "synthetic generator differs on this host"
        ws[name] = to_cuda_bf16(bits)
    specs = [fr.get_format(f) for f in FMTS]
    costs, outs = enc.sweep_and_export(ws, specs)      # one read: every cost format + NVFP4 codes
    for name, d in dg.items():
        for f in FMTS:
            assert_rel(costs[name][f], d[f"mse/{f}"], 1e-5, f"{name} {f}")
        p, s, g = outs[name]
        assert O.digest(u8_of(p), u8_of(s), _f32(g)) == d["nvfp4"], name
        w = ws[name]
        for f in FMTS:
            assert O.digest(bits_of(fr.get_format(f).quantize_dequantize(w))) == d[f"qdq/{f}"], (name, f)
        q, sc = enc.quantize_dequantize_mxfp8(w)
        assert O.digest(u8_of(q), u8_of(sc)) == d["mxfp8"], name
        q, sc = enc.quantize_dequantize_fp8_dynamic(w)
        assert O.digest(u8_of(q), _f32(sc)) == d["fp8dyn"], name
        del q, sc
    torch.cuda.empty_cache()


def test_moe30b_layer_packed_experts(fix):
    dg = fix["moe30b_layer"]

    class PackedExperts(torch.nn.Module):   # class name holds "expert"; owns the packed parameters
        def __init__(self, params):
            super().__init__()
            for n, t in params.items():
                self.register_parameter(n, torch.nn.Parameter(t, requires_grad=False))

    params = {}
    for name, d in dg.items():
        bits = O.synthetic_weight_bits(tuple(d["shape"]), seed=name_seed(name))
        params[name.rsplit(".", 1)[1]] = to_cuda_bf16(bits)
    model = torch.nn.Module()
    model.add_module("experts", PackedExperts(params))
    for name, d in dg.items():
        assert O.digest(bits_of(getattr(model.experts, name.rsplit(".", 1)[1]))) == d["input"]
    specs = [fr.get_format(f) for f in FMTS]
    accum = {}
    mqc._measure_packed_experts(model, {"experts.gate_up_proj", "experts.down_proj"}, specs, "cuda",
                                torch.bfloat16, accum)
    table = mqc._finalize_results(accum)
    for name, d in dg.items():
        pn = name.rsplit(".", 1)[1]
        got, want = table["experts." + pn], d["table"]
        assert set(got) == set(want)
        for f in FMTS:
            for k in ("weight_mse", "output_mse", "rel_output_mse"):
                assert_rel(got[f][k], want[f][k], 1e-5, f"{pn} {f} {k}")
        W = getattr(model.experts, pn)
        for f in FMTS:
            assert O.digest(bits_of(mqc._batched_quantize(fr.get_format(f), W))) == d[f"qdq/{f}"], (pn, f)
        p, s, g = enc.quantize_dequantize_nvfp4_packed(W)
        assert O.digest(u8_of(p), u8_of(s), _f32(g)) == d["nvfp4_packed"], pn
        del p, s, g
        torch.cuda.empty_cache()
