"""The toy model behind tests/golden/cost_pipeline.json: four bf16 Linears of three shapes and one
packed-experts module, with seeded activations and per-weight / per-channel Fisher diagonals.
Shared by make_golden.py (which runs the reference on it) and the GPU tests (which run the B200
path on the same inputs); nothing here imports the reference."""
from __future__ import annotations

import numpy as np
import torch

from oracle import pq_oracle as O

PIPE_LINEARS = {"model.layers.0.self_attn.q_proj": (64, 128), "model.layers.0.self_attn.k_proj": (64, 128),
                "model.layers.0.self_attn.o_proj": (128, 64), "model.layers.0.mlp.down_proj": (48, 96)}
PIPE_EXPERTS = ("model.layers.0.mlp.experts", (4, 32, 64))   # gate_up_proj [E, M, N]


def to_t(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def pipeline_inputs():
    """Seeded bf16 weights, activations [rows, in] and H (per weight for Linears, [E, M] for the
    packed experts)."""
    ws = {n: O.synthetic_weight_bits(s, seed=100 + i, outlier_frac=0.01) for i, (n, s) in enumerate(PIPE_LINEARS.items())}
    acts = {n: O.synthetic_weight_bits((24 + 8 * i, s[1]), seed=200 + i, std=1.0)
            for i, (n, s) in enumerate(PIPE_LINEARS.items())}
    rng = np.random.default_rng(300)
    hs = {n: (rng.random(s, dtype=np.float32) * np.float32(5.0)) for n, s in PIPE_LINEARS.items()}
    e_name, e_shape = PIPE_EXPERTS
    ws[e_name + ".gate_up_proj"] = O.synthetic_weight_bits(e_shape, seed=400, std=0.05)
    hs[e_name + ".gate_up_proj"] = rng.random(e_shape[:2], dtype=np.float32) * np.float32(3.0)
    return ws, acts, hs


class Index:
    """The activation / H index interface the cost functions use: `name in idx`, `idx.load(name)`."""

    def __init__(self, d):
        self.d = d

    def __contains__(self, n):
        return n in self.d

    def load(self, n):
        return self.d[n]


class PackedExperts(torch.nn.Module):   # class name holds "expert" and it owns a packed 3-D parameter
    def __init__(self, w):
        super().__init__()
        self.gate_up_proj = torch.nn.Parameter(w)


def build_pipeline_model(ws, device="cpu"):
    root = torch.nn.Module()
    for name, shape in PIPE_LINEARS.items():
        parent = root
        parts = name.split(".")
        for p in parts[:-1]:
            if not hasattr(parent, p):
                parent.add_module(p, torch.nn.Module())
            parent = getattr(parent, p)
        lin = torch.nn.Linear(shape[1], shape[0], bias=False, dtype=torch.bfloat16, device=device)
        with torch.no_grad():
            lin.weight.copy_(to_t(ws[name]).to(device))
        parent.add_module(parts[-1], lin)
    e_name, _ = PIPE_EXPERTS
    parent = root
    for p in e_name.split(".")[:-1]:
        parent = getattr(parent, p)
    parent.add_module(e_name.split(".")[-1], PackedExperts(to_t(ws[e_name + ".gate_up_proj"]).to(device)))
    return root


def run_cost_pipeline(mqc, fr, device):
    """The three cost entry points with H, all registry formats; mqc / fr are either the
    reference's modules or this package's."""
    ws, acts, hs = pipeline_inputs()
    model = build_pipeline_model(ws, device=device)
    act = Index({n: to_t(a) for n, a in acts.items()})
    hd = Index({n: torch.from_numpy(h) for n, h in hs.items()})
    specs = [fr.get_format(n) for n in fr.REGISTRY]
    targets = set(PIPE_LINEARS)
    out = {"batched": mqc.measure_batched_gpu(model, act, targets, specs, device, torch.bfloat16, chunk_size=2,
                                              h_detail=hd),
           "unbatched": mqc.measure_unbatched(model, act, targets, specs, device, torch.bfloat16, h_detail=hd)}
    accum = {}
    mqc._measure_packed_experts(model, {PIPE_EXPERTS[0] + ".gate_up_proj"}, specs, device, torch.bfloat16, accum,
                                h_detail=hd)
    out["packed"] = mqc._finalize_results(accum)
    return out
