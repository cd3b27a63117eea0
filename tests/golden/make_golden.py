"""Generate the golden fixtures under tests/golden/ by running the REFERENCE
prismaquant implementation (imported read-only from a local checkout) on
seeded inputs.

    PYTHONPATH=oracle/_shim:<reference checkout> python tests/golden/make_golden.py

Outputs:
  small_cases.npz     inputs (bf16 bit patterns) and the reference's outputs
                      for every hot-path function on small edge-case tensors
  cost_pipeline.json  the reference's cost tables (measure_batched_gpu, measure_unbatched,
                      _measure_packed_experts, with per-weight / per-channel H) for a
                      toy model rebuilt from seeds by the GPU tests
  full_digests.json   SHA-256 digests of the reference's outputs on the
                      single-Linear sweep (4096x4096 with 0.1 % x20 outliers,
                      seed 0) and on the fused-sibling q/k/v + gate/up group
                      (seeds 1..5), plus their MSE_W values
  config_digests.json (`configs`) the same for one full-shape Llama-8B decoder
                      layer + lm_head rows 0-4095, and one Qwen3-30B-A3B-like
                      MoE layer through _measure_packed_experts, the batched
                      W_hat and the packed NVFP4 export
  fisher_bridge_bf16.npz (`fisher_bridge`) FisherAccumulator at one token per
                      backward on bf16-valued inputs and gradients
  fisher_detail.npz   (`fisher_detail`) FisherAccumulator with h_detail_dir
  qconfig_cases.json  (`qconfig`) build_quantization_config / write_config_with_quantization
                      on recipe assignments (dense, packed and per-expert MoE, MTP, fused
                      siblings), with the profile's answers recorded as tables

Only this script touches the reference; the committed fixtures travel, the
reference does not.
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle import pq_oracle as O  # noqa: E402

from prismaquant import format_registry as fr  # noqa: E402
from prismaquant import measure_quant_cost as mqc  # noqa: E402
from prismaquant import export_native_compressed as enc  # noqa: E402
from prismaquant import sensitivity_probe as sp  # noqa: E402

torch.set_num_threads(os.cpu_count() or 1)

COST_FMTS = ["NVFP4", "MXFP8", "FP8_E4M3", "BF16"]
# the rest of the registry (quantize_dequantize only; served by the exact codebook kernel)
EXT_FMTS = ["MXFP4", "MXFP6_E3M2", "MXFP6_E2M3", "MXFP8_E5M2", "FP8_E5M2", "NVFP3", "INT3", "INT2",
            "INT8_W8A16", "INT4_W4A16_g128", "FP8_SOURCE"]


def to_t(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def bits_of(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def u8_of(t):
    return t.contiguous().view(torch.uint8).numpy().copy()


def bf16_bits_from_f32(vals):
    return O.f32_to_bf16_bits(np.asarray(vals, dtype=np.float32))


def tie_case():
    """Rows whose scaled values land exactly on codebook midpoints.

    Row r: first element fixes amax so that scale is an exact power of two
    for NVFP4 (amax = 6 * 2^-4 -> s = 2^-4) and for FP8-per-channel the row
    amax = 448 * 2^-8; the rest are +-midpoints in that grid.
    """
    s = 2.0 ** -4
    e2m1_mid = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0]
    rows = []
    for sign in (1.0, -1.0):
        row = [6.0 * s] + [sign * m * s for m in e2m1_mid] + [-0.0, 0.0] + [sign * 0.1 * s] * 6
        rows.append(row[:16] + row[:16])
    # e4m3 midpoints for MX / FP8 channel: grid at scale 1 (amax 448)
    mids = [448.0, 9.0, 17.0, 0.5 + 1 / 32, 2 ** -7 + 2 ** -10, 2 ** -10, 3 * 2 ** -10,
            -9.0, -17.0, -(2 ** -10), -(3 * 2 ** -10), 104.0, -104.0, 232.0, 464.0, -0.0]
    rows.append(mids + [-m for m in mids])
    rows.append([v * 2.0 ** -20 for v in mids + mids])
    return bf16_bits_from_f32(np.array(rows, dtype=np.float32))


def small_cases():
    cases = {}
    cases["rand_64x128"] = O.synthetic_weight_bits((64, 128), seed=11, outlier_frac=0.01)
    cases["rand_33x256"] = O.synthetic_weight_bits((33, 256), seed=12, std=1.0, outlier_frac=0.003)
    cases["ties_4x32"] = tie_case()
    z = np.zeros((3, 64), dtype=np.float32)
    z[1, :16] = -0.0
    z[2, 5] = 1e-30
    z[2, 40] = -3e-39        # bf16 subnormal
    cases["zeros_3x64"] = bf16_bits_from_f32(z)
    wide = np.random.default_rng(5).standard_normal((8, 96)).astype(np.float32)
    wide *= np.float32(10.0) ** np.random.default_rng(6).integers(-30, 30, (8, 1)).astype(np.float32)
    cases["wide_range_8x96"] = bf16_bits_from_f32(wide)
    cases["row1_1x4096"] = O.synthetic_weight_bits((1, 4096), seed=13)
    cases["cols16_5x16"] = O.synthetic_weight_bits((5, 16), seed=14)
    cases["cols48_7x48"] = O.synthetic_weight_bits((7, 48), seed=15)    # MXFP8 cannot group 48
    cases["cols8_4x8"] = O.synthetic_weight_bits((4, 8), seed=16)        # whole-row groups
    cases["packed_4x32x64"] = O.synthetic_weight_bits((4, 32, 64), seed=17, std=0.05)
    cases["packed_3x16x96"] = O.synthetic_weight_bits((3, 16, 96), seed=18, outlier_frac=0.01)
    # 4096 distinct finite bf16 patterns (both zeros, subnormals, the largest finite), rows of 32
    allv = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    fin = allv[np.isfinite(O.bf16_bits_to_f32(allv))]
    pick = np.random.default_rng(19).choice(fin, 4096 - 6, replace=False)
    edge = np.array([0x0000, 0x8000, 0x0001, 0x8001, 0x7F7F, 0xFF7F], dtype=np.uint16)
    cases["bf16mix_128x32"] = np.random.default_rng(20).permutation(np.concatenate([pick, edge])).reshape(128, 32)
    return cases


def run_cost(bits):
    out = {}
    W = to_t(bits)
    for fmt in COST_FMTS + EXT_FMTS:
        spec = fr.get_format(fmt)
        try:
            if W.dim() == 3:
                What = mqc._batched_quantize(spec, W)
            else:
                What = spec.quantize_dequantize(W.clone())
            err = (W - What).float()
            out[f"cost/{fmt}/qdq"] = bits_of(What)
            out[f"cost/{fmt}/mse"] = np.array([float(err.pow(2).mean().item())], dtype=np.float64)
        except Exception as e:  # the reference records {"error": str(e)}
            out[f"cost/{fmt}/error"] = np.array([str(e)])
    return out


def run_export(bits):
    out = {}
    W = to_t(bits).float()
    if W.dim() == 2:
        rows, cols = W.shape
        if cols % 16 == 0:
            wp, ws, wg = enc.quantize_dequantize_nvfp4(W)
            out["nvfp4/packed"], out["nvfp4/scale"], out["nvfp4/global"] = u8_of(wp), u8_of(ws), wg.numpy()
            gr = enc.compute_nvfp4_global_real(W)
            out["nvfp4/global_real"] = np.array([gr.item()], dtype=np.float32)
            ov = torch.tensor(float(gr.item()) * 3.0)
            wp, ws, wg = enc.quantize_dequantize_nvfp4(W, global_real_override=ov)
            out["nvfp4_ovr/override"] = np.array([ov.item()], dtype=np.float32)
            out["nvfp4_ovr/packed"], out["nvfp4_ovr/scale"], out["nvfp4_ovr/global"] = u8_of(wp), u8_of(ws), wg.numpy()
            q = enc._quantize_2d(W, "NVFP4")
            out["q2d_nvfp4/input_global_scale"] = q["input_global_scale"].numpy()
        if cols % 32 == 0:
            w8, s8 = enc.quantize_dequantize_mxfp8(W)
            out["mxfp8/weight"], out["mxfp8/scale"] = u8_of(w8), u8_of(s8)
        wf, sf = enc.quantize_dequantize_fp8_dynamic(W)
        out["fp8dyn/weight"], out["fp8dyn/scale"] = u8_of(wf), sf.numpy()
    else:
        E, M, N = W.shape
        if N % 16 == 0:
            wp, ws, wg = enc.quantize_dequantize_nvfp4_packed(W)
            out["nvfp4p/packed"], out["nvfp4p/scale"], out["nvfp4p/global"] = u8_of(wp), u8_of(ws), wg.numpy()
        if N % 32 == 0:
            w8, s8 = enc.quantize_dequantize_mxfp8_packed(W)
            out["mxfp8p/weight"], out["mxfp8p/scale"] = u8_of(w8), u8_of(s8)
            g = enc._quantize_2d_group_same_shape(W, "MXFP8")
            out["grouped_mxfp8/weight"], out["grouped_mxfp8/scale"] = u8_of(g["weight"]), u8_of(g["weight_scale"])
        wf, sf = enc.quantize_dequantize_fp8_dynamic_packed(W)
        out["fp8dynp/weight"], out["fp8dynp/scale"] = u8_of(wf), sf.numpy()
    return out


def run_fisher(bits):
    """_GradNormCapture.backward on the tensor used as a packed-expert gradient."""
    out = {}
    g = to_t(bits)
    if g.dim() == 3:
        acc, ch = {}, {}
        w = torch.zeros(g.shape, dtype=torch.bfloat16, requires_grad=True)
        y = sp._GradNormCapture.apply(w, "p", acc, ch, None)
        y.backward(g)
        out["gradnorm/scalar"] = np.array([acc["p"]], dtype=np.float64)
        out["gradnorm/channel"] = ch["p"].numpy()
    return out


def fisher_bridge():
    """FisherAccumulator on a toy Linear with ONE token per backward: the
    reference's ||gy^T x||^2 equals the per-token product of squared norms."""
    torch.manual_seed(3)
    model = torch.nn.Sequential(torch.nn.Linear(64, 48, bias=False), torch.nn.Linear(48, 32, bias=False))
    model = model.to(torch.float32)
    tracked = ["0", "1"]
    acc = sp.FisherAccumulator(model, tracked, {}, hook_packed_experts=False)
    xs, gys = {n: [] for n in tracked}, {n: [] for n in tracked}
    mods = dict(model.named_modules())
    hooks = []
    for n in tracked:
        hooks.append(mods[n].register_forward_hook(lambda m, i, o, n=n: xs[n].append(i[0].detach().clone())))
        hooks.append(mods[n].register_full_backward_hook(lambda m, gi, go, n=n: gys[n].append(go[0].detach().clone())))
    inputs = torch.randn(5, 1, 64)
    for i in range(inputs.shape[0]):
        y = model(inputs[i])
        y.pow(2).sum().backward()
    acc.finalize(None)
    for h in hooks:
        h.remove()
    out = {}
    for n in tracked:
        out[f"bridge/{n}/x"] = torch.cat(xs[n]).numpy()
        out[f"bridge/{n}/gy"] = torch.cat(gys[n]).numpy()
        out[f"bridge/{n}/h_trace_raw"] = np.array([acc.stats[n]["h_trace_raw"]], dtype=np.float64)
        out[f"bridge/{n}/n_tokens_seen"] = np.array([acc.stats[n]["n_tokens_seen"]], dtype=np.int64)
    return out


def fisher_detail():
    """FisherAccumulator with h_detail_dir on a toy bf16 model, several tokens per backward: each
    backward's inputs and output gradients, the h_diag files the reference writes and its exact
    stats (h_trace_raw = sum of bf16(grad_w)^2, h_w2_sum_raw, n_tokens_seen)."""
    import tempfile
    torch.manual_seed(5)
    model = torch.nn.Sequential(torch.nn.Linear(64, 48, bias=False), torch.nn.Linear(48, 32, bias=False))
    model = model.to(torch.bfloat16)
    tracked = ["0", "1"]
    out = {}
    with tempfile.TemporaryDirectory() as d:
        acc = sp.FisherAccumulator(model, tracked, {}, hook_packed_experts=False, h_detail_dir=Path(d))
        xs, gys = {n: [] for n in tracked}, {n: [] for n in tracked}
        mods = dict(model.named_modules())
        hooks = []
        for n in tracked:
            hooks.append(mods[n].register_forward_hook(lambda m, i, o, n=n: xs[n].append(i[0].detach().clone())))
            hooks.append(mods[n].register_full_backward_hook(
                lambda m, gi, go, n=n: gys[n].append(go[0].detach().clone())))
        inputs = torch.randn(5, 16, 64).to(torch.bfloat16)
        for i in range(inputs.shape[0]):
            y = model(inputs[i])
            y.float().pow(2).sum().backward()
        acc.finalize(None)
        for h in hooks:
            h.remove()
        for n in tracked:
            blob = torch.load(Path(d) / (n + ".pt"), weights_only=False)
            out[f"detail/{n}/x"] = torch.stack(xs[n]).view(torch.int16).numpy()
            out[f"detail/{n}/gy"] = torch.stack(gys[n]).view(torch.int16).numpy()
            out[f"detail/{n}/w"] = mods[n].weight.detach().view(torch.int16).numpy()
            out[f"detail/{n}/h_diag"] = blob["h_diag"].numpy()
            out[f"detail/{n}/kind"] = np.array([blob["kind"]])
            for k in ("h_trace_raw", "h_w2_sum_raw"):
                out[f"detail/{n}/{k}"] = np.array([acc.stats[n][k]], dtype=np.float64)
            out[f"detail/{n}/n_tokens_seen"] = np.array([acc.stats[n]["n_tokens_seen"]], dtype=np.int64)
            out[f"detail/{n}/h_detail_path"] = np.array([acc.stats[n]["h_detail_path"]])
    return out


def known_answers():
    out = {}
    v = torch.tensor([0.25, 0.75, -0.75, 1.25, -1.25, 2.5, -2.5, 5.0, -5.0, -0.0, -0.1, 0.0, 0.5, 1.0, 6.0, -6.0, 7.0, -7.0])
    out["ka/round_to_codebook/in"] = v.numpy()
    out["ka/round_to_codebook/out"] = enc._round_to_codebook(v).numpy()
    # cost-path signed-codebook RTN on a row whose amax is 6 (scale exactly 1)
    c = torch.tensor([[0.25, 0.75, -0.75, 1.25, -1.25, 2.5, -2.5, 5.0, -5.0, -0.0, -0.1, 6.0]])
    out["ka/cost_e2m1/in"] = c.numpy()
    out["ka/cost_e2m1/out"] = fr._rtn_fp_codebook(c, fr._CODEBOOKS["fp4_e2m1"], 0).numpy()
    idx = torch.tensor([[1, 2, 3, 4]])
    out["ka/pack/out"] = enc.pack_fp4_indices(idx, 4).numpy()
    return out


def cost_pipeline():
    """The reference's cost tables for the toy model of tests/golden/pipeline_model.py."""
    from tests.golden.pipeline_model import run_cost_pipeline
    return run_cost_pipeline(mqc, fr, "cpu")


def fisher_bridge_bf16():
    """FisherAccumulator (fp32 model, ONE token per backward) on inputs and output gradients that
    are all bf16 values, so the B200 per-token kernels can take the very same numbers: then the
    reference's ||gy^T x||_F^2 (fp32 GEMM, square, sum) equals sum_t ||x_t||^2 ||g_t||^2 up to fp32
    rounding.  Two Linears, each fed its own input and output gradient (no chain rule between
    them, so every recorded gradient stays a bf16 value)."""
    torch.manual_seed(7)
    model = torch.nn.ModuleDict({"0": torch.nn.Linear(64, 48, bias=False), "1": torch.nn.Linear(48, 32, bias=False)})
    tracked = ["0", "1"]
    acc = sp.FisherAccumulator(model, tracked, {}, hook_packed_experts=False)
    bf = lambda t: t.to(torch.bfloat16).float()   # noqa: E731
    xs = {"0": bf(torch.randn(6, 1, 64)), "1": bf(torch.randn(6, 1, 48) * 3)}
    gs = {"0": bf(torch.randn(6, 1, 48) * 0.01), "1": bf(torch.randn(6, 1, 32) * 0.1)}
    for i in range(6):
        ys = [model[n](xs[n][i].clone().requires_grad_(True)) for n in tracked]
        torch.autograd.backward(ys, [gs[n][i] for n in tracked])
    acc.finalize(None)
    out = {}
    for n in tracked:
        out[f"bridge16/{n}/x"] = xs[n].reshape(6, -1).to(torch.bfloat16).view(torch.int16).numpy()
        out[f"bridge16/{n}/gy"] = gs[n].reshape(6, -1).to(torch.bfloat16).view(torch.int16).numpy()
        out[f"bridge16/{n}/w"] = model[n].weight.detach().to(torch.bfloat16).view(torch.int16).numpy()
        out[f"bridge16/{n}/h_trace_raw"] = np.array([acc.stats[n]["h_trace_raw"]], dtype=np.float64)
        out[f"bridge16/{n}/n_tokens_seen"] = np.array([acc.stats[n]["n_tokens_seen"]], dtype=np.int64)
    return out


def name_seed(name: str) -> int:
    """Per-tensor seed of the full-shape configuration fixtures (the GPU tests derive the same)."""
    import hashlib
    return int.from_bytes(hashlib.sha256(name.encode()).digest()[:6], "little")


# Llama-8B decoder layer (config 2: hidden 4096, intermediate 14336, 32 / 8 heads of 128) and the
# first 4096 rows of lm_head [128256, 4096]
LLAMA8B_LAYER = {"model.layers.0.self_attn.q_proj": (4096, 4096), "model.layers.0.self_attn.k_proj": (1024, 4096),
                 "model.layers.0.self_attn.v_proj": (1024, 4096), "model.layers.0.self_attn.o_proj": (4096, 4096),
                 "model.layers.0.mlp.gate_proj": (14336, 4096), "model.layers.0.mlp.up_proj": (14336, 4096),
                 "model.layers.0.mlp.down_proj": (4096, 14336), "lm_head": (4096, 4096)}
LLAMA8B_SIBLINGS = {"qkv": ["model.layers.0.self_attn.q_proj", "model.layers.0.self_attn.k_proj",
                            "model.layers.0.self_attn.v_proj"],
                    "gate_up": ["model.layers.0.mlp.gate_proj", "model.layers.0.mlp.up_proj"]}
# one Qwen3-30B-A3B-like MoE layer (config 3): 128 experts, hidden 2048, expert intermediate 768
MOE_LAYER = {"model.layers.0.mlp.experts.gate_up_proj": (128, 1536, 2048),
             "model.layers.0.mlp.experts.down_proj": (128, 2048, 768)}


class _PackedExperts(torch.nn.Module):   # class name holds "expert"; owns packed 3-D parameters
    def __init__(self, params):
        super().__init__()
        for n, t in params.items():
            self.register_parameter(n, torch.nn.Parameter(t, requires_grad=False))


def config_fixtures():
    """The reference on one full-shape config-2 decoder layer (+ lm_head rows) and one config-3
    MoE layer: per tensor the MSE_W of each cost format and SHA-256 digests of W_hat, of the NVFP4
    export (fused-sibling joint globals for q/k/v and gate/up) and of the MXFP8 / FP8 exports;
    for the packed experts, _measure_packed_experts' table, the batched W_hat and the per-expert
    NVFP4 export."""
    out = {"llama8b_layer": {}, "moe30b_layer": {}}
    joint = {}
    for members in LLAMA8B_SIBLINGS.values():
        g = torch.stack([enc.compute_nvfp4_global_real(
            to_t(O.synthetic_weight_bits(LLAMA8B_LAYER[m], seed=name_seed(m))).float()) for m in members]).max()
        for m in members:
            joint[m] = g
    for name, shape in LLAMA8B_LAYER.items():
        bits = O.synthetic_weight_bits(shape, seed=name_seed(name))
        d = full_case(bits, joint=joint.get(name))
        d["seed"] = name_seed(name)
        if name in joint:
            d["joint_global_real"] = float(joint[name].item())
        out["llama8b_layer"][name] = d
        print("[config2]", name, flush=True)
    model = torch.nn.Module()
    model.add_module("experts", _PackedExperts({n.rsplit(".", 1)[1]: to_t(O.synthetic_weight_bits(s, seed=name_seed(n)))
                                                 for n, s in MOE_LAYER.items()}))
    specs = [fr.get_format(f) for f in COST_FMTS]
    accum = {}
    mqc._measure_packed_experts(model, {"experts.gate_up_proj", "experts.down_proj"}, specs, "cpu", torch.bfloat16,
                                accum)
    table = mqc._finalize_results(accum)
    for name, shape in MOE_LAYER.items():
        pn = name.rsplit(".", 1)[1]
        W = getattr(model.experts, pn).detach()
        d = {"seed": name_seed(name), "shape": list(shape), "input": O.digest(bits_of(W)),
             "table": table["experts." + pn]}
        for fmt in COST_FMTS:
            d[f"qdq/{fmt}"] = O.digest(bits_of(mqc._batched_quantize(fr.get_format(fmt), W)))
        wp, ws, wg = enc.quantize_dequantize_nvfp4_packed(W.float())
        d["nvfp4_packed"] = O.digest(u8_of(wp), u8_of(ws), wg.numpy())
        out["moe30b_layer"][name] = d
        print("[config3]", name, flush=True)
    return out


class _RecordingProfile:
    """Wraps one of the reference's model profiles and records every answer the config
    builder asks of it, so the test can replay the profile as plain tables."""

    def __init__(self, inner):
        self.inner, self.names = inner, {}

    def to_vllm_internal_name(self, name):
        self.names[name] = self.inner.to_vllm_internal_name(name)
        return self.names[name]

    def __getattr__(self, attr):
        return getattr(self.inner, attr)


def _qconfig_cases():
    L = "model.layers"
    dense = {}
    for i in range(2):
        dense.update({f"{L}.{i}.self_attn.q_proj": "NVFP4", f"{L}.{i}.self_attn.k_proj": "NVFP4",
                      f"{L}.{i}.self_attn.v_proj": "NVFP4", f"{L}.{i}.self_attn.o_proj": "MXFP8",
                      f"{L}.{i}.mlp.gate_proj": "NVFP4", f"{L}.{i}.mlp.up_proj": "NVFP4",
                      f"{L}.{i}.mlp.down_proj": "BF16"})
    dense[f"{L}.1.self_attn.v_proj"] = "MXFP8"          # a mixed fused group: no fused target
    per_expert = {f"{L}.{l}.mlp.experts.{e}.{p}_proj": ("NVFP4" if l != 10 else "MXFP8")
                  for l in (2, 10) for e in range(8) for p in ("gate", "up", "down")}
    per_expert.update({f"{L}.3.mlp.experts.{e}.gate_proj": "MXFP8" for e in (0, 2, 5)})
    per_expert.update({f"{L}.3.mlp.experts.{e}.up_proj": "BF16" for e in (1, 4)})
    packed = {f"{L}.{l}.mlp.experts.{p}": f for l, f in ((0, "NVFP4"), (1, "MXFP8"), (2, "BF16"))
              for p in ("gate_up_proj", "down_proj")}
    packed.update({f"{L}.{l}.self_attn.q_proj": "NVFP4" for l in range(3)})
    packed.update({"mtp.layers.0.mlp.experts.gate_up_proj": "BF16", "mtp.layers.0.mlp.experts.down_proj": "BF16"})
    mixtral = {f"{L}.0.block_sparse_moe.experts.w{k}": "BF16" for k in (1, 2, 3)}
    mixtral.update({f"{L}.0.self_attn.{p}_proj": "INT3" for p in "qkvo"})
    mixtral.update({f"{L}.0.mlp.gate": "NVINT2", "lm_head": "FP8_SOURCE", "mtp.experts.down_proj": "BF16"})
    llama_map = {"qkv_proj": ["q_proj", "k_proj", "v_proj"], "gate_up_proj": ["gate_proj", "up_proj"]}
    qwen_map = {**llama_map, "qkv": ["qkv"], "in_proj_qkvz": ["in_proj_qkv", "in_proj_z"]}
    return [
        # the reference's own test scenarios (tests/test_prismaquant_export_native_compressed.py:353-520)
        ("qwen3_5", {**{f"{L}.{i}.self_attn.k_proj": "MXFP8" for i in range(2)},
                     **{f"{L}.{i}.mlp.experts.down_proj": "NVFP4" for i in range(5)}}, ["lm_head"], [], None),
        ("qwen3_5", {f"{L}.0.mlp.gate_proj": "NVFP4", f"{L}.0.mlp.shared_expert_gate": "BF16"}, ["lm_head"],
         [f"{L}.0.mlp.gate"], None),
        ("qwen3_5", {f"{L}.0.mlp.experts.gate_up_proj": "NVFP4", f"{L}.0.mlp.experts.down_proj": "NVFP4",
                     f"{L}.0.self_attn.q_proj": "NVFP4"}, [], [], None),
        ("qwen3_5", {f"{L}.0.mlp.experts.gate_up_proj": "NVFP4", f"{L}.0.mlp.experts.down_proj": "NVFP4",
                     "mtp.layers.0.mlp.experts.gate_up_proj": "BF16", "mtp.layers.0.mlp.experts.down_proj": "BF16"},
         [], [], None),
        ("qwen3_5", {f"{L}.0.mlp.experts.gate_up_proj": "NVFP4", f"{L}.0.mlp.experts.down_proj": "MXFP8"}, [], [], None),
        # wider cases
        ("qwen3_5", packed, ["lm_head", "model.embed_tokens"], [f"{L}.0.mlp.gate"], qwen_map),
        ("qwen3_5", {**packed, f"{L}.0.linear_attn.in_proj_qkv": "MXFP8", f"{L}.0.linear_attn.in_proj_z": "MXFP8",
                     f"{L}.1.linear_attn.in_proj_qkv": "BF16"}, [], [], qwen_map),
        ("default", dense, ["lm_head"], [], llama_map),
        ("default", dense, ["lm_head"], [], None),
        ("default", {f"{L}.0.self_attn.k_proj": "BF16", f"{L}.0.mlp.up_proj": "BF16",
                     f"{L}.0.mlp.down_proj": "NVFP4"}, [], [], llama_map),
        ("default", per_expert, [], ["router"], None),
        ("qwen3_5", per_expert, [], [], None),
        ("default", packed, ["lm_head"], [], None),
        ("default", mixtral, [], [], None),
        ("default", {f"{L}.0.mlp.gate_proj": "MXFP8", f"{L}.0.mlp.up_proj": "NVFP4"}, [], [], None),   # size tie
        ("default", {f"{L}.0.mlp.down_proj": "BF16"}, ["lm_head"], [], None),                        # nothing quantized
        ("default", {f"{L}.0.mlp.down_proj": "FP8_E4M3", f"{L}.1.mlp.down_proj": "NVFP4"}, [], [], None),  # no scheme
    ]


def qconfig_fixtures():
    """The reference's config builder on recipe assignments (mode `qconfig`)."""
    import tempfile
    from prismaquant.model_profiles import vllm_registry as vr
    from prismaquant.model_profiles.default import DefaultProfile
    from prismaquant.model_profiles.qwen3_5 import Qwen3_5Profile
    out = {"build": [], "write": []}
    real_pm = vr.packed_modules_mapping_from_class
    for kind, assignment, passthrough, extra, mapping in _qconfig_cases():
        prof = _RecordingProfile(Qwen3_5Profile() if kind == "qwen3_5" else DefaultProfile())
        vr.packed_modules_mapping_from_class = (lambda _cls, m=mapping: dict(m or {}))
        try:
            want = enc.build_quantization_config(assignment, set(passthrough), extra, profile=prof)
        except (RuntimeError, KeyError) as e:
            want = {"error": type(e).__name__}
        finally:
            vr.packed_modules_mapping_from_class = real_pm
        out["build"].append({"assignment": assignment, "bf16_passthrough": passthrough, "extra_ignore": extra,
                             "packed_mapping": mapping or {}, "names": prof.names,
                             "moe_regex": prof.per_expert_moe_regex(), "mtp_regex": prof.per_expert_mtp_regex(),
                             "want": want})
    # config.json: quantization_config and the pruned expert counts (the profile is detected from it)
    src_cfg = {"architectures": ["ToyMoeForCausalLM"], "model_type": "toy_moe", "num_experts": 8,
               "num_local_experts": 8, "hidden_size": 64, "text_config": {"n_routed_experts": 8, "vocab_size": 32}}
    for assignment, prune in ((_qconfig_cases()[7][1], None),
                              ({"model.layers.0.mlp.experts.gate_up_proj": "NVFP4",
                                "model.layers.0.mlp.experts.down_proj": "NVFP4"},
                               {"model.layers.0.mlp": {"num_experts_kept": 6}}),
                              ({"model.layers.0.mlp.down_proj": "BF16"}, None)):
        with tempfile.TemporaryDirectory() as src, tempfile.TemporaryDirectory() as dst:
            Path(src, "config.json").write_text(json.dumps(src_cfg))
            enc.write_config_with_quantization(src, Path(dst), assignment, {"lm_head"}, (), prune)
            out["write"].append({"src_config": src_cfg, "assignment": assignment, "bf16_passthrough": ["lm_head"],
                                 "prune_manifest": prune, "want_text": Path(dst, "config.json").read_text()})
    return out


def main():
    if "qconfig" in sys.argv[1:]:         # only the quantization_config fixtures
        with open(HERE / "qconfig_cases.json", "w") as f:
            json.dump(qconfig_fixtures(), f, indent=1)
        return
    if "fisher_detail" in sys.argv[1:]:   # only the per-weight Fisher fixture
        np.savez_compressed(HERE / "fisher_detail.npz", **fisher_detail())
        return
    if "fisher_bridge" in sys.argv[1:]:   # only the bf16-valued Fisher bridge
        np.savez_compressed(HERE / "fisher_bridge_bf16.npz", **fisher_bridge_bf16())
        return
    if "configs" in sys.argv[1:]:         # only the full-shape config-2 / config-3 fixtures
        with open(HERE / "config_digests.json", "w") as f:
            json.dump(config_fixtures(), f, indent=1, sort_keys=True)
        return
    arrays = {}
    for name, bits in small_cases().items():
        arrays[f"{name}/input"] = bits
        for k, v in {**run_cost(bits), **run_export(bits), **run_fisher(bits)}.items():
            arrays[f"{name}/{k}"] = v
    arrays.update(fisher_bridge())
    arrays.update(known_answers())
    np.savez_compressed(HERE / "small_cases.npz", **arrays)

    digests = {}
    # single-Linear sweep: 4096x4096, N(0, 0.02^2), 0.1 % x20 outliers, seed 0
    w0 = O.synthetic_weight_bits((4096, 4096), seed=0, outlier_frac=0.001)
    digests["linear4096"] = full_case(w0)
    # fused siblings: q/k/v share one NVFP4 global, gate/up share one
    sib_shapes = {"q_proj": (4096, 4096), "k_proj": (1024, 4096), "v_proj": (1024, 4096),
                  "gate_proj": (14336, 4096), "up_proj": (14336, 4096)}
    sib = {n: O.synthetic_weight_bits(s, seed=i + 1) for i, (n, s) in enumerate(sib_shapes.items())}
    groups = {"qkv": ["q_proj", "k_proj", "v_proj"], "gate_up": ["gate_proj", "up_proj"]}
    dg = {}
    for gname, members in groups.items():
        joint = torch.stack([enc.compute_nvfp4_global_real(to_t(sib[m]).float()) for m in members]).max()
        for m in members:
            d = full_case(sib[m], joint=joint)
            d["joint_global_real"] = float(joint.item())
            d["seed"] = list(sib_shapes).index(m) + 1
            dg[m] = d
    digests["siblings"] = dg
    with open(HERE / "full_digests.json", "w") as f:
        json.dump(digests, f, indent=1, sort_keys=True)
    with open(HERE / "cost_pipeline.json", "w") as f:
        json.dump(cost_pipeline(), f, indent=1, sort_keys=True)
    print("wrote", HERE / "small_cases.npz", HERE / "full_digests.json")


def full_case(bits, joint=None):
    W = to_t(bits)
    d = {"input": O.digest(bits), "shape": list(bits.shape)}
    for fmt in COST_FMTS:
        What = fr.get_format(fmt).quantize_dequantize(W.clone())
        d[f"mse/{fmt}"] = float((W - What).float().pow(2).mean().item())
        d[f"qdq/{fmt}"] = O.digest(bits_of(What))
    Wf = W.float()
    wp, ws, wg = enc.quantize_dequantize_nvfp4(Wf, global_real_override=joint)
    d["nvfp4"] = O.digest(u8_of(wp), u8_of(ws), wg.numpy())
    d["nvfp4_global_div"] = float(wg.item())
    w8, s8 = enc.quantize_dequantize_mxfp8(Wf)
    d["mxfp8"] = O.digest(u8_of(w8), u8_of(s8))
    wf, sf = enc.quantize_dequantize_fp8_dynamic(Wf)
    d["fp8dyn"] = O.digest(u8_of(wf), sf.numpy())
    return d


if __name__ == "__main__":
    main()
