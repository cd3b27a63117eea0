"""Benchmark: full-model multi-format cost sweep + NVFP4 export.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

One step = one pass of the hot path over one synthetic model: every Linear
is scored for NVFP4, MXFP8 and FP8-per-channel (BF16 error is 0) and exported
to NVFP4 (codes, E4M3 block scales, fused-sibling joint globals), then the
cost table is all-gathered across ranks.  Default workload: Llama-style 8B
dense (32 layers, hidden 4096, intermediate 14336, 32/8 heads of 128,
lm_head 128256 x 4096; 7.50e9 Linear params, 15.01 GB bf16) with random
N(0, 0.02^2) weights.  Multi-GPU is strong scaling by default: the one model's
units (Linears, expert tensors; fused siblings together) are split across the
ranks by bytes, each rank sweeps and exports its shard, and one all-gather
assembles the cost table; value = model bytes / max-rank time.  `--scaling weak`
gives each rank its own model instance instead.

metric "weight GB/s scored" = bf16 weight bytes swept per second (all formats
from one read); inputs (15 GB/rank) are far larger than L2, so no flush is needed.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

PEAKS = REPO / "MEASURED_PEAKS.json"
PROFILE_TRAFFIC = REPO / "profiles" / "traffic.json"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="llama8b",
                    choices=["llama8b", "siblings", "lmhead", "linear4096", "moe30b", "fisher1b", "outerr8b", "kernels",
                             "costtable8b", "fishermoe"])
    ap.add_argument("--moe-tokens", type=int, default=8192, help="tokens per step of the fishermoe workload")
    ap.add_argument("--fisher-seqs", type=int, default=64, help="calibration sequences (split across ranks)")
    ap.add_argument("--fisher-batch", type=int, default=4, help="sequences per backward on each rank")
    ap.add_argument("--fisher-detail", action="store_true",
                    help="per-weight Fisher diagonal (h_detail) on the tensor cores, the reference's exact stats")
    ap.add_argument("--outerr-layers", type=int, default=32,
                    help="decoder layers whose Linears the output-error workload stacks by shape")
    ap.add_argument("--scaling", default="auto", choices=["auto", "strong", "weak"],
                    help="N > 1: strong = one model sharded across the ranks by whole units (fused siblings "
                         "kept together), weak = one model instance per rank; auto = strong")
    ap.add_argument("--pipeline-chunks", type=int, default=1,
                    help="sweep launches per step, each chunk's NVFP4 scale pass overlapping the next chunk")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=3)
    return ap.parse_args()


def run_fisher(a, rank, world, local):
    """Fisher-trace probe on a random-init Llama-style 1B model (16 layers, hidden 2048,
    intermediate 8192, 16 heads, vocab 32000, bf16): calibration ids drawn uniformly from
    [0, 32000) (64 x 2048 by default, seed 0), split across ranks (data parallel); every
    Linear tracked with the per-token estimator; per-rank traces combined with one all_reduce.
    One step = one backward of --fisher-batch sequences on every rank."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from prismaquant_b200 import _lib
    from prismaquant_b200 import distributed as D
    from prismaquant_b200 import sensitivity_probe as sp
    from prismaquant_b200 import synthetic as S
    from transformers import LlamaForCausalLM

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    torch.manual_seed(0)
    cfg = S.llama_1b_config()
    model = LlamaForCausalLM(cfg).to(device=dev, dtype=torch.bfloat16)
    for p in model.parameters():
        p.requires_grad_(False)
    tracked = [n for n, m in model.named_modules() if isinstance(m, torch.nn.Linear)]
    g = torch.Generator().manual_seed(0)
    calib = torch.randint(0, cfg.vocab_size, (a.fisher_seqs, 2048), generator=g)
    mine = calib[rank::world]
    B = a.fisher_batch

    # time the hook kernels with events on the launching stream
    kev = []
    orig_rn, orig_td = _lib.rownorm2, _lib.tokennorm_dot
    kbytes = [0]

    def timed(fn, nbytes):
        def w(*args, **kw):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            out = fn(*args, **kw)
            e1.record()
            kev.append((e0, e1))
            kbytes[0] += nbytes(*args)
            return out
        return w
    sp._lib.rownorm2 = timed(orig_rn, lambda x: x.numel() * 2 + (x.numel() // x.shape[-1]) * 4)
    sp._lib.tokennorm_dot = timed(orig_td, lambda g_, xn, acc, token_idx=None: g_.numel() * 2 + xn.numel() * 4)
    detail_dir = None
    if a.fisher_detail:   # the tensor-core per-weight diagonal: work counted in FLOP (2 t m n)
        import tempfile
        detail_dir = tempfile.mkdtemp(prefix="pq_hdetail_")
        orig_gs = _lib.grad_sq_acc
        sp._lib.grad_sq_acc = timed(orig_gs, lambda gy, x, h, sums, w=None: 2 * gy.shape[0] * gy.shape[1] * x.shape[1])

    acc = sp.FisherAccumulator(model, tracked, {}, h_detail_dir=detail_dir)
    model.train()
    emb = model.get_input_embeddings()

    def step(i):
        ids = mine[(i * B) % len(mine):(i * B) % len(mine) + B].to(dev)
        with torch.no_grad():
            e = emb(ids)
        e.requires_grad_(True)
        logits = model(inputs_embeds=e).logits
        lp = torch.nn.functional.log_softmax(logits[:, :-1].reshape(-1, logits.size(-1)).float(), dim=-1)
        loss = -lp.gather(1, ids[:, 1:].reshape(-1, 1)).sum()
        loss.backward()
        acc._xnorm.clear()
        acc._saved_inputs.clear()
        if world > 1:
            D.all_reduce_traces(acc.trace_buffer.clone())

    for i in range(a.warmup):
        step(i)
    torch.cuda.synchronize()
    kev.clear()
    kbytes[0] = 0
    if world > 1:
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        t0.record()
        for i in range(a.steps):
            step(i)
        t1.record()
        torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    ms_t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    kern_ms = sum(e0.elapsed_time(e1) for e0, e1 in kev)
    tokens = world * a.steps * B * 2048
    hbm, peak_kind = peaks()
    achieved = kbytes[0] / (kern_ms / 1e3) / 1e9 if kern_ms > 0 else 0.0
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
            "frac": round(achieved / hbm, 4), "traffic": None, "peak_kind": peak_kind,
            "kernel": "rownorm2 + tokennorm_dot (hook kernels)",
            "kernel_ms_per_step": round(kern_ms / a.steps, 4), "hook_share_of_step": round(kern_ms / ms, 4)}
    if a.fisher_detail:
        try:
            tf_peak = float(json.loads(PEAKS.read_text())["bf16_tflops"])
        except Exception:
            tf_peak = 1590.0
        tf = kbytes[0] / (kern_ms / 1e3) / 1e12 if kern_ms > 0 else 0.0
        roof = {"bound": "tensor", "achieved": round(tf, 1), "peak": tf_peak, "unit": "TFLOP/s",
                "frac": round(tf / tf_peak, 4), "traffic": None, "peak_kind": "measured (burst)",
                "kernel": "gradsq_kernel (per-weight Fisher diagonal, tcgen05)",
                "kernel_ms_per_step": round(kern_ms / a.steps, 4), "hook_share_of_step": round(kern_ms / ms, 4)}
    if rank == 0:
        print(json.dumps({
            "metric": "Fisher probe tokens/s (fwd+bwd with per-token trace hooks)", "value": round(tokens / (ms_max / 1e3), 1),
            "unit": "tokens/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": round(ms_max / a.steps, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic: random-init weights, uniform token ids",
            "config": {"workload": "llama1b_fisher_probe" + ("_h_detail" if a.fisher_detail else ""),
                       "seq_len": 2048, "seqs_per_step_per_rank": B, "tracked_linears": len(tracked),
                       "parallelism": f"data-parallel x{world}, traces all-reduced"},
            "roofline": roof,
            "clocks": clk.summary(), "gpu_launches": len(kev)}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


OUTERR_GROUPS = [  # a Llama-8B decoder layer's Linears by shape: (name, per layer, out, in)
    ("q_proj+o_proj", 2, 4096, 4096), ("k_proj+v_proj", 2, 1024, 4096),
    ("gate_proj+up_proj", 2, 14336, 4096), ("down_proj", 1, 4096, 14336)]
OUTERR_ROWS = 256          # cached activation rows per Linear (the probe's input_rows)
OUTERR_FORMATS = ("NVFP4", "MXFP8", "FP8_E4M3")


def run_outerr(a, rank, world, local):
    """Output-error pass of the cost table (measure_quant_cost.py:599-605, 630-635) over the
    Linears of --outerr-layers Llama-8B decoder layers (default 32: the whole model but lm_head),
    stacked by shape as measure_batched_gpu stacks them (its chunk_size of 256 holds each group
    whole), with 256 cached activation rows each (N(0,1) activations, N(0, 0.02^2) weights,
    rank-seeded).  One step = per shape group y_ref and its energy once (pq_output_ref) and the
    output error of
    NVFP4, MXFP8 and FP8-per-channel (pq_output_err on the formats' W_hat / X_hat, made before
    the timed region).  The reference's torch chain on the same tensors (bmm y_ref once, then per
    format bmm + (y_ref - y_q).float().pow(2).mean) is timed right after and reported beside it.
    Replicas when world > 1 (each rank its own layer; max-rank time)."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from prismaquant_b200 import _lib
    from prismaquant_b200 import format_registry as fr
    from prismaquant_b200 import measure_quant_cost as mqc

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    groups = []
    flops = 0
    hbm_bytes = 0
    for name, per_layer, out, k in OUTERR_GROUPS:
        b = per_layer * a.outerr_layers
        W = torch.empty(b, out, k, dtype=torch.bfloat16, device=dev)
        for i in range(b):   # one Linear at a time keeps the fp32 temporary small
            W[i] = (torch.randn(out, k, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        X = torch.randn(b, OUTERR_ROWS, k, device=dev, generator=g).to(torch.bfloat16)
        fmts = []
        for f in OUTERR_FORMATS:
            spec = fr.get_format(f)
            fmts.append((f, mqc._batched_quantize(spec, W), spec.activation_quantize_dequantize(X.clone())))
        y = torch.empty(b, OUTERR_ROWS, out, dtype=torch.bfloat16, device=dev)
        groups.append((name, W, X, fmts, y))
        flops += 2 * b * OUTERR_ROWS * out * k * (1 + len(fmts))
        # algorithmic bytes: W, X, y_ref written once; per format W_hat, X_hat, y_ref read
        hbm_bytes += (W.numel() + X.numel() + y.numel()) * 2 + len(fmts) * (W.numel() + X.numel() + y.numel()) * 2
    sums = torch.zeros(len(groups), 1 + len(OUTERR_FORMATS), max(gr[1].shape[0] for gr in groups),
                       dtype=torch.float64, device=dev)
    launches = [0]

    def ours():
        for gi, (_, W, X, fmts, y) in enumerate(groups):
            b = W.shape[0]
            _lib.output_ref(X, W, sums[gi, 0, :b], y)
            for fi, (_, Wh, Xh) in enumerate(fmts):
                _lib.output_err(Xh, Wh, y, sums[gi, 1 + fi, :b])
            launches[0] += 1 + len(fmts)

    def torch_chain():
        res = []
        for _, W, X, fmts, _ in groups:
            y_ref = torch.bmm(X, W.transpose(1, 2))
            res.append(y_ref.float().pow(2).mean(dim=(1, 2)))
            for _, Wh, Xh in fmts:
                res.append((y_ref - torch.bmm(Xh, Wh.transpose(1, 2))).float().pow(2).mean(dim=(1, 2)))
        return res

    def timed(fn, steps):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(a.warmup):
        ours()
    launches[0] = 0
    with ClockSampler(local) as clk:
        ms = timed(ours, a.steps)
    n_launch = launches[0]
    if _lib.device_error() != 0:
        raise RuntimeError("output-error kernels reported a device error")
    # parity with the torch chain on the same tensors (summation order and bf16 rounding of
    # differently ordered fp32 sums differ: 2e-2 relative on the error, 1e-3 on the energy)
    sums.zero_()
    ours()
    ref_res = torch_chain()
    got = []
    for gi, (_, W, _, fmts, _) in enumerate(groups):
        b = W.shape[0]
        n_out = OUTERR_ROWS * W.shape[1]
        got += [sums[gi, j, :b] / n_out for j in range(1 + len(fmts))]
    worst = max(float(((x - r.double()).abs() / r.double().abs().clamp_min(1e-30)).max()) for x, r in zip(got, ref_res))
    for _ in range(a.warmup):
        torch_chain()
    ms_torch = timed(torch_chain, a.steps)
    peak = None
    peak_kind = "fallback"
    try:
        peak = float(json.loads(PEAKS.read_text())["bf16_tflops"])
        peak_kind = "measured (burst)"
    except Exception:
        peak = 1590.0
    hbm, _ = peaks()
    tflops = flops * a.steps / (ms / 1e3) / 1e12 * world
    per_gpu = flops / (ms / a.steps / 1e3) / 1e12
    if rank == 0:
        print(json.dumps({
            "metric": "output-error TFLOP/s (y_ref once + 3 formats, fused error epilogue)",
            "value": round(tflops, 1), "unit": "TFLOP/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": round(ms / a.steps, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 (fp32 accumulate)",
            "data": "synthetic: N(0,1) activations, N(0,0.02^2) weights",
            "config": {"workload": f"llama8b_output_error_{a.outerr_layers}_layers", "rows": OUTERR_ROWS,
                       "groups": [f"{n} [{b * a.outerr_layers},{o},{k}]" for n, b, o, k in OUTERR_GROUPS],
                       "formats": list(OUTERR_FORMATS),
                       "l2": f"operands per step {hbm_bytes / 1e9:.1f} GB > L2, no flush"},
            "roofline": {"bound": "tensor", "achieved": round(per_gpu, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(per_gpu / peak, 4), "peak_kind": peak_kind,
                         "hbm_achieved_gbs": round(hbm_bytes / (ms / a.steps / 1e3) / 1e9, 1), "hbm_peak_gbs": hbm,
                         "hbm_bound_ms": round(hbm_bytes / hbm / 1e6, 4),
                         "tensor_bound_ms": round(flops / peak / 1e9, 4),
                         "kernel": "outerr_kernel (tcgen05 cta_group::2, TMA ring)"},
            "torch_chain": {"ms_per_step": round(ms_torch / a.steps, 4),
                            "speedup": round(ms_torch / ms, 3), "max_rel_diff": worst},
            "clocks": clk.summary(), "gpu_launches": n_launch}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_kernels(a, local):
    """Per-kernel table: every library kernel timed alone (CUDA events, back-to-back calls after
    warm-up) on inputs larger than L2, with its algorithmic bytes per call and the fraction of the
    measured HBM bandwidth (TFLOP/s of the measured bf16 peak for the output-error GEMM).
    Weights: one [32768, 4096] bf16 tensor (268 MB), N(0, 0.02^2); H: fp32 of the same shape;
    activations / gradients: [65536, 4096] bf16."""
    import torch

    from prismaquant_b200 import _lib

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev).manual_seed(7)
    R, C = 32768, 4096
    n = R * C
    W = (torch.randn(R, C, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    H = torch.rand(R, C, device=dev, generator=g)
    X = torch.randn(65536, C, device=dev, generator=g).to(torch.bfloat16)
    xnorm = _lib.rownorm2(X)
    acc2 = torch.zeros(2, dtype=torch.float64, device=dev)
    sse = torch.zeros(1, 4, dtype=torch.float64, device=dev)
    s0 = torch.zeros((), dtype=torch.float64, device=dev)
    s3 = torch.zeros(3, dtype=torch.float64, device=dev)
    codes = torch.empty(R, C // 2, dtype=torch.uint8, device=dev)
    amax = torch.empty(R, C // 16, dtype=torch.int16, device=dev)
    tmax = torch.zeros(1, dtype=torch.int32, device=dev)
    Xo = torch.randn(16, 256, C, device=dev, generator=g).to(torch.bfloat16)
    Wo = (torch.randn(16, 4096, C, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    Yo = torch.empty(16, 256, 4096, dtype=torch.bfloat16, device=dev)
    eo = torch.zeros(16, dtype=torch.float64, device=dev)
    _lib.output_ref(Xo, Wo, eo, Yo)
    hbm, _ = peaks()
    try:
        tf_peak = float(json.loads(PEAKS.read_text())["bf16_tflops"])
    except Exception:
        tf_peak = 1590.0
    gb = lambda b: b / 1e9
    table = [   # name, call, algorithmic bytes (or FLOP for the GEMM), unit
        ("sweep_fast_kernel: NVFP4+MXFP8+FP8-channel MSE_W", lambda: _lib.sweep_sse([W], [7], sse=sse), 2 * n, "GB/s"),
        ("sweep_fast_kernel + NVFP4 codes (export pass 1)",
         lambda: _lib.sweep_sse([W], [15], nvfp4_outputs=[(codes, amax, tmax)], sse=sse), 2.625 * n, "GB/s"),
        ("nvfp4_pack (codes + E4M3 scales + global)", lambda: _lib.nvfp4_pack(W), (2 + 0.5 + 1 / 16 + 0.25) * n, "GB/s"),
        ("mxfp8_pack", lambda: _lib.mxfp8_pack(W), (2 + 1 + 1 / 32) * n, "GB/s"),
        ("fp8_channel_pack", lambda: _lib.fp8_channel_pack(W), 3 * n, "GB/s"),
        ("cost_qdq NVFP4 (W_hat)", lambda: _lib.cost_qdq(W, "NVFP4"), 4 * n, "GB/s"),
        ("cost_qdq MXFP8 (W_hat)", lambda: _lib.cost_qdq(W, "MXFP8"), 4 * n, "GB/s"),
        ("cost_qdq FP8_E4M3 (W_hat)", lambda: _lib.cost_qdq(W, "FP8_E4M3"), 4 * n, "GB/s"),
        ("xfmt2_kernel cost_qdq MXFP4 (W_hat)", lambda: _lib.cost_qdq(W, "MXFP4"), 4 * n, "GB/s"),
        ("xfmt2_kernel cost_qdq MXFP6_E3M2 (W_hat)", lambda: _lib.cost_qdq(W, "MXFP6_E3M2"), 4 * n, "GB/s"),
        ("xfmt2_kernel cost_qdq NVFP3 (W_hat)", lambda: _lib.cost_qdq(W, "NVFP3"), 4 * n, "GB/s"),
    ]
    for f in ("MXFP4", "MXFP6_E3M2", "FP8_E5M2", "NVFP3", "INT3", "INT4_W4A16_g128", "INT8_W8A16", "FP8_E4M3_G128"):
        kname = ("mxsse_kernel" if f.startswith("MX") else "fp3sse_kernel" if f == "NVFP3" else
                 "intsse_kernel" if f in ("INT2", "INT3", "INT4_W4A16_g128") else "xfmt2_kernel")
        table.append((f"{kname} format_sse {f}", (lambda f=f: _lib.format_sse(W, f, s0)), 2 * n, "GB/s"))
    mx4 = ["MXFP4", "MXFP6_E3M2", "MXFP6_E2M3", "MXFP8_E5M2"]
    s4 = torch.zeros(len(mx4), dtype=torch.float64, device=dev)
    table.append(("mxsse_kernel format_sse_multi " + "+".join(mx4), lambda: _lib.format_sse_multi(W, mx4, s4),
                  2 * n, "GB/s"))
    table += [
        ("xfmt2_kernel weighted_sse NVFP4 (predicted_dloss)", lambda: _lib.weighted_sse(W, "NVFP4", H, s0), 6 * n, "GB/s"),
        ("sweep_fast_kernel weighted NVFP4+MXFP8+FP8-channel (predicted_dloss)",
         lambda: _lib.weighted_sse_fused(W, _lib.FUSED_FMTS, H, s3), 6 * n, "GB/s"),
        ("rownorm2 (Fisher forward hook)", lambda: _lib.rownorm2(X), X.numel() * 2 + X.shape[0] * 4, "GB/s"),
        ("tokennorm_dot (Fisher backward hook)", lambda: _lib.tokennorm_dot(X, xnorm, acc2), X.numel() * 2 + X.shape[0] * 4,
         "GB/s"),
        ("outerr_kernel ERR [16, 256, 4096] x [16, 4096, 4096]", lambda: _lib.output_err(Xo, Wo, Yo, eo),
         2 * 16 * 256 * 4096 * C, "TFLOP/s"),
    ]
    rows = []
    with ClockSampler(local) as clk:
        for name, fn, work, unit in table:
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.steps):
                fn()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / a.steps
            if unit == "GB/s":
                v = gb(work) / (ms / 1e3)
                rows.append({"kernel": name, "ms": round(ms, 4), "bytes": int(work), "GB/s": round(v, 1),
                             "frac_hbm": round(v / hbm, 4)})
            else:
                v = work / (ms / 1e3) / 1e12
                rows.append({"kernel": name, "ms": round(ms, 4), "flop": int(work), "TFLOP/s": round(v, 1),
                             "frac_bf16": round(v / tf_peak, 4)})
    if _lib.device_error() != 0:
        raise RuntimeError("a kernel reported a device error")
    print(json.dumps({"metric": "per-kernel throughput (each kernel alone)", "unit": "GB/s | TFLOP/s",
                      "steps": a.steps, "data": "synthetic: N(0,0.02^2) weights, N(0,1) activations",
                      "config": {"workload": "kernel_table", "weight": [R, C], "activations": list(X.shape),
                                 "l2": "every input > 126 MB L2, no flush"},
                      "peaks": {"hbm_gbs": hbm, "bf16_tflops": tf_peak}, "kernels": rows,
                      "clocks": clk.summary()}), flush=True)


def run_fisher_moe(a, local):
    """Routed packed-expert Fisher probe on one Qwen3-30B-A3B-shaped sparse MoE block (hidden 2048,
    128 experts of intermediate 768, top-8 routing, bf16, random init): one step = forward +
    backward of --moe-tokens tokens with the per-token estimator installed
    (install_routed_expert_hooks: one pq_rownorm2 per projection input and one
    pq_tokennorm_dot_seg per projection's output gradient).  Reports tokens/s and the hook
    kernels' own time and HBM bytes (x and h read for their norms, the two output gradients read
    once) against the measured HBM peak."""
    import torch
    from transformers import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeSparseMoeBlock

    from prismaquant_b200 import _lib
    from prismaquant_b200 import sensitivity_probe as sp
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg = Qwen3MoeConfig(hidden_size=2048, moe_intermediate_size=768, num_experts=128, num_experts_per_tok=8,
                         norm_topk_prob=True)
    torch.manual_seed(0)
    blk = Qwen3MoeSparseMoeBlock(cfg).to(device=dev, dtype=torch.bfloat16)
    with torch.no_grad():
        for p in blk.parameters():
            p.normal_(std=0.02)
            p.requires_grad_(False)
    acc = {}
    sp.install_routed_expert_hooks(blk, acc)
    kev, kbytes = [], [0]
    orig_rn, orig_seg = _lib.rownorm2, _lib.tokennorm_dot_seg

    def timed(fn, nbytes):
        def w(*args, **kw):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            out = fn(*args, **kw)
            e1.record()
            kev.append((e0, e1))
            kbytes[0] += nbytes(*args, **kw)
            return out
        return w
    sp._lib.rownorm2 = timed(orig_rn, lambda x: x.numel() * 2 + (x.numel() // x.shape[-1]) * 4)
    sp._lib.tokennorm_dot_seg = timed(orig_seg, lambda g, xn, seg, acc_, token_idx=None: g.numel() * 2 + 8 * (
        g.numel() // g.shape[-1]))
    T = a.moe_tokens
    gx = torch.Generator(device=dev).manual_seed(1)
    xs = [torch.randn(1, T, 2048, device=dev, dtype=torch.bfloat16, generator=gx) for _ in range(2)]

    def step(i):
        x = xs[i % 2].clone().requires_grad_(True)
        out = blk(x)
        out = out[0] if isinstance(out, tuple) else out
        out.float().pow(2).sum().backward()

    for i in range(a.warmup):
        step(i)
    torch.cuda.synchronize()
    kev.clear()
    kbytes[0] = 0
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        t0.record()
        for i in range(a.steps):
            step(i)
        t1.record()
        torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    k_ms = sum(e0.elapsed_time(e1) for e0, e1 in kev)
    hbm, peak_kind = peaks()
    achieved = kbytes[0] / (k_ms / 1e3) / 1e9 if k_ms > 0 else 0.0
    line = {"metric": "routed MoE Fisher probe tokens/s (one Qwen3-30B-A3B-shaped MoE block)",
            "value": round(a.steps * T / (ms / 1e3), 1), "unit": "tokens/s", "n_gpus": 1, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: random-init N(0, 0.02^2) bf16 block, N(0, 1) hidden states",
            "config": {"workload": "qwen3_30b_a3b_moe_block_routed_fisher", "tokens_per_step": T, "experts": 128,
                       "top_k": 8, "hidden": 2048, "moe_intermediate": 768},
            "hook_kernels": {"launches": len(kev), "ms_per_step": round(k_ms / a.steps, 4),
                             "share_of_step": round(k_ms / ms, 4),
                             "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                                          "frac": round(achieved / hbm, 4), "peak_kind": peak_kind,
                                          "bytes_per_step": kbytes[0] // a.steps}},
            "clocks": clk.summary()}
    print(json.dumps(line), flush=True)


def run_costtable(a, local):
    """The reference's cost-table entry point end to end: measure_quant_cost.measure_batched_gpu
    (measure_quant_cost.py:551-685) on a random-init Llama-8B-shaped model (the 224 decoder
    Linears of 32 layers, N(0, 0.02^2) bf16 weights) with 256 cached activation rows per Linear
    (N(0,1); one tensor per input width, shared), for NVFP4, MXFP8 and FP8 per channel: weight_mse
    from the fused sweep, W_hat per format, the activation quantizers and output_mse /
    rel_output_mse from the tensor-core output-error kernels, with the reference's cost-table
    schema as the result.  One step = one full call (its host syncs included)."""
    import contextlib
    import io

    import torch
    import torch.nn as nn

    from prismaquant_b200 import _lib
    from prismaquant_b200 import format_registry as fr
    from prismaquant_b200 import measure_quant_cost as mqc

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    torch.manual_seed(0)
    model = nn.Module()
    layers = nn.ModuleList()
    shapes = {"self_attn": {"q_proj": (4096, 4096), "k_proj": (4096, 1024), "v_proj": (4096, 1024),
                            "o_proj": (4096, 4096)},
              "mlp": {"gate_proj": (4096, 14336), "up_proj": (4096, 14336), "down_proj": (14336, 4096)}}
    with torch.no_grad():
        for _ in range(32):
            layer = nn.Module()
            for block, projs in shapes.items():
                mod = nn.Module()
                for pn, (fin, fout) in projs.items():
                    lin = nn.Linear(fin, fout, bias=False, device=dev, dtype=torch.bfloat16)
                    lin.weight.normal_(0.0, 0.02)
                    setattr(mod, pn, lin)
                setattr(layer, block, mod)
            layers.append(layer)
    model.layers = layers
    names = {n for n, m in model.named_modules() if isinstance(m, nn.Linear)}
    params = sum(m.weight.numel() for m in model.modules() if isinstance(m, nn.Linear))
    acts_by_width = {w_: torch.randn(256, w_, device=dev).to(torch.bfloat16) for w_ in (4096, 14336)}
    in_of = {n: m.in_features for n, m in model.named_modules() if isinstance(m, nn.Linear)}

    class Acts:
        def __contains__(self, n):
            return n in in_of

        def load(self, n):
            return acts_by_width[in_of[n]]

    specs = [fr.get_format(f) for f in ("NVFP4", "MXFP8", "FP8_E4M3")]
    run = lambda: mqc.measure_batched_gpu(model, Acts(), names, specs, "cuda", torch.bfloat16)
    with contextlib.redirect_stdout(io.StringIO()):
        for _ in range(max(1, a.warmup)):
            table = run()
        torch.cuda.synchronize()
        with ClockSampler(local) as clk:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.steps):
                table = run()
            e1.record()
            torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.steps
    if _lib.device_error() != 0:
        raise RuntimeError("a kernel reported a device error")
    assert len(table) == len(names) and all("error" not in v for e in table.values() for v in e.values())
    sample = table["layers.0.mlp.down_proj"]
    print(json.dumps({
        "metric": "cost table: measure_batched_gpu over an 8B model (weight_mse + output_mse, 3 formats)",
        "value": round(params * 2 / (ms / 1e3) / 1e9, 1), "unit": "GB/s (bf16 weights per second)",
        "n_gpus": 1, "steps": a.steps, "warmup": max(1, a.warmup), "ms_per_step": round(ms, 2),
        "higher_is_better": True, "data": "synthetic: N(0,0.02^2) weights, N(0,1) activations",
        "config": {"workload": "llama8b_cost_table", "linears": len(names), "params": params, "rows": 256,
                   "formats": [s_.name for s_ in specs], "chunk_size": 256},
        "sample_entry": {"layers.0.mlp.down_proj": {f: {k: float(f"{v:.6g}") for k, v in e.items()}
                                                    for f, e in sample.items()}},
        "clocks": clk.summary()}), flush=True)


def workload_shapes(name):
    from prismaquant_b200 import synthetic as S
    if name == "llama8b":
        return S.llama_dense_linears(), "llama8b_dense_sweep_nvfp4_export"
    if name == "siblings":
        return S.fused_sibling_group(), "fused_sibling_qkv_gateup_sweep_nvfp4_export"
    if name == "lmhead":
        return [("lm_head", (128256, 4096))], "llama8b_lm_head_sweep_nvfp4_export"
    if name == "linear4096":
        return [("model.layers.0.self_attn.o_proj", (4096, 4096))], "single_linear_4096_sweep_nvfp4_export"
    if name == "moe30b":
        return S.moe_expert_params(), "qwen3_30b_a3b_packed_expert_sweep"
    if name == "fisher1b":
        return S.llama_dense_linears(n_layers=16, hidden=2048, inter=8192, n_heads=16, n_kv=16, head_dim=128,
                                     vocab=32000), "llama1b_fisher_probe"
    raise ValueError(name)


def peaks():
    try:
        d = json.loads(PEAKS.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """SM clock and clock-event reasons of the rank's GPU during the timed region: read-only NVML
    queries, one sample when the region opens, one when it closes and one every 2 ms between
    (short regions still get samples); nvidia-smi at 200 ms when NVML cannot be loaded."""

    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples = []   # (sm_mhz, max_mhz, {reason, ...})
        self.proc = None
        self.nvml = None
        self.stop = threading.Event()

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        try:   # the CUDA device's PCI address, so the two orderings cannot disagree
            pr = torch.cuda.get_device_properties(self.index)
            bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def _sample_nvml(self):
        nv, h = self.nvml
        bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        masks = (nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                 nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap)
        self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                             float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)),
                             {n for n, m in zip(self.NAMES, masks) if bits & m}))

    def _poll(self):
        while not self.stop.wait(0.002):
            try:
                self._sample_nvml()
            except Exception:
                return

    def __enter__(self):
        try:
            self.nvml = self._nvml_handle()
            self._sample_nvml()
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            return self
        except Exception:
            self.nvml = None
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.index)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                self.samples.append((float(parts[1]), float(parts[2]) if parts[2].replace(".", "").isdigit() else 0.0,
                                     {n for n, v in zip(self.NAMES, parts[5:9]) if v.lower() == "active"}))

    def __exit__(self, *a):
        if self.nvml is not None:
            self.stop.set()
            self.t.join(timeout=5)
            try:
                self._sample_nvml()
            except Exception:
                pass
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(s[0] for s in self.samples),
                "sm_max_mhz": max(s[1] for s in self.samples),
                "reasons": sorted(set().union(*(s[2] for s in self.samples))), "samples": len(self.samples),
                "source": "nvml" if self.nvml is not None else "nvidia-smi"}


# ---------------------------------------------------------------------------
# CPU baseline (oracle port on the host cores, spawn pool)
# ---------------------------------------------------------------------------

def _oracle_rows(args):
    """Oracle work on a row block: all cost formats + NVFP4 codes/scales of the block."""
    bits, = args
    from oracle import pq_oracle as O
    for f in ("NVFP4", "MXFP8", "FP8_E4M3"):
        O.cost_sse(bits, f)
    O.nvfp4_pack(O.bf16_bits_to_f32(bits))
    return bits.size


def cpu_sample_rate(pool, cores, rows=4096, cols=4096, seed=0):
    """Bf16 weight GB/s of the oracle port on one 4096x4096 Linear split by rows over `cores` processes."""
    import numpy as np
    from oracle import pq_oracle as O
    bits = O.synthetic_weight_bits((rows, cols), seed=seed)
    blocks = np.array_split(bits, max(cores, 1) * 2, axis=0)
    t0 = time.perf_counter()
    n = sum(pool.map(_oracle_rows, [(b,) for b in blocks]))
    dt = time.perf_counter() - t0
    return 2.0 * n / dt / 1e9, dt


def make_pool():
    import multiprocessing as mp
    cores = os.cpu_count() or 1
    return mp.get_context("spawn").Pool(cores), cores


# ---------------------------------------------------------------------------

def result_digest(plan, mine, first, table, n_units, world, strong, dev):
    """A checksum of the run's outputs, outside the timed region: per unit an integer checksum of
    its NVFP4 codes, block scales and global (64-bit word sums, exact and order-free, so the row
    blocks of a unit cut into pieces add up to the whole unit's; the global counted by the first
    block only), gathered in unit order and hashed; and the cost table's weight MSE averaged over
    all weights per format.  The codes digest is the same at every N of a strong-scaling run (the
    same model).  mine / first: each plan entry's unit and whether it starts at row 0."""
    import hashlib

    import torch
    import torch.distributed as dist
    n_local = len(mine)
    cs = torch.zeros(max(n_local, 1), 3, dtype=torch.int64, device=dev)
    if plan.export:
        for j, (c, sc, g) in enumerate(plan.outputs):
            for k, t in enumerate((c, sc.view(torch.uint8), g.view(torch.uint8))):
                b = t.reshape(-1)
                pad = (-b.numel()) % 8
                if pad:
                    b = torch.cat([b, torch.zeros(pad, dtype=torch.uint8, device=dev)])
                v = b.view(torch.int64)
                cs[j, k] = v.sum() + (v * 0x9E3779B97F4A7C1).sum() if (k < 2 or first[j]) else 0
    numel = float(sum(plan.numel))
    if world > 1:
        caps = torch.tensor([n_local], device=dev)
        dist.all_reduce(caps, op=dist.ReduceOp.MAX)
        cap = max(1, int(caps.item()))
        rec = torch.full((cap, 4), -1, dtype=torch.int64, device=dev)
        rec[:n_local, 0] = torch.tensor(mine, device=dev)
        rec[:n_local, 1:] = cs[:n_local]
        out = torch.empty(world * cap, 4, dtype=torch.int64, device=dev)
        dist.all_gather_into_tensor(out, rec)
        out = out.cpu()
        if not strong:   # one instance per rank: rank r's units follow rank r-1's
            out[:, 0] += torch.arange(world).repeat_interleave(cap) * n_units * (out[:, 0] >= 0)
        rows = sorted((int(r[0]), r[1:].tolist()) for r in out if r[0] >= 0)
        total = torch.tensor([numel], dtype=torch.float64, device=dev)
        dist.all_reduce(total)
        numel = float(total.item())
    else:
        rows = list(zip(mine, cs[:n_local].cpu().tolist()))
    agg: dict[int, list[int]] = {}   # a unit's pieces add up (64-bit wrap-around, as the sums on the device)
    for uid, vals in rows:
        acc = agg.setdefault(int(uid), [0, 0, 0])
        for k, v in enumerate(vals):
            acc[k] = ((acc[k] + int(v) + (1 << 63)) % (1 << 64)) - (1 << 63)
    h = hashlib.sha256()
    for uid in sorted(agg):
        h.update(uid.to_bytes(8, "little", signed=True))
        for v in agg[uid]:
            h.update(int(v).to_bytes(8, "little", signed=True))
    sse = table.double().sum(dim=0).cpu().tolist()
    return {"nvfp4_export_sha256_16": h.hexdigest()[:16] if plan.export else None,
            "mean_weight_mse": {f: float("%.7g" % (sse[i] / numel)) for i, f in
                                enumerate(("NVFP4", "MXFP8", "FP8_E4M3", "BF16"))}}


def main():
    a = parse()
    if a.warmup < 3:
        a.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if a.workload == "fisher1b" and a.impl == "ours":
        return run_fisher(a, rank, world, local)
    if a.workload == "fishermoe":
        if a.impl == "ours" and rank == 0:
            run_fisher_moe(a, local)
        elif a.impl == "reference" and rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the routed MoE Fisher workload has no CPU "
                              "reference arm (the reference's hooks run the same model on the GPU)"}))
        return
    if a.workload == "costtable8b":
        if a.impl == "ours" and rank == 0:
            run_costtable(a, local)
        elif a.impl == "reference" and rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the cost-table workload has no reference arm on "
                              "the GPU box (the reference is Python and does not travel)"}))
        return
    if a.workload == "kernels":
        if a.impl == "ours" and rank == 0:
            run_kernels(a, local)
        elif a.impl == "reference" and rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the kernel table has no reference arm"}))
        return
    if a.workload == "outerr8b":
        if a.impl == "ours":
            return run_outerr(a, rank, world, local)
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the output-error workload's reference arm is the "
                              "torch bmm chain, timed on the GPU beside ours (torch_chain in its line)"}), flush=True)
        return
    shapes, wl_name = workload_shapes(a.workload)
    params = sum(int(__import__("math").prod(s)) for _, s in shapes)
    metric, unit = "weight GB/s scored across all formats", "GB/s"
    hbm, peak_kind = peaks()

    if a.impl == "reference":
        if rank != 0:
            return
        pool, cores = make_pool()   # spawned before any CUDA use
        for _ in range(a.warmup):
            cpu_sample_rate(pool, cores, rows=512)
        vals, dts = [], []
        for _ in range(a.steps):
            v, dt = cpu_sample_rate(pool, cores)
            vals.append(v)
            dts.append(dt)
        pool.close()
        v = statistics.median(vals)
        line = {"impl": "reference", "metric": metric, "value": round(v, 4), "unit": unit, "n_gpus": a.gpus,
                "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(1e3 * statistics.median(dts), 2),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic", "config": {"workload": wl_name, "model_params": params,
                                                "sample": "one 4096x4096 Linear per step"},
                "cpu_baseline": {"value": round(v, 4), "unit": unit, "cores": cores, "kind": "port",
                                 "sample": "one 4096x4096 bf16 Linear per step: NVFP4/MXFP8/FP8 cost + NVFP4 pack, "
                                           "numpy oracle over a spawn pool"},
                "e2e": {"value": round(v, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    pool = cores = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        pool, cores = make_pool()

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from prismaquant_b200 import distributed as D
    from prismaquant_b200 import export_native_compressed as enc
    from prismaquant_b200 import format_registry as fr
    from prismaquant_b200 import synthetic as S

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    specs = [fr.get_format(f) for f in ("NVFP4", "MXFP8", "FP8_E4M3", "BF16")]
    strong = world > 1 and a.scaling in ("auto", "strong")
    n_units = len(shapes)
    split_slots = split_ids = None
    n_split = 0
    if strong:   # one model: this rank's pieces only, the same per-name seeds at every N
        pieces, owner = D.plan_pieces(shapes, world, [enc.sibling_group_key(n) for n, _ in shapes])
        mine_p = [i for i in range(len(pieces)) if owner[i] == rank]
        cap = D.max_units_per_rank(owner, world)
        n_pieces = [0] * n_units
        for u, _, _ in pieces:
            n_pieces[u] += 1
        split_of = {}
        for u in range(n_units):
            if n_pieces[u] > 1:
                split_of[u] = len(split_of)
        n_split = len(split_of)
        weights, mine, first, slots, sids = {}, [], [], [], []
        for j, i in enumerate(mine_p):   # a row block of a unit cut into pieces: generate the unit, keep the rows
            u, r0, r1 = pieces[i]
            name, sh = shapes[u]
            w = S.cuda_weights([(name, sh)], dev, base_seed=0)[name]
            whole = r0 == 0 and r1 == sh[0]
            weights[name if whole else f"{name}[{r0}:{r1}]"] = w if whole else w[r0:r1].contiguous()
            mine.append(u)
            first.append(r0 == 0)
            if u in split_of:
                slots.append(j)
                sids.append(split_of[u])
        split_slots = torch.tensor(slots, dtype=torch.int64, device=dev)
        split_ids = torch.tensor(sids, dtype=torch.int64, device=dev)
        my_params = sum(w.numel() for w in weights.values())
    else:
        mine = list(range(n_units))
        first = [True] * n_units
        weights = S.cuda_weights(shapes, dev, base_seed=1_000_003 * rank)
        my_params = params
    plan = enc.SweepExportPlan(weights, specs, export_nvfp4=a.workload != "moe30b", pipeline_chunks=a.pipeline_chunks)
    my_ids = torch.tensor(mine, dtype=torch.int64, device=dev)

    def gather():
        if strong:
            return D.all_gather_costs(my_ids, plan.sse, n_units, cap)
        if world > 1:
            return D.all_gather_costs(my_ids + rank * n_units, plan.sse, n_units * world, n_units)
        return plan.sse

    sweep_ms = []

    def step(timed):
        plan.sse.zero_()
        if plan.export:
            plan.tmax.zero_()
        if timed:   # the sweep's device time: its launches on this stream, between two events
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        if n_split:   # units cut into row blocks: the whole sweep, their NVFP4 maximum over all ranks, scales
            plan.launch_sweep()
            D.reduce_split_tmax(plan.tmax, split_slots, split_ids, n_split)
            side = plan.launch_scales_side()
        else:   # each chunk's scale pass on a side stream while the next chunk is swept
            side = plan.launch_pipelined()
        if timed:
            e1.record()
            sweep_ms.append((e0, e1))
        out = gather()   # overlaps the last chunk's scale pass
        if side is not None:
            torch.cuda.current_stream(dev).wait_stream(side)
        return out

    for _ in range(a.warmup):
        step(False)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        t0.record()
        for _ in range(a.steps):
            step(True)
        t1.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = t0.elapsed_time(t1)
    ms_t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    kern_ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in sweep_ms)
    bytes_w = 2.0 * params                       # one model
    job_bytes = bytes_w if strong else world * bytes_w
    value = job_bytes * a.steps / (ms_max / 1e3) / 1e9
    digest = result_digest(plan, mine, first, gather(), n_units, world, strong, dev)

    # dominant kernel roofline: fused sweep + NVFP4 codes; reads 2 B/param, writes 0.5 B/param of codes
    alg_bytes = my_params * (2.0 + (0.5 if plan.export else 0.0))
    achieved = alg_bytes / (kern_ms / 1e3) / 1e9
    traffic = None
    try:
        tr = json.loads(PROFILE_TRAFFIC.read_text())
        traffic = tr.get(wl_name)
        if traffic is not None:   # the capture is of the whole model: this rank's share of it
            traffic = int(traffic * my_params / params)
    except Exception:
        pass

    # end to end through the public API with host buffers: the weights start in pinned host
    # memory; StreamingSweepExport overlaps their H2D copy, the sweep + export and the D2H copy of
    # the packed outputs chunk by chunk; the cost table comes back at the end
    e2e = None
    if not a.no_e2e:
        host = {n: w.cpu().pin_memory() for n, w in weights.items()}
        streamer = enc.StreamingSweepExport(host, specs, export_nvfp4=plan.export, device=dev)
        h2d, d2h = streamer.h2d_bytes, streamer.d2h_bytes
        es = []
        for i in range(a.e2e_steps + 1):
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            streamer.run()
            table = streamer.sse_host()
            s1.record()
            torch.cuda.synchronize()
            if i > 0:
                es.append(s0.elapsed_time(s1))
        d2h += table.numel() * 8
        del streamer
        e_ms = torch.tensor([statistics.mean(es)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
        e2e = {"value": round(job_bytes / (float(e_ms.item()) / 1e3) / 1e9, 3), "unit": unit,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": a.e2e_steps}

    cpu = None
    if pool is not None:
        cpu_sample_rate(pool, cores, rows=256)
        v, dt = cpu_sample_rate(pool, cores)
        pool.close()
        cpu = {"value": round(v, 4), "unit": unit, "cores": cores, "kind": "port",
               "sample": f"one 4096x4096 bf16 Linear ({dt:.1f} s): NVFP4/MXFP8/FP8 cost + NVFP4 pack, numpy oracle "
                         f"over a spawn pool of {cores} processes"}

    if rank == 0:
        line = {
            "metric": metric, "value": round(value, 2), "unit": unit, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms_max / a.steps, 4), "higher_is_better": True,
            "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: random-init N(0, 0.02^2) bf16 weights of the named shapes, generated on the device",
            "config": {"workload": wl_name, "model_params": params, "tensors": n_units,
                       "rank0_params": my_params, "rank0_tensors": len(mine),
                       "formats": ["NVFP4", "MXFP8", "FP8_E4M3", "BF16"], "nvfp4_export": plan.export,
                       "l2": "inputs (2 B/param per rank) far larger than the 126 MB L2; no flush",
                       "parallelism": (f"one model, units sharded by bytes x{world} (strong), cost table "
                                       f"all-gathered" if strong else
                                       f"one model instance per rank x{world} (weak), cost table all-gathered")},
            "hbm_frac": round(value / world / hbm, 4),
            "digest": digest,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "traffic": traffic, "peak_kind": peak_kind,
                         "kernel": "sweep_fast_kernel (fused sweep + NVFP4 codes)",
                         "kernel_ms": round(kern_ms, 4), "algorithmic_bytes_per_launch": alg_bytes},
            "clocks": clk.summary(),
            "gpu_launches": a.steps * (len(plan.chunks) * (2 if plan.export else 1)),   # sweep + scale per chunk
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
