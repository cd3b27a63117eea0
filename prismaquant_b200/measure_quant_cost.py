"""Per-(Linear, format) quantization cost on B200.

Drop-in for the weight-error half of prismaquant/measure_quant_cost.py:
  * `_batched_quantize(spec, stacked_w)`            (:532-548)
  * `measure_batched_gpu(...)` / `measure_unbatched(...)` (:551-685, :266-327)
  * `_measure_packed_experts(...)`                 (:381-449)
  * `_accumulate_result` / `_finalize_results`     (:57-101), same cost-table schema.

The new primitive is `sweep_weight_mse`: ONE kernel pass over every weight
scores all requested formats (NVFP4, MXFP8, FP8 per channel; BF16 is 0 by
definition) and a single device->host copy returns the whole table, where the
reference runs a quantize + subtract + square + mean chain per (chunk,
format) with a host sync each.  `output_mse` / `predicted_dloss` keep the
reference's definitions: the reconstruction comes from the CUDA
quantize-dequantize kernel, and the two products with the error between them
run on the tensor cores (`pq_output_ref` once per chunk, `pq_output_err` per
format), so neither bf16 output of the format is written to memory.
"""
from __future__ import annotations

import math
import re
import time

import torch
import torch.nn as nn

from . import _lib
from . import format_registry as fr

FLT_MAX = float(torch.finfo(torch.float32).max)
_KBIT = {"NVFP4": 1 << _lib.FMT_NVFP4, "MXFP8": 1 << _lib.FMT_MXFP8, "FP8_E4M3": 1 << _lib.FMT_FP8_CHANNEL,
         "BF16": 1 << _lib.FMT_BF16}
_KCOL = {"NVFP4": _lib.FMT_NVFP4, "MXFP8": _lib.FMT_MXFP8, "FP8_E4M3": _lib.FMT_FP8_CHANNEL, "BF16": _lib.FMT_BF16}
_GROUP = {"NVFP4": 16, "MXFP8": 32, "MXFP4": 32, "MXFP6_E3M2": 32, "MXFP6_E2M3": 32, "MXFP8_E5M2": 32,
          "NVFP3": 16, "INT3": 16, "INT2": 16, "INT4_W4A16_g128": 128, "FP8_E4M3_G128": 128}
_FUSED = ("NVFP4", "MXFP8", "FP8_E4M3", "BF16")   # kernel formats of the fused sweep

# measure_quant_cost._batched_quantize (measure_quant_cost.py:516-548) picks the RTN by element dtype:
# codebook dtypes with the spec's group size (E8M0-snapped for family "mx"), integer dtypes with the
# spec's bits and group size, bfloat16 as a clone, and raises for anything else (fp3_e2m0 = NVFP3).
# (element dtype, group size, E8M0) -> kernel format
_BATCHED_CODEBOOK = {
    ("fp4_e2m1", 16, False): "NVFP4", ("fp4_e2m1", 32, True): "MXFP4",
    ("fp6_e3m2", 32, True): "MXFP6_E3M2", ("fp6_e2m3", 32, True): "MXFP6_E2M3",
    ("fp8_e4m3", 32, True): "MXFP8", ("fp8_e4m3", 0, False): "FP8_E4M3",
    ("fp8_e4m3", 128, False): "FP8_E4M3_G128",
    ("fp8_e5m2", 32, True): "MXFP8_E5M2", ("fp8_e5m2", 0, False): "FP8_E5M2",
}
_BATCHED_INT = {(3, 16): "INT3", (2, 16): "INT2", (8, 0): "INT8_W8A16", (4, 128): "INT4_W4A16_g128"}


def canonical_linear_name(name: str) -> str:
    """measure_quant_cost.py:41-55: per-expert Linears -> packed-expert cost keys."""
    m = re.match(r"^(.+\.mlp\.experts)\.(\d+)\.(gate_proj|up_proj|down_proj)$", name)
    if not m:
        return name
    prefix, eid, proj = m.groups()
    return f"{prefix}.gate_up_proj.{eid}" if proj in {"gate_proj", "up_proj"} else f"{prefix}.down_proj.{eid}"


def _kernel_format(spec: fr.FormatSpec) -> str:
    k = getattr(spec, "kernel_format", None)
    if k is None:
        raise NotImplementedError(f"format {spec.name} has no B200 kernel")
    return k


def batched_kernel_format(spec: fr.FormatSpec) -> str:
    """Kernel format of the reference's batched cost path for `spec` (measure_quant_cost.py:535-548);
    raises ValueError with the reference's message for an element dtype it does not take."""
    elt = spec.weight_element_dtype
    if elt in ("fp4_e2m1", "fp6_e3m2", "fp6_e2m3", "fp8_e4m3", "fp8_e5m2"):
        key = (elt, spec.group_size, spec.family == "mx")
        if key not in _BATCHED_CODEBOOK:
            raise NotImplementedError(f"no B200 kernel for {elt} groups of {spec.group_size}")
        return _BATCHED_CODEBOOK[key]
    if elt.startswith("int"):
        key = (spec.weight_bits, spec.group_size)
        if key not in _BATCHED_INT:
            raise NotImplementedError(f"no B200 kernel for INT{spec.weight_bits} groups of {spec.group_size}")
        return _BATCHED_INT[key]
    if elt == "bfloat16":
        return "BF16"
    raise ValueError(f"Unknown weight_element_dtype {elt!r} for batched RTN")


def shape_error(kfmt: str, cols: int) -> str | None:
    """The reference reshapes rows into groups (format_registry.py:208-212); a row
    that does not divide raises there and is recorded as {"error": ...}."""
    g = _GROUP.get(kfmt)
    if g is not None and cols > g and cols % g:
        return f"shape '[-1, {cols // g}, {g}]' is invalid for a row of {cols} elements"
    return None


# ---------------------------------------------------------------------------
# cost-table schema (measure_quant_cost.py:57-101)
# ---------------------------------------------------------------------------

def _accumulate_result(bucket: dict, name: str, fmt: str, weight_mse: float, output_mse: float,
                       rel_output_mse: float, predicted_dloss: float | None = None):
    acc = bucket.setdefault(name, {}).setdefault(fmt, {
        "_count": 0, "_weight_mse_sum": 0.0, "_output_mse_sum": 0.0, "_rel_output_mse_sum": 0.0,
        "_predicted_dloss_sum": 0.0, "_predicted_dloss_count": 0})
    if "error" in acc:
        return
    acc["_count"] += 1
    acc["_weight_mse_sum"] += weight_mse
    acc["_output_mse_sum"] += output_mse
    acc["_rel_output_mse_sum"] += rel_output_mse
    if predicted_dloss is not None:
        acc["_predicted_dloss_sum"] += predicted_dloss
        acc["_predicted_dloss_count"] += 1


def _finalize_results(bucket: dict) -> dict:
    out = {}
    for name, per in bucket.items():
        out[name] = {}
        for fmt, acc in per.items():
            if "error" in acc:
                out[name][fmt] = acc
                continue
            n = max(int(acc["_count"]), 1)
            entry = {"weight_mse": acc["_weight_mse_sum"] / n, "output_mse": acc["_output_mse_sum"] / n,
                     "rel_output_mse": acc["_rel_output_mse_sum"] / n}
            if acc["_predicted_dloss_count"] > 0:
                entry["predicted_dloss"] = acc["_predicted_dloss_sum"] / acc["_predicted_dloss_count"]
            out[name][fmt] = entry
    return out


# ---------------------------------------------------------------------------
# the fused sweep
# ---------------------------------------------------------------------------

def sweep_sse_async(weights: list[torch.Tensor], specs: list[fr.FormatSpec], nvfp4_outputs=None,
                    sse: torch.Tensor | None = None):
    """Launch the fused sweep; returns (sse [n, 4] fp64 on device, errors).

    errors[i][spec.name] holds the reference's error text for a (tensor,
    format) whose grouping the shape cannot take; that format is left out of
    the tensor's mask."""
    kf = [_kernel_format(s) for s in specs]
    masks, errors = [], []
    for w in weights:
        cols = w.shape[-1]
        m, err = 0, {}
        for s, k in zip(specs, kf):
            e = shape_error(k, cols)
            if e:
                err[s.name] = e
            elif k in _KBIT:
                m |= _KBIT[k]
        masks.append(m & 0x7)
        errors.append(err)
    sse = _lib.sweep_sse(weights, masks, nvfp4_outputs=nvfp4_outputs, sse=sse)
    return sse, errors


def _mse_from_sse(sse: float, n: int) -> float:
    if not math.isfinite(sse) or sse > FLT_MAX:
        return float("inf") if not math.isnan(sse) else sse
    return sse / max(n, 1)


def sweep_weight_mse(named_weights, specs: list[fr.FormatSpec],
                     per_linear: bool = False) -> dict[str, dict[str, float | dict]]:
    """{name: {spec.name: weight_mse | {"error": msg}}} for bf16 CUDA weights
    ([out, in] Linears or [E, M, N] packed experts), the fused formats in one pass.

    Each spec is quantized as the batched cost path does (`_batched_quantize`), or, with
    `per_linear`, as its own quantize_dequantize does (measure_unbatched); the two differ only for
    NVFP3 (an error in the batched path) and FP8_SOURCE (E4M3 g128 there, a clone per Linear)."""
    items = list(named_weights.items()) if isinstance(named_weights, dict) else list(named_weights)
    names = [n for n, _ in items]
    weights = [_lib.as_bf16_cuda(w.detach(), "sweep_weight_mse") for _, w in items]
    if not weights:
        return {}
    # the kernel format of each spec as the batched cost path quantizes it
    kf: dict[str, str | None] = {}
    dtype_err: dict[str, str] = {}
    for s in specs:
        try:
            kf[s.name] = _kernel_format(s) if per_linear else batched_kernel_format(s)
        except ValueError as e:
            kf[s.name], dtype_err[s.name] = None, str(e)
    fused = [s for s in specs if kf[s.name] in _FUSED]
    ext = [s for s in specs if kf[s.name] is not None and kf[s.name] not in _FUSED]
    sse, errors = sweep_sse_async(weights, [_as_kernel_spec(s, kf[s.name]) for s in fused])
    ext_sse = torch.zeros(len(weights), max(len(ext), 1), dtype=torch.float64, device=weights[0].device)
    for i, w in enumerate(weights):
        bad = {s.name: shape_error(kf[s.name], w.shape[-1]) for s in ext}
        if ext and not any(bad.values()):   # the MX formats among them from one read
            _lib.format_sse_multi(w, [kf[s.name] for s in ext], ext_sse[i])
            continue
        for j, s in enumerate(ext):
            if bad[s.name]:
                errors[i][s.name] = bad[s.name]
            else:
                _lib.format_sse(w, kf[s.name], ext_sse[i, j])
    host, ext_host = sse.cpu().tolist(), ext_sse.cpu().tolist()   # the device->host copies
    _lib.raise_on_device_error("sweep_weight_mse")
    out = {}
    for i, (name, w) in enumerate(zip(names, weights)):
        per = {}
        for s in specs:
            if s.name in dtype_err:
                per[s.name] = {"error": dtype_err[s.name]}
            elif s.name in errors[i]:
                per[s.name] = {"error": errors[i][s.name]}
            elif kf[s.name] in _FUSED:
                per[s.name] = _mse_from_sse(host[i][_KCOL[kf[s.name]]], w.numel())
            else:
                per[s.name] = _mse_from_sse(ext_host[i][ext.index(s)], w.numel())
        out[name] = per
    return out


def _as_kernel_spec(spec: fr.FormatSpec, kfmt: str) -> fr.FormatSpec:
    """`spec` with kernel_format set to the batched path's kernel format (FP8_SOURCE's
    per-Linear kernel format is a clone; its batched one is not)."""
    if spec.kernel_format == kfmt:
        return spec
    import dataclasses
    return dataclasses.replace(spec, kernel_format=kfmt)


def _batched_quantize(spec: fr.FormatSpec, stacked_w: torch.Tensor) -> torch.Tensor:
    """measure_quant_cost.py:532-548: W_hat of a stacked [N, out, in] weight, the RTN picked by the
    spec's element dtype as the reference does (so NVFP3 raises and FP8_SOURCE is an E4M3 g128 RTN)."""
    k = batched_kernel_format(spec)
    if k == "BF16":
        return stacked_w.clone()
    return _lib.cost_qdq(stacked_w, k)


# ---------------------------------------------------------------------------
# reference entry points
# ---------------------------------------------------------------------------

def _fused_w_hats(W: torch.Tensor, specs, budget: int | None = None):
    """W_hat of every spec whose batched RTN is NVFP4, MXFP8 or FP8 per channel, and each W[n]'s
    squared-error sum for those specs, from one read of the stacked weight (pq_cost_qdq_fused_sse)
    when two or more of them are asked for and the extra slices fit in a quarter of the free
    device memory: ({spec name: W_hat}, {spec name: (fp64 device tensor [N] of sums, elements per
    W[n])}); weight_mse is sum / elements.  ({}, {}) otherwise, or on a shape error (the
    per-format path then reports each format's own error)."""
    by_kernel: dict[str, list[str]] = {}
    for spec in specs:
        try:
            k = batched_kernel_format(spec)
        except Exception:
            continue
        if k in _lib.FUSED_FMTS:
            by_kernel.setdefault(k, []).append(spec.name)
    if len(by_kernel) < 2:
        return {}, {}
    if budget is None:
        budget = torch.cuda.mem_get_info(W.device)[0] // 4
    if W.numel() * 2 * len(by_kernel) > budget:
        return {}, {}
    try:
        hats, sse = _lib.cost_qdq_fused_sse(W, list(by_kernel))
    except ValueError:
        return {}, {}
    per = W[0].numel() if W.dim() == 3 else W.numel()
    out = {name: hats[k] for k, names in by_kernel.items() for name in names}
    mse = {name: (sse[:, _KCOL[k]], per) for k, names in by_kernel.items() for name in names}
    return out, mse


def _fused_w_hats_list(ws, specs, dev: torch.device, budget: int | None = None):
    """_fused_w_hats for a chunk's weights as they are (bf16, contiguous, on `dev`, one shape),
    without stacking them first: the same read also writes the stacked weight
    (pq_cost_qdq_fused_sse_list).  Returns (W_hat dict, sums dict, stacked weight), or
    ({}, {}, None) when the chunk does not qualify; the caller then stacks as the reference does."""
    by_kernel: dict[str, list[str]] = {}
    for spec in specs:
        try:
            k = batched_kernel_format(spec)
        except Exception:
            continue
        if k in _lib.FUSED_FMTS:
            by_kernel.setdefault(k, []).append(spec.name)
    if len(by_kernel) < 2 or not ws:
        return {}, {}, None
    shape = ws[0].shape
    if dev.type == "cuda" and dev.index is None:   # "cuda" names the current device
        dev = torch.device("cuda", torch.cuda.current_device())
    if any(w.device != dev or w.dtype != torch.bfloat16 or w.dim() != 2 or w.shape != shape or
           not w.is_contiguous() for w in ws):
        return {}, {}, None
    if budget is None:
        budget = torch.cuda.mem_get_info(dev)[0] // 4
    if len(ws) * ws[0].numel() * 2 * (len(by_kernel) + 1) > budget:
        return {}, {}, None
    try:
        hats, W, sse = _lib.cost_qdq_fused_sse_list(ws, list(by_kernel))
    except ValueError:
        return {}, {}, None
    per = ws[0].numel()
    out = {name: hats[k] for k, names in by_kernel.items() for name in names}
    mse = {name: (sse[:, _KCOL[k]], per) for k, names in by_kernel.items() for name in names}
    return out, mse, W


def _fused_predicted_dloss(W: torch.Tensor, specs, h: torch.Tensor, per_row: bool = False) -> dict:
    """predicted_dloss of every spec whose batched RTN is NVFP4, MXFP8 or FP8 per channel, from one
    read of each W[n] and h[n], all in one launch (pq_weighted_sse_fused_batch), when two or more
    of them are asked for:
    {spec name: [0.5 * sum(h[n] * err^2) for each n]}; {} otherwise, or on a shape error (the
    per-format path then reports each format's own error)."""
    by_kernel: dict[str, list[str]] = {}
    for spec in specs:
        try:
            k = batched_kernel_format(spec)
        except Exception:
            continue
        if k in _lib.FUSED_FMTS:
            by_kernel.setdefault(k, []).append(spec.name)
    if len(by_kernel) < 2:
        return {}
    try:
        W3 = W if W.dim() == 3 else W.reshape(W.size(0), -1, W.shape[-1])   # packed [1, E, M, N] -> [1, E*M, N]
        out = _lib.weighted_sse_fused_batch(W3, list(by_kernel), h.float(), per_row=per_row)
    except ValueError:
        return {}
    vals = (0.5 * out).cpu()
    return {name: vals[:, _lib.FMT_IDS[k]].tolist() for k, names in by_kernel.items() for name in names}


def _group_by_shape(model: nn.Module, target_names: set[str]):
    groups: dict[tuple[int, int], list[tuple[str, nn.Linear]]] = {}
    for name, mod in model.named_modules():
        cname = canonical_linear_name(name)
        if isinstance(mod, nn.Linear) and cname in target_names:
            groups.setdefault((mod.in_features, mod.out_features), []).append((cname, mod))
    return groups


def _predicted_dloss(W: torch.Tensor, spec: fr.FormatSpec, h: torch.Tensor, per_row: bool,
                     per_linear: bool) -> list[float]:
    """0.5 * sum(h * err^2) for each W[n] of a stacked weight, on the exact kernel (one D2H).
    h[n] has W[n]'s shape, or (per_row) one value per row of W[n]."""
    k = _kernel_format(spec) if per_linear else batched_kernel_format(spec)
    out = torch.zeros(W.size(0), dtype=torch.float64, device=W.device)
    if k != "BF16":
        for n in range(W.size(0)):
            _lib.weighted_sse(W[n], k, h[n].float(), out[n], per_row=per_row)
    return (0.5 * out).cpu().tolist()


def _weight_mse_or_errors(W_list, specs, per_linear=False):
    """Weight MSE of each weight for each spec (one fused pass), as python floats."""
    res = sweep_weight_mse([(str(i), w) for i, w in enumerate(W_list)], specs, per_linear=per_linear)
    return [res[str(i)] for i in range(len(W_list))]


def measure_batched_gpu(model: nn.Module, act_cache, target_names: set[str], specs: list[fr.FormatSpec],
                        device: str, dtype: torch.dtype, chunk_size: int = 256, h_detail=None,
                        _per_linear: bool = False) -> dict:
    """measure_quant_cost.py:551-685 with the weight error from the fused sweep.  `_per_linear`
    (used by measure_unbatched) quantizes with each spec's own quantize_dequantize instead."""
    dev = torch.device(device)
    groups = _group_by_shape(model, target_names)
    accum: dict = {}
    processed, t0 = 0, time.time()
    total = sum(len(v) for v in groups.values())
    # Results stay on the device until the end and come back in one copy (the GPU never waits for
    # the host in between); entries are replayed in processing order, errors included.
    pending: list = []
    dev_parts: list = []
    # memory budget for the fused W_hat slices, read once: cudaMemGetInfo waits for the device, so
    # a query per chunk would stop the host from queueing work ahead
    budget = torch.cuda.mem_get_info(dev)[0] // 4 if dev.type == "cuda" else 0

    def stash(t: torch.Tensor) -> int:
        dev_parts.append(t.detach().reshape(-1).to(torch.float64))
        return len(dev_parts) - 1

    for (_in_f, _out_f), entries in groups.items():
        entries = [(n, m) for n, m in entries if n in act_cache]
        for i in range(0, len(entries), chunk_size):
            chunk = entries[i:i + chunk_size]
            names = [n for n, _ in chunk]
            acts = [act_cache.load(n) for n in names]
            rows = min(a.size(0) for a in acts)
            # W_hat and weight_mse of the fused formats from one read of each weight, which also
            # stacks the weights; the reference's stack (measure_quant_cost.py:595-597) otherwise
            w_hat_pre, mse_pre, W = ({}, {}, None)
            if dtype == torch.bfloat16 and not _per_linear:
                w_hat_pre, mse_pre, W = _fused_w_hats_list([m.weight.detach() for _, m in chunk], specs, dev, budget)
            if W is None:
                W = torch.stack([m.weight.detach().to(device=dev, dtype=dtype) for _, m in chunk])
                if dtype == torch.bfloat16 and not _per_linear:
                    w_hat_pre, mse_pre = _fused_w_hats(W, specs, budget)
            X = torch.stack([a[:rows].to(device=dev, dtype=dtype) for a in acts])
            # tensor cores with fused epilogues for bf16 operands with k % 8 == 0: y_ref (bf16) and
            # its energy once per chunk (pq_output_ref), then one GEMM per format whose epilogue
            # reduces the error against it (pq_output_err); the bmm's otherwise
            fused_out = dtype == torch.bfloat16 and X.shape[-1] % 8 == 0 and rows > 0 and W.shape[1] > 0
            n_out = rows * W.shape[1]
            if fused_out:
                y_ref = torch.empty(W.shape[0], rows, W.shape[1], dtype=torch.bfloat16, device=dev)
                ref = torch.zeros(W.shape[0], dtype=torch.float64, device=dev)
                _lib.output_ref(X, W, ref, y_ref)
                ref_energy = ref / n_out
            else:
                y_ref = torch.bmm(X, W.transpose(1, 2))
                ref_energy = y_ref.float().pow(2).mean(dim=(1, 2))
            h_stacked = None
            if h_detail is not None and all(n in h_detail for n in names):
                hs = [h_detail.load(n) for n in names]
                if all(tuple(h.shape) == tuple(W.shape[1:]) for h in hs):
                    h_stacked = torch.stack([h.to(dev).float() for h in hs])
            wmse = None
            mse_dev = {sname: (stash(t), per) for sname, (t, per) in mse_pre.items()}
            if dtype == torch.bfloat16:
                rest = [s for s in specs if s.name not in mse_pre]
                wmse = (_weight_mse_or_errors(list(W.unbind(0)), rest, _per_linear) if rest
                        else [{} for _ in names])
            dl_pre = (_fused_predicted_dloss(W, specs, h_stacked)
                      if h_stacked is not None and dtype == torch.bfloat16 and not _per_linear else {})
            for spec in specs:
                try:
                    if wmse is None and spec.weight_element_dtype != "bfloat16":
                        raise NotImplementedError(f"B200 cost kernels take bf16 weights, got {dtype}")
                    W_hat = w_hat_pre.get(spec.name)
                    if W_hat is None and not _per_linear and batched_kernel_format(spec) == "BF16":
                        W_hat = W   # the reference's clone (measure_quant_cost.py:544-545) is only read here
                    if W_hat is None:
                        W_hat = spec.quantize_dequantize(W) if _per_linear else _batched_quantize(spec, W)
                    X_hat = spec.activation_quantize_dequantize(X.clone())
                    if fused_out:
                        err = torch.zeros(W.shape[0], dtype=torch.float64, device=dev)
                        _lib.output_err(X_hat, W_hat, y_ref, err)
                        out_mse = err / n_out
                    else:
                        y_q = torch.bmm(X_hat, W_hat.transpose(1, 2))
                        out_mse = (y_ref - y_q).float().pow(2).mean(dim=(1, 2))
                    rel = out_mse / ref_energy.clamp_min(1e-12)
                    dl = None
                    if h_stacked is not None:   # 0.5 * sum(H * err^2) per Linear (measure_quant_cost.py:638-640)
                        dl = dl_pre.get(spec.name)
                        if dl is None:
                            dl = _predicted_dloss(W, spec, h_stacked, per_row=False, per_linear=_per_linear)
                    if spec.name in mse_dev:
                        wm = mse_dev[spec.name]
                    else:
                        wm = [0.0 if wmse is None else wmse[j][spec.name] for j in range(len(names))]
                        for v in wm:
                            if isinstance(v, dict):
                                raise ValueError(v["error"])
                    pending.append((names, spec.name, wm, stash(out_mse), stash(rel), dl))
                except Exception as e:  # measure_quant_cost.py:673-675
                    pending.append((names, spec.name, str(e)))
            processed += len(chunk)
            if processed % (chunk_size * 4) == 0 or processed == total:
                print(f"[cost] {processed}/{total} ({time.time() - t0:.1f}s)", flush=True)
    host = torch.cat(dev_parts).cpu() if dev_parts else None   # the one device->host copy
    _lib.raise_on_device_error("measure_batched_gpu")
    offs = [0]
    for t in dev_parts:
        offs.append(offs[-1] + t.numel())
    part = lambda i: host[offs[i]:offs[i + 1]].tolist()
    for rec in pending:
        if len(rec) == 3:
            names, sname, msg = rec
            for name in names:
                accum.setdefault(name, {})[sname] = {"error": msg}
            continue
        names, sname, wm, i_om, i_rl, dl = rec
        if isinstance(wm, tuple):   # device sums of the fused formats
            sums, per = part(wm[0]), wm[1]
            wm = [_mse_from_sse(v, per) for v in sums]
        om, rl = part(i_om), part(i_rl)
        for j, name in enumerate(names):
            _accumulate_result(accum, name, sname, float(wm[j]), float(om[j]), float(rl[j]),
                               predicted_dloss=None if dl is None else float(dl[j]))
    return _finalize_results(accum)


def measure_unbatched(model: nn.Module, act_cache, target_names: set[str], specs: list[fr.FormatSpec],
                      device: str, dtype: torch.dtype, h_detail=None) -> dict:
    """measure_quant_cost.py:266-327: one Linear at a time, each spec's own quantize_dequantize."""
    accum: dict = {}
    for name, mod in model.named_modules():
        cname = canonical_linear_name(name)
        if not isinstance(mod, nn.Linear) or cname not in target_names or cname not in act_cache:
            continue
        sub = nn.Module()
        sub.add_module("lin", mod)
        one = measure_batched_gpu(sub, _Renamed(act_cache, cname), {"lin"}, specs, device, dtype, 1,
                                  _Renamed(h_detail, cname) if h_detail is not None else None, _per_linear=True)
        for fmt, entry in one.get("lin", {}).items():
            if "error" in entry:
                accum.setdefault(cname, {})[fmt] = entry
            else:
                _accumulate_result(accum, cname, fmt, entry["weight_mse"], entry["output_mse"],
                                   entry["rel_output_mse"], entry.get("predicted_dloss"))
    return _finalize_results(accum)


class _Renamed:
    def __init__(self, index, real_name):
        self.index, self.real = index, real_name

    def __contains__(self, name):
        return self.real in self.index

    def load(self, name):
        return self.index.load(self.real)


_PACKED_EXPERT_PARAM_NAMES = {"gate_up_proj", "down_proj", "w1", "w2", "w3", "gate_proj", "up_proj"}


def _is_packed_experts_module(module: nn.Module) -> bool:
    """sensitivity_probe.py:507-530: class name contains "expert" and it owns a
    3-D parameter with a known packed-expert name."""
    if "expert" not in type(module).__name__.lower():
        return False
    return any(p.dim() == 3 and n in _PACKED_EXPERT_PARAM_NAMES for n, p in module.named_parameters(recurse=False))


def _packed_experts_param_names(module: nn.Module) -> list[str]:
    return sorted(n for n, p in module.named_parameters(recurse=False)
                  if p.dim() == 3 and n in _PACKED_EXPERT_PARAM_NAMES)


def _enumerate_packed_experts(model: nn.Module, target_names: set[str]):
    out = []
    for qname, mod in model.named_modules():
        if not _is_packed_experts_module(mod):
            continue
        for pn in _packed_experts_param_names(mod):
            full = f"{qname}.{pn}" if qname else pn
            if full in target_names:
                out.append((full, getattr(mod, pn)))
    return out


def _measure_packed_experts(model: nn.Module, target_names: set[str], specs: list[fr.FormatSpec], device: str,
                            dtype: torch.dtype, accum: dict, h_detail=None) -> None:
    """measure_quant_cost.py:381-449: weight_mse of every packed [E, M, N]
    parameter for every spec in one fused pass (output_mse recorded as 0)."""
    dev = torch.device(device)
    entries = _enumerate_packed_experts(model, target_names)
    if not entries:
        return
    ws = [p.detach().to(device=dev, dtype=dtype) for _, p in entries]
    res = sweep_weight_mse([(n, w) for (n, _), w in zip(entries, ws)], specs)
    for (name, _), w in zip(entries, ws):
        h_em = None
        if h_detail is not None and name in h_detail:
            h = h_detail.load(name).to(dev).float()
            if tuple(h.shape) == (w.size(0), w.size(1)):
                h_em = h
        dl_pre = (_fused_predicted_dloss(w.unsqueeze(0), specs, h_em.unsqueeze(0), per_row=True)
                  if h_em is not None and dtype == torch.bfloat16 else {})
        for spec in specs:
            v = res[name][spec.name]
            if isinstance(v, dict):
                accum.setdefault(name, {})[spec.name] = v
                continue
            dl = None
            if h_em is not None:   # 0.5 * N * sum(H_em * mean_n err^2) (measure_quant_cost.py:430-437)
                dl = dl_pre[spec.name][0] if spec.name in dl_pre else \
                    _predicted_dloss(w.unsqueeze(0), spec, h_em.unsqueeze(0), per_row=True, per_linear=False)[0]
            _accumulate_result(accum, name, spec.name, float(v), 0.0, 0.0, predicted_dloss=dl)


def measure_weight_costs(model: nn.Module, target_names: set[str], specs: list[fr.FormatSpec],
                         device: str = "cuda", dtype: torch.dtype = torch.bfloat16) -> dict:
    """Whole-model weight-error table in one fused pass: every target Linear
    and packed-expert tensor, every spec.  Entries carry weight_mse (what the
    allocator consumes when no predicted_dloss is present,
    allocator_candidates.py:120-131) and zero output_mse / rel_output_mse."""
    dev = torch.device(device)
    named = []
    for name, mod in model.named_modules():
        cname = canonical_linear_name(name)
        if isinstance(mod, nn.Linear) and cname in target_names:
            named.append((cname, mod.weight.detach().to(device=dev, dtype=dtype)))
    named += [(n, p.detach().to(device=dev, dtype=dtype)) for n, p in _enumerate_packed_experts(model, target_names)]
    res = sweep_weight_mse(named, specs)
    accum: dict = {}
    for name, per in res.items():
        for fmt, v in per.items():
            if isinstance(v, dict):
                accum.setdefault(name, {})[fmt] = v
            else:
                _accumulate_result(accum, name, fmt, float(v), 0.0, 0.0)
    return _finalize_results(accum)
