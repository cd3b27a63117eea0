"""Fisher-trace statistics on B200.

Drop-in for the hot path of prismaquant/sensitivity_probe.py:
  * `_GradNormCapture` (:413-504): identity forward; backward reduces the
    packed-expert weight gradient to sum(g^2) and the [E, M] channel diagonal
    with one HBM pass (pq_sumsq_rows) into DEVICE accumulators, where the
    reference syncs once per 1M-element chunk and copies [E, M] to the host
    every backward.
  * `install_packed_expert_hooks` (:555-728), same patching and metadata.
  * `FisherAccumulator` (:959-1241) with the per-token estimator
        h_trace_raw += sum_t ||x_t||^2 ||g_t||^2
    — forward hook keeps ||x_t||^2 (T floats) instead of X, backward hook
    reduces ||g_t||^2 against it — replacing grad_w = gy^T x followed by
    sum(grad_w^2) (:1115-1152).  It equals the reference when one token flows
    through each backward and is the per-token (diagonal-in-t) empirical
    Fisher otherwise.  Packed experts either keep the reference's weight-grad
    norm (`packed_estimator="grad_norm"`) or use the same per-token estimator
    over each expert's routed tokens (`packed_estimator="per_token"`).
All accumulators stay on the device; `finalize` does one device->host copy.
"""
from __future__ import annotations

import re
from collections import defaultdict
from pathlib import Path

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from .measure_quant_cost import _PACKED_EXPERT_PARAM_NAMES, _is_packed_experts_module, _packed_experts_param_names


def _device_acc(store: dict, name: str, device, shape=(1,), dtype=torch.float64) -> torch.Tensor:
    """Accumulator tensor for `name`; a prior python float in the dict is folded in."""
    cur = store.get(name)
    if isinstance(cur, torch.Tensor) and cur.device == device and cur.dtype == dtype and tuple(cur.shape) == tuple(shape):
        return cur
    t = torch.zeros(shape, dtype=dtype, device=device)
    if isinstance(cur, torch.Tensor):
        t += cur.to(device=device, dtype=dtype).reshape(shape)
    elif cur is not None:
        t += float(cur)
    store[name] = t
    return t


class _GradNormCapture(torch.autograd.Function):
    """sensitivity_probe.py:413-504.  Accumulators are device tensors: the
    scalar one a [1] float64 (float() of it gives the reference's number), the
    channel one [E, M] float32."""

    @staticmethod
    def forward(ctx, weight, name, scalar_accumulator, channel_accumulator, full_accumulator):
        ctx.name = name
        ctx.scalar_acc = scalar_accumulator
        ctx.channel_acc = channel_accumulator
        ctx.full_acc = full_accumulator
        return weight

    @staticmethod
    def backward(ctx, grad_output):
        if grad_output is None:
            return None, None, None, None, None
        g = grad_output.detach()
        total = _device_acc(ctx.scalar_acc, ctx.name, g.device)
        per_row = None
        if ctx.channel_acc is not None and g.dim() in (2, 3):
            per_row = _device_acc(ctx.channel_acc, ctx.name, g.device, tuple(g.shape[:-1]), torch.float32)
        if ctx.full_acc is not None and g.dim() >= 2:
            # the per-weight [E, M, N] accumulator (sensitivity_probe.py:486-503), kept on the
            # device (the reference streams each backward's gradient to a host copy); a
            # caller-provided tensor elsewhere is updated from a device copy
            cur = ctx.full_acc.get(ctx.name)
            if cur is None:
                cur = ctx.full_acc[ctx.name] = torch.zeros(g.shape, dtype=torch.float32, device=g.device)
            if cur.device == g.device and cur.is_contiguous():
                _lib.sumsq_rows_full(g, total, per_row, cur)
            else:
                tmp = cur.to(g.device).contiguous()
                _lib.sumsq_rows_full(g, total, per_row, tmp)
                cur.copy_(tmp)
        else:
            _lib.sumsq_rows(g, total, per_row)
        return None, None, None, None, None


class _TokenNormCapture(torch.autograd.Function):
    """Identity on a Linear's output y; backward adds sum_t xnorm[t] * ||dy_t||^2
    (and the token count) into `acc` without touching the gradient."""

    @staticmethod
    def forward(ctx, y, xnorm, acc):
        ctx.save_for_backward(xnorm)
        ctx.acc = acc
        return y.view_as(y)

    @staticmethod
    def backward(ctx, gy):
        (xnorm,) = ctx.saved_tensors
        _lib.tokennorm_dot(gy.detach().reshape(-1, gy.shape[-1]), xnorm, ctx.acc)
        return gy, None, None


_PATCH = "_prismaquant_packed_expert_patch"
_CHANNEL = "_prismaquant_packed_expert_channel_patch"
_FULL = "_prismaquant_packed_expert_full_patch"


def _packed_meta(qname: str, pn: str, p: torch.Tensor) -> dict:
    shape = tuple(p.shape)
    return {"h_trace_raw": 0.0, "h_w2_sum_raw": 0.0, "w_max_abs": None if p.is_meta else float(p.detach().abs().max()),
            "w_norm_sq": None if p.is_meta else float(p.detach().float().pow(2).sum()),
            "n_params": int(p.numel()), "in_features": int(shape[2]), "out_features": int(shape[1]),
            "num_experts": int(shape[0]), "n_tokens_seen": 0, "route_prob": None, "router_path": None,
            "expert_id": None, "_packed_experts_module": qname, "_packed_param": pn}


def install_packed_expert_hooks(model: nn.Module, accumulator: dict, channel_accumulator: dict | None = None,
                                full_accumulator: dict | None = None) -> dict[str, dict]:
    """Route every packed-experts parameter through _GradNormCapture
    (sensitivity_probe.py:555-728); idempotent re-binding of accumulators."""
    meta = {}
    for qname, module in model.named_modules():
        if not _is_packed_experts_module(module):
            continue
        names = _packed_experts_param_names(module)
        for pn in names:
            p = module._parameters.get(pn)
            if p is not None:
                meta[f"{qname}.{pn}" if qname else pn] = _packed_meta(qname, pn, p)
        already = hasattr(module, _PATCH)
        setattr(module, _PATCH, accumulator)
        setattr(module, _CHANNEL, channel_accumulator)
        setattr(module, _FULL, full_accumulator)
        if already:
            continue
        for pn in names:
            getattr(module, pn).requires_grad_(True)
        original = module.forward
        fulls = [f"{qname}.{pn}" if qname else pn for pn in names]

        def patched(*args, _ns=tuple(names), _full=tuple(fulls), _orig=original, _mod=module, **kwargs):
            acc = getattr(_mod, _PATCH, None)
            if acc is None:
                return _orig(*args, **kwargs)
            ch, fu = getattr(_mod, _CHANNEL, None), getattr(_mod, _FULL, None)
            saved = {}
            for pn, fn in zip(_ns, _full):
                saved[pn] = _mod._parameters.pop(pn)
                _mod.__dict__[pn] = _GradNormCapture.apply(saved[pn], fn, acc, ch, fu)
            try:
                return _orig(*args, **kwargs)
            finally:
                for pn in _ns:
                    _mod.__dict__.pop(pn, None)
                    _mod._parameters[pn] = saved[pn]

        module.forward = patched
    return meta


class _SegTokenNormCapture(torch.autograd.Function):
    """Identity on the row-stacked outputs of a routed packed projection (rows grouped by expert);
    backward adds, for every expert, sum over its rows of xnorm[token] * ||dy_row||^2 and its row
    count into acc [E, 2], in one launch (pq_tokennorm_dot_seg), without touching the gradient.
    `tok` empty: xnorm is already one value per row."""

    @staticmethod
    def forward(ctx, y, xnorm, tok, seg, acc):
        ctx.save_for_backward(xnorm, tok, seg)
        ctx.acc = acc
        return y.view_as(y)

    @staticmethod
    def backward(ctx, gy):
        xnorm, tok, seg = ctx.saved_tensors
        _lib.tokennorm_dot_seg(gy.detach().reshape(-1, gy.shape[-1]), xnorm, seg, ctx.acc,
                               token_idx=tok if tok.numel() else None)
        return gy, None, None, None, None


def install_routed_expert_hooks(model: nn.Module, accumulator: dict) -> dict[str, dict]:
    """Per-token estimator for packed experts with gate_up_proj [E, 2I, H] / down_proj [E, H, I]
    (HF Qwen3MoeExperts layout), the reference's per-expert loop (sensitivity_probe.py:555-728)
    with its Fisher capture fused: the experts forward keeps the model's own arithmetic (one GEMM
    per hit expert, act(gate) * up, routing-weighted index_add in expert order, so its output is
    bit-identical), but each projection's outputs are stacked by expert and captured ONCE: the
    forward takes ||x_t||^2 of every token (pq_rownorm2) and ||h_r||^2 of every routed row, and
    the backward runs one pq_tokennorm_dot_seg launch per projection that adds, for each expert,
    sum over its routed tokens of ||x_t||^2 ||g_{t,e}||^2.  accumulator[name] is a [E, 2]
    float64 device tensor (trace, tokens) per packed parameter."""
    meta = {}
    for qname, module in model.named_modules():
        if not _is_packed_experts_module(module):
            continue
        if not (hasattr(module, "gate_up_proj") and hasattr(module, "down_proj") and hasattr(module, "act_fn")):
            continue
        gu_name, dn_name = f"{qname}.gate_up_proj", f"{qname}.down_proj"
        for pn in ("gate_up_proj", "down_proj"):
            meta[f"{qname}.{pn}"] = _packed_meta(qname, pn, getattr(module, pn))
        E = module.gate_up_proj.shape[0]
        dev = module.gate_up_proj.device
        acc_gu = _device_acc(accumulator, gu_name, dev, (E, 2))
        acc_dn = _device_acc(accumulator, dn_name, dev, (E, 2))

        def routed(hidden_states, top_k_index, top_k_weights, _m=module, _gu=acc_gu, _dn=acc_dn):
            final = torch.zeros_like(hidden_states)
            with torch.no_grad():
                mask = F.one_hot(top_k_index, num_classes=_m.gate_up_proj.shape[0]).permute(2, 1, 0)
                hit = torch.greater(mask.sum(dim=(-1, -2)), 0).nonzero()
            experts = hit.flatten().tolist()
            if not experts:
                return final
            toks, poss = [], []
            for e in experts:
                p_, t_ = torch.where(mask[e])
                poss.append(p_)
                toks.append(t_)
            sizes = [t.numel() for t in toks]
            tok, pos = torch.cat(toks), torch.cat(poss)
            seg = torch.repeat_interleave(torch.tensor(experts, dtype=torch.int32, device=tok.device),
                                          torch.tensor(sizes, device=tok.device))
            xn = _lib.rownorm2(hidden_states.detach())
            gu = torch.cat([F.linear(hidden_states[t], _m.gate_up_proj[e]) for e, t in zip(experts, toks)])
            gu = _SegTokenNormCapture.apply(gu, xn, tok, seg, _gu)
            gate, up = gu.chunk(2, dim=-1)
            h = _m.act_fn(gate) * up
            hn = _lib.rownorm2(h.detach())
            dn = torch.cat([F.linear(he, _m.down_proj[e]) for e, he in zip(experts, torch.split(h, sizes))])
            dn = _SegTokenNormCapture.apply(dn, hn, tok.new_empty(0), seg, _dn)
            dn = dn * top_k_weights[tok, pos, None]
            for t_, o in zip(toks, torch.split(dn, sizes)):
                final.index_add_(0, t_, o.to(final.dtype))
            return final

        module.forward = routed
    return meta


class FisherAccumulator:
    """sensitivity_probe.py:959-1241 with the per-token estimator and device accumulators.

    With `h_detail_dir`, every backward of a tracked Linear also forms the reference's per-weight
    Fisher diagonal on the tensor cores (pq_grad_sq_acc: grad_w = bf16(gy^T x), h_full +=
    bf16(grad_w^2)), so the Linear's stats are the reference's exact ones (h_trace_raw = the sum
    over backwards of bf16(sum grad_w^2), h_w2_sum_raw likewise with bf16(w^2)) rather than the
    per-token estimate, and finalize writes the reference's h_detail files (sensitivity_probe.py:
    1114-1152, 1200-1235) for measure_quant_cost's predicted_dloss."""

    def __init__(self, model: nn.Module, tracked: list[str], expert_info: dict[str, tuple[str, str]],
                 act_cache_dir: Path | None = None, input_rows: int = 256, hook_packed_experts: bool = True,
                 h_detail_dir: Path | None = None, packed_estimator: str = "grad_norm",
                 estimator: str | None = None):
        """`estimator` picks the dense Linears' statistic: "exact" is the reference's own (each
        backward forms grad_w on the tensor cores and keeps the per-weight diagonal on the device;
        the files are written only with `h_detail_dir`), "per_token" the per-token estimate.  The
        default is "exact" with `h_detail_dir` and "per_token" without."""
        self.h_detail_dir = Path(h_detail_dir) if h_detail_dir else None
        if estimator is None:
            estimator = "exact" if self.h_detail_dir is not None else "per_token"
        if estimator not in ("exact", "per_token"):
            raise ValueError(f"unknown estimator {estimator!r}")
        self.estimator = estimator
        self._detail = estimator == "exact"
        self._saved_inputs: dict[str, torch.Tensor] = {}
        self._h_full: dict[str, torch.Tensor] = {}
        self.stats: dict[str, dict] = {}
        self.tracked = set(tracked)
        self.expert_info = expert_info
        self.cache_dir = Path(act_cache_dir) if act_cache_dir else None
        self.input_rows = input_rows
        self._fwd_handles, self._bwd_handles = [], []
        self._xnorm: dict[str, torch.Tensor] = {}
        self._input_snaps: dict[str, list[torch.Tensor]] = defaultdict(list)
        self._rows_got: dict[str, int] = defaultdict(int)
        self._packed_grad_acc: dict = {}
        self._h_packed_channel: dict = {}
        self._packed_sample_count: dict[str, torch.Tensor] = {}
        self._names: list[str] = []
        lin = [(n, m) for n, m in model.named_modules() if n in self.tracked and isinstance(m, nn.Linear)]
        dev = lin[0][1].weight.device if lin else torch.device("cuda")
        # one [n, 2] fp64 accumulator (raw trace, tokens) per tracked Linear
        self._acc = torch.zeros(len(lin), 2, dtype=torch.float64, device=dev)
        if self._detail:
            odd = [n for n, m in lin if m.in_features % 8 or m.out_features % 8]
            if odd:
                raise NotImplementedError(f"per-weight Fisher detail needs in/out features that are multiples of 8: {odd}")
            # (trace, w^2 sum) per Linear, each backward's sums rounded to bf16 as the reference's
            # .sum() of a bf16 tensor returns them; and one scratch pair per backward
            self._exact = torch.zeros(len(lin), 2, dtype=torch.float64, device=dev)
            self._call_sums = torch.zeros(2, dtype=torch.float64, device=dev)
        wstats = []
        for i, (name, mod) in enumerate(lin):
            self._names.append(name)
            router, eid = expert_info.get(name, (None, None))
            w = mod.weight.detach()
            wstats.append(torch.stack([w.abs().max().float(), w.float().pow(2).sum()]))
            self.stats[name] = {"h_trace_raw": 0.0, "h_w2_sum_raw": 0.0, "w_max_abs": None, "w_norm_sq": None,
                                "n_params": int(w.numel()), "in_features": mod.in_features,
                                "out_features": mod.out_features, "n_tokens_seen": 0, "route_prob": None,
                                "router_path": router, "expert_id": eid}
            self._fwd_handles.append(mod.register_forward_hook(self._make_fwd(name)))
            self._bwd_handles.append(mod.register_full_backward_hook(self._make_bwd(name, i, mod)))
        if wstats:
            host = torch.stack(wstats).cpu().tolist()   # one sync for every Linear's weight stats
            for (name, _), (mx, n2) in zip(lin, host):
                self.stats[name]["w_max_abs"], self.stats[name]["w_norm_sq"] = mx, n2
        self.packed_estimator = packed_estimator
        if hook_packed_experts:
            if packed_estimator == "grad_norm":
                meta = install_packed_expert_hooks(model, self._packed_grad_acc, self._h_packed_channel)
            elif packed_estimator == "per_token":
                meta = install_routed_expert_hooks(model, self._packed_grad_acc)
            else:
                raise ValueError(f"unknown packed_estimator {packed_estimator!r}")
            for full, m in meta.items():
                qn = m.pop("_packed_experts_module")
                m.pop("_packed_param", None)
                layer = ".".join(qn.split(".")[:3])
                if any(t.startswith(layer + ".") for t in self.tracked):
                    self.stats[full] = m
                    mod = model.get_submodule(qn)
                    cnt = self._packed_sample_count.setdefault(
                        full, torch.zeros(1, dtype=torch.int64, device=dev))

                    def _exp_fwd(_m, inp, _out, _c=cnt):
                        x = inp[0] if isinstance(inp, tuple) else inp
                        if isinstance(x, torch.Tensor):
                            _c += x.reshape(-1, x.size(-1)).size(0)
                    self._fwd_handles.append(mod.register_forward_hook(_exp_fwd))

    def _make_fwd(self, name: str):
        def hook(module, inp, out):
            x = inp[0] if isinstance(inp, tuple) else inp
            x2 = x.detach().reshape(-1, x.size(-1))
            if self._detail:
                self._saved_inputs[name] = x2   # the reference's saved input (:1094)
            else:
                self._xnorm[name] = _lib.rownorm2(x2)
            if self.cache_dir is not None:
                need = self.input_rows - self._rows_got[name]
                if need > 0:
                    flat = x2
                    if flat.size(0) > need:
                        flat = flat.index_select(0, torch.randperm(flat.size(0), device=flat.device)[:need])
                    self._input_snaps[name].append(flat.to("cpu"))
                    self._rows_got[name] += flat.size(0)
        return hook

    def _make_bwd(self, name: str, idx: int, mod: nn.Linear):
        def hook(module, grad_input, grad_output):
            gy = grad_output[0]
            if self._detail:
                x2 = self._saved_inputs.pop(name, None)
                if x2 is None or gy is None:
                    return
                gy2 = gy.reshape(-1, gy.size(-1))
                h = self._h_full.get(name)
                if h is None:
                    h = self._h_full[name] = torch.zeros(mod.out_features, mod.in_features, dtype=torch.float32,
                                                         device=gy2.device)
                w = mod.weight
                wd = w.detach() if (w is not None and not w.is_meta) else None
                self._call_sums.zero_()
                _lib.grad_sq_acc(gy2, x2, h, self._call_sums, wd)
                self._exact[idx] += self._call_sums.float().to(torch.bfloat16).double()
                self._acc[idx, 1] += gy2.size(0)
                return
            xn = self._xnorm.pop(name, None)
            if xn is None or gy is None:
                return
            _lib.tokennorm_dot(gy.reshape(-1, gy.size(-1)), xn, self._acc[idx])
        return hook

    @property
    def trace_buffer(self) -> torch.Tensor:
        """[n_linears, 2] float64 (raw trace, tokens): what a data-parallel run all-reduces."""
        return self._acc

    def finalize(self, tracker=None):
        host = self._acc.cpu().tolist()
        exact = self._exact.cpu().tolist() if self._detail else [None] * len(host)
        for name, (tr, tok), ex in zip(self._names, host, exact):
            if ex is not None:   # the reference's exact statistics
                self.stats[name]["h_trace_raw"] += ex[0]
                self.stats[name]["h_w2_sum_raw"] += ex[1]
            else:
                self.stats[name]["h_trace_raw"] += tr
            self.stats[name]["n_tokens_seen"] += int(round(tok))
        for full, raw in self._packed_grad_acc.items():
            if full not in self.stats:
                continue
            if isinstance(raw, torch.Tensor) and raw.dim() == 2:   # per-token routed [E, 2]
                self.stats[full]["h_trace_raw"] += float(raw[:, 0].sum())
                self.stats[full]["expert_trace_raw"] = raw[:, 0].cpu().tolist()
            else:
                self.stats[full]["h_trace_raw"] += float(raw)
            self.stats[full]["n_tokens_seen"] = int(self._packed_sample_count.get(full, torch.zeros(1)).item())
        if tracker is not None:
            for s in self.stats.values():
                if s["router_path"]:
                    s["route_prob"] = tracker.prob(s["router_path"], s["expert_id"])
        for s in self.stats.values():
            tokens = max(s["n_tokens_seen"], 1)
            rp = s["route_prob"]
            div = tokens * rp if (rp is not None and rp > 0) else tokens
            s["h_trace"] = s["h_trace_raw"] / div
            s["h_w2_sum"] = s["h_w2_sum_raw"] / div
        if self.cache_dir is not None:
            self.cache_dir.mkdir(parents=True, exist_ok=True)
            for name, snaps in self._input_snaps.items():
                if snaps:
                    X = torch.cat(snaps).to(torch.bfloat16).contiguous()
                    torch.save({"inputs": X, "name": name},
                               self.cache_dir / (re.sub(r"[^A-Za-z0-9_-]", "__", name) + ".pt"))
        if self.h_detail_dir is not None:   # sensitivity_probe.py:1200-1235, the same files and keys
            self.h_detail_dir.mkdir(parents=True, exist_ok=True)
            sub = re.compile(r"[^A-Za-z0-9_-]")
            for name, acc in self._h_full.items():
                if name not in self.stats:
                    continue
                tokens = max(self.stats[name]["n_tokens_seen"], 1)
                rp = self.stats[name].get("route_prob")
                h = acc.to(torch.float32).cpu() / (tokens * rp if (rp is not None and rp > 0) else tokens)
                fname = sub.sub("__", name) + ".pt"
                torch.save({"h_diag": h, "name": name, "kind": "linear", "shape": list(h.shape)},
                           self.h_detail_dir / fname)
                self.stats[name]["h_detail_path"] = fname
            for full_name, ch in self._h_packed_channel.items():
                if full_name not in self.stats:
                    continue
                tokens = max(self.stats[full_name]["n_tokens_seen"], 1)
                h = ch.to(torch.float32).cpu() / tokens
                fname = sub.sub("__", full_name) + ".pt"
                torch.save({"h_diag": h, "name": full_name, "kind": "packed", "shape": list(h.shape)},
                           self.h_detail_dir / fname)
                self.stats[full_name]["h_detail_path"] = fname

    def remove_hooks(self):
        for h in self._fwd_handles + self._bwd_handles:
            h.remove()
        self._fwd_handles.clear()
        self._bwd_handles.clear()


def probe_pass(model: nn.Module, calib: torch.Tensor, tracked: list[str], batch_size: int = 1,
               acc: FisherAccumulator | None = None, all_reduce=None) -> FisherAccumulator:
    """The probe loop of run_probe_pass (sensitivity_probe.py:1509-1576): per
    batch of calibration sequences, sum-reduced next-token cross entropy and
    one backward; the hooks accumulate on the device.  `all_reduce`, if
    given, is called on the trace buffer before finalize (data parallel)."""
    if acc is None:
        acc = FisherAccumulator(model, tracked, {})
    model.train()
    emb = model.get_input_embeddings()
    for i in range(0, calib.size(0), batch_size):
        ids = calib[i:i + batch_size].to(emb.weight.device)
        with torch.no_grad():
            e = emb(ids)
        e.requires_grad_(True)
        logits = model(inputs_embeds=e).logits
        lp = F.log_softmax(logits[:, :-1].reshape(-1, logits.size(-1)).float(), dim=-1)
        loss = -lp.gather(1, ids[:, 1:].reshape(-1, 1)).sum()
        loss.backward()
        acc._xnorm.clear()
        acc._saved_inputs.clear()
    if all_reduce is not None:
        all_reduce(acc.trace_buffer)
    return acc


def make_layer_fisher_hooks(saved_inputs: dict, acc_stats: dict, acc_h_full: dict | None):
    """Drop-in for the per-layer hook pair of the production probe's whole-batch backward
    (incremental_probe.py:1222-1262, `make_fwd` / `make_bwd`): returns (make_fwd, make_bwd) with
    the same closures' contract, computed on the tensor cores.

      make_fwd(name)          forward hook: keeps the Linear's input in `saved_inputs[name]`
      make_bwd(name, module)  backward hook: pops it and, with grad_w = bf16(gy^T x) and
                              g2 = bf16(grad_w^2) formed by pq_grad_sq_acc (never stored),
                              adds bf16(sum g2) to acc_stats[name]["h_trace_raw"],
                              bf16(sum bf16(g2 * bf16(w^2))) to "h_w2_sum_raw", the row count to
                              "n_tokens_seen", and, when `acc_h_full` is a dict, g2 into
                              acc_h_full[name] (fp32 [out, in], created on the host as the
                              reference does, or used where the caller put it).

    The activation-snapshot side of the reference's forward hook is the caller's (it is not on
    the Fisher path); chain it before this one if it is needed."""
    scratch: dict[tuple, torch.Tensor] = {}

    def make_fwd(name: str):
        def hook(module, inp, out):
            x = inp[0] if isinstance(inp, tuple) else inp
            saved_inputs[name] = x.detach()
        return hook

    def make_bwd(name: str, mod_ref: nn.Module):
        def hook(module, grad_input, grad_output):
            gy = grad_output[0]
            x = saved_inputs.pop(name, None)
            if x is None or gy is None:
                return
            gy2 = gy.reshape(-1, gy.size(-1))
            x2 = x.reshape(-1, x.size(-1))
            m, n = gy2.size(1), x2.size(1)
            key = (gy2.device, m, n)
            h = scratch.get(key)
            if h is None:
                h = scratch[key] = torch.empty(m, n, dtype=torch.float32, device=gy2.device)
            h.zero_()
            sums = torch.zeros(2, dtype=torch.float64, device=gy2.device)
            w = getattr(mod_ref, "weight", None)
            wd = w.detach() if (w is not None and not w.is_meta) else None
            _lib.grad_sq_acc(gy2, x2, h, sums, wd)
            if acc_h_full is not None:
                acc = acc_h_full.get(name)
                if acc is None:
                    acc = acc_h_full[name] = torch.zeros(m, n, dtype=torch.float32, device="cpu")
                acc.add_(h.to(acc.device))
            s = sums.float().to(torch.bfloat16).double().cpu().tolist()   # .sum() of a bf16 tensor is bf16
            st = acc_stats[name]
            st["h_trace_raw"] += s[0]
            if wd is not None:
                st["h_w2_sum_raw"] += s[1]
            st["n_tokens_seen"] += x2.size(0)
        return hook

    return make_fwd, make_bwd


def run_probe_pass(model: nn.Module, tokenizer, calib: torch.Tensor, model_name: str, dataset_name: str,
                   seqlen: int, dtype_name: str, requested_device: str, load_device_map, exec_device,
                   linear_include: str, linear_exclude: str, importance_weighting: bool,
                   activation_cache_dir: str | None, output_path: str, h_detail_dir: str | None = None,
                   *, expert_info: dict | None = None, tracker=None, top_k: int | None = None,
                   estimator: str = "exact") -> FisherAccumulator:
    """sensitivity_probe.py:1456-1590 with the same arguments and the same pickle: every Linear
    matching `linear_include` and not `linear_exclude` is tracked; one sequence per backward under
    the sum-reduced next-token cross entropy (optionally importance-weighted per token, weights
    clamped to [0.25, 4] around their mean); the statistics come from this package's
    FisherAccumulator (`estimator="exact"`: the reference's own numbers, on the tensor cores).

    Router bookkeeping of ModuleList MoE models (the reference's discover_moe_structure /
    RouterTracker) is model-structure code outside this path: pass `expert_info`, `tracker` (an
    object with .prob(router, expert), .counts, .total_tokens and .remove_hooks()) and `top_k`
    to have route_prob filled in; a dense model needs none of them."""
    import pickle
    import time

    inc, exc = re.compile(linear_include), re.compile(linear_exclude)
    tracked = [n for n, m in model.named_modules() if isinstance(m, nn.Linear) and inc.search(n) and not exc.search(n)]
    print(f"[probe] tracking {len(tracked)} Linear layers", flush=True)
    expert_info = {k: v for k, v in (expert_info or {}).items() if k in tracked}
    cache_dir = Path(activation_cache_dir) if activation_cache_dir else None
    acc = FisherAccumulator(model, tracked, expert_info, cache_dir,
                            h_detail_dir=Path(h_detail_dir) if h_detail_dir else None, estimator=estimator)
    model.train()
    emb = model.get_input_embeddings()
    t_fwd = t_bwd = 0.0
    for i in range(calib.size(0)):
        ids = calib[i:i + 1].to(exec_device)
        t0 = time.time()
        with torch.no_grad():
            e = emb(ids)
        e.requires_grad_(True)
        logits = model(inputs_embeds=e).logits
        t_fwd += time.time() - t0
        t0 = time.time()
        lp = F.log_softmax(logits[..., :-1, :].reshape(-1, logits.size(-1)), dim=-1)
        nll = -lp.gather(1, ids[..., 1:].reshape(-1, 1)).squeeze(1)
        if importance_weighting:
            with torch.no_grad():
                tok = F.cross_entropy(logits.detach()[..., :-1, :].reshape(-1, logits.size(-1)),
                                      ids[..., 1:].reshape(-1), reduction="none")
                wts = (tok / max(float(tok.mean().item()), 1e-6)).clamp(0.25, 4.0)
            loss = (nll * wts).sum()
        else:
            loss = nll.sum()
        loss.backward()
        t_bwd += time.time() - t0
        if (i + 1) % 4 == 0 or i == 0:
            print(f"[probe] sample {i + 1}/{calib.size(0)} loss={float(loss.detach()) / max(nll.numel(), 1):.3f} "
                  f"fwd_avg={t_fwd / (i + 1):.2f}s bwd_avg={t_bwd / (i + 1):.2f}s", flush=True)
        acc._saved_inputs.clear()
        acc._xnorm.clear()
    acc.finalize(tracker)
    acc.remove_hooks()
    if tracker is not None:
        tracker.remove_hooks()
    out = Path(output_path)
    out.parent.mkdir(parents=True, exist_ok=True)
    with open(out, "wb") as f:
        pickle.dump({"stats": acc.stats,
                     "router_counts": dict(tracker.counts) if tracker else {},
                     "router_totals": dict(tracker.total_tokens) if tracker else {},
                     "expert_info": expert_info,
                     "meta": {"model": model_name, "dataset": dataset_name, "nsamples": calib.size(0),
                              "seqlen": seqlen, "dtype": dtype_name, "device_map": str(load_device_map),
                              "execution_device": str(exec_device), "top_k": top_k if top_k is not None else 2,
                              "importance_weighting": importance_weighting,
                              "activation_cache_dir": str(cache_dir) if cache_dir else None,
                              "linear_include": linear_include, "linear_exclude": linear_exclude}}, f)
    print(f"[probe] wrote {out}", flush=True)
    return acc
