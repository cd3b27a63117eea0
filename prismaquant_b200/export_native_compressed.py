"""NVFP4 / MXFP8 / FP8 packing into compressed-tensors layouts on B200.

Drop-in for the packing math of prismaquant/export_native_compressed.py:
  compute_nvfp4_global_real (:1045-1055), quantize_dequantize_nvfp4[_packed]
  (:1058-1129), quantize_dequantize_mxfp8[_packed] (:1135-1194),
  quantize_dequantize_fp8_dynamic[_packed] (:1197-1226), _quantize_2d NVFP4 /
  MXFP8 / BF16 branches (:1691-1896), _quantize_3d_packed and
  _quantize_2d_group_same_shape (:1930-1981), the fused-sibling joint global
  (:1577-1599, :1650-1685, :2036-2099).
Outputs have the reference's dtypes, shapes and bytes (bit-exact).

`export_nvfp4_many` and `sweep_and_export` are the batched forms: pass 1 (codes,
group amax, tensor amax) runs over every tensor, fused with the cost sweep
when asked, and one pass-2 launch writes every E4M3 block scale with the joint
global of each fused-sibling group.
"""
from __future__ import annotations

import re
from collections import defaultdict

import torch
import torch.nn as nn

from . import _lib
from . import measure_quant_cost as mqc
# the checkpoint's serving configuration, at the reference's module path
from .quantization_config import (SCHEMES as FORMAT_SCHEME, build_quantization_config,  # noqa: F401
                                  write_config_with_quantization)

FLOAT_TO_E2M1 = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
NVFP4_MAX = 6.0
FP8_E4M3_MAX = 448.0
MXFP8_E4M3_MAX = 448.0
DEFAULT_INPUT_GLOBAL_SCALE = 1.0


def _need_group(group_size: int, expected: int, fmt: str):
    if group_size != expected:
        raise NotImplementedError(f"{fmt} on B200 uses group_size={expected}, got {group_size}")


def compute_nvfp4_global_real(weight: torch.Tensor, group_size: int = 16) -> torch.Tensor:
    """(max over 16-groups of max(amax,1e-12)/6) / 448, clamped at 1e-12; the max of
    the rounded per-group quotients equals the quotient of the tensor amax.  A 0-d fp32
    tensor on the weight's device, as the reference returns."""
    _need_group(group_size, 16, "NVFP4")
    rows, cols = weight.shape
    if cols % group_size:
        raise ValueError(f"NVFP4 group_size={group_size} ∤ {cols}")
    return _lib.nvfp4_global_real(weight, 1)[0]   # one read, one kernel (pq_nvfp4_global_real)


def quantize_dequantize_nvfp4(weight: torch.Tensor, group_size: int = 16,
                              global_real_override: torch.Tensor | None = None):
    """(weight_packed u8 [rows, cols/2], weight_scale e4m3 [rows, cols/16],
    weight_global_scale f32 [1] = 1/global_real)."""
    _need_group(group_size, 16, "NVFP4")
    if weight.dim() != 2:
        raise ValueError(f"expected a 2-D weight, got {tuple(weight.shape)}")
    if weight.shape[1] % group_size:
        raise ValueError(f"NVFP4 group_size={group_size} ∤ {weight.shape[1]}")
    return _lib.nvfp4_pack(weight, override=global_real_override)


def quantize_dequantize_nvfp4_packed(packed: torch.Tensor, group_size: int = 16):
    """Per-expert globals: (u8 [E, M, N/2], e4m3 [E, M, N/16], f32 [E])."""
    _need_group(group_size, 16, "NVFP4")
    if packed.dim() != 3:
        raise ValueError(f"expected [E, M, N], got {tuple(packed.shape)}")
    if packed.shape[2] % group_size:
        raise ValueError(f"NVFP4 group_size={group_size} ∤ {packed.shape[2]}")
    return _lib.nvfp4_pack(packed)


def quantize_dequantize_mxfp8(weight: torch.Tensor, group_size: int = 32):
    _need_group(group_size, 32, "MXFP8")
    if weight.shape[-1] % group_size:
        raise ValueError(f"MXFP8 group_size={group_size} ∤ {weight.shape[-1]}")
    return _lib.mxfp8_pack(weight)


def quantize_dequantize_mxfp8_packed(packed: torch.Tensor, group_size: int = 32):
    _need_group(group_size, 32, "MXFP8")
    if packed.shape[-1] % group_size:
        raise ValueError(f"MXFP8 group_size={group_size} ∤ {packed.shape[-1]}")
    return _lib.mxfp8_pack(packed)


def quantize_dequantize_fp8_dynamic(weight: torch.Tensor):
    """(fp8 [out, in], fp32 per-channel scale [out, 1])."""
    return _lib.fp8_channel_pack(weight)


def quantize_dequantize_fp8_dynamic_packed(packed: torch.Tensor):
    """(fp8 [E, M, N], fp32 scale [E, M, 1])."""
    return _lib.fp8_channel_pack(packed)


def _canonical_export_format(fmt: str) -> str:
    return {"NVINT2": "INT2", "NVINT3": "INT3"}.get(fmt, fmt)


def _quantize_2d(weight: torch.Tensor, fmt: str, nvfp4_global_real_override: torch.Tensor | None = None,
                 input_global_scale_override: float | None = None, linear_name: str | None = None,
                 awq_enabled: bool = False, gptq_enabled: bool = False, awq_round_enabled: bool = False,
                 scale_sweep_enabled: bool = False, cached_activations: torch.Tensor | None = None):
    """On-disk tensors of one Linear (export_native_compressed.py:1691-1896), RTN only."""
    fmt = _canonical_export_format(fmt)
    if awq_enabled or gptq_enabled or awq_round_enabled or scale_sweep_enabled:
        raise NotImplementedError("activation-aware NVFP4 passes are not on the B200 path")
    if fmt == "NVFP4":
        wp, ws, wg = quantize_dequantize_nvfp4(weight, 16, nvfp4_global_real_override)
        scale = DEFAULT_INPUT_GLOBAL_SCALE if input_global_scale_override is None else input_global_scale_override
        return {"weight_packed": wp, "weight_scale": ws, "weight_global_scale": wg,
                "input_global_scale": torch.tensor([float(scale)], dtype=torch.float32, device=wp.device)}
    if fmt == "MXFP8":
        w, ws = quantize_dequantize_mxfp8(weight, 32)
        return {"weight": w, "weight_scale": ws}
    if fmt == "BF16":
        return {"weight": weight.to(torch.bfloat16)}
    raise ValueError(f"unsupported format: {fmt}")


def _quantize_3d_packed(packed: torch.Tensor, fmt: str):
    fmt = _canonical_export_format(fmt)
    if fmt == "BF16":
        return {"weight": packed.to(torch.bfloat16)}
    if fmt == "NVFP4":
        wp, ws, wg = quantize_dequantize_nvfp4_packed(packed, 16)
        return {"weight_packed": wp, "weight_scale": ws, "weight_global_scale": wg}
    if fmt == "MXFP8":
        w, ws = quantize_dequantize_mxfp8_packed(packed, 32)
        return {"weight": w, "weight_scale": ws}
    raise ValueError(f"unsupported format for packed-MoE: {fmt}")


def _quantize_2d_group_same_shape(stacked_weights: torch.Tensor, fmt: str):
    fmt = _canonical_export_format(fmt)
    if stacked_weights.dim() != 3:
        raise ValueError("same-shape export grouping expects [B, out, in] weights; "
                         f"got shape={tuple(stacked_weights.shape)}")
    if fmt == "MXFP8":
        w, ws = quantize_dequantize_mxfp8_packed(stacked_weights, 32)
        return {"weight": w, "weight_scale": ws}
    raise ValueError(f"unsupported grouped 2D export format: {fmt}")


# ---------------------------------------------------------------------------
# fused siblings (export_native_compressed.py:1577-1599, 2036-2099)
# ---------------------------------------------------------------------------
_FUSED_DENSE_PATTERNS = [
    (re.compile(r"^(?P<pre>.+)\.self_attn\.(?P<sib>q_proj|k_proj|v_proj)$"), ("q_proj", "k_proj", "v_proj")),
    (re.compile(r"^(?P<pre>.+)\.mlp\.(?P<sib>gate_proj|up_proj)$"), ("gate_proj", "up_proj")),
    (re.compile(r"^(?P<pre>.+)\.mlp\.shared_expert\.(?P<sib>gate_proj|up_proj)$"), ("gate_proj", "up_proj")),
    (re.compile(r"^(?P<pre>.+)\.linear_attn\.(?P<sib>in_proj_qkv|in_proj_z)$"), ("in_proj_qkv", "in_proj_z")),
    (re.compile(r"^(?P<pre>.+)\.linear_attn\.(?P<sib>in_proj_a|in_proj_b)$"), ("in_proj_a", "in_proj_b")),
]

_FUSED_SIBLINGS = {
    "q_proj": "qkv", "k_proj": "qkv", "v_proj": "qkv",
    "gate_proj": "gate_up", "up_proj": "gate_up",
    "in_proj_qkv": "qkvz", "in_proj_z": "qkvz",
    "in_proj_b": "ba", "in_proj_a": "ba",
}


def _fused_dense_group(name: str):
    for pat, members in _FUSED_DENSE_PATTERNS:
        m = pat.match(name)
        if m:
            return (m.group("pre"), members)
    return None


def sibling_group_key(name: str) -> str | None:
    """Key shared by the fused siblings of `name` (parent module + family), None if unfused."""
    parent, _, leaf = name.rpartition(".")
    fam = _FUSED_SIBLINGS.get(leaf)
    return None if fam is None else f"{parent}::{fam}"


def _compute_nvfp4_joint_global(model: nn.Module, assignment: dict[str, str]) -> dict[str, torch.Tensor]:
    groups = defaultdict(list)
    for qname, mod in model.named_modules():
        if isinstance(mod, nn.Linear) and assignment.get(qname) == "NVFP4":
            g = _fused_dense_group(qname)
            if g is not None:
                groups[g].append((qname, mod))
    out = {}
    for sib in groups.values():
        joint = torch.stack([compute_nvfp4_global_real(m.weight.detach()) for _, m in sib]).max()
        for q, _ in sib:
            out[q] = joint
    return out


def _compute_layer_joint_nvfp4(layer_mod: nn.Module, layer_qname: str, assignment: dict[str, str],
                               profile) -> dict[str, torch.Tensor]:
    groups = defaultdict(list)
    for sub, mod in layer_mod.named_modules():
        if not isinstance(mod, nn.Linear):
            continue
        fam = _FUSED_SIBLINGS.get(sub.rsplit(".", 1)[-1])
        if fam is None:
            continue
        parent = sub.rsplit(".", 1)[0] if "." in sub else ""
        groups[(parent, fam)].append((sub, mod))
    out = {}
    for members in groups.values():
        keyed = []
        for sub, mod in members:
            full = f"{layer_qname}.{sub}" if sub else layer_qname
            rk = profile.live_to_recipe_name(full)
            keyed.append((rk, assignment.get(rk), mod))
        if {f for _, f, _ in keyed} != {"NVFP4"}:
            continue
        joint = torch.stack([compute_nvfp4_global_real(m.weight.detach()) for _, _, m in keyed]).max()
        for rk, _, _ in keyed:
            out[rk] = joint
    return out


# ---------------------------------------------------------------------------
# batched export (+ fused cost sweep)
# ---------------------------------------------------------------------------

def _alloc_nvfp4(w: torch.Tensor):
    lead, cols = w.shape[:-1], w.shape[-1]
    dev = w.device
    return (torch.empty(*lead, cols // 2, dtype=torch.uint8, device=dev),
            torch.empty(*lead, cols // 16, dtype=torch.int16, device=dev))


def export_nvfp4_many(weights: list[torch.Tensor], group_keys: list[str | None] | None = None,
                      fuse_sweep_specs=None, sse: torch.Tensor | None = None):
    """NVFP4-export many 2-D bf16 CUDA weights; tensors with the same non-None
    group key share one joint global (fused siblings).

    With `fuse_sweep_specs`, pass 1 is the fused multi-format cost sweep (one
    read of each weight gives MSE_W for every spec AND the NVFP4 codes).
    Returns (outputs, sse, errors): outputs[i] = (weight_packed u8,
    weight_scale e4m3, weight_global_scale f32 [1])."""
    n = len(weights)
    ws = [_lib.as_bf16_cuda(w, "export_nvfp4_many") for w in weights]
    for w in ws:
        if w.dim() != 2 or w.shape[1] % 16:
            raise ValueError(f"NVFP4 export needs [rows, cols%16==0], got {tuple(w.shape)}")
    dev = ws[0].device
    codes, amax = zip(*[_alloc_nvfp4(w) for w in ws]) if n else ((), ())
    tmax = torch.zeros(n, dtype=torch.int32, device=dev)
    errors = None
    if fuse_sweep_specs is not None:
        outs = [(c, a, tmax[i:i + 1]) for i, (c, a) in enumerate(zip(codes, amax))]
        sse, errors = mqc.sweep_sse_async(ws, fuse_sweep_specs, nvfp4_outputs=outs, sse=sse)
    else:
        for i, w in enumerate(ws):
            _lib.nvfp4_codes(w, 1, codes[i], amax[i], tmax[i:i + 1])
    gdiv = torch.empty(n, dtype=torch.float32, device=dev)
    scales = [torch.empty(a.shape, dtype=torch.uint8, device=dev) for a in amax]
    ids: dict[str, int] = {}
    grp = [-1 if (group_keys is None or k is None) else ids.setdefault(k, len(ids)) for k in
           (group_keys or [None] * n)]
    step = 256
    for b0 in range(0, n, step):
        sl = slice(b0, min(n, b0 + step))
        sub_grp = grp[sl]
        # a joint group must not straddle launches: fall back to own-slice scope if it would
        if any(g >= 0 and (grp.count(g) != sub_grp.count(g)) for g in sub_grp):
            raise ValueError("fused-sibling groups must be adjacent within 256 tensors")
        _lib.nvfp4_scales(list(amax[sl]), tmax[sl], scales[sl], gdiv[sl], group_of=sub_grp)
    outputs = [(codes[i], scales[i].view(torch.float8_e4m3fn), gdiv[i:i + 1]) for i in range(n)]
    return outputs, sse, errors


def sweep_and_export(named_weights, specs, export_nvfp4: bool = True):
    """One pass over every weight: MSE_W for all `specs` (cost table) and,
    if `export_nvfp4`, the NVFP4 export of every tensor with fused-sibling
    joint globals.  Returns (cost dict {name: {fmt: weight_mse}}, {name: (packed, scale, global)})."""
    items = list(named_weights.items()) if isinstance(named_weights, dict) else list(named_weights)
    names = [n for n, _ in items]
    ws = [w for _, w in items]
    # NVFP4 / MXFP8 / FP8 per channel / BF16 ride on the export's read; the rest of the registry
    # (exact codebook / integer kernel, NVFP3's batched-path error) is a second, separate sweep
    fused = [s for s in specs if s.kernel_format in mqc._FUSED and s.name != "FP8_SOURCE"]
    rest = [s for s in specs if s not in fused]
    if export_nvfp4:
        outs, sse, errors = export_nvfp4_many(ws, [sibling_group_key(n) for n in names], fuse_sweep_specs=fused)
    else:
        sse, errors = mqc.sweep_sse_async([_lib.as_bf16_cuda(w, "sweep") for w in ws], fused)
        outs = None
    other = mqc.sweep_weight_mse(list(zip(names, ws)), rest) if rest else {}
    host = sse.cpu().tolist()
    costs = {}
    for name, w, row, err in zip(names, ws, host, errors):
        per = {}
        for s in specs:
            if s in rest:
                per[s.name] = other[name][s.name]
            else:
                per[s.name] = {"error": err[s.name]} if s.name in err else \
                    mqc._mse_from_sse(row[mqc._KCOL[mqc._kernel_format(s)]], w.numel())
        costs[name] = per
    return costs, (dict(zip(names, outs)) if outs is not None else None)


def _plan_chunks(sizes: list[int], keys: list[str | None], target: int) -> list[tuple[int, int]]:
    """[b0, b1) runs of tensors for a pipelined plan: up to `target` runs of about equal size, at
    most 256 tensors each, never cutting between two members of one fused-sibling group (wherever
    they sit in the list)."""
    n = len(sizes)
    first: dict[str, int] = {}
    last: dict[str, int] = {}
    for i, k in enumerate(keys):
        if k is not None:
            first.setdefault(k, i)
            last[k] = i
    blocked = set()
    for k in first:
        blocked.update(range(first[k] + 1, last[k] + 1))   # a cut before index p splits the group
    per = sum(sizes) / max(target, 1)
    chunks, b0, acc = [], 0, 0
    for i in range(n):
        acc += sizes[i]
        p = i + 1
        if p < n and p not in blocked and (acc >= per * (len(chunks) + 1) or p - b0 >= 256):
            chunks.append((b0, p))
            b0 = p
        elif p - b0 > 256:
            raise ValueError("a fused-sibling group spans more than 256 tensors")
    if b0 < n or not chunks:
        chunks.append((b0, n))
    return chunks


class SweepExportPlan:
    """Cost sweep (+ NVFP4 export) of a fixed set of device-resident bf16
    weights, planned once and run many times: the descriptor table, outputs
    and scratch are built at construction; `run()` is a memset plus two
    kernel launches (the fused sweep with NVFP4 codes, then the block-scale
    pass with fused-sibling joint globals) and no host synchronisation.

    After run(): `sse` [n, 4] fp64 holds sum(err^2) per (tensor, format),
    `outputs[i]` the NVFP4 (weight_packed, weight_scale, weight_global_scale).

    With the export and `pipeline_chunks` > 1 the tensors are cut into up to that many runs of
    about equal bytes (never inside a fused-sibling group, at most 256 tensors each): a chunk's
    scale pass runs on a side stream while the next chunk is swept (`launch_pipelined`), so only
    the last chunk's scale pass follows the sweep.  On the 8B model 4 chunks gain 0.3 % a step: the
    extra launches' tails and the scale passes sharing the SMs take most of the 0.31 ms the overlap
    hides, so the default is one chunk (runs of 256 tensors at most)."""

    def __init__(self, named_weights, specs, export_nvfp4: bool = True, pipeline_chunks: int = 1):
        import ctypes
        items = list(named_weights.items()) if isinstance(named_weights, dict) else list(named_weights)
        self.names = [n for n, _ in items]
        self.weights = [_lib.as_bf16_cuda(w, "SweepExportPlan") for _, w in items]
        self.specs = list(specs)
        self.numel = [w.numel() for w in self.weights]
        n = len(self.weights)
        dev = self.weights[0].device
        self.device = dev
        self.sse = torch.zeros(n, 4, dtype=torch.float64, device=dev)
        self.tmax = torch.zeros(max(n, 1), dtype=torch.int32, device=dev)
        kf = [mqc._kernel_format(s) for s in self.specs]
        if any(k not in mqc._FUSED or s.name == "FP8_SOURCE" for s, k in zip(self.specs, kf)):
            raise ValueError("SweepExportPlan takes the fused-sweep formats (NVFP4, MXFP8, FP8_E4M3, BF16 and "
                             "their aliases); use sweep_and_export for the rest of the registry")
        self.errors = []
        masks = []
        for w in self.weights:
            m, err = 0, {}
            for s, k in zip(self.specs, kf):
                e = mqc.shape_error(k, w.shape[-1])
                if e:
                    err[s.name] = e
                else:
                    m |= mqc._KBIT[k]
            masks.append(m & 0x7)
            self.errors.append(err)
        self.export = export_nvfp4
        self.codes, self.amax, self.scales = [], [], []
        arr = (_lib.SweepTensor * n)()
        for i, (w, m) in enumerate(zip(self.weights, masks)):
            cols = w.shape[-1]
            arr[i].w, arr[i].rows, arr[i].cols, arr[i].fmt_mask = w.data_ptr(), w.numel() // cols, cols, m
            if export_nvfp4:
                if w.dim() != 2 or cols % 16:
                    raise ValueError(f"NVFP4 export needs [rows, cols%16==0], got {tuple(w.shape)}")
                c, a = _alloc_nvfp4(w)
                self.codes.append(c)
                self.amax.append(a)
                self.scales.append(torch.empty(a.shape, dtype=torch.uint8, device=dev))
                arr[i].nvfp4_codes, arr[i].nvfp4_amax = c.data_ptr(), a.data_ptr()
                arr[i].nvfp4_tmax = self.tmax.data_ptr() + 4 * i
        self._arr = arr
        self._n = n
        self.gdiv = torch.empty(max(n, 1), dtype=torch.float32, device=dev)
        keys = [sibling_group_key(nm) for nm in self.names]
        self.chunks = _plan_chunks(self.numel, keys, pipeline_chunks if export_nvfp4 else 1)
        tsize = ctypes.sizeof(_lib.SweepTensor)
        self._sweep_calls = [(ctypes.cast(ctypes.addressof(arr) + b0 * tsize, ctypes.POINTER(_lib.SweepTensor)),
                              b1 - b0, self.sse.data_ptr() + 32 * b0) for b0, b1 in self.chunks]
        if export_nvfp4:
            ids: dict[str, int] = {}
            grp = [(-1 if k is None else ids.setdefault(k, len(ids))) for k in keys]
            self._scale_calls = []   # one per chunk: a fused-sibling group never straddles two
            for b0, b1 in self.chunks:
                sl = slice(b0, b1)
                A = (ctypes.c_void_p * (b1 - b0))(*[a.data_ptr() for a in self.amax[sl]])
                G = (ctypes.c_int64 * (b1 - b0))(*[a.numel() for a in self.amax[sl]])
                S = (ctypes.c_void_p * (b1 - b0))(*[s.data_ptr() for s in self.scales[sl]])
                Q = (ctypes.c_int32 * (b1 - b0))(*grp[sl])
                self._scale_calls.append((b1 - b0, A, G, S, Q, self.tmax.data_ptr() + 4 * b0,
                                          self.gdiv.data_ptr() + 4 * b0))
        self.outputs = [(self.codes[i], self.scales[i].view(torch.float8_e4m3fn), self.gdiv[i:i + 1])
                        for i in range(n)] if export_nvfp4 else None

    def launch_sweep(self):
        import ctypes
        lib = _lib.load()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        for arr, k, sse_ptr in self._sweep_calls:
            _lib._check(lib.pq_sweep_sse(arr, k, ctypes.c_void_p(sse_ptr), stream), "pq_sweep_sse")

    def launch_pipelined(self):
        """The sweep chunk by chunk on the current stream, each chunk's NVFP4 scale pass on the
        plan's side stream once that chunk is swept; returns the side stream, which the current
        stream must wait on before the scales and globals are read.  (Without the export: the
        sweep, and None.)"""
        import ctypes
        if not self.export:
            self.launch_sweep()
            return None
        lib = _lib.load()
        cur = torch.cuda.current_stream(self.device)
        if getattr(self, "_side", None) is None:
            self._side = torch.cuda.Stream(self.device)
        for (arr, k, sse_ptr), (n, A, G, S, Q, tptr, gptr) in zip(self._sweep_calls, self._scale_calls):
            _lib._check(lib.pq_sweep_sse(arr, k, ctypes.c_void_p(sse_ptr), cur.cuda_stream), "pq_sweep_sse")
            self._side.wait_stream(cur)
            _lib._check(lib.pq_nvfp4_scales(n, A, G, ctypes.c_void_p(tptr), Q, None, S, ctypes.c_void_p(gptr),
                                            self._side.cuda_stream), "pq_nvfp4_scales")
        return self._side

    def launch_scales(self):
        import ctypes
        lib = _lib.load()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        for (n, A, G, S, Q, tptr, gptr) in self._scale_calls:
            _lib._check(lib.pq_nvfp4_scales(n, A, G, ctypes.c_void_p(tptr), Q, None, S, ctypes.c_void_p(gptr),
                                            stream), "pq_nvfp4_scales")

    def launch_scales_side(self):
        """The NVFP4 scale pass on the plan's side stream, after what the current stream has
        enqueued (the sweep); returns that stream, which the current stream must wait on before
        the scales and globals are read.  Work enqueued on the current stream meanwhile (the
        cost-table all-gather) overlaps the scale pass."""
        cur = torch.cuda.current_stream(self.device)
        if getattr(self, "_side", None) is None:
            self._side = torch.cuda.Stream(self.device)
        self._side.wait_stream(cur)
        with torch.cuda.stream(self._side):
            self.launch_scales()
        return self._side

    def run(self, then=None, between=None):
        """Sweep, then the NVFP4 scale pass, chunk by chunk (launch_pipelined).  `then` (a
        callable, e.g. the all-gather of the cost table) is enqueued on the current stream after
        the sweep, overlapping the scale passes still running; the current stream waits for them
        before run() returns `then()`'s result (else the per-tensor sums).  `between` runs after
        the whole sweep and before any scale pass (e.g. distributed.reduce_split_tmax for tensors
        cut into row blocks across ranks)."""
        self.sse.zero_()
        if self.export:
            self.tmax.zero_()
        if between is None:
            side = self.launch_pipelined()
            out = then() if then is not None else self.sse
            if side is not None:
                torch.cuda.current_stream(self.device).wait_stream(side)
            return out
        self.launch_sweep()
        between()
        if then is None:
            if self.export:
                self.launch_scales()
            return self.sse
        side = self.launch_scales_side() if self.export else None
        out = then()
        if side is not None:
            torch.cuda.current_stream(self.device).wait_stream(side)
        return out

    def costs(self) -> dict:
        host = self.sse.cpu().tolist()
        _lib.raise_on_device_error("SweepExportPlan")
        out = {}
        for name, n, row, err in zip(self.names, self.numel, host, self.errors):
            out[name] = {s.name: ({"error": err[s.name]} if s.name in err else
                                  mqc._mse_from_sse(row[mqc._KCOL[mqc._kernel_format(s)]], n)) for s in self.specs}
        return out


class StreamingSweepExport:
    """Cost sweep + NVFP4 export of HOST-resident bf16 weights with the transfers overlapped.

    The weights are split into chunks of whole fused-sibling groups (about `chunk_bytes` each).
    Chunk c's host->device copy runs on one copy stream while chunk c-1 is swept and exported on
    the compute stream and chunk c-2's packed outputs go device->host on another copy stream, so a
    run costs about max(H2D, D2H) of the link instead of their sum.  Each chunk is a
    SweepExportPlan, so the numbers and bytes are those of the resident path.

    `run()` returns nothing and does not synchronise the host; `costs()` (one device->host read
    of the cost tables) and `host_outputs` are valid once the current stream has passed `run()`'s
    work.  host_outputs[name] = (weight_packed u8, weight_scale float8_e4m3fn, weight_global_scale
    f32 [1]) in pinned host memory."""

    def __init__(self, named_host_weights, specs, export_nvfp4: bool = True, chunk_bytes: int = 512 << 20,
                 device=None):
        items = list(named_host_weights.items()) if isinstance(named_host_weights, dict) else \
            list(named_host_weights)
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.specs = list(specs)
        self.export = export_nvfp4
        self.names = [n for n, _ in items]
        host = {}
        for n, w in items:
            if w.device.type != "cpu" or w.dtype != torch.bfloat16:
                raise TypeError(f"{n}: StreamingSweepExport takes bf16 host tensors")
            w = w.contiguous()
            host[n] = w if w.is_pinned() else w.pin_memory()
        self.host_weights = host
        # chunks of whole sibling groups, in first-appearance order
        groups: dict[str, list[str]] = {}
        for n in self.names:
            groups.setdefault(sibling_group_key(n) or f"\0{n}", []).append(n)
        self.chunks: list[list[str]] = [[]]
        size = 0
        for members in groups.values():
            if self.chunks[-1] and size >= chunk_bytes:
                self.chunks.append([])
                size = 0
            self.chunks[-1].extend(members)
            size += sum(host[m].numel() * 2 for m in members)
        self.dev_weights = {n: torch.empty(host[n].shape, dtype=torch.bfloat16, device=dev) for n in self.names}
        self.plans = [SweepExportPlan([(n, self.dev_weights[n]) for n in c], specs, export_nvfp4) for c in self.chunks]
        self.host_outputs = {}
        if export_nvfp4:
            for plan in self.plans:
                for i, n in enumerate(plan.names):
                    c, s, g = plan.outputs[i]
                    self.host_outputs[n] = (torch.empty(c.shape, dtype=torch.uint8).pin_memory(),
                                            torch.empty(s.shape, dtype=torch.uint8).pin_memory(),
                                            torch.empty(1, dtype=torch.float32).pin_memory())
        self.h2d = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        self._chunk_done = [torch.cuda.Event() for _ in self.chunks]   # chunk's outputs are on the host
        self.h2d_bytes = sum(w.numel() * 2 for w in host.values())
        self.d2h_bytes = sum(c.numel() + s.numel() + 4 for c, s, _ in self.host_outputs.values())

    def run(self):
        comp = torch.cuda.current_stream(self.device)
        self.h2d.wait_stream(comp)    # the previous run's readers of the device weights are done
        self.d2h.wait_stream(comp)
        for chunk, plan in zip(self.chunks, self.plans):
            with torch.cuda.stream(self.h2d):
                for n in chunk:
                    self.dev_weights[n].copy_(self.host_weights[n], non_blocking=True)
            comp.wait_stream(self.h2d)
            plan.run()
            if self.export:
                self.d2h.wait_stream(comp)
                with torch.cuda.stream(self.d2h):
                    for i, n in enumerate(plan.names):
                        hc, hs, hg = self.host_outputs[n]
                        c, s, g = plan.outputs[i]
                        hc.copy_(c, non_blocking=True)
                        hs.copy_(s.view(torch.uint8), non_blocking=True)
                        hg.copy_(g, non_blocking=True)
                    self._chunk_done[self.plans.index(plan)].record(self.d2h)
        comp.wait_stream(self.d2h)

    def costs(self) -> dict:
        out = {}
        for plan in self.plans:
            out.update(plan.costs())
        return out

    def sse_host(self) -> torch.Tensor:
        """All chunks' [n, 4] error sums in one device->host copy (synchronising)."""
        return torch.cat([p.sse for p in self.plans]).cpu()

    def export_to(self, writer, input_global_scale: float = DEFAULT_INPUT_GLOBAL_SCALE) -> None:
        """run(), then hand every tensor's NVFP4 entries to `writer.add_tensors` (an
        IncrementalSafetensorsWriter) chunk by chunk as each chunk's outputs reach the host, from a
        background thread, so the disk writes of one chunk overlap the GPU work and transfers of the
        next.  Keys are `{name}.weight_packed / .weight_scale / .weight_global_scale /
        .input_global_scale` as _quantize_2d emits them (export_native_compressed.py:1844-1865), so
        names are module prefixes.  Returns once everything is written; the caller finalizes."""
        import threading
        if not self.export:
            raise ValueError("export_to needs export_nvfp4=True")
        igs = torch.tensor([float(input_global_scale)], dtype=torch.float32)
        failure: list[BaseException] = []

        def writer_loop():
            try:
                for chunk, done in zip(self.chunks, self._chunk_done):
                    done.synchronize()
                    entries = {}
                    for n in chunk:
                        hc, hs, hg = self.host_outputs[n]
                        entries[f"{n}.weight_packed"] = hc
                        entries[f"{n}.weight_scale"] = hs.view(torch.float8_e4m3fn)
                        entries[f"{n}.weight_global_scale"] = hg
                        entries[f"{n}.input_global_scale"] = igs.clone()
                    writer.add_tensors(entries)
            except BaseException as e:   # re-raised on the caller's thread
                failure.append(e)

        self.run()
        t = threading.Thread(target=writer_loop, name="pq-safetensors-writer")
        t.start()
        t.join()
        if failure:
            raise failure[0]

    def outputs(self) -> dict:
        """{name: (weight_packed, weight_scale as float8_e4m3fn, weight_global_scale)} on the host."""
        return {n: (c, s.view(torch.float8_e4m3fn), g) for n, (c, s, g) in self.host_outputs.items()}
