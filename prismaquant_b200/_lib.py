"""ctypes binding of libprismaquant_b200.so (the C ABI in include/prismaquant_b200.h).

Every function here takes CUDA torch tensors, checks dtype / device /
contiguity, hands raw pointers plus the current CUDA stream to the library
and returns torch tensors the caller owns.  There is no CPU path: if the
shared library is missing or a tensor is not on a CUDA device, the call
raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_NAME = "libprismaquant_b200.so"
LIB_PATH = Path(os.environ.get("PQ_B200_LIB", Path(__file__).resolve().parent / LIB_NAME))

PQ_OK, PQ_ERR_NULL, PQ_ERR_SHAPE, PQ_ERR_ALIGN, PQ_ERR_FORMAT, PQ_ERR_CUDA, PQ_ERR_LIMIT, PQ_ERR_DEVICE = range(8)
FMT_NVFP4, FMT_MXFP8, FMT_FP8_CHANNEL, FMT_BF16 = range(4)
FMT_IDS = {"NVFP4": FMT_NVFP4, "MXFP8": FMT_MXFP8, "FP8_E4M3": FMT_FP8_CHANNEL, "BF16": FMT_BF16}
# the rest of the registry (pq_format ids 4..14), served by the exact codebook / integer kernel
EXT_FMT_IDS = {"MXFP4": 4, "MXFP6_E3M2": 5, "MXFP6_E2M3": 6, "MXFP8_E5M2": 7, "FP8_E5M2": 8, "NVFP3": 9,
               "INT3": 10, "INT2": 11, "INT8_W8A16": 12, "INT4_W4A16_g128": 13, "FP8_E4M3_G128": 14}
FMT_IDS.update(EXT_FMT_IDS)
NUM_FMTS_ALL = 15

EXPORTED = [
    "pq_sweep_sse", "pq_cost_qdq", "pq_nvfp4_codes", "pq_nvfp4_scales", "pq_nvfp4_pack",
    "pq_mxfp8_pack", "pq_fp8_channel_pack", "pq_sumsq_rows", "pq_rownorm2", "pq_tokennorm_dot",
    "pq_device_error", "pq_last_cuda_error", "pq_status_string", "pq_version", "pq_nvfp4_pack_noalloc",
    "pq_format_sse", "pq_weighted_sse", "pq_output_sse", "pq_output_ref", "pq_output_err", "pq_cost_qdq_fused",
    "pq_weighted_sse_fused", "pq_cost_qdq_fused_sse", "pq_weighted_sse_fused_batch",
    "pq_cost_qdq_fused_sse_list", "pq_grad_sq_acc", "pq_set_wait_limit", "pq_default_wait_limit",
    "pq_sumsq_rows_full", "pq_nvfp4_global_real", "pq_tokennorm_dot_seg", "pq_format_sse_multi",
]


class SweepTensor(ctypes.Structure):
    """Mirror of pq_sweep_tensor."""
    _fields_ = [
        ("w", ctypes.c_void_p),
        ("rows", ctypes.c_int64),
        ("cols", ctypes.c_int64),
        ("fmt_mask", ctypes.c_uint32),
        ("_pad", ctypes.c_uint32),
        ("nvfp4_codes", ctypes.c_void_p),
        ("nvfp4_amax", ctypes.c_void_p),
        ("nvfp4_tmax", ctypes.c_void_p),
    ]


_LIB = None


def load() -> ctypes.CDLL:
    """Load the shared library (once).  Raises if it has not been built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m prismaquant_b200.build` "
            "(the B200 kernels have no CPU fallback)")
    lib = ctypes.CDLL(str(LIB_PATH))
    P, I64, I, V = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
    sig = {
        "pq_sweep_sse": [ctypes.POINTER(SweepTensor), I, P, V],
        "pq_cost_qdq": [P, I64, I64, I, P, V],
        "pq_cost_qdq_fused": [P, I64, I64, ctypes.c_uint32, P, V],
        "pq_weighted_sse_fused": [P, I64, I64, ctypes.c_uint32, P, I, P, V],
        "pq_cost_qdq_fused_sse": [P, I64, I64, I64, ctypes.c_uint32, P, P, V],
        "pq_weighted_sse_fused_batch": [P, I64, I64, I64, ctypes.c_uint32, P, I, P, V],
        "pq_cost_qdq_fused_sse_list": [P, I64, I64, I64, ctypes.c_uint32, P, P, V],
        "pq_format_sse": [P, I64, I64, I, P, V],
        "pq_format_sse_multi": [P, I64, I64, P, I, P, V],
        "pq_weighted_sse": [P, I64, I64, I, P, I, P, V],
        "pq_output_sse": [P, P, P, P, I64, I64, I64, I64, P, P, P, P, V],
        "pq_output_ref": [P, P, I64, I64, I64, I64, P, P, V],
        "pq_output_err": [P, P, P, I64, I64, I64, I64, P, V],
        "pq_grad_sq_acc": [P, P, P, I64, I64, I64, P, P, V],
        "pq_nvfp4_codes": [P, I64, I64, I64, P, P, P, V],
        "pq_nvfp4_scales": [I, ctypes.POINTER(P), ctypes.POINTER(I64), P, ctypes.POINTER(ctypes.c_int32), P,
                            ctypes.POINTER(P), P, V],
        "pq_nvfp4_pack": [P, I64, I64, I64, P, P, P, P, P, P, V],
        "pq_nvfp4_global_real": [P, I64, I64, I64, P, P, V],
        "pq_nvfp4_pack_noalloc": [P, I64, I64, I64, P, P, P, P, V],
        "pq_mxfp8_pack": [P, I64, I64, P, P, V],
        "pq_fp8_channel_pack": [P, I64, I64, P, P, V],
        "pq_sumsq_rows": [P, I64, I64, P, P, V],
        "pq_sumsq_rows_full": [P, I64, I64, P, P, P, V],
        "pq_rownorm2": [P, I64, I64, P, V],
        "pq_tokennorm_dot": [P, I64, I64, P, P, P, V],
        "pq_tokennorm_dot_seg": [P, I64, I64, P, P, P, I64, P, V],
        "pq_device_error": [ctypes.POINTER(ctypes.c_int)],
        "pq_set_wait_limit": [ctypes.c_uint32],
        "pq_default_wait_limit": [],
        "pq_last_cuda_error": [],
        "pq_status_string": [I],
        "pq_version": [],
    }
    for name, args in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = (ctypes.c_char_p if name == "pq_status_string" else
                      ctypes.c_uint32 if name == "pq_default_wait_limit" else ctypes.c_int)
    _LIB = lib
    return lib


def _check(status: int, what: str, shape_msg: str | None = None):
    if status == PQ_OK:
        return
    lib = load()
    msg = lib.pq_status_string(status).decode()
    if status == PQ_ERR_SHAPE:
        raise ValueError(shape_msg or f"{what}: {msg}")
    if status == PQ_ERR_CUDA:
        raise RuntimeError(f"{what}: {msg} (cudaError {lib.pq_last_cuda_error()})")
    raise RuntimeError(f"{what}: {msg}")


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def as_bf16_cuda(w: torch.Tensor, what: str) -> torch.Tensor:
    """Return a contiguous CUDA bf16 view of `w`.

    float32 inputs are accepted when every value is a bf16 value (the
    reference's export path feeds `weight.float()` of bf16 weights); other
    float32 tensors are rejected rather than rounded silently.
    """
    if not w.is_cuda:
        raise RuntimeError(f"{what}: tensor is on {w.device}; the B200 kernels need a CUDA tensor")
    if w.dtype == torch.bfloat16:
        return w.contiguous()
    if w.dtype == torch.float32:
        b = w.to(torch.bfloat16)
        if not torch.equal(b.float(), w):
            raise NotImplementedError(
                f"{what}: float32 input with values that are not bf16-representable is not supported")
        return b.contiguous()
    raise TypeError(f"{what}: unsupported dtype {w.dtype}")


def device_error() -> int:
    code = ctypes.c_int(0)
    _check(load().pq_device_error(ctypes.byref(code)), "pq_device_error")
    return code.value


def raise_on_device_error(what: str) -> None:
    """Raise if a kernel's bounded wait gave up since the last check (reads and clears the
    device error word; a host synchronisation point)."""
    code = device_error()
    if code:
        raise RuntimeError(f"{what}: a kernel's bounded wait gave up (device error {code}); its results are "
                           "incomplete")


def set_wait_limit(iterations: int | None) -> None:
    """Iteration limit of the sweep kernels' stage waits (None: the default).  A test hook for
    the failure-detection path: 0 makes those waits give up at once."""
    lib = load()
    n = lib.pq_default_wait_limit() if iterations is None else int(iterations)
    _check(lib.pq_set_wait_limit(n), "pq_set_wait_limit")


# ---------------------------------------------------------------------------
# Cost path
# ---------------------------------------------------------------------------

def sweep_sse(weights, masks, nvfp4_outputs=None, sse: torch.Tensor | None = None) -> torch.Tensor:
    """Fused multi-format error sweep.  `weights` are 2-D (or 3-D packed)
    bf16 CUDA tensors, `masks` one format bitmask each.  Returns (or adds
    into) a [n, 4] float64 tensor of sum((W - qdq_f(W))^2).

    `nvfp4_outputs`, if given, is a list (per tensor, or None) of
    (codes u8 [rows, cols/2], amax bf16-scratch [rows, cols/16], tmax u32 [1])
    filled in the same pass."""
    lib = load()
    n = len(weights)
    if n == 0:
        return torch.zeros(0, 4, dtype=torch.float64)
    dev = weights[0].device
    if sse is None:
        sse = torch.zeros(n, 4, dtype=torch.float64, device=dev)
    arr = (SweepTensor * n)()
    keep = []
    for i, (w, m) in enumerate(zip(weights, masks)):
        if w.device != dev:
            raise RuntimeError("sweep_sse: all tensors must be on one device")
        if w.dtype != torch.bfloat16 or not w.is_contiguous():
            raise TypeError("sweep_sse: weights must be contiguous bf16")
        keep.append(w)
        cols = w.shape[-1] if w.dim() else 1
        rows = w.numel() // cols if cols else 0
        arr[i].w = w.data_ptr()
        arr[i].rows = rows
        arr[i].cols = cols
        arr[i].fmt_mask = int(m)
        if nvfp4_outputs is not None and nvfp4_outputs[i] is not None:
            codes, amax, tmax = nvfp4_outputs[i]
            arr[i].nvfp4_codes = codes.data_ptr()
            arr[i].nvfp4_amax = amax.data_ptr()
            arr[i].nvfp4_tmax = tmax.data_ptr()
    _check(lib.pq_sweep_sse(arr, n, _ptr(sse), _stream(sse)), "pq_sweep_sse")
    return sse


def cost_qdq(w: torch.Tensor, fmt: str) -> torch.Tensor:
    """Cost-path quantize->dequantize (bf16 in, bf16 out, same shape)."""
    lib = load()
    wb = as_bf16_cuda(w, "quantize_dequantize")
    out = torch.empty_like(wb)
    if wb.numel() == 0:
        return out.to(w.dtype)
    cols = wb.shape[-1]
    rows = wb.numel() // cols
    fid = FMT_IDS[fmt]
    _check(lib.pq_cost_qdq(_ptr(wb), rows, cols, fid, _ptr(out), _stream(wb)), "pq_cost_qdq",
           f"cannot reshape rows of {cols} into groups for {fmt}")
    return out if w.dtype == torch.bfloat16 else out.to(w.dtype)


FUSED_FMTS = ("NVFP4", "MXFP8", "FP8_E4M3")


def cost_qdq_fused(w: torch.Tensor, fmts) -> dict:
    """Cost-path W_hat of several of NVFP4 / MXFP8 / FP8_E4M3 (per channel) from one read of W:
    {fmt: bf16 tensor of w's shape}, each equal to cost_qdq(w, fmt)."""
    wb = as_bf16_cuda(w, "quantize_dequantize")
    want = [f for f in FUSED_FMTS if f in set(fmts)]
    if len(want) != len(set(fmts)):
        raise ValueError(f"cost_qdq_fused: formats must be among {FUSED_FMTS}, got {list(fmts)}")
    out = torch.empty((len(want),) + tuple(wb.shape), dtype=torch.bfloat16, device=wb.device)
    if wb.numel():
        cols = wb.shape[-1] if wb.dim() else 1
        mask = sum(1 << FMT_IDS[f] for f in want)
        _check(load().pq_cost_qdq_fused(_ptr(wb), wb.numel() // cols, cols, mask, _ptr(out), _stream(wb)),
               "pq_cost_qdq_fused", f"cannot reshape rows of {cols} into groups for {want}")
    return {f: out[i] for i, f in enumerate(want)}


def cost_qdq_fused_sse(w: torch.Tensor, fmts) -> tuple[dict, torch.Tensor]:
    """cost_qdq_fused of a stacked weight [batch, rows, cols] (a 2-D weight is batch 1) together
    with each w[b]'s error sums, from one read of w: ({fmt: bf16 tensor of w's shape},
    fp64 [batch, 4] device tensor whose column FMT_IDS[fmt] holds sum((w[b] - W_hat)^2))."""
    wb = as_bf16_cuda(w, "quantize_dequantize")
    want = [f for f in FUSED_FMTS if f in set(fmts)]
    if len(want) != len(set(fmts)) or not want:
        raise ValueError(f"cost_qdq_fused_sse: formats must be among {FUSED_FMTS}, got {list(fmts)}")
    if wb.dim() not in (2, 3):
        raise ValueError(f"cost_qdq_fused_sse: expected a [rows, cols] or [batch, rows, cols] weight, got "
                         f"{tuple(wb.shape)}")
    w3 = wb.unsqueeze(0) if wb.dim() == 2 else wb
    batch, rows, cols = w3.shape
    out = torch.empty((len(want),) + tuple(wb.shape), dtype=torch.bfloat16, device=wb.device)
    sse = torch.zeros(batch, 4, dtype=torch.float64, device=wb.device)
    if w3.numel():
        mask = sum(1 << FMT_IDS[f] for f in want)
        _check(load().pq_cost_qdq_fused_sse(_ptr(w3), batch, rows, cols, mask, _ptr(out), _ptr(sse), _stream(wb)),
               "pq_cost_qdq_fused_sse", f"cannot reshape rows of {cols} into groups for {want}")
    return {f: out[i] for i, f in enumerate(want)}, sse


def cost_qdq_fused_sse_list(ws, fmts) -> tuple[dict, torch.Tensor, torch.Tensor]:
    """cost_qdq_fused_sse for a list of same-shape [rows, cols] bf16 CUDA weights that are not
    stacked: ({fmt: W_hat [batch, rows, cols]}, the weights stacked [batch, rows, cols], fp64
    [batch, 4] sums), all from one read of each weight."""
    want = [f for f in FUSED_FMTS if f in set(fmts)]
    if len(want) != len(set(fmts)) or not want:
        raise ValueError(f"cost_qdq_fused_sse_list: formats must be among {FUSED_FMTS}, got {list(fmts)}")
    wl = [as_bf16_cuda(w, "quantize_dequantize") for w in ws]
    if not wl or any(w.dim() != 2 or w.shape != wl[0].shape or w.device != wl[0].device for w in wl):
        raise ValueError("cost_qdq_fused_sse_list: expected same-shape [rows, cols] weights on one device")
    batch, (rows, cols) = len(wl), wl[0].shape
    out = torch.empty((len(want) + 1, batch, rows, cols), dtype=torch.bfloat16, device=wl[0].device)
    sse = torch.zeros(batch, 4, dtype=torch.float64, device=wl[0].device)
    if out.numel():
        ptrs = (ctypes.c_void_p * batch)(*[w.data_ptr() for w in wl])
        mask = sum(1 << FMT_IDS[f] for f in want)
        _check(load().pq_cost_qdq_fused_sse_list(ptrs, batch, rows, cols, mask, _ptr(out), _ptr(sse), _stream(wl[0])),
               "pq_cost_qdq_fused_sse_list", f"cannot reshape rows of {cols} into groups for {want}")
    return {f: out[i] for i, f in enumerate(want)}, out[len(want)], sse


def format_sse(w: torch.Tensor, fmt: str, sse: torch.Tensor) -> None:
    """Adds sum((W - qdq_fmt(W))^2) into the fp64 device scalar `sse` (one of the extended
    formats, or BF16); asynchronous on the current stream."""
    wb = as_bf16_cuda(w, "format_sse")
    if wb.numel() == 0:
        return
    cols = wb.shape[-1]
    _check(load().pq_format_sse(_ptr(wb), wb.numel() // cols, cols, FMT_IDS[fmt], _ptr(sse), _stream(wb)),
           "pq_format_sse", f"cannot reshape rows of {cols} into groups for {fmt}")


def format_sse_multi(w: torch.Tensor, fmts: list[str], sse: torch.Tensor) -> None:
    """format_sse of several formats: adds each format's sum into sse[f] (a contiguous fp64 device
    vector of len(fmts)); the MX formats among them come from one read of the weights."""
    wb = as_bf16_cuda(w, "format_sse_multi")
    if wb.numel() == 0 or not fmts:
        return
    if sse.dtype != torch.float64 or not sse.is_contiguous() or sse.numel() < len(fmts):
        raise ValueError("format_sse_multi: sse must be a contiguous fp64 vector with one entry per format")
    cols = wb.shape[-1]
    ids = (ctypes.c_int32 * len(fmts))(*[FMT_IDS[f] for f in fmts])
    _check(load().pq_format_sse_multi(_ptr(wb), wb.numel() // cols, cols, ctypes.cast(ids, ctypes.c_void_p),
                                      len(fmts), _ptr(sse), _stream(wb)),
           "pq_format_sse_multi", f"cannot reshape rows of {cols} into groups for one of {fmts}")


def weighted_sse(w: torch.Tensor, fmt: str, h: torch.Tensor, sse: torch.Tensor, per_row: bool = False) -> None:
    """Adds sum(h * (W - qdq_fmt(W))^2) into the fp64 device scalar `sse`; h is fp32 with W's
    shape, or (per_row) one weight per row of W viewed as [numel / cols, cols]."""
    wb = as_bf16_cuda(w, "weighted_sse")
    if wb.numel() == 0:
        return
    cols = wb.shape[-1]
    rows = wb.numel() // cols
    hh = h.detach()
    if hh.device != wb.device or hh.dtype != torch.float32:
        raise TypeError("weighted_sse: h must be float32 on the weight's device")
    hh = hh.contiguous()
    if hh.numel() != (rows if per_row else rows * cols):
        raise ValueError(f"weighted_sse: h has {hh.numel()} values for a [{rows}, {cols}] weight")
    _check(load().pq_weighted_sse(_ptr(wb), rows, cols, FMT_IDS[fmt], _ptr(hh), int(per_row), _ptr(sse),
                                  _stream(wb)), "pq_weighted_sse", f"cannot reshape rows of {cols} into groups for {fmt}")


def weighted_sse_fused(w: torch.Tensor, fmts, h: torch.Tensor, sse: torch.Tensor | None = None,
                       per_row: bool = False) -> torch.Tensor:
    """weighted_sse of several of NVFP4 / MXFP8 / FP8_E4M3 (per channel) from one read of W and h:
    adds each format's sum into sse[FMT_IDS[fmt]] of the fp64 device vector `sse` (3 entries; a
    new zero vector when None) and returns it."""
    wb = as_bf16_cuda(w, "weighted_sse")
    want = [f for f in FUSED_FMTS if f in set(fmts)]
    if len(want) != len(set(fmts)) or not want:
        raise ValueError(f"weighted_sse_fused: formats must be among {FUSED_FMTS}, got {list(fmts)}")
    if sse is None:
        sse = torch.zeros(3, dtype=torch.float64, device=wb.device)
    _check_sums(sse, 3, wb.device, "weighted_sse_fused")
    if wb.numel() == 0:
        return sse
    cols = wb.shape[-1]
    rows = wb.numel() // cols
    hh = h.detach()
    if hh.device != wb.device or hh.dtype != torch.float32:
        raise TypeError("weighted_sse_fused: h must be float32 on the weight's device")
    hh = hh.contiguous()
    if hh.numel() != (rows if per_row else rows * cols):
        raise ValueError(f"weighted_sse_fused: h has {hh.numel()} values for a [{rows}, {cols}] weight")
    mask = sum(1 << FMT_IDS[f] for f in want)
    _check(load().pq_weighted_sse_fused(_ptr(wb), rows, cols, mask, _ptr(hh), int(per_row), _ptr(sse),
                                        _stream(wb)),
           "pq_weighted_sse_fused", f"cannot reshape rows of {cols} into groups for {want}")
    return sse


def weighted_sse_fused_batch(w: torch.Tensor, fmts, h: torch.Tensor, per_row: bool = False) -> torch.Tensor:
    """weighted_sse_fused of each w[b] of a stacked [batch, rows, cols] weight with its own h[b]
    ([rows, cols], or [rows] when per_row), in one launch: a new fp64 [batch, 3] device tensor
    whose column FMT_IDS[fmt] holds w[b]'s sum(h[b] * err^2)."""
    wb = as_bf16_cuda(w, "weighted_sse")
    want = [f for f in FUSED_FMTS if f in set(fmts)]
    if len(want) != len(set(fmts)) or not want:
        raise ValueError(f"weighted_sse_fused_batch: formats must be among {FUSED_FMTS}, got {list(fmts)}")
    if wb.dim() != 3:
        raise ValueError(f"weighted_sse_fused_batch: expected a [batch, rows, cols] weight, got {tuple(wb.shape)}")
    batch, rows, cols = wb.shape
    hh = h.detach()
    if hh.device != wb.device or hh.dtype != torch.float32:
        raise TypeError("weighted_sse_fused_batch: h must be float32 on the weight's device")
    hh = hh.contiguous()
    if hh.numel() != batch * (rows if per_row else rows * cols):
        raise ValueError(f"weighted_sse_fused_batch: h has {hh.numel()} values for a {tuple(wb.shape)} weight")
    sse = torch.zeros(batch, 3, dtype=torch.float64, device=wb.device)
    if wb.numel():
        mask = sum(1 << FMT_IDS[f] for f in want)
        _check(load().pq_weighted_sse_fused_batch(_ptr(wb), batch, rows, cols, mask, _ptr(hh), int(per_row),
                                                  _ptr(sse), _stream(wb)),
               "pq_weighted_sse_fused_batch", f"cannot reshape rows of {cols} into groups for {want}")
    return sse


def output_sse(x: torch.Tensor, w: torch.Tensor, x_hat: torch.Tensor, w_hat: torch.Tensor,
               err_sse: torch.Tensor | None, ref_sse: torch.Tensor | None,
               y_ref: torch.Tensor | None = None, y_q: torch.Tensor | None = None) -> None:
    """Adds, per stacked Linear b, sum(bf16(y_ref - y_q)^2) into err_sse[b] and sum(y_ref^2) into
    ref_sse[b] (fp64 [batch] on the device), y_ref = bf16(X W^T), y_q = bf16(X_hat W_hat^T)
    computed on the tensor cores.  x, x_hat: [batch, rows, k] (or [rows, k]); w, w_hat:
    [batch, out, k] (or [out, k]); k a multiple of 8.  y_ref / y_q (fp32 [batch, rows, out])
    optionally receive the unrounded accumulators."""
    xs = [as_bf16_cuda(t, "output_sse") for t in (x, w, x_hat, w_hat)]
    squeeze = xs[0].dim() == 2
    if squeeze:
        xs = [t.unsqueeze(0) for t in xs]
    xb, wb, xqb, wqb = xs
    if any(t.dim() != 3 for t in xs) or xb.shape != xqb.shape or wb.shape != wqb.shape or \
            xb.shape[0] != wb.shape[0] or xb.shape[2] != wb.shape[2]:
        raise ValueError(f"output_sse: shapes {[tuple(t.shape) for t in (x, w, x_hat, w_hat)]} do not match")
    batch, rows, k = xb.shape
    out = wb.shape[1]
    for name, t in (("err_sse", err_sse), ("ref_sse", ref_sse)):
        if t is not None and (t.dtype != torch.float64 or t.device != xb.device or t.numel() != batch
                              or not t.is_contiguous()):
            raise TypeError(f"output_sse: {name} must be a contiguous float64 [{batch}] tensor on the device")
    for name, t in (("y_ref", y_ref), ("y_q", y_q)):
        if t is not None and (t.dtype != torch.float32 or t.device != xb.device or t.numel() != batch * rows * out
                              or not t.is_contiguous()):
            raise TypeError(f"output_sse: {name} must be a contiguous float32 [{batch}, {rows}, {out}] tensor")
    _check(load().pq_output_sse(_ptr(xb), _ptr(wb), _ptr(xqb), _ptr(wqb), batch, rows, out, k, _ptr(err_sse),
                                _ptr(ref_sse), _ptr(y_ref), _ptr(y_q), _stream(xb)),
           "pq_output_sse", f"k = {k} must be a multiple of 8")


def _outerr_operands(x: torch.Tensor, w: torch.Tensor, what: str):
    xb, wb = as_bf16_cuda(x, what), as_bf16_cuda(w, what)
    if xb.dim() == 2:
        xb, wb = xb.unsqueeze(0), wb.unsqueeze(0)
    if xb.dim() != 3 or wb.dim() != 3 or xb.shape[0] != wb.shape[0] or xb.shape[2] != wb.shape[2]:
        raise ValueError(f"{what}: shapes {tuple(x.shape)} and {tuple(w.shape)} do not match")
    return xb, wb


def _check_sums(t, batch, dev, what):
    if t is not None and (t.dtype != torch.float64 or t.device != dev or t.numel() != batch or not t.is_contiguous()):
        raise TypeError(f"{what} must be a contiguous float64 [{batch}] tensor on the device")


def output_ref(x: torch.Tensor, w: torch.Tensor, ref_sse: torch.Tensor | None,
               y_ref: torch.Tensor | None = None) -> None:
    """y_ref = bf16(X W^T) on the tensor cores: written into `y_ref` (bf16 [batch, rows, out], may be
    None) and sum(y_ref^2) added into ref_sse[b] (fp64 [batch] on the device)."""
    xb, wb = _outerr_operands(x, w, "output_ref")
    batch, rows, k = xb.shape
    out = wb.shape[1]
    _check_sums(ref_sse, batch, xb.device, "output_ref: ref_sse")
    if y_ref is not None and (y_ref.dtype != torch.bfloat16 or y_ref.device != xb.device or
                              y_ref.numel() != batch * rows * out or not y_ref.is_contiguous()):
        raise TypeError(f"output_ref: y_ref must be a contiguous bfloat16 [{batch}, {rows}, {out}] tensor")
    _check(load().pq_output_ref(_ptr(xb), _ptr(wb), batch, rows, out, k, _ptr(y_ref), _ptr(ref_sse), _stream(xb)),
           "pq_output_ref", f"k = {k} must be a multiple of 8")


def output_err(x_hat: torch.Tensor, w_hat: torch.Tensor, y_ref: torch.Tensor, err_sse: torch.Tensor) -> None:
    """Adds sum(bf16(y_ref - bf16(X_hat W_hat^T))^2) into err_sse[b]; y_ref is the bf16 output of
    output_ref for the same shapes."""
    xb, wb = _outerr_operands(x_hat, w_hat, "output_err")
    batch, rows, k = xb.shape
    out = wb.shape[1]
    _check_sums(err_sse, batch, xb.device, "output_err: err_sse")
    if y_ref.dtype != torch.bfloat16 or y_ref.device != xb.device or y_ref.numel() != batch * rows * out or \
            not y_ref.is_contiguous():
        raise TypeError(f"output_err: y_ref must be a contiguous bfloat16 [{batch}, {rows}, {out}] tensor")
    _check(load().pq_output_err(_ptr(xb), _ptr(wb), _ptr(y_ref), batch, rows, out, k, _ptr(err_sse), _stream(xb)),
           "pq_output_err", f"k = {k} must be a multiple of 8")


def grad_sq_acc(gy: torch.Tensor, x: torch.Tensor, h: torch.Tensor, sums: torch.Tensor,
                w: torch.Tensor | None = None) -> None:
    """One backward's per-weight Fisher diagonal on the tensor cores: with grad_w = bf16(gy^T x)
    (gy [t, m], x [t, n]) and g2 = bf16(grad_w^2), h (fp32 [m, n]) += g2, sums[0] += sum(g2) and,
    given the bf16 weight w [m, n], sums[1] += sum(bf16(g2 * bf16(w^2)))."""
    gb, xb = as_bf16_cuda(gy, "grad_sq_acc"), as_bf16_cuda(x, "grad_sq_acc")
    gb, xb = gb.reshape(-1, gb.shape[-1]), xb.reshape(-1, xb.shape[-1])
    t, m = gb.shape
    n = xb.shape[1]
    if xb.shape[0] != t or tuple(h.shape) != (m, n) or h.dtype != torch.float32 or not h.is_contiguous():
        raise ValueError(f"grad_sq_acc: gy {tuple(gy.shape)}, x {tuple(x.shape)}, h {tuple(h.shape)} do not match")
    if sums.dtype != torch.float64 or sums.numel() < 2 or not sums.is_contiguous():
        raise TypeError("grad_sq_acc: sums must be a contiguous float64 tensor of 2")
    wb = None if w is None else as_bf16_cuda(w, "grad_sq_acc")
    if wb is not None and tuple(wb.shape) != (m, n):
        raise ValueError(f"grad_sq_acc: w {tuple(wb.shape)} is not [{m}, {n}]")
    _check(load().pq_grad_sq_acc(_ptr(gb), _ptr(xb), _ptr(wb), t, m, n, _ptr(h), _ptr(sums), _stream(gb)),
           "pq_grad_sq_acc", f"grad_w [{m}, {n}]: both sides must be multiples of 8")


# ---------------------------------------------------------------------------
# Export path
# ---------------------------------------------------------------------------

def nvfp4_global_real(w: torch.Tensor, batch: int = 1) -> torch.Tensor:
    """compute_nvfp4_global_real of each of `batch` equal slices of w, from one read: fp32 [batch]."""
    wb = as_bf16_cuda(w, "nvfp4_global_real")
    cols = wb.shape[-1]
    rows = wb.numel() // cols // max(batch, 1)
    out = torch.empty(batch, dtype=torch.float32, device=wb.device)
    scratch = torch.empty(batch + 1, dtype=torch.int32, device=wb.device)
    _check(load().pq_nvfp4_global_real(_ptr(wb), batch, rows, cols, _ptr(scratch), _ptr(out), _stream(wb)),
           "pq_nvfp4_global_real", f"NVFP4 group_size=16 ∤ {cols}")
    return out


def nvfp4_codes(w: torch.Tensor, batch: int, codes: torch.Tensor, amax: torch.Tensor, tmax: torch.Tensor):
    cols = w.shape[-1]
    rows = w.numel() // cols // max(batch, 1)
    _check(load().pq_nvfp4_codes(_ptr(w), batch, rows, cols, _ptr(codes), _ptr(amax), _ptr(tmax), _stream(w)),
           "pq_nvfp4_codes", f"NVFP4 group_size=16 ∤ {cols}")


def nvfp4_scales(amax_list, tmax: torch.Tensor | None, scales_list, global_div: torch.Tensor,
                 group_of=None, override: torch.Tensor | None = None):
    n = len(amax_list)
    lib = load()
    A = (ctypes.c_void_p * n)(*[a.data_ptr() for a in amax_list])
    G = (ctypes.c_int64 * n)(*[a.numel() for a in amax_list])
    S = (ctypes.c_void_p * n)(*[s.data_ptr() for s in scales_list])
    grp = None if group_of is None else (ctypes.c_int32 * n)(*[int(g) for g in group_of])
    _check(lib.pq_nvfp4_scales(n, A, G, _ptr(tmax), grp, _ptr(override), S, _ptr(global_div),
                               _stream(global_div)), "pq_nvfp4_scales")


def nvfp4_pack(w: torch.Tensor, override: torch.Tensor | None = None):
    """NVFP4 export of [rows, cols] (one global) or [E, M, N] (per-expert globals).

    Returns (weight_packed u8, weight_scale float8_e4m3fn, weight_global_scale f32)."""
    wb = as_bf16_cuda(w, "quantize_dequantize_nvfp4")
    if wb.dim() not in (2, 3):
        raise ValueError(f"NVFP4 export expects a 2-D or 3-D weight, got {tuple(wb.shape)}")
    batch = 1 if wb.dim() == 2 else wb.shape[0]
    cols = wb.shape[-1]
    if cols % 16:
        raise ValueError(f"NVFP4 group_size=16 ∤ {cols}")
    lead = wb.shape[:-1]
    dev = wb.device
    codes = torch.empty(*lead, cols // 2, dtype=torch.uint8, device=dev)
    scales = torch.empty(*lead, cols // 16, dtype=torch.uint8, device=dev)
    gdiv = torch.empty(batch, dtype=torch.float32, device=dev)
    amax = torch.empty(*lead, cols // 16, dtype=torch.int16, device=dev)
    tmax = torch.empty(batch, dtype=torch.int32, device=dev)
    if override is not None:
        override = override.to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
        if override.numel() == 1 and batch > 1:
            override = override.expand(batch).contiguous()
    rows = wb.numel() // cols // batch
    _check(load().pq_nvfp4_pack(_ptr(wb), batch, rows, cols, _ptr(override), _ptr(codes), _ptr(scales),
                                _ptr(gdiv), _ptr(amax), _ptr(tmax), _stream(wb)), "pq_nvfp4_pack")
    return codes, scales.view(torch.float8_e4m3fn), gdiv


def mxfp8_pack(w: torch.Tensor):
    wb = as_bf16_cuda(w, "quantize_dequantize_mxfp8")
    cols = wb.shape[-1]
    if cols % 32:
        raise ValueError(f"MXFP8 group_size=32 ∤ {cols}")
    q = torch.empty(wb.shape, dtype=torch.uint8, device=wb.device)
    sc = torch.empty(*wb.shape[:-1], cols // 32, dtype=torch.uint8, device=wb.device)
    _check(load().pq_mxfp8_pack(_ptr(wb), wb.numel() // cols, cols, _ptr(q), _ptr(sc), _stream(wb)),
           "pq_mxfp8_pack")
    return q.view(torch.float8_e4m3fn), sc


def fp8_channel_pack(w: torch.Tensor):
    wb = as_bf16_cuda(w, "quantize_dequantize_fp8_dynamic")
    cols = wb.shape[-1]
    q = torch.empty(wb.shape, dtype=torch.uint8, device=wb.device)
    s = torch.empty(*wb.shape[:-1], 1, dtype=torch.float32, device=wb.device)
    _check(load().pq_fp8_channel_pack(_ptr(wb), wb.numel() // cols, cols, _ptr(q), _ptr(s), _stream(wb)),
           "pq_fp8_channel_pack")
    return q.view(torch.float8_e4m3fn), s


# ---------------------------------------------------------------------------
# Fisher statistics
# ---------------------------------------------------------------------------

def sumsq_rows(g: torch.Tensor, total: torch.Tensor, per_row: torch.Tensor | None = None):
    """total[0] += sum(g^2) (fp64); per_row (fp32, g.shape[:-1]) += row sums."""
    gb = as_bf16_cuda(g, "sumsq_rows")
    cols = gb.shape[-1]
    _check(load().pq_sumsq_rows(_ptr(gb), gb.numel() // cols, cols, _ptr(total), _ptr(per_row), _stream(gb)),
           "pq_sumsq_rows")


def sumsq_rows_full(g: torch.Tensor, total: torch.Tensor, per_row: torch.Tensor | None, h_full: torch.Tensor):
    """sumsq_rows plus h_full (fp32, g's shape, on g's device) += g.float()^2, one read of g."""
    gb = as_bf16_cuda(g, "sumsq_rows_full")
    cols = gb.shape[-1]
    if (h_full.dtype != torch.float32 or not h_full.is_contiguous() or h_full.numel() != gb.numel()
            or h_full.device != gb.device):
        raise ValueError(f"sumsq_rows_full: h_full must be a contiguous float32 tensor of {tuple(gb.shape)} on "
                         f"{gb.device}")
    _check(load().pq_sumsq_rows_full(_ptr(gb), gb.numel() // cols, cols, _ptr(total), _ptr(per_row), _ptr(h_full),
                                     _stream(gb)), "pq_sumsq_rows_full")


def rownorm2(x: torch.Tensor) -> torch.Tensor:
    xb = as_bf16_cuda(x, "rownorm2")
    d = xb.shape[-1]
    out = torch.empty(xb.numel() // d, dtype=torch.float32, device=xb.device)
    _check(load().pq_rownorm2(_ptr(xb), out.numel(), d, _ptr(out), _stream(xb)), "pq_rownorm2")
    return out


def tokennorm_dot_seg(g: torch.Tensor, xnorm: torch.Tensor, seg: torch.Tensor, acc: torch.Tensor,
                      token_idx: torch.Tensor | None = None):
    """Routed experts in one launch: rows of g [R, d] sorted by expert seg[r] (int32);
    acc[e, 0] += sum over e's rows of xnorm[token_idx[r]] * ||g_r||^2, acc[e, 1] += row count."""
    gb = as_bf16_cuda(g, "tokennorm_dot_seg")
    d = gb.shape[-1]
    R = gb.numel() // d
    if acc.dtype != torch.float64 or not acc.is_contiguous() or acc.dim() != 2 or acc.shape[1] != 2:
        raise TypeError("tokennorm_dot_seg: acc must be a contiguous float64 [E, 2] tensor")
    seg = seg.to(torch.int32).contiguous()
    if token_idx is not None:
        token_idx = token_idx.to(torch.int64).contiguous()
    _check(load().pq_tokennorm_dot_seg(_ptr(gb), R, d, _ptr(xnorm), _ptr(token_idx), _ptr(seg), acc.shape[0],
                                       _ptr(acc), _stream(gb)), "pq_tokennorm_dot_seg")


def tokennorm_dot(g: torch.Tensor, xnorm: torch.Tensor, acc: torch.Tensor, token_idx: torch.Tensor | None = None):
    """acc[0] += sum_t xnorm[idx(t)] * ||g_t||^2; acc[1] += T."""
    gb = as_bf16_cuda(g, "tokennorm_dot")
    d = gb.shape[-1]
    T = gb.numel() // d
    if token_idx is not None:
        token_idx = token_idx.to(torch.int64).contiguous()
    _check(load().pq_tokennorm_dot(_ptr(gb), T, d, _ptr(xnorm), _ptr(token_idx), _ptr(acc), _stream(gb)),
           "pq_tokennorm_dot")
