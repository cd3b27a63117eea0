"""Install the B200 kernels behind an existing prismaquant process.

    import prismaquant_b200.install as pqi
    pqi.patch_prismaquant()          # after `import prismaquant`

Rebinds, in the already-imported reference modules, the functions on the
quantization-cost path to their B200 versions:

  format_registry.REGISTRY[f].quantize_dequantize       every registry format
      (and .activation_quantize_dequantize where the format quantizes activations)
  measure_quant_cost._batched_quantize                  (measure_quant_cost.py:532-548)
  measure_quant_cost.measure_batched_gpu,
      measure_unbatched, _measure_packed_experts        (measure_quant_cost.py:266-449, 551-685)
  export_native_compressed.compute_nvfp4_global_real,
      quantize_dequantize_nvfp4[_packed], quantize_dequantize_mxfp8[_packed],
      quantize_dequantize_fp8_dynamic[_packed]          (export_native_compressed.py:1045-1226)
  sensitivity_probe._GradNormCapture,
      install_packed_expert_hooks, FisherAccumulator    (sensitivity_probe.py:413-728, 959-1241)

and the same names in the production modules that imported them by name, so the
shard runners reach the kernels too:

  incremental_measure_quant_cost: measure_batched_gpu, measure_unbatched,
      _measure_packed_experts                           (incremental_measure_quant_cost.py:53-62)
  incremental_probe: FisherAccumulator, install_packed_expert_hooks
                                                        (incremental_probe.py:55-67)

The installed FisherAccumulator computes the reference's exact statistics by
default (grad_w = gy^T x on the tensor cores, the per-weight diagonal kept on
the device): a plain install does not change the probe's numbers.
`patch_prismaquant(fisher="per_token")` selects the per-token estimate instead.

The cost entry points take the caller's reference FormatSpecs and map them by
name to this package's registry.  A call whose device is not CUDA, or that
names a format this package does not know, runs the reference's own function
(the B200 kernels need CUDA tensors; nothing here computes on the CPU).
Production modules that fail to import are skipped.  Returns the list of
rebound names; `unpatch_prismaquant()` restores the originals.
"""
from __future__ import annotations

import functools
import importlib
import inspect

import torch

_SAVED: list[tuple[object, str, object]] = []

_COST_NAMES = ("measure_batched_gpu", "measure_unbatched", "_measure_packed_experts")
_PROBE_NAMES = ("FisherAccumulator", "install_packed_expert_hooks")
# production modules that import the names above into their own namespace
_IMPORTERS = {"incremental_measure_quant_cost": _COST_NAMES, "incremental_probe": _PROBE_NAMES}


def _rebind(obj, name: str, value, done: list[str], label: str):
    _SAVED.append((obj, name, getattr(obj, name)))
    setattr(obj, name, value)
    done.append(label)


def _is_cuda(device) -> bool:
    try:
        return torch.device(device).type == "cuda"
    except (TypeError, RuntimeError):
        return False


def _cost_wrapper(ours, theirs, our_fr):
    """measure_* with the reference's signature: specs mapped by name; non-CUDA devices and
    unknown formats go to the reference's function."""
    sig = inspect.signature(theirs)

    @functools.wraps(theirs)
    def wrapped(*args, **kwargs):
        bound = dict(sig.bind(*args, **kwargs).arguments)
        specs, device = bound.get("specs"), bound.get("device")
        if specs is None or not _is_cuda(device) or any(s.name not in our_fr.REGISTRY for s in specs):
            return theirs(*args, **kwargs)
        bound["specs"] = [our_fr.REGISTRY[s.name] for s in specs]
        return ours(**bound)
    wrapped.__prismaquant_b200__ = ours
    return wrapped


def patch_prismaquant(package: str = "prismaquant", fisher: str = "exact") -> list[str]:
    from . import _lib
    from . import export_native_compressed as our_enc
    from . import format_registry as our_fr
    from . import measure_quant_cost as our_mqc
    from . import sensitivity_probe as our_sp

    if fisher not in ("exact", "per_token"):
        raise ValueError(f"fisher must be 'exact' or 'per_token', got {fisher!r}")
    _lib.load()   # fail here, loudly, if the kernels are not built
    done: list[str] = []
    # import the production modules before anything is rebound, so the names they import from the
    # reference's modules are the reference's own (what unpatch must restore)
    importers = {}
    for mod_name in _IMPORTERS:
        try:
            importers[mod_name] = importlib.import_module(f"{package}.{mod_name}")
        except Exception:   # a production module whose own dependencies are absent here
            continue
    fr = importlib.import_module(f"{package}.format_registry")
    for name, spec in list(fr.REGISTRY.items()):
        ours = our_fr.REGISTRY.get(name)
        if ours is None or ours.kernel_format is None:
            continue
        _rebind(spec, "quantize_dequantize", ours.quantize_dequantize, done, f"format_registry.{name}.quantize_dequantize")
        if ours.activation_quantize_dequantize is not our_fr._identity:
            _rebind(spec, "activation_quantize_dequantize", ours.activation_quantize_dequantize, done,
                    f"format_registry.{name}.activation_quantize_dequantize")
    mqc = importlib.import_module(f"{package}.measure_quant_cost")
    ref_batched = mqc._batched_quantize

    def _batched_quantize(spec, stacked_w):
        ours = our_fr.REGISTRY.get(spec.name)
        if ours is not None and ours.kernel_format is not None:
            return our_mqc._batched_quantize(ours, stacked_w)   # CUDA tensors only; raises otherwise
        return ref_batched(spec, stacked_w)                      # formats without a B200 kernel

    _rebind(mqc, "_batched_quantize", _batched_quantize, done, "measure_quant_cost._batched_quantize")
    cost = {n: _cost_wrapper(getattr(our_mqc, n), getattr(mqc, n), our_fr) for n in _COST_NAMES}
    for n, fn in cost.items():
        _rebind(mqc, n, fn, done, f"measure_quant_cost.{n}")

    enc = importlib.import_module(f"{package}.export_native_compressed")
    for name in ("compute_nvfp4_global_real", "quantize_dequantize_nvfp4", "quantize_dequantize_nvfp4_packed",
                 "quantize_dequantize_mxfp8", "quantize_dequantize_mxfp8_packed",
                 "quantize_dequantize_fp8_dynamic", "quantize_dequantize_fp8_dynamic_packed"):
        _rebind(enc, name, getattr(our_enc, name), done, f"export_native_compressed.{name}")

    sp = importlib.import_module(f"{package}.sensitivity_probe")
    _rebind(sp, "_GradNormCapture", our_sp._GradNormCapture, done, "sensitivity_probe._GradNormCapture")

    class FisherAccumulator(our_sp.FisherAccumulator):
        """The B200 FisherAccumulator with the reference's constructor; statistics per
        patch_prismaquant(fisher=...)."""

        def __init__(self, model, tracked, expert_info, act_cache_dir=None, input_rows=256,
                     hook_packed_experts=True, h_detail_dir=None, **kw):
            kw.setdefault("estimator", fisher)
            super().__init__(model, tracked, expert_info, act_cache_dir, input_rows, hook_packed_experts,
                             h_detail_dir, **kw)

    FisherAccumulator.__module__ = our_sp.__name__
    probe = {"FisherAccumulator": FisherAccumulator, "install_packed_expert_hooks": our_sp.install_packed_expert_hooks}
    for n, fn in probe.items():
        _rebind(sp, n, fn, done, f"sensitivity_probe.{n}")

    for mod_name, mod in importers.items():
        for n in _IMPORTERS[mod_name]:
            if hasattr(mod, n):
                _rebind(mod, n, cost[n] if n in cost else probe[n], done, f"{mod_name}.{n}")
    return done


def unpatch_prismaquant() -> None:
    while _SAVED:
        obj, name, value = _SAVED.pop()
        setattr(obj, name, value)
