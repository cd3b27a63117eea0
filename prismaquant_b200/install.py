"""Install the B200 kernels behind an existing prismaquant process.

    import prismaquant_b200.install as pqi
    pqi.patch_prismaquant()          # after `import prismaquant`

Rebinds, in the already-imported reference modules, exactly the functions on
the quantization-cost path to their B200 versions:

  format_registry.REGISTRY[f].quantize_dequantize      NVFP4, NVFP4A16, MXFP8,
                                                       MXFP8_E4M3, MXFP8A16, FP8_E4M3
  measure_quant_cost._batched_quantize                 (measure_quant_cost.py:532-548)
  export_native_compressed.compute_nvfp4_global_real,
      quantize_dequantize_nvfp4[_packed], quantize_dequantize_mxfp8[_packed],
      quantize_dequantize_fp8_dynamic[_packed]         (export_native_compressed.py:1045-1226)
  sensitivity_probe._GradNormCapture                   (sensitivity_probe.py:413-504)

Formats without a B200 kernel keep the reference's implementation.  Returns
the list of rebound names; `unpatch_prismaquant()` restores the originals.
"""
from __future__ import annotations

import importlib

_SAVED: list[tuple[object, str, object]] = []


def _rebind(obj, name: str, value, done: list[str], label: str):
    _SAVED.append((obj, name, getattr(obj, name)))
    setattr(obj, name, value)
    done.append(label)


def patch_prismaquant(package: str = "prismaquant") -> list[str]:
    from . import _lib
    from . import export_native_compressed as our_enc
    from . import format_registry as our_fr
    from . import measure_quant_cost as our_mqc
    from . import sensitivity_probe as our_sp

    _lib.load()   # fail here, loudly, if the kernels are not built
    done: list[str] = []
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
    enc = importlib.import_module(f"{package}.export_native_compressed")
    for name in ("compute_nvfp4_global_real", "quantize_dequantize_nvfp4", "quantize_dequantize_nvfp4_packed",
                 "quantize_dequantize_mxfp8", "quantize_dequantize_mxfp8_packed",
                 "quantize_dequantize_fp8_dynamic", "quantize_dequantize_fp8_dynamic_packed"):
        _rebind(enc, name, getattr(our_enc, name), done, f"export_native_compressed.{name}")
    sp = importlib.import_module(f"{package}.sensitivity_probe")
    _rebind(sp, "_GradNormCapture", our_sp._GradNormCapture, done, "sensitivity_probe._GradNormCapture")
    return done


def unpatch_prismaquant() -> None:
    while _SAVED:
        obj, name, value = _SAVED.pop()
        setattr(obj, name, value)
