"""FormatSpec / REGISTRY / get_format with CUDA quantize-dequantize.

Drop-in for prismaquant/format_registry.py (FormatSpec :31-119, REGISTRY and
register_format :126-136, get_format :585-590) with every registered format:
NVFP4 (+ NVFP4A16), MXFP8 (+ MXFP8_E4M3, MXFP8A16) and FP8_E4M3 per output
channel run on the fused sweep kernels; MXFP4, MXFP6 E3M2/E2M3, MXFP8_E5M2,
FP8_E5M2, NVFP3, INT2/INT3 (aliases NVINT2/NVINT3), INT8_W8A16 and
INT4_W4A16_g128 on the exact codebook / integer kernel; BF16 and FP8_SOURCE
are clones.  The metadata of each format (bits, group size, scale dtype,
family) is the reference's, so shape-aware bit counts and allocator inputs
are unchanged; `quantize_dequantize` runs the sm_100a kernel of the same
cost-path arithmetic (format_registry.py:147-233) on a bf16 CUDA tensor.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable

import torch

from . import _lib


@dataclass
class FormatSpec:
    name: str
    weight_bits: int
    group_size: int          # 0 = per output channel (one scale per row)
    scale_bits: int
    scale_dtype_name: str
    weight_element_dtype: str
    scale_block_shape: tuple[int, int] | None = None
    act_bits: int | None = None
    act_dtype_name: str | None = None
    act_group_size: int | None = None
    family: str = "generic"
    min_capability_sm: int = 80
    autoround_config: Callable[[], dict] = field(default=lambda: {})
    quantize_dequantize: Callable[[torch.Tensor], torch.Tensor] = field(default=lambda x: x)
    activation_quantize_dequantize: Callable[[torch.Tensor], torch.Tensor] = field(default=lambda x: x)
    # Which kernel format computes this spec's weight error (None: not on the B200 path).
    kernel_format: str | None = None

    @property
    def effective_bits(self) -> float:
        if self.group_size == 0:
            return float(self.weight_bits) if self.scale_bits == 0 else float(self.weight_bits) + 0.02
        if self.scale_block_shape is not None:
            r, c = self.scale_block_shape
            return float(self.weight_bits) + float(self.scale_bits) / (r * c)
        return float(self.weight_bits) + float(self.scale_bits) / self.group_size

    def scale_count_for_shape(self, shape: tuple[int, ...]) -> int:
        if len(shape) == 0 or self.scale_bits == 0:
            return 0
        if self.scale_block_shape is not None:
            r, c = self.scale_block_shape
            if len(shape) < 2:
                return math.ceil(int(shape[0]) / (r * c))
            outer = int(math.prod(shape[:-2])) if len(shape) > 2 else 1
            return outer * math.ceil(int(shape[-2]) / r) * math.ceil(int(shape[-1]) / c)
        if self.group_size == 0:
            return int(shape[0])
        if len(shape) == 1:
            return math.ceil(int(shape[0]) / self.group_size)
        return int(math.prod(shape[:-1])) * math.ceil(int(shape[-1]) / self.group_size)

    def memory_bytes_for_shape(self, shape: tuple[int, ...]) -> int:
        n = int(math.prod(shape)) if len(shape) else 1
        return math.ceil(n * self.weight_bits / 8.0) + math.ceil(self.scale_count_for_shape(shape) * self.scale_bits / 8.0)

    def effective_bits_for_shape(self, shape: tuple[int, ...]) -> float:
        n = int(math.prod(shape)) if len(shape) else 1
        return 8.0 * self.memory_bytes_for_shape(shape) / max(n, 1)


REGISTRY: dict[str, FormatSpec] = {}
FORMAT_ALIASES: dict[str, str] = {"NVINT2": "INT2", "NVINT3": "INT3"}   # format_registry.py:120-123


def register_format(spec: FormatSpec) -> FormatSpec:
    REGISTRY[spec.name] = spec
    return spec


def canonical_format_name(name: str) -> str:
    return FORMAT_ALIASES.get(name, name)


def aliases_for(name: str) -> tuple[str, ...]:
    canonical = canonical_format_name(name)
    return (canonical, *[a for a, t in FORMAT_ALIASES.items() if t == canonical])


def get_format(name: str) -> FormatSpec:
    canonical = canonical_format_name(name)
    if canonical not in REGISTRY:
        raise KeyError(f"Unknown format '{name}'. Available: {sorted((*REGISTRY, *FORMAT_ALIASES))}")
    return REGISTRY[canonical]


def list_formats(family: str | None = None) -> list[FormatSpec]:
    specs = REGISTRY.values() if family is None else [s for s in REGISTRY.values() if s.family == family]
    return sorted(specs, key=lambda s: s.effective_bits)


def _kernel_qdq(kfmt: str) -> Callable[[torch.Tensor], torch.Tensor]:
    def qdq(w: torch.Tensor) -> torch.Tensor:
        return _lib.cost_qdq(w, kfmt)
    qdq.__name__ = f"qdq_{kfmt.lower()}"
    return qdq


def _identity(x: torch.Tensor) -> torch.Tensor:
    return x


def _clone(x: torch.Tensor) -> torch.Tensor:
    return x.clone()


def _nv_cfg(act_bits: int):
    return dict(bits=4, group_size=16, sym=True, data_type="nv_fp", act_bits=act_bits, act_group_size=16,
                act_sym=True, act_data_type="nv_fp4_with_static_gs", act_dynamic=True)


def _mx_cfg(act_bits: int):
    return dict(bits=8, group_size=32, sym=True, data_type="mx_fp", act_bits=act_bits, act_group_size=32,
                act_sym=True, act_data_type="mx_fp", act_dynamic=True)


# name, weight_bits, group, scale_bits, scale dtype, element dtype, act bits, family, sm, kernel fmt, act quant
_TABLE = [
    ("NVFP4", 4, 16, 8, "fp8_e4m3", "fp4_e2m1", 4, "nv", 100, "NVFP4", True),
    ("NVFP4A16", 4, 16, 8, "fp8_e4m3", "fp4_e2m1", None, "nv", 100, "NVFP4", False),
    ("MXFP8", 8, 32, 8, "uint8_e8m0", "fp8_e4m3", 8, "mx", 100, "MXFP8", True),
    ("MXFP8_E4M3", 8, 32, 8, "uint8_e8m0", "fp8_e4m3", 8, "mx", 100, "MXFP8", True),
    ("MXFP8A16", 8, 32, 8, "uint8_e8m0", "fp8_e4m3", None, "mx", 80, "MXFP8", False),
    ("FP8_E4M3", 8, 0, 32, "fp32", "fp8_e4m3", 8, "fp", 90, "FP8_E4M3", True),
]

for (_n, _wb, _g, _sb, _sd, _ed, _ab, _fam, _sm, _kf, _aq) in _TABLE:
    register_format(FormatSpec(
        name=_n, weight_bits=_wb, group_size=_g, scale_bits=_sb, scale_dtype_name=_sd,
        weight_element_dtype=_ed, act_bits=_ab, act_dtype_name=_ed if _ab else None,
        act_group_size=(_g if _ab else None), family=_fam, min_capability_sm=_sm,
        autoround_config=(lambda _f=_fam, _a=_ab: _nv_cfg(_a or 16) if _f == "nv" else
                          _mx_cfg(_a or 16) if _f == "mx" else
                          dict(bits=8, group_size=-1, sym=True, data_type="fp8_e4m3", act_bits=8,
                               act_group_size=-1, act_sym=True, act_data_type="fp8_e4m3", act_dynamic=True)),
        quantize_dequantize=_kernel_qdq(_kf),
        activation_quantize_dequantize=_kernel_qdq(_kf) if _aq else _identity,
        kernel_format=_kf,
    ))

register_format(FormatSpec(
    name="BF16", weight_bits=16, group_size=0, scale_bits=0, scale_dtype_name="none",
    weight_element_dtype="bfloat16", family="fp", min_capability_sm=75,
    autoround_config=lambda: dict(bits=16, group_size=0, data_type="float", act_bits=16, act_data_type="float"),
    quantize_dequantize=_clone, activation_quantize_dequantize=_clone, kernel_format="BF16",
))


# The rest of the registry (format_registry.py:391-576).  Autoround metadata as the reference's
# _mx_autoround / _int_autoround / _plain_fp8_autoround build it (format_registry.py:337-365).
def _mx_ar(bits: int, act_bits: int) -> dict:
    return dict(bits=bits, group_size=32, sym=True, data_type="mx_fp", act_bits=act_bits, act_group_size=32,
                act_sym=True, act_data_type="mx_fp", act_dynamic=True)


def _int_ar(bits: int, gsize: int, act_bits: int = 16) -> dict:
    return dict(bits=bits, group_size=gsize, sym=True, data_type="int", act_bits=act_bits,
                act_group_size=gsize if act_bits <= 8 else 0, act_sym=True,
                act_data_type="int" if act_bits <= 8 else "float", act_dynamic=True)


def _fp8_ar(elt: str, act_bits: int = 8) -> dict:
    return dict(bits=8, group_size=-1, sym=True, data_type=elt, act_bits=act_bits, act_group_size=-1, act_sym=True,
                act_data_type=elt if act_bits == 8 else "float", act_dynamic=True)


for _n, _wb, _ed in (("MXFP4", 4, "fp4_e2m1"), ("MXFP6_E3M2", 6, "fp6_e3m2"), ("MXFP6_E2M3", 6, "fp6_e2m3"),
                     ("MXFP8_E5M2", 8, "fp8_e5m2")):
    register_format(FormatSpec(
        name=_n, weight_bits=_wb, group_size=32, scale_bits=8, scale_dtype_name="uint8_e8m0",
        weight_element_dtype=_ed, act_bits=_wb, act_dtype_name=_ed, act_group_size=32, family="mx",
        min_capability_sm=100, autoround_config=(lambda _b=_wb: _mx_ar(_b, _b)),
        quantize_dequantize=_kernel_qdq(_n), activation_quantize_dequantize=_kernel_qdq(_n), kernel_format=_n,
    ))

register_format(FormatSpec(
    name="FP8_E5M2", weight_bits=8, group_size=0, scale_bits=32, scale_dtype_name="fp32",
    weight_element_dtype="fp8_e5m2", act_bits=8, act_dtype_name="fp8_e5m2", act_group_size=0, family="fp",
    min_capability_sm=90, autoround_config=lambda: _fp8_ar("fp8_e5m2", 8),
    quantize_dequantize=_kernel_qdq("FP8_E5M2"), activation_quantize_dequantize=_kernel_qdq("FP8_E5M2"),
    kernel_format="FP8_E5M2",
))

for _n, _wb, _ed, _g, _sb, _sd, _fam, _sm, _ar in (
        ("INT3", 3, "int3", 16, 8, "fp8_e4m3", "nv", 100, lambda: _int_ar(3, 16, 16)),
        ("INT2", 2, "int2", 16, 8, "fp8_e4m3", "nv", 100, lambda: _int_ar(2, 16, 16)),
        ("NVFP3", 3, "fp3_e2m0", 16, 8, "fp8_e4m3", "nv", 100, lambda: _int_ar(3, 16, 16)),
        ("INT8_W8A16", 8, "int8", 0, 16, "fp16", "int", 70, lambda: _int_ar(8, -1, 16)),
        ("INT4_W4A16_g128", 4, "int4", 128, 16, "fp16", "int", 70, lambda: _int_ar(4, 128, 16))):
    register_format(FormatSpec(
        name=_n, weight_bits=_wb, group_size=_g, scale_bits=_sb, scale_dtype_name=_sd, weight_element_dtype=_ed,
        act_bits=None, family=_fam, min_capability_sm=_sm, autoround_config=_ar,
        quantize_dequantize=_kernel_qdq(_n), activation_quantize_dequantize=_identity, kernel_format=_n,
    ))

# Source-FP8 passthrough: the per-Linear quantize_dequantize is a clone (format_registry.py:563-576);
# the batched cost path quantizes it by its element dtype (E4M3, groups of 128, real scale).
register_format(FormatSpec(
    name="FP8_SOURCE", weight_bits=8, group_size=128, scale_bits=32, scale_dtype_name="fp32",
    weight_element_dtype="fp8_e4m3", scale_block_shape=(128, 128), act_bits=None, family="fp",
    min_capability_sm=89,
    autoround_config=lambda: dict(bits=8, group_size=128, data_type="fp8_e4m3", sym=True, act_bits=16,
                                  act_data_type="float"),
    quantize_dequantize=_clone, activation_quantize_dequantize=_clone, kernel_format="BF16",
))

# Registration order of the reference (format_registry.py:368-576); list_formats sorts stably,
# so formats of equal effective bits keep this order.
_REFERENCE_ORDER = ("NVFP4", "NVFP4A16", "MXFP4", "MXFP6_E3M2", "MXFP6_E2M3", "MXFP8", "MXFP8_E4M3", "MXFP8_E5M2",
                    "MXFP8A16", "FP8_E4M3", "FP8_E5M2", "INT3", "INT2", "NVFP3", "INT8_W8A16", "INT4_W4A16_g128",
                    "BF16", "FP8_SOURCE")
_ordered = {n: REGISTRY[n] for n in _REFERENCE_ORDER}
REGISTRY.clear()
REGISTRY.update(_ordered)
