"""The compressed-tensors `quantization_config` of a mixed-format checkpoint, and the
`config.json` that carries it (export_native_compressed.py:3206-3478, 4134-4186).

Host-side only: it turns the per-Linear format assignment into the serving configuration
that vLLM's compressed-tensors loader dispatches on.  What it emits:

* one config group per format, each with the format's fixed scheme (the tables below are the
  compressed-tensors scheme dicts the reference writes, export_native_compressed.py:2989-3083),
  the format with the most targets last, as the catch-all, with the profile's per-expert regexes;
* targets as anchored regexes in the serving engine's internal naming (the profile's
  `to_vllm_internal_name`), per-expert Linears collapsed to one regex per (layer, projection);
* packed 3-D expert tensors (`<block>.experts.gate_up_proj` / `.down_proj`) replaced by one
  regex over that block's per-expert projections, which is the form the MoE scheme dispatch
  probes; gate_up and down of one block must share a format;
* with the engine's packed-module mapping (`{"qkv_proj": ["q_proj", "k_proj", "v_proj"], ...}`),
  the fused module's name beside its siblings when all of them share a format, and every
  sibling of a BF16 member in `ignore`;
* `ignore`: BF16 Linears, the passthrough set, `extra_ignore`, and the per-layer regexes of BF16
  packed experts.

The profile is any object with the reference's profile methods (`to_vllm_internal_name`,
`per_expert_moe_regex`, `per_expert_mtp_regex`, optionally `vllm_architecture_class`); the
reference's own profiles qualify.  Without one, names are kept as they are and there are no
per-expert regexes.  The packed-module mapping is passed in, or looked up in vLLM's model
registry from the profile's architecture when vLLM can be imported (empty otherwise).
"""
from __future__ import annotations

import copy
import json
import re
from collections import defaultdict
from pathlib import Path
from typing import Iterable

__all__ = ["SCHEMES", "MOE_EXPERT_COUNT_FIELDS", "IdentityProfile", "build_target_list",
           "packed_expert_ignore_regexes", "build_quantization_config",
           "write_config_with_quantization", "vllm_packed_mapping"]

# compressed-tensors scheme per format (export_native_compressed.py:2989-3083, 3195-3203): the
# loader reads these keys, so they are kept as the reference writes them
_NVFP4 = {
    "format": "nvfp4-pack-quantized",
    "weights": {"num_bits": 4, "type": "float", "strategy": "tensor_group", "group_size": 16,
                "symmetric": True, "dynamic": False, "scale_dtype": "torch.float8_e4m3fn",
                "zp_dtype": "torch.float8_e4m3fn", "observer": "memoryless_minmax"},
    "input_activations": {"num_bits": 4, "type": "float", "strategy": "tensor_group", "group_size": 16,
                          "symmetric": True, "dynamic": "local", "observer": "static_minmax",
                          "scale_dtype": "torch.float8_e4m3fn", "zp_dtype": "torch.float8_e4m3fn"},
}
_MXFP8 = {
    "format": "mxfp8-quantized",
    "weights": {"num_bits": 8, "type": "float", "strategy": "group", "group_size": 32,
                "symmetric": True, "dynamic": False, "scale_dtype": "torch.uint8",
                "zp_dtype": "torch.uint8", "observer": "memoryless_minmax"},
    "input_activations": {"num_bits": 8, "type": "float", "strategy": "group", "group_size": 32,
                          "symmetric": True, "dynamic": True, "scale_dtype": "torch.uint8",
                          "zp_dtype": "torch.uint8"},
}


def _int_scheme(bits: int) -> dict:
    """Symmetric integer weights in the NVFP4 scale envelope (g16, E4M3 group scales), no
    activation quantization."""
    return {"format": "pack-quantized",
            "weights": {"num_bits": bits, "type": "int", "strategy": "tensor_group", "group_size": 16,
                        "symmetric": True, "dynamic": False, "scale_dtype": "torch.float8_e4m3fn",
                        "zp_dtype": "torch.float8_e4m3fn", "observer": "memoryless_minmax"}}


_FP8_SOURCE = {   # the source checkpoint's 128x128 block FP8, copied through
    "format": "float-quantized",
    "weights": {"num_bits": 8, "type": "float", "strategy": "block", "block_structure": [128, 128],
                "symmetric": True, "dynamic": False, "observer": "memoryless_minmax"},
    "input_activations": {"num_bits": 8, "type": "float", "strategy": "tensor", "symmetric": True,
                          "dynamic": True, "observer": "memoryless_minmax"},
}
SCHEMES = {"NVFP4": _NVFP4, "MXFP8": _MXFP8, "INT2": _int_scheme(2), "INT3": _int_scheme(3),
           "NVINT2": _int_scheme(2), "NVINT3": _int_scheme(3), "FP8_SOURCE": _FP8_SOURCE}

# config.json fields that hold an MoE expert count (export_native_compressed.py:1559-1564)
MOE_EXPERT_COUNT_FIELDS = ("num_experts", "num_local_experts", "num_routed_experts", "n_routed_experts")


class IdentityProfile:
    """Names kept as they are, no per-expert regexes, no engine architecture."""

    def to_vllm_internal_name(self, name: str) -> str:
        return name

    def per_expert_moe_regex(self):
        return None

    def per_expert_mtp_regex(self):
        return None

    def vllm_architecture_class(self):
        return None


def vllm_packed_mapping(profile) -> dict[str, list[str]]:
    """`{fused: [siblings]}` of the engine's model class for the profile's architecture
    (its `packed_modules_mapping`), or {} when there is no architecture, vLLM cannot be
    imported or does not know the class (model_profiles/vllm_registry.py:25-117)."""
    arch_of = getattr(profile, "vllm_architecture_class", None)
    arch = arch_of() if callable(arch_of) else None
    if not arch:
        return {}
    try:   # the registry's lazy entry: importing the one model module is enough
        from vllm.model_executor.models.registry import ModelRegistry
        entry = ModelRegistry.models.get(arch)
        cls = entry.load_model_cls() if entry is not None else None
    except Exception:
        return {}
    pm = getattr(cls, "packed_modules_mapping", None)
    if not isinstance(pm, dict):
        return {}
    return {k: list(v) for k, v in pm.items() if isinstance(v, list) and v}


def _anchored(name: str) -> str:
    return "re:^" + name.replace(".", "[.]") + "$"


# a per-expert Linear in the engine's naming, e.g. model.layers.10.mlp.experts.0.gate_proj
# (export_native_compressed.py:1311-1315)
_EXPERT_LINEAR = re.compile(r"^(?P<prefix>.*[.])layers[.](?P<L>\d+)[.](?P<inner>.*mlp)[.]"
                            r"experts[.](?P<E>\d+)[.](?P<proj>gate|up|down)_proj$")


def build_target_list(names: Iterable[str]) -> list[str]:
    """Regex targets of one config group (export_native_compressed.py:1318-1382): per-expert
    Linears become one regex per (prefix, layer, inner path, projection), `[0-9]+` when the
    experts present are exactly 0..n-1, else an alternation of the indices; other names become
    anchored regexes; names that already are regexes (`re:`) pass through.  Order: anchored
    names sorted by name, then the pass-through regexes sorted, then the collapsed ones sorted."""
    experts: dict[tuple[str, int, str, str], set[int]] = defaultdict(set)
    plain: list[str] = []
    given: list[str] = []
    for n in names:
        if n.startswith("re:"):
            given.append(n)
            continue
        m = _EXPERT_LINEAR.match(n)
        if m is None:
            plain.append(n)
        else:
            experts[(m["prefix"], int(m["L"]), m["inner"], m["proj"])].add(int(m["E"]))
    collapsed = []
    for (prefix, layer, inner, proj), ids in sorted(experts.items()):
        span = "[0-9]+" if ids == set(range(max(ids) + 1)) else "(" + "|".join(map(str, sorted(ids))) + ")"
        collapsed.append(f"re:^{prefix.replace('.', '[.]')}layers[.]{layer}[.]{inner.replace('.', '[.]')}"
                         f"[.]experts[.]{span}[.]{proj}_proj$")
    return [_anchored(n) for n in sorted(plain)] + sorted(given) + sorted(collapsed)


_PACKED_KEY = re.compile(r"^(.*\.)(experts)\.(gate_up_proj|down_proj|w\d|gate_proj|up_proj)$")
_LAYER_IN_KEY = re.compile(r"\.layers\.(\d+)\.")
_ANY_LAYER = re.compile(r"layers\[\.\]\[0-9\]\+")


def _pin(profile_regex: str, layer, projections: str) -> str:
    """The profile's per-expert regex narrowed to one layer and the given projections."""
    body = _ANY_LAYER.sub(lambda _m: f"layers[.]{layer}", profile_regex[3:], count=1)
    return "re:" + body.replace("(gate|up|down)_proj", f"({projections})")


def packed_expert_ignore_regexes(recipe_key: str, profile) -> list[str]:
    """`ignore` regexes for a BF16 packed-expert tensor (export_native_compressed.py:3085-3192):
    its per-expert projection names at dispatch time (gate_up splits into gate and up).  MTP
    keys (`mtp.`) use the profile's MTP regex or an `mtp.layers.N` pattern; body keys the
    profile's MoE regex, or both common layouts (`language_model.model.layers.N` and
    `model.layers.N`).  [] for other keys, or when a fallback pattern has no layer index."""
    m = _PACKED_KEY.match(recipe_key)
    if m is None:
        return []
    param = m.group(3)
    projections = {"gate_up_proj": "gate_proj|up_proj", "down_proj": "down_proj"}.get(param) or re.escape(param)
    lm = _LAYER_IN_KEY.search(recipe_key)
    layer = lm.group(1) if lm else None
    if recipe_key.startswith("mtp."):
        base = profile.per_expert_mtp_regex() if profile else None
        if base and base.startswith("re:"):
            return [_pin(base, layer, projections)]
        if layer is None:
            return []
        return [f"re:^mtp[.]layers[.]{layer}[.](?:moe[.])?experts[.][0-9]+[.]({projections})$"]
    base = profile.per_expert_moe_regex() if profile else None
    if base and base.startswith("re:"):
        return [_pin(base, layer, projections)]
    if layer is None:
        return []
    return [f"re:^{root}layers[.]{layer}[.](?:moe[.])?experts[.][0-9]+[.]({projections})$"
            for root in ("language_model[.]model[.]", "model[.]")]


_PACKED_TARGET = re.compile(r"^(.+\.experts)\.(gate_up_proj|down_proj)$")


def _block_regex(block: str) -> str:
    return "re:^" + block.replace(".", "[.]") + "[.][0-9]+[.](gate_proj|up_proj|down_proj)$"


def build_quantization_config(assignment: dict[str, str], bf16_passthrough: Iterable[str],
                              extra_ignore: Iterable[str] = (), *, profile=None,
                              packed_mapping: dict[str, list[str]] | None = None) -> dict:
    """The `quantization_config` dict for `assignment` ({recipe name: format}); {} when no
    name is quantized.  Same signature and output as export_native_compressed.py:3206-3478,
    plus `packed_mapping` (the engine's fused-module map; looked up from the profile when None).
    Raises RuntimeError when a packed expert block's gate_up and down differ in format, and
    KeyError for a format without a scheme (as the reference does)."""
    profile = profile or IdentityProfile()
    to_engine = profile.to_vllm_internal_name
    groups: dict[str, list[str]] = {}      # format -> engine names, in order of first use
    ignore: list[str] = [to_engine(n) for n in bf16_passthrough]
    ignore += [to_engine(n) for n in extra_ignore]
    for name, fmt in sorted(assignment.items()):
        if fmt == "BF16":
            ignore.append(to_engine(name))
            ignore += packed_expert_ignore_regexes(name, profile)
        else:
            groups.setdefault(fmt, []).append(to_engine(name))

    mapping = vllm_packed_mapping(profile) if packed_mapping is None else packed_mapping
    fused_of = {sib: fused for fused, sibs in mapping.items() for sib in sibs}
    if mapping:   # every sibling of a BF16 member is ignored too, seen or not
        ignored = set(ignore)
        for name, fmt in assignment.items():
            leaf = name.rsplit(".", 1)[-1]
            if fmt != "BF16" or leaf not in fused_of:
                continue
            for sib in mapping[fused_of[leaf]]:
                eng = to_engine(name[: -len(leaf)] + sib)
                if eng not in ignored:
                    ignore.append(eng)
                    ignored.add(eng)

    # packed 3-D expert tensors -> one regex over the block's per-expert projections
    block_state: dict[str, set[str]] = {}
    for fmt in groups:
        keep = []
        for eng in groups[fmt]:
            m = _PACKED_TARGET.match(eng)
            if m:
                block_state.setdefault(m.group(1), set()).add(fmt)
            else:
                keep.append(eng)
        groups[fmt] = keep
    keep = []
    for eng in ignore:
        m = None if eng.startswith("re:") else _PACKED_TARGET.match(eng)
        if m:
            block_state.setdefault(m.group(1), set()).add("IGNORE")
        else:
            keep.append(eng)
    ignore = keep
    for block, states in block_state.items():
        if len(states) > 1:
            raise RuntimeError(f"[export-stream] FusedMoE at {block!r} has mixed states across projections "
                               f"{states}; promote_moe_pair should have forced gate_up_proj and down_proj to "
                               f"share a scheme before this point.")
        (state,) = states
        if state == "IGNORE":
            ignore.append(_block_regex(block))
        else:
            groups.setdefault(state, []).append(_block_regex(block))

    if mapping:   # the fused module's name beside siblings that all share one state
        state_of: dict[tuple[str, str], str] = {}
        for fmt, names in groups.items():
            for eng in names:
                if "." in eng:
                    parent, leaf = eng.rsplit(".", 1)
                    state_of[(parent, leaf)] = fmt
        for eng in set(ignore):
            if "." in eng:
                parent, leaf = eng.rsplit(".", 1)
                state_of.setdefault((parent, leaf), "IGNORE")
        emitted: set[str] = set()
        for parent in {p for p, _ in state_of}:
            for fused, sibs in mapping.items():
                if len(sibs) < 2:
                    continue
                states = {state_of.get((parent, s)) for s in sibs}
                if None in states or len(states) != 1:
                    continue
                full = f"{parent}.{fused}"
                if full in emitted:
                    continue
                emitted.add(full)
                (state,) = states
                if state == "IGNORE":
                    ignore.append(full)
                else:
                    groups.setdefault(state, []).append(full)

    if not groups:
        return {}
    catchall = max(groups, key=lambda f: len(groups[f]))   # the first of the largest
    config_groups = {}
    for fmt in [f for f in groups if f != catchall] + [catchall]:
        scheme = copy.deepcopy(SCHEMES[fmt])
        scheme["targets"] = build_target_list(groups[fmt])
        if fmt == catchall:
            scheme["targets"] += [r for r in (profile.per_expert_moe_regex(), profile.per_expert_mtp_regex())
                                  if r is not None]
        config_groups[f"group_{len(config_groups)}"] = scheme
    return {"quant_method": "compressed-tensors", "format": "mixed-precision", "config_groups": config_groups,
            "ignore": sorted(set(ignore)), "quantization_status": "compressed"}


def write_config_with_quantization(src_model, out_dir, assignment: dict[str, str], bf16_passthrough: Iterable[str],
                                   extra_ignore: Iterable[str] = (), prune_manifest: dict[str, dict] | None = None,
                                   *, profile=None, packed_mapping: dict[str, list[str]] | None = None) -> None:
    """`out_dir/config.json`: the source model's config.json with `quantization_config` set
    (when any name is quantized) and, with a prune manifest, every MoE expert-count field (top
    level and `text_config`) set to the kept count (export_native_compressed.py:4134-4186).
    The reference detects the profile from the source model; here it is passed in."""
    cfg = json.loads((Path(src_model) / "config.json").read_text())
    qc = build_quantization_config(assignment, bf16_passthrough, extra_ignore, profile=profile,
                                   packed_mapping=packed_mapping)
    if qc:
        cfg["quantization_config"] = qc
    if prune_manifest:
        kept = {int(e["num_experts_kept"]) for e in prune_manifest.values()}
        if len(kept) != 1:
            raise RuntimeError(f"[export-stream] prune: manifest has inconsistent num_experts_kept across layers "
                               f"({sorted(kept)}). HF config carries a single scalar field — mixed per-layer counts "
                               f"need a schema change.")
        (k,) = kept
        for d in (cfg, cfg.get("text_config")):
            if isinstance(d, dict):
                for field in MOE_EXPERT_COUNT_FIELDS:
                    if isinstance(d.get(field), int) and d[field] != k:
                        print(f"[export-stream] config: {field} {d[field]} → {k}", flush=True)
                        d[field] = k
    with open(Path(out_dir) / "config.json", "w") as f:
        json.dump(cfg, f, indent=2)
