"""The compressed-tensors quantization_config builder and the config.json writer against the
reference's own outputs (tests/golden/qconfig_cases.json, made by tests/golden/make_golden.py
`qconfig` from export_native_compressed.py:3206-3478, 4134-4186).  The reference's model
profiles are replayed as the tables recorded beside each case."""
import json
import re
from pathlib import Path

import pytest

from prismaquant_b200 import quantization_config as qc

GOLDEN = json.loads((Path(__file__).parent / "golden" / "qconfig_cases.json").read_text())


class TableProfile:
    """A model profile answered from recorded tables."""

    def __init__(self, names, moe=None, mtp=None):
        self.names, self.moe, self.mtp = names, moe, mtp

    def to_vllm_internal_name(self, name):
        return self.names[name]

    def per_expert_moe_regex(self):
        return self.moe

    def per_expert_mtp_regex(self):
        return self.mtp


def _profile(case):
    return TableProfile(case["names"], case["moe_regex"], case["mtp_regex"])


@pytest.mark.parametrize("i", range(len(GOLDEN["build"])))
def test_build_matches_reference(i):
    case = GOLDEN["build"][i]
    args = (case["assignment"], set(case["bf16_passthrough"]), case["extra_ignore"])
    kw = dict(profile=_profile(case), packed_mapping=case["packed_mapping"])
    if "error" in case["want"]:
        with pytest.raises({"RuntimeError": RuntimeError, "KeyError": KeyError}[case["want"]["error"]]):
            qc.build_quantization_config(*args, **kw)
        return
    got = qc.build_quantization_config(*args, **kw)
    assert json.dumps(got) == json.dumps(case["want"])   # same keys, values and order


@pytest.mark.parametrize("i", range(len(GOLDEN["write"])))
def test_config_json_matches_reference(i, tmp_path):
    case = GOLDEN["write"][i]
    src, dst = tmp_path / "src", tmp_path / "dst"
    src.mkdir()
    dst.mkdir()
    (src / "config.json").write_text(json.dumps(case["src_config"]))
    qc.write_config_with_quantization(src, dst, case["assignment"], set(case["bf16_passthrough"]), (),
                                      case["prune_manifest"], packed_mapping={})
    assert (dst / "config.json").read_text() == case["want_text"]


def test_prune_manifest_must_agree(tmp_path):
    (tmp_path / "config.json").write_text(json.dumps({"num_experts": 8}))
    with pytest.raises(RuntimeError):
        qc.write_config_with_quantization(tmp_path, tmp_path, {"a.b": "NVFP4"}, set(), (),
                                          {"x": {"num_experts_kept": 4}, "y": {"num_experts_kept": 6}})


def test_target_list_collapses_experts_and_matches_every_name():
    names = [f"model.layers.{l}.mlp.experts.{e}.{p}_proj" for l in (1, 12) for e in range(64)
             for p in ("gate", "up", "down")]
    sparse = [f"model.layers.3.mlp.experts.{e}.down_proj" for e in (0, 7, 9)]
    plain = ["model.layers.0.self_attn.q_proj", "lm_head"]
    targets = qc.build_target_list(names + sparse + plain + ["re:^x$"])
    assert len(targets) == 2 + 1 + 6 + 1
    pats = [re.compile(t[3:]) for t in targets]
    for n in names + sparse + plain:
        assert any(p.match(n) for p in pats), n
    assert not any(p.match("model.layers.3.mlp.experts.1.down_proj") for p in pats)


def test_packed_expert_regexes_pin_layer_and_projections():
    moe = "re:^language_model[.]model[.]layers[.][0-9]+[.]mlp[.]experts[.][0-9]+[.](gate|up|down)_proj$"
    prof = TableProfile({}, moe=moe)
    (r,) = qc.packed_expert_ignore_regexes("model.layers.7.mlp.experts.gate_up_proj", prof)
    pat = re.compile(r[3:])
    assert pat.match("language_model.model.layers.7.mlp.experts.3.up_proj")
    assert not pat.match("language_model.model.layers.7.mlp.experts.3.down_proj")
    assert not pat.match("language_model.model.layers.17.mlp.experts.3.up_proj")
    two = qc.packed_expert_ignore_regexes("model.layers.7.mlp.experts.down_proj", TableProfile({}))
    assert len(two) == 2 and all("layers[.]7[.]" in t for t in two)
    assert qc.packed_expert_ignore_regexes("model.layers.7.mlp.down_proj", prof) == []
