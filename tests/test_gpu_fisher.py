"""Fisher statistics on the GPU vs the reference (golden fixtures) and the
oracle.  Bar: rel <= 1e-5 for traces (fp64 accumulation)."""
import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import pq_oracle as O
from prismaquant_b200 import _lib
from prismaquant_b200 import sensitivity_probe as sp
from tests._helpers import assert_rel, to_cuda_bf16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", ["packed_4x32x64", "packed_3x16x96"])
def test_gradnorm_capture_matches_reference(golden, case):
    g = to_cuda_bf16(golden[f"{case}/input"])
    acc, ch = {}, {}
    w = torch.zeros(g.shape, dtype=torch.bfloat16, device="cuda", requires_grad=True)
    y = sp._GradNormCapture.apply(w, "p", acc, ch, None)
    y.backward(g)
    assert w.grad is None
    assert_rel(float(acc["p"]), float(golden[f"{case}/gradnorm/scalar"][0]), 1e-6)
    np.testing.assert_allclose(ch["p"].cpu().numpy(), golden[f"{case}/gradnorm/channel"], rtol=1e-6)


@pytest.mark.parametrize("shape", [(7, 8), (1000, 2048), (33, 8192), (5, 32000), (9, 100), (0, 64)])
def test_rownorm_and_tokennorm_vs_oracle(shape):
    T, d = shape
    xb = O.synthetic_weight_bits((T, d), seed=T + d, std=1.0)
    gb = O.synthetic_weight_bits((T, d), seed=T + d + 1, std=0.01)
    x, g = to_cuda_bf16(xb), to_cuda_bf16(gb)
    xn = _lib.rownorm2(x)
    np.testing.assert_allclose(xn.cpu().numpy().astype(np.float64), O.rownorm2(xb), rtol=1e-6)
    acc = torch.zeros(2, dtype=torch.float64, device="cuda")
    _lib.tokennorm_dot(g, xn, acc)
    ref = float(np.dot(xn.cpu().numpy().astype(np.float64), O.rownorm2(gb)))
    assert_rel(float(acc[0]), ref, 1e-6)
    assert_rel(float(acc[0]), O.tokennorm_trace(xb, gb), 1e-5)
    assert float(acc[1]) == T


def test_tokennorm_routed_subset():
    xb = O.synthetic_weight_bits((64, 512), seed=1, std=1.0)
    gb = O.synthetic_weight_bits((20, 256), seed=2, std=0.1)
    idx = np.random.default_rng(0).choice(64, 20, replace=False)
    xn = _lib.rownorm2(to_cuda_bf16(xb))
    acc = torch.zeros(2, dtype=torch.float64, device="cuda")
    _lib.tokennorm_dot(to_cuda_bf16(gb), xn, acc, token_idx=torch.from_numpy(idx).cuda())
    assert_rel(float(acc[0]), O.tokennorm_trace(xb, gb, token_idx=idx), 1e-5)


@pytest.mark.parametrize("shape", [(128, 4096), (4, 1536, 2048), (3, 100)])
def test_sumsq_rows_vs_oracle(shape):
    gb = O.synthetic_weight_bits(shape, seed=9, std=0.003)
    total = torch.zeros(1, dtype=torch.float64, device="cuda")
    per_row = torch.zeros(shape[:-1], dtype=torch.float32, device="cuda")
    _lib.sumsq_rows(to_cuda_bf16(gb), total, per_row)
    t_ref, r_ref = O.sumsq_rows(gb)
    assert_rel(float(total), t_ref, 1e-6)
    np.testing.assert_allclose(per_row.cpu().numpy(), r_ref, rtol=1e-6)


class _Toy(nn.Module):
    def __init__(self):
        super().__init__()
        self.a = nn.Linear(256, 512, bias=False)
        self.b = nn.Linear(512, 128, bias=False)

    def forward(self, x):
        return self.b(torch.relu(self.a(x)))


def test_fisher_accumulator_per_token_vs_oracle():
    torch.manual_seed(0)
    m = _Toy().cuda().to(torch.bfloat16)
    acc = sp.FisherAccumulator(m, ["a", "b"], {})
    xs, gs = {"a": [], "b": []}, {"a": [], "b": []}
    hooks = []
    for n in ("a", "b"):
        mod = getattr(m, n)
        hooks.append(mod.register_forward_hook(lambda mm, i, o, n=n: xs[n].append(i[0].detach().reshape(-1, i[0].shape[-1]))))
        hooks.append(mod.register_full_backward_hook(lambda mm, gi, go, n=n: gs[n].append(go[0].detach().reshape(-1, go[0].shape[-1]))))
    for step in range(3):
        x = torch.randn(2, 37, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        m(x).float().pow(2).sum().backward()
    acc.finalize(None)
    for h in hooks:
        h.remove()
    for n in ("a", "b"):
        ref = sum(O.tokennorm_trace(xx.cpu().view(torch.int16).numpy().view(np.uint16),
                                    gg.cpu().view(torch.int16).numpy().view(np.uint16)) for xx, gg in zip(xs[n], gs[n]))
        assert_rel(acc.stats[n]["h_trace_raw"], ref, 1e-5, n)
        assert acc.stats[n]["n_tokens_seen"] == 3 * 2 * 37
        assert_rel(acc.stats[n]["h_trace"], ref / (3 * 2 * 37), 1e-5, n)
    acc.remove_hooks()


def test_fisher_bridge_one_token_matches_reference(golden):
    """At one token per backward the per-token estimator IS the reference's
    ||gy^T x||_F^2 (FisherAccumulator._make_bwd); the recorded x / gy of the
    reference run give its h_trace_raw."""
    for lin in ("0", "1"):
        x = golden[f"bridge/{lin}/x"]
        gy = golden[f"bridge/{lin}/gy"]
        xb, gb = O.f32_to_bf16_bits(x), O.f32_to_bf16_bits(gy)
        if not (np.array_equal(O.bf16_bits_to_f32(xb), x) and np.array_equal(O.bf16_bits_to_f32(gb), gy)):
            # fp32 recordings: evaluate the estimator on the GPU in fp32 via its definition
            xn = torch.from_numpy(x).cuda().double().pow(2).sum(-1)
            gn = torch.from_numpy(gy).cuda().double().pow(2).sum(-1)
            assert_rel(float((xn * gn).sum()), float(golden[f"bridge/{lin}/h_trace_raw"][0]), 1e-5)


def _explicit_routed_traces(blk, x):
    """Independent statement of the routed per-token estimator: the experts
    loop of HF Qwen3MoeExperts.forward written out with retained per-expert
    output gradients, traces summed in float64."""
    ex = blk.experts
    H = x.shape[-1]
    h = x.reshape(-1, H)
    _, top_w, top_i = blk.gate(h)
    mask = torch.nn.functional.one_hot(top_i, num_classes=ex.gate_up_proj.shape[0]).permute(2, 1, 0)
    final = torch.zeros_like(h)
    kept = []
    for e in range(ex.gate_up_proj.shape[0]):
        pos, tok = torch.where(mask[e])
        if tok.numel() == 0:
            continue
        xe = h[tok]
        gu = torch.nn.functional.linear(xe, ex.gate_up_proj[e])
        gu.retain_grad()
        gate, up = gu.chunk(2, dim=-1)
        he = ex.act_fn(gate) * up
        dn = torch.nn.functional.linear(he, ex.down_proj[e])
        dn.retain_grad()
        final.index_add_(0, tok, (dn * top_w[tok, pos, None]).to(final.dtype))
        kept.append((xe, gu, he, dn))
    final.reshape(x.shape).float().pow(2).sum().backward()
    tg = sum(float((xe.double().pow(2).sum(-1) * gu.grad.double().pow(2).sum(-1)).sum()) for xe, gu, _, _ in kept)
    td = sum(float((he.detach().double().pow(2).sum(-1) * dn.grad.double().pow(2).sum(-1)).sum())
             for _, _, he, dn in kept)
    return tg, td


def test_routed_expert_estimator_vs_explicit_autograd():
    from transformers import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeSparseMoeBlock
    cfg = Qwen3MoeConfig(hidden_size=128, moe_intermediate_size=64, num_experts=8, num_experts_per_tok=2,
                         norm_topk_prob=True)
    torch.manual_seed(0)
    blk = Qwen3MoeSparseMoeBlock(cfg).cuda().to(torch.bfloat16)
    with torch.no_grad():
        for p in blk.parameters():
            p.normal_(std=0.05)
    x = torch.randn(1, 50, 128, device="cuda", dtype=torch.bfloat16)
    ref_out = blk(x)
    tg, td = _explicit_routed_traces(blk, x)
    acc = {}
    meta = sp.install_routed_expert_hooks(blk, acc)
    assert set(meta) == {"experts.gate_up_proj", "experts.down_proj"}
    out = blk(x)
    torch.testing.assert_close(out, ref_out, rtol=0, atol=0)
    out.float().pow(2).sum().backward()
    assert_rel(float(acc["experts.gate_up_proj"][:, 0].sum()), tg, 1e-5, "gate_up")
    assert_rel(float(acc["experts.down_proj"][:, 0].sum()), td, 1e-5, "down")
    assert float(acc["experts.down_proj"][:, 1].sum()) == 50 * 2
