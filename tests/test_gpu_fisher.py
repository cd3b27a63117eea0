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


@pytest.mark.parametrize("shape", [(4, 96, 64), (3, 16, 100), (2, 40)])
def test_gradnorm_capture_full_accumulator(shape):
    """_GradNormCapture with all three accumulators (sensitivity_probe.py:451-503): the [E, M, N]
    accumulator is h += g.float()^2 in fp32, bit-exact with the reference's add, over two
    backwards; the scalar and channel sums as before."""
    gs = [to_cuda_bf16(O.synthetic_weight_bits(shape, seed=40 + k, std=0.01)) for k in range(2)]
    acc, ch, full = {}, {}, {}
    for g in gs:
        w = torch.zeros(shape, dtype=torch.bfloat16, device="cuda", requires_grad=True)
        sp._GradNormCapture.apply(w, "p", acc, ch, full).backward(g)
        assert w.grad is None
    want = torch.zeros(shape, dtype=torch.float32)
    for g in gs:
        want.add_(g.cpu().float().pow(2))          # the reference's CPU accumulation
    assert torch.equal(full["p"].cpu(), want)
    tot = sum(float(g.double().pow(2).sum()) for g in gs)
    assert_rel(float(acc["p"]), tot, 1e-6)
    if len(shape) >= 2:
        np.testing.assert_allclose(ch["p"].cpu().numpy(), sum(g.float().pow(2).sum(-1) for g in gs).cpu().numpy(),
                                   rtol=1e-5)


class _PackedExpertsToy(nn.Module):   # class name holds "expert"; owns packed gate_up_proj / down_proj
    def __init__(self, E=4, H=64, I=32):
        super().__init__()
        self.gate_up_proj = nn.Parameter(torch.randn(E, 2 * I, H) * 0.05)
        self.down_proj = nn.Parameter(torch.randn(E, H, I) * 0.05)

    def forward(self, x):   # every expert sees every token (dense mixture), enough for the hooks
        h = torch.einsum("th,emh->etm", x, self.gate_up_proj)
        g, u = h.chunk(2, dim=-1)
        return torch.einsum("eti,ehi->th", torch.nn.functional.silu(g) * u, self.down_proj)


class _MoEToy(nn.Module):
    def __init__(self):
        super().__init__()
        self.model = nn.Module()
        self.model.layers = nn.ModuleList([nn.Module()])
        self.model.layers[0].mlp = nn.Module()
        self.model.layers[0].mlp.experts = _PackedExpertsToy()
        self.model.layers[0].mlp.up = nn.Linear(64, 64, bias=False)

    def forward(self, x):
        return self.model.layers[0].mlp.experts(self.model.layers[0].mlp.up(x))


def _packed_grads(model, xs):
    """The packed parameters' plain autograd gradients for each backward (the reference's g)."""
    ex = model.model.layers[0].mlp.experts
    out = []
    for x in xs:
        ex.zero_grad(set_to_none=True)
        model(x).float().pow(2).sum().backward()
        out.append({n: getattr(ex, n).grad.detach().clone() for n in ("gate_up_proj", "down_proj")})
    return out


def test_install_packed_expert_hooks_through_a_packed_module():
    """install_packed_expert_hooks on a module that owns packed experts (sensitivity_probe.py:555-728):
    the forward is unchanged, no .grad is kept on the packed leaves, and the scalar / channel / full
    accumulators equal sum(g^2) / sum_n g^2 / g^2 of the plain autograd gradients."""
    torch.manual_seed(0)
    model = _MoEToy().cuda().to(torch.bfloat16)
    xs = [torch.randn(37, 64, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
    ref_out = model(xs[0]).detach()
    grads = _packed_grads(model, xs)
    ex = model.model.layers[0].mlp.experts
    ex.zero_grad(set_to_none=True)
    scalar, chan, full = {}, {}, {}
    meta = sp.install_packed_expert_hooks(model, scalar, chan, full)
    q = "model.layers.0.mlp.experts"
    assert set(meta) == {f"{q}.gate_up_proj", f"{q}.down_proj"}
    assert meta[f"{q}.gate_up_proj"]["num_experts"] == 4 and meta[f"{q}.down_proj"]["in_features"] == 32
    torch.testing.assert_close(model(xs[0]).detach(), ref_out, rtol=0, atol=0)
    ex.zero_grad(set_to_none=True)
    for x in xs:
        model(x).float().pow(2).sum().backward()
    assert ex.gate_up_proj.grad is None and ex.down_proj.grad is None
    for pn in ("gate_up_proj", "down_proj"):
        name = f"{q}.{pn}"
        g = [gr[pn] for gr in grads]
        assert_rel(float(scalar[name]), sum(float(t.double().pow(2).sum()) for t in g), 1e-5, pn)
        np.testing.assert_allclose(chan[name].cpu().numpy(), sum(t.float().pow(2).sum(-1) for t in g).cpu().numpy(),
                                   rtol=1e-5)
        want = torch.zeros_like(full[name])
        for t in g:
            want.add_(t.float().pow(2))
        assert torch.equal(full[name], want)


def test_fisher_accumulator_hooks_packed_experts():
    """FisherAccumulator(hook_packed_experts=True) on a model with packed experts: the packed
    parameters get stats entries with the reference's schema, h_trace_raw = sum over backwards of
    sum(g^2), tokens counted by the experts' forward hook, and the tracked Linear its own stats."""
    torch.manual_seed(1)
    model = _MoEToy().cuda().to(torch.bfloat16)
    xs = [torch.randn(21, 64, device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    grads = _packed_grads(model, xs)
    model.model.layers[0].mlp.experts.zero_grad(set_to_none=True)
    acc = sp.FisherAccumulator(model, ["model.layers.0.mlp.up"], {}, hook_packed_experts=True)
    for x in xs:
        model(x).float().pow(2).sum().backward()
    acc.finalize(None)
    q = "model.layers.0.mlp.experts"
    for pn in ("gate_up_proj", "down_proj"):
        st = acc.stats[f"{q}.{pn}"]
        assert {"h_trace_raw", "h_w2_sum_raw", "n_params", "num_experts", "n_tokens_seen", "h_trace"} <= set(st)
        assert_rel(st["h_trace_raw"], sum(float(gr[pn].double().pow(2).sum()) for gr in grads), 1e-5, pn)
        assert st["n_tokens_seen"] == 3 * 21
        assert st["h_trace"] == pytest.approx(st["h_trace_raw"] / 63)
    assert acc.stats["model.layers.0.mlp.up"]["n_tokens_seen"] == 63
    acc.remove_hooks()


BRIDGE = __import__("pathlib").Path(__file__).resolve().parent / "golden" / "fisher_bridge_bf16.npz"


@pytest.mark.parametrize("n", ["0", "1"])
def test_fisher_bridge_kernels_match_reference(n):
    """At one token per backward the reference's ||gy^T x||_F^2 is the per-token product of squared
    norms.  The reference ran FisherAccumulator on bf16-valued inputs and output gradients
    (tests/golden/fisher_bridge_bf16.npz); the same numbers go through this package's
    FisherAccumulator on the GPU (its hooks call pq_rownorm2 and pq_tokennorm_dot), and its
    h_trace_raw must match the reference's within 1e-5."""
    d = np.load(BRIDGE)
    x = torch.from_numpy(d[f"bridge16/{n}/x"]).view(torch.bfloat16).cuda()
    gy = torch.from_numpy(d[f"bridge16/{n}/gy"]).view(torch.bfloat16).cuda()
    w = torch.from_numpy(d[f"bridge16/{n}/w"]).view(torch.bfloat16).cuda()
    lin = nn.Linear(w.shape[1], w.shape[0], bias=False, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(w)
    model = nn.ModuleDict({n: lin})
    calls = []
    orig = _lib.tokennorm_dot

    def counted(*a, **k):
        calls.append(1)
        return orig(*a, **k)
    sp._lib.tokennorm_dot = counted
    try:
        acc = sp.FisherAccumulator(model, [n], {}, hook_packed_experts=False, estimator="per_token")
        for t in range(x.shape[0]):
            xi = x[t:t + 1].clone().requires_grad_(True)
            lin(xi).backward(gy[t:t + 1])
        acc.finalize(None)
    finally:
        sp._lib.tokennorm_dot = orig
    assert len(calls) == x.shape[0]
    assert acc.stats[n]["n_tokens_seen"] == int(d[f"bridge16/{n}/n_tokens_seen"][0])
    assert_rel(acc.stats[n]["h_trace_raw"], float(d[f"bridge16/{n}/h_trace_raw"][0]), 1e-5, n)


def test_tokennorm_seg_vs_oracle():
    """pq_tokennorm_dot_seg: rows of g grouped by expert, each expert's sum of xnorm[token] *
    ||g_r||^2 and its row count, against the per-expert oracle (rel 1e-5); empty experts stay 0."""
    rng = np.random.default_rng(4)
    T, d, E = 300, 768, 9
    xb = O.synthetic_weight_bits((T, 2048), seed=5, std=1.0)
    sizes = [37, 0, 120, 1, 64, 0, 250, 8, 40]
    toks = [rng.choice(T, n, replace=False) for n in sizes]
    tok = np.concatenate(toks).astype(np.int64)
    seg = np.repeat(np.arange(E, dtype=np.int32), sizes)
    gb = O.synthetic_weight_bits((tok.size, d), seed=6, std=0.02)
    xn = _lib.rownorm2(to_cuda_bf16(xb))
    acc = torch.zeros(E, 2, dtype=torch.float64, device="cuda")
    _lib.tokennorm_dot_seg(to_cuda_bf16(gb), xn, torch.from_numpy(seg).cuda(), acc,
                           token_idx=torch.from_numpy(tok).cuda())
    off = 0
    for e, n in enumerate(sizes):
        if n == 0:
            assert float(acc[e, 0]) == 0.0 and float(acc[e, 1]) == 0.0
            continue
        want = O.tokennorm_trace(xb, gb[off:off + n], token_idx=tok[off:off + n])
        assert_rel(float(acc[e, 0]), want, 1e-5, str(e))
        assert float(acc[e, 1]) == n
        off += n


def test_routed_hooks_one_launch_per_projection(monkeypatch):
    """The routed estimator's backward is one pq_tokennorm_dot_seg launch per projection,
    whatever the number of experts hit."""
    from transformers import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeSparseMoeBlock
    cfg = Qwen3MoeConfig(hidden_size=128, moe_intermediate_size=64, num_experts=16, num_experts_per_tok=4,
                         norm_topk_prob=True)
    torch.manual_seed(2)
    blk = Qwen3MoeSparseMoeBlock(cfg).cuda().to(torch.bfloat16)
    calls = []
    orig = _lib.tokennorm_dot_seg
    monkeypatch.setattr(_lib, "tokennorm_dot_seg", lambda *a, **k: (calls.append(1), orig(*a, **k))[1])
    acc = {}
    sp.install_routed_expert_hooks(blk, acc)
    x = torch.randn(1, 200, 128, device="cuda", dtype=torch.bfloat16)
    blk(x).float().pow(2).sum().backward()
    assert len(calls) == 2
    assert float(acc["experts.gate_up_proj"][:, 1].sum()) == 200 * 4
