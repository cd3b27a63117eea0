"""pq_grad_sq_acc: the per-weight Fisher diagonal of one backward on the tensor cores
(sensitivity_probe.py:1114-1152): grad_w = bf16(gy^T x), g2 = bf16(grad_w^2), h += g2,
sums += (sum g2, sum bf16(g2 * bf16(w^2))).

grad_w is an fp32 accumulation over the tokens, so its bf16 rounding can differ from another
accumulation order (the reference's cuBLAS, or the fp64 product used here) by one bf16 ulp on a
few elements: h is held to bit equality on >= 99 % of elements and to 2^-5 relative on all.  The
sums are checked against the kernel's own h (its g2 values) at fp32-partial precision."""
import pytest
import torch

from oracle import pq_oracle as O
from tests._helpers import to_cuda_bf16

pytestmark = pytest.mark.gpu


def _bf16(x):
    return x.to(torch.bfloat16).float()


@pytest.mark.parametrize("t,m,n", [(300, 264, 520), (2048, 1024, 2048), (64, 8, 8), (1000, 512, 256),
                                   (4096, 256, 1536)])
def test_grad_sq_matches_fp64_product(t, m, n):
    from prismaquant_b200 import _lib
    gy = to_cuda_bf16(O.synthetic_weight_bits((t, m), seed=t + m, std=0.05))
    x = to_cuda_bf16(O.synthetic_weight_bits((t, n), seed=t + n + 1, std=1.0))
    w = to_cuda_bf16(O.synthetic_weight_bits((m, n), seed=m * n, std=0.02))
    h = torch.zeros(m, n, dtype=torch.float32, device="cuda")
    sums = torch.zeros(2, dtype=torch.float64, device="cuda")
    _lib.grad_sq_acc(gy, x, h, sums, w)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    d = gy.double().t() @ x.double()
    g = _bf16(d.float())
    want = _bf16(g * g)
    exact = (h == want).double().mean().item()
    assert exact >= 0.99, exact
    # grad_w's fp32 accumulation error is bounded by (t/16 + 4) 2^-23 sum_t |gy||x| (B).  Near a
    # bf16 rounding boundary bf16(grad_w) may move by one ulp (<= 2^-7 relative; the kernel and
    # cuBLAS agree there, the fp64 product rounds the other way), so g2 by 2 * 2^-7 plus its own
    # two bf16 roundings: 2^-5 relative; where terms cancel, by about 2 |d| B more
    b = (gy.double().abs().t() @ x.double().abs()) * ((t / 16 + 4) * 2.0 ** -23)
    tol = want.double().abs() * 2.0 ** -5 + 4.0 * (d.abs() + b) * b + 1e-30
    assert ((h.double() - want.double()).abs() <= tol).all()
    # the sums are those of the kernel's own g2 (= h after one call from zero)
    torch.testing.assert_close(sums[0], h.double().sum(), rtol=1e-6, atol=0)
    w2 = _bf16(w.float() * w.float())
    torch.testing.assert_close(sums[1], _bf16(h * w2).double().sum(), rtol=1e-6, atol=0)


def test_accumulates_over_backwards_and_without_weight():
    from prismaquant_b200 import _lib
    t, m, n = 512, 264, 384
    h = torch.zeros(m, n, dtype=torch.float32, device="cuda")
    sums = torch.zeros(2, dtype=torch.float64, device="cuda")
    ones = []
    for k in range(2):
        gy = to_cuda_bf16(O.synthetic_weight_bits((t, m), seed=10 + k, std=0.05))
        x = to_cuda_bf16(O.synthetic_weight_bits((t, n), seed=20 + k, std=1.0))
        h1 = torch.zeros_like(h)
        s1 = torch.zeros_like(sums)
        _lib.grad_sq_acc(gy, x, h1, s1)
        _lib.grad_sq_acc(gy, x, h, sums)
        ones.append((h1, s1))
    torch.cuda.synchronize()
    assert torch.equal(h, ones[0][0] + ones[1][0])   # h += g2 is exact per call, deterministic
    torch.testing.assert_close(sums, ones[0][1] + ones[1][1], rtol=1e-12, atol=0)
    assert sums[1].item() == 0.0


def test_validation():
    from prismaquant_b200 import _lib
    gy = torch.zeros(4, 12, dtype=torch.bfloat16, device="cuda")
    x = torch.zeros(4, 16, dtype=torch.bfloat16, device="cuda")
    h = torch.zeros(12, 16, dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError):
        _lib.grad_sq_acc(gy, x, h, torch.zeros(2, dtype=torch.float64, device="cuda"))   # m = 12


from pathlib import Path   # noqa: E402

import numpy as np   # noqa: E402

DETAIL = Path(__file__).resolve().parent / "golden" / "fisher_detail.npz"


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).view(torch.bfloat16).cuda()


@pytest.mark.parametrize("n", ["0", "1"])
def test_kernel_against_reference_fixture(n):
    """Each recorded backward of the reference's FisherAccumulator (tests/golden/fisher_detail.npz)
    through pq_grad_sq_acc, its sums rounded to bf16 per backward as the reference's .sum() of a
    bf16 tensor: h_diag and the exact stats against the reference's own outputs.  The reference
    ran on the CPU (its bf16 GEMM accumulates in another order), so a few grad_w roundings differ."""
    from prismaquant_b200 import _lib
    d = np.load(DETAIL)
    x, gy, w = _t(d[f"detail/{n}/x"]), _t(d[f"detail/{n}/gy"]), _t(d[f"detail/{n}/w"])
    h = torch.zeros(w.shape, dtype=torch.float32, device="cuda")
    trace = w2 = 0.0
    for c in range(x.shape[0]):
        s = torch.zeros(2, dtype=torch.float64, device="cuda")
        _lib.grad_sq_acc(gy[c], x[c], h, s, w)
        trace += s.float().to(torch.bfloat16).double()[0].item()
        w2 += s.float().to(torch.bfloat16).double()[1].item()
    tokens = int(d[f"detail/{n}/n_tokens_seen"][0])
    got = (h.cpu() / tokens).numpy()
    want = d[f"detail/{n}/h_diag"]
    assert (got == want).mean() >= 0.9
    np.testing.assert_allclose(got, want, rtol=2.0 ** -5, atol=1e-6 * float(np.abs(want).max()))
    assert trace == pytest.approx(float(d[f"detail/{n}/h_trace_raw"][0]), rel=2.0 ** -7)
    assert w2 == pytest.approx(float(d[f"detail/{n}/h_w2_sum_raw"][0]), rel=2.0 ** -7)


def test_accumulator_writes_the_reference_detail_files(tmp_path):
    """FisherAccumulator(h_detail_dir=...) on the fixture's toy model on the GPU: the reference's
    file names and keys, stats with h_detail_path and the exact trace, and values equal to the
    reference's algorithm run in torch on the same GPU activations."""
    from prismaquant_b200 import sensitivity_probe as sp
    d = np.load(DETAIL)
    model = torch.nn.Sequential(torch.nn.Linear(64, 48, bias=False), torch.nn.Linear(48, 32, bias=False))
    model = model.to(device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        for n in ("0", "1"):
            model.get_submodule(n).weight.copy_(_t(d[f"detail/{n}/w"]))
    tracked = ["0", "1"]
    acc = sp.FisherAccumulator(model, tracked, {}, hook_packed_experts=False, h_detail_dir=tmp_path)
    xs, gys = {n: [] for n in tracked}, {n: [] for n in tracked}
    hooks = []
    for n in tracked:
        m = model.get_submodule(n)
        hooks.append(m.register_forward_hook(lambda mm, i, o, n=n: xs[n].append(i[0].detach().clone())))
        hooks.append(m.register_full_backward_hook(lambda mm, gi, go, n=n: gys[n].append(go[0].detach().clone())))
    inputs = _t(d["detail/0/x"])
    for c in range(inputs.shape[0]):
        model(inputs[c]).float().pow(2).sum().backward()
    acc.finalize(None)
    for h in hooks:
        h.remove()
    for n in tracked:
        blob = torch.load(tmp_path / f"{n}.pt", weights_only=False)
        assert set(blob) == {"h_diag", "name", "kind", "shape"} and blob["kind"] == "linear" and blob["name"] == n
        assert acc.stats[n]["h_detail_path"] == f"{n}.pt" and acc.stats[n]["n_tokens_seen"] == 80
        # the reference's algorithm (sensitivity_probe.py:1120-1141) in torch on the same activations
        h_ref = torch.zeros(blob["shape"], dtype=torch.float32, device="cuda")
        tr = w2 = 0.0
        wd = model.get_submodule(n).weight.detach()
        for x, gy in zip(xs[n], gys[n]):
            g2 = (gy.reshape(-1, gy.shape[-1]).t() @ x.reshape(-1, x.shape[-1])).pow(2)
            h_ref += g2.float()
            tr += float(g2.sum())
            w2 += float((g2 * wd.pow(2)).sum())
        got, want = blob["h_diag"].numpy(), (h_ref.cpu() / 80).numpy()
        assert (got == want).mean() >= 0.9
        np.testing.assert_allclose(got, want, rtol=2.0 ** -5, atol=1e-6 * float(np.abs(want).max()))
        assert acc.stats[n]["h_trace_raw"] == pytest.approx(tr, rel=2.0 ** -7)
        assert acc.stats[n]["h_w2_sum_raw"] == pytest.approx(w2, rel=2.0 ** -7)
        assert acc.stats[n]["h_trace"] == pytest.approx(acc.stats[n]["h_trace_raw"] / 80)


@pytest.mark.parametrize("n", ["0", "1"])
def test_production_layer_hooks_against_reference_fixture(n):
    """make_layer_fisher_hooks (the production probe's whole-batch hook pair,
    incremental_probe.py:1222-1262) on the fixture's recorded backwards: the reference's stats and
    its fp32 host accumulator of grad_w^2, within the same one-bf16-ulp allowance as above."""
    from prismaquant_b200 import sensitivity_probe as sp
    d = np.load(DETAIL)
    x, gy, w = _t(d[f"detail/{n}/x"]), _t(d[f"detail/{n}/gy"]), _t(d[f"detail/{n}/w"])
    lin = torch.nn.Linear(w.shape[1], w.shape[0], bias=False, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(w)
    saved, h_full = {}, {}
    stats = {n: {"h_trace_raw": 0.0, "h_w2_sum_raw": 0.0, "n_tokens_seen": 0}}
    make_fwd, make_bwd = sp.make_layer_fisher_hooks(saved, stats, h_full)
    fwd, bwd = make_fwd(n), make_bwd(n, lin)
    for c in range(x.shape[0]):
        fwd(lin, (x[c],), None)
        bwd(lin, None, (gy[c],))
    assert not saved
    st = stats[n]
    assert st["n_tokens_seen"] == int(d[f"detail/{n}/n_tokens_seen"][0])
    assert st["h_trace_raw"] == pytest.approx(float(d[f"detail/{n}/h_trace_raw"][0]), rel=2.0 ** -7)
    assert st["h_w2_sum_raw"] == pytest.approx(float(d[f"detail/{n}/h_w2_sum_raw"][0]), rel=2.0 ** -7)
    assert h_full[n].device.type == "cpu" and h_full[n].dtype == torch.float32
    got = (h_full[n] / st["n_tokens_seen"]).numpy()
    want = d[f"detail/{n}/h_diag"]
    assert (got == want).mean() >= 0.9
    np.testing.assert_allclose(got, want, rtol=2.0 ** -5, atol=1e-6 * float(np.abs(want).max()))


def test_run_probe_pass_reference_signature_and_pickle(tmp_path):
    """run_probe_pass with the reference's arguments (sensitivity_probe.py:1456-1472) on a small
    random-init bf16 Llama: one sequence per backward, the exact statistics from the tensor cores,
    the reference's pickle keys; each Linear's h_trace_raw equals the reference's algorithm
    (bf16 gy^T x per backward, squared, summed) run in torch on the same GPU activations."""
    import pickle

    from transformers import LlamaConfig, LlamaForCausalLM

    from prismaquant_b200 import sensitivity_probe as sp
    cfg = LlamaConfig(vocab_size=256, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=64,
                      tie_word_embeddings=False)
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg).cuda().to(torch.bfloat16)
    for p in model.parameters():
        p.requires_grad_(False)
    calib = torch.randint(0, 256, (3, 32), generator=torch.Generator().manual_seed(1))
    # record what the reference's hook would see, with plain hooks beside ours
    names = [n for n, m in model.named_modules() if isinstance(m, torch.nn.Linear) and "mlp" in n]
    xs, gys, hooks = {n: [] for n in names}, {n: [] for n in names}, []
    for n in names:
        m = model.get_submodule(n)
        hooks.append(m.register_forward_hook(lambda mm, i, o, n=n: xs[n].append(i[0].detach().clone())))
        hooks.append(m.register_full_backward_hook(lambda mm, gi, go, n=n: gys[n].append(go[0].detach().clone())))
    out = tmp_path / "probe.pkl"
    acc = sp.run_probe_pass(model, None, calib, "toy", "synthetic", 32, "bfloat16", "cuda", "cuda",
                            torch.device("cuda"), r"mlp\.", r"^$", False, None, str(out))
    for h in hooks:
        h.remove()
    blob = pickle.loads(out.read_bytes())
    assert set(blob) == {"stats", "router_counts", "router_totals", "expert_info", "meta"}
    assert blob["meta"]["nsamples"] == 3 and blob["meta"]["linear_include"] == r"mlp\."
    assert set(blob["stats"]) == set(names)
    for n in names:
        tr = 0.0
        for x, gy in zip(xs[n], gys[n]):
            g2 = (gy.reshape(-1, gy.shape[-1]).t() @ x.reshape(-1, x.shape[-1])).pow(2)
            tr += float(g2.sum())
        st = blob["stats"][n]
        assert st["n_tokens_seen"] == 3 * 32
        assert st["h_trace_raw"] == pytest.approx(tr, rel=2.0 ** -6), n
        assert st["h_trace"] == pytest.approx(st["h_trace_raw"] / 96)
    assert acc.estimator == "exact"
