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
