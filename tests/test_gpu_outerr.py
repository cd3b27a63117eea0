"""pq_output_sse: the output error of a quantized Linear on the tcgen05 tensor cores.

Three layers of checks: the raw fp32 accumulators against a torch fp32 matmul of the same
bf16 operands (tolerance from the fp32 accumulation order: (k/16 + 4) 2^-23 of sum |x||w| per element);
the two sums against the same epilogue recomputed in fp64 on the host from the kernel's own
accumulators (fp32 partial sums of 64 squares: 4e-6 relative); and output_mse / ref_energy against the
reference's bmm formulation (measure_quant_cost.py:599-605, 630-635) through cuBLAS, whose bf16
roundings of differently ordered fp32 sums differ on a few elements (2e-2 relative)."""
import pytest
import torch

from oracle import pq_oracle as O
from prismaquant_b200 import format_registry as fr
from tests._helpers import to_cuda_bf16

pytestmark = pytest.mark.gpu

SHAPES = [  # batch, rows, out, k
    (1, 128, 128, 64), (2, 200, 300, 320), (3, 1, 1, 8), (1, 129, 257, 72), (1, 64, 40, 4096), (2, 384, 256, 136),
]


def _bf16(shape, seed, std=1.0):
    return to_cuda_bf16(O.synthetic_weight_bits(shape, seed=seed, std=std, outlier_frac=0.01))


def _operands(b, m, n, k, seed):
    x = _bf16((b, m, k), seed)
    w = _bf16((b, n, k), seed + 1, std=0.05)
    xq = _bf16((b, m, k), seed + 2)
    wq = (w.float() + 0.01 * torch.randn(w.shape, device="cuda", generator=torch.Generator("cuda").manual_seed(seed))
          ).to(torch.bfloat16)
    return x, w, xq, wq


def _run(x, w, xq, wq, want_y=True):
    from prismaquant_b200 import _lib
    b, m, _ = x.shape
    n = w.shape[1]
    err = torch.zeros(b, dtype=torch.float64, device="cuda")
    ref = torch.zeros(b, dtype=torch.float64, device="cuda")
    yr = torch.full((b, m, n), float("nan"), device="cuda") if want_y else None
    yq = torch.full((b, m, n), float("nan"), device="cuda") if want_y else None
    _lib.output_sse(x, w, xq, wq, err, ref, yr, yq)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    return err, ref, yr, yq


@pytest.mark.parametrize("shape", SHAPES)
def test_accumulators_match_fp32_matmul(shape):
    x, w, xq, wq = _operands(*shape, seed=11)
    _, _, yr, yq = _run(x, w, xq, wq)
    for a, bm, y in ((x, w, yr), (xq, wq, yq)):
        want = torch.bmm(a.double(), bm.double().transpose(1, 2))
        # fp32 accumulation over k / 16 MMA steps: gamma_n * sum |x||w| with n = k / 16 + 4, u = 2^-23
        n_acc = a.shape[-1] / 16 + 4
        bound = torch.bmm(a.double().abs(), bm.double().abs().transpose(1, 2)) * (n_acc * 2.0 ** -23) + 1e-30
        assert torch.isfinite(y).all()
        assert ((y.double() - want).abs() <= bound).all(), float(((y.double() - want).abs() / bound).max())


@pytest.mark.parametrize("shape", SHAPES)
def test_sums_match_epilogue_on_host(shape):
    x, w, xq, wq = _operands(*shape, seed=23)
    err, ref, yr, yq = _run(x, w, xq, wq)
    a = yr.to(torch.bfloat16)
    d = (a - yq.to(torch.bfloat16)).double()
    want_err = (d * d).sum(dim=(1, 2))
    want_ref = (a.double() ** 2).sum(dim=(1, 2))
    # fp32 partial sums of <= 64 squares, then fp64: 64 * 2^-24 relative at most
    torch.testing.assert_close(err, want_err, rtol=4e-6, atol=0)
    torch.testing.assert_close(ref, want_ref, rtol=4e-6, atol=0)
    # without the fp32 outputs the sums are the same
    err2, ref2, _, _ = _run(x, w, xq, wq, want_y=False)
    assert torch.equal(err, err2) and torch.equal(ref, ref2)


@pytest.mark.parametrize("fmt", ["NVFP4", "MXFP8", "FP8_E4M3", "MXFP4"])
def test_output_mse_matches_bmm(fmt):
    spec = fr.get_format(fmt)
    b, m, n, k = 4, 256, 384, 512
    x = _bf16((b, m, k), 5)
    w = _bf16((b, n, k), 6, std=0.05)
    w_hat = torch.stack([spec.quantize_dequantize(t) for t in w])
    x_hat = spec.activation_quantize_dequantize(x.clone())
    err, ref, _, _ = _run(x, w, x_hat, w_hat, want_y=False)
    y_ref = torch.bmm(x, w.transpose(1, 2))
    y_q = torch.bmm(x_hat, w_hat.transpose(1, 2))
    out_mse = (y_ref - y_q).float().pow(2).mean(dim=(1, 2)).double()
    ref_energy = y_ref.float().pow(2).mean(dim=(1, 2)).double()
    torch.testing.assert_close(err / (m * n), out_mse, rtol=2e-2, atol=0)
    torch.testing.assert_close(ref / (m * n), ref_energy, rtol=1e-3, atol=0)


def test_identity_operands_give_zero_error():
    x, w, _, _ = _operands(2, 130, 140, 96, seed=3)
    err, ref, _, _ = _run(x, w, x, w, want_y=False)
    assert (err == 0).all() and (ref > 0).all()


def test_validation():
    from prismaquant_b200 import _lib
    x = torch.zeros(1, 4, 12, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(1, 5, 12, dtype=torch.bfloat16, device="cuda")
    s = torch.zeros(1, dtype=torch.float64, device="cuda")
    with pytest.raises(ValueError):
        _lib.output_sse(x, w, x, w, s, s)          # k = 12 is not a multiple of 8
    with pytest.raises(ValueError):
        _lib.output_sse(x, w[:, :, :8], x, w, s, s)
    e = torch.zeros(0, 4, 16, dtype=torch.bfloat16, device="cuda")
    _lib.output_sse(e, torch.zeros(0, 5, 16, dtype=torch.bfloat16, device="cuda"), e,
                    torch.zeros(0, 5, 16, dtype=torch.bfloat16, device="cuda"), None, None)
    assert _lib.device_error() == 0


def _ref_err(x, w, xq, wq):
    from prismaquant_b200 import _lib
    b, m, _ = x.shape
    n = w.shape[1]
    y = torch.empty(b, m, n, dtype=torch.bfloat16, device="cuda")
    ref = torch.zeros(b, dtype=torch.float64, device="cuda")
    err = torch.zeros_like(ref)
    _lib.output_ref(x, w, ref, y)
    _lib.output_err(xq, wq, y, err)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    return y, ref, err


@pytest.mark.parametrize("shape", SHAPES)
def test_ref_and_err_modes_match_dual(shape):
    """The split kernels (y_ref stored once, one GEMM per format) against the one-pass dual kernel
    and against an fp64 product of the same operands."""
    x, w, xq, wq = _operands(*shape, seed=29)
    y, ref, err = _ref_err(x, w, xq, wq)
    derr, dref, yr, _ = _run(x, w, xq, wq)
    want = torch.bmm(x.double(), w.double().transpose(1, 2))
    bound = torch.bmm(x.double().abs(), w.double().abs().transpose(1, 2)) * ((x.shape[-1] / 16 + 4) * 2.0 ** -23)
    # y_ref is bf16 of an fp32 accumulator within the bound: half a bf16 ulp more at most
    assert ((y.double() - want).abs() <= bound + want.abs() * 2.0 ** -8 + 1e-30).all()
    # the split kernels may sum K in parts (a CTA cluster per tile) where the dual kernel runs K in
    # one pass: bf16 roundings of a few outputs can differ, nothing more
    assert ((y.double() - yr.double()).abs() <= bound + yr.double().abs() * 2.0 ** -8 + 1e-30).all()
    torch.testing.assert_close(ref, dref, rtol=2e-3, atol=0)
    torch.testing.assert_close(err, derr, rtol=2e-3, atol=0)


def test_err_mode_of_the_reference_operands_is_zero():
    x, w, _, _ = _operands(3, 300, 520, 200, seed=41)
    _, ref, err = _ref_err(x, w, x, w)
    assert (err == 0).all() and (ref > 0).all()


def test_ref_mode_without_output_and_validation():
    from prismaquant_b200 import _lib
    x, w, _, _ = _operands(2, 64, 96, 40, seed=43)
    y, ref, _ = _ref_err(x, w, x, w)
    ref2 = torch.zeros_like(ref)
    _lib.output_ref(x, w, ref2, None)
    torch.cuda.synchronize()
    assert torch.equal(ref, ref2)
    with pytest.raises(TypeError):
        _lib.output_err(x, w, y.float(), ref2)
    with pytest.raises(ValueError):
        _lib.output_ref(x[:, :, :36], w[:, :, :36], ref2)    # k = 36 is not a multiple of 8
