"""Past 2^31 elements: one bf16 tensor of 2.18e9 elements (4.4 GB) built from R copies of a
[256, 4096] block.  Every format groups within a row, so the tensor's error sums are R times the
block's and each copy's W_hat and NVFP4 codes equal the block's bit for bit:
size-independent properties that would catch a 32-bit index anywhere in the kernels.  The sums
fold fp32 partials of up to 64 exact squares at different boundaries in the two tensors, hence
1e-7 rather than exact equality."""
import pytest
import torch

from oracle import pq_oracle as O
from tests._helpers import to_cuda_bf16

pytestmark = pytest.mark.gpu

R = 2080                 # 2080 * 256 * 4096 = 2,181,038,080 elements > 2^31


@pytest.fixture(scope="module")
def tiled():
    block = to_cuda_bf16(O.synthetic_weight_bits((256, 4096), seed=21, outlier_frac=0.002))
    big = block.repeat(R, 1)
    assert big.numel() > 2 ** 31
    yield block, big
    del big
    torch.cuda.empty_cache()


def test_sweep_sums_scale_with_copies(tiled):
    from prismaquant_b200 import _lib
    block, big = tiled
    s_block = _lib.sweep_sse([block], [7])
    s_big = _lib.sweep_sse([big], [7])
    torch.testing.assert_close(s_big[0, :3], s_block[0, :3] * R, rtol=1e-7, atol=0)
    for f in ("MXFP4", "INT4_W4A16_g128"):
        a = torch.zeros((), dtype=torch.float64, device="cuda")
        b = torch.zeros((), dtype=torch.float64, device="cuda")
        _lib.format_sse(block, f, a)
        _lib.format_sse(big, f, b)
        torch.testing.assert_close(b, a * R, rtol=1e-7, atol=0)
    assert _lib.device_error() == 0


def test_w_hat_and_codes_of_every_copy(tiled):
    from prismaquant_b200 import _lib
    block, big = tiled
    want = _lib.cost_qdq(block, "NVFP4")
    got = _lib.cost_qdq(big, "NVFP4").view(R, 256, 4096)
    assert torch.equal(got, want.unsqueeze(0).expand(R, -1, -1))
    del got
    codes_b, _, _ = _lib.nvfp4_pack(block)
    codes, _, _ = _lib.nvfp4_pack(big)
    assert torch.equal(codes.view(R, 256, 2048), codes_b.unsqueeze(0).expand(R, -1, -1))
    assert _lib.device_error() == 0
