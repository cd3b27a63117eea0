"""The allocation-free NVFP4 export entry point, pq_nvfp4_pack_noalloc.

It exists for callers that cannot allocate device memory (their memory belongs
to another allocator, their host forbids device allocations, or a cudaMalloc's
device-wide synchronisation is not acceptable), so it keeps its scratch in a
fixed array inside the library instead of taking scratch buffers.  These
tests call it through the C ABI and require the same bytes as pq_nvfp4_pack
(which takes caller-provided scratch) on two calls in a row: the second call
has a smaller maximum than the first, so a per-slice maximum left over in the
shared array would change its global scale and block scales.  This file is
named to be collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import pq_oracle as O
from prismaquant_b200 import _lib

pytestmark = pytest.mark.gpu


def _w(shape, seed, std):
    bits = O.synthetic_weight_bits(shape, seed=seed, std=std, outlier_frac=0.001)
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()


def _outputs(batch, rows, cols):
    dev = torch.device("cuda")
    return (torch.empty(batch * rows * cols // 2, dtype=torch.uint8, device=dev),
            torch.empty(batch * rows * cols // 16, dtype=torch.uint8, device=dev),
            torch.empty(batch, dtype=torch.float32, device=dev))


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _pack_with_scratch(w, batch, override):
    lib = _lib.load()
    rows, cols = w.numel() // w.shape[-1] // batch, w.shape[-1]
    codes, scales, gdiv = _outputs(batch, rows, cols)
    amax = torch.empty(batch * rows * cols // 16, dtype=torch.int16, device="cuda")
    tmax = torch.empty(batch, dtype=torch.int32, device="cuda")
    st = lib.pq_nvfp4_pack(_ptr(w), batch, rows, cols, _ptr(override), _ptr(codes), _ptr(scales), _ptr(gdiv),
                           _ptr(amax), _ptr(tmax), torch.cuda.current_stream().cuda_stream)
    assert st == _lib.PQ_OK, st
    return codes, scales, gdiv


def _pack_noalloc(w, batch, override):
    lib = _lib.load()
    rows, cols = w.numel() // w.shape[-1] // batch, w.shape[-1]
    codes, scales, gdiv = _outputs(batch, rows, cols)
    st = lib.pq_nvfp4_pack_noalloc(_ptr(w), batch, rows, cols, _ptr(override), _ptr(codes), _ptr(scales),
                                   _ptr(gdiv), torch.cuda.current_stream().cuda_stream)
    assert st == _lib.PQ_OK, st
    return codes, scales, gdiv


@pytest.mark.parametrize("with_override", [False, True])
def test_noalloc_matches_scratch_entry_point_on_two_calls(with_override):
    first = (_w((8, 256, 2048), seed=1, std=1.0), 8)       # 8 experts, per-expert globals, larger values
    second = (_w((1536, 4096), seed=2, std=0.02), 1)       # one Linear, much smaller maximum
    results = []
    for w, batch in (first, second):                       # two noalloc calls in a row
        ov = torch.full((batch,), 3e-4, dtype=torch.float32, device="cuda") if with_override else None
        results.append((_pack_noalloc(w, batch, ov), (w, batch, ov)))
    torch.cuda.synchronize()
    for got, (w, batch, ov) in results:
        want = _pack_with_scratch(w, batch, ov)
        for g, r in zip(got, want):
            assert torch.equal(g, r)
    assert _lib.device_error() == 0


def test_noalloc_rejects_sizes_beyond_its_array():
    lib = _lib.load()
    # 8,388,608 groups is the limit: 2 x 4096 x 65,552 bf16 is above it; 257 slices is above 256
    assert lib.pq_nvfp4_pack_noalloc(None, 2, 65552, 4096, None, None, None, None, None) == _lib.PQ_ERR_LIMIT
    assert lib.pq_nvfp4_pack_noalloc(None, 257, 16, 16, None, None, None, None, None) == _lib.PQ_ERR_LIMIT


def test_noalloc_at_its_exact_limit_and_with_empty_slices():
    """At exactly 8,388,608 groups (the array's size: 2 slices of 4096 x 16384) and with rows == 0
    (no groups at all: each slice's global still comes from the override, or from a zero maximum),
    the entry point gives pq_nvfp4_pack's bytes."""
    w = _w((2, 4096, 16384), seed=5, std=0.02)
    got = _pack_noalloc(w, 2, None)
    want = _pack_with_scratch(w, 2, None)
    for g, r in zip(got, want):
        assert torch.equal(g, r)
    lib = _lib.load()
    for ov in (None, torch.tensor([2e-3, 5e-4, 1e-3], dtype=torch.float32, device="cuda")):
        e = torch.empty(0, dtype=torch.bfloat16, device="cuda")
        g_na = torch.full((3,), -1.0, dtype=torch.float32, device="cuda")
        g_sc = torch.full((3,), -2.0, dtype=torch.float32, device="cuda")
        s = torch.cuda.current_stream().cuda_stream
        assert lib.pq_nvfp4_pack_noalloc(_ptr(e), 3, 0, 64, _ptr(ov), None, None, _ptr(g_na), s) == _lib.PQ_OK
        tm = torch.empty(3, dtype=torch.int32, device="cuda")
        assert lib.pq_nvfp4_pack(_ptr(e), 3, 0, 64, _ptr(ov), None, None, _ptr(g_sc), None, _ptr(tm), s) == \
            _lib.PQ_OK
        torch.cuda.synchronize()
        assert torch.equal(g_na, g_sc)
    assert _lib.device_error() == 0


def test_noalloc_limit_checks_do_not_overflow():
    lib = _lib.load()
    # rows * cols / 16 would overflow int64 if formed before the check
    assert lib.pq_nvfp4_pack_noalloc(None, 1, 2 ** 62, 2 ** 20, None, None, None, None, None) == _lib.PQ_ERR_LIMIT
