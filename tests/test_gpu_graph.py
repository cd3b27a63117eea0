"""The hot-path entry points launch without host synchronisation or device-side descriptor
buffers (the sweep's work list travels as kernel parameters), so a step can be captured once in
a CUDA graph and replayed.  This captures the fused sweep, the NVFP4 export, the fused W_hat and
the tensor-core output error, replays them, and checks every output against an eager run."""
import pytest
import torch

from oracle import pq_oracle as O
from tests._helpers import to_cuda_bf16

pytestmark = pytest.mark.gpu


def test_capture_and_replay_matches_eager():
    from prismaquant_b200 import _lib
    w = to_cuda_bf16(O.synthetic_weight_bits((512, 4096), seed=3, outlier_frac=0.001))
    x = to_cuda_bf16(O.synthetic_weight_bits((1, 256, 4096), seed=4, std=1.0))
    sse = torch.zeros(1, 4, dtype=torch.float64, device="cuda")
    codes = torch.empty(512, 2048, dtype=torch.uint8, device="cuda")
    amax = torch.empty(512, 256, dtype=torch.int16, device="cuda")
    tmax = torch.zeros(1, dtype=torch.int32, device="cuda")
    y = torch.empty(1, 256, 512, dtype=torch.bfloat16, device="cuda")
    ref = torch.zeros(1, dtype=torch.float64, device="cuda")
    err = torch.zeros(1, dtype=torch.float64, device="cuda")
    hats = {}

    def step():
        sse.zero_()
        tmax.zero_()
        ref.zero_()
        err.zero_()
        _lib.sweep_sse([w], [15], nvfp4_outputs=[(codes, amax, tmax)], sse=sse)
        hats.update(_lib.cost_qdq_fused(w, ("NVFP4", "MXFP8", "FP8_E4M3")))
        _lib.output_ref(x, w.unsqueeze(0), ref, y)
        _lib.output_err(x, hats["NVFP4"].unsqueeze(0), y, err)

    step()   # eager, also loads the library and sets kernel attributes outside the capture
    torch.cuda.synchronize()
    eager = [t.clone() for t in (sse, codes, amax, tmax, y, ref, err)] + [hats[f].clone() for f in sorted(hats)]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):   # warm the side stream, as torch's capture recipe does
        step()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    got = [sse, codes, amax, tmax, y, ref, err] + [hats[f] for f in sorted(hats)]
    for a, b in zip(got, eager):
        if a.dtype == torch.float64:   # fp64 atomics across CTAs: the last bits may differ
            torch.testing.assert_close(a, b, rtol=1e-12, atol=0)
        else:
            assert torch.equal(a, b)
