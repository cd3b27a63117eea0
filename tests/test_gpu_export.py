"""Export packing on the GPU vs the reference (golden fixtures, full-size
digests) and the oracle.  Bar: bit-exact codes, scales and globals."""
import numpy as np
import pytest
import torch

from oracle import pq_oracle as O
from prismaquant_b200 import export_native_compressed as enc
from prismaquant_b200 import format_registry as fr
from prismaquant_b200 import measure_quant_cost as mqc
from tests._helpers import assert_rel, to_cuda_bf16, u8_of

pytestmark = pytest.mark.gpu

CASES2D = ["rand_64x128", "rand_33x256", "ties_4x32", "zeros_3x64", "wide_range_8x96", "row1_1x4096",
           "cols16_5x16", "cols48_7x48", "cols8_4x8"]


def f32(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("case", CASES2D)
def test_export_2d_matches_reference(golden, case):
    w = to_cuda_bf16(golden[f"{case}/input"])
    if f"{case}/nvfp4/packed" in golden:
        p, s, g = enc.quantize_dequantize_nvfp4(w)
        np.testing.assert_array_equal(u8_of(p), golden[f"{case}/nvfp4/packed"])
        np.testing.assert_array_equal(u8_of(s), golden[f"{case}/nvfp4/scale"])
        np.testing.assert_array_equal(f32(g), golden[f"{case}/nvfp4/global"])
        assert s.dtype == torch.float8_e4m3fn and p.dtype == torch.uint8 and g.dtype == torch.float32
        gr = enc.compute_nvfp4_global_real(w)
        assert float(gr) == float(golden[f"{case}/nvfp4/global_real"][0])
        ov = torch.tensor(float(golden[f"{case}/nvfp4_ovr/override"][0]))
        p, s, g = enc.quantize_dequantize_nvfp4(w, global_real_override=ov)
        np.testing.assert_array_equal(u8_of(p), golden[f"{case}/nvfp4_ovr/packed"])
        np.testing.assert_array_equal(u8_of(s), golden[f"{case}/nvfp4_ovr/scale"])
        np.testing.assert_array_equal(f32(g), golden[f"{case}/nvfp4_ovr/global"])
        q = enc._quantize_2d(w, "NVFP4")
        assert float(q["input_global_scale"]) == float(golden[f"{case}/q2d_nvfp4/input_global_scale"][0])
    else:
        with pytest.raises(ValueError):
            enc.quantize_dequantize_nvfp4(w)
    if f"{case}/mxfp8/weight" in golden:
        q, sc = enc.quantize_dequantize_mxfp8(w)
        np.testing.assert_array_equal(u8_of(q), golden[f"{case}/mxfp8/weight"])
        np.testing.assert_array_equal(u8_of(sc), golden[f"{case}/mxfp8/scale"])
    q, sc = enc.quantize_dequantize_fp8_dynamic(w)
    np.testing.assert_array_equal(u8_of(q), golden[f"{case}/fp8dyn/weight"])
    np.testing.assert_array_equal(f32(sc), golden[f"{case}/fp8dyn/scale"])


@pytest.mark.parametrize("case", ["packed_4x32x64", "packed_3x16x96"])
def test_export_packed_matches_reference(golden, case):
    w = to_cuda_bf16(golden[f"{case}/input"])
    p, s, g = enc.quantize_dequantize_nvfp4_packed(w)
    np.testing.assert_array_equal(u8_of(p), golden[f"{case}/nvfp4p/packed"])
    np.testing.assert_array_equal(u8_of(s), golden[f"{case}/nvfp4p/scale"])
    np.testing.assert_array_equal(f32(g), golden[f"{case}/nvfp4p/global"])
    q, sc = enc.quantize_dequantize_mxfp8_packed(w)
    np.testing.assert_array_equal(u8_of(q), golden[f"{case}/mxfp8p/weight"])
    np.testing.assert_array_equal(u8_of(sc), golden[f"{case}/mxfp8p/scale"])
    gq = enc._quantize_2d_group_same_shape(w, "MXFP8")
    np.testing.assert_array_equal(u8_of(gq["weight"]), golden[f"{case}/grouped_mxfp8/weight"])
    q, sc = enc.quantize_dequantize_fp8_dynamic_packed(w)
    np.testing.assert_array_equal(u8_of(q), golden[f"{case}/fp8dynp/weight"])
    np.testing.assert_array_equal(f32(sc), golden[f"{case}/fp8dynp/scale"])


@pytest.mark.parametrize("shape,seed,std", [((512, 4096), 1, 0.02), ((64, 14336), 2, 0.02), ((8, 64, 768), 3, 0.02),
                                            ((257, 2048), 4, 1e-20), ((33, 1024), 5, 1e20)])
def test_export_vs_oracle(shape, seed, std):
    bits = O.synthetic_weight_bits(shape, seed=seed, std=std, outlier_frac=0.001)
    w = to_cuda_bf16(bits)
    wf = O.bf16_bits_to_f32(bits)
    ref = O.nvfp4_pack(wf) if len(shape) == 2 else O.nvfp4_pack_packed(wf)
    got = enc.quantize_dequantize_nvfp4(w) if len(shape) == 2 else enc.quantize_dequantize_nvfp4_packed(w)
    for r, g in zip(ref, got):
        np.testing.assert_array_equal(u8_of(g) if g.dtype != torch.float32 else f32(g), r)
    q, sc = enc.quantize_dequantize_mxfp8(w)
    rq, rsc = O.mxfp8_pack(wf)
    np.testing.assert_array_equal(u8_of(q), rq)
    np.testing.assert_array_equal(u8_of(sc), rsc)
    q, sc = enc.quantize_dequantize_fp8_dynamic(w)
    rq, rsc = O.fp8_dynamic_pack(wf)
    np.testing.assert_array_equal(u8_of(q), rq)
    np.testing.assert_array_equal(f32(sc), rsc)


def test_linear4096_export_digests(full_digests):
    d = full_digests["linear4096"]
    bits = O.synthetic_weight_bits((4096, 4096), seed=0, outlier_frac=0.001)
    w = to_cuda_bf16(bits)
    p, s, g = enc.quantize_dequantize_nvfp4(w)
    assert O.digest(u8_of(p), u8_of(s), f32(g)) == d["nvfp4"]
    q, sc = enc.quantize_dequantize_mxfp8(w)
    assert O.digest(u8_of(q), u8_of(sc)) == d["mxfp8"]
    q, sc = enc.quantize_dequantize_fp8_dynamic(w)
    assert O.digest(u8_of(q), f32(sc)) == d["fp8dyn"]


def test_fused_siblings_joint_global(full_digests):
    """q/k/v and gate/up share one NVFP4 global (max of their natural ones);
    fused sweep + export in one pass reproduces the reference's packed bytes
    and MSE_W for every sibling."""
    dg = full_digests["siblings"]
    names = list(dg)
    prefix = {"q_proj": "model.layers.0.self_attn.", "k_proj": "model.layers.0.self_attn.",
              "v_proj": "model.layers.0.self_attn.", "gate_proj": "model.layers.0.mlp.",
              "up_proj": "model.layers.0.mlp."}
    ws = {}
    for n in names:
        bits = O.synthetic_weight_bits(tuple(dg[n]["shape"]), seed=dg[n]["seed"])
        assert O.digest(bits) == dg[n]["input"]
        ws[prefix[n] + n] = to_cuda_bf16(bits)
    specs = [fr.get_format(f) for f in ("NVFP4", "MXFP8", "FP8_E4M3", "BF16")]
    costs, outs = enc.sweep_and_export(ws, specs)
    for full, n in zip(ws, names):
        p, s, g = outs[full]
        assert O.digest(u8_of(p), u8_of(s), f32(g)) == dg[n]["nvfp4"], n
        for f in ("NVFP4", "MXFP8", "FP8_E4M3", "BF16"):
            assert_rel(costs[full][f], dg[n][f"mse/{f}"], 1e-5, f"{n} {f}")
    # same bytes through the one-tensor API with the joint override
    for full, n in zip(ws, names):
        p, s, g = enc.quantize_dequantize_nvfp4(ws[full], global_real_override=torch.tensor(dg[n]["joint_global_real"]))
        assert O.digest(u8_of(p), u8_of(s), f32(g)) == dg[n]["nvfp4"], n


def test_fused_sweep_export_equals_separate():
    bits = [O.synthetic_weight_bits(s, seed=40 + i) for i, s in enumerate([(256, 4096), (128, 14336), (96, 1024)])]
    ws = {f"model.layers.0.mlp.x{i}": to_cuda_bf16(b) for i, b in enumerate(bits)}
    specs = [fr.get_format(f) for f in ("NVFP4", "MXFP8", "FP8_E4M3")]
    costs, outs = enc.sweep_and_export(ws, specs)
    sep = mqc.sweep_weight_mse(ws, specs)
    for k, w in ws.items():
        for f in ("NVFP4", "MXFP8", "FP8_E4M3"):
            assert costs[k][f] == sep[k][f]
        p, s, g = enc.quantize_dequantize_nvfp4(w)
        torch.testing.assert_close(outs[k][0], p, rtol=0, atol=0)
        assert torch.equal(outs[k][1].view(torch.uint8), s.view(torch.uint8))
        assert torch.equal(outs[k][2], g)


def test_shape_errors_raise():
    w = torch.zeros(4, 40, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        enc.quantize_dequantize_nvfp4(w)
    with pytest.raises(ValueError):
        enc.quantize_dequantize_mxfp8(w)
    with pytest.raises(ValueError):
        fr.get_format("MXFP8").quantize_dequantize(torch.zeros(4, 48, dtype=torch.bfloat16, device="cuda"))


def test_nvfp4_scales_every_bf16_amax():
    """pq_nvfp4_scales over every positive bf16 group maximum, for globals that put many quotients
    exactly on E4M3 midpoints (1, 1/2, 7/6, ...), the 1e-12 floor (also reached from below), a
    global outside the bracket's range, and a misaligned tail slice (scalar path)."""
    from prismaquant_b200 import _lib
    bits = np.arange(0, 0x7F80, dtype=np.uint16)                 # 0 .. largest finite bf16
    amax = torch.from_numpy(bits.view(np.int16)).cuda()
    globs = [1.0, 0.5, 3.0, 7.0 / 6.0, 1.0 / 448.0, 2.0 ** -20, 1e-12, 1e-20, 1e31, 12.25]
    slices = [amax] * len(globs) + [amax[1:]]                    # last: 2-byte offset, scalar path
    over = torch.tensor(globs + [0.75], dtype=torch.float32, device="cuda")
    scales = [torch.empty(s.numel(), dtype=torch.uint8, device="cuda") for s in slices]
    gdiv = torch.empty(len(slices), dtype=torch.float32, device="cuda")
    _lib.nvfp4_scales(slices, None, scales, gdiv, override=over)
    torch.cuda.synchronize()
    a32 = O.bf16_bits_to_f32(bits)
    s_g = (np.maximum(a32, np.float32(1e-12)) / np.float32(6.0)).astype(np.float32)
    for i, g in enumerate(globs + [0.75]):
        glob = np.float32(max(np.float32(g), np.float32(1e-12)))
        want = O.f32_to_e4m3fn_bits(np.clip((s_g / glob).astype(np.float32), np.float32(0), np.float32(448)))
        if i == len(globs):
            want = want[1:]
        got = scales[i].cpu().numpy()
        bad = np.nonzero(got != want)[0]
        assert bad.size == 0, (g, bad[:5], got[bad[:5]], want[bad[:5]])
        assert gdiv[i].item() == float(np.float32(1.0) / glob)
    assert _lib.device_error() == 0


def test_streaming_sweep_export_equals_resident():
    """StreamingSweepExport (host weights, chunked H2D / sweep + export / D2H on three streams)
    gives the resident plan's cost table and packed bytes, fused-sibling joint globals included,
    on two consecutive runs."""
    shapes = {"model.layers.0.self_attn.q_proj": (256, 512), "model.layers.0.self_attn.k_proj": (64, 512),
              "model.layers.0.self_attn.v_proj": (64, 512), "model.layers.0.self_attn.o_proj": (512, 256),
              "model.layers.0.mlp.gate_proj": (384, 512), "model.layers.0.mlp.up_proj": (384, 512),
              "model.layers.0.mlp.down_proj": (512, 384), "lm_head": (1000, 512)}
    host = {n: torch.from_numpy(O.synthetic_weight_bits(s, seed=60 + i, outlier_frac=0.01).view(np.int16))
            .view(torch.bfloat16) for i, (n, s) in enumerate(shapes.items())}
    specs = [fr.get_format(f) for f in ("NVFP4", "MXFP8", "FP8_E4M3", "BF16")]
    st = enc.StreamingSweepExport(host, specs, chunk_bytes=200_000)   # several chunks, groups kept whole
    assert len(st.chunks) > 3
    plan = enc.SweepExportPlan({n: h.cuda() for n, h in host.items()}, specs)
    plan.run()
    want_costs = plan.costs()
    for _ in range(2):
        st.run()
        torch.cuda.synchronize()
        assert st.costs() == want_costs
        outs = st.outputs()
        for i, n in enumerate(plan.names):
            c, s, g = plan.outputs[i]
            hc, hs, hg = outs[n]
            assert torch.equal(hc, c.cpu())
            assert torch.equal(hs.view(torch.uint8), s.view(torch.uint8).cpu())
            assert torch.equal(hg, g.cpu())


def test_plan_run_with_overlapped_collective_equals_run():
    """SweepExportPlan.run(then=...): the scale pass on a side stream while `then` is enqueued on
    the current one gives run()'s packed bytes, globals and sums, and returns `then`'s result."""
    shapes = {"model.layers.0.self_attn.q_proj": (256, 512), "model.layers.0.self_attn.k_proj": (64, 512),
              "model.layers.0.self_attn.v_proj": (64, 512), "model.layers.0.mlp.down_proj": (512, 384)}
    ws = {n: to_cuda_bf16(O.synthetic_weight_bits(s, seed=90 + i, outlier_frac=0.01)) for i, (n, s) in enumerate(shapes.items())}
    specs = [fr.get_format(f) for f in ("NVFP4", "MXFP8", "FP8_E4M3", "BF16")]
    plan = enc.SweepExportPlan(ws, specs)
    plan.run()
    want = [(c.clone(), s.view(torch.uint8).clone(), g.clone()) for c, s, g in plan.outputs]
    want_sse = plan.sse.clone()
    for _ in range(2):
        got = plan.run(then=lambda: plan.sse.clone())
        torch.cuda.synchronize()
        assert torch.equal(got, want_sse) and torch.equal(plan.sse, want_sse)
        for (c, s, g), (wc, ws_, wg) in zip(plan.outputs, want):
            assert torch.equal(c, wc) and torch.equal(s.view(torch.uint8), ws_) and torch.equal(g, wg)


def test_streaming_export_to_safetensors():
    """export_to streams every chunk's NVFP4 entries into IncrementalSafetensorsWriter shards while
    later chunks are on the GPU; the checkpoint on disk holds the resident path's bytes under the
    reference's keys."""
    import tempfile
    from pathlib import Path

    from safetensors.torch import load_file
    from prismaquant_b200 import safetensors_io as S
    shapes = {"model.layers.0.self_attn.q_proj": (256, 512), "model.layers.0.self_attn.k_proj": (64, 512),
              "model.layers.0.self_attn.v_proj": (64, 512), "model.layers.0.mlp.gate_proj": (384, 512),
              "model.layers.0.mlp.up_proj": (384, 512), "model.layers.0.mlp.down_proj": (512, 384)}
    host = {n: torch.from_numpy(O.synthetic_weight_bits(s, seed=80 + i).view(np.int16)).view(torch.bfloat16)
            for i, (n, s) in enumerate(shapes.items())}
    specs = [fr.get_format(f) for f in ("NVFP4", "MXFP8", "FP8_E4M3")]
    st = enc.StreamingSweepExport(host, specs, chunk_bytes=300_000)
    costs, packed = enc.sweep_and_export({n: h.cuda() for n, h in host.items()}, specs)
    with tempfile.TemporaryDirectory() as d:
        w = S.IncrementalSafetensorsWriter(Path(d), shard_bytes=150_000)
        st.export_to(w)
        w.finalize()
        assert st.costs() == costs
        files = sorted(p.name for p in Path(d).iterdir())
        assert "model.safetensors.index.json" in files and len(files) > 2
        loaded = {}
        for f in files:
            if f.endswith(".safetensors"):
                loaded.update(load_file(str(Path(d) / f)))
        assert set(loaded) == {f"{n}.{k}" for n in shapes for k in
                               ("weight_packed", "weight_scale", "weight_global_scale", "input_global_scale")}
        for n in shapes:
            p, s, g = packed[n]
            assert torch.equal(loaded[f"{n}.weight_packed"], p.cpu())
            assert torch.equal(loaded[f"{n}.weight_scale"].view(torch.uint8), s.view(torch.uint8).cpu())
            assert torch.equal(loaded[f"{n}.weight_global_scale"], g.cpu())
            assert loaded[f"{n}.input_global_scale"].tolist() == [1.0]


def test_global_real_kernel_batched_and_joint(full_digests, monkeypatch):
    """pq_nvfp4_global_real: per-slice globals of a stacked tensor equal the one-slice call and the
    oracle, and the fused-sibling joint globals of the full-size q/k/v + gate/up group equal the
    reference's (full_digests.json).  No torch reduction runs on the path (abs/amax are poisoned)."""
    from prismaquant_b200 import _lib
    bits = O.synthetic_weight_bits((6, 96, 256), seed=3, std=0.05, outlier_frac=0.01)
    w = to_cuda_bf16(bits)
    got = _lib.nvfp4_global_real(w, 6)
    for b in range(6):
        assert float(got[b]) == float(O.nvfp4_global_real(O.bf16_bits_to_f32(bits[b])))
        assert float(got[b]) == float(enc.compute_nvfp4_global_real(w[b]))

    def boom(*a, **k):
        raise AssertionError("torch reduction on the global path")
    dg = full_digests["siblings"]
    ws = {n: to_cuda_bf16(O.synthetic_weight_bits(tuple(dg[n]["shape"]), seed=dg[n]["seed"])) for n in dg}
    monkeypatch.setattr(torch.Tensor, "amax", boom)
    monkeypatch.setattr(torch.Tensor, "abs", boom)
    for group in (("q_proj", "k_proj", "v_proj"), ("gate_proj", "up_proj")):
        joint = max(float(enc.compute_nvfp4_global_real(ws[n])) for n in group)
        for n in group:
            assert joint == dg[n]["joint_global_real"], n


def test_pipelined_plan_equals_one_chunk():
    """A plan swept and scaled in several chunks (scale passes on a side stream) gives the packed
    bytes, globals (fused-sibling joint ones included) and sums of a one-chunk plan."""
    shapes = {}
    for l in range(3):
        for p, sh in (("self_attn.q_proj", (256, 512)), ("self_attn.k_proj", (64, 512)), ("self_attn.v_proj", (64, 512)),
                      ("self_attn.o_proj", (512, 256)), ("mlp.gate_proj", (384, 512)), ("mlp.up_proj", (384, 512)),
                      ("mlp.down_proj", (512, 384))):
            shapes[f"model.layers.{l}.{p}"] = sh
    ws = {n: to_cuda_bf16(O.synthetic_weight_bits(s, seed=70 + i, outlier_frac=0.01)) for i, (n, s) in enumerate(shapes.items())}
    specs = [fr.get_format(f) for f in ("NVFP4", "MXFP8", "FP8_E4M3", "BF16")]
    one = enc.SweepExportPlan(ws, specs, pipeline_chunks=1)
    many = enc.SweepExportPlan(ws, specs, pipeline_chunks=4)
    assert len(one.chunks) == 1 and len(many.chunks) > 2
    one.run()
    for _ in range(2):
        many.run()
        torch.cuda.synchronize()
        assert torch.allclose(many.sse, one.sse, rtol=1e-12, atol=0.0)   # fp64 atomics: order may differ
        for (c, s, g), (c1, s1, g1) in zip(many.outputs, one.outputs):
            assert torch.equal(c, c1) and torch.equal(s.view(torch.uint8), s1.view(torch.uint8)) and torch.equal(g, g1)


def test_fp8_channel_export_ties_and_every_bf16_value():
    """The FP8 per-channel export against the oracle: rows whose maximum has a significand that
    is a multiple of 7 (s = a / 448 exact, so E4M3 midpoints among the quotients are exact ties,
    which round to even), 1.75 x 2^k (s a power of two), and others, each row holding 4095 bf16
    magnitudes drawn from all those up to its maximum, with random signs."""
    rng = np.random.default_rng(12)
    b = np.arange(1 << 15, dtype=np.uint32)
    mags = b[b < 0x7F80]
    rows = []
    for sig in (1.75, 1.3125, 1.09375, 1.0, 1.5390625, 1.9921875):     # 224, 168, 140: multiples of 7
        for k in (-30, -1, 0, 9):
            a_bits = int(O.f32_to_bf16_bits(np.array([sig * 2.0 ** k], np.float32))[0])
            pool = mags[mags <= a_bits]
            row = rng.choice(pool, size=4095, replace=pool.size < 4095).astype(np.uint32)
            row |= rng.integers(0, 2, size=4095).astype(np.uint32) << 15
            rows.append(np.concatenate([[a_bits], row]).astype(np.uint16))
    bits = np.array(rows)
    q, sc = enc.quantize_dequantize_fp8_dynamic(to_cuda_bf16(bits))
    rq, rsc = O.fp8_dynamic_pack(O.bf16_bits_to_f32(bits))
    np.testing.assert_array_equal(f32(sc), rsc)
    got = u8_of(q)
    bad = np.nonzero(got != rq)
    assert bad[0].size == 0, (got[bad][:5], rq[bad][:5], bits[bad][:5])
