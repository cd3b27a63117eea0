"""CPU-side checks of the boundary and the host logic (no GPU needed)."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent


def declared_symbols():
    text = (REPO / "include" / "prismaquant_b200.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:int|uint32_t|const char\*)\s+(pq_\w+)\s*\(", text, re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    from prismaquant_b200 import _lib
    lib = _lib.load()
    syms = declared_symbols()
    assert len(syms) >= 14
    for s in syms:
        assert hasattr(lib, s), s
    assert set(_lib.EXPORTED) == set(syms)
    assert lib.pq_version() >= 1
    assert lib.pq_status_string(2) == b"shape not divisible by the format's group size"


def test_struct_layout_matches_header():
    from prismaquant_b200 import _lib
    assert ctypes.sizeof(_lib.SweepTensor) == 56
    assert _lib.SweepTensor.nvfp4_codes.offset == 32


def test_argument_validation_without_gpu():
    """Shape / null checks happen before any CUDA call."""
    from prismaquant_b200 import _lib
    lib = _lib.load()
    assert lib.pq_mxfp8_pack(None, 4, 48, None, None, None) == _lib.PQ_ERR_SHAPE
    assert lib.pq_nvfp4_codes(None, 1, 4, 40, None, None, None, None) == _lib.PQ_ERR_SHAPE
    assert lib.pq_cost_qdq(None, 4, 64, _lib.NUM_FMTS_ALL, None, None) == _lib.PQ_ERR_FORMAT
    assert lib.pq_cost_qdq(None, 4, 40, _lib.FMT_IDS["INT3"], None, None) == _lib.PQ_ERR_SHAPE    # 16 does not divide 40
    assert lib.pq_cost_qdq(None, 4, 8, _lib.FMT_IDS["INT4_W4A16_g128"], None, None) == _lib.PQ_ERR_NULL  # whole-row group
    assert lib.pq_format_sse(None, 4, 40, _lib.FMT_IDS["MXFP4"], None, None) == _lib.PQ_ERR_SHAPE
    assert lib.pq_format_sse(None, 4, 64, _lib.FMT_NVFP4, None, None) == _lib.PQ_ERR_FORMAT        # fused: pq_sweep_sse
    assert lib.pq_format_sse(None, 4, 64, _lib.FMT_BF16, None, None) == _lib.PQ_OK
    assert lib.pq_format_sse(None, 4, 64, _lib.FMT_IDS["NVFP3"], None, None) == _lib.PQ_ERR_NULL
    assert lib.pq_sumsq_rows(None, 4, 64, None, None, None) == _lib.PQ_ERR_NULL
    assert lib.pq_sweep_sse(None, 0, None, None) == _lib.PQ_OK
    arr = (_lib.SweepTensor * 1)()
    arr[0].rows, arr[0].cols, arr[0].fmt_mask = 4, 48, 1 << _lib.FMT_MXFP8
    arr[0].w = 16
    assert lib.pq_sweep_sse(arr, 1, ctypes.c_void_p(16), None) == _lib.PQ_ERR_SHAPE
    arr[0].fmt_mask = 1 << 7
    assert lib.pq_sweep_sse(arr, 1, ctypes.c_void_p(16), None) == _lib.PQ_ERR_FORMAT
    assert lib.pq_nvfp4_scales(300, None, None, None, None, None, None, None, None) == _lib.PQ_ERR_LIMIT
    mx, nv = 1 << _lib.FMT_MXFP8, 1 << _lib.FMT_NVFP4
    assert lib.pq_weighted_sse_fused(None, 4, 64, 0, None, 0, None, None) == _lib.PQ_ERR_FORMAT
    assert lib.pq_weighted_sse_fused(None, 4, 64, 1 << _lib.FMT_BF16, None, 0, None, None) == _lib.PQ_ERR_FORMAT
    assert lib.pq_weighted_sse_fused(None, 4, 48, mx, None, 0, None, None) == _lib.PQ_ERR_SHAPE
    assert lib.pq_weighted_sse_fused(None, 0, 64, nv | mx, None, 0, None, None) == _lib.PQ_OK
    assert lib.pq_weighted_sse_fused(None, 4, 64, nv | mx, None, 1, None, None) == _lib.PQ_ERR_NULL
    assert lib.pq_cost_qdq_fused_sse(None, -1, 4, 64, nv, None, None, None) == _lib.PQ_ERR_SHAPE
    assert lib.pq_cost_qdq_fused_sse(None, 2, 4, 64, 0, None, None, None) == _lib.PQ_ERR_FORMAT
    assert lib.pq_cost_qdq_fused_sse(None, 2, 4, 48, nv | mx, None, None, None) == _lib.PQ_ERR_SHAPE
    assert lib.pq_cost_qdq_fused_sse(None, 0, 4, 64, nv | mx, None, None, None) == _lib.PQ_OK
    assert lib.pq_cost_qdq_fused_sse(None, 2, 4, 64, nv | mx, None, None, None) == _lib.PQ_ERR_NULL
    assert lib.pq_weighted_sse_fused_batch(None, 2, 4, 48, mx, None, 0, None, None) == _lib.PQ_ERR_SHAPE
    assert lib.pq_weighted_sse_fused_batch(None, 2, 4, 64, 1 << 3, None, 0, None, None) == _lib.PQ_ERR_FORMAT
    assert lib.pq_weighted_sse_fused_batch(None, 0, 4, 64, nv, None, 0, None, None) == _lib.PQ_OK
    assert lib.pq_weighted_sse_fused_batch(None, 2, 4, 64, nv, None, 0, None, None) == _lib.PQ_ERR_NULL


def test_cuda_calls_fail_loudly_on_cpu_tensors():
    import torch
    from prismaquant_b200 import format_registry as fr
    with pytest.raises(RuntimeError):
        fr.get_format("NVFP4").quantize_dequantize(torch.zeros(4, 16, dtype=torch.bfloat16))


def test_e8m0_table_header_matches_oracle():
    from oracle import pq_oracle as O
    text = (REPO / "prismaquant_b200" / "csrc" / "pq_e8m0_tables.h").read_text()
    def arr(name):
        body = re.search(name + r"\[\d+\] = \{([^}]*)\}", text).group(1)
        return [int(v) for v in body.replace("\n", " ").split(",") if v.strip()]
    ceil_last, round_first = arr("PQ_CEIL_LAST"), arr("PQ_ROUND_FIRST")
    t = O.e8m0()
    assert ceil_last == [t.ceil_last[k] for k in range(-127, 128)]
    assert round_first == [t.round_first[k] for k in range(-126, 128)]


def test_format_registry_metadata_matches_reference_formats():
    from prismaquant_b200 import format_registry as fr
    shape = (128, 128)
    assert fr.get_format("NVFP4").effective_bits_for_shape(shape) == pytest.approx(4.5)
    assert fr.get_format("MXFP8").effective_bits_for_shape(shape) == pytest.approx(8.25)
    assert fr.get_format("BF16").effective_bits_for_shape(shape) == pytest.approx(16.0)
    spec = fr.get_format("FP8_E4M3")
    assert spec.scale_count_for_shape((5, 7)) == 5
    assert spec.memory_bytes_for_shape((5, 7)) == 5 * 7 + 5 * 4
    with pytest.raises(KeyError):
        fr.get_format("NOPE")


def test_cost_schema_roundtrip():
    from prismaquant_b200 import measure_quant_cost as mqc
    b = {}
    mqc._accumulate_result(b, "x", "NVFP4", 2.0, 1.0, 0.5, predicted_dloss=3.0)
    mqc._accumulate_result(b, "x", "NVFP4", 4.0, 3.0, 1.5)
    out = mqc._finalize_results(b)
    assert out["x"]["NVFP4"] == {"weight_mse": 3.0, "output_mse": 2.0, "rel_output_mse": 1.0, "predicted_dloss": 3.0}
    assert mqc.shape_error("MXFP8", 48) and mqc.shape_error("MXFP8", 16) is None
    assert mqc.shape_error("NVFP4", 24) and mqc.shape_error("NVFP4", 8) is None
    assert mqc.canonical_linear_name("m.mlp.experts.3.up_proj") == "m.mlp.experts.gate_up_proj.3"


def test_cost_schema_matches_reference_validator():
    """The cost table validates under the reference's own schema checker when it is importable."""
    import sys
    from tests.conftest import REFERENCE, reference_available
    if not reference_available():
        pytest.skip("reference checkout not present")
    sys.path.insert(0, str(REFERENCE))
    try:
        from prismaquant import schemas
    finally:
        sys.path.remove(str(REFERENCE))
    from prismaquant_b200 import measure_quant_cost as mqc
    b = {}
    mqc._accumulate_result(b, "model.layers.0.mlp.up_proj", "NVFP4", 1e-5, 0.0, 0.0)
    table = {"costs": mqc._finalize_results(b), "formats": ["NVFP4"], "meta": {}}
    fn = getattr(schemas, "validate_cost_payload", None)
    if fn is None:
        pytest.skip("reference has no cost validator")
    fn(table)


def test_sibling_keys_and_partition():
    from prismaquant_b200 import export_native_compressed as enc
    from prismaquant_b200 import distributed as D
    from prismaquant_b200 import synthetic as S
    assert enc.sibling_group_key("model.layers.3.self_attn.k_proj") == "model.layers.3.self_attn::qkv"
    assert enc.sibling_group_key("model.layers.3.mlp.down_proj") is None
    assert enc._fused_dense_group("model.layers.5.self_attn.q_proj")[0] == "model.layers.5"
    lin = S.llama_dense_linears()
    assert len(lin) == 32 * 7 + 1
    assert sum(np.prod(s) for _, s in lin) == 7_504_658_432
    sizes = [int(np.prod(s)) for _, s in lin]
    keys = [enc.sibling_group_key(n) for n, _ in lin]
    for world in (1, 2, 4, 8):
        ranks = D.partition_units(sizes, world, keys)
        loads = [sum(s for s, r in zip(sizes, ranks) if r == k) for k in range(world)]
        assert max(loads) / (sum(sizes) / world) < 1.10
        for k in set(x for x in keys if x):
            assert len({r for r, kk in zip(ranks, keys) if kk == k}) == 1


def _gloo_worker(rank, world, port, q):
    import os
    import torch
    import torch.distributed as dist
    from prismaquant_b200 import distributed as D
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n_units = 7
        ranks = [u % world for u in range(n_units)]
        ids = torch.tensor([u for u in range(n_units) if ranks[u] == rank])
        sse = torch.stack([torch.arange(4, dtype=torch.float64) + 10 * u for u in ids.tolist()])
        table = D.all_gather_costs(ids, sse, n_units, D.max_units_per_rank(ranks, world))
        buf = torch.full((3, 2), float(rank + 1), dtype=torch.float64)
        D.all_reduce_traces(buf)
        q.put((rank, table.tolist(), buf.tolist()))
    finally:
        dist.destroy_process_group()


def _gloo_fisher_worker(rank, world, port, q, detail_dir):
    import os
    import torch
    import torch.distributed as dist
    from prismaquant_b200 import distributed as D
    from prismaquant_b200 import sensitivity_probe as sp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        model = torch.nn.Sequential(torch.nn.Linear(16, 8, bias=False), torch.nn.Linear(8, 24, bias=False))
        acc = sp.FisherAccumulator(model, ["0", "1"], {}, hook_packed_experts=False,
                                   h_detail_dir=detail_dir if rank == 0 else detail_dir + f"_{rank}")
        # what each rank's backwards would have left: rank-dependent values
        acc._acc += torch.tensor([[0.0, 10.0], [0.0, 10.0]], dtype=torch.float64) * (rank + 1)
        acc._exact += torch.tensor([[1.0, 0.5], [2.0, 0.25]], dtype=torch.float64) * (rank + 1)
        acc._h_full["0"] = torch.full((8, 16), float(rank + 1))
        acc._h_full["1"] = torch.full((24, 8), 2.0 * (rank + 1))
        D.all_reduce_fisher(acc)
        if rank == 0:
            acc.finalize(None)
            blob = torch.load(os.path.join(detail_dir, "0.pt"), weights_only=False)
            q.put((rank, acc.stats["0"]["h_trace_raw"], acc.stats["1"]["h_w2_sum_raw"], acc.stats["0"]["n_tokens_seen"],
                   float(blob["h_diag"][0, 0]), acc.stats["1"]["h_detail_path"]))
        else:
            q.put((rank, float(acc._exact[0, 0]), float(acc._h_full["1"][0, 0]), None, None, None))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_fisher_detail_reduce(tmp_path):
    """all_reduce_fisher on two gloo ranks: the exact sums, tokens and per-weight diagonals add up,
    and rank 0's finalize writes the reference's h_detail files from the summed values."""
    import multiprocessing as mp
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    d = str(tmp_path / "hd")
    procs = [ctx.Process(target=_gloo_fisher_worker, args=(r, 2, port, q, d)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    r0, r1 = res
    assert r0[1:4] == (3.0, 0.75, 30)            # trace 1+2, w^2 sum 0.25*(1+2), tokens 10+20
    assert r0[4] == pytest.approx(3.0 / 30)      # h_diag = summed h_full / summed tokens
    assert r0[5] == "1.pt"
    assert r1[1:3] == (3.0, 6.0)


def test_gloo_two_ranks_gather_and_reduce():
    import multiprocessing as mp
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, table, buf in res:
        assert table == [[10.0 * u + j for j in range(4)] for u in range(7)]
        assert buf == [[3.0, 3.0]] * 3


def test_patch_prismaquant_rebinds_reference_functions():
    """install.patch_prismaquant rebinds the reference's hot-path functions in place (and restores them)."""
    import sys
    from tests.conftest import REFERENCE, reference_available
    if not reference_available():
        pytest.skip("reference checkout not present")
    shim = str(Path(__file__).resolve().parent.parent / "oracle" / "_shim")
    sys.path[:0] = [shim, str(REFERENCE)]
    try:
        import prismaquant.export_native_compressed as enc
        import prismaquant.format_registry as fr
        import prismaquant.measure_quant_cost as mqc
        import prismaquant.sensitivity_probe as sp
        from prismaquant_b200 import install
        orig = (fr.REGISTRY["NVFP4"].quantize_dequantize, mqc._batched_quantize, enc.quantize_dequantize_nvfp4,
                sp._GradNormCapture, fr.REGISTRY["INT3"].quantize_dequantize)
        done = install.patch_prismaquant()
        assert "measure_quant_cost._batched_quantize" in done
        assert fr.REGISTRY["NVFP4"].quantize_dequantize is not orig[0]
        assert enc.quantize_dequantize_nvfp4.__module__ == "prismaquant_b200.export_native_compressed"
        assert sp._GradNormCapture.__module__ == "prismaquant_b200.sensitivity_probe"
        assert fr.REGISTRY["INT3"].quantize_dequantize is not orig[4]  # the exact codebook / integer kernel
        install.unpatch_prismaquant()
        assert (fr.REGISTRY["NVFP4"].quantize_dequantize, mqc._batched_quantize, enc.quantize_dequantize_nvfp4,
                sp._GradNormCapture) == orig[:4]
    finally:
        for p in (shim, str(REFERENCE)):
            if p in sys.path:
                sys.path.remove(p)


def test_batched_dispatch_matches_oracle():
    """_batched_quantize picks the RTN by element dtype (measure_quant_cost.py:516-548), as the oracle's
    restatement does: NVFP3 raises, FP8_SOURCE is an E4M3 RTN with real groups of 128."""
    from oracle import pq_oracle as O
    from prismaquant_b200 import format_registry as fr
    from prismaquant_b200 import measure_quant_cost as mqc
    kernel = {"NVFP4": ("fp4_e2m1", 16, False), "MXFP4": ("fp4_e2m1", 32, True),
              "MXFP6_E3M2": ("fp6_e3m2", 32, True), "MXFP6_E2M3": ("fp6_e2m3", 32, True),
              "MXFP8": ("fp8_e4m3", 32, True), "FP8_E4M3": ("fp8_e4m3", 0, False),
              "FP8_E4M3_G128": ("fp8_e4m3", 128, False), "MXFP8_E5M2": ("fp8_e5m2", 32, True),
              "FP8_E5M2": ("fp8_e5m2", 0, False)}
    assert set(fr.REGISTRY) == set(O.REGISTRY_DTYPES)
    for name in fr.REGISTRY:
        spec = fr.get_format(name)
        elt, fam, bits, group = O.REGISTRY_DTYPES[name]
        assert (spec.weight_element_dtype, spec.family, spec.weight_bits, spec.group_size) == (elt, fam, bits, group)
        if elt == "fp3_e2m0":
            with pytest.raises(ValueError, match="Unknown weight_element_dtype"):
                mqc.batched_kernel_format(spec)
            continue
        k = mqc.batched_kernel_format(spec)
        if elt.startswith("int"):
            assert k == name
        elif elt == "bfloat16":
            assert k == "BF16"
        else:
            assert kernel[k] == (elt, group, fam == "mx")


def test_registry_matches_reference_registry():
    """Every format, alias and metadata field of the reference's REGISTRY (format_registry.py:368-576)."""
    import sys
    from tests.conftest import REFERENCE, reference_available
    if not reference_available():
        pytest.skip("reference checkout not present")
    from prismaquant_b200 import format_registry as ours
    shim = str(Path(__file__).resolve().parent.parent / "oracle" / "_shim")
    sys.path[:0] = [shim, str(REFERENCE)]
    try:
        import prismaquant.format_registry as ref
        assert set(ref.REGISTRY) == set(ours.REGISTRY)
        assert ref.FORMAT_ALIASES == ours.FORMAT_ALIASES
        fields = ("weight_bits", "group_size", "scale_bits", "scale_dtype_name", "weight_element_dtype",
                  "scale_block_shape", "act_bits", "act_dtype_name", "act_group_size", "family", "min_capability_sm")
        for name, r in ref.REGISTRY.items():
            o = ours.get_format(name)
            for f in fields:
                assert getattr(o, f) == getattr(r, f), (name, f)
            assert o.effective_bits == pytest.approx(r.effective_bits), name
            assert o.autoround_config() == r.autoround_config(), name
            for shape in ((4096, 4096), (7, 96), (3, 64, 256), (100,)):
                assert o.scale_count_for_shape(shape) == r.scale_count_for_shape(shape), (name, shape)
                assert o.memory_bytes_for_shape(shape) == r.memory_bytes_for_shape(shape), (name, shape)
        assert [s.name for s in ours.list_formats()] == [s.name for s in ref.list_formats()]
    finally:
        for p in (shim, str(REFERENCE)):
            if p in sys.path:
                sys.path.remove(p)


def test_safetensors_serializer_matches_safetensors():
    """Our serializer writes the same bytes as safetensors.torch.save_file (every dtype, scalars,
    empty tensors, with and without metadata)."""
    import tempfile

    import torch
    from safetensors.torch import save_file as st_save
    from prismaquant_b200 import safetensors_io as S
    g = torch.Generator().manual_seed(0)
    dts = [torch.bool, torch.uint8, torch.int8, torch.float8_e5m2, torch.float8_e4m3fn, torch.int16, torch.float16,
           torch.bfloat16, torch.int32, torch.float32, torch.float64, torch.int64]
    t = {}
    for i, d in enumerate(dts):
        x = torch.randn(3, 5 + i, generator=g) * 10
        t[f"model.layers.{i}.w{'xyz'[i % 3]}"] = x > 0 if d == torch.bool else x.to(d)
    t["scalar"] = torch.tensor(3.0)
    t["empty"] = torch.zeros(0, 4)
    with tempfile.TemporaryDirectory() as d:
        for md in (None, {"format": "pt"}):
            S.save_file(t, f"{d}/ours.safetensors", metadata=md)
            st_save(t, f"{d}/theirs.safetensors", metadata=md)
            assert Path(f"{d}/ours.safetensors").read_bytes() == Path(f"{d}/theirs.safetensors").read_bytes()


def _tree_bytes(root):
    return {p.name: p.read_bytes() for p in sorted(Path(root).iterdir())}


def test_sharded_writers_match_reference():
    """write_sharded_safetensors and IncrementalSafetensorsWriter write the same files (names,
    bytes, index) as the reference's (export_native_compressed.py:3977-4131)."""
    import sys
    import tempfile

    import torch
    from tests.conftest import REFERENCE, reference_available
    if not reference_available():
        pytest.skip("reference checkout not present")
    from prismaquant_b200 import safetensors_io as S
    shim = str(Path(__file__).resolve().parent.parent / "oracle" / "_shim")
    sys.path[:0] = [shim, str(REFERENCE)]
    try:
        import prismaquant.export_native_compressed as ref
        g = torch.Generator().manual_seed(1)
        tensors = {}
        for i in range(12):
            rows = 40 + 17 * i
            tensors[f"model.layers.{i}.mlp.down_proj.weight_packed"] = torch.randint(0, 255, (rows, 64), dtype=torch.uint8,
                                                                                      generator=g)
            tensors[f"model.layers.{i}.mlp.down_proj.weight_scale"] = (torch.rand(rows, 8, generator=g) * 100).to(
                torch.float8_e4m3fn)
            tensors[f"model.layers.{i}.mlp.down_proj.weight_global_scale"] = torch.rand(1, generator=g)
            tensors[f"model.layers.{i}.self_attn.o_proj.weight"] = torch.randn(32, 48, generator=g).to(torch.bfloat16)
        for shard in (10_000, 30_000, 10_000_000):
            with tempfile.TemporaryDirectory() as a, tempfile.TemporaryDirectory() as b:
                S.write_sharded_safetensors(tensors, Path(a), shard)
                ref.write_sharded_safetensors(tensors, Path(b), shard)
                assert _tree_bytes(a) == _tree_bytes(b)
            with tempfile.TemporaryDirectory() as a, tempfile.TemporaryDirectory() as b:
                wa, wb = S.IncrementalSafetensorsWriter(Path(a), shard), ref.IncrementalSafetensorsWriter(Path(b), shard)
                keys = sorted(tensors)
                for k0 in range(0, len(keys), 7):   # batches as an export would emit them
                    batch = {k: tensors[k] for k in keys[k0:k0 + 7]}
                    wa.add_tensors(batch)
                    wb.add_tensors(batch)
                wa.finalize()
                wb.finalize()
                assert _tree_bytes(a) == _tree_bytes(b)
                assert wa.weight_map == wb.weight_map
    finally:
        for p in (shim, str(REFERENCE)):
            if p in sys.path:
                sys.path.remove(p)


def test_patch_reaches_production_entry_points():
    """patch_prismaquant also rebinds the cost and probe entry points, in the reference's own modules
    and in the production modules that imported them by name (incremental_measure_quant_cost.py:53-62,
    incremental_probe.py:55-67); the installed FisherAccumulator defaults to the exact statistics;
    unpatch restores every name in every namespace."""
    import inspect
    import sys
    from tests.conftest import REFERENCE, reference_available
    if not reference_available():
        pytest.skip("reference checkout not present")
    shim = str(Path(__file__).resolve().parent.parent / "oracle" / "_shim")
    sys.path[:0] = [shim, str(REFERENCE)]
    try:
        import prismaquant.incremental_measure_quant_cost as imqc
        import prismaquant.incremental_probe as ip
        import prismaquant.measure_quant_cost as mqc
        import prismaquant.sensitivity_probe as sp
        from prismaquant_b200 import install
        from prismaquant_b200 import measure_quant_cost as our_mqc
        from prismaquant_b200 import sensitivity_probe as our_sp
        where = {mqc: install._COST_NAMES, imqc: install._COST_NAMES, sp: install._PROBE_NAMES,
                 ip: install._PROBE_NAMES}
        before = {(m, n): getattr(m, n) for m, names in where.items() for n in names}
        done = install.patch_prismaquant()
        for m, names in where.items():
            short = m.__name__.rsplit(".", 1)[1]
            for n in names:
                assert f"{short}.{n}" in done, (short, n)
                got = getattr(m, n)
                assert got is not before[(m, n)]
                if n in install._COST_NAMES:
                    assert got.__prismaquant_b200__ is getattr(our_mqc, n)
                elif n == "FisherAccumulator":
                    assert issubclass(got, our_sp.FisherAccumulator)
                else:
                    assert got is getattr(our_sp, n)
        # the production namespaces hold the very objects the reference modules hold
        assert imqc.measure_batched_gpu is mqc.measure_batched_gpu and ip.FisherAccumulator is sp.FisherAccumulator
        assert inspect.signature(sp.FisherAccumulator.__init__).parameters["h_detail_dir"].default is None
        install.unpatch_prismaquant()
        for (m, n), v in before.items():
            assert getattr(m, n) is v, (m.__name__, n)
        install.patch_prismaquant(fisher="per_token")
        install.unpatch_prismaquant()
        with pytest.raises(ValueError):
            install.patch_prismaquant(fisher="bogus")
    finally:
        for p in (shim, str(REFERENCE)):
            if p in sys.path:
                sys.path.remove(p)


def test_installed_cost_entry_keeps_reference_path_off_cuda():
    """The rebound measure_* functions hand a non-CUDA call (the reference's CPU mode) back to the
    reference's own function with the caller's arguments untouched."""
    from prismaquant_b200 import format_registry as our_fr
    from prismaquant_b200 import install

    calls = []

    def theirs(model, act_cache, target_names, specs, device, dtype, chunk_size=256, h_detail=None):
        calls.append(("theirs", device, chunk_size))
        return "ref"

    def ours(**kw):
        calls.append(("ours", kw["device"], kw["chunk_size"], [s.name for s in kw["specs"]]))
        return "b200"

    class Spec:
        def __init__(self, name):
            self.name = name

    w = install._cost_wrapper(ours, theirs, our_fr)
    assert w(None, None, set(), [Spec("NVFP4")], "cpu", None) == "ref"
    assert w(None, None, set(), [Spec("NVFP4"), Spec("MXFP8")], "cuda", None, chunk_size=8) == "b200"
    assert calls[-1] == ("ours", "cuda", 8, ["NVFP4", "MXFP8"])
    assert w(None, None, set(), [Spec("MY_CUSTOM_FORMAT")], "cuda:0", None) == "ref"


def test_plan_pieces_cuts_units_larger_than_a_share():
    """plan_pieces: every unit's rows covered once, in order; only 2-D units outside sibling groups
    and larger than total / world are cut, into ceil(size / share) near-equal row blocks; siblings
    stay together; one rank keeps everything whole."""
    from prismaquant_b200 import distributed as D
    from prismaquant_b200 import export_native_compressed as enc
    shapes = [("lm_head", (128256, 4096)), ("model.layers.0.self_attn.q_proj", (4096, 4096)),
              ("model.layers.0.self_attn.k_proj", (1024, 4096)), ("model.layers.0.self_attn.v_proj", (1024, 4096)),
              ("model.layers.0.mlp.experts.gate_up_proj", (128, 1536, 2048))]
    keys = [enc.sibling_group_key(n) for n, _ in shapes]
    for world in (1, 2, 4, 8, 16):
        pieces, ranks = D.plan_pieces(shapes, world, keys)
        assert len(ranks) == len(pieces)
        sizes = [int(np.prod(sh)) for _, sh in shapes]
        share = sum(sizes) / world
        for u, (name, sh) in enumerate(shapes):
            mine = [(r0, r1) for uu, r0, r1 in pieces if uu == u]
            assert mine[0][0] == 0 and mine[-1][1] == sh[0]
            assert all(a[1] == b[0] for a, b in zip(mine, mine[1:]))
            cut = world > 1 and keys[u] is None and len(sh) == 2 and sizes[u] > share
            assert len(mine) == (int(np.ceil(sizes[u] / share)) if cut else 1), (world, name)
        for k in {x for x in keys if x}:
            assert len({r for (u, _, _), r in zip(pieces, ranks) if keys[u] == k}) == 1
    assert D.plan_pieces(shapes, 1, keys)[0] == [(u, 0, sh[0]) for u, (_, sh) in enumerate(shapes)]


def _gloo_split_worker(rank, world, port, q):
    import os
    import torch
    import torch.distributed as dist
    from prismaquant_b200 import distributed as D
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # unit 0 cut in two (one block per rank), unit 1 whole on rank 0, unit 2 cut in two with
        # both blocks on rank 1
        pieces = {0: [(0, 0), (2, 0), (1, None)], 1: [(0, 1), (2, 1), (2, 1)]}[rank]
        ids = torch.tensor([u for u, _ in pieces])
        sse = torch.stack([torch.full((4,), 1.0 + u + 10 * rank, dtype=torch.float64) for u, _ in pieces])
        table = D.all_gather_costs(ids, sse, 3, 3)
        tmax = torch.tensor([100 + 7 * rank + j for j in range(len(pieces))], dtype=torch.int32)
        slots = torch.tensor([j for j, (_, s) in enumerate(pieces) if s is not None])
        sids = torch.tensor([{0: 0, 2: 1}[u] for u, s in pieces if s is not None])
        D.reduce_split_tmax(tmax, slots, sids, 2)
        q.put((rank, table.tolist(), tmax.tolist()))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_split_units():
    """Row blocks of one unit on two ranks (or twice on one): the gathered sums add up per unit,
    and reduce_split_tmax leaves every block of a split unit holding the unit's maximum."""
    import multiprocessing as mp
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_split_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (t, m)) for r, t, m in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = [[1.0 + 11.0] * 4, [2.0] * 4, [3.0 + 13.0 + 13.0] * 4]   # unit 2: one block on rank 0, two on rank 1
    for r in (0, 1):
        assert res[r][0] == want
    # unit 0: max(100, 107) on both; unit 2: max(101, 108, 109) on both; unit 1 untouched
    assert res[0][1] == [107, 109, 102]
    assert res[1][1] == [107, 109, 109]


def test_plan_chunks_keep_sibling_groups_whole():
    """SweepExportPlan's chunks: cover the tensors in order, at most 256 each, about equal bytes,
    and never put a cut between two members of one fused-sibling group, even when the members
    are not adjacent in the list."""
    from prismaquant_b200 import export_native_compressed as enc
    names = []
    for l in range(40):
        names += [f"model.layers.{l}.self_attn.{p}_proj" for p in ("q", "o", "k", "v")]   # o between siblings
        names += [f"model.layers.{l}.mlp.{p}_proj" for p in ("gate", "down", "up")]
    sizes = [4096 * 4096 if n.endswith(("q_proj", "o_proj")) else 1024 * 4096 if n.endswith(("k_proj", "v_proj"))
             else 14336 * 4096 for n in names]
    keys = [enc.sibling_group_key(n) for n in names]
    for target in (1, 2, 4, 7):
        chunks = enc._plan_chunks(sizes, keys, target)
        assert chunks[0][0] == 0 and chunks[-1][1] == len(names)
        assert all(a[1] == b[0] for a, b in zip(chunks, chunks[1:]))
        assert all(b - a <= 256 for a, b in chunks)
        where = {i: c for c, (a, b) in enumerate(chunks) for i in range(a, b)}
        for k in {x for x in keys if x}:
            assert len({where[i] for i, kk in enumerate(keys) if kk == k}) == 1, (target, k)
        if target > 1 and len(names) <= 256 * target:
            assert len(chunks) >= min(target, 2)
