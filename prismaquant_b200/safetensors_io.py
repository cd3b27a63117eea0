"""Safetensors shards for the packed checkpoint, written from pinned host memory.

Drop-in for the reference's writers (export_native_compressed.py:3977-4076
`IncrementalSafetensorsWriter`, :4078-4131 `write_sharded_safetensors`): the same
shard boundaries, file names, index JSON and bytes on disk, from a layout planner
(`even_shard_runs`, `shard_file_names`) and a writer of this module's own.  The file layout is
safetensors': an 8-byte little-endian header length, a compact JSON header
(`__metadata__` first, then one entry per tensor in data order) padded with
spaces to a multiple of 8 bytes, then the tensors' bytes back to back.  Data
order is dtype (widest first, in safetensors' dtype order) then name.  The
serializer is this module's own; tests check it byte for byte against
`safetensors.torch.save_file`.

`IncrementalSafetensorsWriter.add_tensors` can be fed from a background thread
while the GPU is still producing later chunks (`StreamingSweepExport.export_to`).
"""
from __future__ import annotations

import json
import os
import struct
from pathlib import Path

import torch

# safetensors' dtype names, in the order it lays data out (first = written first)
_DTYPE_ORDER = ("U64", "I64", "F64", "F32", "U32", "I32", "BF16", "F16", "U16", "I16", "F8_E4M3", "F8_E5M2", "I8",
                "U8", "BOOL")
_RANK = {n: i for i, n in enumerate(_DTYPE_ORDER)}
_DTYPE_NAME = {torch.uint64: "U64", torch.int64: "I64", torch.float64: "F64", torch.float32: "F32",
               torch.uint32: "U32", torch.int32: "I32", torch.bfloat16: "BF16", torch.float16: "F16",
               torch.uint16: "U16", torch.int16: "I16", torch.float8_e4m3fn: "F8_E4M3",
               torch.float8_e5m2: "F8_E5M2", torch.int8: "I8", torch.uint8: "U8", torch.bool: "BOOL"}


def _bytes_of(t: torch.Tensor) -> memoryview:
    t = t.detach()
    if t.device.type != "cpu":
        t = t.cpu()
    t = t.contiguous()
    if t.numel() == 0:
        return memoryview(b"")
    return memoryview(t.reshape(-1).view(torch.uint8).numpy())


def save_file(tensors: dict[str, torch.Tensor], path, metadata: dict[str, str] | None = None) -> None:
    """Write one safetensors file (same bytes as safetensors.torch.save_file)."""
    names = sorted(tensors, key=lambda k: (_RANK[_DTYPE_NAME[tensors[k].dtype]], k))
    header: dict = {}
    if metadata:
        header["__metadata__"] = dict(metadata)
    off = 0
    for k in names:
        t = tensors[k]
        n = t.numel() * t.element_size()
        header[k] = {"dtype": _DTYPE_NAME[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + n]}
        off += n
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * (-(8 + len(hb)) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for k in names:
            f.write(_bytes_of(tensors[k]))


# ---------------------------------------------------------------------------
# shard layout: which tensors go to which file, and the files' names and index
# ---------------------------------------------------------------------------
#
# The on-disk result must be what the reference's writers produce
# (export_native_compressed.py:3977-4131), because its loaders and tools read these
# checkpoints.  The rules that fix it:
#   * names are laid out in sorted order;
#   * one-shot writes aim every shard at the same size, total / ceil(total / budget), and
#     a shard is closed before the tensor that would take it past that size;
#   * streamed writes close a shard before a tensor that would take it past the budget, and
#     also right after a tensor that brings it to the budget or beyond;
#   * a single shard is `model.safetensors` with no index; n > 1 shards are
#     `model-<i>-of-<n>.safetensors` (five-digit, 1-based) plus
#     `model.safetensors.index.json` = {"metadata": {"total_size": bytes}, "weight_map":
#     {tensor: file}} written with two-space indentation;
#   * every file carries the metadata {"format": "pt"}.

_INDEX_NAME = "model.safetensors.index.json"
_FILE_META = {"format": "pt"}


def _nbytes(t: torch.Tensor) -> int:
    return int(t.numel() * t.element_size())


def shard_file_names(n_shards: int) -> list[str]:
    """Final file name of each of `n_shards` shards."""
    if n_shards == 1:
        return ["model.safetensors"]
    return ["model-%05d-of-%05d.safetensors" % (i, n_shards) for i in range(1, n_shards + 1)]


def even_shard_runs(sizes: list[int], shard_bytes: int) -> list[tuple[int, int]]:
    """[start, stop) runs of the (already ordered) sizes for a one-shot write: each run is closed
    before the element that would take it past the common target size."""
    total = sum(sizes)
    n_target = max(1, -(-total // shard_bytes))
    target = -(-total // n_target)
    runs: list[tuple[int, int]] = []
    start, fill = 0, 0
    for i, n in enumerate(sizes):
        if i > start and fill + n > target:
            runs.append((start, i))
            start, fill = i, 0
        fill += n
    runs.append((start, len(sizes)))
    return runs


def _write_index(out_dir: Path, files: list[str], keys_per_file: list[list[str]], total: int) -> None:
    wmap = {}
    for fname, keys in zip(files, keys_per_file):
        wmap.update(dict.fromkeys(keys, fname))
    (out_dir / _INDEX_NAME).write_text(json.dumps({"metadata": {"total_size": total}, "weight_map": wmap}, indent=2))


def write_sharded_safetensors(tensors: dict[str, torch.Tensor], out_dir: Path, shard_bytes: int) -> None:
    """Write `tensors` as near-equal shards of at most about `shard_bytes` each (drop-in for
    export_native_compressed.py:4078-4131; the layout rules are above)."""
    out_dir = Path(out_dir)
    order = sorted(tensors)
    runs = even_shard_runs([_nbytes(tensors[k]) for k in order], shard_bytes)
    files = shard_file_names(len(runs))
    groups = [order[a:b] for a, b in runs]
    for fname, keys in zip(files, groups):
        save_file({k: tensors[k] for k in keys}, out_dir / fname, metadata=_FILE_META)
    if len(files) > 1:
        _write_index(out_dir, files, groups, sum(_nbytes(t) for t in tensors.values()))


class IncrementalSafetensorsWriter:
    """Streamed checkpoint writer (drop-in for export_native_compressed.py:3977-4076).

    Tensors arrive in batches (`add_tensors`, each batch taken in name order).  The open shard
    is held in memory and spilled to a hidden temporary file whenever the streaming rule above
    closes it; `finalize` gives the spilled files their final names (which depend on how many
    there are) and writes the index.  `weight_map` is {tensor name: final file} after finalize."""

    def __init__(self, out_dir: Path, shard_bytes: int):
        self.out_dir = Path(out_dir)
        self.out_dir.mkdir(parents=True, exist_ok=True)
        self.shard_bytes = int(shard_bytes)
        self.weight_map: dict[str, str] = {}
        self._open: list[tuple[str, torch.Tensor]] = []
        self._open_bytes = 0
        self._spilled: list[tuple[Path, list[str]]] = []   # (temporary file, its tensor names)
        self._written: set[str] = set()
        self._total = 0

    def add_tensors(self, tensors: dict[str, torch.Tensor]) -> None:
        for name in sorted(tensors):
            if name in self._written:
                raise RuntimeError(f"tensor {name!r} was already added to this checkpoint")
            t = tensors[name]
            n = _nbytes(t)
            if self._open and self._open_bytes + n > self.shard_bytes:
                self._spill()
            self._open.append((name, t))
            self._open_bytes += n
            self._total += n
            self._written.add(name)
            if self._open_bytes >= self.shard_bytes:
                self._spill()

    def _spill(self) -> None:
        if not self._open:
            return
        tmp = self.out_dir / f".pq-shard-{len(self._spilled):05d}.partial"
        save_file(dict(self._open), tmp, metadata=_FILE_META)
        self._spilled.append((tmp, [name for name, _ in self._open]))
        self._open, self._open_bytes = [], 0

    def finalize(self) -> None:
        self._spill()
        if not self._spilled:
            raise RuntimeError("finalize() on a checkpoint with no tensors")
        files = shard_file_names(len(self._spilled))
        for fname, (tmp, keys) in zip(files, self._spilled):
            os.replace(tmp, self.out_dir / fname)
            self.weight_map.update(dict.fromkeys(keys, fname))
        if len(files) > 1:
            _write_index(self.out_dir, files, [keys for _, keys in self._spilled], self._total)
