"""Safetensors shards for the packed checkpoint, written from pinned host memory.

Drop-in for the reference's writers (export_native_compressed.py:3977-4076
`IncrementalSafetensorsWriter`, :4078-4131 `write_sharded_safetensors`): the same
shard boundaries, file names, index JSON and bytes on disk.  The file layout is
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
import math
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


def write_sharded_safetensors(tensors: dict[str, torch.Tensor], out_dir: Path, shard_bytes: int) -> None:
    """export_native_compressed.py:4078-4131: near-equal shards of the sorted keys; one file
    is `model.safetensors`, several are `model-0000i-of-0000n.safetensors` plus the index."""
    out_dir = Path(out_dir)
    keys = sorted(tensors)
    sizes = {k: tensors[k].numel() * tensors[k].element_size() for k in keys}
    total = sum(sizes.values())
    n_shards = max(1, math.ceil(total / shard_bytes))
    target = math.ceil(total / n_shards)
    shards: list[list[str]] = [[]]
    cur = 0
    for k in keys:
        if cur + sizes[k] > target and shards[-1]:
            shards.append([])
            cur = 0
        shards[-1].append(k)
        cur += sizes[k]
    if len(shards) == 1:
        save_file({k: tensors[k] for k in shards[0]}, out_dir / "model.safetensors", metadata={"format": "pt"})
        return
    weight_map: dict[str, str] = {}
    n = len(shards)
    for i, shard_keys in enumerate(shards):
        name = f"model-{i + 1:05d}-of-{n:05d}.safetensors"
        save_file({k: tensors[k] for k in shard_keys}, out_dir / name, metadata={"format": "pt"})
        for k in shard_keys:
            weight_map[k] = name
    with open(out_dir / "model.safetensors.index.json", "w") as f:
        json.dump({"metadata": {"total_size": total}, "weight_map": weight_map}, f, indent=2)


class IncrementalSafetensorsWriter:
    """export_native_compressed.py:3977-4076: keeps one shard resident, flushes it to a temporary
    file once adding the next tensor would pass `shard_bytes` (a single tensor at or above the
    budget is flushed on its own), and on finalize renames the shards to their final names and
    writes the index (none for a single shard)."""

    def __init__(self, out_dir: Path, shard_bytes: int):
        self.out_dir = Path(out_dir)
        self.shard_bytes = int(shard_bytes)
        self.current: dict[str, torch.Tensor] = {}
        self.current_size = 0
        self.total_size = 0
        self.tmp_shards: list[tuple[Path, list[str]]] = []
        self.weight_map: dict[str, str] = {}
        self.seen_keys: set[str] = set()
        self.out_dir.mkdir(parents=True, exist_ok=True)

    def add_tensors(self, tensors: dict[str, torch.Tensor]) -> None:
        for key in sorted(tensors):
            if key in self.seen_keys:
                raise RuntimeError(f"duplicate tensor key emitted during export: {key}")
            t = tensors[key]
            size = int(t.numel() * t.element_size())
            if self.current and self.current_size + size > self.shard_bytes:
                self._flush_current()
            self.current[key] = t
            self.current_size += size
            self.total_size += size
            self.seen_keys.add(key)
            if self.current_size >= self.shard_bytes:
                self._flush_current()

    def _flush_current(self) -> None:
        if not self.current:
            return
        idx = len(self.tmp_shards) + 1
        tmp = self.out_dir / f".model-{idx:05d}.safetensors.tmp"
        save_file(self.current, tmp, metadata={"format": "pt"})
        self.tmp_shards.append((tmp, list(self.current.keys())))
        self.current = {}
        self.current_size = 0

    def finalize(self) -> None:
        self._flush_current()
        if not self.tmp_shards:
            raise RuntimeError("no tensors were written")
        if len(self.tmp_shards) == 1:
            tmp, keys = self.tmp_shards[0]
            os.replace(tmp, self.out_dir / "model.safetensors")
            for k in keys:
                self.weight_map[k] = "model.safetensors"
            return
        n = len(self.tmp_shards)
        for i, (tmp, keys) in enumerate(self.tmp_shards, start=1):
            name = f"model-{i:05d}-of-{n:05d}.safetensors"
            os.replace(tmp, self.out_dir / name)
            for k in keys:
                self.weight_map[k] = name
        with open(self.out_dir / "model.safetensors.index.json", "w") as f:
            json.dump({"metadata": {"total_size": self.total_size}, "weight_map": self.weight_map}, f, indent=2)
