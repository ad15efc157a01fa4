"""Minimal safetensors reader (mmap, zero-copy tensor views) and writer.

File layout: little-endian u64 header length N, N bytes of JSON
``{name: {"dtype", "shape", "data_offsets": [begin, end]}, "__metadata__": {...}}``,
then the raw tensor bytes (offsets relative to the end of the header).  The reader
maps each file once and returns tensors that alias the mapping, so a loader can copy
expert weights straight into their final home (NUMA-sharded engine memory, pinned
staging or the GPU) without an intermediate host copy.
"""
from __future__ import annotations

import json
import mmap
import os
import struct
from pathlib import Path

import torch

DTYPES = {
    "F64": torch.float64, "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16,
    "F8_E4M3": torch.float8_e4m3fn, "F8_E5M2": torch.float8_e5m2, "I64": torch.int64, "I32": torch.int32,
    "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8, "BOOL": torch.bool,
}
NAMES = {v: k for k, v in DTYPES.items()}


class SafetensorsFile:
    def __init__(self, path: str | Path):
        self.path = str(path)
        self._f = open(self.path, "rb")
        n = struct.unpack("<Q", self._f.read(8))[0]
        self.header = json.loads(self._f.read(n))
        self.meta = self.header.pop("__metadata__", {})
        self.base = 8 + n
        size = os.fstat(self._f.fileno()).st_size
        self._mm = mmap.mmap(self._f.fileno(), size, access=mmap.ACCESS_READ) if size > 0 else None

    def keys(self):
        return self.header.keys()

    def get(self, name: str) -> torch.Tensor:
        h = self.header[name]
        dt = DTYPES[h["dtype"]]
        b, e = h["data_offsets"]
        shape = h["shape"]
        count = (e - b) // torch.tensor([], dtype=dt).element_size()
        if count == 0:
            return torch.empty(shape, dtype=dt)
        import warnings
        with warnings.catch_warnings():       # the mapping is read-only; callers copy what they keep
            warnings.simplefilter("ignore")
            t = torch.frombuffer(self._mm, dtype=dt, count=count, offset=self.base + b)
        return t.view(shape)

    def close(self):
        if self._mm is not None:
            self._mm.close()
            self._mm = None
        self._f.close()


class CheckpointDir:
    """All ``*.safetensors`` files of a checkpoint directory behind one name index."""

    def __init__(self, path: str | Path):
        self.path = Path(path)
        files = sorted(self.path.glob("*.safetensors")) if self.path.is_dir() else [self.path]
        self.files = [SafetensorsFile(f) for f in files]
        self.index = {}
        for f in self.files:
            for k in f.keys():
                self.index[k] = f

    def __contains__(self, name: str) -> bool:
        return name in self.index

    def get(self, name: str) -> torch.Tensor:
        try:
            return self.index[name].get(name)
        except KeyError:
            raise KeyError(f"tensor {name!r} not in checkpoint {self.path}") from None

    def keys(self):
        return self.index.keys()

    def close(self):
        for f in self.files:
            f.close()


def save_file(tensors: dict[str, torch.Tensor], path: str | Path, metadata: dict | None = None) -> None:
    header, off, blobs = {}, 0, []
    for name, t in tensors.items():
        t = t.detach().contiguous().cpu()
        raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": NAMES[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        off += len(raw)
        blobs.append(raw)
    if metadata:
        header["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for raw in blobs:
            f.write(raw)
