"""The `.fni8` weight container: writer, reader and `save_fni8`.

fni8-serve imports `FQReader`, `save_fni8` (fni8serve/loader.py:16) and the streaming
`fni8.format.FQWriter` (fni8serve/convert.py:320-356) from its kernels package; the byte
format is defined inside that package, which is not available, so this module defines
its own and keeps the reference's call contract:

    save_fni8(path, {name: QTensor}, shards=None, meta=None)
    with FQWriter(path) as w: w.add(name, qt); ...; w.finalize(meta=...)
    with FQReader(path) as r:
        r.header["arch"], r.header["quant"], r.header["version"], r.header.get("__meta__")
        r.names, r.shards ({"experts": {id: [names]}, "pp_stages": [[names], ...]})
        r.load_many(names, device) -> {name: QTensor}

Layout (little-endian): an 8-byte magic, the tensor bytes, each part starting on a
4096-byte boundary, then the JSON header, then a 24-byte footer (header offset, header
length, magic). Every part is the resident layout the kernels read (per_row_i8: int8
[N, K] row-major + fp32 scale [N]; per_group_i4: packed uint8 [N, K/2] + fp32 scale
[N, K/group]; raw: the tensor as is), so a load is a page-aligned read of exactly the
requested tensors' bytes and one host-to-device copy: no dequantisation, repacking or
transposition (the contract of fni8serve/loader.py:1-8). A writer streams tensors to
disk as they are added, so peak memory is one tensor (fni8serve/convert.py:313-318).
"""
from __future__ import annotations

import json
import mmap
import os
import struct

import torch

from .qtensor import QTensor

MAGIC = b"FNI8B200"
FORMAT_VERSION = 1
ALIGN = 4096
_FOOTER = struct.Struct("<QQ8s")

_DTYPES = {
    "int8": torch.int8, "uint8": torch.uint8, "int16": torch.int16, "int32": torch.int32, "int64": torch.int64,
    "float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32, "float64": torch.float64,
    "bool": torch.bool,
}
_NAMES = {v: k for k, v in _DTYPES.items()}


class FQWriter:
    """Streams QTensors into a `.fni8` file; `finalize(meta=)` writes the header."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "wb")
        self._f.write(MAGIC)
        self._entries: dict[str, dict] = {}
        self._done = False

    def __enter__(self) -> "FQWriter":
        return self

    def __exit__(self, exc_type, exc, tb) -> None:
        if exc_type is None and not self._done:
            self.finalize()
        self._f.close()
        if exc_type is not None:
            try:
                os.remove(self.path)  # never leave a truncated container behind
            except OSError:
                pass

    def _part(self, t: torch.Tensor) -> dict:
        if t.dtype not in _NAMES:
            raise TypeError(f"fni8 format: unsupported dtype {t.dtype}")
        t = t.detach().contiguous().cpu()
        pad = (-self._f.tell()) % ALIGN
        if pad:
            self._f.write(b"\0" * pad)
        off = self._f.tell()
        nbytes = t.numel() * t.element_size()
        if nbytes:
            self._f.write(t.reshape(-1).view(torch.uint8).numpy())  # the tensor's bytes, no copy
        return {"dtype": _NAMES[t.dtype], "shape": list(t.shape), "offset": off, "nbytes": nbytes}

    def add(self, name: str, qt: QTensor) -> None:
        if self._done:
            raise RuntimeError("fni8 format: add() after finalize()")
        if name in self._entries:
            raise ValueError(f"fni8 format: duplicate tensor {name!r}")
        if not isinstance(qt, QTensor):
            qt = QTensor(qt, None, scheme="raw")
        entry = {"scheme": qt.scheme, "group_size": qt.group_size, "codebook": qt.codebook,
                 "data": self._part(qt.data), "scale": None if qt.scale is None else self._part(qt.scale)}
        self._entries[name] = entry

    def finalize(self, meta: dict | None = None, shards: dict | None = None) -> None:
        if self._done:
            return
        meta = dict(meta or {})
        schemes = {e["scheme"] for e in self._entries.values()} - {"raw"}
        quant = ("int8" if schemes == {"per_row_i8"} else "int4" if schemes == {"per_group_i4"} else
                 "mixed" if schemes else "raw")
        header = {"version": FORMAT_VERSION, "arch": meta.get("arch", ""), "quant": quant, "__meta__": meta,
                  "shards": shards or {}, "tensors": self._entries}
        cfg = meta.get("config")
        if isinstance(cfg, dict):  # model dimensions readable straight from the header
            for k, v in cfg.items():
                header.setdefault(k, v)
        blob = json.dumps(header).encode()
        off = self._f.tell()
        self._f.write(blob)
        self._f.write(_FOOTER.pack(off, len(blob), MAGIC))
        self._f.flush()
        self._done = True


def save_fni8(path: str, tensors: dict, *, shards: dict | None = None, meta: dict | None = None) -> None:
    """Write {name: QTensor} (plain tensors are stored as `raw`) to `path`."""
    if shards:
        known = set(tensors)
        listed = [n for v in shards.get("experts", {}).values() for n in v]
        listed += [n for stage in shards.get("pp_stages", []) for n in stage]
        missing = [n for n in listed if n not in known]
        if missing:
            raise KeyError(f"fni8 format: shard index names unknown tensors {missing[:4]}")
    with FQWriter(path) as w:
        for name, qt in tensors.items():
            w.add(name, qt)
        w.finalize(meta=meta, shards=shards)


class FQReader:
    """Reads a `.fni8` file: header, names, shard index, and partial loads."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        size = os.fstat(self._f.fileno()).st_size
        if size < len(MAGIC) + _FOOTER.size or self._f.read(len(MAGIC)) != MAGIC:
            self._f.close()
            raise ValueError(f"{path}: not a .fni8 container")
        self._f.seek(size - _FOOTER.size)
        off, length, magic = _FOOTER.unpack(self._f.read(_FOOTER.size))
        if magic != MAGIC or off + length + _FOOTER.size != size:
            self._f.close()
            raise ValueError(f"{path}: corrupt .fni8 footer")
        self._f.seek(off)
        self.header = json.loads(self._f.read(length))
        if self.header.get("version") != FORMAT_VERSION:
            self._f.close()
            raise ValueError(f"{path}: .fni8 version {self.header.get('version')} (this reader: {FORMAT_VERSION})")
        self._tensors = self.header["tensors"]
        self.names = list(self._tensors)
        self.shards = self.header.get("shards") or {}
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ) if size else None

    def __enter__(self) -> "FQReader":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def close(self) -> None:
        if self._mm is not None:
            self._mm.close()
            self._mm = None
        if not self._f.closed:
            self._f.close()

    def _tensor(self, part: dict, device) -> torch.Tensor:
        dt = _DTYPES[part["dtype"]]
        shape = part["shape"]
        if part["nbytes"] == 0:
            return torch.empty(shape, dtype=dt, device=device)
        # one copy of exactly this part's bytes (only its pages fault in from the file)
        with memoryview(self._mm) as mv:
            buf = bytearray(mv[part["offset"]:part["offset"] + part["nbytes"]])
        t = torch.frombuffer(buf, dtype=torch.uint8).view(dt).reshape(shape)
        return t.to(device) if torch.device(device).type != "cpu" else t

    def load(self, name: str, device="cpu") -> QTensor:
        e = self._tensors[name]
        data = self._tensor(e["data"], device)
        scale = None if e["scale"] is None else self._tensor(e["scale"], device)
        return QTensor(data, scale, scheme=e["scheme"], group_size=e["group_size"], codebook=e["codebook"])

    def load_many(self, names, device="cpu") -> dict:
        missing = [n for n in names if n not in self._tensors]
        if missing:
            raise KeyError(f"{self.path}: no tensors {missing[:4]}")
        return {n: self.load(n, device) for n in names}
