"""GGUF files: read through the library's C-ABI reader (csrc/qg_gguf.cu) into resident
packs, and written from the public GGUF layout (for tests and tooling).

* `GGUFFile(path)` -- header summary and tensor table (`tensors`, `info`), `read(name)`
  returns a tensor's bytes, `pack(name)` a packs.Pack of a Q4_K / Q5_K / IQ2_S / IQ3_S
  tensor (rows = element count / dims[0], cols = dims[0]).
* `ingest(path, out_dir, names=None, q4k_policy="split-native")` -- the reference packers'
  job (tools/bench/q4k_resident_pack.py, iq_resident_pack.py, q5k_resident_pack.py): the
  selected tensors into resident-pack directories with manifest.json files
  (qgemv_b200/manifest.py), the GGUF offsets recorded as source offsets.
* `write_gguf(path, tensors, metadata)` -- a version-3 GGUF file: magic "GGUF", version,
  tensor and metadata counts, metadata key/value pairs, tensor infos (name, dims, ggml type,
  offset), the data section aligned to general.alignment, each tensor's bytes padded to it.
"""

from __future__ import annotations

import ctypes
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import manifest, packs
from ._lib import CudaError, call, check

GGML_TYPE = {"F32": 0, "F16": 1, "Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "IQ3_S": 21, "IQ2_S": 22}
FORMAT_OF_GGML = {12: packs.Q4K_RAW, 13: packs.Q5K, 21: packs.IQ3S, 22: packs.IQ2S}
GGML_OF_FORMAT = {v: k for k, v in FORMAT_OF_GGML.items()}


class GGUFInfo(ctypes.Structure):
    _fields_ = [("version", ctypes.c_uint32), ("tensor_count", ctypes.c_uint64),
                ("metadata_count", ctypes.c_uint64), ("tensor_info_end_offset", ctypes.c_uint64),
                ("tensor_data_offset", ctypes.c_uint64), ("tensor_data_alignment", ctypes.c_uint64),
                ("supported_tensors", ctypes.c_uint64), ("valid_tensors", ctypes.c_uint64),
                ("expected_data_bytes", ctypes.c_uint64), ("architecture", ctypes.c_char * 64)]


class GGUFTensorInfo(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 256), ("ggml_type", ctypes.c_uint32),
                ("n_dims", ctypes.c_uint32), ("dims", ctypes.c_uint64 * 4),
                ("offset", ctypes.c_uint64), ("absolute_offset", ctypes.c_uint64),
                ("span_bytes", ctypes.c_uint64), ("data_bytes", ctypes.c_uint64),
                ("block_size", ctypes.c_uint32), ("type_size", ctypes.c_uint32),
                ("valid", ctypes.c_uint32)]


@dataclass
class TensorEntry:
    index: int
    name: str
    ggml_type: int
    dims: list
    offset: int
    absolute_offset: int
    span_bytes: int
    data_bytes: int
    valid: bool


class GGUFFile:
    def __init__(self, path: str | Path):
        self.path = Path(path)
        self.handle = ctypes.c_void_p(None)
        check("qg_gguf_open", str(self.path).encode(), ctypes.byref(self.handle))
        info = GGUFInfo()
        check("qg_gguf_summary", self.handle, ctypes.byref(info))
        self.info = {f: getattr(info, f) for f, _ in GGUFInfo._fields_ if f != "architecture"}
        self.info["architecture"] = info.architecture.decode()
        self.tensors: dict[str, TensorEntry] = {}
        for i in range(info.tensor_count):
            t = GGUFTensorInfo()
            check("qg_gguf_tensor", self.handle, i, ctypes.byref(t))
            self.tensors[t.name.decode()] = TensorEntry(
                i, t.name.decode(), t.ggml_type, list(t.dims[: t.n_dims]), t.offset,
                t.absolute_offset, t.span_bytes, t.data_bytes, bool(t.valid))

    def read(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        buf = np.empty(t.data_bytes, np.uint8)
        check("qg_gguf_read", self.handle, t.index, buf.ctypes.data, t.data_bytes)
        return buf

    def pack(self, name: str) -> packs.Pack:
        t = self.tensors[name]
        if t.ggml_type not in FORMAT_OF_GGML:
            raise ValueError(f"{name}: ggml type {t.ggml_type} is not a decode-path format")
        cols = int(t.dims[0])
        rows = int(np.prod(t.dims)) // cols
        return packs.Pack(FORMAT_OF_GGML[t.ggml_type], rows, cols, self.read(name), None)

    def close(self) -> None:
        if self.handle.value:
            call("qg_gguf_close", self.handle)
            self.handle = ctypes.c_void_p(None)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ingest(path: str | Path, out_dir: str | Path, names: list[str] | None = None,
           q4k_policy: str = "split-native") -> dict[str, Path]:
    """GGUF tensors -> resident packs + manifests: {"q4k": manifest, "iq": ..., "q5k": ...}
    for the families present among the selected tensors."""
    out_dir = Path(out_dir)
    result = {}
    with GGUFFile(path) as g:
        sel = [n for n in (names or list(g.tensors)) if g.tensors[n].ggml_type in FORMAT_OF_GGML]
        groups: dict[str, list] = {"q4k": [], "iq": [], "q5k": []}
        for n in sel:
            pk = g.pack(n)
            key = {packs.Q4K_RAW: "q4k", packs.Q5K: "q5k"}.get(pk.fmt, "iq")
            groups[key].append((n, pk, g.tensors[n].absolute_offset))
        for key, items in groups.items():
            if not items:
                continue
            tensors = [(n, pk) for n, pk, _ in items]
            offs = [o for _, _, o in items]
            if key == "q4k":
                result[key] = manifest.write_q4k_manifest(out_dir / key, tensors, q4k_policy,
                                                          model=str(path), source_offsets=offs)
            else:
                result[key] = manifest.write_raw_manifest(out_dir / key, tensors, model=str(path),
                                                          source_offsets=offs)
    return result


# --------------------------------------------------------------------------- writer

def _gguf_string(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _gguf_value(v) -> tuple[int, bytes]:
    if isinstance(v, bool):
        return 7, struct.pack("<?", v)
    if isinstance(v, int):
        return (4, struct.pack("<I", v)) if 0 <= v < 2**32 else (11, struct.pack("<q", v))
    if isinstance(v, float):
        return 6, struct.pack("<f", v)
    if isinstance(v, str):
        return 8, _gguf_string(v)
    if isinstance(v, (list, tuple)):
        if not v:
            return 9, struct.pack("<IQ", 4, 0)
        t0, _ = _gguf_value(v[0])
        body = b"".join(_gguf_value(x)[1] for x in v)
        return 9, struct.pack("<IQ", t0, len(v)) + body
    raise TypeError(f"unsupported metadata value {v!r}")


def write_gguf(path: str | Path, tensors: list[tuple[str, int, list, bytes]],
               metadata: dict | None = None, alignment: int = 32) -> Path:
    """tensors: (name, ggml type id, dims in GGUF order, raw bytes).  Returns the path."""
    meta = {"general.architecture": "llama", "general.alignment": alignment}
    meta.update(metadata or {})
    out = bytearray(b"GGUF")
    out += struct.pack("<IQQ", 3, len(tensors), len(meta))
    for k, v in meta.items():
        t, body = _gguf_value(v)
        out += _gguf_string(k) + struct.pack("<I", t) + body
    offset = 0
    offsets = []
    for name, gtype, dims, data in tensors:
        out += _gguf_string(name) + struct.pack("<I", len(dims))
        out += b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", gtype, offset)
        offsets.append(offset)
        offset += (len(data) + alignment - 1) // alignment * alignment
    out += b"\0" * ((-len(out)) % alignment)
    for (_, _, _, data), off in zip(tensors, offsets):
        out += data
        out += b"\0" * ((-len(data)) % alignment)
    Path(path).write_bytes(bytes(out))
    return Path(path)


__all__ = ["GGUFFile", "ingest", "write_gguf", "GGML_TYPE", "CudaError"]
