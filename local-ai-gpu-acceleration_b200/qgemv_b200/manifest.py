"""Resident-pack manifests in the reference's on-disk format, written and read.

The reference's packers emit one directory per pack set: a payload file per tensor (and,
for Q4_K, a metadata file) plus `manifest.json`, which its C++ loaders read
(runtime/loaders/iq_manifest.h:49-57, runtime/loaders/q4k_manifest.h:53-69):

* raw-block packs (IQ2_S, IQ3_S, Q5_K): `<label>.<type>_raw_blocks.bin` holding the GGUF
  blocks unchanged, one tensor row per entry (tools/bench/iq_resident_pack.py:115-147,
  tools/bench/q5k_resident_pack.py:93-120);
* Q4_K split packs: `<label>.q4k_payload.bin` (128 B/block) + `<label>.q4k_meta.<fmt>.bin`
  (tools/bench/q4k_resident_pack.py:170-222), optionally the raw blocks too.

Checksums are the byte sums the packers and loaders use (iq_resident_pack.py:43-44).
Dimensions follow GGUF: [cols, rows].  `write_*` create packs from `packs.Pack` objects
(synthetic or ingested from a GGUF file); `read_manifest` loads a directory written by
either these functions or the reference's own packers and validates sizes and checksums
the way the C++ loaders do.
"""

from __future__ import annotations

import json
import re
from datetime import datetime, timezone
from pathlib import Path

import numpy as np

from . import packs

TYPE_OF_FORMAT = {packs.IQ2S: "IQ2_S", packs.IQ3S: "IQ3_S", packs.Q5K: "Q5_K", packs.Q4K_RAW: "Q4_K"}
FORMAT_OF_TYPE = {v: k for k, v in TYPE_OF_FORMAT.items()}
BLOCK_TYPE_SIZE = {"IQ2_S": 82, "IQ3_S": 110, "Q5_K": 176, "Q4_K": 144}
RAW_KERNEL = {"IQ2_S": "iq2s_raw_block_probe", "IQ3_S": "iq3s_raw_block_probe",
              "Q5_K": "q5_k_raw_pending"}
# split-policy name in the manifest -> (pack format, metadata format name)
# (q4k_resident_pack.py:82-88)
Q4K_POLICIES = {
    "split-predecoded": (packs.Q4K_PREDECODED, "fp32-products"),
    "split-half": (packs.Q4K_HALF, "fp16-products"),
    "split-compact": (packs.Q4K_COMPACT, "compact-u8"),
    "split-native": (packs.Q4K_NATIVE, "native16"),
}
_LAYER_RE = re.compile(r"^blk\.(?P<layer>\d+)\.(?P<role>.+)$")


def checksum(data) -> int:
    return int(np.frombuffer(bytes(data) if not isinstance(data, np.ndarray) else data.tobytes(),
                             np.uint8).sum(dtype=np.uint64))


def sanitize_label(name: str) -> str:
    return re.sub(r"[^A-Za-z0-9_.-]+", "_", name)


def _role(name: str) -> tuple[int | None, str]:
    m = _LAYER_RE.match(name)
    if m:
        return int(m.group("layer")), m.group("role")
    return None, name  # written as null, which the loaders read as layer -1


# Offsets of the tensors in their (GGUF) source file.  The loaders require a non-zero
# offset; packs made without a source file are given the offsets a GGUF data section
# starting at 1 MiB with 32-byte alignment would give them.
_SOURCE_BASE = 1 << 20


def _source_offsets(sizes: list[int], offsets: list[int] | None) -> list[int]:
    if offsets is not None:
        return list(offsets)
    out, at = [], _SOURCE_BASE
    for n in sizes:
        out.append(at)
        at += (n + 31) // 32 * 32
    return out


def write_raw_manifest(out_dir: Path, tensors: list[tuple[str, packs.Pack]], model: str = "synthetic",
                       tensor_plan: str = "synthetic", source_offsets: list[int] | None = None) -> Path:
    """IQ2_S / IQ3_S / Q5_K raw-block packs and their manifest.json; returns its path.
    `source_offsets`: the tensors' offsets in their source file (GGUF ingest)."""
    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    rows_out, types = [], set()
    offs = _source_offsets([pk.payload.size for _, pk in tensors], source_offsets)
    for (name, pk), src_off in zip(tensors, offs):
        ttype = TYPE_OF_FORMAT[pk.fmt]
        if ttype == "Q4_K":
            raise ValueError("Q4_K tensors use write_q4k_manifest")
        types.add(ttype)
        payload = np.ascontiguousarray(pk.payload, np.uint8)
        label = sanitize_label(name)
        path = out_dir / f"{label}.{ttype.lower()}_raw_blocks.bin"
        path.write_bytes(payload.tobytes())
        layer, role = _role(name)
        cs = checksum(payload)
        rows_out.append({
            "name": name, "type": ttype, "layer": layer, "role": role,
            "dimensions": [pk.cols, pk.rows], "element_count": pk.rows * pk.cols,
            "block_size": 256, "block_type_size": BLOCK_TYPE_SIZE[ttype],
            "block_count": pk.rows * pk.cols // 256, "source_offset": int(src_off),
            "source_bytes": int(payload.size), "source_checksum": cs,
            "payload_path": str(path), "payload_bytes": int(payload.size), "payload_checksum": cs,
            "resident_bytes": int(payload.size), "policy": "raw-blocks",
            "runtime_kernel": RAW_KERNEL[ttype],
        })
    manifest = {
        "path": "iq_resident_pack", "generated_at": datetime.now(timezone.utc).isoformat(),
        "model": model, "tensor_plan": tensor_plan, "output_dir": str(out_dir),
        "types": sorted(types), "tensor_count": len(rows_out),
        "source_bytes": sum(r["source_bytes"] for r in rows_out),
        "payload_bytes": sum(r["payload_bytes"] for r in rows_out),
        "resident_bytes": sum(r["resident_bytes"] for r in rows_out),
        "tensors": rows_out,
    }
    path = out_dir / "manifest.json"
    path.write_text(json.dumps(manifest, indent=2), encoding="utf-8")
    return path


def write_q4k_manifest(out_dir: Path, tensors: list[tuple[str, packs.Pack]], policy: str,
                       write_blocks: bool = True, model: str = "synthetic",
                       tensor_plan: str = "synthetic", source_offsets: list[int] | None = None) -> Path:
    """Q4_K split packs (payload + metadata of `policy`) from raw Q4_K packs."""
    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    fmt, tag = Q4K_POLICIES[policy]
    rows_out = []
    offs = _source_offsets([pk.payload.size for _, pk in tensors], source_offsets)
    for (name, pk), src_off in zip(tensors, offs):
        if pk.fmt != packs.Q4K_RAW:
            raise ValueError("write_q4k_manifest takes raw Q4_K packs")
        blocks = np.ascontiguousarray(pk.payload, np.uint8)
        s_payload, s_meta = packs.split_q4k(blocks, fmt)
        label = sanitize_label(name)
        p_path = out_dir / f"{label}.q4k_payload.bin"
        m_path = out_dir / f"{label}.q4k_meta.{tag}.bin"
        p_path.write_bytes(s_payload.tobytes())
        m_path.write_bytes(s_meta.tobytes())
        b_path = ""
        if write_blocks:
            b_path = str(out_dir / f"{label}.q4k_blocks.bin")
            Path(b_path).write_bytes(blocks.tobytes())
        res = int(s_payload.size + s_meta.size)
        rows_out.append({
            "name": name, "dimensions": [pk.cols, pk.rows], "rows": pk.rows, "cols": pk.cols,
            "block_count": pk.rows * pk.cols // 256, "source_offset": int(src_off),
            "source_bytes": int(blocks.size), "source_checksum": checksum(blocks),
            "policy": policy, "metadata_format": tag, "payload_path": str(p_path),
            "payload_bytes": int(s_payload.size), "payload_checksum": checksum(s_payload),
            "metadata_path": str(m_path), "metadata_bytes": int(s_meta.size),
            "metadata_checksum": checksum(s_meta), "blocks_path": b_path,
            "resident_bytes": res, "compression_ratio_vs_fp16": pk.rows * pk.cols * 2 / float(res),
            "runtime_kernel": policy,
        })
    manifest = {
        "path": "q4k_resident_pack", "generated_at": datetime.now(timezone.utc).isoformat(),
        "model": model, "tensor_plan": tensor_plan, "output_dir": str(out_dir), "policy": policy,
        "write_blocks": write_blocks, "tensor_count": len(rows_out),
        "source_bytes": sum(r["source_bytes"] for r in rows_out),
        "payload_bytes": sum(r["payload_bytes"] for r in rows_out),
        "metadata_bytes": sum(r["metadata_bytes"] for r in rows_out),
        "resident_bytes": sum(r["resident_bytes"] for r in rows_out),
        "tensors": rows_out,
    }
    path = out_dir / "manifest.json"
    path.write_text(json.dumps(manifest, indent=2), encoding="utf-8")
    return path


def _resolve(manifest_path: Path, p: str) -> Path:
    q = Path(p)
    return q if q.is_absolute() else manifest_path.parent / q


def read_manifest(path: Path) -> dict[str, packs.Pack]:
    """Every tensor of a manifest as a packs.Pack (raw blocks, or Q4_K split payload +
    metadata), with the sizes and byte-sum checksums validated like the C++ loaders."""
    path = Path(path)
    m = json.loads(path.read_text(encoding="utf-8"))
    out = {}
    for t in m["tensors"]:
        cols, rows = int(t["dimensions"][0]), int(t["dimensions"][1])
        payload = np.fromfile(_resolve(path, t["payload_path"]), np.uint8)
        if payload.size != int(t["payload_bytes"]) or checksum(payload) != int(t["payload_checksum"]):
            raise ValueError(f"{t['name']}: payload size or checksum does not match the manifest")
        if "metadata_path" in t:
            fmt = Q4K_POLICIES[t["policy"]][0]
            meta = np.fromfile(_resolve(path, t["metadata_path"]), np.uint8)
            if meta.size != int(t["metadata_bytes"]) or checksum(meta) != int(t["metadata_checksum"]):
                raise ValueError(f"{t['name']}: metadata size or checksum does not match the manifest")
        else:
            fmt = FORMAT_OF_TYPE[t["type"]]
            meta = None
            if int(t["block_type_size"]) != BLOCK_TYPE_SIZE[t["type"]]:
                raise ValueError(f"{t['name']}: block type size mismatch")
        if rows * cols // 256 * packs.payload_bytes_per_block(fmt) != payload.size:
            raise ValueError(f"{t['name']}: payload bytes do not match the dimensions")
        out[t["name"]] = packs.Pack(fmt, rows, cols, payload, meta)
    return out
