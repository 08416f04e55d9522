"""GGUF ingest: the library's reader (csrc/qg_gguf.cu) on files written from the public
GGUF layout (qgemv_b200/gguf.py write_gguf), checked against the reference's own probe
(runtime/apps/gguf_probe, built unmodified by local-ai-gpu-acceleration_b200/link/Makefile)
where it is built; the ingested tensors as resident packs in the reference's manifest
format; on the GPU, the kernels on ingested tensors against the oracle."""

import json
import subprocess

import numpy as np
import pytest

from conftest import REPO
from qgemv_b200 import gguf, manifest, packs

PROBE = REPO / "local-ai-gpu-acceleration_b200" / "link" / "_build" / "gguf_probe"

FILE_NOT_FOUND, INVALID_VALUE, INVALID_SYMBOL = 301, 1, 13


def _model(tmp_path, alignment=32):
    """A small llama-style file: one layer of each decode-path format, an F32 norm, an
    F16 tensor and a tensor of a type outside the probe's table (Q4_1 = 3)."""
    spec = [("blk.0.attn_q.weight", packs.IQ3S, 256, 512), ("blk.0.attn_k.weight", packs.IQ3S, 128, 512),
            ("blk.0.ffn_gate.weight", packs.IQ2S, 384, 512), ("blk.0.ffn_down.weight", packs.Q5K, 512, 768),
            ("output.weight", packs.Q4K_RAW, 320, 512)]
    tensors, pks = [], {}
    for i, (name, fmt, rows, cols) in enumerate(spec):
        pk = packs.synthetic_pack(fmt, rows, cols, seed=40 + i)
        pks[name] = pk
        tensors.append((name, gguf.GGML_OF_FORMAT[fmt], [cols, rows], pk.payload.tobytes()))
    norm = np.linspace(0.5, 1.5, 512).astype(np.float32)
    tensors.insert(2, ("blk.0.attn_norm.weight", 0, [512], norm.tobytes()))
    tensors.append(("token_embd.weight", 1, [512, 3], np.ones(1536, np.float16).tobytes()))
    tensors.append(("blk.0.odd.weight", 3, [64], bytes(40)))
    meta = {"general.name": "synthetic", "llama.block_count": 1, "llama.rope.freq_base": 500000.0,
            "tokenizer.ggml.tokens": ["a", "bb", "ccc"], "llama.attention.head_count": 4,
            "general.alignment": alignment}
    path = gguf.write_gguf(tmp_path / "m.gguf", tensors, meta, alignment=alignment)
    return path, pks, norm


@pytest.mark.parametrize("alignment", [32, 64])
def test_reader_table_and_bytes(tmp_path, alignment):
    path, pks, norm = _model(tmp_path, alignment)
    with gguf.GGUFFile(path) as g:
        info = g.info
        assert info["version"] == 3 and info["tensor_count"] == 8 and info["metadata_count"] == 7
        assert info["tensor_data_alignment"] == alignment and info["architecture"] == "llama"
        assert info["tensor_data_offset"] % alignment == 0
        assert info["tensor_data_offset"] >= info["tensor_info_end_offset"]
        # 7 tensors of supported types (the Q4_1 one is not in the table), all valid
        assert info["supported_tensors"] == 7 and info["valid_tensors"] == 7
        for name, pk in pks.items():
            t = g.tensors[name]
            assert t.valid and t.data_bytes == pk.payload.size
            assert t.span_bytes - t.data_bytes < alignment
            assert t.absolute_offset == info["tensor_data_offset"] + t.offset
            got = g.pack(name)
            assert (got.fmt, got.rows, got.cols) == (pk.fmt, pk.rows, pk.cols)
            assert np.array_equal(got.payload, pk.payload)
        assert np.array_equal(g.read("blk.0.attn_norm.weight").view(np.float32), norm)
        assert not g.tensors["blk.0.odd.weight"].valid


def test_reader_matches_reference_probe(tmp_path):
    if not PROBE.exists():
        pytest.skip("reference gguf_probe not built (needs the reference tree)")
    path, _, _ = _model(tmp_path)
    res = subprocess.run([str(PROBE), "--model", str(path)], capture_output=True, text=True)
    assert res.returncode == 2, res.stderr  # the probe's exit code when a tensor is invalid (Q4_1)
    ref = json.loads(res.stdout)
    assert ref["invalid_tensors"] == 1
    with gguf.GGUFFile(path) as g:
        for key in ("version", "tensor_count", "metadata_count", "tensor_info_end_offset",
                    "tensor_data_offset", "tensor_data_alignment", "supported_tensors",
                    "valid_tensors", "expected_data_bytes", "architecture"):
            assert g.info[key] == ref[key], key
        # the probe's Q4_K smoke reads the first block of the first Q4_K tensor
        t = g.tensors[ref["q4k_smoke"]["tensor_name"]]
        assert ref["q4k_smoke"]["absolute_offset"] == t.absolute_offset
        blk = g.read(t.name)[:144]
        assert ref["q4k_smoke"]["scale_checksum"] == int(blk[4:16].sum())
        assert ref["q4k_smoke"]["packed_q4_checksum"] == int(blk[16:144].sum())


def test_reader_errors(tmp_path):
    import ctypes

    import qgemv_b200

    h = ctypes.c_void_p()
    assert qgemv_b200.call("qg_gguf_open", str(tmp_path / "missing.gguf").encode(), ctypes.byref(h)) == FILE_NOT_FOUND
    (tmp_path / "not.gguf").write_bytes(b"GGML" + bytes(60))
    assert qgemv_b200.call("qg_gguf_open", str(tmp_path / "not.gguf").encode(), ctypes.byref(h)) == INVALID_VALUE
    path, _, _ = _model(tmp_path)
    data = path.read_bytes()
    (tmp_path / "cut.gguf").write_bytes(data[:200])  # inside the metadata
    assert qgemv_b200.call("qg_gguf_open", str(tmp_path / "cut.gguf").encode(), ctypes.byref(h)) == INVALID_VALUE
    with gguf.GGUFFile(path) as g:
        idx = ctypes.c_uint64()
        assert qgemv_b200.call("qg_gguf_find", g.handle, b"no.such.tensor", ctypes.byref(idx)) == INVALID_SYMBOL
        buf = np.empty(10, np.uint8)
        t = g.tensors["output.weight"]
        assert qgemv_b200.call("qg_gguf_read", g.handle, t.index, buf.ctypes.data, 10) == INVALID_VALUE


def test_ingest_writes_reference_manifests(tmp_path):
    path, pks, _ = _model(tmp_path)
    out = gguf.ingest(path, tmp_path / "packs", q4k_policy="split-predecoded")
    assert set(out) == {"q4k", "iq", "q5k"}
    loaded = {}
    for m in out.values():
        loaded.update(manifest.read_manifest(m))
    with gguf.GGUFFile(path) as g:
        for name, pk in pks.items():
            got = loaded[name]
            if pk.fmt == packs.Q4K_RAW:
                payload, meta = packs.split_q4k(pk.payload, packs.Q4K_PREDECODED)
                assert got.fmt == packs.Q4K_PREDECODED
                assert np.array_equal(got.payload, payload) and np.array_equal(got.meta, meta)
            else:
                assert got.fmt == pk.fmt and np.array_equal(got.payload, pk.payload)
            rows = json.loads(next(m for m in out.values() if name in m.read_text()).read_text())["tensors"]
            row = next(r for r in rows if r["name"] == name)
            assert row["source_offset"] == g.tensors[name].absolute_offset


@pytest.mark.gpu
def test_ingested_tensors_on_the_gpu(tmp_path, cuda, port):
    import torch

    from test_gpu_parity import assert_rows_close, dev, row_tol
    from qgemv_b200 import ops

    path, _, _ = _model(tmp_path)
    out = gguf.ingest(path, tmp_path / "packs", q4k_policy="split-compact")
    for m in out.values():
        for name, pk in manifest.read_manifest(m).items():
            x = packs.synthetic_activation(pk.cols, 7)
            y = ops.gemv(pk.fmt, dev(pk.payload, cuda), dev(pk.meta, cuda), dev(x, cuda), pk.rows, pk.cols)
            want = port.matvec(pk.fmt, pk.payload, pk.meta, x, pk.rows, pk.cols)
            assert_rows_close(y.cpu().numpy(), want, row_tol(port, pk.fmt, pk.payload, pk.meta, x, pk.rows, pk.cols))
    torch.cuda.synchronize()
