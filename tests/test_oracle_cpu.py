"""The CPU oracle pinned against the reference (no GPU).

Golden vectors in tests/golden were produced by the reference's own CPU functions and
packer (tests/golden/make_golden.py).  The C restatement in oracle/qoracle.c must
reproduce them bit for bit; when the reference tree is present the live reference
(oracle/_ref) is compared too.
"""

import struct
import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import FORMAT_TAGS, GOLDEN, REPO, load_golden
from qgemv_b200 import packs

from qoracle import REFERENCE_ROOT as REF_ROOT  # noqa: E402


def same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    """Bit equality, with every NaN equal to every NaN (the fp16 decode yields one)."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    nan = np.isnan(a) & np.isnan(b)
    return bool(np.array_equal(a.view(np.uint32)[~nan], b.view(np.uint32)[~nan]))


def meta_of(g):
    return g["meta"] if g["meta"].size else None


@pytest.mark.parametrize("fmt", list(FORMAT_TAGS))
@pytest.mark.parametrize("case", ["small", "edge"])
def test_port_dequant_bit_exact(port, fmt, case):
    g = load_golden(fmt, case)
    nblocks = int(g["rows"]) * int(g["cols"]) // 256
    out = port.dequant(fmt, g["payload"], meta_of(g), 0, nblocks)
    assert same_bits(out, g["dequant"])


@pytest.mark.parametrize("fmt", list(FORMAT_TAGS))
@pytest.mark.parametrize("case", ["small", "ragged", "edge"])
def test_port_matvec_token_kv_bit_exact(port, fmt, case):
    g = load_golden(fmt, case)
    rows, cols = int(g["rows"]), int(g["cols"])
    y = port.matvec(fmt, g["payload"], meta_of(g), g["x"], rows, cols)
    assert same_bits(y, g["logits"])
    kv = np.zeros_like(g["kv"])
    port.apply_kv(y, kv, int(g["token_in"]), int(g["page_words"]), int(g["active_pages"]))
    assert same_bits(kv, g["kv"])
    token = (port.argmax(y) + int(g["token_in"]) + 1) % 32000
    assert token == int(g["token_out"])


@pytest.mark.parametrize("fmt", sorted(packs.SPLIT_POLICY))
@pytest.mark.parametrize("case", ["small", "ragged", "edge"])
def test_split_packer_matches_reference_packer(fmt, case):
    g = load_golden(fmt, case)
    payload, meta = packs.split_q4k(g["raw"], fmt)
    assert np.array_equal(payload, g["payload"])
    assert np.array_equal(meta, g["meta"])


def test_q4k_known_answers(port):
    """runtime/tests/unit/test_q4k_resident_pack.py:31-73 known answers."""
    kat = np.load(GOLDEN / "golden_q4k_kat.npz")
    scales = bytes(kat["raw"][4:16])
    assert port.scale_min_k4(0, scales) == (1, 5)
    assert port.scale_min_k4(3, scales) == (4, 8)
    assert port.scale_min_k4(4, scales) == (0, 4)
    assert port.scale_min_k4(5, scales) == (0, 8)
    assert port.scale_min_k4(6, scales) == (0, 12)
    sc, mn = packs.scale_min_k4(kat["raw"][4:16].reshape(1, 12))
    assert (int(sc[0, 0]), int(mn[0, 0])) == (1, 5) and (int(sc[0, 6]), int(mn[0, 6])) == (0, 12)
    pay, meta = packs.split_q4k(kat["raw"], packs.Q4K_PREDECODED)
    assert struct.unpack("<ff", meta[:8].tobytes()) == (0.5, 1.25)
    assert pay[:4].tolist() == [0, 1, 2, 3] and pay[-1] == 127
    _, meta = packs.split_q4k(kat["raw"], packs.Q4K_COMPACT)
    assert meta[:4].tobytes() == kat["raw"][:4].tobytes()
    assert meta[4:8].tolist() == [1, 2, 3, 4] and meta[12:16].tolist() == [5, 6, 7, 8]
    _, meta = packs.split_q4k(kat["raw"], packs.Q4K_NATIVE)
    assert meta.tobytes() == kat["raw"][:16].tobytes()
    assert same_bits(port.dequant(packs.Q4K_RAW, kat["raw"], None, 0, 1), kat["dequant_raw"])
    for fmt in packs.SPLIT_POLICY:
        assert np.array_equal(kat[f"meta_{fmt}"], packs.split_q4k(kat["raw"], fmt)[1])
        out = port.dequant(fmt, kat[f"payload_{fmt}"], kat[f"meta_{fmt}"], 0, 1)
        assert same_bits(out, kat[f"dequant_{fmt}"])


def test_block_byte_sizes():
    """runtime/tests/unit/test_gguf_block_formats.py:19-24 byte counts."""
    assert packs.pack_bytes(packs.Q4K_RAW, 8192, 2048) == 9_437_184
    assert packs.pack_bytes(packs.Q5K, 248320, 2048) == 349_634_560
    assert packs.pack_bytes(packs.IQ2S, 512 * 256, 2048) == 85_983_232
    assert packs.pack_bytes(packs.IQ3S, 2048 * 256, 512) == 115_343_360


def test_feedback_port_matches_reference():
    import qoracle

    g = np.load(GOLDEN / "golden_feedback.npz")
    L = qoracle.Port().lib
    logits = g["logits"]
    lp = logits.ctypes.data
    for eps_tag, eps in (("e6", 1e-6), ("e5", 1e-5)):
        for kind in range(6):
            for acc in ((0, 1) if kind >= 4 else (0,)):
                key = f"k{kind}_{eps_tag}_a{acc}"
                act = g[f"{key}_act_in"].copy()
                cache = g[f"{key}_cache_in"].copy()
                ap, cp = act.ctypes.data, cache.ctypes.data
                n, cols, cc = logits.size, act.size, cache.size
                if kind == 0:
                    L.orc_rmsnorm_feedback(lp, ap, n, cols, eps)
                elif kind == 1:
                    L.orc_silu_rmsnorm_feedback(lp, ap, n, cols, eps)
                elif kind == 2:
                    cache = np.resize(cache, cols).astype(np.float32)  # reference grows the cache
                    cp = cache.ctypes.data
                    L.orc_rmsnorm_feedback_with_silu_cache(lp, ap, cp, n, cols, eps)
                elif kind == 3:
                    L.orc_gated_silu_rmsnorm_feedback(lp, cp, ap, n, cc, cols, eps)
                else:
                    L.orc_rmsnorm_cache(lp, cp, n, cc, eps, 1 if kind == 5 else 0, acc)
                np.testing.assert_allclose(act, g[f"{key}_act"], rtol=1e-6, atol=1e-6)
                if kind != 2:
                    np.testing.assert_allclose(cache, g[f"{key}_cache"], rtol=1e-6, atol=1e-6)
                else:
                    np.testing.assert_allclose(cache[: g[f"{key}_cache"].size][:cols],
                                               g[f"{key}_cache"][:cols], rtol=1e-6, atol=1e-6)


def test_gated_product_port_matches_reference():
    """rmsnorm_cache_and_gated_product (decode_kernels.cu:263-289): the C restatement
    against the reference's own CPU twin (golden vectors)."""
    import qoracle

    g = np.load(GOLDEN / "golden_feedback.npz")
    L = qoracle.Port().lib
    logits = g["logits"]
    for eps_tag, eps in (("e6", 1e-6), ("e5", 1e-5)):
        for acc in (0, 1):
            key = f"k6_{eps_tag}_a{acc}"
            gate, up, act = g[f"{key}_gate"], g[f"{key}_up_in"].copy(), g[f"{key}_act_in"].copy()
            L.orc_rmsnorm_cache_and_gated_product(logits.ctypes.data, gate.ctypes.data, up.ctypes.data,
                                                  act.ctypes.data, logits.size, up.size, act.size, eps, acc)
            assert same_bits(up, g[f"{key}_up"]) and same_bits(act, g[f"{key}_act"]), key


def test_planted_mistake_is_caught(port):
    """A corrupted payload byte must break bit-exactness and the logit tolerance."""
    g = load_golden(packs.Q4K_RAW, "small")
    bad = g["payload"].copy()
    bad[16 + 5] ^= 0xFF  # a quant byte of block 0, row 0
    y = port.matvec(packs.Q4K_RAW, bad, None, g["x"], int(g["rows"]), int(g["cols"]))
    assert not same_bits(y, g["logits"])
    l1 = port.row_l1(packs.Q4K_RAW, g["payload"], None, int(g["rows"]), int(g["cols"]))
    tol = 1e-3 * l1 * np.abs(g["x"]).max()
    assert np.abs(y - g["logits"])[0] > tol[0] * 1e-3


@pytest.mark.skipif(not (REF_ROOT / "runtime").is_dir(), reason="reference tree not present")
def test_iq_grid_header_matches_reference():
    sys.path.insert(0, str(REPO / "oracle"))
    import gen_iq_grids

    got = gen_iq_grids.parse_header(gen_iq_grids.DEFAULT_OUT)
    want = gen_iq_grids.load_reference_tables(REF_ROOT)
    assert got[0] == want[0] and got[1] == want[1]


@pytest.mark.skipif(not (REF_ROOT / "runtime").is_dir(), reason="reference tree not present")
@pytest.mark.parametrize("fmt", list(FORMAT_TAGS))
def test_port_matches_live_reference(port, fmt):
    import qoracle

    ref = qoracle.Ref.load()
    pk = packs.synthetic_pack(fmt, 19, 1280, seed=900 + fmt)
    x = packs.synthetic_activation(1280, 900 + fmt)
    a = port.matvec(fmt, pk.payload, pk.meta, x, 19, 1280)
    b = ref.matvec(fmt, pk.payload, pk.meta, x, 19, 1280)
    assert same_bits(a, b)
    assert same_bits(port.dequant(fmt, pk.payload, pk.meta, 3, 5), ref.dequant(fmt, pk.payload, pk.meta, 3, 5))


def test_codebook_properties_used_by_the_kernels():
    """The GEMV turns IQ3_S magnitudes g into g XOR 0x11 / g XOR 0x0F (= 15 +- g): every
    grid byte must be odd and <= 15; IQ2_S codes are 2-bit by construction."""
    sys.path.insert(0, str(REPO / "oracle"))
    import gen_iq_grids

    iq2s, iq3s = gen_iq_grids.parse_header(gen_iq_grids.DEFAULT_OUT)
    assert len(iq2s) == 1024 and all(0 <= v < 65536 for v in iq2s)
    for v in iq3s:
        for k in range(4):
            b = (v >> (8 * k)) & 0xFF
            assert b % 2 == 1 and b <= 15
