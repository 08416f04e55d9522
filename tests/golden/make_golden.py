"""Generate tests/golden/*.npz from the reference's own code.

Run where the reference tree is present (its root as the argument, else the default
root that oracle/qoracle.py uses):

    python tests/golden/make_golden.py [reference_root]

Sources of truth (all the reference's own, compiled or imported unmodified):
  * oracle/_ref/libref_oracle.so -- runtime/apps/mixed_sequence_benchmark_runner/
    main.cpp:1075-1500 (dequant, reference_stage_logits, argmax_token,
    apply_reference_kv, the feedback math), built by oracle/Makefile;
  * tools/bench/q4k_resident_pack.py -- build_metadata / extract_payload for the
    Q4_K split packs (imported from the reference tree).

Inputs are seeded synthetic blocks with the BASELINE distributions plus a handful
of hand-built edge blocks (zero, negative, subnormal and largest-finite fp16 d).
The GPU box has no reference tree: tests read only the committed .npz files.
"""

from __future__ import annotations

import struct
import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO / "local-ai-gpu-acceleration_b200"))
sys.path.insert(0, str(REPO / "oracle"))

from qgemv_b200 import packs  # noqa: E402
import qoracle  # noqa: E402

OUT = Path(__file__).resolve().parent


def ref_split(raw: np.ndarray, fmt: int, ref_root: Path) -> tuple[np.ndarray, np.ndarray]:
    sys.path.insert(0, str(ref_root))
    from tools.bench.q4k_resident_pack import build_metadata, extract_payload  # noqa: E402

    blocks = raw.tobytes()
    payload = np.frombuffer(extract_payload(blocks), np.uint8).copy()
    meta = np.frombuffer(build_metadata(blocks, packs.SPLIT_POLICY[fmt]), np.uint8).copy()
    return payload, meta


def edge_blocks(fmt_raw: int, fp16_products: bool = False) -> np.ndarray:
    """Six blocks with unusual fp16 scale words, random bodies (fixed seed).  With
    fp16_products the largest words are reduced so d*scale still fits an fp16 (the
    reference packer raises OverflowError otherwise, q4k_resident_pack.py:48-49)."""
    rng = np.random.Generator(np.random.PCG64(4242 + fmt_raw))
    bb = packs.RAW_BLOCK_BYTES[fmt_raw]
    blocks = np.frombuffer(rng.bytes(6 * bb), np.uint8).reshape(6, bb).copy()
    d_words = [0x0000, 0x8000, 0x0001, 0x03FF, 0x7BFF, 0xBC00]  # +0, -0, min subnormal, max subnormal, max finite, -1
    dmin_words = [0x3C00, 0x0000, 0x8001, 0x2E66, 0x0400, 0xFBFF]
    if fp16_products:
        d_words[4], dmin_words[5] = 0x57FF, 0xD7FF  # +-127.9
    for i in range(6):
        blocks[i, 0:2] = np.frombuffer(struct.pack("<H", d_words[i]), np.uint8)
        if fmt_raw in (packs.Q4K_RAW, packs.Q5K):
            blocks[i, 2:4] = np.frombuffer(struct.pack("<H", dmin_words[i]), np.uint8)
    return blocks.reshape(-1)


def sample_q4k_block() -> np.ndarray:
    """The known-answer block of runtime/tests/unit/test_q4k_resident_pack.py:20-27."""
    block = bytearray(144)
    block[0:2] = struct.pack("<e", 0.5)
    block[2:4] = struct.pack("<e", 0.25)
    block[4:16] = bytes([1, 2, 3, 4, 5, 6, 7, 8, 0x40, 0x80, 0xC0, 0x00])
    for i in range(128):
        block[16 + i] = i & 0xFF
    return np.frombuffer(bytes(block), np.uint8).copy()


def make_case(ref: qoracle.Ref, ref_root: Path, fmt: int, rows: int, cols: int, seed: int,
              raw: np.ndarray | None = None, dump_dequant: bool = True) -> dict:
    nblocks = rows * cols // 256
    base = packs.Q4K_RAW if fmt in packs.SPLIT_POLICY else fmt
    if raw is None:
        rng = np.random.Generator(np.random.PCG64(seed))
        raw = packs.synthetic_raw_blocks(base, nblocks, rng)
    if fmt in packs.SPLIT_POLICY:
        payload, meta = ref_split(raw, fmt, ref_root)
    else:
        payload, meta = raw, np.zeros(0, np.uint8)
    x = packs.synthetic_activation(cols, seed)
    m = meta if meta.size else None
    case = {"fmt": np.int32(fmt), "rows": np.int32(rows), "cols": np.int32(cols),
            "raw": raw, "payload": payload, "meta": meta, "x": x}
    if dump_dequant:
        case["dequant"] = ref.dequant(fmt, payload, m, 0, nblocks)
    logits = ref.matvec(fmt, payload, m, x, rows, cols)
    case["logits"] = logits
    token_in = np.uint32(seed * 7919 % 32000)
    kv = np.zeros(rows * 4 + 3, np.float32)
    page_words, active = 4, max(1, rows - 2)
    ref.apply_kv(logits, kv, int(token_in), page_words, active)
    case.update(token_in=token_in, kv=kv, page_words=np.uint32(page_words),
                active_pages=np.uint32(active),
                token_out=np.uint32((ref.argmax(logits) + int(token_in) + 1) % 32000))
    return case


def main(argv: list[str]) -> int:
    ref_root = Path(argv[1]) if len(argv) > 1 else qoracle.REFERENCE_ROOT
    ref = qoracle.Ref.load()
    if ref is None:
        print("reference tree not found; cannot regenerate golden vectors")
        return 2
    for fmt, name in packs.FORMAT_NAMES.items():
        tag = name.replace("/", "_").replace("-", "_").lower()
        small = make_case(ref, ref_root, fmt, rows=8, cols=512, seed=100 + fmt)
        ragged = make_case(ref, ref_root, fmt, rows=37, cols=1024, seed=200 + fmt, dump_dequant=False)
        base = packs.Q4K_RAW if fmt in packs.SPLIT_POLICY else fmt
        edge = make_case(ref, ref_root, fmt, rows=2, cols=768, seed=300 + fmt, raw=edge_blocks(base, fmt == packs.Q4K_HALF))
        arrays = {}
        for prefix, case in (("small", small), ("ragged", ragged), ("edge", edge)):
            arrays.update({f"{prefix}_{k}": v for k, v in case.items()})
        np.savez_compressed(OUT / f"golden_{tag}.npz", **arrays)
        print(f"golden_{tag}.npz")

    # Q4_K packer known answers + the reference's decode of that block.
    kat = sample_q4k_block()
    arrays = {"raw": kat, "dequant_raw": ref.dequant(packs.Q4K_RAW, kat, None, 0, 1)}
    for fmt in packs.SPLIT_POLICY:
        payload, meta = ref_split(kat, fmt, ref_root)
        arrays[f"payload_{fmt}"] = payload
        arrays[f"meta_{fmt}"] = meta
        arrays[f"dequant_{fmt}"] = ref.dequant(fmt, payload, meta, 0, 1)
    np.savez_compressed(OUT / "golden_q4k_kat.npz", **arrays)

    # Feedback math (rmsnorm / silu / caches), eps of the mixed runner and of config 3.
    rng = np.random.Generator(np.random.PCG64(777))
    logits = (rng.standard_normal(37) * 3).astype(np.float32)
    arrays = {"logits": logits}
    for eps in (1e-6, 1e-5):
        for kind in range(6):
            act = (rng.standard_normal(96)).astype(np.float32)
            cache = (rng.standard_normal(64)).astype(np.float32)
            for acc in ((0, 1) if kind >= 4 else (0,)):
                a2, c2 = act.copy(), cache.copy()
                ref.feedback(kind, logits, a2, c2, eps, acc)
                key = f"k{kind}_e{int(round(-np.log10(eps)))}_a{acc}"
                arrays.update({f"{key}_act_in": act, f"{key}_cache_in": cache,
                               f"{key}_act": a2, f"{key}_cache": c2})
    # rmsnorm_cache_and_gated_product: the up cache takes the normalised logits (overwritten
    # or accumulated), the activation is gate x up (decode_kernels.cu:263-289 as the mixed
    # runner's CPU reference applies it).
    for eps in (1e-6, 1e-5):
        for acc in (0, 1):
            gate = rng.standard_normal(96).astype(np.float32)
            up = rng.standard_normal(96).astype(np.float32)
            act = rng.standard_normal(96).astype(np.float32)
            u2, a2 = up.copy(), act.copy()
            ref.cache_gated_product(logits, gate, u2, a2, eps, acc)
            key = f"k6_e{int(round(-np.log10(eps)))}_a{acc}"
            arrays.update({f"{key}_gate": gate, f"{key}_up_in": up, f"{key}_act_in": act,
                           f"{key}_up": u2, f"{key}_act": a2})
    np.savez_compressed(OUT / "golden_feedback.npz", **arrays)
    print("done")
    return 0


if __name__ == "__main__":
    raise SystemExit(main(sys.argv))
