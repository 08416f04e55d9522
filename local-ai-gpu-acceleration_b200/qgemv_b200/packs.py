"""Resident packs: the byte layouts of the reference's packers and seeded synthetic packs.

Layouts (unchanged from the reference):
  * Q4_K raw blocks and the four Q4_K split packs -- payload = block[16:144] per block
    plus a metadata stream (tools/bench/q4k_resident_pack.py:82-145).
  * Q5_K / IQ2_S / IQ3_S raw GGUF blocks (tools/bench/iq_resident_pack.py:115-147,
    tools/bench/q5k_resident_pack.py).

`split_q4k` restates the packer's `build_metadata` / `extract_payload` with numpy
(tests pin it byte-for-byte against the reference packer).  `synthetic_pack`
draws the BASELINE distributions: every byte uniform, then fp16 d (and dmin for the
K-quants) uniform in [1e-3, 1e-2].
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

# Format ids: include/qgemv_b200.h qg_format.
Q4K_RAW, Q4K_PREDECODED, Q4K_HALF, Q4K_COMPACT, Q4K_NATIVE, Q5K, IQ2S, IQ3S = range(8)
FORMAT_NAMES = {
    Q4K_RAW: "Q4_K", Q4K_PREDECODED: "Q4_K/split-predecoded", Q4K_HALF: "Q4_K/split-half",
    Q4K_COMPACT: "Q4_K/split-compact", Q4K_NATIVE: "Q4_K/split-native", Q5K: "Q5_K",
    IQ2S: "IQ2_S", IQ3S: "IQ3_S",
}
SPLIT_POLICY = {
    Q4K_PREDECODED: "split-predecoded", Q4K_HALF: "split-half",
    Q4K_COMPACT: "split-compact", Q4K_NATIVE: "split-native",
}
RAW_BLOCK_BYTES = {Q4K_RAW: 144, Q5K: 176, IQ2S: 82, IQ3S: 110}
PAYLOAD_BYTES = {Q4K_RAW: 144, Q4K_PREDECODED: 128, Q4K_HALF: 128, Q4K_COMPACT: 128,
                 Q4K_NATIVE: 128, Q5K: 176, IQ2S: 82, IQ3S: 110}
META_BYTES = {Q4K_PREDECODED: 64, Q4K_HALF: 32, Q4K_COMPACT: 20, Q4K_NATIVE: 16}


def payload_bytes_per_block(fmt: int) -> int:
    return PAYLOAD_BYTES[fmt]


def meta_bytes_per_block(fmt: int) -> int:
    return META_BYTES.get(fmt, 0)


def pack_bytes(fmt: int, rows: int, cols: int) -> int:
    """Algorithmic weight bytes of a rows x cols pack (payload + metadata)."""
    blocks = rows * (cols // 256)
    return blocks * (payload_bytes_per_block(fmt) + meta_bytes_per_block(fmt))


def scale_min_k4(scales: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Vectorised get_scale_min_k4 (q4k_resident_pack.py:52-57): scales [n, 12] u8 ->
    (scale [n, 8], min [n, 8]) u8."""
    s = scales.astype(np.uint8)
    sc = np.empty((s.shape[0], 8), np.uint8)
    mn = np.empty((s.shape[0], 8), np.uint8)
    sc[:, :4] = s[:, 0:4] & 63
    mn[:, :4] = s[:, 4:8] & 63
    sc[:, 4:] = (s[:, 8:12] & 0x0F) | ((s[:, 0:4] >> 6) << 4)
    mn[:, 4:] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    return sc, mn


def split_q4k(raw: np.ndarray, fmt: int) -> tuple[np.ndarray, np.ndarray]:
    """Raw 144-B Q4_K blocks -> (payload, metadata) of split pack `fmt`
    (q4k_resident_pack.py:82-145)."""
    blocks = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1, 144)
    payload = np.ascontiguousarray(blocks[:, 16:144]).reshape(-1)
    if fmt == Q4K_NATIVE:
        return payload, np.ascontiguousarray(blocks[:, 0:16]).reshape(-1)
    sc, mn = scale_min_k4(blocks[:, 4:16])
    if fmt == Q4K_COMPACT:
        meta = np.concatenate([blocks[:, 0:4], sc, mn], axis=1)
        return payload, np.ascontiguousarray(meta).reshape(-1)
    d = blocks[:, 0:2].copy().view("<f2").astype(np.float64)
    dmin = blocks[:, 2:4].copy().view("<f2").astype(np.float64)
    prod = np.empty((blocks.shape[0], 8, 2), np.float64)
    prod[:, :, 0] = d * sc.astype(np.float64)
    prod[:, :, 1] = dmin * mn.astype(np.float64)
    if fmt == Q4K_PREDECODED:
        return payload, prod.astype("<f4").reshape(-1).view(np.uint8).copy()
    if fmt == Q4K_HALF:
        return payload, prod.astype("<f2").reshape(-1).view(np.uint8).copy()
    raise ValueError(f"not a Q4_K split format: {fmt}")


@dataclass
class Pack:
    fmt: int
    rows: int
    cols: int
    payload: np.ndarray          # uint8
    meta: np.ndarray | None      # uint8 or None

    @property
    def weight_bytes(self) -> int:
        return self.payload.nbytes + (0 if self.meta is None else self.meta.nbytes)


def synthetic_raw_blocks(fmt_raw: int, nblocks: int, rng: np.random.Generator) -> np.ndarray:
    """Uniform random bytes with fp16 d (and dmin for K-quants) ~ U[1e-3, 1e-2]."""
    bb = RAW_BLOCK_BYTES[fmt_raw]
    blocks = np.frombuffer(rng.bytes(nblocks * bb), np.uint8).reshape(nblocks, bb).copy()
    nscale = 2 if fmt_raw in (Q4K_RAW, Q5K) else 1
    vals = rng.uniform(1e-3, 1e-2, size=(nblocks, nscale)).astype(np.float16)
    blocks[:, 0 : 2 * nscale] = vals.view(np.uint8).reshape(nblocks, 2 * nscale)
    return blocks.reshape(-1)


def synthetic_pack(fmt: int, rows: int, cols: int, seed: int) -> Pack:
    if cols <= 0 or cols % 256 or rows <= 0:
        raise ValueError(f"bad shape {rows}x{cols}")
    rng = np.random.Generator(np.random.PCG64(seed))
    nblocks = rows * (cols // 256)
    if fmt in SPLIT_POLICY:
        raw = synthetic_raw_blocks(Q4K_RAW, nblocks, rng)
        payload, meta = split_q4k(raw, fmt)
        return Pack(fmt, rows, cols, payload, meta)
    return Pack(fmt, rows, cols, synthetic_raw_blocks(fmt, nblocks, rng), None)


def synthetic_activation(cols: int, seed: int, batch: int = 1) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed + 0x5EED))
    x = rng.standard_normal((batch, cols), dtype=np.float32)
    return x[0] if batch == 1 else x
