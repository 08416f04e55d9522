"""ctypes front end of the CPU checkers -- TEST INFRASTRUCTURE ONLY.

  * `Port`  -> oracle/_build/libqoracle.so: this project's C restatement
    (oracle/qoracle.c) of the reference's CPU decode path.
  * `Ref`   -> oracle/_ref/libref_oracle.so: the reference's own CPU functions
    (runtime/apps/mixed_sequence_benchmark_runner/main.cpp:1075-1500) compiled
    unmodified by oracle/Makefile.  Present only where the reference tree was
    available at build time (it is copied to GPU boxes as a prebuilt file).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs
use this module; the product path never does.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import c_double, c_float, c_int, c_uint32, c_uint64, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_LIB = HERE / "_build" / "libqoracle.so"
REF_LIB = HERE / "_ref" / "libref_oracle.so"
# The reference tree: QG_REFERENCE_ROOT, else a checkout named "reference" beside this
# repository (absent on machines that only run the prebuilt files).
REFERENCE_ROOT = Path(os.environ.get("QG_REFERENCE_ROOT", str(HERE.parent.parent / "reference")))


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(c_void_p)


def build_port() -> Path:
    if not PORT_LIB.exists() or PORT_LIB.stat().st_mtime < (HERE / "qoracle.c").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)
    return PORT_LIB


def build_ref() -> Path | None:
    """Build oracle/_ref from the reference tree when it is present."""
    if REF_LIB.exists():
        return REF_LIB
    if not (REFERENCE_ROOT / "runtime").is_dir():
        return None
    subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF={REFERENCE_ROOT}"], check=True)
    return REF_LIB if REF_LIB.exists() else None


class Port:
    def __init__(self) -> None:
        self.lib = ctypes.CDLL(str(build_port()))
        L = self.lib
        L.orc_fp16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_fp16_to_f32.restype = c_float
        L.orc_dequant_blocks.argtypes = [c_int, c_void_p, c_void_p, c_uint64, c_uint64, c_void_p]
        L.orc_matvec_rows.argtypes = [c_int, c_void_p, c_void_p, c_void_p, c_uint32, c_uint32, c_uint32, c_void_p]
        L.orc_matvec.argtypes = [c_int, c_void_p, c_void_p, c_void_p, c_uint32, c_uint32, c_void_p]
        L.orc_row_l1.argtypes = [c_int, c_void_p, c_void_p, c_uint32, c_uint32, c_void_p]
        L.orc_argmax.argtypes = [c_void_p, c_uint32]
        L.orc_argmax.restype = c_uint32
        L.orc_apply_kv.argtypes = [c_void_p, c_uint32, c_void_p, c_uint64, c_uint32, c_uint32, c_uint32]
        L.orc_output_token_sample.argtypes = [c_void_p, c_uint32, c_uint32, c_uint32]
        L.orc_output_token_sample.restype = c_uint32
        L.orc_scale_min_k4.argtypes = [c_int, c_void_p, c_void_p, c_void_p]
        for name in ("orc_rmsnorm_feedback", "orc_silu_rmsnorm_feedback"):
            getattr(L, name).argtypes = [c_void_p, c_void_p, c_uint32, c_uint32, c_float]
        L.orc_rmsnorm_feedback_with_silu_cache.argtypes = [c_void_p, c_void_p, c_void_p, c_uint32, c_uint32, c_float]
        L.orc_gated_silu_rmsnorm_feedback.argtypes = [c_void_p, c_void_p, c_void_p, c_uint32, c_uint32, c_uint32, c_float]
        L.orc_rmsnorm_cache.argtypes = [c_void_p, c_void_p, c_uint32, c_uint32, c_float, c_int, c_int]
        L.orc_rmsnorm_cache_and_gated_product.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_uint32, c_uint32, c_uint32, c_float, c_int]
        L.orc_weighted_rmsnorm.argtypes = [c_void_p, c_void_p, c_uint32, c_float, c_void_p]
        L.orc_silu_gate.argtypes = [c_void_p, c_void_p, c_uint32, c_void_p]
        L.orc_residual_add.argtypes = [c_void_p, c_void_p, c_uint32, c_void_p]

    def dequant(self, fmt, payload, meta, first_block, count) -> np.ndarray:
        out = np.empty(count * 256, np.float32)
        self.lib.orc_dequant_blocks(fmt, _p(payload), _p(meta), first_block, count, _p(out))
        return out

    def matvec(self, fmt, payload, meta, x, rows, cols, row_begin=0, row_end=None) -> np.ndarray:
        row_end = rows if row_end is None else row_end
        y = np.empty(row_end - row_begin, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        self.lib.orc_matvec_rows(fmt, _p(payload), _p(meta), _p(x), cols, row_begin, row_end, _p(y))
        return y

    def row_l1(self, fmt, payload, meta, rows, cols) -> np.ndarray:
        out = np.empty(rows, np.float32)
        self.lib.orc_row_l1(fmt, _p(payload), _p(meta), rows, cols, _p(out))
        return out

    def argmax(self, v: np.ndarray) -> int:
        v = np.ascontiguousarray(v, np.float32)
        return int(self.lib.orc_argmax(_p(v), v.size))

    def apply_kv(self, logits, kv, token, page_words, active_pages) -> None:
        logits = np.ascontiguousarray(logits, np.float32)
        self.lib.orc_apply_kv(_p(logits), logits.size, _p(kv), kv.size, token, page_words, active_pages)

    def scale_min_k4(self, index: int, packed: bytes) -> tuple[int, int]:
        buf = np.frombuffer(bytes(packed), np.uint8).copy()
        sc = np.zeros(1, np.uint8)
        mn = np.zeros(1, np.uint8)
        self.lib.orc_scale_min_k4(index, _p(buf), _p(sc), _p(mn))
        return int(sc[0]), int(mn[0])


class Ref:
    """The reference's own CPU functions (None-safe constructor: use Ref.load())."""

    def __init__(self, path: Path) -> None:
        self.lib = ctypes.CDLL(str(path))
        L = self.lib
        L.ref_stage_logits.argtypes = [c_int, c_void_p, c_void_p, c_void_p, c_uint32, c_uint32, c_uint32, c_void_p]
        L.ref_stage_logits.restype = c_int
        L.ref_dequant_blocks.argtypes = [c_int, c_void_p, c_void_p, c_uint64, c_uint64, c_void_p]
        L.ref_dequant_blocks.restype = c_int
        L.ref_argmax.argtypes = [c_void_p, c_uint32]
        L.ref_argmax.restype = c_uint32
        L.ref_apply_kv.argtypes = [c_void_p, c_uint32, c_void_p, c_uint64, c_uint32, c_uint32, c_uint32]
        L.ref_feedback.argtypes = [c_int, c_void_p, c_uint32, c_void_p, c_uint32, c_void_p, c_uint32, c_float, c_int]
        L.ref_cache_gated_product.argtypes = [c_void_p, c_uint32, c_void_p, c_uint32, c_void_p, c_uint32,
                                              c_void_p, c_uint32, c_float, c_int]
        L.ref_time_stage_logits.argtypes = [c_int, c_void_p, c_void_p, c_void_p, c_uint32, c_uint32, c_uint32, c_void_p]
        L.ref_time_stage_logits.restype = c_double

    @staticmethod
    def load(build: bool = True) -> "Ref | None":
        path = build_ref() if build else (REF_LIB if REF_LIB.exists() else None)
        return Ref(path) if path is not None else None

    def matvec(self, fmt, payload, meta, x, rows, cols, row_begin=0, row_end=None) -> np.ndarray:
        row_end = rows if row_end is None else row_end
        y = np.empty(row_end - row_begin, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        rc = self.lib.ref_stage_logits(fmt, _p(payload), _p(meta), _p(x), cols, row_begin, row_end, _p(y))
        if rc != 0:
            raise ValueError("ref_stage_logits rejected the arguments")
        return y

    def dequant(self, fmt, payload, meta, first_block, count) -> np.ndarray:
        out = np.empty(count * 256, np.float32)
        if self.lib.ref_dequant_blocks(fmt, _p(payload), _p(meta), first_block, count, _p(out)) != 0:
            raise ValueError("bad format")
        return out

    def argmax(self, v: np.ndarray) -> int:
        v = np.ascontiguousarray(v, np.float32)
        return int(self.lib.ref_argmax(_p(v), v.size))

    def apply_kv(self, logits, kv, token, page_words, active_pages) -> None:
        logits = np.ascontiguousarray(logits, np.float32)
        self.lib.ref_apply_kv(_p(logits), logits.size, _p(kv), kv.size, token, page_words, active_pages)

    def feedback(self, kind, logits, act, cache, eps, accumulate=0) -> None:
        logits = np.ascontiguousarray(logits, np.float32)
        self.lib.ref_feedback(kind, _p(logits), logits.size, _p(act), act.size,
                              _p(cache), 0 if cache is None else cache.size, eps, accumulate)

    def cache_gated_product(self, logits, gate, up, act, eps, accumulate) -> None:
        logits = np.ascontiguousarray(logits, np.float32)
        self.lib.ref_cache_gated_product(_p(logits), logits.size, _p(gate), gate.size, _p(up), up.size,
                                         _p(act), act.size, eps, accumulate)

    def time_matvec(self, fmt, payload, meta, x, rows, cols, threads) -> tuple[float, np.ndarray]:
        y = np.empty(rows, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        t = self.lib.ref_time_stage_logits(fmt, _p(payload), _p(meta), _p(x), rows, cols, threads, _p(y))
        if t < 0:
            raise ValueError("bad arguments")
        return float(t), y
