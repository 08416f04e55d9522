"""ctypes binding of libqgemv_b200.so (include/qgemv_b200.h).

The library is the product; this module only declares its C signatures so Python
tests and bench.py can call the same entry points a C/C++ caller links against.
Loading never falls back to anything: if the shared library is missing and cannot
be built, `lib()` raises.
"""

from __future__ import annotations

import ctypes
import os
import re
from ctypes import c_float, c_int, c_uint32, c_uint64, c_void_p
from pathlib import Path

from . import build as _build

HEADER = Path(__file__).resolve().parents[2] / "include" / "qgemv_b200.h"

P = c_void_p
U32 = c_uint32
U64 = c_uint64
ERR = c_int  # cudaError_t

_COMPAT_DECODE = [P, P, P, P, P, U32, U32, U32, U32, U32, P]          # Q4_K raw launchers
_COMPAT_SPLIT = [P, P, P, P, P, P, U32, U32, U32, U32, U32, P]        # Q4_K split / predecoded
_COMPAT_PROBE = [P, P, P, P, P, U32, U32, U32, U32, U32, U32, P]      # IQ / Q5_K decode probes

SIGNATURES: dict[str, list] = {
    "rtxllm_launch_q4k_matvec_decode": _COMPAT_DECODE,
    "rtxllm_launch_q4k_matvec_decode_shared": _COMPAT_DECODE,
    "rtxllm_launch_q4k_matvec_decode_warp": _COMPAT_DECODE,
    "rtxllm_launch_q4k_matvec_decode_warp_broadcast": _COMPAT_DECODE,
    "rtxllm_launch_q4k_matvec_decode_warp_broadcast_vec4": _COMPAT_DECODE,
    "rtxllm_launch_q4k_matvec_decode_warp_broadcast_vec4x2": _COMPAT_DECODE,
    "rtxllm_launch_q4k_matvec_decode_warp_broadcast_vec4x4": _COMPAT_DECODE,
    "rtxllm_launch_q4k_matvec_decode_predecoded_vec4x4": _COMPAT_SPLIT,
    "rtxllm_launch_q4k_matvec_decode_split_predecoded_vec4x4": _COMPAT_SPLIT,
    "rtxllm_launch_q4k_matvec_decode_split_half_vec4x4": _COMPAT_SPLIT,
    "rtxllm_launch_q4k_matvec_decode_split_compact_vec4x4": _COMPAT_SPLIT,
    "rtxllm_launch_q4k_matvec_decode_split_native_vec4x4": _COMPAT_SPLIT,
    "rtxllm_launch_q5k_matvec_decode_probe": _COMPAT_PROBE,
    "rtxllm_launch_iq2s_matvec_probe": [P, P, P, U32, U32, U32, P],
    "rtxllm_launch_iq2s_matvec_decode_probe": _COMPAT_PROBE,
    "rtxllm_launch_iq3s_matvec_decode_probe": _COMPAT_PROBE,
    "rtxllm_launch_output_token_sample": [P, P, U32, U32, U32, P],
    "rtxllm_launch_rmsnorm_feedback": [P, P, U32, U32, c_float, P],
    "rtxllm_launch_silu_rmsnorm_feedback": [P, P, U32, U32, c_float, P],
    "rtxllm_launch_rmsnorm_feedback_with_silu_cache": [P, P, P, U32, U32, c_float, P],
    "rtxllm_launch_gated_silu_rmsnorm_feedback": [P, P, P, U32, U32, U32, c_float, P],
    "rtxllm_launch_rmsnorm_silu_cache": [P, P, U32, U32, c_float, U32, P],
    "rtxllm_launch_rmsnorm_cache": [P, P, U32, U32, c_float, U32, P],
    "rtxllm_launch_rmsnorm_cache_and_gated_product": [P, P, P, P, U32, U32, U32, c_float, U32, P],
    "qg_gemv": [c_int, P, P, P, P, U32, U32, P],
    "qg_act_bytes": [U32, P],
    "qg_act_prepare": [P, U32, P, P],
    "qg_gemv_act": [c_int, P, P, P, P, P, U32, U32, P],
    "qg_decode_stage": [c_int, P, P, P, P, P, P, U32, U32, U32, U32, U32, P],
    "qg_gemv_batched": [c_int, P, P, P, P, U32, U32, U32, P],
    "qg_dequantize": [c_int, P, P, U64, U64, P, P],
    "qg_argmax_token": [P, U32, P, U32, U32, U32, P],
    "qg_get_error": [P],
    "qg_gemv_plan": [c_int, U32, U32, P, P, P, P],
    "qg_gemv_plan_sms": [c_int, U32, U32, U32, P, P, P, P],
    "qg_layer_slice_workspace_bytes": [P, P],
    "qg_layer_slice_buffers": [P, P, P],
    "qg_gemm_batched_workspace_bytes": [c_int, U32, U32, U32, P],
    "qg_gemm_batched": [c_int, P, P, P, P, U32, U32, U32, P, P],
    "qg_layer_slice_forward": [P, P, P, P, P],
    "qg_layer_slice_forward_static": [P, P, P, P],
    "qg_layer_slice_batched_workspace_bytes": [P, U32, P],
    "qg_layer_slice_forward_batched": [P, P, P, U32, P, P],
    "qg_layer_slice_batched_buffers": [P, U32, P, P],
    "qg_slice_buckets_create": [P, P, U32, P, P],
    "qg_slice_buckets_bucket": [P, U32, P],
    "qg_slice_buckets_run": [P, P, P, U32, P],
    "qg_slice_buckets_destroy": [P],
    "qg_graph_begin": [P],
    "qg_graph_end": [P, P],
    "qg_graph_launch": [P, P],
    "qg_graph_destroy": [P],
    "qg_nccl_unique_id": [P],
    "qg_decoder_workspace_bytes": [P, P],
    "qg_decoder_shard": [P, P, P, P, P, P],
    "qg_decoder_create": [P, P, P, P, P, P, P, P],
    "qg_decoder_exchange_bytes": [P, P],
    "qg_decoder_create_in": [P, P, P, P, P, P, P, P, P],
    "qg_decoder_step": [P, P, U32, P, P],
    "qg_decoder_step_at": [P, P, P, U32, U32, P, P],
    "qg_decoder_views": [P, P, P],
    "qg_decoder_stage_buffers": [P, P],
    "qg_decoder_destroy": [P],
    "qg_gguf_open": [ctypes.c_char_p, P],
    "qg_gguf_summary": [P, P],
    "qg_gguf_tensor": [P, U64, P],
    "qg_gguf_find": [P, ctypes.c_char_p, P],
    "qg_gguf_read": [P, U64, P, U64],
    "qg_gguf_close": [P],
}

_LIB: ctypes.CDLL | None = None


class CudaError(RuntimeError):
    def __init__(self, fn: str, code: int):
        super().__init__(f"{fn} returned cudaError_t {code}")
        self.code = code


def header_functions(header: Path = HEADER) -> list[str]:
    """Every function name the public header declares."""
    text = header.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\bcudaError_t\s+(\w+)\s*\(", text)))


def lib() -> ctypes.CDLL:
    """The library: the in-tree build (rebuilt when a source is newer), or the build
    named by QG_LIBRARY (another build of the same sources, e.g. with different tuning
    macros, for side-by-side measurements)."""
    global _LIB
    if _LIB is None:
        override = os.environ.get("QG_LIBRARY")
        path = Path(override) if override else _build.build()
        handle = ctypes.CDLL(str(path))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = argtypes
            fn.restype = ERR
        _LIB = handle
    return _LIB


def call(name: str, *args) -> int:
    """Call an entry point and return its cudaError_t (0 = success)."""
    return int(getattr(lib(), name)(*args))


def check(name: str, *args) -> None:
    code = call(name, *args)
    if code != 0:
        raise CudaError(name, code)
