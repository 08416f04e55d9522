"""The C-ABI library builds for sm_100a, loads, and exports the header's entry points
(no GPU: only host-side argument validation is exercised)."""

import ctypes

import pytest

import qgemv_b200
from qgemv_b200 import _lib

INVALID_VALUE = 1           # cudaErrorInvalidValue
INVALID_CONFIGURATION = 9   # cudaErrorInvalidConfiguration


def test_library_exports_every_header_symbol():
    lib = qgemv_b200.lib()
    names = qgemv_b200.header_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert missing == []
    # every exported name has a declared ctypes signature
    assert set(names) <= set(_lib.SIGNATURES)


def test_reference_launcher_names_are_all_present():
    """The hot launchers of runtime/kernels/decode/decode_kernels.h:345-583."""
    want = [
        "rtxllm_launch_q4k_matvec_decode", "rtxllm_launch_q4k_matvec_decode_shared",
        "rtxllm_launch_q4k_matvec_decode_warp", "rtxllm_launch_q4k_matvec_decode_warp_broadcast",
        "rtxllm_launch_q4k_matvec_decode_warp_broadcast_vec4",
        "rtxllm_launch_q4k_matvec_decode_warp_broadcast_vec4x2",
        "rtxllm_launch_q4k_matvec_decode_warp_broadcast_vec4x4",
        "rtxllm_launch_q4k_matvec_decode_predecoded_vec4x4",
        "rtxllm_launch_q4k_matvec_decode_split_predecoded_vec4x4",
        "rtxllm_launch_q4k_matvec_decode_split_half_vec4x4",
        "rtxllm_launch_q4k_matvec_decode_split_compact_vec4x4",
        "rtxllm_launch_q4k_matvec_decode_split_native_vec4x4",
        "rtxllm_launch_q5k_matvec_decode_probe", "rtxllm_launch_iq2s_matvec_probe",
        "rtxllm_launch_iq2s_matvec_decode_probe", "rtxllm_launch_iq3s_matvec_decode_probe",
        "rtxllm_launch_output_token_sample", "rtxllm_launch_rmsnorm_feedback",
        "rtxllm_launch_silu_rmsnorm_feedback", "rtxllm_launch_rmsnorm_feedback_with_silu_cache",
        "rtxllm_launch_gated_silu_rmsnorm_feedback", "rtxllm_launch_rmsnorm_silu_cache",
        "rtxllm_launch_rmsnorm_cache", "rtxllm_launch_rmsnorm_cache_and_gated_product",
    ]
    assert set(want) <= set(qgemv_b200.header_functions())


@pytest.mark.parametrize("name", ["rtxllm_launch_q5k_matvec_decode_probe",
                                  "rtxllm_launch_iq2s_matvec_decode_probe",
                                  "rtxllm_launch_iq3s_matvec_decode_probe"])
@pytest.mark.parametrize("rows,cols,limit", [(0, 256, 1), (4, 0, 1), (4, 256, 0), (4, 300, 4)])
def test_probe_launchers_validate_like_reference(name, rows, cols, limit):
    """decode_kernels.cu:4046-4048: zero dims or cols % 256 != 0 -> cudaErrorInvalidValue,
    returned before any launch."""
    code = qgemv_b200.call(name, 1, 1, 1, 1, 1, rows, cols, limit, 0, 0, 0, None)
    assert code == INVALID_VALUE


def test_q4k_launcher_zero_rows_is_a_launch_error():
    code = qgemv_b200.call("rtxllm_launch_q4k_matvec_decode", 1, 1, 1, 1, 1, 0, 256, 0, 0, 0, None)
    assert code == INVALID_CONFIGURATION


def test_output_sampler_validation():
    assert qgemv_b200.call("rtxllm_launch_output_token_sample", None, 1, 4, 10, 0, None) == INVALID_VALUE
    assert qgemv_b200.call("rtxllm_launch_output_token_sample", 1, 1, 0, 10, 0, None) == INVALID_VALUE
    assert qgemv_b200.call("rtxllm_launch_output_token_sample", 1, 1, 4, 0, 0, None) == INVALID_VALUE


@pytest.mark.parametrize("args", [
    (99, 1, 1, 1, 1, 4, 256, None),      # unknown format
    (0, 1, 1, 1, 1, 4, 255, None),       # cols not a multiple of 256
    (0, 1, 1, 1, 1, 0, 256, None),       # no rows
    (1, 1, None, 1, 1, 4, 256, None),    # split pack without metadata
    (0, None, None, 1, 1, 4, 256, None), # no payload
])
def test_qg_gemv_rejects_bad_arguments(args):
    assert qgemv_b200.call("qg_gemv", *args) == INVALID_VALUE


def test_batched_rejects_batch_out_of_range():
    assert qgemv_b200.call("qg_gemv_batched", 0, 1, None, 1, 1, 0, 4, 256, None) == INVALID_VALUE
    assert qgemv_b200.call("qg_gemv_batched", 0, 1, None, 1, 1, 33, 4, 256, None) == INVALID_VALUE


def test_feedback_cache_validation():
    assert qgemv_b200.call("rtxllm_launch_rmsnorm_cache", 1, 1, 4, 0, 1e-6, 0, None) == INVALID_VALUE
    assert qgemv_b200.call("rtxllm_launch_rmsnorm_silu_cache", 1, 1, 4, 0, 1e-6, 0, None) == INVALID_VALUE
    assert qgemv_b200.call("rtxllm_launch_rmsnorm_cache_and_gated_product",
                           1, 1, 1, 1, 4, 0, 8, 1e-6, 0, None) == INVALID_VALUE


def test_get_error_rejects_null():
    assert qgemv_b200.call("qg_get_error", None) == INVALID_VALUE


def test_layer_slice_rejects_bad_dims():
    from qgemv_b200.slice import LayerSliceC

    c = LayerSliceC()
    c.hidden, c.q_rows, c.kv_rows, c.ffn = 4096, 4096, 1024, 1000  # ffn not a multiple of 256
    n = ctypes.c_size_t(0)
    assert qgemv_b200.call("qg_layer_slice_workspace_bytes", ctypes.byref(c), ctypes.byref(n)) == 1
