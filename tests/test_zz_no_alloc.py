"""qg_layer_slice_forward_static (library-owned scratch, no workspace argument) against
qg_layer_slice_forward with a caller workspace, on the same slice and inputs, for two
calls in a row.  Named to be collected last, so it also runs after every other test
has used the device."""

import ctypes

import numpy as np
import pytest
import torch

import qgemv_b200
from qgemv_b200 import ops, packs
from qgemv_b200._lib import check
from qgemv_b200.slice import LayerSlice, LayerSliceC

INVALID_VALUE = 1  # cudaErrorInvalidValue
SCRATCH_MAX = 1 << 20  # QG_SLICE_STATIC_SCRATCH_BYTES


def _dims_only(hidden, q_rows, kv_rows, ffn):
    c = LayerSliceC()
    c.hidden, c.q_rows, c.kv_rows, c.ffn = hidden, q_rows, kv_rows, ffn
    c.eps, c.norm_weight = 1e-5, 1
    for n in ("wq", "wk", "wv", "wo", "wg", "wu", "wd"):
        setattr(c, n, 1)
    c.attn_fmt = c.ffn_fmt = c.down_fmt = packs.Q4K_RAW
    return c


def test_static_scratch_covers_70b_slice_and_rejects_larger():
    """Host-side checks only (no launch): the 70B-class slice fits the scratch, a slice
    whose workspace is larger is rejected before any CUDA call."""
    n = ctypes.c_size_t(0)
    check("qg_layer_slice_workspace_bytes", ctypes.byref(_dims_only(8192, 8192, 1024, 28672)), ctypes.byref(n))
    assert n.value <= SCRATCH_MAX
    big = _dims_only(32768, 32768, 8192, 32768)
    check("qg_layer_slice_workspace_bytes", ctypes.byref(big), ctypes.byref(n))
    assert n.value > SCRATCH_MAX
    out = ctypes.c_void_p(1)
    assert qgemv_b200.call("qg_layer_slice_forward_static", ctypes.byref(big), 1, out, None) == INVALID_VALUE
    bad = _dims_only(4096, 4096, 1024, 1000)  # ffn not a multiple of 256
    assert qgemv_b200.call("qg_layer_slice_forward_static", ctypes.byref(bad), 1, out, None) == INVALID_VALUE
    ok = _dims_only(512, 512, 256, 1536)
    assert qgemv_b200.call("qg_layer_slice_forward_static", ctypes.byref(ok), None, out, None) == INVALID_VALUE


@pytest.mark.gpu
@pytest.mark.parametrize("dims", [
    dict(hidden=512, q_rows=512, kv_rows=256, ffn=1536),
    dict(hidden=4096, q_rows=4096, kv_rows=1024, ffn=14336),
])
def test_static_matches_workspace_forward_twice(cuda, dims):
    sl = LayerSlice(**dims, seed=21)
    stream = torch.cuda.current_stream()
    for call, seed in enumerate((301, 302)):
        x = torch.from_numpy(packs.synthetic_activation(dims["hidden"], seed)).to(cuda)
        want = sl.forward(x)
        got = torch.full_like(x, float("nan"))
        check("qg_layer_slice_forward_static", ctypes.byref(sl.c), x.data_ptr(), got.data_ptr(),
              stream.cuda_stream)
        torch.cuda.synchronize()
        w, g = want.cpu().numpy(), got.cpu().numpy()
        assert np.isfinite(g).all(), f"call {call}: output not fully written"
        # same kernels on the same inputs: expected identical, checked within 1e-6 relative
        np.testing.assert_allclose(g, w, rtol=1e-6, atol=1e-6 * float(np.abs(w).max()),
                                   err_msg=f"call {call}")


@pytest.mark.gpu
def test_static_back_to_back_on_one_stream(cuda):
    """Three static calls enqueued on one stream with no host synchronisation between them
    (each kernel's prologue may overlap the previous kernel through programmatic dependent
    launch while they share the one scratch array); every output must equal its
    workspace-path result and the library's error word must stay clear."""
    dims = dict(hidden=4096, q_rows=4096, kv_rows=1024, ffn=14336)
    sl = LayerSlice(**dims, seed=23)
    stream = torch.cuda.current_stream()
    xs = [torch.from_numpy(packs.synthetic_activation(dims["hidden"], 400 + i)).to(cuda) for i in range(3)]
    wants = [sl.forward(x) for x in xs]
    torch.cuda.synchronize()
    assert ops.get_error() == 0  # read and clear before the static calls
    outs = [torch.full_like(x, float("nan")) for x in xs]
    for x, o in zip(xs, outs):
        check("qg_layer_slice_forward_static", ctypes.byref(sl.c), x.data_ptr(), o.data_ptr(),
              stream.cuda_stream)
    torch.cuda.synchronize()
    for i, (w, o) in enumerate(zip(wants, outs)):
        w, g = w.cpu().numpy(), o.cpu().numpy()
        assert np.isfinite(g).all(), f"call {i}: output not fully written"
        np.testing.assert_allclose(g, w, rtol=1e-6, atol=1e-6 * float(np.abs(w).max()),
                                   err_msg=f"call {i}")
    assert ops.get_error() == 0
