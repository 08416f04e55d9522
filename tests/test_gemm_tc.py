"""Batched GEMM on the tensor cores (qg_gemm_batched) against the
oracle, row by row and batch row by batch row, within the north_star bound
max |err| <= 1e-3 * ||w_row||_1 * ||x_b||_inf.  Shapes cover partial 128-row tiles,
tiles split between CTAs (the stream-K fixup), every supported format and batch
sizes on both sides of the N=16 / N=32 switch; the config-4 shapes run in full on
the GPU with sampled rows checked."""

import ctypes

import numpy as np
import pytest
import torch

import qgemv_b200
from qgemv_b200 import ops, packs
from test_gpu_parity import assert_rows_close, dev, row_tol

TC_FORMATS = [packs.Q4K_RAW, packs.Q5K, packs.IQ2S, packs.IQ3S]
INVALID_VALUE = 1


def check_rows(port, pk, x, y, rows, cols, r0=0, r1=None):
    r1 = rows if r1 is None else r1
    bpr = cols // 256
    pb = packs.payload_bytes_per_block(pk.fmt)
    sub = pk.payload[r0 * bpr * pb : r1 * bpr * pb]
    for b in range(x.shape[0]):
        want = port.matvec(pk.fmt, pk.payload, None, x[b], rows, cols, r0, r1)
        tol = row_tol(port, pk.fmt, sub, None, x[b], r1 - r0, cols)
        assert_rows_close(y[b, r0:r1], want, tol)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", TC_FORMATS)
@pytest.mark.parametrize("rows,cols,batch", [
    (128, 256, 16),     # one unit
    (300, 512, 8),      # ragged last tile, every tile split over two CTAs
    (1000, 2048, 17),   # N=32 with padded batch rows, tiles split over 8 CTAs
    (2048, 4096, 32),   # uneven stream-K ranges over all SMs
    (200, 1024, 1),
    (100, 512, 16),     # fewer rows than one tile: per-row copies instead of the tensor map
])
def test_gemm_batched_vs_oracle(cuda, port, fmt, rows, cols, batch):
    pk = packs.synthetic_pack(fmt, rows, cols, seed=rows * 7 + cols + fmt)
    x = packs.synthetic_activation(cols, rows + batch, batch=batch).reshape(batch, cols)
    y = ops.gemm_batched(fmt, dev(pk.payload, cuda), None, dev(x, cuda), rows, cols).cpu().numpy()
    assert np.all(np.isfinite(y))
    check_rows(port, pk, x, y, rows, cols)
    assert ops.get_error() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", [packs.Q4K_RAW, packs.IQ2S])
def test_gemm_batched_deterministic_and_scaled_inputs(cuda, port, fmt):
    """Two calls give identical bits; batch rows with very different magnitudes (per-row
    power-of-two scaling) and an all-zero row stay within the bound."""
    rows, cols, batch = 640, 3072, 24
    pk = packs.synthetic_pack(fmt, rows, cols, seed=5)
    x = packs.synthetic_activation(cols, 9, batch=batch).reshape(batch, cols)
    x[1] *= 1e-20
    x[2] *= 3e15
    x[3] = 0.0
    x[4, ::7] = 0.0
    p = dev(pk.payload, cuda)
    xd = dev(x, cuda)
    ws = torch.empty(ops.gemm_batched_workspace_bytes(fmt, batch, rows, cols), dtype=torch.uint8, device=cuda)
    y1 = ops.gemm_batched(fmt, p, None, xd, rows, cols, workspace=ws).cpu().numpy()
    y2 = ops.gemm_batched(fmt, p, None, xd, rows, cols, workspace=ws).cpu().numpy()
    assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32))
    assert np.all(y1[3] == 0.0)
    check_rows(port, pk, x, y1, rows, cols)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", [packs.Q4K_RAW, packs.IQ2S])
@pytest.mark.parametrize("rows,cols", [(28672, 8192), (8192, 28672)])
@pytest.mark.parametrize("batch", [8, 16, 32])
def test_gemm_batched_config4_sampled_rows(cuda, port, fmt, rows, cols, batch):
    """BASELINE config 4 shapes in full on the GPU; three 16-row windows against the oracle."""
    pk = packs.synthetic_pack(fmt, rows, cols, seed=rows + cols + fmt)
    x = packs.synthetic_activation(cols, batch, batch=batch).reshape(batch, cols)
    y = ops.gemm_batched(fmt, dev(pk.payload, cuda), None, dev(x, cuda), rows, cols).cpu().numpy()
    assert np.all(np.isfinite(y))
    for r0 in (0, rows // 2 - 9, rows - 16):
        check_rows(port, pk, x, y, rows, cols, r0, r0 + 16)


@pytest.mark.gpu
def test_gemm_batched_unaligned_iq_tail(cuda, port):
    """IQ rows whose block windows reach the payload's unaligned end (82 * blocks not a
    multiple of 16): the last bytes are fetched with plain loads."""
    rows, cols, batch = 129, 768, 16   # 129 * 3 * 82 = 31734 bytes, 6 past a 16-B boundary
    pk = packs.synthetic_pack(packs.IQ2S, rows, cols, seed=44)
    assert pk.payload.size % 16 != 0
    buf = torch.empty(pk.payload.size, dtype=torch.uint8, device=cuda)
    buf.copy_(dev(pk.payload, cuda))
    x = packs.synthetic_activation(cols, 3, batch=batch).reshape(batch, cols)
    y = ops.gemm_batched(packs.IQ2S, buf, None, dev(x, cuda), rows, cols).cpu().numpy()
    check_rows(port, pk, x, y, rows, cols)


@pytest.mark.parametrize("args", [
    (packs.Q4K_PREDECODED, 8, 128, 256),  # split packs are not supported here
    (packs.Q4K_RAW, 0, 128, 256),
    (packs.Q4K_RAW, 33, 128, 256),
    (packs.Q4K_RAW, 8, 0, 256),
    (packs.Q4K_RAW, 8, 128, 300),
])
def test_gemm_batched_rejects_bad_arguments(args):
    fmt, batch, rows, cols = args
    n = ctypes.c_size_t(0)
    assert qgemv_b200.call("qg_gemm_batched_workspace_bytes", fmt, batch, rows, cols, ctypes.byref(n)) == INVALID_VALUE
    assert qgemv_b200.call("qg_gemm_batched", fmt, 16, None, 16, 16, batch, rows, cols, 256, None) == INVALID_VALUE


def test_gemm_batched_rejects_misaligned_pointers():
    assert qgemv_b200.call("qg_gemm_batched", packs.Q4K_RAW, 8, None, 16, 16, 8, 128, 256, 256, None) == INVALID_VALUE
    assert qgemv_b200.call("qg_gemm_batched", packs.Q4K_RAW, 16, None, 16, 16, 8, 128, 256, 128, None) == INVALID_VALUE
    assert qgemv_b200.call("qg_gemm_batched", packs.Q4K_RAW, 16, None, 16, 16, 8, 128, 256, None, None) == INVALID_VALUE
