"""Multi-vector GEMV on the CUDA cores (csrc/qg_gemv_batch.cu): qg_gemv_batched for every
format, and qg_gemm_batched below its tensor-core threshold (batch 5), against the oracle vector by vector.

The kernel reads each weight once per group of up to 8 vectors, holds x as int16 with one
scale per (vector, column slice) and sums exact int32 products per 32-column sub-block, so
its bound, 1.6e-5 * ||w_row||_1 * ||x_b||_inf plus fp32 rounding, is checked here at
1e-4 (ten times tighter than the north_star bound of 1e-3).  Shapes cover one-slice and
multi-slice rows (slices chained as y += ...), 2-, 4- and 8-vector kernels with padded
vectors, groups beyond 8 vectors (the ninth alone takes the batch-1 GEMV), ragged unit
tails, IQ rows whose windows reach an unaligned payload end, misaligned packs (vector by
vector fallback) and misaligned x (scalar loads)."""

import numpy as np
import pytest
import torch

from qgemv_b200 import ops, packs
from test_gpu_parity import FORMAT_TAGS, assert_rows_close, dev

TIGHT = 1e-4


def tight_tol(port, pk, x, rows, cols):
    l1 = port.row_l1(pk.fmt, pk.payload, pk.meta, rows, cols)
    return TIGHT * l1 * float(np.abs(x).max()) + 1e-30


def check_all(port, pk, x, y, rows, cols):
    for b in range(x.shape[0]):
        want = port.matvec(pk.fmt, pk.payload, pk.meta, x[b], rows, cols)
        assert_rows_close(y[b], want, tight_tol(port, pk, x[b], rows, cols))


SHAPES = [
    (37, 256, 2),      # one block per row, 2-vector kernel, ragged unit
    (300, 4096, 3),    # 4-vector kernel with one padded vector
    (129, 768, 5),     # 8-vector kernel, IQ payload end off a 16-B boundary
    (1000, 8192, 8),   # one slice of 8 full warps
    (64, 14336, 7),    # two slices (8-vector), one (4-vector)
    (96, 28672, 8),    # four 7-warp slices
    (333, 2304, 9),    # 8 vectors, then one on the batch-1 GEMV
    (100, 1024, 12),   # 8 + 4
]


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", list(FORMAT_TAGS))
@pytest.mark.parametrize("rows,cols,batch", SHAPES)
def test_gemv_batched_vs_oracle(cuda, port, fmt, rows, cols, batch):
    pk = packs.synthetic_pack(fmt, rows, cols, seed=rows * 3 + cols + fmt)
    x = packs.synthetic_activation(cols, rows + batch, batch=batch).reshape(batch, cols)
    y = ops.gemv_batched(fmt, dev(pk.payload, cuda), dev(pk.meta, cuda), dev(x, cuda), rows, cols)
    y = y.cpu().numpy()
    assert np.all(np.isfinite(y))
    check_all(port, pk, x, y, rows, cols)
    assert ops.get_error() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", [packs.Q4K_RAW, packs.Q5K, packs.IQ2S, packs.IQ3S])
@pytest.mark.parametrize("batch", [2, 3, 4])
def test_gemm_batched_below_the_tensor_core_threshold_runs_the_cuda_core_path(cuda, port, fmt, batch):
    """qg_gemm_batched below batch 5 gives the same bits as qg_gemv_batched."""
    rows, cols = 700, 14336
    pk = packs.synthetic_pack(fmt, rows, cols, seed=batch + fmt)
    x = packs.synthetic_activation(cols, batch, batch=batch).reshape(batch, cols)
    p, xd = dev(pk.payload, cuda), dev(x, cuda)
    y1 = ops.gemm_batched(fmt, p, None, xd, rows, cols).cpu().numpy()
    y2 = ops.gemv_batched(fmt, p, None, xd, rows, cols).cpu().numpy()
    assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32))
    check_all(port, pk, x, y1, rows, cols)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", [packs.Q4K_RAW, packs.IQ2S, packs.Q4K_COMPACT])
def test_gemv_batched_deterministic_and_scaled_vectors(cuda, port, fmt):
    """Identical bits on repeat; vectors of very different magnitudes (one scale per
    vector), an all-zero vector and a partly zero one stay within the tight bound."""
    rows, cols, batch = 640, 28672, 8
    pk = packs.synthetic_pack(fmt, rows, cols, seed=5)
    x = packs.synthetic_activation(cols, 9, batch=batch).reshape(batch, cols)
    x[1] *= 1e-20
    x[2] *= 3e15
    x[3] = 0.0
    x[4, ::7] = 0.0
    x[5, : cols // 2] = 0.0   # whole slices of zeros
    p, m, xd = dev(pk.payload, cuda), dev(pk.meta, cuda), dev(x, cuda)
    y1 = ops.gemv_batched(fmt, p, m, xd, rows, cols).cpu().numpy()
    y2 = ops.gemv_batched(fmt, p, m, xd, rows, cols).cpu().numpy()
    assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32))
    assert np.all(y1[3] == 0.0)
    check_all(port, pk, x, y1, rows, cols)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", [packs.Q4K_RAW, packs.IQ3S, packs.Q4K_NATIVE])
def test_gemv_batched_misaligned_pack_and_x(cuda, port, fmt):
    """A payload 2 bytes off a 16-B boundary takes the vector-by-vector fallback; x one
    float off a 16-B boundary takes the kernel's scalar loads."""
    rows, cols, batch = 150, 2048, 6
    pk = packs.synthetic_pack(fmt, rows, cols, seed=77)
    x = packs.synthetic_activation(cols, 4, batch=batch).reshape(batch, cols)
    # misaligned x, aligned pack
    xb = torch.zeros(batch * cols + 1, dtype=torch.float32, device=cuda)
    xb[1:].copy_(dev(x.reshape(-1), cuda))
    xv = xb[1:].view(batch, cols)
    y = ops.gemv_batched(fmt, dev(pk.payload, cuda), dev(pk.meta, cuda), xv, rows, cols).cpu().numpy()
    check_all(port, pk, x, y, rows, cols)
    # misaligned pack
    pb = torch.zeros(pk.payload.size + 2, dtype=torch.uint8, device=cuda)
    pb[2:].copy_(dev(pk.payload, cuda))
    y = ops.gemv_batched(fmt, pb[2:], dev(pk.meta, cuda), dev(x, cuda), rows, cols).cpu().numpy()
    for b in range(batch):
        want = port.matvec(fmt, pk.payload, pk.meta, x[b], rows, cols)
        l1 = port.row_l1(fmt, pk.payload, pk.meta, rows, cols)
        assert_rows_close(y[b], want, 1e-3 * l1 * float(np.abs(x[b]).max()) + 1e-30)
    assert ops.get_error() == 0
