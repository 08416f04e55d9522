"""Batched layer slice (qg_layer_slice_forward_batched) and its batch-bucket graphs
(qg_slice_buckets_*): every stage of every row against the oracle on the GPU's own
input to that stage (the north_star bound per GEMV), each row's RMSNorm bit-equal to the
single-vector slice, bucket replays bit-equal to eager runs at the bucket's batch with
the rows padded, and the bucket selection.  CPU: argument validation and the workspace
size (no GPU call)."""

import ctypes

import numpy as np
import pytest
import torch

import qgemv_b200
from qgemv_b200 import packs
from qgemv_b200.slice import LayerSlice, LayerSliceC, SliceBuckets
from test_gpu_parity import assert_rows_close, row_tol
from test_layer_slice import oracle_silu_gate, oracle_weighted_rmsnorm

INVALID_VALUE = 1
SMALL = dict(hidden=512, q_rows=512, kv_rows=256, ffn=1536)


def stage_rows(port, sl, name, x_in, y_gpu):
    pk = sl.host[name]
    rows, cols = sl.shapes[name]
    for b in range(x_in.shape[0]):
        want = port.matvec(pk.fmt, pk.payload, pk.meta, x_in[b], rows, cols)
        assert_rows_close(y_gpu[b], want, row_tol(port, pk.fmt, pk.payload, pk.meta, x_in[b], rows, cols))


@pytest.mark.gpu
@pytest.mark.parametrize("dims,batch", [
    (SMALL, 2),     # CUDA-core multi-vector GEMVs
    (SMALL, 7),     # tensor-core tiles (batch >= 5)
    (dict(hidden=4096, q_rows=4096, kv_rows=1024, ffn=14336), 3),   # config-3 dims
])
def test_batched_slice_stagewise(cuda, port, dims, batch):
    sl = LayerSlice(**dims, seed=7, keep_host=True)
    x = packs.synthetic_activation(dims["hidden"], 5, batch=batch).reshape(batch, dims["hidden"])
    xd = torch.from_numpy(x).to(cuda)
    out = sl.forward_batched(xd).cpu().numpy()
    v = {k: t.cpu().numpy() for k, t in sl.batched_views(batch).items()}
    # each row's h: the oracle RMSNorm, and bit for bit the single-vector slice
    for b in range(batch):
        np.testing.assert_allclose(v["h"][b], oracle_weighted_rmsnorm(port, x[b], sl.norm_host, sl.eps),
                                   rtol=2e-6, atol=1e-6)
        sl.forward(xd[b].contiguous())
        torch.cuda.synchronize()
        h1 = sl.views()["h"].cpu().numpy()
        assert np.array_equal(h1.view(np.uint32), v["h"][b].view(np.uint32))
    for name, src, dst in (("wq", "h", "q"), ("wk", "h", "k"), ("wv", "h", "v"), ("wo", "q", "o"),
                           ("wg", "o", "gate"), ("wu", "o", "up")):
        stage_rows(port, sl, name, v[src], v[dst])
    for b in range(batch):
        np.testing.assert_allclose(v["act"][b], oracle_silu_gate(port, v["gate"][b], v["up"][b]),
                                   rtol=1e-5, atol=1e-6)
    pk = sl.host["wd"]
    rows, cols = sl.shapes["wd"]
    for b in range(batch):
        want = x[b] + port.matvec(pk.fmt, pk.payload, pk.meta, v["act"][b], rows, cols)
        tol = row_tol(port, pk.fmt, pk.payload, pk.meta, v["act"][b], rows, cols) + 1e-6 * np.abs(x[b])
        assert_rows_close(out[b], want, tol)


@pytest.mark.gpu
def test_buckets_replay_like_eager_runs(cuda):
    sl = LayerSlice(**SMALL, seed=3)
    buckets = SliceBuckets(sl, [1, 2, 4, 8, 16])
    x = torch.from_numpy(packs.synthetic_activation(SMALL["hidden"], 11, batch=16).reshape(16, -1)).to(cuda)
    for batch, bucket in [(1, 1), (2, 2), (3, 4), (4, 4), (5, 8), (8, 8), (11, 16), (16, 16)]:
        assert buckets.bucket(batch) == bucket
        got = buckets.run(x[:batch].contiguous())
        # eager at the bucket's batch over the padded rows (the rows past `batch` are those
        # an earlier run left in the bucket: any value, here x's own rows)
        want = sl.forward_batched(x[:bucket].contiguous())
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int32), want[:batch].view(torch.int32)), (batch, bucket)
    # a second replay of the same bucket with other rows
    y = x.flip(0).contiguous()
    got = buckets.run(y[:6].contiguous())
    want = sl.forward_batched(y[:8].contiguous())
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int32), want[:6].view(torch.int32))
    with pytest.raises(qgemv_b200.CudaError):
        buckets.run(torch.zeros(17, SMALL["hidden"], device=cuda))
    buckets.close()


def _fake_slice():
    # non-null pointers that are never dereferenced: argument checks only
    return LayerSliceC(512, 512, 256, 1536, 1e-5, 16, packs.IQ3S, 16, 16, 16, 16, None, None, None, None,
                       packs.IQ2S, 16, 16, None, None, packs.Q5K, 16, None)


def test_buckets_reject_bad_arguments():
    s = _fake_slice()
    h = ctypes.c_void_p()
    for batches in ([4, 2], [0, 1], [1, 33], [2, 2]):
        arr = (ctypes.c_uint32 * len(batches))(*batches)
        assert qgemv_b200.call("qg_slice_buckets_create", ctypes.byref(s), arr, len(batches), None,
                               ctypes.byref(h)) == INVALID_VALUE
    assert qgemv_b200.call("qg_slice_buckets_create", ctypes.byref(s), None, 1, None, ctypes.byref(h)) == INVALID_VALUE
    assert qgemv_b200.call("qg_slice_buckets_run", None, 16, 16, 1, None) == INVALID_VALUE
    assert qgemv_b200.call("qg_layer_slice_forward_batched", ctypes.byref(s), 16, 16, 0, 256, None) == INVALID_VALUE
    assert qgemv_b200.call("qg_layer_slice_forward_batched", ctypes.byref(s), 16, 16, 33, 256, None) == INVALID_VALUE


def test_batched_workspace_grows_with_the_batch():
    s = _fake_slice()
    sizes = []
    for batch in (1, 2, 4, 5, 16):
        n = ctypes.c_size_t(0)
        assert qgemv_b200.call("qg_layer_slice_batched_workspace_bytes", ctypes.byref(s), batch,
                               ctypes.byref(n)) == 0
        sizes.append(n.value)
    assert sizes == sorted(sizes) and len(set(sizes)) == len(sizes)
    # from batch 5 the tensor-core workspace joins the activations
    act_per_row = 4 * (3 * 512 + 2 * 256 + 512 + 3 * 1536)
    assert sizes[3] - sizes[2] > act_per_row
