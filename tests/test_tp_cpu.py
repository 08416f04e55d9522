"""Tensor-parallel sharding arithmetic on CPU ranks (gloo, world size 2, 4 and 8): each rank runs
the oracle decode step on its own shards (row shards of Wq/Wk/Wv/Wg/Wu/head, column
shards of Wo/Wd, its kv heads), with the residual on rank 0 and real gloo all-reduce /
all-gather, and must reproduce the single-rank step."""

import os
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import REPO

SPEC_KW = dict(layers=2, hidden=512, n_q_heads=4, n_kv_heads=2, head_dim=128, ffn=1024,
               vocab=1000, ctx_max=64)
# shards four ways: every rank 2 q heads, 1 kv head, 512 ffn rows, 256 vocab rows
SPEC_KW_TP4 = dict(layers=2, hidden=1024, n_q_heads=8, n_kv_heads=4, head_dim=128, ffn=2048,
                   vocab=1024, ctx_max=64)
# eight ways: every rank 2 q heads, 1 kv head, 256 ffn rows, 128 vocab rows
SPEC_KW_TP8 = dict(layers=2, hidden=1024, n_q_heads=16, n_kv_heads=8, head_dim=128, ffn=2048,
                   vocab=1024, ctx_max=64)
POS = 37


def _rank_main(rank, world, port_no, q, spec_kw):
    sys.path.insert(0, str(REPO / "local-ai-gpu-acceleration_b200"))
    sys.path.insert(0, str(REPO / "oracle"))
    import torch
    import torch.distributed as dist

    import decode_oracle
    import qoracle
    from qgemv_b200 import decoder, packs

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port_no))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        spec = decoder.ModelSpec(**spec_kw)
        model = decoder.HostModel.synthetic(spec, seed=4)
        w = decoder.rank_weights(model, rank, world)
        x = packs.synthetic_activation(spec.hidden, 5)

        def allreduce(a):
            t = torch.from_numpy(np.ascontiguousarray(a, np.float32))
            dist.all_reduce(t)
            return t.numpy()

        def allgather(c):
            out = [None] * world
            dist.all_gather_object(out, c)
            return out

        tok, hid = decode_oracle.step(qoracle.Port(), spec, w, x, POS, tp=world, rank=rank,
                                      allreduce=allreduce, allgather=allgather)
        q.put((rank, tok, hid))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,spec_kw", [(2, SPEC_KW), (4, SPEC_KW_TP4), (8, SPEC_KW_TP8)],
                         ids=["tp2", "tp4", "tp8"])
def test_tp_sharding_matches_single_rank(port, world, spec_kw):
    sys.path.insert(0, str(REPO / "oracle"))
    import decode_oracle
    from qgemv_b200 import decoder, packs

    spec = decoder.ModelSpec(**spec_kw)
    model = decoder.HostModel.synthetic(spec, seed=4)
    x = packs.synthetic_activation(spec.hidden, 5)
    tok1, hid1 = decode_oracle.step(port, spec, decoder.rank_weights(model, 0, 1), x, POS)

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port_no = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank_main, args=(r, world, port_no + world, q, spec_kw))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, tok, hid in res:
        assert tok == tok1
        np.testing.assert_allclose(hid, hid1, rtol=2e-4, atol=2e-4 * np.abs(hid1).max())


def test_shard_shapes_cover_the_model():
    from qgemv_b200 import decoder

    spec = decoder.ModelSpec()  # the 70B-class config
    for tp in (1, 2, 4, 8):
        rows = [decoder.shard_shape(spec, r, tp) for r in range(tp)]
        assert sum(s["q_rows"] for s in rows) == spec.q_rows
        assert sum(s["kv_rows"] for s in rows) == spec.kv_rows
        assert sum(s["ffn_rows"] for s in rows) == spec.ffn
        assert sum(s["vocab_rows"] for s in rows) == spec.vocab
        offs = [s["vocab_offset"] for s in rows]
        assert offs[0] == 0 and all(offs[i] + rows[i]["vocab_rows"] == offs[i + 1] for i in range(tp - 1))
    # 70B layer: 376,832,000 packed bytes; 30.74 GB with the head
    assert spec.layer_weight_bytes() == 376_832_000
    assert spec.weight_bytes() == 80 * 376_832_000 + 591_003_648
