"""Decode step on the GPU against the CPU restatement
(oracle/decode_oracle.py; GEMVs through the C oracle pinned to the reference)."""

import copy
import os
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import REPO

pytestmark = pytest.mark.gpu

SMALL = dict(layers=2, hidden=512, n_q_heads=4, n_kv_heads=2, head_dim=128, ffn=1024,
             vocab=1000, ctx_max=64)
# a model that shards four ways (every rank: 2 q heads, 1 kv head, 512 ffn rows, 256 vocab rows)
SMALL_TP4 = dict(layers=2, hidden=1024, n_q_heads=8, n_kv_heads=4, head_dim=128, ffn=2048,
                 vocab=1024, ctx_max=64)


def _oracle(port, model, x, pos):
    sys.path.insert(0, str(REPO / "oracle"))
    import decode_oracle
    from qgemv_b200 import decoder

    w = copy.deepcopy(decoder.rank_weights(model, 0, 1))
    return decode_oracle.step(port, model.spec, w, x, pos)


def _check(hidden, want, tok, want_tok, logits_margin_ok=True):
    scale = np.abs(want).max()
    err = np.abs(hidden - want).max()
    assert err <= 3e-3 * scale, f"max err {err} vs scale {scale}"
    if logits_margin_ok:
        assert tok == want_tok


@pytest.mark.parametrize("pos", [0, 37, 63])
def test_decoder_tp1_small_vs_oracle(cuda, port, pos):
    from qgemv_b200 import decoder, packs

    spec = decoder.ModelSpec(**SMALL)
    model = decoder.HostModel.synthetic(spec, seed=11)
    x = packs.synthetic_activation(spec.hidden, 12)
    want_tok, want_hidden = _oracle(port, model, x, pos)
    dec = decoder.Decoder(spec, decoder.rank_weights(model, 0, 1))
    tok = int(dec.step(torch.from_numpy(x).to(cuda), pos).item())
    torch.cuda.synchronize()
    _check(dec.hidden().cpu().numpy(), want_hidden, tok, want_tok)
    dec.close()


def test_decoder_real_layer_dims_vs_oracle(cuda, port):
    """One layer at the 70B-class dimensions (hidden 8192, 64/8 heads, ffn 28672, full
    4096-position cache), vocab cut to 4096 so the CPU oracle finishes in seconds."""
    from qgemv_b200 import decoder, packs

    spec = decoder.ModelSpec(layers=1, vocab=4096)
    model = decoder.HostModel.synthetic(spec, seed=3)
    x = packs.synthetic_activation(spec.hidden, 4)
    pos = spec.ctx_max - 1
    want_tok, want_hidden = _oracle(port, model, x, pos)
    dec = decoder.Decoder(spec, decoder.rank_weights(model, 0, 1))
    tok = int(dec.step(torch.from_numpy(x).to(cuda), pos).item())
    torch.cuda.synchronize()
    _check(dec.hidden().cpu().numpy(), want_hidden, tok, want_tok)
    dec.close()


def test_decoder_graph_replay_matches_eager(cuda):
    from qgemv_b200 import decoder
    from qgemv_b200.slice import StepGraph

    spec = decoder.ModelSpec(**SMALL)
    model = decoder.HostModel.synthetic(spec, seed=2)
    dec = decoder.Decoder(spec, decoder.rank_weights(model, 0, 1))
    x = torch.randn(spec.hidden, device=cuda)
    tok = int(dec.step(x, 20).item())
    hid = dec.hidden().clone()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    g = StepGraph(stream, lambda: dec.step(x, 20, stream))
    for _ in range(3):
        g.launch()
    stream.synchronize()
    g.close()
    assert int(dec.token.item()) == tok
    assert torch.equal(dec.hidden(), hid)
    dec.close()


TP_STEPS = (30, 31, 32)  # positions; the middle step runs as a captured graph


def _tp_rank(rank, world, q_in, q_out, spec_kw):
    sys.path.insert(0, str(REPO / "local-ai-gpu-acceleration_b200"))
    import torch

    from qgemv_b200 import decoder, packs
    from qgemv_b200.slice import StepGraph

    torch.cuda.set_device(rank)
    spec = decoder.ModelSpec(**spec_kw)
    model = decoder.HostModel.synthetic(spec, seed=21)
    if rank == 0:
        nid = decoder.nccl_unique_id()
        for _ in range(world - 1):
            q_in.put(nid)
    else:
        nid = q_in.get(timeout=120)
    dev = f"cuda:{rank}"
    dec = decoder.Decoder(spec, decoder.rank_weights(model, rank, world), rank=rank, tp=world,
                          nccl_id=nid, device=dev)
    out = []
    for i, pos in enumerate(TP_STEPS):
        x = torch.from_numpy(packs.synthetic_activation(spec.hidden, 22 + i)).to(dev)
        if i == 1:
            stream = torch.cuda.Stream(dev)
            stream.wait_stream(torch.cuda.current_stream(dev))
            g = StepGraph(stream, lambda: dec.step(x, pos, stream))
            g.launch()
            stream.synchronize()
            g.close()
            tok = int(dec.token.item())
        else:
            tok = int(dec.step(x, pos).item())
        torch.cuda.synchronize()
        out.append((tok, dec.hidden().cpu().numpy()))
    q_out.put((rank, out))
    dec.close()


@pytest.mark.parametrize("world,spec_kw", [(2, SMALL), (4, SMALL_TP4)], ids=["tp2", "tp4"])
def test_decoder_tp_matches_oracle(port, world, spec_kw):
    """World ranks over NVLink (fused exchange in the Wo / Wd GEMVs, NCCL only for the
    token all-gather): three consecutive steps -- eager, captured graph, eager -- against
    the oracle stepping the same model with its caches carried along."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    sys.path.insert(0, str(REPO / "oracle"))
    import decode_oracle
    from qgemv_b200 import decoder, packs

    spec = decoder.ModelSpec(**spec_kw)
    model = decoder.HostModel.synthetic(spec, seed=21)
    w = copy.deepcopy(decoder.rank_weights(model, 0, 1))
    want = []
    for i, pos in enumerate(TP_STEPS):
        x = packs.synthetic_activation(spec.hidden, 22 + i)
        want.append(decode_oracle.step(port, spec, w, x, pos))
    ctx = mp.get_context("spawn")
    q_in, q_out = ctx.Queue(), ctx.Queue()
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    procs = [ctx.Process(target=_tp_rank, args=(r, world, q_in, q_out, spec_kw)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q_out.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for _, steps in res:
        for (tok, hid), (want_tok, want_hidden) in zip(steps, want):
            _check(hid, want_hidden, tok, want_tok)
    # every rank holds the same bits of the replicated hidden state
    for _, other in res[1:]:
        for (_, a), (_, b) in zip(res[0][1], other):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
