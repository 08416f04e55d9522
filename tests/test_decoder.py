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


def _tp_rank(rank, world, q_in, q_out):
    sys.path.insert(0, str(REPO / "local-ai-gpu-acceleration_b200"))
    import torch

    from qgemv_b200 import decoder, packs

    torch.cuda.set_device(rank)
    spec = decoder.ModelSpec(**SMALL)
    model = decoder.HostModel.synthetic(spec, seed=21)
    if rank == 0:
        nid = decoder.nccl_unique_id()
        for _ in range(world - 1):
            q_in.put(nid)
    else:
        nid = q_in.get(timeout=120)
    dec = decoder.Decoder(spec, decoder.rank_weights(model, rank, world), rank=rank, tp=world,
                          nccl_id=nid, device=f"cuda:{rank}")
    x = torch.from_numpy(packs.synthetic_activation(spec.hidden, 22)).to(f"cuda:{rank}")
    tok = int(dec.step(x, 30).item())
    torch.cuda.synchronize()
    q_out.put((rank, tok, dec.hidden().cpu().numpy()))
    dec.close()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_decoder_tp2_matches_oracle(port):
    from qgemv_b200 import decoder, packs

    spec = decoder.ModelSpec(**SMALL)
    model = decoder.HostModel.synthetic(spec, seed=21)
    x = packs.synthetic_activation(spec.hidden, 22)
    want_tok, want_hidden = _oracle(port, model, x, 30)
    ctx = mp.get_context("spawn")
    q_in, q_out = ctx.Queue(), ctx.Queue()
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, q_in, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q_out.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for _, tok, hid in res:
        _check(hid, want_hidden, tok, want_tok)
