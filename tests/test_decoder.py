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
# eight ways (every rank: 2 q heads, 1 kv head, 256 ffn rows, 128 vocab rows)
SMALL_TP8 = dict(layers=2, hidden=1024, n_q_heads=16, n_kv_heads=8, head_dim=128, ffn=2048,
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


def test_step_at_matches_step_and_replays_across_tokens(cuda):
    """The step with its position in device memory: bit-identical to the host-position
    step; one graph captured per context bucket, replayed for successive tokens with the
    position advanced on the device, equals the eager steps; a position past the bucket
    writes nothing and sets QG_ERR_POSITION."""
    from qgemv_b200 import decoder, ops
    from qgemv_b200.slice import StepGraph

    spec = decoder.ModelSpec(**SMALL)
    model = decoder.HostModel.synthetic(spec, seed=31)
    a = decoder.Decoder(spec, copy.deepcopy(decoder.rank_weights(model, 0, 1)))
    b = decoder.Decoder(spec, copy.deepcopy(decoder.rank_weights(model, 0, 1)))
    x = torch.randn(spec.hidden, device=cuda)
    pos = torch.zeros(1, dtype=torch.int32, device=cuda)
    for p in (0, 9, 40, 63):  # eager: device position vs host position, no advance
        pos.fill_(p)
        tb = int(b.step_at(x, pos, ctx_bucket=64, advance=False).item())
        ta = int(a.step(x, p).item())
        torch.cuda.synchronize()
        assert ta == tb and torch.equal(a.hidden(), b.hidden()), p
        assert int(pos.item()) == p
    # buckets: a 32-position graph for tokens 10..12, then a 64-position graph for 33, 34
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    pos.fill_(10)
    torch.cuda.synchronize()
    graphs = {c: StepGraph(stream, lambda c=c: b.step_at(x, pos, ctx_bucket=c, advance=True, stream=stream))
              for c in (32, 64)}
    for p in (10, 11, 12):
        graphs[32].launch()
        stream.synchronize()
        ta = int(a.step(x, p).item())
        torch.cuda.synchronize()
        assert int(b.token.item()) == ta and torch.equal(a.hidden(), b.hidden()), p
    assert int(pos.item()) == 13
    pos.fill_(33)
    torch.cuda.synchronize()
    for p in (33, 34):
        graphs[64].launch()
        stream.synchronize()
        ta = int(a.step(x, p).item())
        torch.cuda.synchronize()
        assert int(b.token.item()) == ta and torch.equal(a.hidden(), b.hidden()), p
    assert ops.get_error() == 0
    # position 40 in the 32-position bucket: refused on the device, caches untouched
    caches = [c.clone() for c in b.caches[0]]
    pos.fill_(40)
    torch.cuda.synchronize()
    graphs[32].launch()
    stream.synchronize()
    assert ops.get_error() & 0x2  # QG_ERR_POSITION
    assert all(torch.equal(c, d) for c, d in zip(caches, b.caches[0]))
    for g in graphs.values():
        g.close()
    a.close()
    b.close()


TP_STEPS = (30, 31, 32)  # positions; the middle step runs as a captured graph


def _run_steps(dec, spec, dev):
    from qgemv_b200 import packs
    from qgemv_b200.slice import StepGraph

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
    return out


def _tp_rank(rank, world, q_in, q_out, spec_kw, collective, caller_exchange=False):
    sys.path.insert(0, str(REPO / "local-ai-gpu-acceleration_b200"))
    import torch

    from qgemv_b200 import decoder, ops

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
    exchange = None
    if caller_exchange:
        # the exchange region inside a larger caller allocation, at a 256-B offset (the way
        # a superallocator arena sits inside its pool)
        n = decoder.exchange_bytes(spec, rank, world)
        pool = torch.zeros(n + 4096, dtype=torch.uint8, device=dev)
        exchange = pool[768 + 256 * rank:][:n]
    dec = decoder.Decoder(spec, decoder.rank_weights(model, rank, world), rank=rank, tp=world,
                          nccl_id=nid, device=dev, collective=collective, exchange=exchange)
    out = _run_steps(dec, spec, dev)
    q_out.put((rank, out, ops.get_error()))
    dec.close()


@pytest.mark.parametrize("world,spec_kw,collective,caller_exchange", [
    (2, SMALL, 0, False), (2, SMALL, 1, False), (2, SMALL, 0, True), (4, SMALL_TP4, 0, False),
    (8, SMALL_TP8, 0, False)],
    ids=["tp2", "tp2-nccl", "tp2-caller-exchange", "tp4", "tp8"])
def test_decoder_tp_matches_oracle_and_tp1(port, world, spec_kw, collective, caller_exchange):
    """World ranks over NVLink (exchange fused into the Wo / Wd GEMVs; or, tp2-nccl, the
    same exchange words moved by ncclAllGather): three consecutive steps -- eager, captured
    graph, eager -- against the oracle stepping the same model with its caches carried
    along, and bit for bit against the same three steps on one GPU (TP 1): the token and
    every bit of the hidden state on every rank."""
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
    procs = [ctx.Process(target=_tp_rank, args=(r, world, q_in, q_out, spec_kw, collective,
                                                caller_exchange)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q_out.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for _, steps, err in res:
        assert err == 0
        for (tok, hid), (want_tok, want_hidden) in zip(steps, want):
            _check(hid, want_hidden, tok, want_tok)
    # TP 1 on cuda:0, the same model, steps and caches
    dec1 = decoder.Decoder(spec, decoder.rank_weights(model, 0, 1), device="cuda:0")
    single = _run_steps(dec1, spec, "cuda:0")
    dec1.close()
    for rank, steps, _ in res:
        for k, ((tok, hid), (tok1, hid1)) in enumerate(zip(steps, single)):
            assert tok == tok1, f"rank {rank} step {k}: token {tok} vs TP1 {tok1}"
            assert np.array_equal(hid.view(np.uint32), hid1.view(np.uint32)), \
                f"rank {rank} step {k}: hidden state differs from TP1"
