"""Decode step (BASELINE config 5 widths) stage by stage: every GEMV output of the last
layer of a 2-layer step against the oracle GEMV of the GPU's own input to that stage,
row by row, within TIGHT * ||w_row||_1 * ||x||_inf (ten times tighter than the
north_star bound), plus the KV append, the attention output and the SiLU gate.  The
intermediates come from qg_decoder_stage_buffers.

Attention runs its dot products on the tensor cores with fp16 operands (q and the
softmax weights rounded to fp16, K and V are the fp16 cache), so its check uses the bound
those roundings give: a score error of at most
delta = (2^-11 + 3e-4) * max_t sum_i |q_i K_ti| / sqrt(d) per head (q's rounding and its
fp32 rotation angle) moves each softmax weight by a factor within exp(+-2 delta), and P's
own rounding adds 2^-11; the output, a convex combination of V rows, then moves by at
most (exp(2 delta) - 1 + 2^-10) * max|V|."""

import sys

import numpy as np
import pytest
import torch

from conftest import REPO
from test_gpu_parity import assert_rows_close

pytestmark = pytest.mark.gpu

TIGHT = 1e-4


def _oracle_module():
    sys.path.insert(0, str(REPO / "oracle"))
    import decode_oracle

    return decode_oracle


def _check_gemv(port, pk, x, got, base=None, name=""):
    want = port.matvec(pk.fmt, pk.payload, pk.meta, x, pk.rows, pk.cols).astype(np.float64)
    tol = TIGHT * port.row_l1(pk.fmt, pk.payload, pk.meta, pk.rows, pk.cols) * float(np.abs(x).max())
    if base is not None:  # residual add: one more fp32 rounding of the sum
        want = want + base.astype(np.float64)
        tol = tol + np.abs(want) * 2.0 ** -23
    assert got.shape == want.shape, name
    assert_rows_close(got, want, tol + 1e-30)


def test_decoder_stages_real_dims_two_layers(cuda, port):
    from qgemv_b200 import decoder, packs

    D = _oracle_module()
    spec = decoder.ModelSpec(layers=2, vocab=4096)
    model = decoder.HostModel.synthetic(spec, seed=7)
    w = decoder.rank_weights(model, 0, 1)
    dec = decoder.Decoder(spec, w)
    x = packs.synthetic_activation(spec.hidden, 21)
    pos = 1500
    dec.step(torch.from_numpy(x).to(cuda), pos)
    torch.cuda.synchronize()
    V = {k: (None if t is None else t.cpu().numpy()) for k, t in dec.stage_views().items()}
    kc, vc = (c.cpu().numpy() for c in dec.caches[-1])
    dec.close()
    L = w["layers"][-1]
    nq, nkv, d = spec.n_q_heads, spec.n_kv_heads, spec.head_dim

    # attention block
    assert V["layer_input"] is not None and np.all(np.isfinite(V["layer_input"]))
    h = D.wrmsnorm(V["layer_input"], L["attn_norm"], spec.eps)
    _check_gemv(port, L["wq"], h, V["q"], name="q")
    _check_gemv(port, L["wk"], h, V["k"], name="k")
    _check_gemv(port, L["wv"], h, V["v"], name="v")
    # KV append: the rotated k and v at `pos`, fp16 (the GPU's angle pos * inv_freq is an
    # fp32 product: up to ~1e-4 rad off at pos 1500, against the fp64 rotation here)
    k_rot = D.rope(V["k"], nkv, pos, spec.rope_base)
    np.testing.assert_allclose(kc[:, pos, :].astype(np.float32), k_rot.reshape(nkv, d),
                               rtol=2.0 ** -10, atol=3e-4 * float(np.abs(k_rot).max()))
    np.testing.assert_array_equal(vc[:, pos, :], V["v"].reshape(nkv, d).astype(np.float16))
    q_rot = D.rope(V["q"], nq, pos, spec.rope_base)
    want = D.attention(q_rot, kc, vc, nq, nkv, pos + 1).reshape(nq, d).astype(np.float64)
    got = V["attn"].reshape(nq, d).astype(np.float64)
    group = nq // nkv
    for hq in range(nq):
        K = kc[hq // group, : pos + 1].astype(np.float64)
        Vv = vc[hq // group, : pos + 1].astype(np.float64)
        # q's fp16 rounding plus its rotation angle (fp32 on the GPU)
        delta = (2.0 ** -11 + 3e-4) * float((np.abs(K) @ np.abs(q_rot[hq * d:(hq + 1) * d])).max()) / np.sqrt(d)
        bound = (np.expm1(2.0 * delta) + 2.0 ** -10) * float(np.abs(Vv).max()) + 1e-6
        err = float(np.abs(got[hq] - want[hq]).max())
        assert err <= bound, f"head {hq}: attention err {err} > bound {bound}"
    _check_gemv(port, L["wo"], V["attn"], V["x1"], base=V["layer_input"], name="x1")

    # feed-forward block
    h2 = D.wrmsnorm(V["x1"], L["ffn_norm"], spec.eps)
    _check_gemv(port, L["wg"], h2, V["g"], name="g")
    _check_gemv(port, L["wu"], h2, V["u"], name="u")
    np.testing.assert_allclose(V["a"], D.silu_gate(V["g"], V["u"]), rtol=1e-5, atol=1e-6)
    _check_gemv(port, L["wd"], V["a"], V["hidden"], base=V["x1"], name="hidden")

    # vocab head
    hf = D.wrmsnorm(V["hidden"], w["final_norm"], spec.eps)
    _check_gemv(port, w["head"], hf, V["logits"], name="logits")


def test_decoder_stage_buffers_before_a_step(cuda):
    """cudaErrorNotReady until a step has been enqueued."""
    from qgemv_b200 import decoder

    spec = decoder.ModelSpec(layers=1, hidden=512, n_q_heads=4, n_kv_heads=2, head_dim=128,
                             ffn=1024, vocab=1000, ctx_max=64)
    model = decoder.HostModel.synthetic(spec, seed=1)
    dec = decoder.Decoder(spec, decoder.rank_weights(model, 0, 1))
    with pytest.raises(RuntimeError):
        dec.stage_views()
    dec.close()
