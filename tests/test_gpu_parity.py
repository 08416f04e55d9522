"""GPU parity: the sm_100a kernels, called through the C-ABI, against the oracle.

* dequantization: bit-exact against the reference's golden vectors;
* GEMV / decode stages: max |err| <= 1e-3 * ||w_row||_1 * ||x||_inf per row (the
  north_star tolerance under fp32 accumulation), tokens and KV words equal;
* BASELINE full sizes: every row computed on the GPU, a sample of rows checked
  against the oracle (the oracle decodes ~10^7 values/s).
"""

import numpy as np
import pytest
import torch

from conftest import FORMAT_TAGS, load_golden
from qgemv_b200 import ops, packs
from test_oracle_cpu import same_bits

pytestmark = pytest.mark.gpu

TOL = 1e-3


def meta_of(g):
    return g["meta"] if g["meta"].size else None


def dev(a, device):
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(device)


def row_tol(port, fmt, payload, meta, x, rows, cols):
    l1 = port.row_l1(fmt, payload, meta, rows, cols)
    return TOL * l1 * float(np.abs(x).max()) + 1e-30


def assert_rows_close(got, want, tol):
    err = np.abs(np.asarray(got, np.float64) - np.asarray(want, np.float64))
    bad = np.nonzero(~(err <= tol))[0]
    assert bad.size == 0, f"{bad.size} rows out of tolerance, first {bad[:5]}: err {err[bad[:5]]} tol {tol[bad[:5]]}"


@pytest.mark.parametrize("fmt", list(FORMAT_TAGS))
@pytest.mark.parametrize("case", ["small", "edge"])
def test_dequant_bit_exact_vs_golden(cuda, fmt, case):
    g = load_golden(fmt, case)
    nblocks = int(g["rows"]) * int(g["cols"]) // 256
    out = ops.dequantize(fmt, dev(g["payload"], cuda), dev(meta_of(g), cuda), 0, nblocks)
    assert same_bits(out.cpu().numpy(), g["dequant"])
    # an offset window
    out = ops.dequantize(fmt, dev(g["payload"], cuda), dev(meta_of(g), cuda), 3, 2)
    assert same_bits(out.cpu().numpy(), g["dequant"][3 * 256 : 5 * 256])


@pytest.mark.parametrize("fmt", list(FORMAT_TAGS))
@pytest.mark.parametrize("case", ["small", "ragged", "edge"])
def test_gemv_vs_golden(cuda, port, fmt, case):
    g = load_golden(fmt, case)
    rows, cols = int(g["rows"]), int(g["cols"])
    y = ops.gemv(fmt, dev(g["payload"], cuda), dev(meta_of(g), cuda), dev(g["x"], cuda), rows, cols)
    tol = row_tol(port, fmt, g["payload"], meta_of(g), g["x"], rows, cols)
    assert_rows_close(y.cpu().numpy(), g["logits"], tol)


COMPAT = {
    packs.Q4K_RAW: "rtxllm_launch_q4k_matvec_decode_warp_broadcast_vec4x4",
    packs.Q4K_PREDECODED: "rtxllm_launch_q4k_matvec_decode_split_predecoded_vec4x4",
    packs.Q4K_HALF: "rtxllm_launch_q4k_matvec_decode_split_half_vec4x4",
    packs.Q4K_COMPACT: "rtxllm_launch_q4k_matvec_decode_split_compact_vec4x4",
    packs.Q4K_NATIVE: "rtxllm_launch_q4k_matvec_decode_split_native_vec4x4",
    packs.Q5K: "rtxllm_launch_q5k_matvec_decode_probe",
    packs.IQ2S: "rtxllm_launch_iq2s_matvec_decode_probe",
    packs.IQ3S: "rtxllm_launch_iq3s_matvec_decode_probe",
}


@pytest.mark.parametrize("fmt", list(FORMAT_TAGS))
@pytest.mark.parametrize("case", ["small", "ragged"])
def test_reference_launchers_logits_kv_token(cuda, port, fmt, case):
    import qgemv_b200

    g = load_golden(fmt, case)
    rows, cols = int(g["rows"]), int(g["cols"])
    payload, meta, x = dev(g["payload"], cuda), dev(meta_of(g), cuda), dev(g["x"], cuda)
    y = torch.full((rows,), float("nan"), device=cuda)
    kv = torch.zeros(g["kv"].size, device=cuda)
    token = torch.tensor([int(g["token_in"])], dtype=torch.int32, device=cuda)
    s = torch.cuda.current_stream().cuda_stream
    name = COMPAT[fmt]
    kvw, pw, ap = g["kv"].size, int(g["page_words"]), int(g["active_pages"])
    if fmt in (packs.Q5K, packs.IQ2S, packs.IQ3S):
        code = qgemv_b200.call(name, payload.data_ptr(), x.data_ptr(), y.data_ptr(), kv.data_ptr(),
                               token.data_ptr(), rows, cols, rows + 5, kvw, pw, ap, s)
    elif fmt == packs.Q4K_RAW:
        code = qgemv_b200.call(name, payload.data_ptr(), x.data_ptr(), y.data_ptr(), kv.data_ptr(),
                               token.data_ptr(), rows, cols, kvw, pw, ap, s)
    else:
        code = qgemv_b200.call(name, payload.data_ptr(), meta.data_ptr(), x.data_ptr(), y.data_ptr(),
                               kv.data_ptr(), token.data_ptr(), rows, cols, kvw, pw, ap, s)
    assert code == 0
    torch.cuda.synchronize()
    tol = row_tol(port, fmt, g["payload"], meta_of(g), g["x"], rows, cols)
    assert_rows_close(y.cpu().numpy(), g["logits"], tol)
    assert int(token.item()) == int(g["token_out"])
    got_kv = kv.cpu().numpy()
    written = g["kv"] != 0
    assert np.array_equal(got_kv != 0, written)
    assert np.all(np.abs(got_kv - g["kv"]) <= tol.max())


def test_rows_limit_caps_launched_rows(cuda, port):
    import qgemv_b200

    pk = packs.synthetic_pack(packs.IQ3S, 40, 1024, seed=7)
    x = packs.synthetic_activation(1024, 7)
    y = torch.full((40,), 12345.0, device=cuda)
    token = torch.zeros(1, dtype=torch.int32, device=cuda)
    p, xd = dev(pk.payload, cuda), dev(x, cuda)
    code = qgemv_b200.call("rtxllm_launch_iq3s_matvec_decode_probe", p.data_ptr(), xd.data_ptr(),
                           y.data_ptr(), None, token.data_ptr(), 40, 1024, 9, 0, 0, 0,
                           torch.cuda.current_stream().cuda_stream)
    assert code == 0
    yc = y.cpu().numpy()
    assert np.all(yc[9:] == 12345.0)
    want = port.matvec(packs.IQ3S, pk.payload, None, x, 40, 1024, 0, 9)
    assert int(token.item()) == (port.argmax(want) + 1) % 32000
    assert_rows_close(yc[:9], want, row_tol(port, packs.IQ3S, pk.payload, None, x, 40, 1024)[:9])


# (5, 8192), (6, 4096), (9, 8192): two or three row passes in all, so the planner shrinks
# the four-pass stage to two (the two-row transposed reduction); (250, 2048): one warp
# per row, four-pass stages, a partial last tile.
SHAPES = [(1, 256), (5, 768), (37, 1792), (64, 3584), (33, 14336), (130, 4096), (17, 28672),
          (3, 33024), (1000, 1024), (5, 8192), (6, 4096), (9, 8192), (250, 2048)]


@pytest.mark.parametrize("fmt", list(FORMAT_TAGS))
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_gemv_shapes_vs_oracle(cuda, port, fmt, rows, cols):
    pk = packs.synthetic_pack(fmt, rows, cols, seed=rows * 31 + cols + fmt)
    x = packs.synthetic_activation(cols, rows + fmt)
    y = ops.gemv(fmt, dev(pk.payload, cuda), dev(pk.meta, cuda), dev(x, cuda), rows, cols)
    want = port.matvec(fmt, pk.payload, pk.meta, x, rows, cols)
    assert_rows_close(y.cpu().numpy(), want, row_tol(port, fmt, pk.payload, pk.meta, x, rows, cols))


@pytest.mark.parametrize("fmt", list(FORMAT_TAGS))
def test_gemv_4096_square_vs_oracle(cuda, port, fmt):
    """BASELINE config 1 shape, every row checked."""
    pk = packs.synthetic_pack(fmt, 4096, 4096, seed=11 + fmt)
    x = packs.synthetic_activation(4096, 11 + fmt)
    y = ops.gemv(fmt, dev(pk.payload, cuda), dev(pk.meta, cuda), dev(x, cuda), 4096, 4096)
    want = port.matvec(fmt, pk.payload, pk.meta, x, 4096, 4096)
    assert_rows_close(y.cpu().numpy(), want, row_tol(port, fmt, pk.payload, pk.meta, x, 4096, 4096))


@pytest.mark.parametrize("fmt", [packs.Q4K_RAW, packs.IQ3S])
@pytest.mark.parametrize("shift", [2, 6])
def test_unaligned_pack_pointer(cuda, port, fmt, shift):
    """Packs that do not start on a 16-B boundary take the all-thread copy path."""
    rows, cols = 50, 2048
    pk = packs.synthetic_pack(fmt, rows, cols, seed=5)
    x = packs.synthetic_activation(cols, 5)
    buf = torch.zeros(pk.payload.size + 64, dtype=torch.uint8, device=cuda)
    buf[shift : shift + pk.payload.size] = dev(pk.payload, cuda)
    y = ops.gemv(fmt, buf[shift:], None, dev(x, cuda), rows, cols)
    want = port.matvec(fmt, pk.payload, None, x, rows, cols)
    assert_rows_close(y.cpu().numpy(), want, row_tol(port, fmt, pk.payload, None, x, rows, cols))


FULL = [(14336, 4096), (4096, 14336), (128256, 8192)]


@pytest.mark.parametrize("fmt", [packs.Q4K_RAW, packs.Q4K_PREDECODED, packs.Q5K, packs.IQ2S, packs.IQ3S])
@pytest.mark.parametrize("rows,cols", FULL)
def test_full_size_sampled_rows(cuda, port, fmt, rows, cols):
    """BASELINE config 2 shapes: full GPU GEMV, oracle on 3 row windows."""
    pk = packs.synthetic_pack(fmt, rows, cols, seed=rows + cols + fmt)
    x = packs.synthetic_activation(cols, fmt)
    y = ops.gemv(fmt, dev(pk.payload, cuda), dev(pk.meta, cuda), dev(x, cuda), rows, cols)
    yc = y.cpu().numpy()
    assert np.all(np.isfinite(yc))
    for r0 in (0, rows // 2 - 7, rows - 16):
        want = port.matvec(fmt, pk.payload, pk.meta, x, rows, cols, r0, r0 + 16)
        sub_payload, sub_meta = _row_slice(pk, r0, r0 + 16)
        tol = row_tol(port, fmt, sub_payload, sub_meta, x, 16, cols)
        assert_rows_close(yc[r0 : r0 + 16], want, tol)


def _row_slice(pk, r0, r1):
    bpr = pk.cols // 256
    pb, mb = packs.payload_bytes_per_block(pk.fmt), packs.meta_bytes_per_block(pk.fmt)
    payload = pk.payload[r0 * bpr * pb : r1 * bpr * pb]
    meta = None if pk.meta is None else pk.meta[r0 * bpr * mb : r1 * bpr * mb]
    return payload, meta


def test_argmax_ties_and_nan(cuda, port):
    rng = np.random.default_rng(3)
    for n in (1, 7, 1000, 4099, 128256):
        v = rng.standard_normal(n).astype(np.float32)
        if n > 10:
            v[n // 3] = v[n // 5] = v.max() + 1.0   # tie: the lower index must win
            v[n // 7] = np.nan
        for add, off, mod in ((1, 1, 32000), (0, 5, 32000), (0, 0, 1000)):
            tok0 = 1234
            t = torch.tensor([tok0], dtype=torch.int32, device=cuda)
            ops.argmax_token(dev(v, cuda), t, off, add, mod)
            want = (port.argmax(v) + off + (tok0 if add else 0)) % mod
            assert int(t.item()) == want
    # all -inf / NaN: index 0, like the reference's running best of -FLT_MAX
    v = np.full(300, -np.inf, np.float32)
    v[5] = np.nan
    t = torch.tensor([0], dtype=torch.int32, device=cuda)
    ops.argmax_token(dev(v, cuda), t, 0, 0, 32000)
    assert int(t.item()) == 0


def test_output_token_sample_launcher(cuda, port):
    import qgemv_b200

    v = np.random.default_rng(4).standard_normal(128256).astype(np.float32)
    t = torch.tensor([99], dtype=torch.int32, device=cuda)
    vd = dev(v, cuda)
    assert qgemv_b200.call("rtxllm_launch_output_token_sample", vd.data_ptr(), t.data_ptr(),
                           128256, 32000, 7, torch.cuda.current_stream().cuda_stream) == 0
    assert int(t.item()) == (port.argmax(v) + 7) % 32000


def test_feedback_launchers_vs_golden(cuda):
    import qgemv_b200
    from conftest import GOLDEN

    g = np.load(GOLDEN / "golden_feedback.npz")
    logits = dev(g["logits"], cuda)
    n = g["logits"].size
    s = torch.cuda.current_stream().cuda_stream
    for eps_tag, eps in (("e6", 1e-6), ("e5", 1e-5)):
        for kind in range(6):
            for acc in ((0, 1) if kind >= 4 else (0,)):
                key = f"k{kind}_{eps_tag}_a{acc}"
                act = dev(g[f"{key}_act_in"], cuda)
                cache_in = g[f"{key}_cache_in"]
                cols, cc = act.numel(), cache_in.size
                if kind == 2:
                    cache = torch.zeros(cols, device=cuda)
                    cache[:cc] = dev(cache_in, cuda)
                else:
                    cache = dev(cache_in, cuda)
                if kind == 0:
                    code = qgemv_b200.call("rtxllm_launch_rmsnorm_feedback", logits.data_ptr(), act.data_ptr(), n, cols, eps, s)
                elif kind == 1:
                    code = qgemv_b200.call("rtxllm_launch_silu_rmsnorm_feedback", logits.data_ptr(), act.data_ptr(), n, cols, eps, s)
                elif kind == 2:
                    code = qgemv_b200.call("rtxllm_launch_rmsnorm_feedback_with_silu_cache", logits.data_ptr(), act.data_ptr(), cache.data_ptr(), n, cols, eps, s)
                elif kind == 3:
                    code = qgemv_b200.call("rtxllm_launch_gated_silu_rmsnorm_feedback", logits.data_ptr(), cache.data_ptr(), act.data_ptr(), n, cc, cols, eps, s)
                elif kind == 4:
                    code = qgemv_b200.call("rtxllm_launch_rmsnorm_cache", logits.data_ptr(), cache.data_ptr(), n, cc, eps, acc, s)
                else:
                    code = qgemv_b200.call("rtxllm_launch_rmsnorm_silu_cache", logits.data_ptr(), cache.data_ptr(), n, cc, eps, acc, s)
                assert code == 0
                np.testing.assert_allclose(act.cpu().numpy(), g[f"{key}_act"], rtol=2e-6, atol=2e-6)
                want_cache = g[f"{key}_cache"]
                np.testing.assert_allclose(cache.cpu().numpy()[: want_cache.size], want_cache, rtol=2e-6, atol=2e-6)


def test_gated_product_launcher_vs_golden(cuda):
    """rtxllm_launch_rmsnorm_cache_and_gated_product (decode_kernels.cu:263-289; the mixed
    runner's finalising FFN edge, main.cpp:4113) against the reference's CPU twin: up cache
    overwritten or accumulated, activation = gate x up."""
    import qgemv_b200
    from conftest import GOLDEN

    g = np.load(GOLDEN / "golden_feedback.npz")
    logits = dev(g["logits"], cuda)
    n = g["logits"].size
    s = torch.cuda.current_stream().cuda_stream
    for eps_tag, eps in (("e6", 1e-6), ("e5", 1e-5)):
        for acc in (0, 1):
            key = f"k6_{eps_tag}_a{acc}"
            gate, up, act = dev(g[f"{key}_gate"], cuda), dev(g[f"{key}_up_in"], cuda), dev(g[f"{key}_act_in"], cuda)
            cols = act.numel()
            code = qgemv_b200.call("rtxllm_launch_rmsnorm_cache_and_gated_product", logits.data_ptr(),
                                   gate.data_ptr(), up.data_ptr(), act.data_ptr(), n, up.numel(), cols,
                                   eps, acc, s)
            assert code == 0
            np.testing.assert_allclose(up.cpu().numpy(), g[f"{key}_up"], rtol=2e-6, atol=2e-6, err_msg=key)
            np.testing.assert_allclose(act.cpu().numpy(), g[f"{key}_act"], rtol=2e-6, atol=2e-6, err_msg=key)
    # validation as decode_kernels.cu:3227-3229: zero cache or output columns are
    # cudaErrorInvalidValue; zero rows launch a kernel that returns at once (nothing written)
    up0 = torch.ones(4, device=cuda)
    call = lambda rows, cc, oc: qgemv_b200.call(  # noqa: E731
        "rtxllm_launch_rmsnorm_cache_and_gated_product", logits.data_ptr(), up0.data_ptr(),
        up0.data_ptr(), up0.data_ptr(), rows, cc, oc, 1e-6, 0, s)
    assert call(n, 0, 4) == 1 and call(n, 4, 0) == 1
    assert call(0, 4, 4) == 0
    torch.cuda.synchronize()
    assert torch.equal(up0, torch.ones(4, device=cuda))


def test_batched_vs_oracle(cuda, port):
    for fmt in (packs.Q4K_RAW, packs.IQ2S):
        rows, cols, batch = 96, 2048, 5
        pk = packs.synthetic_pack(fmt, rows, cols, seed=17)
        x = packs.synthetic_activation(cols, 17, batch=batch)
        y = ops.gemv_batched(fmt, dev(pk.payload, cuda), dev(pk.meta, cuda), dev(x, cuda), rows, cols)
        tol = row_tol(port, fmt, pk.payload, pk.meta, np.abs(x).max(axis=0), rows, cols)
        for b in range(batch):
            want = port.matvec(fmt, pk.payload, pk.meta, x[b], rows, cols)
            assert_rows_close(y[b].cpu().numpy(), want, tol)


def test_error_word_is_clear(cuda):
    torch.cuda.synchronize()
    assert ops.get_error() == 0


@pytest.mark.parametrize("fmt", list(FORMAT_TAGS))
@pytest.mark.parametrize("rows,cols", [(37, 1792), (300, 4096), (64, 14336)])
def test_prepared_activation_gemv_vs_oracle(cuda, port, fmt, rows, cols):
    """qg_act_prepare once, then qg_gemv_act: same tolerance as qg_gemv."""
    pk = packs.synthetic_pack(fmt, rows, cols, seed=rows + 7 * cols + fmt)
    x = packs.synthetic_activation(cols, fmt + 3)
    xd = dev(x, cuda)
    act = ops.act_prepare(xd)
    y = ops.gemv_act(fmt, dev(pk.payload, cuda), dev(pk.meta, cuda), xd, act, rows, cols)
    want = port.matvec(fmt, pk.payload, pk.meta, x, rows, cols)
    assert_rows_close(y.cpu().numpy(), want, row_tol(port, fmt, pk.payload, pk.meta, x, rows, cols))
    y2 = ops.gemv(fmt, dev(pk.payload, cuda), dev(pk.meta, cuda), xd, rows, cols)
    assert torch.equal(y, y2)  # same planes, same arithmetic


def test_activation_extremes(cuda, port):
    """x with zeros, one huge value and tiny values: the per-32-column scale handles it."""
    rows, cols = 40, 2048
    pk = packs.synthetic_pack(packs.Q4K_RAW, rows, cols, seed=3)
    x = packs.synthetic_activation(cols, 3)
    x[:64] = 0.0
    x[100] = 3.0e4
    x[200:260] *= 1e-6
    y = ops.gemv(packs.Q4K_RAW, dev(pk.payload, cuda), None, dev(x, cuda), rows, cols)
    want = port.matvec(packs.Q4K_RAW, pk.payload, None, x, rows, cols)
    assert_rows_close(y.cpu().numpy(), want, row_tol(port, packs.Q4K_RAW, pk.payload, None, x, rows, cols))
