"""CPU restatement of the tensor-parallel decode step -- TEST INFRASTRUCTURE ONLY.

The reference has no attention core and no multi-GPU path (its attention kernels are
synthetic surrogates, runtime/kernels/decode/decode_kernels.cu:311-1136), so this is
a plain restatement of the Llama-style decode step the decoder implements:
GEMVs through the C oracle (oracle/qoracle.c, pinned to the reference), the rest in
numpy fp32 / fp64:

  h = x / sqrt(mean(x^2) + eps) * w_attn
  q, k, v = Wq h, Wk h, Wv h;  RoPE on q and k (adjacent pairs, angle pos * base^(-2i/d))
  cache[pos] = fp16(k), fp16(v);  per q head: softmax(q . K[0..pos] / sqrt(d)) . V
  x1 = x + Wo attn;  h2 = rmsnorm(x1) * w_ffn;  x2 = x1 + Wd (silu(Wg h2) * (Wu h2))
  after the layers: logits = head (rmsnorm(x) * w_final); token = argmax (lowest index)

`step(..., tp, rank)` computes what one rank contributes (its shards, partial Wo/Wd
products with the residual on rank 0), with `allreduce` / `allgather` callbacks, so the
same code checks the sharding arithmetic on CPU ranks (gloo) and, with tp=1, the whole
step.
"""

from __future__ import annotations

import numpy as np


def wrmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = x.astype(np.float32)
    ms = np.float32(np.sum(x.astype(np.float64) ** 2) / x.size)
    return (x / np.sqrt(ms + np.float32(eps)) * w).astype(np.float32)


def rope(vec: np.ndarray, heads: int, pos: int, base: float, d: int = 128) -> np.ndarray:
    out = vec.astype(np.float64).reshape(heads, d).copy()
    j = np.arange(d // 2, dtype=np.float64)
    ang = pos * base ** (-2.0 * j / d)
    c, s = np.cos(ang), np.sin(ang)
    a, b = out[:, 0::2].copy(), out[:, 1::2].copy()
    out[:, 0::2] = a * c - b * s
    out[:, 1::2] = a * s + b * c
    return out.reshape(-1).astype(np.float32)


def attention(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, n_q: int, n_kv: int, ctx_len: int,
              d: int = 128) -> np.ndarray:
    group = n_q // n_kv
    out = np.empty((n_q, d), np.float64)
    qh = q.astype(np.float64).reshape(n_q, d) / np.sqrt(d)
    for h in range(n_q):
        K = kc[h // group, :ctx_len].astype(np.float64)
        V = vc[h // group, :ctx_len].astype(np.float64)
        s = K @ qh[h]
        p = np.exp(s - s.max())
        out[h] = (p / p.sum()) @ V
    return out.reshape(-1).astype(np.float32)


def silu_gate(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g64 = g.astype(np.float64)
    return (g64 / (1.0 + np.exp(-g64)) * u).astype(np.float32)


def argmax_first(v: np.ndarray) -> int:
    return int(np.argmax(v))  # first index of the maximum


def step(port, spec, weights: dict, x: np.ndarray, pos: int, tp: int = 1, rank: int = 0,
         allreduce=None, allgather=None):
    """One decode step of rank `rank` of `tp` over `weights` (rank_weights layout; the
    caches are updated in place).  Returns (token, final hidden state)."""
    allreduce = allreduce or (lambda a: a)
    nq, nkv = spec.n_q_heads // tp, spec.n_kv_heads // tp

    def mv(pk, vec):
        return port.matvec(pk.fmt, pk.payload, pk.meta, vec, pk.rows, pk.cols)

    cur = x.astype(np.float32)
    for L in weights["layers"]:
        h = wrmsnorm(cur, L["attn_norm"], spec.eps)
        q = rope(mv(L["wq"], h), nq, pos, spec.rope_base)
        k = rope(mv(L["wk"], h), nkv, pos, spec.rope_base)
        v = mv(L["wv"], h)
        L["k_cache"][:, pos, :] = k.reshape(nkv, -1).astype(np.float16)
        L["v_cache"][:, pos, :] = v.reshape(nkv, -1).astype(np.float16)
        attn = attention(q, L["k_cache"], L["v_cache"], nq, nkv, pos + 1)
        o = mv(L["wo"], attn)
        x1 = allreduce(o + cur if rank == 0 else o)
        h2 = wrmsnorm(x1, L["ffn_norm"], spec.eps)
        a = silu_gate(mv(L["wg"], h2), mv(L["wu"], h2))
        dn = mv(L["wd"], a)
        cur = allreduce(dn + x1 if rank == 0 else dn)
    hf = wrmsnorm(cur, weights["final_norm"], spec.eps)
    logits = mv(weights["head"], hf)
    i = argmax_first(logits)
    cand = (float(logits[i]), i + weights["shard"]["vocab_offset"])
    cands = allgather(cand) if allgather else [cand]
    best = max(cands, key=lambda c: (c[0], -c[1]))
    return best[1], cur
