"""Tensor-parallel decode step on top of qg_decoder_*.

* `ModelSpec` -- architecture and pack formats (defaults: the 70B-class config).
* `HostModel` -- seeded global weights on the host (numpy), for parity tests at
  small sizes; `rank_weights(model, rank, tp)` cuts one rank's shards out of it the
  way the decoder expects them (row shards of Wq/Wk/Wv/Wg/Wu/head, column shards of
  Wo/Wd on 256-column block boundaries, the rank's kv heads of the cache).
* `synthetic_rank_weights(spec, rank, tp, ...)` -- one seeded global model drawn
  directly on the GPU, cut into the same shard shapes (full-size benchmark: ~31 GB of
  packs at tp=1); identical weights at every tensor-parallel degree.
* `Decoder` -- one rank's qg_decoder plus its workspace.
"""

from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_uint32, c_void_p
from dataclasses import dataclass, field

import numpy as np
import torch

from . import packs
from ._lib import check


@dataclass
class ModelSpec:
    layers: int = 80
    hidden: int = 8192
    n_q_heads: int = 64
    n_kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 28672
    vocab: int = 128256
    ctx_max: int = 4096
    eps: float = 1e-5
    rope_base: float = 500000.0
    attn_fmt: int = packs.IQ3S
    ffn_fmt: int = packs.IQ2S
    down_fmt: int = packs.Q5K
    head_fmt: int = packs.Q4K_RAW

    @property
    def q_rows(self) -> int:
        return self.n_q_heads * self.head_dim

    @property
    def kv_rows(self) -> int:
        return self.n_kv_heads * self.head_dim

    def layer_weight_bytes(self) -> int:
        h, q, kv, f = self.hidden, self.q_rows, self.kv_rows, self.ffn
        return (packs.pack_bytes(self.attn_fmt, q, h) + 2 * packs.pack_bytes(self.attn_fmt, kv, h)
                + packs.pack_bytes(self.attn_fmt, h, q) + 2 * packs.pack_bytes(self.ffn_fmt, f, h)
                + packs.pack_bytes(self.down_fmt, h, f))

    def weight_bytes(self) -> int:
        return self.layers * self.layer_weight_bytes() + packs.pack_bytes(self.head_fmt, self.vocab, self.hidden)

    def kv_bytes_read(self, ctx_len: int) -> int:
        return self.layers * 2 * self.n_kv_heads * ctx_len * self.head_dim * 2


class DecoderDims(ctypes.Structure):
    _fields_ = [(n, c_uint32) for n in ("layers", "hidden", "n_q_heads", "n_kv_heads", "head_dim",
                                         "ffn", "vocab", "ctx_max")] + [
        ("eps", c_float), ("rope_base", c_float),
        ("attn_fmt", c_int), ("ffn_fmt", c_int), ("down_fmt", c_int), ("head_fmt", c_int),
        ("tp_rank", c_uint32), ("tp_size", c_uint32), ("collective", c_uint32)]


LAYER_MATS = ("wq", "wk", "wv", "wo", "wg", "wu", "wd")


class DecoderLayerC(ctypes.Structure):
    _fields_ = ([("attn_norm", c_void_p), ("ffn_norm", c_void_p)]
                + [(n, c_void_p) for n in LAYER_MATS]
                + [(n + "_meta", c_void_p) for n in LAYER_MATS]
                + [("k_cache", c_void_p), ("v_cache", c_void_p)])


COLLECTIVE_NVLINK = 0  # exchanges fused into the GEMVs over NVLink peer memory
COLLECTIVE_NCCL = 1    # the same exchange words moved by ncclAllGather between the kernels


def dims_struct(spec: ModelSpec, rank: int, tp: int, collective: int = COLLECTIVE_NVLINK) -> DecoderDims:
    return DecoderDims(spec.layers, spec.hidden, spec.n_q_heads, spec.n_kv_heads, spec.head_dim,
                       spec.ffn, spec.vocab, spec.ctx_max, spec.eps, spec.rope_base,
                       spec.attn_fmt, spec.ffn_fmt, spec.down_fmt, spec.head_fmt, rank, tp, collective)


def shard_shape(spec: ModelSpec, rank: int, tp: int) -> dict:
    vals = [c_uint32() for _ in range(5)]
    d = dims_struct(spec, rank, tp)
    check("qg_decoder_shard", ctypes.byref(d), *[ctypes.byref(v) for v in vals])
    q, kv, f, vr, vo = (v.value for v in vals)
    return dict(q_rows=q, kv_rows=kv, ffn_rows=f, vocab_rows=vr, vocab_offset=vo)


# --------------------------------------------------------------------------- shards

def rows_of(pk: packs.Pack, r0: int, r1: int) -> packs.Pack:
    bpr = pk.cols // 256
    pb, mb = packs.payload_bytes_per_block(pk.fmt), packs.meta_bytes_per_block(pk.fmt)
    payload = pk.payload[r0 * bpr * pb: r1 * bpr * pb].copy()
    meta = None if pk.meta is None else pk.meta[r0 * bpr * mb: r1 * bpr * mb].copy()
    return packs.Pack(pk.fmt, r1 - r0, pk.cols, payload, meta)


def cols_of(pk: packs.Pack, c0: int, c1: int) -> packs.Pack:
    assert c0 % 256 == 0 and c1 % 256 == 0
    bpr = pk.cols // 256
    b0, b1 = c0 // 256, c1 // 256
    pb, mb = packs.payload_bytes_per_block(pk.fmt), packs.meta_bytes_per_block(pk.fmt)
    payload = pk.payload.reshape(pk.rows, bpr, pb)[:, b0:b1, :].copy().reshape(-1)
    meta = None if pk.meta is None else pk.meta.reshape(pk.rows, bpr, mb)[:, b0:b1, :].copy().reshape(-1)
    return packs.Pack(pk.fmt, pk.rows, c1 - c0, payload, meta)


@dataclass
class HostModel:
    spec: ModelSpec
    layers: list = field(default_factory=list)      # dicts: attn_norm, ffn_norm, w*, k_cache, v_cache
    final_norm: np.ndarray | None = None
    head: packs.Pack | None = None

    @staticmethod
    def synthetic(spec: ModelSpec, seed: int = 0) -> "HostModel":
        rng = np.random.Generator(np.random.PCG64(seed))
        m = HostModel(spec)
        shapes = dict(wq=(spec.q_rows, spec.hidden), wk=(spec.kv_rows, spec.hidden),
                      wv=(spec.kv_rows, spec.hidden), wo=(spec.hidden, spec.q_rows),
                      wg=(spec.ffn, spec.hidden), wu=(spec.ffn, spec.hidden),
                      wd=(spec.hidden, spec.ffn))
        fmts = dict(wq=spec.attn_fmt, wk=spec.attn_fmt, wv=spec.attn_fmt, wo=spec.attn_fmt,
                    wg=spec.ffn_fmt, wu=spec.ffn_fmt, wd=spec.down_fmt)
        for l in range(spec.layers):
            layer = dict(attn_norm=(1 + 0.02 * rng.standard_normal(spec.hidden)).astype(np.float32),
                         ffn_norm=(1 + 0.02 * rng.standard_normal(spec.hidden)).astype(np.float32))
            for i, n in enumerate(LAYER_MATS):
                layer[n] = packs.synthetic_pack(fmts[n], *shapes[n], seed=seed * 1000 + l * 10 + i)
            shape = (spec.n_kv_heads, spec.ctx_max, spec.head_dim)
            layer["k_cache"] = rng.standard_normal(shape).astype(np.float16)
            layer["v_cache"] = rng.standard_normal(shape).astype(np.float16)
            m.layers.append(layer)
        m.final_norm = (1 + 0.02 * rng.standard_normal(spec.hidden)).astype(np.float32)
        m.head = packs.synthetic_pack(spec.head_fmt, spec.vocab, spec.hidden, seed=seed * 1000 + 999)
        return m


def rank_weights(model: HostModel, rank: int, tp: int) -> dict:
    """This rank's shards of a host model (numpy)."""
    spec = model.spec
    sh = shard_shape(spec, rank, tp)
    q0, q1 = rank * sh["q_rows"], (rank + 1) * sh["q_rows"]
    k0, k1 = rank * sh["kv_rows"], (rank + 1) * sh["kv_rows"]
    f0, f1 = rank * sh["ffn_rows"], (rank + 1) * sh["ffn_rows"]
    h0, h1 = rank * (spec.n_kv_heads // tp), (rank + 1) * (spec.n_kv_heads // tp)
    layers = []
    for L in model.layers:
        layers.append(dict(
            attn_norm=L["attn_norm"], ffn_norm=L["ffn_norm"],
            wq=rows_of(L["wq"], q0, q1), wk=rows_of(L["wk"], k0, k1), wv=rows_of(L["wv"], k0, k1),
            wo=cols_of(L["wo"], q0, q1), wg=rows_of(L["wg"], f0, f1), wu=rows_of(L["wu"], f0, f1),
            wd=cols_of(L["wd"], f0, f1),
            k_cache=L["k_cache"][h0:h1].copy(), v_cache=L["v_cache"][h0:h1].copy()))
    v0 = sh["vocab_offset"]
    return dict(layers=layers, final_norm=model.final_norm,
                head=rows_of(model.head, v0, v0 + sh["vocab_rows"]), shard=sh)


def _gpu_pack(fmt: int, rows: int, cols: int, gen: torch.Generator, device) -> tuple:
    """Seeded synthetic pack drawn on the GPU (BASELINE distributions)."""
    nblocks = rows * (cols // 256)
    pb = packs.payload_bytes_per_block(fmt)
    payload = torch.randint(0, 256, (nblocks, pb), dtype=torch.uint8, device=device, generator=gen)
    nscale = 2 if fmt in (packs.Q4K_RAW, packs.Q5K) else 1
    d = torch.empty(nblocks, nscale, device=device).uniform_(1e-3, 1e-2, generator=gen).half()
    payload[:, : 2 * nscale] = d.view(torch.uint8).view(nblocks, 2 * nscale)
    if fmt in packs.SPLIT_POLICY:
        raise ValueError("GPU-side synthetic packs are raw-block formats only")
    return payload.view(-1), None


def _rows_view(p: tuple, fmt: int, cols: int, r0: int, r1: int) -> tuple:
    payload, _ = p
    row = (cols // 256) * packs.payload_bytes_per_block(fmt)
    return payload.view(-1, row)[r0:r1].reshape(-1), None


def _cols_copy(p: tuple, fmt: int, rows: int, cols: int, c0: int, c1: int) -> tuple:
    payload, _ = p
    pb = packs.payload_bytes_per_block(fmt)
    blocks = payload.view(rows, cols // 256, pb)[:, c0 // 256: c1 // 256, :]
    return blocks.contiguous().view(-1), None


def synthetic_rank_weights(spec: ModelSpec, rank: int, tp: int, device, seed: int = 0,
                           keep_full: bool = False) -> dict:
    """This rank's shards (shapes as rank_weights) of one seeded global model drawn on the
    GPU: every rank draws the same global tensors in the same order from a generator with
    the same seed and keeps its own rows / columns / kv heads, so the shards of every
    tensor-parallel degree are cut from identical weights (the step is comparable across
    degrees).  With keep_full the global weights are returned as well (`full`, the tp=1
    shards; the rank's shards are then views into them where they are contiguous)."""
    sh = shard_shape(spec, rank, tp)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed * 7919 + 17)
    q, kv, f = sh["q_rows"], sh["kv_rows"], sh["ffn_rows"]
    q0, k0, f0 = rank * q, rank * kv, rank * f
    h0, h1 = rank * (spec.n_kv_heads // tp), (rank + 1) * (spec.n_kv_heads // tp)
    full_shapes = dict(wq=(spec.attn_fmt, spec.q_rows, spec.hidden),
                       wk=(spec.attn_fmt, spec.kv_rows, spec.hidden),
                       wv=(spec.attn_fmt, spec.kv_rows, spec.hidden),
                       wo=(spec.attn_fmt, spec.hidden, spec.q_rows),
                       wg=(spec.ffn_fmt, spec.ffn, spec.hidden),
                       wu=(spec.ffn_fmt, spec.ffn, spec.hidden),
                       wd=(spec.down_fmt, spec.hidden, spec.ffn))
    row_cut = dict(wq=(q0, q0 + q), wk=(k0, k0 + kv), wv=(k0, k0 + kv), wg=(f0, f0 + f), wu=(f0, f0 + f))
    col_cut = dict(wo=(q0, q0 + q), wd=(f0, f0 + f))
    layers, full_layers = [], []
    for _ in range(spec.layers):
        L = {"attn_norm": 1 + 0.02 * torch.randn(spec.hidden, device=device, generator=gen),
             "ffn_norm": 1 + 0.02 * torch.randn(spec.hidden, device=device, generator=gen)}
        F = dict(L)
        for n, (fmt, r, c) in full_shapes.items():
            full = _gpu_pack(fmt, r, c, gen, device)
            F[n] = full
            if n in row_cut:
                part = _rows_view(full, fmt, c, *row_cut[n])
                L[n] = part if keep_full else (part[0].clone(), None)
            else:
                L[n] = _cols_copy(full, fmt, r, c, *col_cut[n])
        cache = (spec.n_kv_heads, spec.ctx_max, spec.head_dim)
        kc = torch.randn(cache, device=device, generator=gen).half()
        vc = torch.randn(cache, device=device, generator=gen).half()
        F["k_cache"], F["v_cache"] = kc, vc
        L["k_cache"] = kc[h0:h1] if keep_full else kc[h0:h1].clone()
        L["v_cache"] = vc[h0:h1] if keep_full else vc[h0:h1].clone()
        layers.append(L)
        if keep_full:
            full_layers.append(F)
    final_norm = 1 + 0.02 * torch.randn(spec.hidden, device=device, generator=gen)
    head_full = _gpu_pack(spec.head_fmt, spec.vocab, spec.hidden, gen, device)
    v0 = sh["vocab_offset"]
    head = _rows_view(head_full, spec.head_fmt, spec.hidden, v0, v0 + sh["vocab_rows"])
    out = dict(layers=layers, final_norm=final_norm,
               head=head if keep_full else (head[0].clone(), None), shard=sh, on_device=True)
    if keep_full:
        out["full"] = dict(layers=full_layers, final_norm=final_norm, head=head_full,
                           shard=shard_shape(spec, 0, 1), on_device=True)
    return out


# --------------------------------------------------------------------------- runtime

class Decoder:
    """One rank's decoder: device-resident shards, workspace and the qg_decoder."""

    def __init__(self, spec: ModelSpec, weights: dict, rank: int = 0, tp: int = 1,
                 nccl_id: bytes | None = None, device="cuda", collective: int = COLLECTIVE_NVLINK,
                 exchange: torch.Tensor | None = None):
        self.spec, self.rank, self.tp = spec, rank, tp
        self.device = torch.device(device)
        self._keep = []
        dev = self.device

        def t(a):
            if isinstance(a, torch.Tensor):
                return a
            return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

        def pack_ptrs(p):
            if isinstance(p, tuple):  # (payload tensor, meta tensor or None) on the device
                payload, meta = p
            else:
                payload = t(p.payload)
                meta = None if p.meta is None else t(p.meta)
            self._keep.append((payload, meta))
            return payload.data_ptr(), (None if meta is None else meta.data_ptr())

        arr = (DecoderLayerC * spec.layers)()
        self.caches = []
        for i, L in enumerate(weights["layers"]):
            an, fn = t(L["attn_norm"]).float().contiguous(), t(L["ffn_norm"]).float().contiguous()
            kc, vc = t(L["k_cache"]).contiguous(), t(L["v_cache"]).contiguous()
            self._keep += [an, fn]
            self.caches.append((kc, vc))
            fields = dict(attn_norm=an.data_ptr(), ffn_norm=fn.data_ptr(),
                          k_cache=kc.data_ptr(), v_cache=vc.data_ptr())
            for n in LAYER_MATS:
                p, m = pack_ptrs(L[n])
                fields[n] = p
                fields[n + "_meta"] = m
            arr[i] = DecoderLayerC(**fields)
        self.layers_c = arr
        fnorm = t(weights["final_norm"]).float().contiguous()
        self._keep.append(fnorm)
        head_p, head_m = pack_ptrs(weights["head"])
        self.vocab_rows = (weights.get("shard") or {}).get("vocab_rows",
                                                           getattr(weights["head"], "rows", None))
        self.dims = dims_struct(spec, rank, tp, collective)
        n = ctypes.c_size_t(0)
        check("qg_decoder_workspace_bytes", ctypes.byref(self.dims), ctypes.byref(n))
        self.workspace = torch.empty(n.value, dtype=torch.uint8, device=dev)
        self.token = torch.zeros(1, dtype=torch.int32, device=dev)
        self.handle = c_void_p(None)
        idbuf = None
        if tp > 1:
            idbuf = ctypes.create_string_buffer(bytes(nccl_id), 128)
        if exchange is None:
            check("qg_decoder_create", ctypes.byref(self.dims), arr, fnorm.data_ptr(), head_p, head_m,
                  self.workspace.data_ptr(), idbuf, ctypes.byref(self.handle))
        else:  # caller-owned exchange region (qg_decoder_create_in)
            self._keep.append(exchange)
            check("qg_decoder_create_in", ctypes.byref(self.dims), arr, fnorm.data_ptr(), head_p,
                  head_m, self.workspace.data_ptr(), exchange.data_ptr(), idbuf,
                  ctypes.byref(self.handle))

    def step(self, x: torch.Tensor, pos: int, stream=None) -> torch.Tensor:
        s = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        check("qg_decoder_step", self.handle, x.data_ptr(), pos, self.token.data_ptr(), s)
        return self.token

    def step_at(self, x: torch.Tensor, pos_dev: torch.Tensor, ctx_bucket: int, advance: bool = True,
                stream=None) -> torch.Tensor:
        """The step with the position read from pos_dev (a 1-element int32 device tensor)."""
        s = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        check("qg_decoder_step_at", self.handle, x.data_ptr(), pos_dev.data_ptr(), ctx_bucket,
              1 if advance else 0, self.token.data_ptr(), s)
        return self.token

    def exchange_bytes(self) -> int:
        n = ctypes.c_size_t(0)
        check("qg_decoder_exchange_bytes", ctypes.byref(self.dims), ctypes.byref(n))
        return n.value

    def hidden(self) -> torch.Tensor:
        hp, lp = c_void_p(), c_void_p()
        check("qg_decoder_views", self.handle, ctypes.byref(hp), ctypes.byref(lp))
        off = hp.value - self.workspace.data_ptr()
        return self.workspace[off: off + 4 * self.spec.hidden].view(torch.float32)

    STAGES = ("layer_input", "q", "k", "v", "attn", "x1", "g", "u", "a", "hidden", "logits")

    def stage_views(self) -> dict:
        """The last step's vectors of its last layer (qg_decoder_stage_buffers) as float32
        views of the workspace; the layer input is None when it is the caller's x (a
        one-layer model)."""
        raw = (c_void_p * len(self.STAGES))()
        check("qg_decoder_stage_buffers", self.handle, ctypes.byref(raw))
        s = self.spec
        q_rows = s.n_q_heads // self.tp * s.head_dim
        kv_rows = s.n_kv_heads // self.tp * s.head_dim
        ffn = s.ffn // self.tp
        sizes = dict(layer_input=s.hidden, q=q_rows, k=kv_rows, v=kv_rows, attn=q_rows,
                     x1=s.hidden, g=ffn, u=ffn, a=ffn, hidden=s.hidden,
                     logits=self.vocab_rows)
        base, end = self.workspace.data_ptr(), self.workspace.data_ptr() + self.workspace.numel()
        out = {}
        for name, ptr in zip(self.STAGES, raw):
            n = sizes[name]
            if ptr is None or not (base <= ptr < end) or n is None:
                out[name] = None
                continue
            off = ptr - base
            out[name] = self.workspace[off: off + 4 * n].view(torch.float32)
        return out

    def close(self) -> None:
        if self.handle.value:
            check("qg_decoder_destroy", self.handle)
            self.handle = c_void_p(None)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def exchange_bytes(spec: ModelSpec, rank: int, tp: int) -> int:
    n = ctypes.c_size_t(0)
    d = dims_struct(spec, rank, tp)
    check("qg_decoder_exchange_bytes", ctypes.byref(d), ctypes.byref(n))
    return n.value


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    check("qg_nccl_unique_id", buf)
    return buf.raw
