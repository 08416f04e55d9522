"""Mixed-format layer slice on top of qg_layer_slice_forward.

`LayerSlice` holds seeded synthetic packs for one Llama-style slice (RMSNorm weights
N(1, 0.02), Q/K/V/O in attn_fmt, gate/up in ffn_fmt, down in down_fmt), resident on
the GPU, plus a caller-owned workspace.  Host copies of the packs are kept when
`keep_host` is set (tests compare against the CPU oracle).
"""

from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_uint32, c_void_p

import numpy as np
import torch

from . import packs
from ._lib import check


class LayerSliceC(ctypes.Structure):
    _fields_ = [
        ("hidden", c_uint32), ("q_rows", c_uint32), ("kv_rows", c_uint32), ("ffn", c_uint32),
        ("eps", c_float), ("norm_weight", c_void_p),
        ("attn_fmt", c_int), ("wq", c_void_p), ("wk", c_void_p), ("wv", c_void_p), ("wo", c_void_p),
        ("wq_meta", c_void_p), ("wk_meta", c_void_p), ("wv_meta", c_void_p), ("wo_meta", c_void_p),
        ("ffn_fmt", c_int), ("wg", c_void_p), ("wu", c_void_p), ("wg_meta", c_void_p), ("wu_meta", c_void_p),
        ("down_fmt", c_int), ("wd", c_void_p), ("wd_meta", c_void_p),
    ]


class LayerSliceViews(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in ("h", "q", "k", "v", "o", "gate", "up", "act")]


NAMES = ("wq", "wk", "wv", "wo", "wg", "wu", "wd")


class LayerSlice:
    def __init__(self, hidden=4096, q_rows=4096, kv_rows=1024, ffn=14336,
                 attn_fmt=packs.IQ3S, ffn_fmt=packs.IQ2S, down_fmt=packs.Q5K,
                 eps=1e-5, seed=0, device="cuda", keep_host=False):
        self.dims = dict(hidden=hidden, q_rows=q_rows, kv_rows=kv_rows, ffn=ffn)
        self.fmts = dict(wq=attn_fmt, wk=attn_fmt, wv=attn_fmt, wo=attn_fmt,
                         wg=ffn_fmt, wu=ffn_fmt, wd=down_fmt)
        shapes = dict(wq=(q_rows, hidden), wk=(kv_rows, hidden), wv=(kv_rows, hidden),
                      wo=(hidden, q_rows), wg=(ffn, hidden), wu=(ffn, hidden), wd=(hidden, ffn))
        self.shapes = shapes
        self.eps = eps
        self.device = torch.device(device)
        rng = np.random.Generator(np.random.PCG64(seed))
        self.norm_host = (1.0 + 0.02 * rng.standard_normal(hidden)).astype(np.float32)
        self.norm = torch.from_numpy(self.norm_host).to(self.device)
        self.host = {}
        self.dev = {}
        for i, name in enumerate(NAMES):
            pk = packs.synthetic_pack(self.fmts[name], *shapes[name], seed=seed * 101 + i)
            if keep_host:
                self.host[name] = pk
            payload = torch.from_numpy(pk.payload).to(self.device)
            meta = None if pk.meta is None else torch.from_numpy(pk.meta).to(self.device)
            self.dev[name] = (payload, meta)
        self.c = LayerSliceC(hidden, q_rows, kv_rows, ffn, eps, self.norm.data_ptr(),
                             attn_fmt, *[self.dev[n][0].data_ptr() for n in ("wq", "wk", "wv", "wo")],
                             *[self._meta_ptr(n) for n in ("wq", "wk", "wv", "wo")],
                             ffn_fmt, self.dev["wg"][0].data_ptr(), self.dev["wu"][0].data_ptr(),
                             self._meta_ptr("wg"), self._meta_ptr("wu"),
                             down_fmt, self.dev["wd"][0].data_ptr(), self._meta_ptr("wd"))
        n = ctypes.c_size_t(0)
        check("qg_layer_slice_workspace_bytes", ctypes.byref(self.c), ctypes.byref(n))
        self.workspace = torch.empty(n.value, dtype=torch.uint8, device=self.device)

    def _meta_ptr(self, name):
        meta = self.dev[name][1]
        return None if meta is None else meta.data_ptr()

    @property
    def weight_bytes(self) -> int:
        return sum(packs.pack_bytes(self.fmts[n], *self.shapes[n]) for n in NAMES)

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        if out is None:
            out = torch.empty_like(x)
        s = (stream or torch.cuda.current_stream()).cuda_stream
        check("qg_layer_slice_forward", ctypes.byref(self.c), x.data_ptr(), out.data_ptr(),
              self.workspace.data_ptr(), s)
        return out

    def batched_workspace(self, batch: int) -> torch.Tensor:
        n = ctypes.c_size_t(0)
        check("qg_layer_slice_batched_workspace_bytes", ctypes.byref(self.c), batch, ctypes.byref(n))
        return torch.empty(n.value, dtype=torch.uint8, device=self.device)

    def forward_batched(self, x: torch.Tensor, out: torch.Tensor | None = None,
                        workspace: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """x: [batch, hidden] fp32 -> [batch, hidden] (qg_layer_slice_forward_batched)."""
        batch = x.shape[0]
        if out is None:
            out = torch.empty_like(x)
        if workspace is None:
            workspace = self.batched_workspace(batch)
        self._batched_ws = workspace
        s = (stream or torch.cuda.current_stream()).cuda_stream
        check("qg_layer_slice_forward_batched", ctypes.byref(self.c), x.data_ptr(), out.data_ptr(), batch,
              workspace.data_ptr(), s)
        return out

    def batched_views(self, batch: int, workspace: torch.Tensor | None = None) -> dict[str, torch.Tensor]:
        """[batch, n] views of the intermediates of the last forward_batched."""
        ws = workspace if workspace is not None else self._batched_ws
        v = LayerSliceViews()
        check("qg_layer_slice_batched_buffers", ctypes.byref(self.c), batch, ws.data_ptr(), ctypes.byref(v))
        return self._views_of(v, ws, batch)

    def _views_of(self, v, ws, batch):
        d = self.dims
        sizes = dict(h=d["hidden"], q=d["q_rows"], k=d["kv_rows"], v=d["kv_rows"], o=d["hidden"],
                     gate=d["ffn"], up=d["ffn"], act=d["ffn"])
        out = {}
        base = ws.data_ptr()
        for name, size in sizes.items():
            off = getattr(v, name) - base
            t = ws[off : off + 4 * size * batch].view(torch.float32)
            out[name] = t if batch == 0 else t.view(batch, size)
        return out

    def views(self) -> dict[str, torch.Tensor]:
        v = LayerSliceViews()
        check("qg_layer_slice_buffers", ctypes.byref(self.c), self.workspace.data_ptr(), ctypes.byref(v))
        d = self.dims
        sizes = dict(h=d["hidden"], q=d["q_rows"], k=d["kv_rows"], v=d["kv_rows"], o=d["hidden"],
                     gate=d["ffn"], up=d["ffn"], act=d["ffn"])
        out = {}
        base = self.workspace.data_ptr()
        for name, size in sizes.items():
            off = getattr(v, name) - base
            out[name] = self.workspace[off : off + 4 * size].view(torch.float32)
        return out


class SliceBuckets:
    """One captured graph per batch bucket of the batched slice (qg_slice_buckets_*)."""

    def __init__(self, sl: LayerSlice, batches, stream: torch.cuda.Stream | None = None):
        self.slice = sl  # keeps the weights alive
        self.stream = stream or torch.cuda.current_stream(sl.device)
        arr = (ctypes.c_uint32 * len(batches))(*batches)
        self.handle = c_void_p(None)
        check("qg_slice_buckets_create", ctypes.byref(sl.c), arr, len(batches), self.stream.cuda_stream,
              ctypes.byref(self.handle))

    def bucket(self, batch: int) -> int:
        b = ctypes.c_uint32(0)
        check("qg_slice_buckets_bucket", self.handle, batch, ctypes.byref(b))
        return b.value

    def run(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if out is None:
            out = torch.empty_like(x)
        check("qg_slice_buckets_run", self.handle, x.data_ptr(), out.data_ptr(), x.shape[0],
              self.stream.cuda_stream)
        return out

    def close(self) -> None:
        if self.handle.value:
            check("qg_slice_buckets_destroy", self.handle)
            self.handle = c_void_p(None)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class StepGraph:
    """A decode step captured with qg_graph_begin/qg_graph_end and replayed with
    qg_graph_launch (the C-ABI graph API)."""

    def __init__(self, stream: torch.cuda.Stream, enqueue):
        self.stream = stream
        self.handle = c_void_p(None)
        with torch.cuda.stream(stream):
            check("qg_graph_begin", stream.cuda_stream)
            try:
                enqueue()
            finally:
                check("qg_graph_end", stream.cuda_stream, ctypes.byref(self.handle))

    def launch(self) -> None:
        check("qg_graph_launch", self.handle, self.stream.cuda_stream)

    def close(self) -> None:
        if self.handle.value:
            check("qg_graph_destroy", self.handle)
            self.handle = c_void_p(None)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
