"""torch-tensor front end of the C-ABI (device memory and streams only; every
computation happens in libqgemv_b200.so).  Raises if CUDA or the library is absent."""

from __future__ import annotations

import torch

from . import packs
from ._lib import check

QG_ERR_WAIT_TIMEOUT = 0x1


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream: torch.cuda.Stream | None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def require_cuda() -> None:
    if not torch.cuda.is_available():
        raise RuntimeError("qgemv_b200 ops need a CUDA device (there is no CPU path)")


def to_device(pack: packs.Pack, device: str | torch.device = "cuda") -> tuple[torch.Tensor, torch.Tensor | None]:
    payload = torch.from_numpy(pack.payload).to(device)
    meta = None if pack.meta is None else torch.from_numpy(pack.meta).to(device)
    return payload, meta


def gemv(fmt: int, payload: torch.Tensor, meta: torch.Tensor | None, x: torch.Tensor, rows: int,
         cols: int, y: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    require_cuda()
    if y is None:
        y = torch.empty(rows, dtype=torch.float32, device=x.device)
    check("qg_gemv", fmt, _ptr(payload), _ptr(meta), _ptr(x), _ptr(y), rows, cols, _stream(stream))
    return y


def act_bytes(cols: int) -> int:
    import ctypes

    n = ctypes.c_size_t(0)
    check("qg_act_bytes", cols, ctypes.addressof(n))
    return n.value


def act_prepare(x: torch.Tensor, act: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    require_cuda()
    cols = x.numel()
    if act is None:
        act = torch.empty(act_bytes(cols), dtype=torch.uint8, device=x.device)
    check("qg_act_prepare", _ptr(x), cols, _ptr(act), _stream(stream))
    return act


def gemv_act(fmt: int, payload, meta, x: torch.Tensor, act: torch.Tensor, rows: int, cols: int,
             y: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    require_cuda()
    if y is None:
        y = torch.empty(rows, dtype=torch.float32, device=x.device)
    check("qg_gemv_act", fmt, _ptr(payload), _ptr(meta), _ptr(x), _ptr(act), _ptr(y), rows, cols,
          _stream(stream))
    return y


def gemv_batched(fmt: int, payload, meta, x: torch.Tensor, rows: int, cols: int,
                 y: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    require_cuda()
    batch = x.shape[0]
    if y is None:
        y = torch.empty(batch, rows, dtype=torch.float32, device=x.device)
    check("qg_gemv_batched", fmt, _ptr(payload), _ptr(meta), _ptr(x), _ptr(y), batch, rows, cols,
          _stream(stream))
    return y


def gemm_batched_workspace_bytes(fmt: int, batch: int, rows: int, cols: int) -> int:
    import ctypes

    n = ctypes.c_size_t(0)
    check("qg_gemm_batched_workspace_bytes", fmt, batch, rows, cols, ctypes.byref(n))
    return n.value


def gemm_batched(fmt: int, payload, meta, x: torch.Tensor, rows: int, cols: int,
                 y: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                 stream=None) -> torch.Tensor:
    """Y[b] = W x[b] on the tensor cores (qg_gemm_batched); x is [batch, cols] fp32."""
    require_cuda()
    batch = x.shape[0]
    if y is None:
        y = torch.empty(batch, rows, dtype=torch.float32, device=x.device)
    if workspace is None:
        workspace = torch.empty(gemm_batched_workspace_bytes(fmt, batch, rows, cols),
                                dtype=torch.uint8, device=x.device)
    check("qg_gemm_batched", fmt, _ptr(payload), _ptr(meta), _ptr(x), _ptr(y), batch, rows, cols,
          _ptr(workspace), _stream(stream))
    return y


def decode_stage(fmt: int, payload, meta, x, y, kv, token, rows: int, cols: int,
                 kv_words: int, page_words: int, active_pages: int, stream=None) -> None:
    require_cuda()
    check("qg_decode_stage", fmt, _ptr(payload), _ptr(meta), _ptr(x), _ptr(y), _ptr(kv),
          _ptr(token), rows, cols, kv_words, page_words, active_pages, _stream(stream))


def dequantize(fmt: int, payload, meta, first_block: int, block_count: int,
               out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    require_cuda()
    if out is None:
        out = torch.empty(block_count * 256, dtype=torch.float32, device=payload.device)
    check("qg_dequantize", fmt, _ptr(payload), _ptr(meta), first_block, block_count, _ptr(out),
          _stream(stream))
    return out


def argmax_token(values: torch.Tensor, token: torch.Tensor, token_offset: int, add_token: int,
                 modulus: int, stream=None) -> None:
    require_cuda()
    check("qg_argmax_token", _ptr(values), values.numel(), _ptr(token), token_offset, add_token,
          modulus, _stream(stream))


def gemv_plan(fmt: int, rows: int, cols: int, sms: int | None = None) -> dict:
    """The tiled GEMV's launch plan for a shape (qg_gemv_plan): on the current device, or,
    with `sms`, for a device of that many SMs (host-side, no device needed)."""
    import ctypes

    vals = [ctypes.c_uint32(0) for _ in range(4)]
    refs = [ctypes.addressof(v) for v in vals]
    if sms is None:
        check("qg_gemv_plan", fmt, rows, cols, *refs)
    else:
        check("qg_gemv_plan_sms", fmt, rows, cols, sms, *refs)
    grid, threads, rows_per_tile, stages = (v.value for v in vals)
    return dict(grid=grid, threads=threads, rows_per_tile=rows_per_tile, stages=stages)


def get_error() -> int:
    import ctypes

    v = ctypes.c_uint32(0)
    check("qg_get_error", ctypes.addressof(v))
    return v.value
