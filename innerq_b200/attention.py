"""Fused decode attention over the packed InnerQ cache (host side).

``decode_attention`` is the consumer half of the hot path: for one query
token per sequence it computes ``softmax(q K^T * scale) V`` over
``[sink | packed middle | recent]`` directly from the packed store, in place
of the reference's full dequantize (``src/innerq/cache.py:278-281``) followed
by Hugging Face sdpa with ``repeat_kv``.  Split-KV partials are merged with a
log-sum-exp merge; ``decode_attention_partials`` + ``lse_merge`` expose the
two halves for context sharding across GPUs.
"""
from __future__ import annotations

import ctypes as C
import math

import torch

from . import _lib
from .store import PackedSide, dtype_code, require_cuda, stream_ptr

_WORKSPACE: dict = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    key = (device.type, device.index)
    t = _WORKSPACE.get(key)
    if t is None or t.numel() < nbytes:
        t = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WORKSPACE[key] = t
    return t


def _q3(q: torch.Tensor) -> torch.Tensor:
    if q.dim() == 4:
        if q.shape[2] != 1:
            raise ValueError("decode attention takes one query token per sequence")
        q = q[:, :, 0]
    if q.stride(-1) != 1:
        q = q.contiguous()
    return q


def build_args(q: torch.Tensor, k: PackedSide, v: PackedSide, scale: float | None = None,
               n_splits: int = 0, tile_range: tuple[int, int] | None = None) -> _lib.AttnArgs:
    require_cuda(q, "query")
    q = _q3(q)
    B, Hq, D = q.shape
    if q.dtype != k.dtype:
        raise TypeError(f"query dtype {q.dtype} != cache dtype {k.dtype}")
    a = _lib.AttnArgs()
    a.struct_size = C.sizeof(_lib.AttnArgs)
    a.dtype = dtype_code(q.dtype)
    a.B, a.Hq, a.Hkv, a.D = B, Hq, k.H, D
    a.q = q.data_ptr()
    a.q_sb, a.q_sh = q.stride(0), q.stride(1)
    a.key_norm = k.norm_f.data_ptr() if (k.normalize and k.norm_f is not None and k.n_q) else None
    a.k = k.side_struct()
    a.v = v.side_struct()
    a.softmax_scale = float(scale if scale is not None else 1.0 / math.sqrt(D))
    a.n_splits = int(n_splits)
    if tile_range is not None:
        a.tile_lo, a.tile_hi = tile_range
    a._keep = q  # keep a contiguous copy alive for the launch
    return a


class DecodeAttention:
    """Per-layer launcher that keeps its C argument struct and output buffer
    between decode steps and only refreshes what changes (query pointer,
    token counts, recent-window pointer), to keep host time per layer low."""

    def __init__(self):
        self.args = _lib.AttnArgs()
        self.args.struct_size = C.sizeof(_lib.AttnArgs)
        self.out = None
        self._lib = _lib.load()

    def _fill(self, q, k, v, scale, step):
        if not q.is_cuda or q.dtype != k.dtype:
            require_cuda(q, "query")
            raise TypeError(f"query dtype {q.dtype} != cache dtype {k.dtype}")
        if q.dim() == 4 and q.shape[2] != 1:
            raise ValueError("decode attention takes one query token per sequence")
        if q.stride(-1) != 1:
            q = q.contiguous()
        a = self.args
        B, Hq, D = q.shape[0], q.shape[1], q.shape[-1]
        a.dtype = dtype_code(q.dtype)
        a.B, a.Hq, a.Hkv, a.D = B, Hq, k.H, D
        a.q = q.data_ptr()
        a.q_sb, a.q_sh = q.stride(0), q.stride(1)
        a.key_norm = k.norm_f.data_ptr() if (k.normalize and k.norm_f is not None and k.n_q) else None
        graph = step is not None
        k.fill_side(a.k, graph)
        v.fill_side(a.v, graph)
        a.step = step.data_ptr() if graph else None
        a.softmax_scale = float(scale if scale is not None else 1.0 / math.sqrt(D))
        return a, q

    def _ws(self, a, device):
        ws_bytes = self._lib.innerq_decode_attn_workspace(C.byref(a))
        if ws_bytes < 0:
            raise _lib.InnerqError("innerq_decode_attn_workspace", -1, _lib.last_error())
        return _workspace(device, ws_bytes)

    def __call__(self, q: torch.Tensor, k: PackedSide, v: PackedSide, scale: float | None = None,
                 out: torch.Tensor | None = None, step: torch.Tensor | None = None) -> torch.Tensor:
        """step: graph mode (the stores' step-0 state plus the device step
        counter; the launch can be recorded in a CUDA graph and replayed)."""
        a, q = self._fill(q, k, v, scale, step)
        a.n_splits = 0
        ws = self._ws(a, q.device)
        B, Hq, D = a.B, a.Hq, a.D
        if out is None:
            if self.out is None or self.out.shape != (B, Hq, D) or self.out.dtype != q.dtype:
                self.out = torch.empty((B, Hq, D), dtype=q.dtype, device=q.device)
            out = self.out
        _lib.call("innerq_decode_attn", C.byref(a), ws.data_ptr(), ws.numel(), out.data_ptr(),
                  out.stride(0), out.stride(1), None, stream_ptr(q.device))
        return out

    def partials(self, q: torch.Tensor, k: PackedSide, v: PackedSide, po: torch.Tensor,
                 pm: torch.Tensor, pl: torch.Tensor, scale: float | None = None,
                 step: torch.Tensor | None = None) -> None:
        """Exactly po.shape[2] split partials of this store into po
        [B, Hq, s, D], pm / pl [B, Hq, s] (fp32, contiguous; e.g. the send
        block of a sharding.ContextMerge)."""
        a, q = self._fill(q, k, v, scale, step)
        a.n_splits = po.shape[2]
        ws = self._ws(a, q.device)
        _lib.call("innerq_decode_attn_partials", C.byref(a), po.data_ptr(), pm.data_ptr(),
                  pl.data_ptr(), ws.data_ptr(), ws.numel(), stream_ptr(q.device))


def plan(args: _lib.AttnArgs) -> tuple[int, int]:
    nt, ns = C.c_int32(), C.c_int32()
    _lib.call("innerq_attn_plan", C.byref(args), C.byref(nt), C.byref(ns))
    return nt.value, ns.value


def decode_attention(q: torch.Tensor, k: PackedSide, v: PackedSide, scale: float | None = None,
                     n_splits: int = 0, out: torch.Tensor | None = None,
                     lse: torch.Tensor | None = None) -> torch.Tensor:
    """out [B, Hq, D] in the query dtype."""
    args = build_args(q, k, v, scale, n_splits)
    ws_bytes = _lib.load().innerq_decode_attn_workspace(C.byref(args))
    if ws_bytes < 0:
        raise _lib.InnerqError("innerq_decode_attn_workspace", -1, _lib.last_error())
    ws = _workspace(q.device, ws_bytes)
    if out is None:
        out = torch.empty((args.B, args.Hq, args.D), dtype=q.dtype, device=q.device)
    _lib.call("innerq_decode_attn", C.byref(args), ws.data_ptr(), ws.numel(), out.data_ptr(),
              out.stride(0), out.stride(1), None if lse is None else lse.data_ptr(),
              stream_ptr(q.device))
    return out


def decode_attention_partials(q: torch.Tensor, k: PackedSide, v: PackedSide,
                              scale: float | None = None, n_splits: int = 0,
                              tile_range: tuple[int, int] | None = None):
    """Split partials (o [B,Hq,S,D] fp32 unnormalised, m, l [B,Hq,S] log2 domain)."""
    args = build_args(q, k, v, scale, n_splits, tile_range)
    _, ns = plan(args)
    B, Hq, D = args.B, args.Hq, args.D
    po = torch.empty((B, Hq, ns, D), dtype=torch.float32, device=q.device)
    pm = torch.empty((B, Hq, ns), dtype=torch.float32, device=q.device)
    pl = torch.empty((B, Hq, ns), dtype=torch.float32, device=q.device)
    ws_bytes = _lib.load().innerq_decode_attn_workspace(C.byref(args))
    if ws_bytes < 0:
        raise _lib.InnerqError("innerq_decode_attn_workspace", -1, _lib.last_error())
    ws = _workspace(q.device, ws_bytes)
    _lib.call("innerq_decode_attn_partials", C.byref(args), po.data_ptr(), pm.data_ptr(),
              pl.data_ptr(), ws.data_ptr(), ws.numel(), stream_ptr(q.device))
    return po, pm, pl


def lse_merge(po: torch.Tensor, pm: torch.Tensor, pl: torch.Tensor, dtype: torch.dtype,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """Merge split partials along dim 2 into out [B, Hq, D] of dtype."""
    require_cuda(po, "partials")
    po, pm, pl = po.contiguous(), pm.contiguous(), pl.contiguous()
    B, Hq, ns, D = po.shape
    if out is None:
        out = torch.empty((B, Hq, D), dtype=dtype, device=po.device)
    _lib.call("innerq_lse_merge", po.data_ptr(), pm.data_ptr(), pl.data_ptr(), B, Hq, ns, D,
              dtype_code(dtype), out.data_ptr(), out.stride(0), out.stride(1), None,
              stream_ptr(po.device))
    return out
