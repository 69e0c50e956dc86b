"""CPU baseline (test and benchmark infrastructure only): the reference's
decode step restated with the same torch ops, run on the host cores.

The reference's decode step per layer is ``InnerqDynamicLayer.update``
(``src/innerq/cache.py:382-396``): append the new token to the recent window
and pop ``flush`` tokens when it holds that many (``:283-312``), quantize them
(``quant.py:58-131`` via ``:314-365``) and ``torch.cat`` them onto the whole
store, then dequantize the whole store in fp32, undo the key normalisation,
concatenate sink / store / recent and cast to the model dtype
(``get_deq_tensors``, ``:235-281``), after which the Hugging Face consumer runs
``scaled_dot_product_attention`` over the repeated KV heads.  This module
repeats those torch ops on CPU tensors, so ``torch.set_num_threads`` spreads
them over every host core the way the reference's own CPU run would.

``bench.py`` times it as the CPU baseline (``cpu_baseline`` and
``--impl reference``); ``tests/test_oracle_golden.py`` checks that its K/V
are bit-identical with the numpy oracle, which is pinned to the reference's
fixtures.  Symmetric and asymmetric modes, channel and token groups (hybrid
is not needed by the benchmarked configurations).  Nothing in the product
imports this module.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def _quantize(x: torch.Tensor, group: int, bits: int, dim: int, sym: bool):
    """quant.py:58-73 (asym) and :95-111 (sym): groups of `group` along `dim`."""
    shape = x.shape
    ng = shape[dim] // group
    assert shape[dim] % group == 0
    gshape = shape[:dim] + (ng, group) + shape[dim + 1:]
    sshape = shape[:dim] + (ng,) + shape[dim + 1:]
    if sym:
        top = 2 ** (bits - 1) - 1
        signs = x.sign()
        a = x.reshape(gshape).abs()
        scale = a.max(dim=dim + 1, keepdim=True)[0] / top
        a.div_(scale)
        codes = a.clamp_(0, top).round_().to(torch.int32).reshape(shape)
        return codes, scale.reshape(sshape), signs
    top = 2 ** bits - 1
    g = x.reshape(gshape)
    mn = g.min(dim=dim + 1, keepdim=True)[0]
    scale = (g.max(dim=dim + 1, keepdim=True)[0] - mn) / top
    y = g - mn
    y.div_(scale)
    codes = y.clamp_(0, top).round_().to(torch.int32).reshape(shape)
    return codes, scale.reshape(sshape), mn.reshape(sshape)


def _dequantize(codes, scale, zs, group: int, over_token: bool, sym: bool):
    """quant.py:83-93 (asym) and :121-131 (sym), op dtype fp32."""
    if over_token:
        gshape = codes.shape[:-2] + (scale.shape[-2], group, codes.shape[-1])
        r = codes.view(gshape).to(torch.float32) * scale.unsqueeze(-2).to(torch.float32)
        if not sym:
            r = r + zs.unsqueeze(-2).to(torch.float32)
    else:
        gshape = codes.shape[:-1] + (scale.shape[-1], group)
        r = codes.view(gshape).to(torch.float32) * scale.unsqueeze(-1).to(torch.float32)
        if not sym:
            r = r + zs.unsqueeze(-1).to(torch.float32)
    r = r.view(codes.shape)
    return r * zs if sym else r


class _Side:
    def __init__(self, bits, group, w_recent, w_sink, flush, over_token, mode, normalize):
        self.bits, self.group, self.w_recent, self.w_sink = bits, group, w_recent, w_sink
        self.flush, self.over_token, self.sym = flush, over_token, mode == "symmetric"
        self.normalize = normalize
        self.factor = None
        self.codes = self.scale = self.zs = None

    def _q(self, x):
        if self.normalize:
            if self.factor is None:  # cache.py:121-126, from the first quantized tokens
                self.factor = x.abs().max(dim=-2, keepdim=True).values.sqrt()
            x = x / self.factor
        return _quantize(x, self.group, self.bits, x.dim() - (2 if self.over_token else 1), self.sym)

    def prefill(self, x):  # cache.py:135-210
        ns = min(self.w_sink, x.shape[-2])
        self.sink, x = x[:, :, :ns], x[:, :, ns:]
        r = min(self.w_recent, x.shape[-2])
        if self.over_token:
            while (x.shape[-2] - r) % self.flush:
                r -= 1
        nq = x.shape[-2] - r
        self.recent = x[:, :, nq:].contiguous()
        if nq:
            self.codes, self.scale, self.zs = self._q(x[:, :, :nq].contiguous())

    def append(self, x):  # cache.py:283-312, 314-380
        self.recent = torch.cat([self.recent, x], dim=-2)
        n = self.flush if self.recent.shape[-2] >= self.flush else 0
        out, self.recent = self.recent[:, :, :n], self.recent[:, :, n:]
        if out.numel():
            c, s, z = self._q(out)
            if self.codes is None:
                self.codes, self.scale, self.zs = c, s, z
            else:
                self.codes = torch.cat([self.codes, c], dim=2)
                self.scale = torch.cat([self.scale, s], dim=2)
                self.zs = torch.cat([self.zs, z], dim=2)

    def deq(self, dtype):  # cache.py:235-276, then the cast of :278-281
        parts = [self.sink] if self.sink.numel() else []
        if self.codes is not None:
            d = _dequantize(self.codes, self.scale, self.zs, self.group, self.over_token, self.sym)
            if self.normalize:
                d = d * self.factor
            parts.append(d)
        if self.recent.numel():
            parts.append(self.recent)
        out = torch.tensor([], dtype=dtype)
        for p in parts:
            out = torch.cat([out, p], dim=-2)
        return out.to(dtype)


class TorchRefLayer:
    """One cache layer of the reference (the sym/asym configurations)."""

    def __init__(self, k_bits=16, v_bits=16, key_group_size=32, value_group_size=32,
                 key_w_recent=32, value_w_recent=32, key_w_sink=0, value_w_sink=0,
                 key_flush_size=32, value_flush_size=32, key_normalize=False,
                 key_quantize_over_token=False, value_quantize_over_token=True,
                 key_quantize_mode="symmetric", value_quantize_mode="symmetric"):
        assert k_bits < 16 and v_bits < 16, "the baseline covers quantized caches"
        self.k = _Side(k_bits, key_group_size, key_w_recent, key_w_sink, key_flush_size,
                       key_quantize_over_token, key_quantize_mode, bool(key_normalize))
        self.v = _Side(v_bits, value_group_size, value_w_recent, value_w_sink, value_flush_size,
                       value_quantize_over_token, value_quantize_mode, False)
        self.dtype = None

    def update(self, k: torch.Tensor, v: torch.Tensor):
        """cache.py:382-396: prefill returns the inputs, a decode step the
        dequantized K/V in the model dtype."""
        if self.dtype is None:
            self.dtype = k.dtype
            self.k.prefill(k)
            self.v.prefill(v)
            return k, v
        self.k.append(k)
        self.v.append(v)
        return self.k.deq(self.dtype), self.v.deq(self.dtype)


def consumer_attention(q: torch.Tensor, K: torch.Tensor, V: torch.Tensor) -> torch.Tensor:
    """The Hugging Face sdpa consumer: KV heads repeated to the query heads,
    then scaled_dot_product_attention (scale head_dim^-0.5) in the model dtype."""
    rep = q.shape[1] // K.shape[1]
    if rep > 1:
        B, H, S, D = K.shape
        K = K[:, :, None].expand(B, H, rep, S, D).reshape(B, H * rep, S, D)
        V = V[:, :, None].expand(B, H, rep, S, D).reshape(B, H * rep, S, D)
    return F.scaled_dot_product_attention(q, K, V)


def ref_cache(n_layers: int, **kw):
    """A Hugging Face cache whose layers are TorchRefLayer (the reference's
    cache on CPU), for timing a full model's decode step on the host."""
    from transformers.cache_utils import Cache, CacheLayerMixin

    class _Layer(CacheLayerMixin):
        is_sliding = False

        def __init__(self):
            super().__init__()
            self.ref = TorchRefLayer(**kw)
            self.n = 0

        def lazy_initialization(self, key_states, value_states):
            self.dtype, self.device = key_states.dtype, key_states.device
            self.is_initialized = True

        def update(self, key_states, value_states, *args, **kwargs):
            if not self.is_initialized:
                self.lazy_initialization(key_states, value_states)
            self.n += key_states.shape[-2]
            return self.ref.update(key_states, value_states)

        def get_mask_sizes(self, query_length):
            q = query_length if isinstance(query_length, int) else query_length.shape[0]
            return self.n + q, 0

        def get_seq_length(self):
            return self.n

        def get_max_cache_shape(self):
            return -1

    return Cache(layers=[_Layer() for _ in range(n_layers)])
