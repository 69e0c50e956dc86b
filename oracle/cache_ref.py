"""CPU oracle (test infrastructure only) for the InnerQ KV-cache layer.

A numpy restatement of ``InnerqDynamicLayer`` (``src/innerq/cache.py:61-419``)
of mthcom/innerq: sink / quantized middle / recent split at prefill, the
recent-window flush rule on every decode step, key normalisation, and the full
dequantize-and-concatenate the reference returns from ``update``.  Plus the
attention the Hugging Face consumer runs on those tensors
(``softmax(q K^T * scale) V`` with grouped-query heads).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
may use this module; the product path never does.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import quant_ref as Q


@dataclass
class CacheConfig:
    """The 15 quantisation attributes read by cache.py:70-91, same defaults."""
    k_bits: int = 16
    v_bits: int = 16
    key_group_size: int = 32
    value_group_size: int = 32
    key_w_recent: int = 32
    value_w_recent: int = 32
    key_w_sink: int = 0
    value_w_sink: int = 0
    key_flush_size: int = 32
    value_flush_size: int = 32
    key_normalize: bool = False
    key_quantize_over_token: bool = False
    value_quantize_over_token: bool = True
    key_quantize_mode: str = "symmetric"
    value_quantize_mode: str = "symmetric"


PRESETS = {
    # scripts/run_lmeval.sh:94-113 (innerq_base), 114-133 (innerq_small), 54-72 (kivi)
    "innerq_base": dict(k_bits=3, v_bits=3, key_flush_size=1, value_flush_size=32,
                        key_group_size=32, value_group_size=32, key_w_recent=96,
                        value_w_recent=96, key_w_sink=32, value_w_sink=32,
                        key_normalize=True, key_quantize_over_token=False,
                        value_quantize_over_token=True, key_quantize_mode="symmetric",
                        value_quantize_mode="symmetric"),
    "innerq_small": dict(k_bits=3, v_bits=2, key_flush_size=1, value_flush_size=32,
                         key_group_size=32, value_group_size=32, key_w_recent=96,
                         value_w_recent=96, key_w_sink=32, value_w_sink=32,
                         key_normalize=True, key_quantize_over_token=False,
                         value_quantize_over_token=True, key_quantize_mode="symmetric",
                         value_quantize_mode="symmetric"),
    "kivi": dict(k_bits=2, v_bits=2, key_flush_size=32, value_flush_size=1,
                 key_group_size=32, value_group_size=32, key_w_recent=128,
                 value_w_recent=128, key_w_sink=0, value_w_sink=0,
                 key_normalize=False, key_quantize_over_token=True,
                 value_quantize_over_token=False, key_quantize_mode="asymmetric",
                 value_quantize_mode="asymmetric"),
}

_MODE = {"symmetric": "sym", "asymmetric": "asym"}


class _Side:
    """One of K or V: sink, quantized store and recent window."""

    def __init__(self, bits, group, w_recent, w_sink, flush, over_token, mode, dtype,
                 normalize=False):
        self.bits, self.group, self.w_recent, self.w_sink = bits, group, w_recent, w_sink
        self.flush, self.over_token, self.dtype = flush, over_token, dtype
        self.quantize = bits < 16
        m = mode.strip().lower()
        if m not in _MODE:
            raise ValueError("mode must be symmetric or asymmetric in the oracle")
        self.mode = _MODE[m]
        self.qf, self.df = Q.QUANT[(self.mode, "token" if over_token else "channel")]
        self.normalize = normalize
        self.factor = None
        self.codes = self.scale = self.zp = None

    # cache.py:121-126
    def _norm(self, x):
        if self.normalize:
            if self.factor is None:
                self.factor = Q.key_norm_factor(x, self.dtype)
            x = Q.normalize_keys(x, self.factor, self.dtype)
        return x

    def _q(self, x):
        x = self._norm(x)
        return self.qf(x, self.group, self.bits, self.dtype)

    # cache.py:135-155, 157-185, 187-210
    def prefill(self, x):
        T = x.shape[-2]
        n_sink = min(self.w_sink, T) if self.quantize else 0
        self.sink = x[:, :, :n_sink]
        x = x[:, :, n_sink:]
        if self.quantize:
            r = min(self.w_recent, x.shape[-2])
            if self.over_token:
                while (x.shape[-2] - r) % self.flush != 0:
                    r -= 1
        else:
            r = x.shape[-2]
        nq = x.shape[-2] - r
        self.recent = x[:, :, nq:].copy()
        mid = x[:, :, :nq]
        if self.quantize and mid.size != 0:
            self.codes, self.scale, self.zp = self._q(mid)

    # cache.py:283-307 then 314-380
    def append(self, x):
        self.recent = np.concatenate([self.recent, x], axis=-2)
        n = self.flush if (self.quantize and self.recent.shape[-2] >= self.flush) else 0
        out = self.recent[:, :, :n]
        self.recent = self.recent[:, :, n:]
        if out.size != 0:
            c, s, z = self._q(out)
            if self.codes is None:
                self.codes, self.scale, self.zp = c, s, z
            else:
                self.codes = np.concatenate([self.codes, c], axis=2)
                self.scale = np.concatenate([self.scale, s], axis=2)
                self.zp = np.concatenate([self.zp, z], axis=2)

    def n_quantized(self):
        return 0 if self.codes is None else self.codes.shape[2]

    # cache.py:235-281: fp32 dequant, unnormalise, concatenate, cast to the dtype
    def dequant_fp32(self):
        if self.codes is None:
            return None
        d = self.df(self.codes, self.scale, self.zp, self.group)
        if self.normalize:
            d = d * self.factor
        return d.astype(np.float32)

    def full(self):
        parts = [self.sink]
        d = self.dequant_fp32()
        if d is not None:
            parts.append(Q.rnd(d, self.dtype))
        parts.append(self.recent)
        return np.concatenate(parts, axis=-2)


class OracleLayer:
    """Restatement of InnerqDynamicLayer (cache.py:61-419) on numpy arrays."""

    def __init__(self, cfg: CacheConfig, dtype: str = "fp16"):
        self.cfg, self.dtype = cfg, dtype
        self.k = _Side(cfg.k_bits, cfg.key_group_size, cfg.key_w_recent, cfg.key_w_sink,
                       cfg.key_flush_size, cfg.key_quantize_over_token, cfg.key_quantize_mode,
                       dtype, normalize=cfg.key_normalize)
        self.v = _Side(cfg.v_bits, cfg.value_group_size, cfg.value_w_recent, cfg.value_w_sink,
                       cfg.value_flush_size, cfg.value_quantize_over_token,
                       cfg.value_quantize_mode, dtype)
        self.cumulative_length = 0
        self.initialized = False

    # cache.py:382-396
    def update(self, k, v):
        k = np.asarray(k, np.float32)
        v = np.asarray(v, np.float32)
        self.cumulative_length += k.shape[-2]
        if not self.initialized:
            self.k.prefill(k)
            self.v.prefill(v)
            self.initialized = True
            return k, v
        self.k.append(k)
        self.v.append(v)
        return self.k.full(), self.v.full()

    def get_seq_length(self):
        return self.cumulative_length


def attention(q, k, v, scale=None):
    """softmax(q K^T * scale) V with GQA; q [B,Hq,Lq,D], k/v [B,Hkv,S,D].
    Computed in float64 from the given values (the reference hands the cast
    K/V to HF sdpa; this is its exact-arithmetic counterpart)."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    B, Hq, Lq, D = q.shape
    Hkv = k.shape[1]
    rep = Hq // Hkv
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    kk = np.repeat(k, rep, axis=1)
    vv = np.repeat(v, rep, axis=1)
    logits = np.einsum("bhqd,bhsd->bhqs", q, kk) * scale
    m = logits.max(axis=-1, keepdims=True)
    p = np.exp(logits - m)
    l = p.sum(axis=-1, keepdims=True)
    return np.einsum("bhqs,bhsd->bhqd", p / l, vv), logits


def lse_merge(o, m, l):
    """Merge split-KV partials: o [..., S, D] (unnormalised sums), m, l [..., S].
    out = sum_s exp(m_s - M) o_s / sum_s exp(m_s - M) l_s."""
    o = np.asarray(o, np.float64)
    m = np.asarray(m, np.float64)
    l = np.asarray(l, np.float64)
    M = m.max(axis=-1, keepdims=True)
    w = np.exp(m - M)
    return (o * w[..., None]).sum(axis=-2) / (l * w).sum(axis=-1)[..., None]
