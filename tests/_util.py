"""Shared helpers for the parity tests: seeded inputs and oracle comparisons."""
from __future__ import annotations

import types

import numpy as np
import torch

from oracle import cache_ref as C

TDT = {"fp16": torch.float16, "bf16": torch.bfloat16}


def synth_kv(B, H, T, D=128, dtype="fp16", seed=0, device="cuda"):
    """K = N(0,1) x exp(N(0,1)) per channel (channel outliers), V = N(0,1)."""
    g = torch.Generator().manual_seed(seed)
    k = torch.randn((B, H, T, D), generator=g) * torch.exp(torch.randn(D, generator=g))
    v = torch.randn((B, H, T, D), generator=g)
    return k.to(TDT[dtype]).to(device), v.to(TDT[dtype]).to(device)


def synth_q(B, Hq, D=128, dtype="fp16", seed=1, device="cuda"):
    g = torch.Generator().manual_seed(seed)
    return torch.randn((B, Hq, 1, D), generator=g).to(TDT[dtype]).to(device)


def to_np32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def cfg(**kw):
    """An attribute bag standing in for the HF config (cache.py reads getattr)."""
    return types.SimpleNamespace(**kw)


def oracle_layer(kw, dtype):
    return C.OracleLayer(C.CacheConfig(**kw), dtype)


def assert_close_rel(out, ref, tol=1e-3, what=""):
    """max |out - ref| <= tol * max |ref| (the 1e-3 relative bar)."""
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = max(np.abs(ref).max(), 1e-30)
    err = np.abs(out - ref).max()
    assert err <= tol * scale, f"{what}: max err {err:.3e} > {tol:g} x max|ref| {scale:.3e}"


def merge_np(po, pm, pl):
    """float64 merge of split partials (log2 domain), for tight comparisons."""
    po = np.asarray(po, np.float64)
    pm = np.asarray(pm, np.float64)
    pl = np.asarray(pl, np.float64)
    M = pm.max(axis=-1, keepdims=True)
    w = np.where(np.isneginf(pm), 0.0, np.exp2(pm - np.where(np.isneginf(M), 0, M)))
    num = (po * w[..., None]).sum(axis=-2)
    den = (pl * w).sum(axis=-1)
    return num / den[..., None], (M[..., 0] + np.log2(den))
