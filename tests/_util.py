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


def synth_kv_dev(B, H, T, D=128, dtype="fp16", seed=0, device="cuda"):
    """synth_kv drawn by the device generator (full-size caches: seconds, not
    minutes, and no host copy of the cache)."""
    g = torch.Generator(device=device).manual_seed(seed)
    k = torch.randn((B, H, T, D), device=device, generator=g)
    k *= torch.exp(torch.randn(D, device=device, generator=g))
    k = k.to(TDT[dtype])
    v = torch.randn((B, H, T, D), device=device, generator=g).to(TDT[dtype])
    return k, v


def side_fp32(side, normalize_f=None):
    """[sink | fp32 dequantization | recent] of one packed side, the dequantized
    part from the reference-format views (innerq_unpack_ref, then the
    quant.py:83-93 / 121-131 dequantize restated by innerq_dequant_ref), i.e.
    independent of the fused attention kernel."""
    from innerq_b200 import _lib
    from innerq_b200 import quant as M
    parts = []
    if side.sink is not None and side.sink.shape[2]:
        parts.append(side.sink.float())
    codes, scale, zs = side.ref_views()
    if codes is not None:
        d = M._dequantize(codes, scale, zs, side.group, torch.float32, side.mode, side.over_token)
        del codes, scale, zs
        if normalize_f is not None:
            d *= normalize_f.float().unsqueeze(2)
        parts.append(d)
    if side.n_recent:
        parts.append(side.recent.float())
    return torch.cat(parts, dim=2)


def gpu_ref_attention(layer, q):
    """softmax(q K^T / sqrt(D)) V in fp64 over the reference fp32 dequantized
    K/V (cache.py:235-281 without the final cast), one sequence at a time,
    query heads grouped per KV head (GQA).  q [B, Hq, 1, D] -> [B, Hq, D]."""
    import math
    ks, vs = layer.key_side, layer.value_side
    K = side_fp32(ks, ks.norm_f if ks.normalize else None)
    V = side_fp32(vs)
    B, Hkv, S, D = K.shape
    R = q.shape[1] // Hkv
    out = torch.empty((B, q.shape[1], D), dtype=torch.float64, device=q.device)
    for b in range(B):
        kb, vb = K[b].double(), V[b].double()
        qb = q[b, :, 0].double().view(Hkv, R, D)
        lg = (qb @ kb.transpose(-1, -2)) / math.sqrt(D)
        out[b] = (torch.softmax(lg, dim=-1) @ vb).reshape(Hkv * R, D)
    return out


def assert_attn_close(out, ref, dtype="fp16"):
    """The 1e-3 bar: |out - ref| <= 1e-3 max|ref| plus the model dtype's
    rounding of each output element."""
    r = ref.float().cpu().numpy()
    o = out.float().cpu().numpy()
    ulp = 2.0 ** -8 if dtype == "bf16" else 2.0 ** -11
    err = np.abs(o - r)
    bound = 1e-3 * np.abs(r).max() + ulp * np.abs(r)
    assert (err <= bound).all(), f"max err {err.max():.3e}, bound at argmax {bound.flat[err.argmax()]:.3e}"


def hybrid_side_fp32(side):
    """[sink | fp32 hybrid dequantization | recent] of a HybridSide: both code
    sets dequantized by the reference-format kernels and combined with the
    mask as quant.py:159-176 does (symmetric where the mask is set)."""
    from innerq_b200 import quant as M
    parts = []
    if side.sink is not None and side.sink.shape[2]:
        parts.append(side.sink.float())
    codes, scale, zs = side.ref_views()
    if codes is not None:
        sym = M._dequantize(codes["nozp"], scale["nozp"], zs["nozp"], side.group, torch.float32,
                            side.mode, side.over_token)
        asym = M._dequantize(codes["zp"], scale["zp"], zs["zp"], side.group, torch.float32, 1,
                             side.over_token)
        m = scale["mask"].repeat_interleave(side.group, dim=2 if side.over_token else 3)
        parts.append(torch.where(m, sym, asym))
    if side.n_recent:
        parts.append(side.recent.float())
    return torch.cat(parts, dim=2)
