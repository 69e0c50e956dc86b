"""CPU oracle (test infrastructure only) for the InnerQ group quantizer.

This is a numpy restatement of the reference quantizer in ``src/innerq/quant.py``
of mthcom/innerq.  It exists to CHECK the CUDA path; nothing in the product
imports it.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may use it.

Arithmetic model.  The reference runs every torch op in the input dtype
(fp16 for lm-eval, bf16 for LongBench).  A torch CPU/GPU half op computes in
fp32 and rounds the result to the dtype with round-to-nearest-even.  Because
fp32 has more than 2p+2 bits for p = 11 (fp16) and p = 8 (bf16), an fp32
division or square root rounded once more to the dtype is the correctly
rounded dtype result, so this file reproduces the reference bit for bit by
computing each op in float32 and calling :func:`rnd` after it.

Pinned against fixtures produced by running the reference itself
(``tests/golden/make_golden.py``); see ``tests/test_oracle_golden.py``.
"""
from __future__ import annotations

import numpy as np

INT32_MIN = np.iinfo(np.int32).min


# ----------------------------------------------------------------------------
# dtype helpers: values are carried as float32 arrays holding exactly
# representable fp16 / bf16 numbers.
# ----------------------------------------------------------------------------
def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 -> bfloat16 (RNE), returned as float32."""
    x = np.asarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    return np.where(nan, x, out).astype(np.float32)


def rnd(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round a float32 result to the reference op dtype ('fp16' or 'bf16')."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "fp16":
        with np.errstate(over="ignore"):
            return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        return bf16_round(x)
    raise ValueError(dtype)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def _to_codes(q: np.ndarray) -> np.ndarray:
    """float -> int32 the way the reference's ``.to(torch.int32)`` does on x86:
    NaN (the 0/0 of an all-zero group) becomes INT32_MIN."""
    out = np.full(q.shape, INT32_MIN, dtype=np.int64)
    ok = ~np.isnan(q)
    out[ok] = q[ok].astype(np.int64)
    return out.astype(np.int32)


def _group_view(x: np.ndarray, group: int, axis: int):
    """Split ``axis`` into (n_groups, group) exactly as quant.py:63 reshapes."""
    shape = x.shape
    assert shape[axis] % group == 0, "group size must divide the quantized dim"
    new_shape = shape[:axis] + (shape[axis] // group, group) + shape[axis + 1:]
    return x.reshape(new_shape), axis + 1


# ----------------------------------------------------------------------------
# quant.py:58-73  quantize_asym
# ----------------------------------------------------------------------------
def quantize_asym(x, group, bit, axis, dtype):
    x = np.asarray(x, dtype=np.float32)
    shape = x.shape
    xg, gax = _group_view(x, group, axis)
    mn = xg.min(axis=gax, keepdims=True)
    mx = xg.max(axis=gax, keepdims=True)
    qmax = float(2 ** bit - 1)
    with np.errstate(invalid="ignore", divide="ignore"):
        scale = rnd(rnd(mx - mn, dtype) / np.float32(qmax), dtype)
        q = rnd(rnd(xg - mn, dtype) / scale, dtype)
    q = np.rint(np.clip(q, 0.0, qmax))
    codes = _to_codes(q).reshape(shape)
    sshape = shape[:axis] + (shape[axis] // group,) + shape[axis + 1:]
    return codes, scale.reshape(sshape), mn.reshape(sshape)


# quant.py:95-111  quantize_sym (one bit goes to the sign)
def quantize_sym(x, group, bit, axis, dtype):
    x = np.asarray(x, dtype=np.float32)
    shape = x.shape
    signs = np.sign(x).astype(np.float32)
    xg, gax = _group_view(np.abs(x), group, axis)
    mx = xg.max(axis=gax, keepdims=True)
    qmax = float(2 ** (bit - 1) - 1)
    with np.errstate(invalid="ignore", divide="ignore"):
        scale = rnd(mx / np.float32(qmax), dtype)
        q = rnd(xg / scale, dtype)
    q = np.rint(np.clip(q, 0.0, qmax))
    codes = _to_codes(q).reshape(shape)
    sshape = shape[:axis] + (shape[axis] // group,) + shape[axis + 1:]
    return codes, scale.reshape(sshape), signs


# quant.py:75-81, 113-119: channel-dim groups the last axis, token-dim the one before
def quantize_channeldim_asym(x, group, bit, dtype="fp16"):
    return quantize_asym(x, group, bit, x.ndim - 1, dtype)


def quantize_tokendim_asym(x, group, bit, dtype="fp16"):
    return quantize_asym(x, group, bit, x.ndim - 2, dtype)


def quantize_channeldim_sym(x, group, bit, dtype="fp16"):
    return quantize_sym(x, group, bit, x.ndim - 1, dtype)


def quantize_tokendim_sym(x, group, bit, dtype="fp16"):
    return quantize_sym(x, group, bit, x.ndim - 2, dtype)


# ----------------------------------------------------------------------------
# quant.py:83-93, 121-131  dequantize_* in fp32 (op_dtype)
# ----------------------------------------------------------------------------
def _expand(scale, group, axis):
    return np.repeat(scale, group, axis=axis)


def dequantize_channeldim_asym(codes, scale, mn, group):
    ax = codes.ndim - 1
    return codes.astype(np.float32) * _expand(scale, group, ax) + _expand(mn, group, ax)


def dequantize_tokendim_asym(codes, scale, mn, group):
    ax = codes.ndim - 2
    return codes.astype(np.float32) * _expand(scale, group, ax) + _expand(mn, group, ax)


def dequantize_channeldim_sym(codes, scale, signs, group):
    ax = codes.ndim - 1
    return codes.astype(np.float32) * _expand(scale, group, ax) * signs


def dequantize_tokendim_sym(codes, scale, signs, group):
    ax = codes.ndim - 2
    return codes.astype(np.float32) * _expand(scale, group, ax) * signs


QUANT = {
    ("sym", "channel"): (quantize_channeldim_sym, dequantize_channeldim_sym),
    ("sym", "token"): (quantize_tokendim_sym, dequantize_tokendim_sym),
    ("asym", "channel"): (quantize_channeldim_asym, dequantize_channeldim_asym),
    ("asym", "token"): (quantize_tokendim_asym, dequantize_tokendim_asym),
}


def signed_codes(codes, signs):
    """codes x sign, the quantity the packed format stores for symmetric mode.
    An all-zero group's INT32_MIN code maps to 0 (its dequantized value is 0)."""
    c = np.where(codes == INT32_MIN, 0, codes).astype(np.int64)
    return (c * np.sign(signs).astype(np.int64)).astype(np.int32)


# ----------------------------------------------------------------------------
# cache.py:121-126 key normalisation factor and division
# ----------------------------------------------------------------------------
def key_norm_factor(k, dtype):
    """f = sqrt(max_t |K|) per (b, h, channel), in the dtype; shape [..., 1, D]."""
    mx = np.abs(np.asarray(k, np.float32)).max(axis=-2, keepdims=True)
    return rnd(np.sqrt(mx), dtype)


def normalize_keys(k, f, dtype):
    with np.errstate(invalid="ignore", divide="ignore"):
        return rnd(np.asarray(k, np.float32) / f, dtype)
