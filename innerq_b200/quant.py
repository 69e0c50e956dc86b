"""Drop-in for ``innerq.quant`` (``src/innerq/quant.py`` of mthcom/innerq) on B200.

Same names, signatures, return values and errors as the reference:

* ``quantize_{channeldim,tokendim}_{sym,asym}(tensor, group_size, bit)``
  return ``(int32 codes, scale, signs | min)`` with scale / min in the input
  dtype, bit-exact with the reference (``quant.py:58-119``).  The codes are
  computed by the sm_100a quantize-and-pack kernel and read back through the
  reference-format unpack kernel.  One documented difference: an all-zero
  group, where the reference divides 0/0 and stores INT32_MIN, yields code 0
  here; both dequantize to the same values.
* ``dequantize_*(tensor, scale, zp_or_sign, group_size, op_dtype=fp32)``
  (``quant.py:83-93, 121-131``) run the reference-format dequant kernel.
* ``quantize_hybrid`` / ``dequantize_hybrid`` factories and ``QMode``
  (``quant.py:43-56, 133-176``) compose the functions above the way the
  reference does.

Tensors must be CUDA float16 / bfloat16 with a last dimension of 128 and
2/3/4-bit codes (1-bit asymmetric, the low half of hybrid mode), group sizes
32/64/128 (what the kernels are built for);
anything else raises.  There is no CPU path.
"""
from __future__ import annotations

from enum import Enum

import torch

from . import _lib
from .store import dtype_code, require_cuda, stream_ptr

__all__ = [
    "QMode", "quantize_asym", "quantize_sym",
    "quantize_channeldim_asym", "quantize_tokendim_asym",
    "quantize_channeldim_sym", "quantize_tokendim_sym",
    "dequantize_channeldim_asym", "dequantize_tokendim_asym",
    "dequantize_channeldim_sym", "dequantize_tokendim_sym",
    "quantize_hybrid", "dequantize_hybrid",
]


class QMode(Enum):
    """quant.py:43-56."""
    SYM = 'symmetric'
    ASYM = 'asymmetric'
    HYBRID = 'hybrid'

    @classmethod
    def from_str(cls, value: str):
        normalized = value.strip().lower()
        for member in cls:
            if member.value == normalized:
                return member
        raise ValueError("Value of Enum should be form the choices 'symmetric', 'asymmetric', "
                         "and 'hybrid'.")


def _quantize(tensor: torch.Tensor, group_size: int, bit: int, expanded_dim: int, mode: int):
    require_cuda(tensor, "tensor")
    shape = tensor.shape
    assert shape[expanded_dim] % group_size == 0  # quant.py:61, 99
    nd = tensor.dim()
    if expanded_dim not in (nd - 1, nd - 2):
        raise NotImplementedError("groups along the last or second-to-last dim only")
    over_token = expanded_dim == nd - 2
    T, D = shape[-2], shape[-1]
    if D != 128:
        raise NotImplementedError(f"last dim {D}: the packed kernels are built for 128")
    if bit not in (1, 2, 3, 4) or (bit == 1 and mode == _lib.SYM):
        raise NotImplementedError(f"{bit}-bit codes are not built (2, 3, 4; 1 for asymmetric)")
    if group_size not in (32, 64, 128):
        raise NotImplementedError(f"group size {group_size} is not built (32, 64, 128 are)")
    dt = dtype_code(tensor.dtype)
    x = tensor.reshape(-1, 1, T, D)
    if x.stride(-1) != 1 or x.data_ptr() % 8:
        x = x.contiguous()
    N = x.shape[0]
    role = _lib.ROLE_V if over_token else _lib.ROLE_K
    tb = _lib.load().innerq_tile_bytes(bit)
    cap_tiles = max(1, (T + 31) // 32)
    if over_token:
        cap_tiles = (cap_tiles * 32 + group_size - 1) // group_size * group_size // 32
    dev = tensor.device
    codes = torch.empty((N, 1, cap_tiles, tb), dtype=torch.uint8, device=dev)
    if over_token:
        sshape = (N, 1, cap_tiles * 32 // group_size, D)
        rshape = shape[:-2] + (T // group_size, D)
    else:
        sshape = (N, 1, cap_tiles * 32, D // group_size)
        rshape = shape[:-1] + (D // group_size,)
    scale_st = torch.empty(sshape, dtype=tensor.dtype, device=dev)
    zero_st = torch.empty(sshape, dtype=tensor.dtype, device=dev) if mode == _lib.ASYM else None
    s = stream_ptr(dev)
    _lib.call("innerq_quant_pack", x.data_ptr(), dt, N, 1, T, D, x.stride(0), x.stride(1),
              x.stride(2), bit, group_size, mode, role, int(over_token), None, codes.data_ptr(),
              scale_st.data_ptr(), None if zero_st is None else zero_st.data_ptr(), cap_tiles, 0, s)
    out_codes = torch.empty(shape, dtype=torch.int32, device=dev)
    out_scale = torch.empty(rshape, dtype=tensor.dtype, device=dev)
    out_zero = torch.empty(rshape, dtype=tensor.dtype, device=dev) if mode == _lib.ASYM else None
    _lib.call("innerq_unpack_ref", codes.data_ptr(), scale_st.data_ptr(),
              None if zero_st is None else zero_st.data_ptr(), dt, N, 1, 0, T, D, bit, group_size,
              mode, role, int(over_token), cap_tiles, out_codes.data_ptr(), None,
              out_scale.data_ptr(), None if out_zero is None else out_zero.data_ptr(), s)
    if mode == _lib.ASYM:
        return out_codes, out_scale, out_zero
    return out_codes, out_scale, tensor.sign()


def quantize_asym(tensor, group_size, bit, expanded_dim):
    """quant.py:58-73."""
    return _quantize(tensor, group_size, bit, expanded_dim, _lib.ASYM)


def quantize_sym(tensor, group_size, bit, expanded_dim):
    """quant.py:95-111 (one of the bits holds the sign)."""
    return _quantize(tensor, group_size, bit, expanded_dim, _lib.SYM)


def quantize_channeldim_asym(tensor, group_size, bit):
    return quantize_asym(tensor, group_size, bit, tensor.dim() - 1)


def quantize_tokendim_asym(tensor, group_size, bit):
    return quantize_asym(tensor, group_size, bit, tensor.dim() - 2)


def quantize_channeldim_sym(tensor, group_size, bit):
    return quantize_sym(tensor, group_size, bit, tensor.dim() - 1)


def quantize_tokendim_sym(tensor, group_size, bit):
    return quantize_sym(tensor, group_size, bit, tensor.dim() - 2)


def _dequantize(tensor, scale, zp_or_sign, group_size, op_dtype, mode, over_token):
    require_cuda(tensor, "tensor")
    if tensor.dtype != torch.int32:
        tensor = tensor.to(torch.int32)
    tensor = tensor.contiguous()
    scale = scale.contiguous()
    zp_or_sign = zp_or_sign.to(scale.dtype).contiguous()
    T, D = tensor.shape[-2], tensor.shape[-1]
    n_outer = tensor.numel() // max(1, T * D)
    out = torch.empty(tensor.shape, dtype=torch.float32, device=tensor.device)
    _lib.call("innerq_dequant_ref", tensor.data_ptr(), scale.data_ptr(), zp_or_sign.data_ptr(),
              dtype_code(scale.dtype), n_outer, T, D, group_size, mode, int(over_token),
              out.data_ptr(), stream_ptr(tensor.device))
    return out if op_dtype == torch.float32 else out.to(op_dtype)


def dequantize_channeldim_asym(tensor, scale, zero_points, group_size, op_dtype=torch.float32):
    return _dequantize(tensor, scale, zero_points, group_size, op_dtype, _lib.ASYM, False)


def dequantize_tokendim_asym(tensor, scale, zero_points, group_size, op_dtype=torch.float32):
    return _dequantize(tensor, scale, zero_points, group_size, op_dtype, _lib.ASYM, True)


def dequantize_channeldim_sym(tensor, scale, signs, group_size, op_dtype=torch.float32):
    return _dequantize(tensor, scale, signs, group_size, op_dtype, _lib.SYM, False)


def dequantize_tokendim_sym(tensor, scale, signs, group_size, op_dtype=torch.float32):
    return _dequantize(tensor, scale, signs, group_size, op_dtype, _lib.SYM, True)


def _grouped_shape(scale_shape, tensor_shape, group_size):
    q_dim = next(i for i, (a, b) in enumerate(zip(scale_shape, tensor_shape)) if a != b)
    return q_dim, list(scale_shape[:q_dim]) + [scale_shape[q_dim], group_size] + list(scale_shape[q_dim + 1:])


def quantize_hybrid(zp_func, nozp_func, zp_deq_func, nozp_deq_func):
    """quant.py:133-151: asym at bit-1 bits and sym at bit bits per group; the
    mask selects sym where its fp32 L1 error is lower."""
    def hybrid_func(tensor, group_size, bit):
        q_zp = zp_func(tensor, group_size, bit - 1)
        q_nozp = nozp_func(tensor, group_size, bit)
        deq_zp = zp_deq_func(*q_zp, group_size)
        deq_nozp = nozp_deq_func(*q_nozp, group_size)
        q_dim, gshape = _grouped_shape(q_zp[1].shape, tensor.shape, group_size)
        err_zp = (deq_zp - tensor).view(gshape).abs().sum(q_dim + 1)
        err_nozp = (deq_nozp - tensor).view(gshape).abs().sum(q_dim + 1)
        mask = err_zp > err_nozp
        return ({'zp': q_zp[0], 'nozp': q_nozp[0]},
                {'zp': q_zp[1], 'nozp': q_nozp[1], 'mask': mask},
                {'zp': q_zp[2], 'nozp': q_nozp[2]})
    return hybrid_func


def dequantize_hybrid(zp_func, nozp_func):
    """quant.py:153-176."""
    def hybrid_func(tensor, scale, sign_or_zp, group_size, op_dtype=torch.float32):
        q_dim, gshape = _grouped_shape(scale['zp'].shape, tensor['zp'].shape, group_size)
        mask = scale['mask'].unsqueeze(q_dim + 1).expand(gshape)
        zp_deq = zp_func(tensor['zp'], scale['zp'], sign_or_zp['zp'], group_size, op_dtype).reshape(gshape)
        nozp_deq = nozp_func(tensor['nozp'], scale['nozp'], sign_or_zp['nozp'], group_size,
                             op_dtype).reshape(gshape)
        return torch.where(mask, nozp_deq, zp_deq).view(tensor['zp'].shape)
    return hybrid_func
