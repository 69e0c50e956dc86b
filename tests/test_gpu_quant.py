"""GPU parity of the quantize-and-pack kernel (through innerq_b200.quant and the
C ABI) against fixtures produced by the reference quant.py itself, and against
the oracle at sizes the fixtures do not cover."""
import numpy as np
import pytest
import torch

from oracle import quant_ref as Q
from tests._util import TDT, synth_kv, to_np32

pytestmark = pytest.mark.gpu

FUNCS = ["channel_sym", "token_sym", "channel_asym", "token_asym"]


def _ours():
    from innerq_b200 import quant as M
    return {
        "channel_sym": (M.quantize_channeldim_sym, M.dequantize_channeldim_sym),
        "token_sym": (M.quantize_tokendim_sym, M.dequantize_tokendim_sym),
        "channel_asym": (M.quantize_channeldim_asym, M.dequantize_channeldim_asym),
        "token_asym": (M.quantize_tokendim_asym, M.dequantize_tokendim_asym),
    }


def _x(g, dtype):
    x = g[f"{dtype}/x"]
    if dtype == "bf16":
        return torch.from_numpy(x.view(np.int16).copy()).view(torch.bfloat16).cuda()
    return torch.from_numpy(x.copy()).cuda()


def _bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _golden_bits(arr, dtype):
    if dtype == "bf16":
        return arr
    return arr.view(np.uint16)


def test_quantize_bit_exact_vs_reference_fixtures(quant_golden):
    g = quant_golden
    ours = _ours()
    keys = sorted(k.rsplit("/", 1)[0] for k in g if k.endswith("/codes"))
    assert len(keys) >= 40
    for key in keys:
        dtype, name, b, gs = key.split("/")
        bits, group = int(b[1:]), int(gs[1:])
        x = _x(g, dtype)
        c, s, z = ours[name][0](x, group, bits)
        ref_c = g[key + "/codes"]
        got = c.cpu().numpy()
        nan_group = ref_c == Q.INT32_MIN
        # all-zero groups: the reference's 0/0 gives INT32_MIN, the packed format 0
        assert (got[nan_group] == 0).all(), key
        np.testing.assert_array_equal(got[~nan_group], ref_c[~nan_group], err_msg=key)
        np.testing.assert_array_equal(_bits16(s), _golden_bits(g[key + "/scale"], dtype), err_msg=key)
        np.testing.assert_array_equal(_bits16(z), _golden_bits(g[key + "/zp"], dtype), err_msg=key)
        if key + "/deq" in g:
            # dequantized values agree everywhere, the all-zero groups included
            d = ours[name][1](c, s, z, group)
            np.testing.assert_array_equal(d.cpu().numpy(), g[key + "/deq"], err_msg=key)


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("name", FUNCS)
def test_quantize_vs_oracle_larger(dtype, bits, name):
    """C0-shaped K ([1, 8, 4096, 128]) through every quantizer vs the oracle."""
    k, v = synth_kv(1, 8, 4096, dtype=dtype, seed=bits)
    x = k if "channel" in name else v
    ours = _ours()
    c, s, z = ours[name][0](x, 32, bits)
    xo = to_np32(x)
    axis = xo.ndim - 1 if "channel" in name else xo.ndim - 2
    fn = Q.quantize_sym if "_sym" in name else Q.quantize_asym
    rc, rs, rz = fn(xo, 32, bits, axis, dtype)
    rc = np.where(rc == Q.INT32_MIN, 0, rc)
    np.testing.assert_array_equal(c.cpu().numpy(), rc)
    np.testing.assert_array_equal(to_np32(s), rs)
    np.testing.assert_array_equal(to_np32(z), rz)
    # codes use the full range (sanity on the synthetic distribution)
    top = (1 << (bits - 1)) - 1 if "_sym" in name else (1 << bits) - 1
    assert c.max().item() == top


def test_bad_inputs_raise():
    from innerq_b200 import quant as M
    from innerq_b200._lib import InnerqError
    x = torch.randn(1, 1, 64, 128, device="cuda", dtype=torch.float16)
    with pytest.raises(AssertionError):
        M.quantize_tokendim_sym(x[:, :, :48], 32, 4)  # quant.py:99 divisibility
    with pytest.raises(NotImplementedError):
        M.quantize_channeldim_sym(x, 32, 8)
    with pytest.raises(NotImplementedError):
        M.quantize_channeldim_sym(torch.randn(1, 1, 64, 64, device="cuda", dtype=torch.float16), 32, 4)
    with pytest.raises(RuntimeError):
        M.quantize_channeldim_sym(x.cpu(), 32, 4)
    with pytest.raises(ValueError):
        M.QMode.from_str("nope")
    assert InnerqError is not None
