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


def _boundary_rows(dtype, bits, asym, n_rows=512, seed=0):
    """Rows of groups of 32 whose elements sit on and a few dtype ulps around
    the values where |x| / s (or (x - min) / s) crosses a half-integer, the
    cases where the rounding of the quotient decides the code."""
    rng = np.random.default_rng(seed)
    qmax = (1 << bits) - 1 if asym else (1 << (bits - 1)) - 1
    out = np.zeros((n_rows, 128), np.float32)
    for r in range(n_rows):
        for g in range(4):
            M = float(Q.rnd(np.float32(rng.uniform(0.05, 30.0)), dtype))
            lo = float(Q.rnd(np.float32(-rng.uniform(0.0, 5.0)), dtype)) if asym else 0.0
            rng_ = float(Q.rnd(np.float32(M - lo), dtype)) if asym else M
            s = float(Q.rnd(np.float32(rng_ / qmax), dtype))
            vals = [M, lo] if asym else [M]
            while len(vals) < 32:
                k = rng.integers(0, qmax)
                base = Q.rnd(np.float32(lo + (k + 0.5) * s), dtype)
                bits16 = (base.astype(np.float16).view(np.uint16) if dtype == "fp16"
                          else Q.f32_to_bf16_bits(base))
                nbi = int(bits16) + int(rng.integers(-3, 4))
                if not 0 <= nbi <= 0xFFFF:
                    continue
                nb = np.uint16(nbi)
                v = (np.array([nb], np.uint16).view(np.float16).astype(np.float32)[0] if dtype == "fp16"
                     else Q.bf16_bits_to_f32(np.array([nb]))[0])
                if not np.isfinite(v) or v > M or v < lo:
                    continue
                if not asym and rng.integers(0, 2):
                    v = -v
                vals.append(v)
            out[r, 32 * g:32 * g + 32] = rng.permutation(np.array(vals, np.float32))
    return out[None, None]


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("asym", [False, True])
@pytest.mark.parametrize("over", ["channel", "token"])
def test_quantize_half_integer_boundaries(dtype, bits, asym, over):
    """Quantizers on inputs built around the rounding boundaries of the
    quotient (the fast path's fallback cases) vs the oracle; token groups get
    the same groups transposed onto the token axis."""
    xo = _boundary_rows(dtype, bits, asym, n_rows=512 if over == "channel" else 128,
                        seed=bits + 10 * asym)
    if over == "token":
        xo = np.ascontiguousarray(xo.swapaxes(-1, -2))
    x = torch.from_numpy(xo).to(TDT[dtype]).cuda()
    ours = _ours()[f"{over}_{'asym' if asym else 'sym'}"][0]
    c, s, z = ours(x, 32, bits)
    fn = Q.quantize_asym if asym else Q.quantize_sym
    rc, rs, rz = fn(to_np32(x), 32, bits, 3 if over == "channel" else 2, dtype)
    rc = np.where(rc == Q.INT32_MIN, 0, rc)
    np.testing.assert_array_equal(c.cpu().numpy(), rc)
    np.testing.assert_array_equal(to_np32(s), rs)
    np.testing.assert_array_equal(to_np32(z), rz)
