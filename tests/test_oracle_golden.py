"""Pin the CPU oracle against fixtures produced by running the reference itself.

Every quantity the oracle restates (codes, scales, zero points, signs,
dequantized values, the key normalisation factor, the cache layer's returned
K/V after prefill + 40 decode steps, the flush trace) must match the
reference bit for bit; attention outputs within fp32 rounding.
"""
import numpy as np
import pytest

from oracle import quant_ref as Q
from oracle import cache_ref as C
from tests.conftest import golden_to_f32

FUNCS = {
    "channel_sym": Q.quantize_channeldim_sym,
    "token_sym": Q.quantize_tokendim_sym,
    "channel_asym": Q.quantize_channeldim_asym,
    "token_asym": Q.quantize_tokendim_asym,
}
DEQ = {
    "channel_sym": Q.dequantize_channeldim_sym,
    "token_sym": Q.dequantize_tokendim_sym,
    "channel_asym": Q.dequantize_channeldim_asym,
    "token_asym": Q.dequantize_tokendim_asym,
}


def _cases(g):
    keys = sorted(k.rsplit("/", 1)[0] for k in g if k.endswith("/codes"))
    return keys


def test_quant_bit_exact(quant_golden):
    g = quant_golden
    n = 0
    for key in _cases(g):
        dtype, name, b, gs = key.split("/")
        bits, group = int(b[1:]), int(gs[1:])
        x = golden_to_f32(g[f"{dtype}/x"], dtype)
        c, s, z = FUNCS[name](x, group, bits, dtype)
        np.testing.assert_array_equal(c, g[key + "/codes"], err_msg=key)
        np.testing.assert_array_equal(s, golden_to_f32(g[key + "/scale"], dtype), err_msg=key)
        np.testing.assert_array_equal(z, golden_to_f32(g[key + "/zp"], dtype), err_msg=key)
        if key + "/deq" in g:
            d = DEQ[name](c, s, z, group)
            ref = g[key + "/deq"]
            np.testing.assert_array_equal(d, ref, err_msg=key)
        n += 1
    assert n >= 40


def test_zero_group_codes_are_int_min(quant_golden):
    """The reference's all-zero group gives 0/0 -> INT32_MIN codes (a quirk the
    packed format replaces by code 0; dequantized values agree)."""
    c = quant_golden["fp16/channel_sym/b4/g32/codes"]
    assert (c[0, 0, 5, 0:32] == Q.INT32_MIN).all()


def test_norm_factor(quant_golden):
    for dtype in ("fp16", "bf16"):
        x = golden_to_f32(quant_golden[f"{dtype}/x"], dtype)
        f = Q.key_norm_factor(x, dtype)
        np.testing.assert_array_equal(f, golden_to_f32(quant_golden[f"{dtype}/norm/f"], dtype))
        xn = Q.normalize_keys(x, f, dtype)
        ref = golden_to_f32(quant_golden[f"{dtype}/norm/xn"], dtype)
        np.testing.assert_array_equal(np.nan_to_num(xn, nan=7.0), np.nan_to_num(ref, nan=7.0))


PRESET_KW = {
    "innerq_base": C.PRESETS["innerq_base"],
    "innerq_small": C.PRESETS["innerq_small"],
    "kivi": C.PRESETS["kivi"],
    "default4": dict(k_bits=4, v_bits=4),
    "asym4_norm": dict(k_bits=4, v_bits=4, key_quantize_mode="asymmetric",
                       value_quantize_mode="asymmetric", key_normalize=True,
                       key_w_sink=4, value_w_sink=4, value_group_size=64,
                       value_flush_size=64),
}


@pytest.mark.parametrize("name", list(PRESET_KW))
def test_cache_layer_bit_exact(cache_golden, name):
    g = cache_golden
    p = f"cache/{name}"
    dtype = str(g[p + "/dtype"])
    kin = golden_to_f32(g[p + "/k_in"], dtype)
    vin = golden_to_f32(g[p + "/v_in"], dtype)
    layer = C.OracleLayer(C.CacheConfig(**PRESET_KW[name]), dtype)
    T0 = kin.shape[2] - 40
    layer.update(kin[:, :, :T0], vin[:, :, :T0])
    trace = []
    for t in range(T0, kin.shape[2]):
        K, V = layer.update(kin[:, :, t:t + 1], vin[:, :, t:t + 1])
        trace.append([layer.k.sink.shape[2], layer.k.n_quantized(), layer.k.recent.shape[2],
                      layer.v.sink.shape[2], layer.v.n_quantized(), layer.v.recent.shape[2]])
    np.testing.assert_array_equal(np.array(trace), g[p + "/trace"])
    np.testing.assert_array_equal(K, golden_to_f32(g[p + "/K"], dtype))
    np.testing.assert_array_equal(V, golden_to_f32(g[p + "/V"], dtype))
    q = golden_to_f32(g[p + "/q"], dtype)
    o, _ = C.attention(q, K, V)
    np.testing.assert_allclose(o, g[p + "/o"], rtol=1e-5, atol=1e-5)


def test_lse_merge_matches_full_softmax():
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, 4, 1, 64))
    k = rng.standard_normal((1, 1, 100, 64))
    v = rng.standard_normal((1, 1, 100, 64))
    full, _ = C.attention(q, k, v)
    os_, ms, ls = [], [], []
    for a, b in ((0, 37), (37, 64), (64, 100)):
        logits = np.einsum("bhqd,bsd->bhqs", q, k[:, 0, a:b]) / 8.0
        m = logits.max(-1)
        p = np.exp(logits - m[..., None])
        os_.append(np.einsum("bhqs,bsd->bhqd", p, v[:, 0, a:b]))
        ms.append(m)
        ls.append(p.sum(-1))
    o = C.lse_merge(np.stack(os_, -2), np.stack(ms, -1), np.stack(ls, -1))
    np.testing.assert_allclose(o, full, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("name", list(PRESET_KW))
def test_torch_baseline_layer_bit_exact(cache_golden, name):
    """The torch CPU restatement timed as the CPU baseline returns the
    reference's K/V bit for bit after prefill + 40 decode steps."""
    import torch

    from oracle.torch_ref import TorchRefLayer, consumer_attention
    g = cache_golden
    p = f"cache/{name}"
    dtype = str(g[p + "/dtype"])
    tdt = torch.float16 if dtype == "fp16" else torch.bfloat16
    kin = torch.from_numpy(golden_to_f32(g[p + "/k_in"], dtype)).to(tdt)
    vin = torch.from_numpy(golden_to_f32(g[p + "/v_in"], dtype)).to(tdt)
    layer = TorchRefLayer(**PRESET_KW[name])
    T0 = kin.shape[2] - 40
    layer.update(kin[:, :, :T0], vin[:, :, :T0])
    for t in range(T0, kin.shape[2]):
        K, V = layer.update(kin[:, :, t:t + 1], vin[:, :, t:t + 1])
    np.testing.assert_array_equal(K.float().numpy(), golden_to_f32(g[p + "/K"], dtype))
    np.testing.assert_array_equal(V.float().numpy(), golden_to_f32(g[p + "/V"], dtype))
    q = torch.from_numpy(golden_to_f32(g[p + "/q"], dtype)).to(tdt)
    o = consumer_attention(q, K, V).float().numpy()
    ref = g[p + "/o"]
    assert np.abs(o - ref).max() <= 2e-2 * np.abs(ref).max()
