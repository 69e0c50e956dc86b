"""GPU parity of the cache layer (append + materialised K/V) and of the fused
decode attention kernel, against the reference fixtures and the oracle."""
import math

import numpy as np
import pytest
import torch

from oracle import cache_ref as C
from tests._util import (TDT, assert_close_rel, cfg, merge_np, oracle_layer, synth_kv, synth_q,
                         to_np32)

pytestmark = pytest.mark.gpu

PRESET_KW = {
    "innerq_base": C.PRESETS["innerq_base"],
    "kivi": C.PRESETS["kivi"],
    # scripts/run_lmeval.sh:134-153; V hybrid (quant.py:133-176), materialised
    "innerq_hybrid": dict(C.PRESETS["innerq_small"], value_quantize_mode="hybrid"),
    "innerq_small": C.PRESETS["innerq_small"],
    "default4": dict(k_bits=4, v_bits=4),
    "asym4_norm": dict(k_bits=4, v_bits=4, key_quantize_mode="asymmetric",
                       value_quantize_mode="asymmetric", key_normalize=True,
                       key_w_sink=4, value_w_sink=4, value_group_size=64,
                       value_flush_size=64),
}


def _from_golden(arr, dtype):
    if dtype == "bf16":
        return torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16).cuda()
    return torch.from_numpy(arr.copy()).cuda()


@pytest.mark.parametrize("name", list(PRESET_KW))
def test_layer_matches_reference_fixture(cache_golden, name):
    from innerq_b200.cache import InnerqDynamicLayer
    g = cache_golden
    p = f"cache/{name}"
    dtype = str(g[p + "/dtype"])
    kin = _from_golden(g[p + "/k_in"], dtype)
    vin = _from_golden(g[p + "/v_in"], dtype)
    layer = InnerqDynamicLayer(cfg(**PRESET_KW[name]), 0)
    T0 = kin.shape[2] - 40
    k0, v0 = layer.update(kin[:, :, :T0], vin[:, :, :T0])
    assert k0.data_ptr() == kin.data_ptr()  # prefill returns the raw states (cache.py:390-392)
    trace = []
    for t in range(T0, kin.shape[2]):
        K, V = layer.update(kin[:, :, t:t + 1], vin[:, :, t:t + 1])
        ks, vs = layer.key_side, layer.value_side
        trace.append([ks.n_sink, ks.n_q, ks.n_recent, vs.n_sink, vs.n_q, vs.n_recent])
    np.testing.assert_array_equal(np.array(trace), g[p + "/trace"])
    # materialised K/V bit-exact with the reference's get_deq_tensors
    np.testing.assert_array_equal(to_np32(K), to_np32(_from_golden(g[p + "/K"], dtype)))
    np.testing.assert_array_equal(to_np32(V), to_np32(_from_golden(g[p + "/V"], dtype)))
    if p + "/kf" in g:
        np.testing.assert_array_equal(to_np32(layer.key_normalization_factor),
                                      to_np32(_from_golden(g[p + "/kf"], dtype)))
    # fused attention over the packed store vs the reference's sdpa on the K/V it
    # returns.  Those are cast to the model dtype (cache.py:279-280), which by
    # itself moves the output by up to a few 1e-3 at 3 bits (1e-2 in bf16); the
    # 1e-3 bar is checked against the fp32 dequantize-then-matmul in
    # test_decode_attention_vs_oracle.
    if layer.key_side.fusable and layer.value_side.fusable:
        q = _from_golden(g[p + "/q"], dtype)
        out = layer.attend(q)
        assert_close_rel(to_np32(out), g[p + "/o"][:, :, 0], 3e-2 if dtype == "bf16" else 1e-2, name)
    assert layer.get_seq_length() == kin.shape[2]
    assert layer.get_mask_sizes(1) == (kin.shape[2] + 1, 0)


def test_kivi_layout_materialised_and_fused():
    """KIVI (keys grouped over tokens, values over channels, asymmetric) runs
    through the packed store and the dequant kernel, bit-exact with the
    reference, and the fused kernel reads it (1e-3 vs the fp32 dequantize);
    GQA 8 and normalised token-grouped keys are refused by the fused kernel."""
    from innerq_b200.attention import decode_attention
    from innerq_b200.cache import InnerqDynamicLayer
    from innerq_b200._lib import InnerqError
    layer = InnerqDynamicLayer(cfg(**C.PRESETS["kivi"]), 0)
    k, v = synth_kv(1, 2, 240, seed=3)
    ol = oracle_layer(C.PRESETS["kivi"], "fp16")
    layer.update(k[:, :, :200], v[:, :, :200])
    ol.update(to_np32(k[:, :, :200]), to_np32(v[:, :, :200]))
    for t in range(200, 240):
        K, V = layer.update(k[:, :, t:t + 1], v[:, :, t:t + 1])
        Kr, Vr = ol.update(to_np32(k[:, :, t:t + 1]), to_np32(v[:, :, t:t + 1]))
    np.testing.assert_array_equal(to_np32(K), Kr)
    np.testing.assert_array_equal(to_np32(V), Vr)
    assert layer.key_side.fusable and layer._fusable()
    q = synth_q(1, 8)
    K32, V32 = _oracle_kv32(ol)
    ref32, _ = C.attention(to_np32(q), K32, V32)
    out = decode_attention(q, layer.key_side, layer.value_side)
    assert_close_rel(to_np32(out), ref32[:, :, 0], 1e-3, "kivi fused")
    with pytest.raises(InnerqError):
        decode_attention(synth_q(1, 16), layer.key_side, layer.value_side)  # GQA 8


def _oracle_kv32(ol):
    """[sink | fp32 dequant (not cast) | recent] of the oracle layer."""
    out = []
    for side in (ol.k, ol.v):
        parts = [side.sink]
        d = side.dequant_fp32()
        if d is not None:
            parts.append(d)
        parts.append(side.recent)
        out.append(np.concatenate(parts, axis=-2))
    return out


CASES = [
    # (k_bits, v_bits, kmode, vmode, R, dtype, gk, gv, sink, recent, normalize, T0, steps)
    (4, 4, "symmetric", "symmetric", 4, "fp16", 32, 32, 0, 32, False, 1000, 5),
    (3, 3, "symmetric", "symmetric", 4, "fp16", 32, 32, 32, 96, True, 700, 40),
    (3, 2, "symmetric", "symmetric", 4, "bf16", 32, 32, 32, 96, True, 517, 33),
    (2, 2, "symmetric", "symmetric", 8, "fp16", 32, 32, 0, 32, False, 2048, 3),
    (4, 4, "asymmetric", "asymmetric", 4, "fp16", 32, 32, 4, 32, True, 900, 7),
    (2, 3, "asymmetric", "symmetric", 1, "bf16", 64, 64, 0, 32, False, 640, 2),
    (4, 2, "symmetric", "asymmetric", 2, "fp16", 128, 128, 0, 128, False, 1100, 2),
    (4, 4, "symmetric", "symmetric", 4, "fp16", 32, 32, 0, 32, False, 20, 3),   # all dense
    (4, 4, "symmetric", "symmetric", 4, "fp16", 32, 32, 0, 32, False, 33, 40),  # tiny middle
    (3, 3, "symmetric", "symmetric", 8, "bf16", 32, 32, 5, 7, True, 76, 31),    # odd sink
]


# values grouped over channels (the BASELINE-literal layout: groups along
# head_dim for K and V); value_flush_size 32 keeps whole packed tiles
CASES_VCH = [
    (4, 4, "symmetric", "symmetric", 4, "fp16", 32, 32, 0, 32, True, 1000, 5),
    (2, 2, "asymmetric", "asymmetric", 8, "bf16", 32, 32, 32, 96, False, 700, 40),
    (3, 3, "symmetric", "asymmetric", 1, "fp16", 64, 64, 4, 32, True, 517, 33),
    (4, 2, "asymmetric", "symmetric", 2, "fp16", 128, 128, 0, 64, False, 900, 3),
]


# keys grouped over tokens (KIVI, cache.py:87; presets kivi / kivi_sink of
# run_lmeval.sh): (case, values over tokens?, value flush)
CASES_KOT = [
    ((2, 2, "asymmetric", "asymmetric", 4, "fp16", 32, 32, 0, 128, False, 1000, 40), False, 1),
    ((2, 2, "asymmetric", "asymmetric", 4, "fp16", 32, 32, 32, 96, False, 700, 33), False, 1),
    ((4, 4, "symmetric", "symmetric", 2, "bf16", 64, 64, 0, 64, False, 900, 5), True, 64),
    ((3, 3, "asymmetric", "symmetric", 1, "fp16", 128, 32, 4, 32, False, 1060, 3), True, 32),
    ((2, 4, "symmetric", "asymmetric", 4, "fp16", 32, 32, 0, 32, False, 40, 30), False, 32),  # tiny middle
]


@pytest.mark.parametrize("case", CASES_KOT, ids=[f"k{i}" for i in range(len(CASES_KOT))])
def test_decode_attention_keys_over_tokens(case):
    c, vot, vflush = case
    _check_case(c, value_over_token=vot, key_over_token=True, value_flush=vflush)


@pytest.mark.parametrize("case", CASES, ids=[f"c{i}" for i in range(len(CASES))])
def test_decode_attention_vs_oracle(case):
    _check_case(case, value_over_token=True)


@pytest.mark.parametrize("case", CASES_VCH, ids=[f"v{i}" for i in range(len(CASES_VCH))])
def test_decode_attention_value_channel_groups(case):
    _check_case(case, value_over_token=False)


def _check_case(case, value_over_token, key_over_token=False, value_flush=None):
    from innerq_b200.attention import decode_attention, decode_attention_partials
    from innerq_b200.cache import InnerqDynamicLayer
    bk, bv, km, vm, R, dtype, gk, gv, sink, recent, norm, T0, steps = case
    if value_flush is None:
        value_flush = gv if value_over_token else 32
    kw = dict(k_bits=bk, v_bits=bv, key_quantize_mode=km, value_quantize_mode=vm,
              key_group_size=gk, value_group_size=gv, key_w_sink=sink, value_w_sink=sink,
              key_w_recent=recent, value_w_recent=recent, key_flush_size=gk if key_over_token else 1,
              value_flush_size=value_flush, key_normalize=norm,
              value_quantize_over_token=value_over_token, key_quantize_over_token=key_over_token)
    Hkv, B = 2, 2
    k, v = synth_kv(B, Hkv, T0 + steps, dtype=dtype, seed=T0)
    layer = InnerqDynamicLayer(cfg(**kw), 0)
    ol = oracle_layer(kw, dtype)
    layer.update(k[:, :, :T0], v[:, :, :T0])
    ol.update(to_np32(k[:, :, :T0]), to_np32(v[:, :, :T0]))
    for t in range(T0, T0 + steps):
        layer.update(k[:, :, t:t + 1], v[:, :, t:t + 1])
        Kr, Vr = ol.update(to_np32(k[:, :, t:t + 1]), to_np32(v[:, :, t:t + 1]))
    assert layer._fusable()
    q = synth_q(B, Hkv * R, dtype=dtype, seed=T0 + 1)
    qn = to_np32(q)
    # (1) the 1e-3 bar: reference fp32 dequantize (quant.py:121-131, cache.py:241-271)
    #     then matmul, softmax and matmul with fp32-or-better accumulation.  The
    #     output is rounded to the model dtype, which adds up to 2^-9 (bf16) or
    #     2^-12 (fp16) of each element on top.
    K32, V32 = _oracle_kv32(ol)
    ref32, logits = C.attention(qn, K32, V32)
    out = decode_attention(q, layer.key_side, layer.value_side)
    r = ref32[:, :, 0]
    ulp = 2.0 ** -8 if dtype == "bf16" else 2.0 ** -11
    err = np.abs(to_np32(out) - r)
    assert (err <= 1e-3 * np.abs(r).max() + ulp * np.abs(r)).all(), err.max()
    # (1b) the reference's returned K/V are cast to the dtype before sdpa; that
    #      cast alone moves the output by up to a few 1e-3 (more in bf16)
    ref, _ = C.attention(qn, Kr, Vr)
    assert_close_rel(to_np32(out), ref[:, :, 0], 3e-2 if dtype == "bf16" else 1e-2, "vs cast K/V")
    # (2) tight: fp64 merge of the partials vs the same fp32 dequant
    for ns in (0, 1, 7):
        po, pm, pl = decode_attention_partials(q, layer.key_side, layer.value_side, n_splits=ns)
        o64, lse2 = merge_np(po.cpu().numpy(), pm.cpu().numpy(), pl.cpu().numpy())
        assert_close_rel(o64, ref32[:, :, 0], 1e-4, f"tight n_splits={ns}")
        lse_ref = np.log2(np.exp(logits - logits.max(-1, keepdims=True)).sum(-1)) \
            + logits.max(-1) / math.log(2)
        np.testing.assert_allclose(lse2, lse_ref[:, :, 0], rtol=0, atol=2e-4)


def test_lse_merge_kernel_and_tile_ranges():
    """Partials of two disjoint tile ranges merged by the CUDA merge kernel equal
    the full pass (the context-sharding path)."""
    from innerq_b200.attention import (build_args, decode_attention, decode_attention_partials,
                                       lse_merge, plan)
    from innerq_b200.cache import InnerqDynamicLayer
    kw = dict(k_bits=4, v_bits=4, key_w_sink=32, value_w_sink=32, key_flush_size=1)
    layer = InnerqDynamicLayer(cfg(**kw), 0)
    k, v = synth_kv(2, 8, 5000, seed=11)
    layer.update(k, v)
    q = synth_q(2, 32, seed=12)
    full = decode_attention(q, layer.key_side, layer.value_side)
    n_tiles, _ = plan(build_args(q, layer.key_side, layer.value_side))
    cut = n_tiles // 3
    parts = [decode_attention_partials(q, layer.key_side, layer.value_side, tile_range=r)
             for r in ((0, cut), (cut, n_tiles))]
    po = torch.cat([p[0] for p in parts], dim=2)
    pm = torch.cat([p[1] for p in parts], dim=2)
    pl = torch.cat([p[2] for p in parts], dim=2)
    merged = lse_merge(po, pm, pl, torch.float16)
    assert_close_rel(to_np32(merged), to_np32(full), 2e-3, "sharded merge")


@pytest.mark.parametrize("B", [1, 8])
def test_full_size_context_32k(B):
    """C1 shape (S = 32768, Hq 32 / Hkv 8, 4-bit G32) against an fp64 attention
    over the reference fp32 dequantization, itself computed on the GPU by the
    reference-format unpack and dequantize kernels (independent of the fused
    attention kernel)."""
    from innerq_b200 import quant as M
    from innerq_b200.cache import InnerqDynamicLayer
    kw = dict(k_bits=4, v_bits=4, key_flush_size=1, key_normalize=True, key_w_sink=32,
              value_w_sink=32, key_w_recent=96, value_w_recent=96)
    layer = InnerqDynamicLayer(cfg(**kw), 0)
    k, v = synth_kv(B, 8, 32768, seed=5)
    layer.update(k, v)
    layer.update(*synth_kv(B, 8, 1, seed=6))
    q = synth_q(B, 32, seed=7)
    out = layer.attend(q)
    kd = M.dequantize_channeldim_sym(layer.keys_q, layer.keys_scale_factor, layer.keys_zp_sign, 32)
    kd = kd * layer.key_normalization_factor.float()
    vd = M.dequantize_tokendim_sym(layer.values_q, layer.values_scale_factor, layer.values_zp_sign, 32)
    K = torch.cat([layer.keys_sink.float(), kd, layer.keys_recent.float()], dim=2).double()
    V = torch.cat([layer.values_sink.float(), vd, layer.values_recent.float()], dim=2).double()
    kk = K.repeat_interleave(4, dim=1)
    vv = V.repeat_interleave(4, dim=1)
    ref = torch.softmax((q.double() @ kk.transpose(-1, -2)) / math.sqrt(128), dim=-1) @ vv
    r = to_np32(ref[:, :, 0])
    err = np.abs(to_np32(out) - r)
    assert (err <= 1e-3 * np.abs(r).max() + 2.0 ** -11 * np.abs(r)).all(), err.max()


def test_prefill_states_are_not_retained():
    """A layer without sink tokens keeps no view of the prefill tensors: after
    the caller drops them their memory is free again (a zero-size slice kept
    as the sink would hold the whole prefill K/V alive)."""
    from innerq_b200.cache import InnerqDynamicLayer
    layer = InnerqDynamicLayer(cfg(k_bits=4, v_bits=4, key_w_sink=0, value_w_sink=0), 0)
    k, v = synth_kv(4, 8, 8192, seed=31)
    torch.cuda.synchronize()
    layer.update(k, v)
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated()
    nbytes = k.numel() * k.element_size() + v.numel() * v.element_size()
    del k, v
    torch.cuda.synchronize()
    assert before - torch.cuda.memory_allocated() >= nbytes


HYBRID_CASES = [
    # (k_bits, v_bits, R, dtype, v_group, T0, steps)
    (3, 2, 4, "fp16", 32, 700, 40),   # the innerq_hybrid preset (scripts/run_lmeval.sh:133-151)
    (3, 2, 8, "bf16", 32, 517, 33),
    (4, 3, 4, "fp16", 64, 900, 5),
    (2, 4, 2, "fp16", 32, 640, 70),
]


@pytest.mark.parametrize("case", HYBRID_CASES, ids=[f"h{i}" for i in range(len(HYBRID_CASES))])
def test_hybrid_values_fused_vs_reference(case):
    """Hybrid values (quant.py:133-176) read by the fused kernel: symmetric or
    asymmetric codes per (group, dim) by the stored mask, against an fp64
    attention over the reference's fp32 hybrid dequantization."""
    from innerq_b200.cache import InnerqDynamicLayer
    from tests._util import gpu_ref_attention, hybrid_side_fp32, side_fp32
    bk, bv, R, dtype, gv, T0, steps = case
    kw = dict(k_bits=bk, v_bits=bv, key_flush_size=1, value_flush_size=gv, key_w_sink=32,
              value_w_sink=32, key_w_recent=96, value_w_recent=96, key_normalize=True,
              value_group_size=gv, value_quantize_mode="hybrid", _attn_implementation="innerq")
    Hkv, B = 2, 2
    k, v = synth_kv(B, Hkv, T0 + steps, dtype=dtype, seed=T0 + bv)
    layer = InnerqDynamicLayer(cfg(**kw), 0)
    layer.update(k[:, :, :T0], v[:, :, :T0])
    for t in range(T0, T0 + steps):
        layer.update(k[:, :, t:t + 1], v[:, :, t:t + 1])
    assert layer._fusable()
    q = synth_q(B, Hkv * R, dtype=dtype, seed=T0 + 1)
    out = layer.attend(q)
    ks = layer.key_side
    K = side_fp32(ks, ks.norm_f if ks.normalize else None).double()
    V = hybrid_side_fp32(layer.value_side).double()
    S = K.shape[2]
    qd = q[:, :, 0].double().view(B, Hkv, R, 128)
    ref = torch.softmax((qd @ K.transpose(-1, -2)) / math.sqrt(128), dim=-1) @ V
    r = to_np32(ref.reshape(B, Hkv * R, 128))
    ulp = 2.0 ** -8 if dtype == "bf16" else 2.0 ** -11
    err = np.abs(to_np32(out) - r)
    assert (err <= 1e-3 * np.abs(r).max() + ulp * np.abs(r)).all(), err.max()
    # and the materialised path agrees with the reference's own get_deq_tensors
    layer.fused = False
    Kd, Vd = layer.get_deq_tensors()
    np.testing.assert_array_equal(to_np32(Vd), to_np32(V.to(Vd.dtype)))
    assert S == T0 + steps
