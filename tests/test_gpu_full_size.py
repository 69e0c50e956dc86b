"""Parity of the fused decode attention at the sizes the benchmark and the
BASELINE configurations use, one layer each, against an fp64 attention over
the reference fp32 dequantization (cache.py:235-281 with quant.py:83-93,
121-131; computed on the GPU by the reference-format unpack and dequantize
kernels, which are bit-exact with the reference fixtures and independent of
the fused kernel).  The bar is the one of the 1e-3 relative tolerance plus the
model dtype's rounding of each output element.

Full-size inputs cannot go through the CPU oracle in seconds; the small-size
tests pin the same kernels to the oracle and the fixtures."""
import types

import pytest
import torch

from tests._util import assert_attn_close, cfg, gpu_ref_attention, synth_kv_dev

pytestmark = pytest.mark.gpu


def _bench_kw(bits, group, v_over_token=True, mode="symmetric"):
    """The cache configuration bench.py uses (sink 32, recent 96, K normalised,
    K flush 1, V flush max(32, group) for token groups)."""
    return dict(k_bits=bits, v_bits=bits, key_group_size=group, value_group_size=group,
                key_flush_size=1, value_flush_size=max(32, group) if v_over_token else 32,
                key_w_sink=32, value_w_sink=32, key_w_recent=96, value_w_recent=96,
                key_normalize=True, value_quantize_over_token=v_over_token,
                key_quantize_mode=mode, value_quantize_mode=mode)


def _run(kw, B, Hkv, Hq, S, steps=3, seed=0):
    from innerq_b200.cache import InnerqDynamicLayer
    layer = InnerqDynamicLayer(cfg(**kw), 0)
    k, v = synth_kv_dev(B, Hkv, S, seed=seed)
    layer.update(k[:, :, :S - steps], v[:, :, :S - steps])
    for t in range(S - steps, S):
        layer.update(k[:, :, t:t + 1], v[:, :, t:t + 1])
    del k, v
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    q = torch.randn((B, Hq, 1, 128), device="cuda", generator=g).half()
    out = layer.attend(q)
    assert layer.get_seq_length() == S
    ref = gpu_ref_attention(layer, q)
    assert_attn_close(out, ref)
    del layer
    torch.cuda.empty_cache()


def test_c1_bench_config_b32():
    """C1 at the benchmark's batch: B 32, Hq 32 / Hkv 8, 32768 tokens, 4-bit G32."""
    _run(_bench_kw(4, 32), 32, 8, 32, 32768)


def test_c1_values_over_channels_b32():
    """C1 B32 with values grouped along head_dim (the BASELINE-literal layout)."""
    _run(_bench_kw(4, 32, v_over_token=False), 32, 8, 32, 32768, seed=3)


def test_c1_asymmetric_b32():
    _run(_bench_kw(4, 32, mode="asymmetric"), 32, 8, 32, 32768, seed=4)


def test_c1_kivi_b32():
    """The kivi preset (run_lmeval.sh:54-72: 2-bit asymmetric keys grouped over
    tokens, values over channels, recent 128, no sink) at C1 B32 x 32768."""
    kw = dict(k_bits=2, v_bits=2, key_group_size=32, value_group_size=32, key_flush_size=32,
              value_flush_size=1, key_w_recent=128, value_w_recent=128, key_quantize_over_token=True,
              value_quantize_over_token=False, key_quantize_mode="asymmetric",
              value_quantize_mode="asymmetric")
    _run(kw, 32, 8, 32, 32768, steps=40, seed=6)


def test_c4_shape_131072():
    """C4: 70B attention shape (Hq 64 / Hkv 8, GQA 8), B 8, 131072 tokens, 2-bit K and V, G32."""
    _run(_bench_kw(2, 32), 8, 8, 64, 131072, seed=5)


@pytest.mark.parametrize("bits,group", [(2, 64), (2, 128), (3, 64), (3, 128)])
def test_c2_65536(bits, group):
    """C2 at its longest context: B 16, 65536 tokens, 2/3-bit, G 64/128."""
    _run(_bench_kw(bits, group), 16, 8, 32, 65536, seed=10 * bits + group)


def test_graph_replay_70_steps_vs_reference():
    """A decode step recorded once and replayed 70 times (more than two V
    flushes of 32 plus the prefill window): the last step's output against the
    reference dequantization of the cache graph mode left behind."""
    from innerq_b200.cache import DynamicCache, InnerqDynamicLayer
    kw = dict(_bench_kw(4, 32), _attn_implementation="innerq")
    B, H, R, T0, steps = 4, 8, 4, 4096, 70
    k, v = synth_kv_dev(B, H, T0 + steps, seed=21)
    layer = InnerqDynamicLayer(types.SimpleNamespace(**kw), 0)
    layer.update(k[:, :, :T0], v[:, :, :T0])
    cache = DynamicCache()
    cache.layers.append(layer)
    cache.graph_begin(steps)
    k_in, v_in = torch.empty_like(k[:, :, :1]), torch.empty_like(v[:, :, :1])
    g = torch.Generator(device="cuda").manual_seed(22)
    q_in = torch.randn((B, H * R, 1, 128), device="cuda", generator=g).half()
    out = torch.empty((B, H * R, 128), dtype=torch.float16, device="cuda")
    stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            cache.graph_advance()
            layer.update(k_in, v_in)
            layer.attend(q_in, out=out)
    torch.cuda.synchronize()
    for i in range(steps):
        k_in.copy_(k[:, :, T0 + i:T0 + i + 1])
        v_in.copy_(v[:, :, T0 + i:T0 + i + 1])
        graph.replay()
    torch.cuda.synchronize()
    got = out.clone()
    assert cache.graph_end() == steps
    assert layer.get_seq_length() == T0 + steps
    assert_attn_close(got, gpu_ref_attention(layer, q_in))


def test_graph_end_rejects_steps_past_the_reservation():
    """graph_begin(n) reserves n steps; a counter advanced past n (no kernel
    run) makes graph_end raise instead of handing back a cache that lost
    tokens."""
    from innerq_b200.cache import DynamicCache, InnerqDynamicLayer
    layer = InnerqDynamicLayer(cfg(_attn_implementation="innerq", **_bench_kw(4, 32)), 0)
    k, v = synth_kv_dev(1, 2, 300, seed=30)
    layer.update(k, v)
    cache = DynamicCache()
    cache.layers.append(layer)
    cache.graph_begin(3)
    for _ in range(5):
        cache.graph_advance()
    with pytest.raises(RuntimeError, match="reserved"):
        cache.graph_end()
