"""Graph mode: a decode step (append + fused attention) recorded once in a
CUDA graph and replayed, the per-step cache state coming from a device step
counter.  Each replayed step must give the eager step's attention output, and
after graph_end the packed stores and recent windows must equal the eager
ones bit for bit."""
import numpy as np
import pytest
import torch

from tests._util import assert_close_rel, cfg, synth_kv, synth_q, to_np32

pytestmark = pytest.mark.gpu

PRESETS = {
    "innerq_base": dict(k_bits=3, v_bits=3, key_flush_size=1, value_flush_size=32, key_w_sink=32,
                        value_w_sink=32, key_w_recent=96, value_w_recent=96, key_normalize=True),
    "v_channels": dict(k_bits=4, v_bits=4, key_flush_size=1, value_flush_size=32,
                       value_quantize_over_token=False, key_w_recent=32, value_w_recent=32),
    # kivi (run_lmeval.sh:54-72): keys grouped over tokens, values over channels
    "kivi": dict(k_bits=2, v_bits=2, key_flush_size=32, value_flush_size=1, key_w_recent=128,
                 value_w_recent=128, key_quantize_over_token=True, value_quantize_over_token=False,
                 key_quantize_mode="asymmetric", value_quantize_mode="asymmetric"),
    "gqa8_2bit_asym": dict(k_bits=2, v_bits=2, key_flush_size=1, value_flush_size=32,
                           key_quantize_mode="asymmetric", value_quantize_mode="asymmetric",
                           key_w_sink=4, value_w_sink=4),
}


@pytest.mark.parametrize("name", list(PRESETS))
def test_graph_replay_matches_eager_steps(name):
    from innerq_b200.cache import DynamicCache, InnerqDynamicLayer
    kw = dict(PRESETS[name], _attn_implementation="innerq")
    R = 8 if "gqa8" in name else 4
    B, H, T0, steps = 2, 2, 700, 40
    k, v = synth_kv(B, H, T0 + steps, seed=5)
    qs = [synth_q(B, H * R, seed=100 + i) for i in range(steps)]
    eager, graphed = InnerqDynamicLayer(cfg(**kw), 0), InnerqDynamicLayer(cfg(**kw), 0)
    for layer in (eager, graphed):
        layer.update(k[:, :, :T0], v[:, :, :T0])
    ref = []
    for i in range(steps):
        t = T0 + i
        eager.update(k[:, :, t:t + 1], v[:, :, t:t + 1])
        ref.append(to_np32(eager.attend(qs[i])))

    cache = DynamicCache()
    cache.layers.append(graphed)
    step = cache.graph_begin(steps)
    k_in = torch.empty_like(k[:, :, :1])
    v_in = torch.empty_like(v[:, :, :1])
    q_in = torch.empty_like(qs[0])
    out = torch.empty((B, H * R, 128), dtype=k.dtype, device=k.device)
    stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            cache.graph_advance()
            graphed.update(k_in, v_in)
            graphed.attend(q_in, out=out)
    torch.cuda.synchronize()
    assert int(step.item()) == 0  # recording runs nothing
    for i in range(steps):
        t = T0 + i
        k_in.copy_(k[:, :, t:t + 1])
        v_in.copy_(v[:, :, t:t + 1])
        q_in.copy_(qs[i])
        graph.replay()
        torch.cuda.synchronize()
        # the split count is fixed at recording time: only the fp32 summation
        # order differs, which can move an element by one ulp of the fp16 output
        got = to_np32(out)
        err = np.abs(got - ref[i])
        assert (err <= 1e-4 * np.abs(ref[i]).max() + 2.0 ** -10 * np.abs(ref[i])).all(), \
            f"{name} step {i}: max err {err.max():.3e}"
    assert cache.graph_end() == steps
    assert graphed.get_seq_length() == eager.get_seq_length()
    for a, b in ((graphed.key_side, eager.key_side), (graphed.value_side, eager.value_side)):
        assert (a.n_q, a.n_recent) == (b.n_q, b.n_recent)
        for x, y in zip(a.ref_views(), b.ref_views()):
            if x is not None:
                np.testing.assert_array_equal(to_np32(x), to_np32(y))
        np.testing.assert_array_equal(to_np32(a.recent), to_np32(b.recent))
    # eager steps continue from the state graph mode left
    t = T0 + steps - 1
    graphed.update(k[:, :, t:t + 1], v[:, :, t:t + 1])
    eager.update(k[:, :, t:t + 1], v[:, :, t:t + 1])
    assert_close_rel(to_np32(graphed.attend(qs[0])), to_np32(eager.attend(qs[0])), 1e-6, "after")
