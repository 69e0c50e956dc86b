"""Saving and restoring the packed cache (DynamicCache.save / load): a cache
restored from disk must hold the same content bit for bit (the materialised
K/V) and continue exactly like the original: the same fused attention output
(or materialised K/V) and the same appends, step after step."""
import pytest
import torch

from tests._util import synth_kv, synth_q

pytestmark = pytest.mark.gpu

PRESETS = {
    # innerq_base (run_lmeval.sh): 3-bit, normalised keys, sinks, recent windows
    "innerq_base": dict(k_bits=3, v_bits=3, key_flush_size=1, value_flush_size=32, key_w_sink=32,
                        value_w_sink=32, key_w_recent=96, value_w_recent=96, key_normalize=True),
    # innerq_hybrid: hybrid values over tokens
    "innerq_hybrid": dict(k_bits=3, v_bits=2, key_flush_size=1, value_flush_size=32, key_w_sink=32,
                          value_w_sink=32, key_w_recent=96, value_w_recent=96, key_normalize=True,
                          value_quantize_mode="hybrid"),
    # kivi: asymmetric keys over tokens, values over channels
    "kivi": dict(k_bits=2, v_bits=2, key_flush_size=32, value_flush_size=1, key_w_recent=128,
                 value_w_recent=128, key_quantize_over_token=True, value_quantize_over_token=False,
                 key_quantize_mode="asymmetric", value_quantize_mode="asymmetric"),
    # values grouped over channels, bf16
    "v_channels_bf16": dict(k_bits=4, v_bits=4, key_flush_size=1, value_flush_size=32,
                            value_quantize_over_token=False, key_w_recent=32, value_w_recent=32),
}


class _Cfg:
    """A model config as DynamicCache reads it (decoder text config, layer count)."""

    def __init__(self, n_layers, **kw):
        self.num_hidden_layers = n_layers
        self._attn_implementation = "innerq"
        for k, v in kw.items():
            setattr(self, k, v)

    def get_text_config(self, decoder=True):
        return self


@pytest.mark.parametrize("name", list(PRESETS))
def test_save_load_continues_bit_for_bit(name, tmp_path):
    from innerq_b200.cache import DynamicCache
    dtype = "bf16" if "bf16" in name else "fp16"
    config = _Cfg(2, **PRESETS[name])
    B, H, R, T0, before, after = 2, 2, 4, 700, 9, 40
    ks, vs = zip(*(synth_kv(B, H, T0 + before + after, dtype=dtype, seed=7 + i) for i in range(2)))
    qs = [synth_q(B, H * R, dtype=dtype, seed=200 + i) for i in range(after)]
    a = DynamicCache(config=config)
    for li, layer in enumerate(a.layers):
        layer.update(ks[li][:, :, :T0], vs[li][:, :, :T0])
        for t in range(T0, T0 + before):
            layer.update(ks[li][:, :, t:t + 1], vs[li][:, :, t:t + 1])
    path = tmp_path / "cache.pt"
    a.save(path)
    b = DynamicCache.load(path, config)
    for la, lb in zip(a.layers, b.layers):
        assert la.get_seq_length() == lb.get_seq_length() == T0 + before
        for x, y in zip(la.get_deq_tensors(), lb.get_deq_tensors()):
            assert torch.equal(x, y)
    # both continue: same appends, same attention output
    for i in range(after):
        t = T0 + before + i
        for li in range(2):
            la, lb = a.layers[li], b.layers[li]
            ra = la.update(ks[li][:, :, t:t + 1], vs[li][:, :, t:t + 1])
            rb = lb.update(ks[li][:, :, t:t + 1], vs[li][:, :, t:t + 1])
            if la._fusable():
                assert torch.equal(la.attend(qs[i]), lb.attend(qs[i]))
            else:
                assert torch.equal(ra[0], rb[0]) and torch.equal(ra[1], rb[1])
    for la, lb in zip(a.layers, b.layers):
        for x, y in zip(la.get_deq_tensors(), lb.get_deq_tensors()):
            assert torch.equal(x, y)


def test_load_rejects_other_config(tmp_path):
    from innerq_b200.cache import DynamicCache
    config = _Cfg(1, **PRESETS["innerq_base"])
    a = DynamicCache(config=config)
    k, v = synth_kv(1, 2, 300, seed=3)
    a.layers[0].update(k, v)
    path = tmp_path / "cache.pt"
    a.save(path)
    other = _Cfg(1, **dict(PRESETS["innerq_base"], k_bits=4))
    with pytest.raises(ValueError, match="bits"):
        DynamicCache.load(path, other)
    with pytest.raises(ValueError, match="layers"):
        DynamicCache.load(path, _Cfg(2, **PRESETS["innerq_base"]))
