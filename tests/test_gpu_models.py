"""The model hooks (src/innerq/models) on the GPU: a small random Llama with
an InnerQ cache decodes through the fused "innerq" attention and matches the
same model decoding through the materialised (reference-exact) K/V + sdpa."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

QCFG = dict(k_bits=4, v_bits=4, key_group_size=32, value_group_size=32, key_flush_size=1,
            value_flush_size=32, key_w_recent=16, value_w_recent=16, key_w_sink=4, value_w_sink=4,
            key_normalize=True)


def _model(cls_name):
    from transformers import LlamaConfig, MistralConfig
    from innerq_b200 import models
    torch.manual_seed(0)
    if cls_name == "llama":
        c = LlamaConfig(num_hidden_layers=2, hidden_size=512, num_attention_heads=4,
                        num_key_value_heads=1, head_dim=128, intermediate_size=256,
                        vocab_size=512, **QCFG)
        m = models.InnerqLlamaForCausalLM(c)
    else:
        c = MistralConfig(num_hidden_layers=2, hidden_size=512, num_attention_heads=8,
                          num_key_value_heads=2, head_dim=128, intermediate_size=256,
                          vocab_size=512, sliding_window=None, **QCFG)
        m = models.InnerqMistralForCausalLM(c)
    return m.to("cuda", torch.float16).eval()


@pytest.mark.parametrize("arch", ["llama", "mistral"])
def test_fused_decode_matches_materialised(arch):
    from innerq_b200.cache import DynamicCache, InnerqDynamicLayer
    m = _model(arch)
    ids = torch.randint(0, 512, (2, 100), device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    steps = torch.randint(0, 512, (2, 40), device="cuda", generator=torch.Generator("cuda").manual_seed(2))
    cfg = m.config.get_text_config(decoder=True)

    def run(fused):
        cache = DynamicCache(config=cfg)
        for layer in cache.layers:
            assert isinstance(layer, InnerqDynamicLayer)
            layer.fused = fused
        out = m(ids, past_key_values=cache, use_cache=True)
        logits = [out.logits[:, -1].float()]
        for t in range(40):  # the same (teacher-forced) tokens for both runs
            out = m(steps[:, t:t + 1], past_key_values=cache, use_cache=True)
            logits.append(out.logits[:, -1].float())
        return torch.stack(logits, 1)

    with torch.no_grad():
        a = run(True)
        b = run(False)
    scale = b.abs().max().item()
    err = (a - b).abs().max().item()
    assert err <= 2e-2 * scale, (err, scale)


def test_generate_installs_innerq_cache():
    from innerq_b200.cache import DynamicCache
    m = _model("llama")
    ids = torch.randint(0, 512, (1, 68), device="cuda")
    with torch.no_grad():
        out = m.generate(ids, max_new_tokens=5, do_sample=False, return_dict_in_generate=True)
    assert isinstance(out.past_key_values, DynamicCache)
    assert out.sequences.shape[1] == 73
    assert out.past_key_values.layers[0].get_seq_length() == 72


def test_sliding_window_layer_returns_the_window():
    """cache.py:421-461: a sliding layer returns the tail of what a full layer
    returns for the same tokens, as many tokens as its get_mask_sizes
    describes (window - 1 + 1 once the window is full; the reference's
    [:, :, -window, :] at cache.py:443-444 would keep one token)."""
    from innerq_b200.cache import InnerqDynamicLayer, InnerqDynamicSlidingWindowLayer
    from tests._util import cfg, synth_kv
    W = 48
    full = InnerqDynamicLayer(cfg(**QCFG), 0)
    sl = InnerqDynamicSlidingWindowLayer(cfg(**QCFG), 0, sliding_window=W)
    k, v = synth_kv(2, 2, 140, seed=9)
    for layer in (full, sl):
        layer.update(k[:, :, :100], v[:, :, :100])
    for t in range(100, 140):
        kv_len, kv_off = sl.get_mask_sizes(1)
        Kf, Vf = full.update(k[:, :, t:t + 1], v[:, :, t:t + 1])
        Ks, Vs = sl.update(k[:, :, t:t + 1], v[:, :, t:t + 1])
        assert Ks.shape[2] == kv_len == W and kv_off == t - W + 1
        torch.testing.assert_close(Ks, Kf[:, :, -W:], rtol=0, atol=0)
        torch.testing.assert_close(Vs, Vf[:, :, -W:], rtol=0, atol=0)
    assert sl.get_max_cache_shape() == W and sl.get_seq_length() == 140


def test_mistral_sliding_window_decodes():
    """A Mistral config with a sliding window gets sliding InnerQ layers and
    decodes through them (HF sliding mask + the cropped dequantized window)."""
    from transformers import MistralConfig
    from innerq_b200 import models
    from innerq_b200.cache import InnerqDynamicSlidingWindowLayer
    torch.manual_seed(0)
    c = MistralConfig(num_hidden_layers=2, hidden_size=512, num_attention_heads=8,
                      num_key_value_heads=2, head_dim=128, intermediate_size=256,
                      vocab_size=512, sliding_window=64, **QCFG)
    m = models.InnerqMistralForCausalLM(c).to("cuda", torch.float16).eval()
    ids = torch.randint(0, 512, (2, 100), device="cuda", generator=torch.Generator("cuda").manual_seed(3))
    with torch.no_grad():
        out = m.generate(ids, max_new_tokens=30, do_sample=False, return_dict_in_generate=True)
    cache = out.past_key_values
    assert all(isinstance(l, InnerqDynamicSlidingWindowLayer) for l in cache.layers)
    assert out.sequences.shape[1] == 130
    assert cache.layers[0].get_seq_length() == 129
