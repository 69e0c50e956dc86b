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
