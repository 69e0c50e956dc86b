"""InnerqLlamaForCausalLM: ``src/innerq/models/llama_innerq.py:6-18``.

Installs the InnerQ ``DynamicCache`` for ``generate`` exactly as the reference
does, and additionally routes attention through the ``"innerq"`` function so
decode steps read the packed cache directly.
"""
from transformers.models.llama.modeling_llama import LlamaForCausalLM

from ..cache import DynamicCache
from .attention_hook import use_innerq_attention


class InnerqLlamaForCausalLM(LlamaForCausalLM):
    def __init__(self, config):
        super().__init__(config)
        use_innerq_attention(self)

    def _prepare_cache_for_generation(self, generation_config, model_kwargs, generation_mode,
                                      batch_size, max_cache_length):
        model_kwargs["past_key_values"] = DynamicCache(config=self.config.get_text_config(decoder=True))
