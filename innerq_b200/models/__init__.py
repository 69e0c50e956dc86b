"""Model hooks: ``src/innerq/models/__init__.py`` of mthcom/innerq."""
from .attention_hook import innerq_attention_forward, register, use_innerq_attention
from .llama_innerq import InnerqLlamaForCausalLM
from .mistral_innerq import InnerqMistralForCausalLM

register()

__all__ = [
    "InnerqLlamaForCausalLM",
    "InnerqMistralForCausalLM",
    "innerq_attention_forward",
    "use_innerq_attention",
]
