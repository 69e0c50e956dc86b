"""The ``"innerq"`` attention function for Hugging Face models.

Registered in ``transformers.AttentionInterface`` (and, for its mask, in
``AttentionMaskInterface`` with the sdpa mask builder).  On a decode step the
InnerQ cache layer hands back the new-token states tagged with the layer
(``innerq_b200.cache.InnerqDynamicLayer.update``); this function then runs
the fused packed-cache attention kernel instead of the reference's
dequantize-everything + sdpa (``src/innerq/cache.py:278-281`` and the HF sdpa
consumer).  Prefill (the reference returns raw K/V there, ``cache.py:390-392``)
and masked decode steps (padding) go to HF sdpa on real tensors, the latter
materialised by the GPU dequant kernel.
"""
from __future__ import annotations

import torch
from transformers import AttentionInterface
from transformers.integrations.sdpa_attention import sdpa_attention_forward
from transformers.masking_utils import AttentionMaskInterface, sdpa_mask

NAME = "innerq"


def _trivial_mask(mask) -> bool:
    if mask is None:
        return True
    if mask.dtype == torch.bool:
        return bool(mask.all())
    return bool((mask == 0).all())


def innerq_attention_forward(module, query, key, value, attention_mask, dropout: float = 0.0,
                             scaling: float | None = None, is_causal: bool | None = None, **kwargs):
    layer = getattr(key, "_innerq_layer", None)
    if layer is not None:
        key._innerq_layer = None
        # graph mode (a recorded decode step) is single-token decode without
        # padding by contract; checking the mask would synchronise the host
        if query.shape[2] == 1 and (layer._gstep is not None or _trivial_mask(attention_mask)):
            out = layer.attend(query, scaling, reuse=True)  # [B, Hq, D]
            return out.unsqueeze(1), None                # [B, q_len=1, Hq, D]
        key, value = layer.get_deq_tensors()
    return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout,
                                  scaling=scaling, is_causal=is_causal, **kwargs)


def register() -> None:
    AttentionInterface.register(NAME, innerq_attention_forward)
    AttentionMaskInterface.register(NAME, sdpa_mask)


def use_innerq_attention(model) -> None:
    """Switch a loaded model to the fused decode attention."""
    register()
    try:
        model.set_attn_implementation(NAME)
    except Exception:
        model.config._attn_implementation = NAME
