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


_mask_seen = [None, False]  # (mask tensor of the current forward, its verdict)


def _trivial_mask(mask) -> bool:
    """True when the mask hides nothing.  Decode without padding gets no mask
    at all (the sdpa mask builder skips it after its own check of the padding
    mask), which costs nothing here.  A mask tensor (padding, or a sliding
    window the builder could not skip) is read once per forward: every layer
    of one forward receives the same tensor, so the host synchronises at most
    once per decode step, not once per layer."""
    if mask is None:
        return True
    if _mask_seen[0] is mask:
        return _mask_seen[1]
    ok = bool(mask.all()) if mask.dtype == torch.bool else bool((mask == 0).all())
    _mask_seen[0], _mask_seen[1] = mask, ok
    return ok


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
