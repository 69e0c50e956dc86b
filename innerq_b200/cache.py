"""Drop-in for ``innerq.cache`` (``src/innerq/cache.py`` of mthcom/innerq) on B200.

``InnerqDynamicLayer`` keeps the reference constructor, the 15 config
attributes with the same defaults (``cache.py:70-119``), the prefill / flush
semantics and the Hugging Face ``CacheLayerMixin`` protocol
(``update`` / ``get_seq_length`` / ``get_mask_sizes`` ...), but stores the
quantized middle packed on the GPU (``innerq_b200.store.PackedSide``) and
appends with the quantize-and-pack kernel instead of ``torch.cat``.

``update`` returns what the reference returns: the raw K/V on the prefill
call (``cache.py:390-392``) and, on decode calls, the full dequantized
``[sink | middle | recent]`` K/V in the model dtype, bit-exact with the
reference's ``get_deq_tensors`` (``cache.py:278-281``).  When the layer is
driven by the ``"innerq"`` attention function (``innerq_b200.models``), the
decode call skips that materialisation and the attention kernel reads the
packed store directly.

The reference-format attributes (``keys_q``, ``keys_scale_factor``,
``keys_zp_sign``, ``keys_sink``, ``keys_recent``,
``key_normalization_factor`` and the ``values_*`` ones) are computed on
access.  Signs read back from the packed store are 0 where the code is 0
(codes x signs is bit-exact; the sign of a value that quantized to 0 is not
stored).
"""
from __future__ import annotations

from collections.abc import Iterable
from typing import Any

import torch
from transformers.cache_utils import Cache, CacheLayerMixin

from . import _lib
from .quant import QMode
from .store import HybridSide, PackedSide


class InnerqDynamicLayer(CacheLayerMixin):
    """cache.py:61-419."""
    is_sliding = False

    def __init__(self, config, layer_idx):
        self.parse_config(config)
        self.layer_idx = layer_idx
        self.cumulative_length = 0
        self.fused = bool(getattr(config, "_attn_implementation", None) == "innerq")
        self._attn = None
        self._gstep = None  # graph mode: the cache's device step counter
        hq, hkv = getattr(config, "num_attention_heads", None), getattr(config, "num_key_value_heads", None)
        self._gqa = hq // hkv if isinstance(hq, int) and isinstance(hkv, int) and hkv > 0 else None
        super().__init__()

    # cache.py:70-119
    def parse_config(self, config):
        self.key_bits = getattr(config, 'k_bits', 16)
        self.value_bits = getattr(config, 'v_bits', 16)
        self.key_quantize = False if self.key_bits >= 16 else True
        self.value_quantize = False if self.value_bits >= 16 else True

        self.key_group_size = getattr(config, 'key_group_size', 32)
        self.value_group_size = getattr(config, 'value_group_size', 32)
        self.key_w_recent = getattr(config, 'key_w_recent', 32)
        self.value_w_recent = getattr(config, 'value_w_recent', 32)
        self.key_w_sink = getattr(config, 'key_w_sink', 0)
        self.value_w_sink = getattr(config, 'value_w_sink', 0)
        self.key_flush_size = getattr(config, 'key_flush_size', 32)
        self.value_flush_size = getattr(config, 'value_flush_size', 32)
        self.key_normalize = getattr(config, 'key_normalize', False)

        self.key_quantize_over_token = getattr(config, 'key_quantize_over_token', False)
        self.value_quantize_over_token = getattr(config, 'value_quantize_over_token', True)

        self.key_quantize_mode = QMode.from_str(getattr(config, 'key_quantize_mode', 'symmetric'))
        self.value_quantize_mode = QMode.from_str(getattr(config, 'value_quantize_mode', 'symmetric'))

        def side(role, qmode, bits, group, over_token, w_sink, w_recent, flush, normalize=False):
            if qmode == QMode.HYBRID:  # quant.py:133-176
                return HybridSide(role, bits, group, over_token, w_sink, w_recent, flush, normalize)
            mode = _lib.ASYM if qmode == QMode.ASYM else _lib.SYM
            return PackedSide(role, bits, group, mode, over_token, w_sink, w_recent, flush, normalize)

        self._k = side(_lib.ROLE_K, self.key_quantize_mode, self.key_bits, self.key_group_size,
                       self.key_quantize_over_token, self.key_w_sink, self.key_w_recent,
                       self.key_flush_size, normalize=bool(self.key_normalize) and self.key_quantize)
        self._v = side(_lib.ROLE_V, self.value_quantize_mode, self.value_bits, self.value_group_size,
                       self.value_quantize_over_token, self.value_w_sink, self.value_w_recent,
                       self.value_flush_size)

    # ----------------------------------------------- reference-format views
    @property
    def key_normalization_factor(self):
        f = self._k.norm_f
        return None if f is None else f.unsqueeze(2)

    @property
    def keys_sink(self):
        return self._k.sink

    @property
    def values_sink(self):
        return self._v.sink

    @property
    def keys_recent(self):
        return self._k.recent

    @property
    def values_recent(self):
        return self._v.recent

    def _kviews(self):
        return self._k.ref_views()

    def _vviews(self):
        return self._v.ref_views()

    @property
    def keys_q(self):
        return self._kviews()[0]

    @property
    def keys_scale_factor(self):
        return self._kviews()[1]

    @property
    def keys_zp_sign(self):
        return self._kviews()[2]

    @property
    def values_q(self):
        return self._vviews()[0]

    @property
    def values_scale_factor(self):
        return self._vviews()[1]

    @property
    def values_zp_sign(self):
        return self._vviews()[2]

    @property
    def key_side(self) -> PackedSide:
        return self._k

    @property
    def value_side(self) -> PackedSide:
        return self._v

    # ------------------------------------------------------------- protocol
    def lazy_initialization(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        """cache.py:226-233."""
        self.dtype, self.device = key_states.dtype, key_states.device
        self._k.prefill(key_states)
        self._v.prefill(value_states)
        self.is_initialized = True

    def add_to_cache(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        """cache.py:367-380."""
        self._k.append(key_states)
        self._v.append(value_states)

    def get_deq_tensors(self) -> tuple[torch.Tensor, torch.Tensor]:
        """cache.py:278-281, materialised by the dequant kernel."""
        return self._k.materialize(), self._v.materialize()

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor,
               cache_kwargs: dict[str, Any] | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """cache.py:382-396."""
        if self._gstep is not None:
            # graph mode: one append launch per side, state on the device
            self._k.append_graph(key_states, self._gstep)
            self._v.append_graph(value_states, self._gstep)
            key_states._innerq_layer = self
            return key_states, value_states
        self.cumulative_length += key_states.shape[-2]
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
            return key_states, value_states
        self.add_to_cache(key_states, value_states)
        if self.fused and key_states.shape[-2] == 1 and self._fusable():
            # the "innerq" attention function reads the packed store
            key_states._innerq_layer = self
            return key_states, value_states
        return self.get_deq_tensors()

    # --------------------------------------------------------- serialisation
    def state_dict(self) -> dict:
        """The layer's cache content as host tensors: both stores
        (PackedSide.state_dict) and the token count."""
        if self._gstep is not None:
            raise RuntimeError("cannot serialise a layer in graph mode (call graph_end first)")
        return {"cumulative_length": self.cumulative_length, "is_initialized": bool(self.is_initialized),
                "sliding_window": getattr(self, "sliding_window", None),
                "k": self._k.state_dict(), "v": self._v.state_dict()}

    def load_state_dict(self, d: dict, device=None) -> None:
        """Restore what state_dict() wrote, onto `device` (default: the
        current CUDA device).  The layer must have been built from the same
        config (bits, groups, windows, modes are checked)."""
        if d.get("sliding_window") != getattr(self, "sliding_window", None):
            raise ValueError(f"saved layer has sliding_window={d.get('sliding_window')!r}, "
                             f"this layer {getattr(self, 'sliding_window', None)!r}")
        self._k.load_state_dict(d["k"], device)
        self._v.load_state_dict(d["v"], device)
        self.cumulative_length = int(d["cumulative_length"])
        self.is_initialized = bool(d["is_initialized"])
        self._attn = None
        if self.is_initialized:
            self.dtype, self.device = self._k.dtype, self._k.device
            if hasattr(self, "_sliding_window_tensor"):
                self._sliding_window_tensor = self._sliding_window_tensor.to(self.device)

    # ------------------------------------------------------------ graph mode
    def graph_begin(self, step: torch.Tensor, max_steps: int) -> None:
        """Enter graph mode (see DynamicCache.graph_begin)."""
        if not (self.is_initialized and self.fused and self._fusable()):
            raise NotImplementedError("graph mode needs a prefilled layer on the fused attention path")
        if isinstance(self._k, HybridSide) or isinstance(self._v, HybridSide):
            raise NotImplementedError("graph mode does not cover hybrid stores")
        self._k.graph_begin(max_steps)
        self._v.graph_begin(max_steps)
        self._gstep = step

    def graph_end(self, n_steps: int) -> None:
        self._k.graph_end(n_steps)
        self._v.graph_end(n_steps)
        self.cumulative_length += n_steps
        self._gstep = None

    def _fusable(self) -> bool:
        """Both stores are in layouts the fused kernel reads: channel-grouped
        values need the keys' group size."""
        k, v = self._k, self._v
        if not (k.fusable and v.fusable):
            return False
        if k.quantize and k.over_token:
            # keys grouped over tokens (KIVI): GQA <= 4, the values' sink
            # size, non-hybrid values, channel-grouped values in groups of 32
            if self._gqa is not None and self._gqa > 4:
                return False
            if isinstance(k, HybridSide) or isinstance(v, HybridSide):
                return False
            if v.quantize and k.w_sink != v.w_sink:
                return False
            return not (v.quantize and not v.over_token and v.group != 32)
        return not (v.quantize and not v.over_token and k.quantize and v.group != k.group)

    def attend(self, query: torch.Tensor, scaling: float | None = None,
               out: torch.Tensor | None = None, reuse: bool = False) -> torch.Tensor:
        """Fused decode attention of query [B, Hq, 1, D] over this layer ->
        [B, Hq, D].  With reuse=True the result lives in a per-layer buffer
        that the next call overwrites (the model hook consumes it at once)."""
        if self._attn is None:
            from .attention import DecodeAttention
            self._attn = DecodeAttention()
        out_ = self._attn(query, self._k, self._v, scaling, out=out, step=self._gstep)
        # the launcher reuses its buffer on the next step: hand out a copy-free
        # view only when the caller gave the destination
        return out_ if (out is not None or reuse) else out_.clone()

    def attend_partials(self, query: torch.Tensor, po: torch.Tensor, pm: torch.Tensor,
                        pl: torch.Tensor, scaling: float | None = None) -> None:
        """Split partials of this layer's tokens (a context chunk when the
        layer is one rank's share of a sharded cache) into po / pm / pl; see
        DecodeAttention.partials."""
        if self._attn is None:
            from .attention import DecodeAttention
            self._attn = DecodeAttention()
        self._attn.partials(query, self._k, self._v, po, pm, pl, scaling, step=self._gstep)

    def get_mask_sizes(self, cache_position) -> tuple[int, int]:
        """cache.py:398-402; also takes the int query_length of transformers >= 5.5."""
        kv_offset = 0
        query_length = cache_position if isinstance(cache_position, int) else cache_position.shape[0]
        kv_length = self.get_seq_length() + query_length
        return kv_length, kv_offset

    def get_seq_length(self) -> int:
        return self.cumulative_length

    def get_max_cache_shape(self) -> int:
        return -1

    def crop(self, max_length: int) -> None:
        raise ValueError('This function is not implementable for quantized cache. It leads to the '
                         'loss of accuracy on the recent tokens')

    def batch_repeat_interleave(self, repeats: int) -> None:
        raise Exception('This function is not implemented yet.')

    def batch_select_indices(self, indices: torch.Tensor) -> None:
        raise Exception('This function is not implemented yet.')


class InnerqDynamicSlidingWindowLayer(InnerqDynamicLayer):
    """cache.py:421-461.  The reference crops with ``[:, :, -window, :]``
    (``cache.py:443-444``), which keeps a single token and drops a dim, and
    only once more than ``window`` tokens preceded the step, one step after
    its own ``get_mask_sizes`` starts sizing the mask for a full window.  This
    layer returns what that mask describes: once ``window`` tokens preceded
    the step, the last ``window - 1 + q_len`` tokens.  The fused path is not
    used for sliding layers."""
    is_sliding = True

    def __init__(self, config, layer_idx: int, sliding_window: int):
        super().__init__(config, layer_idx)
        self.fused = False
        self.sliding_window = sliding_window
        self.cumulative_length = 0
        self._sliding_window_tensor = torch.tensor(self.sliding_window, dtype=torch.long)

    def lazy_initialization(self, key_states, value_states) -> None:
        super().lazy_initialization(key_states, value_states)
        self._sliding_window_tensor = self._sliding_window_tensor.to(self.device)

    def update(self, key_states, value_states, cache_kwargs=None):
        k, v = super().update(key_states, value_states, cache_kwargs)
        q_len = key_states.shape[-2]
        if self.cumulative_length - q_len >= self.sliding_window:  # get_mask_sizes' is_full
            keep = self.sliding_window - 1 + q_len
            k = k[:, :, -keep:, :]
            v = v[:, :, -keep:, :]
        return k, v

    def get_mask_sizes(self, cache_position) -> tuple[int, int]:
        query_length = cache_position if isinstance(cache_position, int) else cache_position.shape[0]
        is_full = self.cumulative_length >= self.sliding_window
        kv_offset = max(self.cumulative_length - self.sliding_window + 1, 0)
        if is_full:
            kv_length = self.sliding_window - 1 + query_length
        else:
            kv_length = self.cumulative_length + query_length
        return kv_length, kv_offset

    def get_max_cache_shape(self) -> int:
        return self.sliding_window


class DynamicCache(Cache):
    """cache.py:463-496: one layer per decoder layer, sliding or full."""

    def __init__(self, ddp_cache_data: Iterable[tuple[torch.Tensor | None, ...]] | None = None,
                 config=None, offloading: bool = False, offload_only_non_sliding: bool = False):
        layers = []
        if config is not None:
            decoder_config = config.get_text_config(decoder=True)
            sliding_window = getattr(decoder_config, "sliding_window", None) or getattr(
                decoder_config, "attention_chunk_size", None)
            layer_types = getattr(decoder_config, "layer_types", None)
            if layer_types is None:
                layer_types = ["sliding_attention" if sliding_window is not None else "full_attention"
                               for _ in range(decoder_config.num_hidden_layers)]
            if hasattr(decoder_config, "num_kv_shared_layers"):
                layer_types = layer_types[: -decoder_config.num_kv_shared_layers]
            for layer_idx, layer_type in enumerate(layer_types):
                if layer_type in ("sliding_attention", "chunked_attention"):
                    layers.append(InnerqDynamicSlidingWindowLayer(config=config, layer_idx=layer_idx,
                                                                  sliding_window=sliding_window))
                else:
                    layers.append(InnerqDynamicLayer(config=config, layer_idx=layer_idx))
        super().__init__(layers=layers, offloading=offloading,
                         offload_only_non_sliding=offload_only_non_sliding)

    # --------------------------------------------------------- serialisation
    FORMAT = "innerq_b200.DynamicCache"
    # 2: scales of keys grouped over tokens in natural dim order
    FORMAT_VERSION = 2

    def state_dict(self) -> dict:
        """Every layer's packed cache as host tensors and plain values (no
        pickled objects: loadable with torch.load(weights_only=True))."""
        return {"format": self.FORMAT, "version": self.FORMAT_VERSION,
                "layers": [layer.state_dict() for layer in self.layers]}

    def load_state_dict(self, sd: dict, device=None) -> None:
        if sd.get("format") != self.FORMAT or sd.get("version") != self.FORMAT_VERSION:
            raise ValueError(f"not a {self.FORMAT} v{self.FORMAT_VERSION} state: "
                             f"{sd.get('format')!r} v{sd.get('version')!r}")
        if len(sd["layers"]) != len(self.layers):
            raise ValueError(f"saved cache has {len(sd['layers'])} layers, this one {len(self.layers)}")
        for layer, d in zip(self.layers, sd["layers"]):
            layer.load_state_dict(d, device)

    def save(self, path) -> None:
        """Write the packed cache to `path` (torch.save of state_dict())."""
        torch.save(self.state_dict(), path)

    @classmethod
    def load(cls, path, config, device=None) -> "DynamicCache":
        """A cache built from `config` (the model config the saved cache was
        built with) holding the content saved at `path`, on `device`."""
        cache = cls(config=config)
        cache.load_state_dict(torch.load(path, map_location="cpu", weights_only=True), device)
        return cache

    # ------------------------------------------------------------ graph mode
    def graph_begin(self, max_steps: int) -> torch.Tensor:
        """Switch every layer to graph mode for up to `max_steps` decode steps:
        the stores reserve the capacity those steps need, and each step's
        appends and attention read the step from a device counter instead of
        from host-side arguments, so a recorded decode step (a CUDA graph)
        replays correctly step after step.  Each recorded step must begin with
        graph_advance().  Returns the counter (int64, 1 element)."""
        layers = [l for l in self.layers if getattr(l, "is_initialized", False)]
        if not layers:
            raise RuntimeError("graph mode needs a prefilled cache")
        self._gstep = torch.zeros(1, dtype=torch.int64, device=layers[0].device)
        for layer in layers:
            layer.graph_begin(self._gstep, max_steps)
        return self._gstep

    def graph_advance(self) -> None:
        """The first operation of every graph-mode decode step."""
        self._gstep.add_(1)

    def graph_end(self) -> int:
        """Leave graph mode; returns the number of steps taken."""
        n = int(self._gstep.item())
        for layer in self.layers:
            if getattr(layer, "_gstep", None) is not None:
                layer.graph_end(n)
        self._gstep = None
        return n

    def __iter__(self):
        for layer in self.layers:
            yield layer.keys, layer.values, getattr(layer, "_sliding_window_tensor", None)
