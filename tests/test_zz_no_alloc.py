"""The allocation-free decode attention entry point.

innerq_decode_attn_noalloc serves callers that cannot allocate device memory
while decoding (a fixed memory arena, or a serving loop that forbids
allocation after warm-up): it keeps its split-KV partials in a fixed device
array of the library instead of a caller workspace.  Here it is called through
the C ABI twice in a row and must agree with innerq_decode_attn each time.
This file is collected last so that a stop-at-first-failure run has already
run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from tests._util import assert_close_rel, cfg, synth_kv, synth_q, to_np32

pytestmark = pytest.mark.gpu


def test_noalloc_matches_workspace_entry_point_twice():
    from innerq_b200 import _lib
    from innerq_b200.attention import build_args, decode_attention
    from innerq_b200.cache import InnerqDynamicLayer
    from innerq_b200.store import stream_ptr

    kw = dict(k_bits=4, v_bits=4, key_flush_size=1, key_normalize=True, key_w_sink=32,
              value_w_sink=32, key_w_recent=96, value_w_recent=96)
    layer = InnerqDynamicLayer(cfg(**kw), 0)
    k, v = synth_kv(2, 8, 6000, seed=21)
    layer.update(k, v)
    for call in range(2):
        q = synth_q(2, 32, seed=30 + call)
        ref = decode_attention(q, layer.key_side, layer.value_side)
        args = build_args(q, layer.key_side, layer.value_side)
        out = torch.full_like(ref, float("nan"))
        _lib.call("innerq_decode_attn_noalloc", ctypes.byref(args), out.data_ptr(),
                  out.stride(0), out.stride(1), None, stream_ptr(q.device))
        torch.cuda.synchronize()
        got = to_np32(out)
        assert np.isfinite(got).all()
        assert_close_rel(got, to_np32(ref), 1e-3, f"noalloc call {call}")


def test_noalloc_rejects_oversized_partials():
    from innerq_b200 import _lib
    from innerq_b200.attention import build_args
    from innerq_b200.cache import InnerqDynamicLayer
    from innerq_b200.store import stream_ptr

    layer = InnerqDynamicLayer(cfg(k_bits=4, v_bits=4, key_flush_size=1), 0)
    k, v = synth_kv(16, 8, 16384, seed=22)
    layer.update(k, v)
    q = synth_q(16, 64, seed=23)
    # one split per tile: 16 x 64 x 513 partial rows, far above the fixed scratch
    args = build_args(q, layer.key_side, layer.value_side, n_splits=100000)
    out = torch.empty((16, 64, 128), dtype=torch.float16, device="cuda")
    with pytest.raises(_lib.InnerqError, match="scratch"):
        _lib.call("innerq_decode_attn_noalloc", ctypes.byref(args), out.data_ptr(),
                  out.stride(0), out.stride(1), None, stream_ptr(q.device))
