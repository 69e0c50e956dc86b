"""Host-side checks that need no GPU: the C-ABI library loads and exports every
function include/innerq_b200.h declares, the ctypes structs match the C
layout, and the drop-in classes keep the reference's config surface."""
import ctypes
import os
import re
import shutil
import subprocess
import types

import pytest
import torch

from tests.conftest import ROOT

HEADER = os.path.join(ROOT, "include", "innerq_b200.h")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(innerq_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from innerq_b200 import _lib
    lib = _lib.load()
    names = _declared()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.EXPORTS, f"{n} has no ctypes signature"
    assert lib.innerq_abi_version() == 5
    assert lib.innerq_tile_bytes(4) == 2048 and lib.innerq_tile_bytes(3) == 1536
    assert lib.innerq_tile_bytes(2) == 1024 and lib.innerq_tile_bytes(5) == -1 and lib.innerq_tile_bytes(1) == 512


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_ctypes_structs_match_c_layout(tmp_path):
    from innerq_b200 import _lib
    c = tmp_path / "s.c"
    c.write_text('#include "innerq_b200.h"\n#include <stdio.h>\n#include <stddef.h>\n'
                 'int main(){printf("%zu %zu %zu %zu %zu %zu %zu %zu %zu\\n", sizeof(innerq_attn_args),'
                 ' sizeof(innerq_side), offsetof(innerq_attn_args, k), offsetof(innerq_attn_args, v),'
                 ' offsetof(innerq_attn_args, softmax_scale), offsetof(innerq_attn_args, step),'
                 ' sizeof(innerq_append_args), offsetof(innerq_append_args, norm_f),'
                 ' offsetof(innerq_append_args, r0));}\n')
    exe = tmp_path / "s"
    subprocess.run(["gcc", "-I", os.path.dirname(HEADER), str(c), "-o", str(exe)], check=True)
    got = list(map(int, subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()))
    A = _lib.AttnArgs
    P = _lib.AppendArgs
    assert got == [ctypes.sizeof(A), ctypes.sizeof(_lib.Side), A.k.offset, A.v.offset,
                   A.softmax_scale.offset, A.step.offset, ctypes.sizeof(P), P.norm_f.offset,
                   P.r0.offset]


def test_append_step_rejects_bad_arguments_without_a_gpu():
    from innerq_b200 import _lib
    lib = _lib.load()
    a = _lib.AppendArgs()
    a.struct_size = ctypes.sizeof(_lib.AppendArgs)
    a.dtype, a.B, a.H, a.D = _lib.DT_F16, 1, 1, 64
    step = ctypes.c_int64(0)
    assert lib.innerq_append_step(ctypes.byref(a), ctypes.byref(step), None) == -2
    assert "head_dim" in _lib.last_error()
    a.D, a.x, a.fifo, a.fifo_cap, a.n_recent, a.r0 = 128, 8, 8, 16, 12, 8
    assert lib.innerq_append_step(ctypes.byref(a), ctypes.byref(step), None) == -1
    assert "FIFO" in _lib.last_error()


def test_argument_errors_are_reported_without_a_gpu():
    """Validation runs before any launch, so bad arguments fail on a CPU box."""
    from innerq_b200 import _lib
    lib = _lib.load()
    rc = lib.innerq_quant_pack(None, 0, 1, 1, 32, 64, 0, 0, 0, 4, 32, 0, 0, 0, None, None, None,
                               None, 1, 0, None)
    assert rc == -2 and "head_dim" in _lib.last_error()
    rc = lib.innerq_quant_pack(None, 0, 1, 1, 32, 128, 0, 0, 0, 5, 32, 0, 0, 0, None, None, None,
                               None, 1, 0, None)
    assert rc == -2 and "bits" in _lib.last_error()
    a = _lib.AttnArgs()
    a.struct_size = 12
    assert lib.innerq_attn_plan(ctypes.byref(a), None, None) == -1
    assert "struct_size" in _lib.last_error()


def test_attention_plan_on_cpu():
    """The split planner is pure host code."""
    from innerq_b200 import _lib
    lib = _lib.load()
    a = _lib.AttnArgs()
    a.struct_size = ctypes.sizeof(_lib.AttnArgs)
    a.dtype, a.B, a.Hq, a.Hkv, a.D = 0, 1, 32, 8, 128
    a.q = 16
    a.k.n_sink, a.k.n_q, a.k.n_recent = 32, 4000, 96
    a.v.n_sink, a.v.n_q, a.v.n_recent = 32, 4064, 32
    for s in (a.k, a.v):
        s.codes = s.scale = 256
        s.cap_tiles, s.bits, s.group = 128, 4, 32
        s.sink = s.recent = 1024
        s.sink_st = s.rec_st = 128
    a.v.over_token = 1
    nt, ns = ctypes.c_int32(), ctypes.c_int32()
    assert lib.innerq_attn_plan(ctypes.byref(a), ctypes.byref(nt), ctypes.byref(ns)) == 0, \
        _lib.last_error()
    assert nt.value == 4128 // 32  # tile grid aligned to the V packed grid (sink 32)
    assert 1 <= ns.value <= nt.value
    a.v.n_recent = 33  # K and V must hold the same number of tokens
    assert lib.innerq_attn_plan(ctypes.byref(a), None, None) == -1


def test_layer_config_surface_matches_reference_defaults():
    from innerq_b200.cache import DynamicCache, InnerqDynamicLayer
    from innerq_b200.quant import QMode
    layer = InnerqDynamicLayer(types.SimpleNamespace(), 3)
    # cache.py:70-91 defaults
    assert (layer.key_bits, layer.value_bits, layer.key_quantize, layer.value_quantize) == (16, 16, False, False)
    assert (layer.key_group_size, layer.value_group_size) == (32, 32)
    assert (layer.key_w_recent, layer.value_w_recent, layer.key_w_sink, layer.value_w_sink) == (32, 32, 0, 0)
    assert (layer.key_flush_size, layer.value_flush_size) == (32, 32)
    assert layer.key_normalize is False and layer.key_normalization_factor is None
    assert layer.key_quantize_over_token is False and layer.value_quantize_over_token is True
    assert layer.key_quantize_mode == QMode.SYM and layer.value_quantize_mode == QMode.SYM
    assert layer.layer_idx == 3 and layer.get_seq_length() == 0 and layer.get_max_cache_shape() == -1
    with pytest.raises(ValueError):
        layer.crop(3)
    with pytest.raises(Exception):
        layer.batch_repeat_interleave(2)
    with pytest.raises(ValueError):
        InnerqDynamicLayer(types.SimpleNamespace(key_quantize_mode="bogus"), 0)
    # the packed store refuses CPU tensors (no CPU path)
    q = InnerqDynamicLayer(types.SimpleNamespace(k_bits=4, v_bits=4), 0)
    with pytest.raises(RuntimeError):
        q.update(torch.zeros(1, 1, 64, 128, dtype=torch.float16), torch.zeros(1, 1, 64, 128, dtype=torch.float16))

    from transformers import LlamaConfig
    c = LlamaConfig(num_hidden_layers=3, hidden_size=256, num_attention_heads=2,
                    num_key_value_heads=1, intermediate_size=64, vocab_size=32)
    cache = DynamicCache(config=c)
    assert len(cache.layers) == 3 and all(isinstance(l, InnerqDynamicLayer) for l in cache.layers)


def test_noalloc_returns_the_plan_status_without_a_gpu():
    """Argument errors are found before any device work: the allocation-free
    entry point returns the same status as innerq_decode_attn (here
    INNERQ_ERR_UNSUPPORTED for a GQA ratio of 3, INNERQ_ERR_ARG for a bad
    struct size) and touches no device."""
    from innerq_b200 import _lib
    lib = _lib.load()
    a = _lib.AttnArgs()
    a.struct_size = ctypes.sizeof(_lib.AttnArgs)
    a.dtype, a.B, a.Hq, a.Hkv, a.D = _lib.DT_F16, 1, 24, 8, 128
    a.q = 16  # never dereferenced: the plan rejects the arguments first
    for expect in (-2, -1):
        if expect == -1:
            a.struct_size = 8
        r1 = lib.innerq_decode_attn(ctypes.byref(a), None, 0, None, 0, 0, None, None)
        r2 = lib.innerq_decode_attn_noalloc(ctypes.byref(a), None, 0, 0, None, None)
        assert r1 == r2 == expect, (r1, r2)


def test_reference_import_names_resolve_to_this_package():
    """`from innerq.cache import ...` (the reference's import paths) reaches
    the B200 modules unchanged."""
    import innerq
    import innerq.cache
    import innerq.models.llama_innerq
    import innerq_b200.cache
    import innerq_b200.models.llama_innerq
    from innerq.cache import DynamicCache, InnerqDynamicLayer  # noqa: F401
    from innerq.models import InnerqLlamaForCausalLM, InnerqMistralForCausalLM  # noqa: F401
    from innerq.quant import QMode, quantize_channeldim_sym  # noqa: F401
    assert innerq.cache is innerq_b200.cache
    assert innerq.models.llama_innerq is innerq_b200.models.llama_innerq
    assert innerq.quant.QMode is innerq_b200.quant.QMode


def test_cache_state_format_without_gpu():
    """An empty cache serialises to plain values (no tensors yet) and loads
    back; a state of another format or layer count is refused."""
    import io

    import torch

    from innerq_b200.cache import DynamicCache

    class Cfg:
        num_hidden_layers = 3
        k_bits, v_bits = 3, 3

        def get_text_config(self, decoder=True):
            return self

    c = DynamicCache(config=Cfg())
    sd = c.state_dict()
    assert sd["format"] == "innerq_b200.DynamicCache" and len(sd["layers"]) == 3
    assert not sd["layers"][0]["k"]["initialized"]
    buf = io.BytesIO()
    torch.save(sd, buf)
    buf.seek(0)
    c2 = DynamicCache(config=Cfg())
    c2.load_state_dict(torch.load(buf, weights_only=True))
    assert c2.get_seq_length() == 0
    with pytest.raises(ValueError):
        c2.load_state_dict(dict(sd, format="other"))
    with pytest.raises(ValueError):
        c2.load_state_dict(dict(sd, layers=sd["layers"][:2]))
