"""Generate the golden fixtures by running the REFERENCE implementation itself.

Run in a container that has the reference checkout (read-only) and transformers:

    python tests/golden/make_golden.py --ref <path to mthcom/innerq checkout>

It imports ``innerq`` from ``<ref>/src`` (with ``lm_eval`` stubbed out, since
``innerq/__init__.py`` imports the lm-eval wrapper), feeds seeded inputs through
``innerq.quant`` and ``innerq.cache.InnerqDynamicLayer`` on the CPU, and writes
the reference's outputs to ``tests/golden/*.npz``.  The GPU box never runs this
script; the tests only read the committed ``.npz`` files.

bf16 tensors are stored as their raw uint16 bit patterns.
"""
from __future__ import annotations

import argparse
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def import_reference(ref_root: str):
    m = types.ModuleType("lm_eval")
    mm = types.ModuleType("lm_eval.models")
    hf = types.ModuleType("lm_eval.models.huggingface")

    class HFLM:  # only needs to exist as a base class
        pass

    hf.HFLM = HFLM
    m.models, mm.huggingface = mm, hf
    sys.modules.update({"lm_eval": m, "lm_eval.models": mm, "lm_eval.models.huggingface": hf})
    sys.path.insert(0, os.path.join(ref_root, "src"))
    import innerq  # noqa: F401
    import innerq.cache
    import innerq.quant
    return innerq


TDT = {"fp16": torch.float16, "bf16": torch.bfloat16}


def to_np(t: torch.Tensor):
    """Lossless numpy form of a reference tensor."""
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float16:
        return t.numpy()
    if t.dtype == torch.int32:
        return t.numpy()
    if t.dtype == torch.float32:
        return t.numpy()
    raise TypeError(t.dtype)


def synth_k(gen, shape, dtype):
    """K = N(0,1) x exp(N(0,1)) per channel (channel outliers), cast to dtype."""
    x = torch.randn(shape, generator=gen)
    ch = torch.exp(torch.randn(shape[-1], generator=gen))
    return (x * ch).to(TDT[dtype])


def quant_cases(innerq):
    Qm = innerq.quant
    funcs = {
        "channel_sym": Qm.quantize_channeldim_sym,
        "token_sym": Qm.quantize_tokendim_sym,
        "channel_asym": Qm.quantize_channeldim_asym,
        "token_asym": Qm.quantize_tokendim_asym,
    }
    deqs = {
        "channel_sym": Qm.dequantize_channeldim_sym,
        "token_sym": Qm.dequantize_tokendim_sym,
        "channel_asym": Qm.dequantize_channeldim_asym,
        "token_asym": Qm.dequantize_tokendim_asym,
    }
    out = {}
    for dtype in ("fp16", "bf16"):
        gen = torch.Generator().manual_seed(1234 if dtype == "fp16" else 4321)
        x = synth_k(gen, (1, 2, 128, 128), dtype)
        # edge groups: an all-zero channel group, an all-zero token group, and a
        # group whose max is a tiny value (its scale underflows in fp16)
        x[0, 0, 5, 0:32] = 0
        x[0, 1, 0:32, 7] = 0
        x[0, 0, 6, 32:64] = 0
        x[0, 0, 6, 40] = 2.0 ** -24 if dtype == "fp16" else 2.0 ** -130
        out[f"{dtype}/x"] = to_np(x)
        cases = [(f, b, 32) for f in funcs for b in (2, 3, 4)]
        if dtype == "fp16":
            cases += [(f, b, g) for f in funcs for b in (2, 3, 4) for g in (64, 128)]
        for name, bits, g in cases:
            c, s, z = funcs[name](x.clone(), g, bits)
            key = f"{dtype}/{name}/b{bits}/g{g}"
            out[key + "/codes"] = c.numpy().astype(np.int32)
            out[key + "/scale"] = to_np(s)
            out[key + "/zp"] = to_np(z)
            if g == 32:
                d = deqs[name](c, s, z, g, op_dtype=torch.float32)
                out[key + "/deq"] = to_np(d.to(torch.float32))
        # key normalisation factor + normalised keys (cache.py:121-126)
        f = x.abs().max(dim=-2, keepdim=True).values.sqrt()
        out[f"{dtype}/norm/f"] = to_np(f)
        out[f"{dtype}/norm/xn"] = to_np(x / f)
    return out


class Cfg:
    """A minimal stand-in for the HF config: cache.py reads it with getattr."""

    def __init__(self, **kw):
        self.__dict__.update(kw)


PRESETS = {
    "innerq_base": dict(k_bits=3, v_bits=3, key_flush_size=1, value_flush_size=32,
                        key_group_size=32, value_group_size=32, key_w_recent=96,
                        value_w_recent=96, key_w_sink=32, value_w_sink=32,
                        key_normalize=True, key_quantize_over_token=False,
                        value_quantize_over_token=True, key_quantize_mode="symmetric",
                        value_quantize_mode="symmetric"),
    "innerq_small": dict(k_bits=3, v_bits=2, key_flush_size=1, value_flush_size=32,
                         key_group_size=32, value_group_size=32, key_w_recent=96,
                         value_w_recent=96, key_w_sink=32, value_w_sink=32,
                         key_normalize=True, key_quantize_over_token=False,
                         value_quantize_over_token=True, key_quantize_mode="symmetric",
                         value_quantize_mode="symmetric"),
    "kivi": dict(k_bits=2, v_bits=2, key_flush_size=32, value_flush_size=1,
                 key_group_size=32, value_group_size=32, key_w_recent=128,
                 value_w_recent=128, key_w_sink=0, value_w_sink=0,
                 key_normalize=False, key_quantize_over_token=True,
                 value_quantize_over_token=False, key_quantize_mode="asymmetric",
                 value_quantize_mode="asymmetric"),
    "default4": dict(k_bits=4, v_bits=4),
    "asym4_norm": dict(k_bits=4, v_bits=4, key_quantize_mode="asymmetric",
                       value_quantize_mode="asymmetric", key_normalize=True,
                       key_w_sink=4, value_w_sink=4, value_group_size=64,
                       value_flush_size=64),
    "innerq_hybrid": dict(k_bits=3, v_bits=2, key_flush_size=1, value_flush_size=32,
                          key_group_size=32, value_group_size=32, key_w_recent=96,
                          value_w_recent=96, key_w_sink=32, value_w_sink=32,
                          key_normalize=True, key_quantize_over_token=False,
                          value_quantize_over_token=True, key_quantize_mode="symmetric",
                          value_quantize_mode="hybrid"),
}


def cache_cases(innerq):
    out = {}
    B, H, D, T0, steps = 1, 2, 128, 200, 40
    for pi, (name, kw) in enumerate(PRESETS.items()):
        dtype = "bf16" if name == "innerq_small" else "fp16"
        gen = torch.Generator().manual_seed(100 + pi)
        layer = innerq.cache.InnerqDynamicLayer(Cfg(**kw), 0)
        k0 = synth_k(gen, (B, H, T0, D), dtype)
        v0 = torch.randn((B, H, T0, D), generator=gen).to(TDT[dtype])
        ks, vs = [k0], [v0]
        layer.update(k0, v0)
        trace = []
        for _ in range(steps):
            k1 = synth_k(gen, (B, H, 1, D), dtype)
            v1 = torch.randn((B, H, 1, D), generator=gen).to(TDT[dtype])
            ks.append(k1)
            vs.append(v1)
            K, V = layer.update(k1, v1)
            def nq(c):
                if c is None:
                    return 0
                return (c["nozp"] if isinstance(c, dict) else c).shape[2]
            nqk, nqv = nq(layer.keys_q), nq(layer.values_q)
            trace.append([layer.keys_sink.shape[2], nqk, layer.keys_recent.shape[2],
                          layer.values_sink.shape[2], nqv, layer.values_recent.shape[2]])
        q = torch.randn((B, 4 * H, 1, D), generator=gen).to(TDT[dtype])
        # the consumer: HF sdpa over the returned (cast) K/V, GQA 4:1, in fp32
        kk = K.float().repeat_interleave(4, dim=1)
        vv = V.float().repeat_interleave(4, dim=1)
        o = torch.nn.functional.scaled_dot_product_attention(q.float(), kk, vv)
        p = f"cache/{name}"
        out[p + "/dtype"] = np.array(dtype)
        out[p + "/k_in"] = to_np(torch.cat(ks, dim=2))
        out[p + "/v_in"] = to_np(torch.cat(vs, dim=2))
        out[p + "/K"] = to_np(K)
        out[p + "/V"] = to_np(V)
        out[p + "/trace"] = np.array(trace, dtype=np.int32)
        out[p + "/q"] = to_np(q)
        out[p + "/o"] = o.numpy()
        if layer.key_normalization_factor is not None:
            out[p + "/kf"] = to_np(layer.key_normalization_factor)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the mthcom/innerq checkout")
    args = ap.parse_args()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    innerq = import_reference(args.ref)
    np.savez_compressed(os.path.join(HERE, "quant_golden.npz"), **quant_cases(innerq))
    np.savez_compressed(os.path.join(HERE, "cache_golden.npz"), **cache_cases(innerq))
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()
