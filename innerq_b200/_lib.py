"""ctypes binding of libinnerq_b200.so (the C ABI in include/innerq_b200.h).

This is the same binding a Python caller of the C ABI would write; the
package's host code calls the library only through it.  Importing works
without a GPU (the CPU test-suite checks the exports); calling a compute entry
point needs CUDA tensors.  There is no fallback: a missing library raises.
"""
from __future__ import annotations

import ctypes as C
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libinnerq_b200.so")

INNERQ_OK = 0
DT_F16, DT_BF16 = 0, 1
SYM, ASYM, HYBRID = 0, 1, 2
ROLE_K, ROLE_V = 0, 1

EXPORTS = (
    "innerq_abi_version", "innerq_last_error", "innerq_tile_bytes", "innerq_norm_factor",
    "innerq_quant_pack", "innerq_unpack_ref", "innerq_dequant", "innerq_attn_plan",
    "innerq_decode_attn_workspace", "innerq_decode_attn", "innerq_decode_attn_partials",
    "innerq_lse_merge", "innerq_dequant_ref", "innerq_decode_attn_noalloc", "innerq_append_step",
    "innerq_partials_rank_floats", "innerq_lse_merge_ranks",
)


class InnerqError(RuntimeError):
    """A negative status from the C ABI (message from innerq_last_error)."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed ({code}): {msg}")
        self.code = code


class Side(C.Structure):
    _fields_ = [
        ("codes", C.c_void_p), ("scale", C.c_void_p), ("zero", C.c_void_p),
        ("cap_tiles", C.c_int64),
        ("sink", C.c_void_p), ("sink_sb", C.c_int64), ("sink_sh", C.c_int64), ("sink_st", C.c_int64),
        ("recent", C.c_void_p), ("rec_sb", C.c_int64), ("rec_sh", C.c_int64), ("rec_st", C.c_int64),
        ("n_sink", C.c_int32), ("n_q", C.c_int32), ("n_recent", C.c_int32),
        ("bits", C.c_int32), ("group", C.c_int32), ("mode", C.c_int32), ("over_token", C.c_int32),
        ("r0", C.c_int32), ("flush", C.c_int32), ("max_steps", C.c_int32),
        ("codes2", C.c_void_p), ("scale2", C.c_void_p), ("zero2", C.c_void_p), ("mask", C.c_void_p),
        ("cap_tiles2", C.c_int64),
    ]


class AppendArgs(C.Structure):
    _fields_ = [
        ("struct_size", C.c_int32), ("dtype", C.c_int32), ("B", C.c_int32), ("H", C.c_int32),
        ("D", C.c_int32),
        ("x", C.c_void_p), ("x_sb", C.c_int64), ("x_sh", C.c_int64),
        ("fifo", C.c_void_p), ("f_sb", C.c_int64), ("f_sh", C.c_int64), ("f_st", C.c_int64),
        ("fifo_cap", C.c_int32),
        ("codes", C.c_void_p), ("scale", C.c_void_p), ("zero", C.c_void_p), ("cap_tiles", C.c_int64),
        ("norm_f", C.c_void_p),
        ("bits", C.c_int32), ("group", C.c_int32), ("mode", C.c_int32), ("role", C.c_int32),
        ("over_token", C.c_int32), ("flush", C.c_int32),
        ("n_q", C.c_int32), ("n_recent", C.c_int32), ("r0", C.c_int32),
        ("max_steps", C.c_int32),
    ]


class AttnArgs(C.Structure):
    _fields_ = [
        ("struct_size", C.c_int32), ("dtype", C.c_int32),
        ("B", C.c_int32), ("Hq", C.c_int32), ("Hkv", C.c_int32), ("D", C.c_int32),
        ("q", C.c_void_p), ("q_sb", C.c_int64), ("q_sh", C.c_int64),
        ("key_norm", C.c_void_p),
        ("k", Side), ("v", Side),
        ("softmax_scale", C.c_float),
        ("n_splits", C.c_int32), ("tile_lo", C.c_int32), ("tile_hi", C.c_int32),
        ("step", C.c_void_p),
    ]


_lib = None


def load() -> C.CDLL:
    """Load the library once; raise loudly when it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m innerq_b200.build` "
            "(innerq_b200 has no CPU fallback)")
    lib = C.CDLL(LIB_PATH)
    vp, i32, i64 = C.c_void_p, C.c_int, C.c_int64
    sig = {
        "innerq_abi_version": (i32, []),
        "innerq_last_error": (C.c_char_p, []),
        "innerq_tile_bytes": (i64, [i32]),
        "innerq_norm_factor": (i32, [vp, i32, i32, i32, i32, i32, i64, i64, i64, vp, vp]),
        "innerq_quant_pack": (i32, [vp, i32, i32, i32, i32, i32, i64, i64, i64, i32, i32, i32, i32,
                                    i32, vp, vp, vp, vp, i64, i64, vp]),
        "innerq_unpack_ref": (i32, [vp, vp, vp, i32, i32, i32, i64, i64, i32, i32, i32, i32, i32,
                                    i32, i64, vp, vp, vp, vp, vp]),
        "innerq_dequant": (i32, [vp, vp, vp, i32, i32, i32, i64, i64, i32, i32, i32, i32, i32, i32,
                                 i64, vp, vp, i64, i64, i64, vp]),
        "innerq_dequant_ref": (i32, [vp, vp, vp, i32, i64, i32, i32, i32, i32, i32, vp, vp]),
        "innerq_attn_plan": (i32, [C.POINTER(AttnArgs), C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
        "innerq_decode_attn_workspace": (i64, [C.POINTER(AttnArgs)]),
        "innerq_decode_attn": (i32, [C.POINTER(AttnArgs), vp, i64, vp, i64, i64, vp, vp]),
        "innerq_decode_attn_partials": (i32, [C.POINTER(AttnArgs), vp, vp, vp, vp, i64, vp]),
        "innerq_decode_attn_noalloc": (i32, [C.POINTER(AttnArgs), vp, i64, i64, vp, vp]),
        "innerq_append_step": (i32, [C.POINTER(AppendArgs), vp, vp]),
        "innerq_lse_merge": (i32, [vp, vp, vp, i32, i32, i32, i32, i32, vp, i64, i64, vp, vp]),
        "innerq_partials_rank_floats": (i64, [i32, i32, i32, i32]),
        "innerq_lse_merge_ranks": (i32, [vp, i32, i64, i32, i32, i32, i32, i32, vp, i64, i64, vp, vp]),
    }
    for name, (res, args) in sig.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    if lib.innerq_abi_version() != 5:
        raise ImportError("libinnerq_b200.so ABI version mismatch; rebuild it")
    _lib = lib
    return lib


# kernels each compute entry point launches (for launch accounting in bench.py)
KERNELS_PER_CALL = {
    "innerq_norm_factor": 1, "innerq_quant_pack": 1, "innerq_unpack_ref": 1, "innerq_dequant": 1,
    "innerq_dequant_ref": 1, "innerq_decode_attn": 3, "innerq_decode_attn_partials": 2,
    "innerq_lse_merge": 1, "innerq_decode_attn_noalloc": 3, "innerq_append_step": 1,
    "innerq_lse_merge_ranks": 1,
}
launch_count = [0]


def call(name: str, *args) -> int:
    """Call a status-returning entry point; raise InnerqError on failure."""
    lib = load()
    rc = getattr(lib, name)(*args)
    launch_count[0] += KERNELS_PER_CALL.get(name, 0)
    if rc != INNERQ_OK:
        raise InnerqError(name, rc, lib.innerq_last_error().decode())
    return rc


def last_error() -> str:
    return load().innerq_last_error().decode()
