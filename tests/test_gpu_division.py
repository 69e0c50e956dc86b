"""The quantizer divides every element by its group's scale (quant.py:107,
:71), and the codes are only bit-exact if that quotient is the IEEE fp32 one.
With fp16 operands the kernels compute it with Markstein's sequence from one
correctly rounded reciprocal per divisor (div_rn, csrc/common.cuh); this test
checks that sequence against CUDA's '/' for every fp16 numerator and every
positive finite fp16 divisor (2 x 10^9 pairs), and with the compile-time
reciprocals of the quantizers' constant divisors 1, 3, 7, 15."""
import ctypes
import os
import shutil
import subprocess
import tempfile

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "innerq_b200", "csrc")


def test_markstein_division_matches_ieee_for_all_fp16_pairs():
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    with tempfile.TemporaryDirectory() as d:
        so = os.path.join(d, "div_check.so")
        subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-shared",
                        "-Xcompiler", "-fPIC", "-I", CSRC, "-o", so,
                        os.path.join(HERE, "cuda", "div_check.cu")], check=True)
        lib = ctypes.CDLL(so)
        n_bad, first = ctypes.c_ulonglong(0), ctypes.c_uint(0)
        assert lib.div_check(ctypes.byref(n_bad), ctypes.byref(first)) == 0
    assert n_bad.value == 0, f"{n_bad.value} mismatches, first a/b bits {first.value:#010x}"


@pytest.mark.parametrize("dtype", [0, 1], ids=["fp16", "bf16"])
def test_code_cuts_match_division_for_all_pairs(dtype):
    """The packers compute codes from per-group cuts instead of dividing each
    element (csrc/common.cuh, code_cuts): checked against rint(clamp(rnd(a/s)))
    with the IEEE quotient for every non-negative a and positive s of the dtype
    (~10^9 pairs), qmax 1, 3, 7, 15."""
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    with tempfile.TemporaryDirectory() as d:
        so = os.path.join(d, "code_check.so")
        subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-shared",
                        "-Xcompiler", "-fPIC", "-I", CSRC, "-o", so,
                        os.path.join(HERE, "cuda", "code_check.cu")], check=True)
        lib = ctypes.CDLL(so)
        n_bad, first = ctypes.c_ulonglong(0), ctypes.c_uint(0)
        assert lib.code_check(dtype, ctypes.byref(n_bad), ctypes.byref(first)) == 0
    assert n_bad.value == 0, f"{n_bad.value} mismatches, first a/s bits {first.value:#010x}"
