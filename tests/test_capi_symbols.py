"""The product library loads without a GPU and exports every function that
include/dsv4_cuda.h declares (no compute call is made here)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dsv4_cuda.h")
LIB = os.path.join(ROOT, "deepseek-v4-flash-0731-in-c_b200", "lib", "libdsv4_cuda.so")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"\b(dsv4\w*)\s*\(", text)
    return sorted(set(n for n in names if not n.isupper()))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        import subprocess, sys
        subprocess.run([sys.executable, os.path.join(ROOT, "deepseek-v4-flash-0731-in-c_b200",
                                                     "build.py")], check=True)
    return ctypes.CDLL(LIB)


def test_header_lists_the_dropin_abi():
    names = declared_functions()
    for n in ("dsv4_gemv_fp4_q", "dsv4_gemv_fp4_pair_q", "dsv4_gemv_fp4_batch_q",
              "dsv4_gemv_fp8_q", "dsv4_gemv_fp8_pair_q", "dsv4_gemv_fp8_batch_q",
              "dsv4_gemv_bf16", "dsv4_gemv_bf16_batch", "dsv4_quant_fp8_codes",
              "dsv4cuda_moe_forward"):
        assert n in names


def test_every_declared_symbol_is_exported(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_no_cpu_fallback_symbols(lib):
    # the product must not carry the oracle
    assert not hasattr(lib, "orc_gemv_fp4_q")
