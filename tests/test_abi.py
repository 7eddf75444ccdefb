"""The C-ABI library loads, exports every function declared in include/qlin.h
and rejects bad arguments before touching the GPU (no compute calls here)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qlin.h")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(qlin_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_hot_path():
    names = declared()
    for fn in ("qlin_gemm_i8", "qlin_gemm_w4", "qlin_proj3", "qlin_proj3_w4", "qlin_mlp_gate_up",
               "qlin_mlp_gate_up_quant", "qlin_mlp_gate_up_quant_w4", "qlin_quant_row"):
        assert fn in names


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg._lib.load()
    for name in declared():
        assert hasattr(lib, name), name
    # the Python binding covers the same set
    assert set(pkg._lib.SIGNATURES) == set(declared())


def test_version_and_status_strings(pkg):
    lib = pkg._lib.load()
    assert lib.qlin_version() >= 100
    assert lib.qlin_status_string(0) == b"ok"
    assert lib.qlin_status_string(2) == b"unsupported shape"


@pytest.mark.parametrize("K", [0, 63, 100])
def test_bad_k_rejected_without_gpu(pkg, K):
    lib = pkg._lib.load()
    rc = lib.qlin_gemm_i8(16, 16, 1, K, 16, 16, 128, 16, 128, None, 0, None)
    assert rc == 2
    assert b"multiple of 64" in lib.qlin_last_error()


def test_bad_n_alignment_rejected(pkg):
    lib = pkg._lib.load()
    assert lib.qlin_gemm_i8(16, 16, 1, 64, 16, 16, 100, 16, 100, None, 0, None) == 3


def test_null_activation_rejected(pkg):
    lib = pkg._lib.load()
    assert lib.qlin_gemm_i8(None, 16, 1, 64, 16, 16, 128, 16, 128, None, 0, None) == 1


def test_bad_w4_group_rejected(pkg):
    lib = pkg._lib.load()
    rc = lib.qlin_gemm_w4(16, 16, 1, 256, 16, 16, None, 128, 48, 16, 128, None, 0, None)
    assert rc == 2


def test_empty_problem_is_noop(pkg):
    lib = pkg._lib.load()
    assert lib.qlin_gemm_i8(16, 16, 0, 64, 16, 16, 128, 16, 128, None, 0, None) == 0
