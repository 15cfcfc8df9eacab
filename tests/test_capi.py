"""The C ABI library (CPU-side checks, no GPU compute).

libmimgpu.so must load and export every entry point include/mimgpu.h
declares, and the Python binding must bind exactly those.
"""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "mimgpu.h")


def declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mimgpu_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared()
    for must in ("mimgpu_open", "mimgpu_upload", "mimgpu_dequant_matmul_a8", "mimgpu_session_run"):
        assert must in names


def test_library_exports_every_declared_symbol():
    import mimgpu
    lib = ctypes.CDLL(mimgpu.LIB_PATH)
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_matches_header():
    import mimgpu
    assert sorted(mimgpu.SIGNATURES) == declared()
    assert mimgpu.lib().mimgpu_abi_version() == 1


def test_open_without_device_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import mimgpu
    h = ctypes.c_void_p()
    rc = mimgpu.lib().mimgpu_open(0, ctypes.byref(h))
    assert rc == mimgpu.ECUDA and not h.value


def test_library_has_no_oracle_dependency():
    """The product library must not link or name the CPU oracle."""
    import mimgpu
    data = open(mimgpu.LIB_PATH, "rb").read()
    assert b"mimoracle" not in data and b"mo_dot_q8k_ref" not in data
