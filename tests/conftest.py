"""Shared pytest configuration.

Markers: `gpu` for tests that need a B200 (run with -m gpu on the GPU box);
everything else runs on the CPU.
"""
import base64
import json
import os
import sys
from fractions import Fraction

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
for sub in ("oracle", "mimir-model_b200"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def round_f32(v: Fraction) -> np.float32:
    """The f32 nearest the rational v, ties to even."""
    f = np.float32(float(v))
    best = f
    for c in (np.nextafter(f, np.float32(-np.inf)), np.nextafter(f, np.float32(np.inf))):
        dc, db = abs(Fraction(float(c)) - v), abs(Fraction(float(best)) - v)
        if dc < db or (dc == db and (int(c.view(np.uint32)) & 1) == 0):
            best = c
    return np.float32(best)


def fma32(a, b, c) -> np.float32:
    """f32 fused multiply-add a*b + c, rounded once (exact rationals)."""
    return round_f32(Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c)))


def f32b64(s: str) -> np.ndarray:
    return np.frombuffer(base64.b64decode(s), np.float32)


def load_tiny(name: str = "llama"):
    """The reference's tiny Llama fixture: (expected dict, {name: (dtype, bytes)})."""
    with open(os.path.join(GOLDEN, f"tiny_{name}.json")) as f:
        e = json.load(f)
    blob = np.fromfile(os.path.join(GOLDEN, f"tiny_{name}.bin"), np.uint8)
    w = {t["name"]: (t["dtype"], blob[t["offset"]:t["offset"] + t["nbytes"]]) for t in e["tensors"]}
    return e, w


@pytest.fixture(scope="session")
def tiny():
    return load_tiny("llama")


@pytest.fixture(scope="session")
def quant_golden():
    with open(os.path.join(GOLDEN, "quant_golden.json")) as f:
        return json.load(f)
