"""ctypes wrapper of the CPU oracle (libmimoracle.so).

TEST INFRASTRUCTURE, NOT PRODUCT.  Only tests/, __graft_entry__.smoke() and
bench.py's CPU legs import this module, as the checker or as the timed CPU
baseline.  The GPU library never calls into it.

Each function restates the Go reference; see mimoracle.h for the file:line
each one follows.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmimoracle.so")

F32, F16, Q8_0, Q4_K, Q6_K = 1, 2, 64, 66, 67
BLOCK = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}


def _cpu_has_avx2() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            flags = f.read()
        return " avx2" in flags and " fma" in flags
    except OSError:
        return False


def build(force: bool = False) -> str:
    """Compiles the oracle with its Makefile (gcc), generic x86-64 when the
    host lacks AVX2/FMA."""
    src = os.path.join(HERE, "mimoracle.c")
    if not force and os.path.exists(LIB_PATH) and os.path.getmtime(LIB_PATH) >= os.path.getmtime(src):
        return LIB_PATH
    arch = "ARCH=-march=x86-64-v3" if _cpu_has_avx2() else "ARCH=-march=x86-64"
    subprocess.run(["make", "-s", "-C", HERE, arch], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(LIB_PATH)
        P, I64, I32, F, D = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_double
        sig = {
            "mo_f16_to_f32": (F, [C.c_uint16]),
            "mo_f32_to_f16": (C.c_uint16, [F]),
            "mo_row_bytes": (I64, [I32, I64]),
            "mo_dequantize": (I32, [I32, P, P, I64]),
            "mo_quantize": (I32, [I32, P, P, I64]),
            "mo_gen_weight": (I32, [I32, C.c_uint64, I64, I64, F, P, I32]),
            "mo_gen_weight_rows": (I32, [I32, C.c_uint64, I64, I64, I64, F, P, I32]),
            "mo_gen_normal": (None, [C.c_uint64, I64, F, F, P]),
            "mo_q8_quantize": (I32, [P, I64, I32, P, P, P, P]),
            "mo_dot_q8k_ref": (I32, [I32, P, P, P, P, I64, P]),
            "mo_set_simd": (None, [I32]),
            "mo_simd_active": (I32, []),
            "mo_dot_q8_b32": (I32, [I32, P, P, P, P, I64, P]),
            "mo_dot_f32": (F, [P, P, I64]),
            "mo_dequant_matmul": (I32, [P, I64, I64, I32, P, I64, P, P, I32]),
            "mo_dequant_matmul_a8": (I32, [P, I64, I64, I32, P, I64, P, I32, P, I32]),
            "mo_rms_norm": (None, [P, I64, I64, P, D, P]),
            "mo_rope": (I32, [P, I32, I32, I32, I32, P, I32, D, I32, I32, P]),
            "mo_attention": (I32, [P, I32, I32, I32, I32, P, P, I32, I32, I32, P, P, D, I32, P]),
            "mo_swiglu": (None, [P, P, I64, P]),
            "mo_embedding": (I32, [I32, P, I64, I64, P, I64, P]),
            "mo_argmax": (I32, [P, I64]),
            "mo_cast_f16": (None, [P, P, I64]),
            "mo_llama_new": (P, [P]),
            "mo_llama_free": (None, [P]),
            "mo_llama_set_weight": (I32, [P, C.c_char_p, I32, P]),
            "mo_llama_reset": (None, [P]),
            "mo_llama_forward": (I32, [P, P, P, I32, P, I32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def set_simd(on: bool) -> None:
    """dotQ8KRef's exact block sums in AVX2 (default) or by the scalar loops:
    the same bits either way (tests/test_oracle.py checks)."""
    lib().mo_set_simd(1 if on else 0)


def simd_active() -> bool:
    return bool(lib().mo_simd_active())


def threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def row_bytes(dt: int, k: int) -> int:
    return int(lib().mo_row_bytes(dt, k))


def dequantize(dt: int, raw: np.ndarray, n: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.empty(n, np.float32)
    if lib().mo_dequantize(dt, _p(raw), _p(out), n) != 0:
        raise ValueError("dequantize: bad dtype or length")
    return out


def quantize(dt: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    be, bb = BLOCK[dt]
    out = np.empty(x.size // be * bb, np.uint8)
    if lib().mo_quantize(dt, _p(x), _p(out), x.size) != 0:
        raise ValueError("quantize: bad dtype or length")
    return out


def gen_weight(dt: int, seed: int, n: int, k: int, sigma: float = 0.02, nthreads: int | None = None) -> np.ndarray:
    out = np.empty(n * row_bytes(dt, k), np.uint8)
    rc = lib().mo_gen_weight(dt, seed, n, k, sigma, _p(out), nthreads or threads())
    if rc != 0:
        raise ValueError("gen_weight: bad dtype or k")
    return out.reshape(n, -1)


def gen_weight_rows(dt: int, seed: int, row0: int, n: int, k: int, sigma: float = 0.02,
                    nthreads: int | None = None) -> np.ndarray:
    """Rows [row0, row0 + n) of gen_weight(dt, seed, ...): a shard, byte for byte."""
    out = np.empty(n * row_bytes(dt, k), np.uint8)
    rc = lib().mo_gen_weight_rows(dt, seed, row0, n, k, sigma, _p(out), nthreads or threads())
    if rc != 0:
        raise ValueError("gen_weight_rows: bad dtype, k or row")
    return out


def gen_normal(seed: int, n: int, mean: float = 0.0, sigma: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().mo_gen_normal(seed, n, mean, sigma, _p(out))
    return out


def q8_quantize(x: np.ndarray, block: int = 256):
    """Returns (ok, q int8[k], d32 f32[k/32], xs i16[k/32], m32 i16[k/2])."""
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    k = x.size
    q = np.zeros(k, np.int8)
    d32 = np.zeros(max(k // 32, 1), np.float32)
    xs = np.zeros(max(k // 32, 1), np.int16)
    m32 = np.zeros(max(k // 2, 1), np.int16)
    ok = lib().mo_q8_quantize(_p(x), k, block, _p(q), _p(d32), _p(xs), _p(m32))
    return bool(ok), q, d32, xs, m32


def dot_q8k_ref(dt: int, row: np.ndarray, q, d32, xs, k: int):
    out = np.zeros(1, np.float32)
    ok = lib().mo_dot_q8k_ref(dt, _p(np.ascontiguousarray(row, np.uint8)), _p(q), _p(d32), _p(xs), k, _p(out))
    return bool(ok), out[0]


def dot_q8_b32(dt: int, row: np.ndarray, q, d32, xs, k: int):
    """RowDot.DotQ8 with blocks of 32 (the AVX2 kernels, restated)."""
    out = np.zeros(1, np.float32)
    ok = lib().mo_dot_q8_b32(dt, _p(np.ascontiguousarray(row, np.uint8)), _p(q), _p(d32), _p(xs), k, _p(out))
    return bool(ok), out[0]


def dot_f32(a: np.ndarray, b: np.ndarray) -> np.float32:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return np.float32(lib().mo_dot_f32(_p(a), _p(b), a.size))


def dequant_matmul(x: np.ndarray, dt: int, w: np.ndarray, n: int, bias=None, nthreads=None) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    k = x.shape[-1]
    rows = x.size // k if k else 0
    y = np.empty(x.shape[:-1] + (n,), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    if lib().mo_dequant_matmul(_p(x), rows, k, dt, _p(np.ascontiguousarray(w, np.uint8)), n, _p(b), _p(y),
                               nthreads or threads()) != 0:
        raise ValueError("dequant_matmul: bad shapes")
    return y


def dequant_matmul_a8(x: np.ndarray, dt: int, w: np.ndarray, n: int, bias=None, block: int = 256,
                      nthreads=None) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    k = x.shape[-1]
    rows = x.size // k if k else 0
    y = np.empty(x.shape[:-1] + (n,), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    if lib().mo_dequant_matmul_a8(_p(x), rows, k, dt, _p(np.ascontiguousarray(w, np.uint8)), n, _p(b), block, _p(y),
                                  nthreads or threads()) != 0:
        raise ValueError("dequant_matmul_a8: bad shapes or block")
    return y


def rms_norm(x: np.ndarray, scale: np.ndarray | None, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    n = x.shape[-1]
    y = np.empty_like(x)
    s = None if scale is None else np.ascontiguousarray(scale, np.float32)
    lib().mo_rms_norm(_p(x), x.size // n, n, _p(s), eps, _p(y))
    return y


def rope(x: np.ndarray, pos: np.ndarray, theta: float, rotary: int | None = None, interleaved: bool = True):
    x = np.ascontiguousarray(x, np.float32)
    B, H, T, D = x.shape
    pos = np.ascontiguousarray(pos, np.int64)
    y = np.empty_like(x)
    if lib().mo_rope(_p(x), B, H, T, D, _p(pos), pos.shape[0], theta, rotary or D, int(interleaved), _p(y)) != 0:
        raise ValueError("rope: bad rotary_dims")
    return y


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, mask: np.ndarray | None = None,
              scale: float | None = None, causal: bool = False) -> np.ndarray:
    """q f32 [B,Hq,Tq,D]; k, v f32 or f16 [B,Hkv,Tk,D]; mask bool, broadcastable."""
    q = np.ascontiguousarray(q, np.float32)
    B, Hq, Tq, D = q.shape
    Hkv, Tk = k.shape[1], k.shape[2]
    kvdt = F16 if k.dtype == np.float16 else F32
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    out = np.empty_like(q)
    ms = None
    if mask is not None:
        mask = np.ascontiguousarray(mask, np.uint8)
        ms = np.array(mask.shape, np.int32)
    sc = scale if scale is not None else 1.0 / np.sqrt(float(D))
    rc = lib().mo_attention(_p(q), B, Hq, Tq, D, _p(k), _p(v), kvdt, Hkv, Tk, _p(mask), _p(ms), sc, int(causal),
                            _p(out))
    if rc != 0:
        raise ValueError("attention: bad heads")
    return out


def swiglu(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    y = np.empty_like(a)
    lib().mo_swiglu(_p(a), _p(b), a.size, _p(y))
    return y


def embedding(dt: int, table: np.ndarray, V: int, E: int, ids: np.ndarray) -> np.ndarray:
    ids = np.ascontiguousarray(ids, np.int32)
    y = np.empty(ids.shape + (E,), np.float32)
    lib().mo_embedding(dt, _p(np.ascontiguousarray(table, np.uint8)), V, E, _p(ids), ids.size, _p(y))
    return y


def argmax(v: np.ndarray) -> int:
    v = np.ascontiguousarray(v, np.float32)
    return int(lib().mo_argmax(_p(v), v.size))


def cast_f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(x.shape, np.uint16)
    lib().mo_cast_f16(_p(x), _p(y), x.size)
    return y


class LlamaConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("layers", "embed", "ffn", "heads", "kv_heads", "head_dim", "rope_dims",
                                       "vocab", "context")] + [("rope_theta", C.c_double), ("norm_eps", C.c_double)] + \
               [(n, C.c_int) for n in ("a8", "cache_f16", "interleaved", "nthreads")]


class Llama:
    """The llama graph of importer/llama.go:317-547 run op by op on the CPU."""

    def __init__(self, cfg: dict, weights: dict):
        c = LlamaConfig(**{k: cfg[k] for k, _ in LlamaConfig._fields_ if k in cfg})
        if c.nthreads <= 0:
            c.nthreads = threads()
        self.cfg = cfg
        self.vocab = c.vocab
        self._h = lib().mo_llama_new(C.byref(c))
        if not self._h:
            raise ValueError("bad llama config")
        self._keep = []
        for name, (dt, arr) in weights.items():
            arr = np.ascontiguousarray(arr)
            self._keep.append(arr)
            if lib().mo_llama_set_weight(self._h, name.encode(), dt, _p(arr)) != 0:
                raise ValueError(f"unknown weight {name}")

    def reset(self):
        lib().mo_llama_reset(self._h)

    def forward(self, tokens, positions, all_rows: bool = False) -> np.ndarray:
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(positions, np.int64)
        T = t.size
        out = np.empty((T if all_rows else 1, self.vocab), np.float32)
        if lib().mo_llama_forward(self._h, _p(t), _p(p), T, _p(out), int(all_rows)) != 0:
            raise ValueError("forward failed (missing weight or position out of range)")
        return out

    def __del__(self):
        if getattr(self, "_h", None):
            lib().mo_llama_free(self._h)
            self._h = None
