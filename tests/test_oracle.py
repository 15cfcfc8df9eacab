"""The CPU oracle against the reference's own golden vectors and known-answer
tests (CPU only).  These pin the oracle before it is trusted as the checker
of the GPU kernels.

Sources of the cases (paths in gsoultan/mimir-model):
  quant_test.go:279-339   golden decode bits (testdata/quant_golden.json)
  quant_test.go:341-477   hand-built blocks
  internal/kernels/q8_test.go:25-165   8-bit activation rules
  internal/kernels/q8k_test.go:32-187  dotQ8KRef and its edge cases
  cmd/mim-run/main_test.go:179-267     tiny Llama logits and greedy ids
"""
import base64

import numpy as np
import pytest

import oracle as O
from conftest import load_tiny, f32b64, fma32 as _fma32

F16 = lambda f: int(O.lib().mo_f32_to_f16(f))  # noqa: E731


def le16(v):
    return bytes([v & 0xFF, v >> 8])


# ---------------------------------------------------------------- decode

@pytest.mark.parametrize("name,dt", [("q8_0", O.Q8_0), ("q4_k", O.Q4_K), ("q6_k", O.Q6_K)])
def test_dequantize_golden(quant_golden, name, dt):
    g = quant_golden[name]
    raw = np.frombuffer(base64.b64decode(g["bytes"]), np.uint8)
    bits = np.array(g["bits"], np.uint32)
    got = O.dequantize(dt, raw, bits.size).view(np.uint32)
    assert np.array_equal(got, bits)


def test_quantize_q8_0_golden(quant_golden):
    """quant_test.go:542-568: the Q8_0 encoder gives gguf's bytes."""
    g = quant_golden["q8_0"]
    x = np.array(g["input_bits"], np.uint32).view(np.float32)
    assert np.array_equal(O.quantize(O.Q8_0, x), np.frombuffer(base64.b64decode(g["bytes"]), np.uint8))


def test_hand_built_q8_0():
    blk = bytearray(le16(F16(0.5)) + bytes(32))
    blk[2], blk[33] = 0x7F, 0x80
    y = O.dequantize(O.Q8_0, np.frombuffer(bytes(blk), np.uint8), 32)
    assert y[0] == 63.5 and y[31] == -64 and y[1] == 0


def test_hand_built_q4_k_scales():
    blk = bytearray(144)
    blk[0:2], blk[2:4] = le16(F16(1)), le16(F16(0))
    sc = memoryview(blk)[4:16]
    for j in range(4):
        sc[j] = j + 1
    for j in range(4, 8):
        v = j + 1
        sc[j + 4] |= v & 0xF
        sc[j - 4] |= (v >> 4) << 6
    for i in range(16, 144):
        blk[i] = 0x11
    y = O.dequantize(O.Q4_K, np.frombuffer(bytes(blk), np.uint8), 256)
    assert all(y[i] == i // 32 + 1 for i in range(256))
    blk = bytearray(144)
    blk[0:2], blk[2:4] = le16(F16(1)), le16(F16(0.5))
    blk[4 + 8], blk[4 + 0], blk[4 + 4] = 0x35, 0x80, 0x40
    blk[16 + 64] = 0x02
    y = O.dequantize(O.Q4_K, np.frombuffer(bytes(blk), np.uint8), 256)
    assert y[128] == np.float32(37 * 2 - 0.5 * 19)
    assert y[129] == np.float32(-0.5 * 19)
    assert y[0] == 0 and y[160] == 0


def test_hand_built_q6_k():
    blk = bytearray(210)
    blk[208:210] = le16(F16(1))
    for i in range(192, 208):
        blk[i] = 1
    blk[0], blk[128], blk[192] = 0xF0, 0x01, 0xFE
    y = O.dequantize(O.Q6_K, np.frombuffer(bytes(blk), np.uint8), 256)
    assert y[0] == 32 and y[64] == -17 and y[32] == -32 and y[255] == -32


def test_f16_conversions():
    """float.go:24-88: exact widening, RNE narrowing, subnormals, inf, NaN."""
    lib = O.lib()
    for h in range(0, 0x10000, 7):
        f = np.float32(lib.mo_f16_to_f32(h))
        ref = np.array([h], np.uint16).view(np.float16).astype(np.float32)[0]
        if np.isnan(ref):
            assert np.isnan(f)
        else:
            assert f.view(np.uint32) == ref.view(np.uint32)
    xs = np.concatenate([np.random.default_rng(1).standard_normal(20000).astype(np.float32) * 1e-3,
                         np.float32([65504, 65520, 1e-8, 6e-8, 3e-8, -2.98e-8, 1e9, np.inf, -np.inf])])
    for x in xs:
        assert lib.mo_f32_to_f16(float(x)) == np.float32(x).astype(np.float16).view(np.uint16)
    assert lib.mo_f32_to_f16(float("nan")) & 0x7E00 == 0x7E00


# ------------------------------------------------------- 8-bit activations

def test_q8_ties_and_refusals():
    y = np.zeros(256, np.float32)
    y[0], y[1], y[2] = 254, 1, 3
    ok, q, d32, xs, _ = O.q8_quantize(y, 256)
    assert ok and (q[0], q[1], q[2]) == (127, 0, 2)
    for bad in (np.inf, -np.inf, np.nan, 1e30):
        y[5] = bad
        assert not O.q8_quantize(y, 256)[0]
    y[5] = 2.0 ** 60
    assert O.q8_quantize(y, 256)[0]
    z = O.gen_normal(3, 512)
    z[300] = 40
    ok, q, d32, xs, _ = O.q8_quantize(z, 256)
    assert ok and q[300] == 127 and np.all(d32[8:16] == np.float32(40) / np.float32(127))
    assert not O.q8_quantize(np.zeros(288, np.float32), 256)[0]
    assert not O.q8_quantize(np.zeros(64, np.float32), 64)[0]


def test_q8_rounding_near_half():
    """q8_test.go TestQuantQ8: values near the half-integer steps."""
    rng = np.random.default_rng(13)
    for _ in range(10):
        amax = np.float32(rng.exponential() * 10)
        h = (rng.integers(0, 255, 4096) - 127) / 2
        x = (h * float(amax) / 127).astype(np.float32)
        for _ in range(2):
            x = np.where(rng.random(4096) < 0.5, np.nextafter(x, np.float32(rng.standard_normal())), x)
        x = np.clip(x, -amax, amax).astype(np.float32)
        x[0] = amax
        ok, q, d32, xs, m32 = O.q8_quantize(x, 256)
        assert ok
        am = np.abs(x.reshape(-1, 256)).max(axis=1).repeat(256)
        want = np.rint(127 * x.astype(np.float64) / am.astype(np.float64)).astype(np.int8)
        assert np.array_equal(q, want)
        assert np.array_equal(xs, q.reshape(-1, 32).astype(np.int16).sum(axis=1).astype(np.int16))
        assert np.array_equal(m32, (32 * (q[0::2].astype(np.int16) + q[1::2])).astype(np.int16))


# ----------------------------------------------------------- dotQ8KRef

def dot_q8k_py(dt, row, q, d32, xs, k):
    """internal/kernels/q8k_test.go:35-117 restated in Python with exact
    rational fma, independent of the C oracle."""
    row = bytes(row)
    tot = off = np.float32(0)
    f16 = lambda b: (np.frombuffer(b, np.float16)[0].astype(np.float32), (b[0] | b[1] << 8) & 0x7C00 != 0x7C00)  # noqa
    for b in range(k // 256):
        y = q[256 * b:256 * b + 256].astype(np.int64)
        dx = d32[8 * b]
        if dt == O.Q4_K:
            blk = row[144 * b:144 * b + 144]
            d, ok1 = f16(blk[0:2])
            dmin, ok2 = f16(blk[2:4])
            if not (ok1 and ok2):
                return False, 0
            s = blk[4:16]
            sc = [s[j] & 63 for j in range(4)] + [(s[j + 8] & 0xF) | ((s[j] >> 6) << 4) for j in range(4)]
            m = [s[j + 4] & 63 for j in range(4)] + [(s[j + 8] >> 4) | ((s[j + 4] >> 6) << 4) for j in range(4)]
            qs = np.frombuffer(blk[16:144], np.uint8).astype(np.int64)
            S = 0
            for c in range(4):
                v = qs[32 * c:32 * c + 32]
                S += sc[2 * c] * int(((v & 15) * y[64 * c:64 * c + 32]).sum())
                S += sc[2 * c + 1] * int(((v >> 4) * y[64 * c + 32:64 * c + 64]).sum())
            M = sum(m[j] * int(xs[8 * b + j]) for j in range(8))
            tot = _fma32(np.float32(S), np.float32(d * dx), tot)
            off = _fma32(np.float32(M), np.float32(dmin * dx), off)
        else:
            blk = row[210 * b:210 * b + 210]
            d, ok = f16(blk[208:210])
            if not ok:
                return False, 0
            full = O.dequantize(O.Q6_K, np.frombuffer(blk[:208] + bytes(le16(0x3C00)), np.uint8), 256)
            # with d = 1 the decode is sc*(q-32) exactly: integers
            S = int((full.astype(np.int64) * y).sum())
            tot = _fma32(np.float32(S), np.float32(d * dx), tot)
    return True, np.float32(tot - off)


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
def test_dot_q8k_ref_edge_cases(dt):
    """q8k_test.go:122-187: tiny and huge activations, a zero block, the
    largest finite scales with all-ones quants, and subnormal scales."""
    k = 2048
    rows = []
    for i in range(4):
        x = O.gen_normal(100 + i, k)
        if i == 1:
            x *= np.float32(1e-30)
        if i == 2:
            x *= np.float32(1e15)
        if i == 3:
            x[:256] = 0
        rows.append(O.q8_quantize(x, 256))
        assert rows[-1][0]
    for trial in range(3):
        w = bytearray(O.gen_weight(dt, 7 + trial, 1, k).tobytes())
        bb = 144 if dt == O.Q4_K else 210
        if trial == 1:
            for o in range(0, len(w), bb):
                if dt == O.Q4_K:
                    w[o:o + 4] = bytes([0xFF, 0x7B, 0xFF, 0x7B])
                    w[o + 4:o + 144] = b"\xff" * 140
                else:
                    w[o + 208:o + 210] = bytes([0xFF, 0x7B])
                    w[o:o + 192] = b"\xff" * 192
                    w[o + 192:o + 208] = b"\x80" * 16
        if trial == 2:
            if dt == O.Q4_K:
                w[0:4] = bytes([0x01, 0x00, 0xFF, 0x03])
            else:
                w[208:210] = bytes([0x01, 0x00])
        row = np.frombuffer(bytes(w), np.uint8)
        for ok, q, d32, xs, _ in rows:
            got = O.dot_q8k_ref(dt, row, q, d32, xs, k)
            want = dot_q8k_py(dt, row, q, d32, xs, k)
            assert got[0] == want[0]
            assert np.float32(got[1]).view(np.uint32) == np.float32(want[1]).view(np.uint32)


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
def test_dot_q8k_simd_equals_scalar(dt):
    """The AVX2 block sums (the timed CPU baseline) and the scalar loops (the
    checker) give the same bits: random rows, rows of all-ones quants with
    the largest scales (the int16 pair sums at their extremes), activations
    saturated at +-127 and alternating signs."""
    if not O.simd_active():
        pytest.skip("oracle built without AVX2")
    k = 4096
    rng = np.random.default_rng(5)
    acts = [O.q8_quantize(O.gen_normal(300 + i, k), 256) for i in range(3)]
    x = np.where(np.arange(k) % 2 == 0, 1.0, -1.0).astype(np.float32)
    acts.append(O.q8_quantize(x, 256))                      # quants +-127
    acts.append(O.q8_quantize(np.ones(k, np.float32), 256))  # quants 127
    bb = 144 if dt == O.Q4_K else 210
    rows = [O.gen_weight(dt, 40 + i, 1, k) for i in range(4)]
    w = bytearray(rows[0].tobytes())
    for o in range(0, len(w), bb):
        if dt == O.Q4_K:
            w[o + 4:o + 144] = b"\xff" * 140
        else:
            w[o:o + 192] = b"\xff" * 192
            w[o + 192:o + 208] = bytes(rng.choice([0x80, 0x7F], 16).astype(np.uint8))
    rows.append(np.frombuffer(bytes(w), np.uint8))
    try:
        for row in rows:
            for ok, q, d32, xs, _ in acts:
                assert ok
                O.set_simd(True)
                a = O.dot_q8k_ref(dt, row, q, d32, xs, k)
                O.set_simd(False)
                b = O.dot_q8k_ref(dt, row, q, d32, xs, k)
                assert a[0] == b[0]
                assert np.float32(a[1]).view(np.uint32) == np.float32(b[1]).view(np.uint32)
        # and a whole product
        wm = O.gen_weight(dt, 77, 64, k)
        xm = O.gen_normal(78, 3 * k).reshape(3, k)
        O.set_simd(True)
        ya = O.dequant_matmul_a8(xm, dt, wm, 64)
        O.set_simd(False)
        yb = O.dequant_matmul_a8(xm, dt, wm, 64)
        assert np.array_equal(ya.view(np.uint32), yb.view(np.uint32))
    finally:
        O.set_simd(True)


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
def test_dot_q8k_refuses_nonfinite_scale(dt):
    k = 512
    w = bytearray(O.gen_weight(dt, 9, 1, k).tobytes())
    if dt == O.Q4_K:
        w[144 + 2:144 + 4] = le16(0x7C00)  # dmin = inf in block 1
    else:
        w[210 + 208:210 + 210] = le16(0x7E00)  # d = NaN in block 1
    ok, q, d32, xs, _ = O.q8_quantize(O.gen_normal(1, k), 256)
    assert O.dot_q8k_ref(dt, np.frombuffer(bytes(w), np.uint8), q, d32, xs, k)[0] is False


# --------------------------------------------------------------- encoders

@pytest.mark.parametrize("dt,tol", [(O.Q4_K, 0.12), (O.Q6_K, 0.03), (O.Q8_0, 0.01)])
def test_encoders_round_trip(dt, tol):
    x = O.gen_normal(5, 4096 * 4, 0.0, 0.02)
    y = O.dequantize(dt, O.quantize(dt, x), x.size)
    rel = np.linalg.norm(y - x) / np.linalg.norm(x)
    assert rel < tol, rel


# -------------------------------------------------------------- composites

def test_a8_matmul_falls_back_on_refused_rows():
    """linearA8 (interp/fast.go:282-379): a row with Inf or NaN, or a weight
    row with a non-finite scale, goes through the f32 product."""
    k, n = 512, 6
    w = bytearray(O.gen_weight(O.Q4_K, 11, n, k).tobytes())
    w[2 * 288:2 * 288 + 2] = le16(0x7C00)  # row 2, block 0: d = inf
    w = np.frombuffer(bytes(w), np.uint8)
    x = O.gen_normal(12, 3 * k).reshape(3, k)
    x[1, 7] = np.inf
    y8 = O.dequant_matmul_a8(x, O.Q4_K, w, n)
    y32 = O.dequant_matmul(x, O.Q4_K, w, n)
    assert np.array_equal(y8[1], y32[1], equal_nan=True)
    assert np.array_equal(y8[:, 2], y32[:, 2], equal_nan=True)
    assert not np.array_equal(y8[0, :2], y32[0, :2])


@pytest.mark.parametrize("name", ["llama", "qwen2"])
def test_tiny_llama_v1_matches_float64_oracle(name):
    """cmd/mim-run/main_test.go:179-216, both fixtures of the reference: the
    tiny Llama and the tiny Qwen 2 (query/key/value biases, rotation of head
    halves).  Prompt and 8 greedy steps of the dequant_matmul.v1 graph (f32
    cache) within 2e-5 of the largest logit, and the same greedy ids."""
    e, w = load_tiny(name)
    V = e["config"]["vocab"]
    m = O.Llama(dict(e["config"], a8=0, cache_f16=0, interleaved=int(name == "llama")), w)
    ids = e["prompt_ids"]
    all_ = m.forward(ids, np.arange(len(ids)), all_rows=True)
    want = f32b64(e["prompt_logits"]).reshape(len(ids), V)
    assert np.abs(all_ - want).max() <= 2e-5 * np.abs(want).max()
    logits, pos = all_[-1], len(ids)
    for i, nxt in enumerate(e["greedy"]):
        w_ = f32b64(e["greedy_logits"][i])
        assert np.abs(logits - w_).max() <= 2e-5 * np.abs(w_).max()
        assert O.argmax(logits) == nxt
        logits = m.forward([nxt], [pos])[0]
        pos += 1


@pytest.mark.parametrize("name", ["llama", "qwen2"])
@pytest.mark.parametrize("cache_f16,bound", [(0, 1.0), (1, 1.1)])
def test_tiny_llama_a8_within_llama_cpp(name, cache_f16, bound):
    """cmd/mim-run/main_test.go:218-267: the a8 graph stays within llama.cpp's
    own distance from the float64 oracle (x1.1 with the f16 cache)."""
    e, w = load_tiny(name)
    V = e["config"]["vocab"]
    m = O.Llama(dict(e["config"], a8=1, cache_f16=cache_f16, interleaved=int(name == "llama")), w)
    ids = e["prompt_ids"]
    all_ = m.forward(ids, np.arange(len(ids)), all_rows=True)
    worst = np.abs(all_ - f32b64(e["prompt_logits"]).reshape(len(ids), V)).max()
    logits, pos = all_[-1], len(ids)
    for i, nxt in enumerate(e["greedy"]):
        worst = max(worst, np.abs(logits - f32b64(e["greedy_logits"][i])).max())
        logits = m.forward([nxt], [pos])[0]
        pos += 1
    assert worst <= e["llama_cpp_max_diff"] * bound


def test_argmax_first_max_and_nan():
    v = np.float32([1, 3, 3, 2])
    assert O.argmax(v) == 1
    v = np.float32([np.nan, 5, 6])
    assert O.argmax(v) == 0
    v = np.float32([1, np.nan, 6, 6])
    assert O.argmax(v) == 2


def test_thread_pool_products_and_fork():
    """The oracle's persistent worker pool: repeated products give the same
    bits as one thread, and a process forked after the pool exists still
    runs products (its pool starts empty)."""
    import os
    import warnings
    w = O.gen_weight(O.Q4_K, 11, 300, 2048)
    x = O.gen_normal(12, 2 * 2048).reshape(2, 2048)
    one = O.dequant_matmul_a8(x, O.Q4_K, w, 300, nthreads=1)
    for _ in range(3):
        assert np.array_equal(O.dequant_matmul_a8(x, O.Q4_K, w, 300, nthreads=8).view(np.uint32), one.view(np.uint32))
    if not hasattr(os, "fork"):
        return
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", DeprecationWarning)
        pid = os.fork()
    if pid == 0:
        ok = np.array_equal(O.dequant_matmul_a8(x, O.Q4_K, w, 300, nthreads=8).view(np.uint32), one.view(np.uint32))
        os._exit(0 if ok else 3)
    _, status = os.waitpid(pid, 0)
    assert os.WIFEXITED(status) and os.WEXITSTATUS(status) == 0
