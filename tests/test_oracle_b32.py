"""The block-32 8-bit product (dequant_matmul_a8.v1) in the oracle.

The reference computes it only with AVX2 assembly (internal/kernels/
kernels_amd64.s:441 dotQ4KQ8AVX2, :763 dotQ6KQ8AVX2, :1007 dotQ8_0Q8AVX2;
RowDot.DotQ8, internal/kernels/q8.go:143-151).  The oracle restates those
kernels lane by lane (mo_dot_q8_b32).  It is pinned here three ways:

* against an independent Python restatement below, which takes the lane
  integers from the pinned dequantizer (decode with d = 1) instead of the C
  bit unpacking, and does every float step as an exact-rational fma;
* against the reference's own test of the kernels, TestRowDotQ8
  (internal/kernels/q8_test.go:183-234): the result within
  (K + 2) * 2^-24 * sum |xq| (|w| + 2 off) of the float64 product of the
  quantized activations and the decoded weights;
* against the refusal rules: TestDotQ8RejectsNonFiniteScales
  (q8_test.go:285-307) and linearA8's f32 fallback (interp/fast.go:324-377).
"""
import numpy as np
import pytest

import oracle as O
from conftest import fma32

BB = {O.Q4_K: 144, O.Q6_K: 210, O.Q8_0: 34}


def _f16(b):
    return np.frombuffer(bytes(b), np.float16)[0].astype(np.float32), (b[0] | b[1] << 8) & 0x7C00 != 0x7C00


def _decode_with(dt, row, k, d=None, dmin=None):
    """The row decoded with its f16 scales replaced (d = 1 makes Q4_K and
    Q6_K decode to sc*q and sc*(q-32), Q8_0 to q: exact integers)."""
    w = bytearray(bytes(row))
    bb = BB[dt]
    for o in range(0, len(w), bb):
        if dt == O.Q4_K:
            w[o:o + 2] = np.float16(d).tobytes()
            w[o + 2:o + 4] = np.float16(dmin).tobytes()
        elif dt == O.Q6_K:
            w[o + 208:o + 210] = np.float16(d).tobytes()
        else:
            w[o:o + 2] = np.float16(d).tobytes()
    return O.dequantize(dt, np.frombuffer(bytes(w), np.uint8), k)


def hsum1(v):
    a = [np.float32(v[i] + v[i + 4]) for i in range(4)]
    return np.float32(np.float32(a[0] + a[1]) + np.float32(a[2] + a[3]))


def dot_q8_b32_py(dt, row, q, d32, xs, k):
    """The AVX2 block-32 kernels restated from the assembly, independently of
    the C oracle: 8 lanes of 4 consecutive elements per run of 32."""
    row = bytes(row)
    y = q.astype(np.int64)
    if dt == O.Q8_0:
        ints = _decode_with(dt, row, k, 1.0).astype(np.int64)
        lanes = (ints * y).reshape(k // 32, 8, 4).sum(axis=2)
        acc = [np.float32(0)] * 8
        for b in range(k // 32):
            d, ok = _f16(row[34 * b:34 * b + 2])
            if not ok:
                return False, 0
            scale = np.float32(d * d32[b])
            acc = [fma32(scale, np.float32(lanes[b, l]), acc[l]) for l in range(8)]
        return True, hsum1(acc)
    nb = k // 256
    ints = _decode_with(dt, row, k, 1.0, 0.0).astype(np.int64)
    lanes = (ints * y).reshape(nb, 8, 8, 4).sum(axis=3)  # [block, run of 32, lane]
    if dt == O.Q4_K:
        mneg = _decode_with(dt, row, k, 0.0, 1.0)  # -m of each run of 32
        m = (-mneg.reshape(nb, 8, 32)[:, :, 0]).astype(np.int64)
    y2 = [np.float32(0)] * 8
    y3 = [np.float32(0)] * 8
    for b in range(nb):
        blk = row[BB[dt] * b:BB[dt] * (b + 1)]
        if dt == O.Q4_K:
            (d, ok1), (dmin, ok2) = _f16(blk[0:2]), _f16(blk[2:4])
            if not (ok1 and ok2):
                return False, 0
            for s in range(8):
                dm = np.float32(dmin * np.float32(m[b, s]))
                dbs = np.float32(d32[8 * b + s] * np.float32(xs[8 * b + s]))
                y3[s] = fma32(dm, dbs, y3[s])
        else:
            d, ok = _f16(blk[208:210])
            if not ok:
                return False, 0
        acc = [[np.float32(0)] * 8, [np.float32(0)] * 8]
        for s in range(8):  # Y0 takes the even runs of 32, Y1 the odd, in order
            for l in range(8):
                acc[s & 1][l] = fma32(d32[8 * b + s], np.float32(lanes[b, s, l]), acc[s & 1][l])
        y2 = [fma32(d, np.float32(acc[0][l] + acc[1][l]), y2[l]) for l in range(8)]
    return True, hsum1([np.float32(y2[l] - y3[l]) for l in range(8)])


def _row(dt, seed, k, edge=0):
    w = bytearray(O.gen_weight(dt, seed, 1, k).tobytes())
    if dt == O.Q8_0:
        w[2] = 0x80  # a weight of -128 (q8_test.go:195-197)
    if edge == 1:  # largest finite scales, all-ones quants
        for o in range(0, len(w), BB[dt]):
            if dt == O.Q4_K:
                w[o:o + 4] = bytes([0xFF, 0x7B, 0xFF, 0x7B])
                w[o + 4:o + 144] = b"\xff" * 140
            elif dt == O.Q6_K:
                w[o + 208:o + 210] = bytes([0xFF, 0x7B])
                w[o:o + 192] = b"\xff" * 192
                w[o + 192:o + 208] = b"\x80" * 16
            else:
                w[o:o + 2] = bytes([0xFF, 0x7B])
                w[o + 2:o + 34] = b"\x81" * 32
    if edge == 2:  # subnormal scales
        if dt == O.Q4_K:
            w[0:4] = bytes([0x01, 0x00, 0xFF, 0x03])
        elif dt == O.Q6_K:
            w[208:210] = bytes([0x01, 0x00])
        else:
            w[0:2] = bytes([0x01, 0x00])
    return np.frombuffer(bytes(w), np.uint8)


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K, O.Q8_0])
def test_b32_matches_independent_restatement(dt):
    k = 1024
    acts = []
    for i in range(4):
        x = O.gen_normal(200 + i, k)
        if i == 1:
            x *= np.float32(1e-30)
        if i == 2:
            x *= np.float32(1e15)
        if i == 3:
            x[:256] = 0
        acts.append(O.q8_quantize(x, 32))
        assert acts[-1][0]
    for edge in range(3):
        row = _row(dt, 30 + edge, k, edge)
        for ok, q, d32, xs, _ in acts:
            got = O.dot_q8_b32(dt, row, q, d32, xs, k)
            want = dot_q8_b32_py(dt, row, q, d32, xs, k)
            assert got[0] == want[0]
            assert np.float32(got[1]).view(np.uint32) == np.float32(want[1]).view(np.uint32), (edge, got, want)


def _offsets(dt, row, k):
    """q8_test.go:166-181: |dmin*m| per weight for Q4_K, zero otherwise."""
    if dt != O.Q4_K:
        return np.zeros(k)
    z = bytearray(bytes(row))
    for b in range(0, len(z), 144):
        z[b + 16:b + 144] = bytes(128)
    return np.abs(O.dequantize(dt, np.frombuffer(bytes(z), np.uint8), k).astype(np.float64))


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K, O.Q8_0])
@pytest.mark.parametrize("k", [256, 2048, 5632])
def test_b32_within_reference_bound(dt, k):
    """TestRowDotQ8 (q8_test.go:183-234) for blocks of 32."""
    row = _row(dt, 7 + k, k)
    w = O.dequantize(dt, row, k).astype(np.float64)
    off = _offsets(dt, row, k)
    for trial in range(3):
        x = O.gen_normal(1000 * trial + k, k)
        if trial == 1:
            x *= np.float32(1e-3)
        x[3] = 0
        ok, q, d32, xs, _ = O.q8_quantize(x, 32)
        assert ok
        xq = q.astype(np.float64) * d32.astype(np.float64)[np.arange(k) // 32]
        want = float((xq * w).sum())
        bound = float((np.abs(xq) * (np.abs(w) + 2 * off)).sum())
        good, got = O.dot_q8_b32(dt, row, q, d32, xs, k)
        assert good
        assert abs(float(got) - want) <= (k + 2) * 2.0**-24 * bound, (dt, k, trial)


@pytest.mark.parametrize("dt,off", [(O.Q4_K, 0), (O.Q4_K, 2), (O.Q6_K, 208), (O.Q8_0, 0)])
def test_b32_refuses_nonfinite_scale(dt, off):
    """TestDotQ8RejectsNonFiniteScales (q8_test.go:285-307): +inf in the
    second block's scale."""
    k = 512
    w = bytearray(O.gen_weight(dt, 8, 1, k).tobytes())
    w[BB[dt] + off:BB[dt] + off + 2] = bytes([0x00, 0x7C])
    ok, q, d32, xs, _ = O.q8_quantize(O.gen_normal(3, k), 32)
    assert O.dot_q8_b32(dt, np.frombuffer(bytes(w), np.uint8), q, d32, xs, k)[0] is False


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K, O.Q8_0])
def test_b32_matmul_rows_and_fallbacks(dt):
    """linearA8 with blocks of 32: each output is the row kernel's value
    (plus bias); a row of x the quantizer refuses, or a weight row with a
    non-finite scale, takes the f32 product."""
    k, n = 512, 5
    w = bytearray(O.gen_weight(dt, 13, n, k).tobytes())
    rb = len(w) // n
    o = 2 * rb + (208 if dt == O.Q6_K else 0)  # row 2, block 0: d = +inf
    w[o:o + 2] = bytes([0x00, 0x7C])
    w = np.frombuffer(bytes(w), np.uint8)
    x = O.gen_normal(14, 3 * k).reshape(3, k)
    x[1, 9] = np.nan
    bias = O.gen_normal(15, n)
    y8 = O.dequant_matmul_a8(x, dt, w, n, bias=bias, block=32)
    y32 = O.dequant_matmul(x, dt, w, n, bias=bias)
    assert np.array_equal(y8[1], y32[1], equal_nan=True)
    assert np.array_equal(y8[:, 2], y32[:, 2], equal_nan=True)
    for i in (0, 2):
        ok, q, d32, xs, _ = O.q8_quantize(x[i], 32)
        assert ok
        for j in (0, 1, 3, 4):
            good, v = O.dot_q8_b32(dt, w[j * rb:(j + 1) * rb], q, d32, xs, k)
            assert good
            assert np.float32(v + bias[j]).view(np.uint32) == y8[i, j].view(np.uint32)
    assert not np.array_equal(y8[0, :2], y32[0, :2])
