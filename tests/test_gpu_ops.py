"""Per-op parity of the GPU fast paths against the CPU oracle, through the
C ABI (libmimgpu.so via ctypes).  Needs a B200.

Bars (reference file:line in gsoultan/mimir-model):
  dequantize           bit-exact (quant.go:197-344, testdata/quant_golden.json)
  dequant_matmul_a8.v2 bit-exact with dotQ8KRef (internal/kernels/q8k_test.go:35-117),
                       batch-invariant (interp/transformer_test.go:297-354)
  dequant_matmul_a8.v1 bit-exact with the AVX2 block-32 kernels (kernels_amd64.s:441,
                       763, 1007) as the oracle restates them; batch-invariant
  dequant_matmul.v1    spec/stdlib.md section 3.3: |err| <= (K+1) u sum|x w| + |bias|,
                       and max relative error <= 1e-3
  rms_norm, rope, swiglu, embedding   bit-exact with the oracle except where a
                       reference float64 step could round differently (noted per test)
  attention            spec/stdlib.md section 6.2: (4 D S + 2 Tk + 64) u V
"""
import base64

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
U = 2.0 ** -24


@pytest.fixture(scope="module")
def ctx():
    import mimgpu
    c = mimgpu.Context(0)
    yield c
    c.close()


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# ------------------------------------------------------------- dequantize

@pytest.mark.parametrize("name,dt", [("q8_0", O.Q8_0), ("q4_k", O.Q4_K), ("q6_k", O.Q6_K)])
def test_dequantize_golden(ctx, quant_golden, name, dt):
    g = quant_golden[name]
    raw = np.frombuffer(base64.b64decode(g["bytes"]), np.uint8)
    want = np.array(g["bits"], np.uint32)
    assert np.array_equal(bits(ctx.dequantize(dt, raw, want.size)), want)


@pytest.mark.parametrize("dt", [O.Q8_0, O.Q4_K, O.Q6_K])
def test_dequantize_random_and_edge_blocks(ctx, dt):
    be, bb = O.BLOCK[dt]
    rng = np.random.default_rng(dt)
    raw = rng.integers(0, 256, 64 * bb, dtype=np.uint8)
    # finite scales in most blocks; keep a few inf/nan/subnormal ones
    want = O.dequantize(dt, raw, 64 * be)
    got = ctx.dequantize(dt, raw, 64 * be)
    # NaN payloads after arithmetic are not specified by IEEE 754; every
    # other value (subnormals and infinities included) must match bit for bit
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(bits(got[~nan]), bits(want[~nan]))


# -------------------------------------------------- 8-bit activation GEMV

def _weights(dt, n, k, seed):
    return O.gen_weight(dt, seed, n, k)


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
@pytest.mark.parametrize("n,k,rows", [(8, 256, 1), (37, 2048, 1), (64, 5632, 3), (300, 4096, 1),
                                      (129, 4096, 5), (96, 11008, 2), (24, 14336, 8), (40, 4096, 16)])
def test_a8_bit_exact(ctx, dt, n, k, rows):
    w = _weights(dt, n, k, 1000 + n)
    x = O.gen_normal(7 + rows, rows * k).reshape(rows, k)
    bias = O.gen_normal(3, n)
    t = ctx.upload(dt, (n, k), w)
    want = O.dequant_matmul_a8(x, dt, w, n, bias)
    got = ctx.dequant_matmul(x, t, bias, a8_block=256)
    assert np.array_equal(bits(got), bits(want))
    t.free()


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
def test_a8_edge_cases(ctx, dt):
    """q8k_test.go:122-187: tiny and huge activations, a zero block, the
    largest finite scales, subnormal scales; plus refused rows (Inf, NaN)
    and a weight row with a non-finite scale (fast.go:282-379)."""
    k, n = 2048, 16
    bb = 144 if dt == O.Q4_K else 210
    w = bytearray(_weights(dt, n, k, 77).tobytes())
    rb = k // 256 * bb
    for o in range(rb, 2 * rb, bb):  # row 1: largest finite scales, all-ones quants
        if dt == O.Q4_K:
            w[o:o + 4] = bytes([0xFF, 0x7B, 0xFF, 0x7B])
            w[o + 4:o + 144] = b"\xff" * 140
        else:
            w[o + 208:o + 210] = bytes([0xFF, 0x7B])
            w[o:o + 192] = b"\xff" * 192
            w[o + 192:o + 208] = b"\x80" * 16
    if dt == O.Q4_K:  # row 2: subnormal scales; row 3: dmin = inf
        w[2 * rb:2 * rb + 4] = bytes([0x01, 0x00, 0xFF, 0x03])
        w[3 * rb + 2:3 * rb + 4] = bytes([0x00, 0x7C])
    else:
        w[2 * rb + 208:2 * rb + 210] = bytes([0x01, 0x00])
        w[3 * rb + 208:3 * rb + 210] = bytes([0x00, 0x7E])
    w = np.frombuffer(bytes(w), np.uint8)
    x = O.gen_normal(5, 6 * k).reshape(6, k)
    x[1] *= np.float32(1e-30)
    x[2] *= np.float32(1e15)
    x[3, :256] = 0
    x[4, 9] = np.inf
    x[5, 100] = np.nan
    t = ctx.upload(dt, (n, k), w)
    want = O.dequant_matmul_a8(x, dt, w, n)
    got = ctx.dequant_matmul(x, t, a8_block=256)
    exact = np.ones_like(want, bool)
    exact[4:, :] = False  # refused rows: f32 product, tolerance
    exact[:, 3] = False   # refused weight row
    assert np.array_equal(bits(got[exact]), bits(want[exact]))
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(np.isinf(got), np.isinf(want))
    fin = ~exact & np.isfinite(want)
    wd = O.dequantize(dt, w, n * k).reshape(n, k).astype(np.float64)
    scale = np.abs(np.nan_to_num(x.astype(np.float64), posinf=0, neginf=0)) @ np.abs(np.nan_to_num(wd)).T
    assert np.all(np.abs(got[fin] - want[fin]) <= (k + 1) * U * 4 * scale[fin] + 1e-30)
    t.free()


@pytest.mark.parametrize("dt,n,k,inf", [(O.Q4_K, 12288, 4096, False), (O.Q6_K, 4096, 14336, False),
                                         (O.Q6_K, 9000, 2048, False), (O.Q4_K, 150, 256, False),
                                         (O.Q6_K, 100, 4096, False), (O.Q4_K, 3000, 4096, True),
                                         (O.Q4_K, 2000, 5632, False), (O.Q6_K, 1200, 6144, False),
                                         (O.Q4_K, 301, 768, False), (O.Q6_K, 4096, 1792, False),
                                         (O.Q6_K, 4096, 3584, False), (O.Q6_K, 2048, 7168, False),
                                         (O.Q6_K, 1003, 3584, False), (O.Q4_K, 900, 1792, False)])
def test_a8_one_row_slabs(ctx, dt, n, k, inf):
    """One activation row (the slab-streaming kernel): matrices whose per-SM
    slabs span several stages of the record ring, fewer rows than SMs, row
    block counts that do not divide 256 (stages of 242, 240 and 255 blocks,
    an odd number of rows per stage), Q6_K rows that are not 16-byte
    multiples (7, 14 and 28 blocks: the ffn_down shards of tensor
    parallelism, cut in units of 8, 4 and 2 rows; a row count that is not a
    whole unit takes the multi-row kernel), and weight rows with a
    non-finite block scale in different stages.  Exact rows equal the oracle bit for bit; refused rows (and a
    refused activation row) equal the multi-row kernel's f32 product."""
    bb = 144 if dt == O.Q4_K else 210
    rb = k // 256 * bb
    w = bytearray(_weights(dt, n, k, 4242 + n).tobytes())
    refused = sorted(r for r in {5, 70, n // 2 + 1, n - 1} if r < n)
    for r in refused:
        o = r * rb + (k // 256 - 1) * bb  # the row's last block
        if dt == O.Q4_K:
            w[o + 2:o + 4] = bytes([0x00, 0x7C])
        else:
            w[o + 208:o + 210] = bytes([0x00, 0x7E])
    w = np.frombuffer(bytes(w), np.uint8)
    x = O.gen_normal(11, 2 * k).reshape(2, k)
    if inf:
        x[0, 17] = np.inf
    x[1] = x[0]
    bias = O.gen_normal(4, n)
    t = ctx.upload(dt, (n, k), w)
    one = ctx.dequant_matmul(x[:1], t, bias, a8_block=256)
    two = ctx.dequant_matmul(x, t, bias, a8_block=256)
    assert np.array_equal(bits(one[0]), bits(two[0]))
    if not inf:
        want = O.dequant_matmul_a8(x[:1], dt, w, n, bias)
        exact = np.ones(n, bool)
        exact[refused] = False
        assert np.array_equal(bits(one[0][exact]), bits(want[0][exact]))
    t.free()


def test_a8_batch_invariance(ctx):
    """interp/transformer_test.go:297-354: each row's result is the same bits
    alone as in any batch."""
    k, n, rows = 1024, 40, 13
    for dt in (O.Q4_K, O.Q6_K):
        w = _weights(dt, n, k, 5)
        x = O.gen_normal(9, rows * k).reshape(rows, k)
        x[4, 3] = np.inf
        t = ctx.upload(dt, (n, k), w)
        together = ctx.dequant_matmul(x, t, a8_block=256)
        for i in range(rows):
            alone = ctx.dequant_matmul(x[i:i + 1], t, a8_block=256)
            assert np.array_equal(bits(alone[0]), bits(together[i]))
        t.free()


@pytest.mark.parametrize("block", [256, 32])
def test_a8_quantizer_rounds_near_half_integers(ctx, block):
    """TestQuantQ8 (internal/kernels/q8_test.go:116-160): activations on
    half-integer steps of amax/127, nudged by a few ulps, where the rounding
    of 127 x / amax decides the quant; every quant shows in the product bits
    (exact integer block sums), compared with the oracle's float64 rounding."""
    rng = np.random.default_rng(13)
    k, n = 4096, 24
    x = np.empty((4, k), np.float32)
    for r in range(4):
        amax = np.float32(rng.exponential(10.0) + 1e-3)
        h = (rng.integers(0, 255, k) - 127) / 2.0
        v = (h * np.float64(amax) / 127).astype(np.float32)
        for _ in range(2):
            nudge = rng.integers(0, 3, k)
            v = np.where(nudge == 1, np.nextafter(v, np.float32(np.inf)), v)
            v = np.where(nudge == 2, np.nextafter(v, np.float32(-np.inf)), v)
        v = np.clip(v, -amax, amax)
        v[::32] = amax  # every run of 32 (so every block) reaches amax exactly
        x[r] = v
    for dt in (O.Q4_K, O.Q6_K):
        w = _weights(dt, n, k, 91)
        t = ctx.upload(dt, (n, k), w)
        want = O.dequant_matmul_a8(x, dt, w, n, block=block)
        got = ctx.dequant_matmul(x, t, a8_block=block)
        assert np.array_equal(bits(got), bits(want))
        t.free()


def test_a8_block_attribute(ctx):
    import mimgpu
    w = _weights(O.Q4_K, 4, 256, 1)
    t = ctx.upload(O.Q4_K, (4, 256), w)
    x = O.gen_normal(1, 256).reshape(1, 256)
    with pytest.raises(mimgpu.MimGPUError) as e:
        ctx.dequant_matmul(x, t, a8_block=64)
    assert e.value.code == mimgpu.EINVAL
    # block 32 on a dtype without a block-32 kernel (F16) is the exact v1
    # product, as the reference falls back (fast.go:254-258)
    wf = O.gen_normal(2, 4 * 256).astype(np.float16)
    tf = ctx.upload(O.F16, (4, 256), wf.view(np.uint8))
    assert np.array_equal(bits(ctx.dequant_matmul(x, tf, a8_block=32)), bits(ctx.dequant_matmul(x, tf)))
    # the v1 key takes no attributes (fastDequantMatmulA8, fast.go:225-230)
    assert ctx.fast_paths["dequant_matmul_a8.v1"]({"block": 256}, [x, t]) == (None, False)
    out, ok = ctx.fast_paths["dequant_matmul_a8.v1"]({}, [x, t])
    assert ok and np.array_equal(bits(out[0]), bits(ctx.dequant_matmul(x, t, a8_block=32)))
    tf.free()
    t.free()


# ------------------------------------- 8-bit activations in blocks of 32 (v1)

B32_BB = {O.Q4_K: 144, O.Q6_K: 210, O.Q8_0: 34}


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K, O.Q8_0])
@pytest.mark.parametrize("n,k,rows", [(8, 256, 1), (37, 2048, 1), (64, 5632, 3), (300, 4096, 1),
                                      (129, 4096, 9), (24, 14336, 8), (40, 4096, 17), (1000, 4096, 1)])
def test_a8_b32_bit_exact(ctx, dt, n, k, rows):
    """dequant_matmul_a8.v1: bit for bit with the oracle's restatement of the
    AVX2 block-32 kernels (kernels_amd64.s:441, 763, 1007)."""
    w = _weights(dt, n, k, 2000 + n)
    x = O.gen_normal(17 + rows, rows * k).reshape(rows, k)
    bias = O.gen_normal(5, n)
    t = ctx.upload(dt, (n, k), w)
    want = O.dequant_matmul_a8(x, dt, w, n, bias, block=32)
    got = ctx.dequant_matmul(x, t, bias, a8_block=32)
    assert np.array_equal(bits(got), bits(want))
    t.free()


@pytest.mark.parametrize("k", [32, 96, 1056])
def test_a8_b32_q8_0_ragged_k(ctx, k):
    """Q8_0 rows need only K % 32 == 0: lengths that are not a whole number
    of 256-element quantizer blocks."""
    n, rows = 45, 3
    w = _weights(O.Q8_0, n, k, 7 + k)
    x = O.gen_normal(k, rows * k).reshape(rows, k)
    t = ctx.upload(O.Q8_0, (n, k), w)
    want = O.dequant_matmul_a8(x, O.Q8_0, w, n, block=32)
    assert np.array_equal(bits(ctx.dequant_matmul(x, t, a8_block=32)), bits(want))
    t.free()


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K, O.Q8_0])
def test_a8_b32_edge_cases(ctx, dt):
    """Tiny and huge activations, a zero block, the largest finite scales,
    subnormal scales and a weight of -128 (q8_test.go:183-234); refused
    activation rows (Inf, NaN) and a weight row with a non-finite scale take
    the f32 product (fast.go:282-379)."""
    k, n = 2048, 16
    bb = B32_BB[dt]
    rb = k // O.BLOCK[dt][0] * bb
    w = bytearray(_weights(dt, n, k, 78).tobytes())
    for o in range(rb, 2 * rb, bb):  # row 1: largest finite scales, extreme quants
        if dt == O.Q4_K:
            w[o:o + 4] = bytes([0xFF, 0x7B, 0xFF, 0x7B])
            w[o + 4:o + 144] = b"\xff" * 140
        elif dt == O.Q6_K:
            w[o + 208:o + 210] = bytes([0xFF, 0x7B])
            w[o:o + 192] = b"\xff" * 192
            w[o + 192:o + 208] = b"\x80" * 16
        else:
            w[o:o + 2] = bytes([0xFF, 0x7B])
            w[o + 2:o + 34] = b"\x80" * 32  # weights of -128
    sc = {O.Q4_K: 0, O.Q6_K: 208, O.Q8_0: 0}[dt]
    w[2 * rb + sc:2 * rb + sc + 2] = bytes([0x01, 0x00])       # row 2: subnormal d
    w[3 * rb + bb + sc:3 * rb + bb + sc + 2] = bytes([0x00, 0x7C])  # row 3: d = inf in block 1
    w = np.frombuffer(bytes(w), np.uint8)
    x = O.gen_normal(6, 6 * k).reshape(6, k)
    x[1] *= np.float32(1e-30)
    x[2] *= np.float32(1e15)
    x[3, :256] = 0
    x[4, 9] = np.inf
    x[5, 100] = np.nan
    t = ctx.upload(dt, (n, k), w)
    want = O.dequant_matmul_a8(x, dt, w, n, block=32)
    got = ctx.dequant_matmul(x, t, a8_block=32)
    exact = np.ones_like(want, bool)
    exact[4:, :] = False  # refused rows: f32 product, tolerance
    exact[:, 3] = False   # refused weight row
    assert np.array_equal(bits(got[exact]), bits(want[exact]))
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(np.isinf(got), np.isinf(want))
    fin = ~exact & np.isfinite(want)
    wd = O.dequantize(dt, w, n * k).reshape(n, k).astype(np.float64)
    scale = np.abs(np.nan_to_num(x.astype(np.float64), posinf=0, neginf=0)) @ np.abs(np.nan_to_num(wd)).T
    assert np.all(np.abs(got[fin] - want[fin]) <= (k + 1) * U * 4 * scale[fin] + 1e-30)
    t.free()


def test_a8_b32_batch_invariance_and_dev_entry(ctx):
    """Each row's bits alone equal its bits in a batch (transformer_test.go:
    297-354), and the device-buffer entry point gives the host call's bits."""
    import ctypes as C
    import torch
    import mimgpu
    k, n, rows = 1024, 40, 13
    for dt in (O.Q4_K, O.Q6_K, O.Q8_0):
        w = _weights(dt, n, k, 6)
        x = O.gen_normal(10, rows * k).reshape(rows, k)
        x[4, 3] = np.inf
        t = ctx.upload(dt, (n, k), w)
        together = ctx.dequant_matmul(x, t, a8_block=32)
        for i in range(rows):
            alone = ctx.dequant_matmul(x[i:i + 1], t, a8_block=32)
            assert np.array_equal(bits(alone[0]), bits(together[i]))
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty((rows, n), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        ctx._check(mimgpu.lib().mimgpu_dequant_matmul_a8_block_dev(
            ctx.h, stream, 32, C.c_void_p(xd.data_ptr()), rows, k, t.h, None, C.c_void_p(yd.data_ptr())))
        torch.cuda.synchronize()
        assert np.array_equal(bits(yd.cpu().numpy()), bits(together))
        t.free()


# ------------------------------------------------------- f32 activations

@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K, O.Q8_0])
@pytest.mark.parametrize("n,k,rows", [(64, 256, 1), (200, 4096, 1), (33, 11008, 2), (16, 14336, 4)])
def test_v1_within_spec_tolerance(ctx, dt, n, k, rows):
    w = _weights(dt, n, k, 300 + n)
    x = O.gen_normal(11, rows * k).reshape(rows, k)
    bias = O.gen_normal(12, n)
    t = ctx.upload(dt, (n, k), w)
    got = ctx.dequant_matmul(x, t, bias).astype(np.float64)
    wd = O.dequantize(dt, w, n * k).reshape(n, k).astype(np.float64)
    exact = x.astype(np.float64) @ wd.T + bias
    bound = (k + 1) * U * (np.abs(x.astype(np.float64)) @ np.abs(wd).T + np.abs(bias))
    assert np.all(np.abs(got - exact) <= bound)
    rel = np.abs(got - exact).max() / np.abs(exact).max()
    assert rel <= 1e-3
    t.free()


# --------------------------------------------------------- per-token ops

def test_rms_norm_matches_oracle(ctx):
    """fast.go:434-485, bit for bit on every row.  The float64 sum of squares
    is a tree sum here and an in-order sum in the reference; where the
    tree's error bound straddles an f32 boundary of the mean, the kernel
    repeats the in-order sum."""
    x = O.gen_normal(21, 64 * 4096).reshape(64, 4096)
    x[3] *= 1e-20
    scale = O.gen_normal(22, 4096, 1.0, 0.02)
    got = ctx.rms_norm(x, scale, 1e-5)
    want = O.rms_norm(x, scale, 1e-5)
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("n", [256, 4096, 8192])
def test_rms_norm_mean_on_an_f32_midpoint(ctx, n):
    """Rows whose mean of squares sits exactly on, or a float64 ulp beside,
    the midpoint between two f32 values: the tree sum cannot settle the f32
    mean there, so these rows take the in-order sum, and must still give the
    reference's bits."""
    a = np.float32(1 + 2.0 ** -12)  # a*a = 1 + 2^-11 + 2^-24: an f32 midpoint
    rows = [np.full(n, a, np.float32)]
    r = np.full(n, a, np.float32)
    r[::7] = np.float32(1 + 2.0 ** -12 + 2.0 ** -23)  # a few ulps away from the midpoint
    rows.append(r)
    rng = np.random.default_rng(5)
    for _ in range(6):
        r = np.full(n, a, np.float32)
        idx = rng.integers(0, n, 3)
        r[idx] = np.nextafter(r[idx], np.float32(2))
        rows.append(r)
    x = np.stack(rows)
    got = ctx.rms_norm(x, None, 1e-5)
    want = O.rms_norm(x, None, 1e-5)
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("interleaved", [True, False])
def test_rope_matches_oracle(ctx, interleaved):
    """fast.go:507-557: cos/sin in float64 rounded to f32; the rotation is
    the same f32 operations, so results are bit-exact unless a float64
    cos/sin differs in its last bit at an f32 rounding boundary."""
    B, H, T, D = 1, 8, 7, 128
    x = O.gen_normal(31, B * H * T * D).reshape(B, H, T, D)
    pos = np.array([[0, 1, 5, 100, 1000, 2303, 131071]], np.int64)
    got = ctx.rope(x, pos, 500000.0, D, interleaved)
    want = O.rope(x, pos, 500000.0, D, interleaved)
    mism = (bits(got) != bits(want)).mean()
    assert mism < 1e-3
    A = float(pos.max())
    assert np.all(np.abs(got - want) <= (16 + 4 * A) * U * np.abs(x).max())


def test_rope_partial_rotary(ctx):
    x = O.gen_normal(32, 2 * 3 * 4 * 64).reshape(2, 3, 4, 64)
    pos = np.array([[1, 2, 3, 4], [7, 8, 9, 10]], np.int64)
    got = ctx.rope(x, pos, 10000.0, 32, False)
    want = O.rope(x, pos, 10000.0, 32, False)
    assert np.array_equal(got[..., 32:], x[..., 32:])
    assert np.allclose(got, want, rtol=0, atol=1e-5)


def test_swiglu_matches_oracle(ctx):
    a = O.gen_normal(41, 100000) * 4
    b = O.gen_normal(42, 100000)
    a[:4] = [np.inf, -np.inf, np.nan, -100.0]
    got = ctx.swiglu(a, b)
    want = O.swiglu(a, b)
    # siluMulF32AVX2's Cephes exp on the first n&~7 elements, float64 on the
    # tail: bit-exact, NaN positions equal
    assert np.array_equal(np.isnan(got), np.isnan(want))
    ok = ~np.isnan(want)
    assert np.array_equal(bits(got[ok]), bits(want[ok]))
    # a length with a tail of 5
    got = ctx.swiglu(a[:1005], b[:1005])
    want = O.swiglu(a[:1005], b[:1005])
    ok = ~np.isnan(want)
    assert np.array_equal(bits(got[ok]), bits(want[ok]))


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K, O.Q8_0])
def test_embedding_exact(ctx, dt):
    V, E = 50, 512
    table = _weights(dt, V, E, 51)
    t = ctx.upload(dt, (V, E), table)
    ids = np.array([0, 49, 7, -1, 50, 7], np.int32)
    got = ctx.embedding(t, ids)
    want = O.embedding(dt, table, V, E, ids)
    assert np.array_equal(bits(got), bits(want))
    assert not got[3].any() and not got[4].any()
    t.free()


def _same(got, want):
    """Bit-exact outside NaN, NaN at the same places."""
    assert np.array_equal(np.isnan(got), np.isnan(want))
    ok = ~np.isnan(want)
    assert np.array_equal(bits(got[ok]), bits(want[ok]))


@pytest.mark.parametrize("kv", [np.float16, np.float32])
def test_attention_cache_mask(ctx, kv):
    """The llama graph's call: one query block over a cache with the mask
    j <= p (importer/llama.go:364-397), GQA 4."""
    B, Hq, Hkv, D, C = 1, 8, 2, 128, 96
    pos = np.array([5, 6, 7, 40], np.int64)
    Tq = pos.size
    q = O.gen_normal(61, B * Hq * Tq * D).reshape(B, Hq, Tq, D)
    k = O.gen_normal(62, B * Hkv * C * D).reshape(B, Hkv, C, D).astype(kv)
    v = O.gen_normal(63, B * Hkv * C * D).reshape(B, Hkv, C, D).astype(kv)
    mask = (np.arange(C)[None, :] <= pos[:, None]).reshape(1, 1, Tq, C)
    got = ctx.attention(q, k, v, mask)
    want = O.attention(q, k, v, mask)
    # the vector path's arithmetic (attn_amd64.s): bit-exact
    _same(got, want)


def test_attention_holes_causal_and_empty(ctx):
    B, Hq, Hkv, Tq, Tk, D = 2, 4, 4, 3, 20, 64
    q = O.gen_normal(71, B * Hq * Tq * D).reshape(B, Hq, Tq, D)
    k = O.gen_normal(72, B * Hkv * Tk * D).reshape(B, Hkv, Tk, D)
    v = O.gen_normal(73, B * Hkv * Tk * D).reshape(B, Hkv, Tk, D)
    rng = np.random.default_rng(7)
    mask = rng.random((B, 1, Tq, Tk)) < 0.6
    mask[0, 0, 1, :] = False  # a row with every key hidden: NaN
    got = ctx.attention(q, k, v, mask, causal=True)
    want = O.attention(q, k, v, mask, causal=True)
    # holes take the scalar path (fast.go:661-716): bit-exact as well
    _same(got, want)


@pytest.mark.parametrize("n", [1, 5, 7, 8, 13, 64, 301])
def test_attention_lengths_and_infinite_scores(ctx, n):
    """Key counts around the group-of-four and lanes-of-eight boundaries, and
    a row whose score overflows (its largest score is not finite, so the
    reference leaves the vector path)."""
    B, Hq, Hkv, D = 1, 4, 2, 64
    q = O.gen_normal(81 + n, B * Hq * 2 * D).reshape(B, Hq, 2, D)
    k = O.gen_normal(82 + n, B * Hkv * n * D).reshape(B, Hkv, n, D).astype(np.float16)
    v = O.gen_normal(83 + n, B * Hkv * n * D).reshape(B, Hkv, n, D).astype(np.float16)
    q[0, 1, 0, :] = 3e38
    got = ctx.attention(q, k, v, None)
    want = O.attention(q, k, v, None)
    _same(got, want)


def test_fast_paths_registry(ctx):
    """The registry keys of interp/fast.go:42-59 this backend serves."""
    for key in ("dequant_matmul.v1", "dequant_matmul_a8.v2", "rms_norm.v1", "rope.v1", "attention.v2",
                "swiglu.v1", "embedding.v1"):
        assert key in ctx.fast_paths
    out, handled = ctx.fast_paths["rope.v1"]({"yarn_factor": 2.0}, [np.zeros((1, 1, 1, 2), np.float32),
                                                                    np.zeros((1, 1), np.int64)])
    assert handled is False
