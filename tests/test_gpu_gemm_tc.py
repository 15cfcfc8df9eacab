"""dequant_matmul_a8.v2 with many activation rows, which libmimgpu runs on the
tensor cores (tcgen05.mma kind::i8, accumulators in TMEM) from 16 rows up.

Bars (reference file:line in gsoultan/mimir-model):
  bit-exact with dotQ8KRef (internal/kernels/q8k_test.go:35-117), like the
  prompt tile kernels, whose per-block float operations are those of the
  one-row kernel (internal/kernels/amx.go:24-51, vnni.go:22-32);
  batch-invariant across the GEMV / GEMM switch (interp/transformer_test.go:297-354);
  refused rows (fast.go:282-379) take the same f32 product as in the GEMV.
"""
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


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
@pytest.mark.parametrize("n,k,rows", [(128, 256, 16), (130, 2048, 32), (257, 4096, 33), (64, 5632, 64),
                                      (300, 1024, 100), (40, 14336, 17)])
def test_gemm_bit_exact(ctx, dt, n, k, rows):
    w = O.gen_weight(dt, 2000 + n, n, k)
    x = O.gen_normal(11 + rows, rows * k).reshape(rows, k)
    bias = O.gen_normal(4, n)
    t = ctx.upload(dt, (n, k), w)
    want = O.dequant_matmul_a8(x, dt, w, n, bias)
    got = ctx.dequant_matmul(x, t, bias, a8_block=256)
    assert np.array_equal(bits(got), bits(want))
    t.free()


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q6_K])
def test_gemm_edge_cases_and_refusals(ctx, dt):
    """The q8k_test.go:122-187 cases in a 24-row launch: tiny and huge
    activations, a zero block, the largest finite scales, subnormal scales,
    refused activation rows (Inf, NaN) and a weight row with a non-finite
    scale; every pair equals its one-row GEMV result bit for bit."""
    k, n, rows = 2048, 140, 24
    bb = 144 if dt == O.Q4_K else 210
    w = bytearray(O.gen_weight(dt, 78, n, k).tobytes())
    rb = k // 256 * bb
    for o in range(rb, 2 * rb, bb):  # row 1: largest finite scales, all-ones quants
        if dt == O.Q4_K:
            w[o:o + 4] = bytes([0xFF, 0x7B, 0xFF, 0x7B])
            w[o + 4:o + 144] = b"\xff" * 140
        else:
            w[o + 208:o + 210] = bytes([0xFF, 0x7B])
            w[o:o + 192] = b"\xff" * 192
            w[o + 192:o + 208] = b"\x80" * 16
    if dt == O.Q4_K:  # row 2: subnormal scales; row 131: dmin = inf (second tile)
        w[2 * rb:2 * rb + 4] = bytes([0x01, 0x00, 0xFF, 0x03])
        w[131 * rb + 2:131 * rb + 4] = bytes([0x00, 0x7C])
    else:
        w[2 * rb + 208:2 * rb + 210] = bytes([0x01, 0x00])
        w[131 * rb + 208:131 * rb + 210] = bytes([0x00, 0x7E])
    w = np.frombuffer(bytes(w), np.uint8)
    x = O.gen_normal(6, rows * k).reshape(rows, k)
    x[1] *= np.float32(1e-30)
    x[2] *= np.float32(1e15)
    x[3, :256] = 0
    x[4, 9] = np.inf
    x[21, 100] = np.nan
    t = ctx.upload(dt, (n, k), w)
    want = O.dequant_matmul_a8(x, dt, w, n)
    got = ctx.dequant_matmul(x, t, a8_block=256)
    exact = np.ones_like(want, bool)
    exact[[4, 21], :] = False  # refused activation rows: f32 product, tolerance
    exact[:, 131] = False      # refused weight row
    assert np.array_equal(bits(got[exact]), bits(want[exact]))
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(np.isinf(got), np.isinf(want))
    fin = ~exact & np.isfinite(want)
    wd = O.dequantize(dt, w, n * k).reshape(n, k).astype(np.float64)
    scale = np.abs(np.nan_to_num(x.astype(np.float64), posinf=0, neginf=0)) @ np.abs(np.nan_to_num(wd)).T
    assert np.all(np.abs(got[fin] - want[fin]) <= (k + 1) * U * 4 * scale[fin] + 1e-30)
    # the same bits as the one-row GEMV, refused pairs included
    for i in (0, 2, 4, 21, 23):
        alone = ctx.dequant_matmul(x[i:i + 1], t, a8_block=256)
        assert np.array_equal(bits(alone[0]), bits(got[i]))
    t.free()


def test_gemm_batch_invariance(ctx):
    """interp/transformer_test.go:297-354 across the GEMV / GEMM switch: a
    row's bits do not depend on how many rows share the launch."""
    k, n = 1536, 200
    for dt in (O.Q4_K, O.Q6_K):
        w = O.gen_weight(dt, 9, n, k)
        x = O.gen_normal(10, 48 * k).reshape(48, k)
        x[7, 3] = -np.inf
        t = ctx.upload(dt, (n, k), w)
        full = ctx.dequant_matmul(x, t, a8_block=256)
        for lo, hi in ((0, 15), (0, 16), (5, 37), (40, 48), (7, 8)):
            part = ctx.dequant_matmul(x[lo:hi], t, a8_block=256)
            assert np.array_equal(bits(part), bits(full[lo:hi]))
        t.free()


def test_prompt_rows_equal_single_token_steps(ctx):
    """Model-level batch invariance (interp/transformer_test.go:297-354): an
    80-token prompt in one pass -- every projection on the tensor-core GEMM,
    two activation-row tiles -- gives the same logits, bit for bit, as the
    same tokens fed one at a time through the GEMV."""
    import mimgpu
    from test_gpu_model import _synthetic
    cfg, w = _synthetic(2, 4096, 32, 8, 14336, 4096)
    T, C = 80, 128
    prompt = np.random.default_rng(5).integers(0, cfg["vocab"], T).astype(np.int32)
    m = mimgpu.Model(ctx, dict(cfg, context=C, a8=1, cache_f16=1, interleaved=1, max_tokens=T), w)
    a = m.session()
    together = a.run(prompt, np.arange(T), all_rows=True)
    b = m.session()
    for i in range(T):
        one = b.run(prompt[i:i + 1], np.arange(i, i + 1))[0]
        assert np.array_equal(bits(one), bits(together[i])), i
    a.free()
    b.free()
    m.free()


@pytest.mark.parametrize("H,Hkv,T", [(64, 8, 37), (32, 8, 9), (16, 16, 21)])
def test_prompt_attention_group_shapes(ctx, H, Hkv, T):
    """The many-row prompt attention for other head groupings (G = 8 as in the
    70B shape, G = 4, G = 1) and prompt lengths that leave a partial tile:
    the prompt's logits equal the one-token steps' bit for bit."""
    import mimgpu
    from test_gpu_model import _synthetic
    E = H * 128
    cfg, w = _synthetic(2, E, H, Hkv, 512, 1024)
    C = 64
    prompt = np.random.default_rng(H + T).integers(0, cfg["vocab"], T).astype(np.int32)
    m = mimgpu.Model(ctx, dict(cfg, context=C, a8=1, cache_f16=1, interleaved=1, max_tokens=T), w)
    a = m.session()
    together = a.run(prompt, np.arange(T), all_rows=True)
    b = m.session()
    for i in range(T):
        one = b.run(prompt[i:i + 1], np.arange(i, i + 1))[0]
        assert np.array_equal(bits(one), bits(together[i])), i
    a.free()
    b.free()
    m.free()
