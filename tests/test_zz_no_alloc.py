"""mimgpu_dequant_matmul_a8_static (the dequant_matmul_a8.v2 product with its
activation scratch in a static device buffer, allocating no device memory)
against the existing entry point, through the C ABI.  Needs a B200.

Tolerance: zero.  Both entry points compute the same exact integer block
sums and the same block-ordered fused multiply-adds of dotQ8KRef
(internal/kernels/q8k_test.go:35-117 of gsoultan/mimir-model), so the
results must agree bit for bit.

The file name sorts last so that the module also runs after every other GPU
test in the same process (the static buffer then holds earlier calls' bytes).
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    import mimgpu
    c = mimgpu.Context(0)
    yield c
    c.close()


def _static(ctx, x_t, rows, k, w, bias_t, y_t):
    import mimgpu
    return mimgpu.lib().mimgpu_dequant_matmul_a8_static(
        ctx.h, None, C.c_void_p(x_t.device_ptr), rows, k, w.h,
        C.c_void_p(bias_t.device_ptr) if bias_t is not None else None, C.c_void_p(y_t.device_ptr))


def _run_static(ctx, x, w, bias=None):
    import mimgpu
    rows, k = x.shape
    n = w.shape[0]
    x_t = ctx.upload(mimgpu.F32, (rows, k), x)
    b_t = ctx.upload(mimgpu.F32, (n,), bias) if bias is not None else None
    y_t = ctx.upload(mimgpu.F32, (rows, n), np.zeros((rows, n), np.float32))
    ctx._check(_static(ctx, x_t, rows, k, w, b_t, y_t))
    y = ctx.download(y_t).view(np.float32).reshape(rows, n)
    for t in (x_t, b_t, y_t):
        if t is not None:
            t.free()
    return y


# 16 rows and more go through the tensor-core GEMM, whose activation tensor
# map then points into the static buffer
@pytest.mark.parametrize("dt,rows,n,k", [(O.Q4_K, 1, 4096, 4096), (O.Q6_K, 3, 1000, 2048), (O.Q4_K, 8, 333, 14336),
                                         (O.Q4_K, 16, 512, 14336), (O.Q6_K, 24, 384, 4096)])
def test_static_matches_a8_entry_two_calls(ctx, dt, rows, n, k):
    w_raw = O.gen_weight(dt, 900 + rows, n, k, 0.02)
    w = ctx.upload(dt, (n, k), w_raw)
    bias = O.gen_normal(950 + rows, n)
    xs = [O.gen_normal(970 + 10 * rows + call, rows * k).reshape(rows, k) for call in range(2)]
    # two calls in a row (different activations; the second with a bias),
    # then the existing entry point on the same inputs
    gots = [_run_static(ctx, xs[call], w, bias if call else None) for call in range(2)]
    for call in range(2):
        want = ctx.dequant_matmul(xs[call], w, bias if call else None, a8_block=256)
        assert np.array_equal(gots[call].view(np.uint32), want.view(np.uint32)), f"call {call}"
        # and the CPU restatement of the reference's kernels (dotQ8KRef)
        ref = O.dequant_matmul_a8(xs[call], dt, w_raw, n, bias if call else None)
        assert np.array_equal(gots[call].view(np.uint32), ref.view(np.uint32)), f"call {call} vs oracle"
    w.free()


def test_static_rejects_oversize_and_other_dtypes(ctx):
    import mimgpu
    k = 16384
    w = ctx.upload(O.Q4_K, (16, k), O.gen_weight(O.Q4_K, 991, 16, k, 0.02))
    x_t = ctx.upload(mimgpu.F32, (64, k), np.zeros((64, k), np.float32))
    y_t = ctx.upload(mimgpu.F32, (64, 16), np.zeros((64, 16), np.float32))
    rc = _static(ctx, x_t, 64, k, w, None, y_t)
    assert rc == mimgpu.EINVAL
    assert "static buffer" in mimgpu.lib().mimgpu_last_error(ctx.h).decode()
    w8 = ctx.upload(O.Q8_0, (16, k), O.gen_weight(O.Q8_0, 992, 16, k, 0.02))
    assert _static(ctx, x_t, 1, k, w8, None, y_t) == mimgpu.ENOTHANDLED
    # the context still works after the refusals
    x = O.gen_normal(993, k).reshape(1, k)
    got = _run_static(ctx, x, w)
    want = ctx.dequant_matmul(x, w, None, a8_block=256)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    for t in (w, x_t, y_t, w8):
        t.free()
