"""Failure detection without a GPU fault (gsoultan/mimir-model turns panics and
errors of a run into run errors, interp/interp.go:416-436; here every wait is
bounded and reports a status instead of hanging).  Needs a GPU.

* A device wait on a flag that nothing sets runs out after the context's
  limit (mimgpu_set_timeout_ms), the next call that waits for the device
  returns MIMGPU_ETIMEOUT, and the context keeps working afterwards.
* A tensor-parallel group whose second rank never joins: mimgpu_tp_new
  returns MIMGPU_ETIMEOUT after the context's timeout instead of hanging the
  host (non-blocking NCCL initialisation, then ncclCommAbort).
"""
import ctypes as C
import multiprocessing as mp
import os
import time

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _flag(ctx, value: int):
    import mimgpu
    return ctx.upload(mimgpu.F32, (1,), np.array([value], np.uint32).view(np.float32))


def _product_ok(ctx):
    """A small a8 product, bit-exact with the oracle: the context still works."""
    w = O.gen_weight(O.Q4_K, 5, 64, 1024)
    x = O.gen_normal(6, 1024).reshape(1, 1024)
    t = ctx.upload(O.Q4_K, (64, 1024), w)
    got = ctx.dequant_matmul(x, t, a8_block=256)
    t.free()
    return np.array_equal(got.view(np.uint32), O.dequant_matmul_a8(x, O.Q4_K, w, 64).view(np.uint32))


def test_device_wait_runs_out_and_the_context_survives():
    import mimgpu
    ctx = mimgpu.Context(0)
    try:
        ctx.set_timeout_ms(200)
        flag = _flag(ctx, 0)
        lib = mimgpu.lib()
        t0 = time.perf_counter()
        ctx._check(lib.mimgpu_stream_wait_value(ctx.h, None, C.c_void_p(flag.device_ptr), 1))
        # a longer host timeout from here on (the new limit is queued behind the wait,
        # which keeps its 200 ms)
        ctx.set_timeout_ms(5000)
        with pytest.raises(mimgpu.MimGPUError) as ei:
            _product_ok(ctx)  # queued behind the wait; the call that syncs reports it
        waited = time.perf_counter() - t0
        assert ei.value.code == mimgpu.ETIMEOUT
        assert 0.2 <= waited < 5.0, waited
        # the status is cleared and the context works
        assert _product_ok(ctx)
        # a flag that is set lets the work through
        flag.free()
        flag = _flag(ctx, 1)
        ctx._check(lib.mimgpu_stream_wait_value(ctx.h, None, C.c_void_p(flag.device_ptr), 1))
        assert _product_ok(ctx)
        flag.free()
    finally:
        ctx.close()


def _lonely_rank(q):
    """Rank 0 of a 2-rank group whose rank 1 never starts."""
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "mimir-model_b200"))
    import mimgpu
    ctx = mimgpu.Context(0)
    ctx.set_timeout_ms(3000)
    t0 = time.perf_counter()
    try:
        mimgpu.TensorParallel(ctx, mimgpu.tp_unique_id(), 2, 0)
        q.put(("joined", time.perf_counter() - t0))
    except mimgpu.MimGPUError as e:
        q.put((e.code, time.perf_counter() - t0))
    ctx.close()


def test_group_with_a_missing_rank_times_out():
    import mimgpu
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_rank, args=(q,))
    p.start()
    try:
        code, took = q.get(timeout=120)
    finally:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert code == mimgpu.ETIMEOUT, code
    assert 3.0 <= took < 60.0, took
