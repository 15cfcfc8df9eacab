"""The one-kernel decode step (k_step.cu) against the kernel-per-op path and
the CPU restatement of the reference.  Needs a B200.

Both paths compute every value with the same arithmetic, so one-token logits
must agree bit for bit, and greedy ids must be identical to each other and to
the oracle's (gsoultan/mimir-model cmd/mim-run/main.go:219-257).
"""
import os
import sys

import numpy as np
import pytest

import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
import bench  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    import mimgpu
    c = mimgpu.Context(0)
    yield c
    c.close()


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("shape,layers,vocab", [("8b", 2, 32000), ("70b", 1, 32000)])
def test_step_kernel_bit_identical_to_op_path(ctx, shape, layers, vocab):
    cfg = dict(bench.SHAPES[shape], layers=layers, vocab=vocab)
    P, C = 24, 96
    model, weights = bench.build_model(ctx, cfg, C, P)
    ids = bench.prompt_ids(vocab, P, seed=11)
    sessions = []
    for use in (True, False):
        s = model.session()
        s.set_step_kernel(use)
        assert s.uses_step_kernel == use
        s.run(ids, np.arange(P))
        sessions.append(s)
    step, ops = sessions
    # one-token runs at successive positions: logits bit for bit
    tok = 7
    for i in range(4):
        a = step.run([tok], [P + i])[0]
        b = ops.run([tok], [P + i])[0]
        assert np.array_equal(_bits(a), _bits(b)), f"position {P + i}"
        tok = int(np.argmax(a))
    # greedy generation: identical ids both ways and to the oracle
    ga = step.generate(tok, P + 4, 24).tolist()
    gb = ops.generate(tok, P + 4, 24).tolist()
    assert ga == gb
    host = {name: (dt, ctx.download(t)) for name, (dt, t) in weights.items()}
    ref = O.Llama(dict(cfg, context=C, a8=1, cache_f16=1, interleaved=1), host)
    ref.forward(ids, np.arange(P))
    cur = 7
    for i in range(4):
        cur = O.argmax(ref.forward([cur], [P + i])[0])
    want = []
    for i in range(24):
        cur = O.argmax(ref.forward([cur], [P + 4 + i])[0])
        want.append(cur)
    assert ga == want
    for s in sessions:
        s.free()
    model.free()
    for _, t in weights.values():
        t.free()


def test_step_kernel_is_opt_in_and_models_that_do_not_qualify_refuse_it(ctx, tiny):
    import mimgpu
    cfg = dict(bench.CFG8B, layers=1, vocab=4096)
    model, weights = bench.build_model(ctx, cfg, 64, 8)
    s = model.session()
    assert not s.uses_step_kernel  # the kernel-per-op path measured faster
    s.set_step_kernel(True)
    assert s.uses_step_kernel
    s.free()
    model.free()
    for _, t in weights.values():
        t.free()
    # the tiny fixture (head size 16) runs op by op
    e, w = tiny
    m = mimgpu.Model(ctx, dict(e["config"], interleaved=1, a8=1, cache_f16=1, max_tokens=8), w)
    s = m.session()
    assert not s.uses_step_kernel
    with pytest.raises(mimgpu.MimGPUError) as ei:
        s.set_step_kernel(True)
    assert ei.value.code == mimgpu.ENOTHANDLED
    s.free()
    m.free()
