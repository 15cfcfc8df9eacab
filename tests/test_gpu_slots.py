"""Batched decoding: a session of several sequences (mimgpu_session_new_slots),
each with its own key-value cache.  Every sequence's logits and greedy ids
are the bits a single-sequence session gives for it -- the batch invariance
of interp/transformer_test.go:297-354 carried to whole decode steps (rows of
the batched step go through the GEMV below 16 rows and the tensor-core GEMM
from 16 rows -- with K split over several CTAs when a matrix has few row
tiles -- the same bits either way)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    import mimgpu
    c = mimgpu.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="module")
def model(ctx):
    import mimgpu
    from test_gpu_model import _synthetic
    cfg, w = _synthetic(2, 4096, 32, 8, 14336, 4096)
    m = mimgpu.Model(ctx, dict(cfg, context=96, a8=1, cache_f16=1, interleaved=1, max_tokens=40), w)
    yield m
    m.free()


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("B", [4, 20, 32])
def test_slots_match_single_sequences(model, B):
    rng = np.random.default_rng(B)
    lens = [int(rng.integers(3, 36)) for _ in range(B)]
    prompts = [rng.integers(0, model.vocab, n).astype(np.int32) for n in lens]
    steps = 6
    # one sequence per session
    want_last, want_ids = [], []
    for p in prompts:
        s = model.session()
        lg = s.run(p, np.arange(p.size))[0]
        want_last.append(lg)
        want_ids.append(s.generate(int(np.argmax(lg)), p.size, steps))
        s.free()
    # all sequences in one session
    bs = model.session(slots=B)
    first = []
    for b, p in enumerate(prompts):
        lg = bs.run_slots(p, np.full(p.size, b), np.arange(p.size))
        assert np.array_equal(bits(lg[-1]), bits(want_last[b])), b
        first.append(int(np.argmax(lg[-1])))
    ids = bs.generate_slots(first, lens, steps)
    for b in range(B):
        assert ids[:, b].tolist() == want_ids[b].tolist(), b
    # one decode row per sequence through run_slots: the logits of each row
    # equal a single-sequence session's for the same token and position
    toks = ids[-1]
    pos = np.array(lens) + steps
    got = bs.run_slots(toks, np.arange(B), pos)
    for b, p in enumerate(prompts[:3]):
        s = model.session()
        s.run(p, np.arange(p.size))
        s.generate(first[b], p.size, steps)
        one = s.run(toks[b:b + 1], pos[b:b + 1])[0]
        assert np.array_equal(bits(one), bits(got[b])), b
        s.free()
    bs.free()


def test_slots_reject_bad_arguments(model):
    import mimgpu
    with pytest.raises(mimgpu.MimGPUError):
        model.session(slots=0)
    with pytest.raises(mimgpu.MimGPUError):
        model.session(slots=41)  # more than max_tokens
    s = model.session(slots=2)
    with pytest.raises(mimgpu.MimGPUError):
        s.run_slots([1], [2], [0])  # no sequence 2
    with pytest.raises(mimgpu.MimGPUError):
        s.generate_slots([1, 2, 3], [0, 0, 0], 2)  # three sequences in a session of two
    s.free()
