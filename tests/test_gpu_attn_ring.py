"""The decode attention at contexts of many key chunks.

attn_decode_kernel streams the earlier tokens' keys and values through a
ring of chunk buffers whose chunk size and depth are chosen at launch: a
one-token grid takes 256-key chunks and as many buffers as fit beside the
scores (three at a 1,100-token cache, two at 8,192); a batched grid of more
blocks than SMs, or a cache whose scores leave no room for two 256-key
buffers (14,000 tokens), takes two 128-key buffers, so that several blocks
share an SM, and blocks of four query heads when the group size allows and
there are still as many blocks as SMs (40 sequences here; 20 keep blocks
of two).  These cases wrap the ring many times, cross chunk boundaries
(a context of 128·k + 1 keys leaves the last value chunk with only the
token's own row) and are checked bit for bit: one-token steps
against the CPU restatement of the reference (attendRow with the amd64
kernels, interp/fast.go:728-751), batched steps against single-sequence
sessions (the batch invariance of interp/transformer_test.go:297-354).
"""
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


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("C", [1100, 8192, 14000])
def test_long_context_steps_bit_exact(ctx, C):
    """A 700-token prompt, then 72 one-token steps (contexts 701-772: 3 to 4
    chunks of 256 keys or 6 to 7 of 128, the 769-key step with an empty last
    value chunk), every step's logits bit for bit with the oracle's, and the
    same greedy ids through mimgpu_session_generate."""
    import mimgpu
    from test_gpu_model import _synthetic
    cfg, w = _synthetic(2, 512, 4, 2, 1024, 700, seed=11)
    P, S = 700, 72
    m = mimgpu.Model(ctx, dict(cfg, context=C, a8=1, cache_f16=1, interleaved=1, max_tokens=P), w)
    ref = O.Llama(dict(cfg, context=C, a8=1, cache_f16=1, interleaved=1), w)
    rng = np.random.default_rng(C)
    prompt = rng.integers(0, cfg["vocab"], P).astype(np.int32)
    s = m.session()
    got = s.run(prompt, np.arange(P))[0]
    want = ref.forward(prompt, np.arange(P))[0]
    assert np.array_equal(bits(got), bits(want))
    tok = O.argmax(want)
    first, want_ids = tok, []
    for i in range(S):
        g = s.run([tok], [P + i])[0]
        wv = ref.forward([tok], [P + i])[0]
        assert np.array_equal(bits(g), bits(wv)), f"step at {P + i + 1} keys"
        tok = O.argmax(wv)
        want_ids.append(tok)
    s.free()
    s = m.session()
    s.run(prompt, np.arange(P))
    assert s.generate(first, P, S).tolist() == want_ids
    s.free()
    m.free()


@pytest.mark.parametrize("B", [20, 40])
def test_batched_long_contexts_match_single_sequences(ctx, B):
    """B sequences of 16 query heads in groups of four (more blocks of two
    heads than SMs: 128-key chunks; at 40 sequences blocks of four heads),
    prompts of 128-600 tokens (including the
    128·k + 1 and 128·k edges), 6 greedy steps: every sequence's ids and
    the logits of one more batched row equal a single-sequence session's."""
    import mimgpu
    from test_gpu_model import _synthetic
    cfg, w = _synthetic(2, 2048, 16, 4, 1024, 700, seed=12)
    steps = 6
    m = mimgpu.Model(ctx, dict(cfg, context=640, a8=1, cache_f16=1, interleaved=1, max_tokens=600), w)
    rng = np.random.default_rng(5)
    lens = [128, 129, 256, 257, 600] + [int(v) for v in rng.integers(130, 600, B - 5)]
    prompts = [rng.integers(0, cfg["vocab"], n).astype(np.int32) for n in lens]
    want_ids, first = [], []
    for p in prompts:
        s = m.session()
        lg = s.run(p, np.arange(p.size))[0]
        first.append(int(np.argmax(lg)))
        want_ids.append(s.generate(first[-1], p.size, steps))
        s.free()
    bs = m.session(slots=B)
    for b, p in enumerate(prompts):
        bs.run_slots(p, np.full(p.size, b), np.arange(p.size))
    ids = bs.generate_slots(first, lens, steps)
    for b in range(B):
        assert ids[:, b].tolist() == want_ids[b].tolist(), b
    toks = ids[-1]
    pos = np.array(lens) + steps
    got = bs.run_slots(toks, np.arange(B), pos)
    for b in (0, 3, 4):
        s = m.session()
        s.run(prompts[b], np.arange(prompts[b].size))
        s.generate(first[b], lens[b], steps)
        one = s.run(toks[b:b + 1], pos[b:b + 1])[0]
        assert np.array_equal(bits(one), bits(got[b])), b
        s.free()
    bs.free()
    m.free()
