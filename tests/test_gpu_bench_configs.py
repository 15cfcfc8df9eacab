"""Parity at the configurations the benchmark times,
against the CPU restatement of the reference (oracle/).  Needs a B200.

Bars (north star of this port; gsoultan/mimir-model cmd/mim-run/main.go:219-257
is the reference's greedy loop, main_test.go:179-267 its identity bar):
  * greedy ids identical to the reference's over 64 steps, on the full 8B
    config-3 model the bench decodes (32 layers, vocab 128256, the bench's
    own 128-token seeded prompt and seeded weights);
  * the prompt GEMM (tcgen05 path) bit-exact with dotQ8KRef at T = 512 on
    the config-4 shapes;
  * two layers at the 70B dimensions (config 5: E 8192, F 28672, 64/8 heads,
    vocab 128256): 32 greedy ids identical.
The prompt logits are bit-identical to the oracle's: every step of the path
(the 8-bit products, RMSNorm, RoPE, attention, SwiGLU) reproduces the
reference's arithmetic bit for bit, so the tolerance here is zero.
"""
import os
import sys

import numpy as np
import pytest

import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
import bench  # noqa: E402  (the benchmark's own model layout and seeds)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    import mimgpu
    c = mimgpu.Context(0)
    yield c
    c.close()


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _greedy_vs_oracle(sess, ref, tok, pos, steps):
    """Greedy ids of the GPU session and of the oracle from (tok, pos); the
    oracle's top-2 margin of every step."""
    gen = sess.generate(tok, pos, steps).tolist()
    cur, want, margins = tok, [], []
    for i in range(steps):
        lg = ref.forward([cur], [pos + i])[0]
        top = np.sort(lg)[-2:]
        margins.append(round(float(top[1] - top[0]), 5))
        cur = O.argmax(lg)
        want.append(cur)
    return gen, want, margins


def _host_weights(ctx, weights):
    return {name: (dt, ctx.download(t)) for name, (dt, t) in weights.items()}


def test_config3_full_8b_64_greedy_ids(ctx):
    """Config 3 exactly as bench.py builds it: the 128-token prompt, then 64
    greedy steps, ids identical to the reference's."""
    cfg = bench.CFG8B
    prompt = bench.PROMPT
    C = prompt + 64 + 8
    model, weights = bench.build_model(ctx, cfg, C, prompt)
    sess = model.session()
    ids = bench.prompt_ids(cfg["vocab"], prompt)
    got = sess.run(ids, np.arange(prompt))[0]
    ref = O.Llama(dict(cfg, context=C, a8=1, cache_f16=1, interleaved=1), _host_weights(ctx, weights))
    want = ref.forward(ids, np.arange(prompt))[0]
    diff = int(np.count_nonzero(_bits(got) != _bits(want)))
    assert diff == 0, f"{diff} prompt logits differ from the oracle"
    tok = O.argmax(want)
    assert int(np.argmax(got)) == tok
    gen, want_ids, margins = _greedy_vs_oracle(sess, ref, tok, prompt, 64)
    print(f"config 3: smallest top-2 margin of the 64 steps {min(margins)}")
    assert gen == want_ids, (gen, want_ids, margins)
    sess.free()
    model.free()
    for _, t in weights.values():
        t.free()


@pytest.mark.parametrize("N,K,dt", [(14336, 4096, O.Q4_K), (4096, 14336, O.Q6_K)])
def test_config4_prompt_gemm_t512_bit_exact(ctx, N, K, dt):
    """The prompt pass's products at T = 512 (config 4), through the
    tensor-core GEMM, bit for bit with dotQ8KRef."""
    w = O.gen_weight(dt, 77 + dt, N, K)
    x = O.gen_normal(78, 512 * K).reshape(512, K)
    t = ctx.upload(dt, (N, K), w)
    got = ctx.dequant_matmul(x, t, a8_block=256)
    want = O.dequant_matmul_a8(x, dt, w, N)
    assert np.array_equal(_bits(got), _bits(want))
    t.free()


def test_config4_prompt_logits_t512(ctx):
    """A 512-token prompt pass (two 8B-shape layers, vocab 32000): every row's
    logits against the oracle's, and the last row's argmax identical."""
    cfg = dict(bench.CFG8B, layers=2, vocab=32000)
    T = 512
    model, weights = bench.build_model(ctx, cfg, T + 8, T)
    sess = model.session()
    ids = bench.prompt_ids(cfg["vocab"], T, seed=20261202)
    got = sess.run(ids, np.arange(T), all_rows=True)
    ref = O.Llama(dict(cfg, context=T + 8, a8=1, cache_f16=1, interleaved=1), _host_weights(ctx, weights))
    want = ref.forward(ids, np.arange(T), all_rows=True)
    diff = int(np.count_nonzero(_bits(got) != _bits(want)))
    assert diff == 0, f"{diff} of {got.size} prompt logits differ from the oracle"
    assert [int(v) for v in np.argmax(got, axis=1)] == [O.argmax(r) for r in want]
    sess.free()
    model.free()
    for _, t in weights.values():
        t.free()


def test_config5_70b_dims_two_layers_32_greedy_ids(ctx):
    """Two layers at the 70B dimensions (E 8192, F 28672, 64 query and 8 kv
    heads, vocab 128256): 16-token prompt, then 32 greedy ids identical to
    the reference's."""
    cfg = dict(bench.CFG70B, layers=2)
    P, C = 16, 64
    model, weights = bench.build_model(ctx, cfg, C, P)
    sess = model.session()
    ids = bench.prompt_ids(cfg["vocab"], P, seed=7)
    got = sess.run(ids, np.arange(P))[0]
    ref = O.Llama(dict(cfg, context=C, a8=1, cache_f16=1, interleaved=1), _host_weights(ctx, weights))
    want = ref.forward(ids, np.arange(P))[0]
    assert np.abs(got - want).max() <= 1e-3 * np.abs(want).max()
    tok = O.argmax(want)
    gen, want_ids, margins = _greedy_vs_oracle(sess, ref, tok, P, 32)
    assert gen == want_ids, (gen, want_ids, margins)
    sess.free()
    model.free()
    for _, t in weights.values():
        t.free()
