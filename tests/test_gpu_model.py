"""The device-resident llama step (mimgpu_session_*) against the reference's
tiny-Llama and tiny-Qwen 2 fixtures and against the CPU oracle.  Needs a B200.

Bars (gsoultan/mimir-model):
  cmd/mim-run/main_test.go:179-216  v1 graph, f32 cache: prompt and step
      logits within 2e-5 of the largest logit of the float64 oracle, and the
      same 8 greedy ids;
  cmd/mim-run/main_test.go:218-267  a8 graph, f16 cache: logits within 1.1x
      llama.cpp's own distance from the float64 oracle;
  token identity: greedy ids identical to the CPU restatement of the
      reference (the a8 products are bit-exact; attention is the only
      tolerance-level step) over 64 steps at 8B layer shapes.
"""
import os
import sys

import numpy as np
import pytest

import oracle as O
from conftest import f32b64, load_tiny

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    import mimgpu
    c = mimgpu.Context(0)
    yield c
    c.close()


def _model(ctx, e, w, **over):
    import mimgpu
    # llama rotates adjacent pairs, qwen2 the halves of each head
    cfg = dict(e["config"], interleaved=int(e["config"]["arch"] == "llama"), max_tokens=len(e["prompt_ids"]))
    cfg.update(over)
    return mimgpu.Model(ctx, cfg, w)


@pytest.mark.parametrize("name", ["llama", "qwen2"])
def test_tiny_llama_v1_matches_float64_oracle(ctx, name):
    e, w = load_tiny(name)
    V = e["config"]["vocab"]
    m = _model(ctx, e, w, a8=0, cache_f16=0)
    s = m.session()
    ids = e["prompt_ids"]
    all_ = s.run(ids, np.arange(len(ids)), all_rows=True)
    want = f32b64(e["prompt_logits"]).reshape(len(ids), V)
    assert np.abs(all_ - want).max() <= 2e-5 * np.abs(want).max()
    logits, pos = all_[-1], len(ids)
    for i, nxt in enumerate(e["greedy"]):
        w_ = f32b64(e["greedy_logits"][i])
        assert np.abs(logits - w_).max() <= 2e-5 * np.abs(w_).max()
        assert int(np.argmax(logits)) == nxt
        logits = s.run([nxt], [pos])[0]
        pos += 1
    s.free()
    m.free()


@pytest.mark.parametrize("name", ["llama", "qwen2"])
@pytest.mark.parametrize("cache_f16,bound", [(0, 1.0), (1, 1.1)])
def test_tiny_llama_a8_within_llama_cpp(ctx, name, cache_f16, bound):
    e, w = load_tiny(name)
    V = e["config"]["vocab"]
    m = _model(ctx, e, w, a8=1, cache_f16=cache_f16)
    s = m.session()
    ids = e["prompt_ids"]
    all_ = s.run(ids, np.arange(len(ids)), all_rows=True)
    worst = np.abs(all_ - f32b64(e["prompt_logits"]).reshape(len(ids), V)).max()
    logits, pos = all_[-1], len(ids)
    for i, nxt in enumerate(e["greedy"]):
        worst = max(worst, np.abs(logits - f32b64(e["greedy_logits"][i])).max())
        logits = s.run([nxt], [pos])[0]
        pos += 1
    assert worst <= e["llama_cpp_max_diff"] * bound
    s.free()
    m.free()


@pytest.mark.parametrize("name", ["llama", "qwen2"])
def test_tiny_llama_a8_matches_cpu_restatement(ctx, name):
    """Prompt logits and 48 greedy ids against the oracle's a8 + f16 graph
    (the Qwen 2 with its query/key/value biases and rotation of halves)."""
    e, w = load_tiny(name)
    m = _model(ctx, e, w, a8=1, cache_f16=1)
    s = m.session()
    ref = O.Llama(dict(e["config"], a8=1, cache_f16=1, interleaved=int(name == "llama")), w)
    ids = e["prompt_ids"]
    got = s.run(ids, np.arange(len(ids)), all_rows=True)
    want = ref.forward(ids, np.arange(len(ids)), all_rows=True)
    assert np.abs(got - want).max() <= 1e-3 * np.abs(want).max()
    tok, pos = int(np.argmax(got[-1])), len(ids)
    gen = s.generate(tok, pos, 48)
    cur, want_ids = tok, []
    for i in range(48):
        lg = ref.forward([cur], [pos + i])[0]
        cur = O.argmax(lg)
        want_ids.append(cur)
    assert gen.tolist() == want_ids
    s.free()
    m.free()


def _synthetic(layers, E, H, Hkv, F, V, seed=1):
    """Random-init llama weights, Q4_K_M layout (Q6_K for attn_v, ffn_down,
    output), f32 norms 1 + N(0, 0.02)."""
    D = E // H
    KV = Hkv * D
    w = {}
    sd = seed * 1000
    def q(name, dt, n, k):
        nonlocal sd
        sd += 1
        w[name] = (dt, O.gen_weight(dt, sd, n, k).ravel())
    def norm(name, n):
        nonlocal sd
        sd += 1
        w[name] = (O.F32, O.gen_normal(sd, n, 1.0, 0.02))
    q("token_embd.weight", O.Q4_K, V, E)
    for l in range(layers):
        p = f"blk.{l}."
        norm(p + "attn_norm.weight", E)
        q(p + "attn_q.weight", O.Q4_K, E, E)
        q(p + "attn_k.weight", O.Q4_K, KV, E)
        q(p + "attn_v.weight", O.Q6_K, KV, E)
        q(p + "attn_output.weight", O.Q4_K, E, E)
        norm(p + "ffn_norm.weight", E)
        q(p + "ffn_gate.weight", O.Q4_K, F, E)
        q(p + "ffn_up.weight", O.Q4_K, F, E)
        q(p + "ffn_down.weight", O.Q6_K, E, F)
    norm("output_norm.weight", E)
    q("output.weight", O.Q6_K, V, E)
    cfg = dict(layers=layers, embed=E, ffn=F, heads=H, kv_heads=Hkv, head_dim=D, rope_dims=D, vocab=V,
               rope_theta=500000.0, norm_eps=1e-5)
    return cfg, w


def test_8b_layer_shapes_token_identity(ctx):
    """Two layers of the 8B shape (E 4096, 32/8 heads, F 14336) with a 32000
    vocabulary: prompt of 16 ids then 64 greedy steps, token-identical to
    the CPU restatement; logits of the prompt close."""
    import mimgpu
    cfg, w = _synthetic(2, 4096, 32, 8, 14336, 32000)
    C = 128
    rng = np.random.default_rng(3)
    prompt = rng.integers(0, cfg["vocab"], 16).astype(np.int32)
    m = mimgpu.Model(ctx, dict(cfg, context=C, a8=1, cache_f16=1, interleaved=1, max_tokens=16), w)
    s = m.session()
    ref = O.Llama(dict(cfg, context=C, a8=1, cache_f16=1, interleaved=1), w)
    got = s.run(prompt, np.arange(16))[0]
    want = ref.forward(prompt, np.arange(16))[0]
    assert np.abs(got - want).max() <= 1e-3 * np.abs(want).max()
    tok = O.argmax(want)
    gen = s.generate(tok, 16, 64)
    cur, want_ids, margins = tok, [], []
    for i in range(64):
        lg = ref.forward([cur], [16 + i])[0]
        top = np.sort(lg)[-2:]
        margins.append(float(top[1] - top[0]))
        cur = O.argmax(lg)
        want_ids.append(cur)
    assert gen.tolist() == want_ids, (gen.tolist(), want_ids, margins)
    s.free()
    m.free()


@pytest.mark.parametrize("T", [8, 24, 160])
def test_refused_rows_same_in_step_and_prompt(ctx, T):
    """Weight rows with a non-finite block scale take the f32 product
    (linearA8, interp/fast.go:282-379) on every path: a one-token step, whose
    GEMVs normalise their own activation row (fused rms_norm) and add the
    residual read at their start, gives the same logits bit for bit as the
    same token as the last row of a prompt pass, whose rms_norm is a kernel
    of its own."""
    import mimgpu
    cfg, w = _synthetic(2, 512, 4, 2, 1024, 700, seed=7)
    rb = {O.Q4_K: 144, O.Q6_K: 210}
    for name, row in (("blk.0.attn_q.weight", 5), ("blk.1.ffn_gate.weight", 100), ("blk.0.ffn_up.weight", 513),
                      ("blk.1.ffn_down.weight", 33), ("output.weight", 17)):
        dt, arr = w[name]
        b = bytearray(arr.tobytes())
        k = 1024 if "ffn_down" in name else 512
        o = row * (k // 256) * rb[dt] + (0 if dt == O.Q4_K else 208)
        b[o:o + 2] = bytes([0x00, 0x7C])  # d = +inf in the row's first block
        w[name] = (dt, np.frombuffer(bytes(b), np.uint8))
    C = 192
    # 24 tokens: the prompt pass's products split K over several CTAs (few
    # row tiles), refused pairs included in the chain kernel; 160 tokens:
    # the prompt pass takes the one-block-per-row rms_norm
    ids = ((np.arange(T) * 37 + 3) % 700).astype(np.int32)
    m = mimgpu.Model(ctx, dict(cfg, context=C, a8=1, cache_f16=1, interleaved=1, max_tokens=T), w)
    s = m.session()
    whole = s.run(ids, np.arange(T), all_rows=True)
    s.reset()
    s.run(ids[:T - 1], np.arange(T - 1))
    step = s.run(ids[T - 1:], np.array([T - 1]))
    assert np.array_equal(np.isnan(step[0]), np.isnan(whole[T - 1]))
    fin = ~np.isnan(whole[T - 1])
    assert np.array_equal(step[0][fin].view(np.uint32), whole[T - 1][fin].view(np.uint32))
    s.free()
    m.free()


def test_tiny_llama_from_the_importers_mim_file(ctx, tiny):
    """The reference importer's own file of the tiny Llama (container 0.2,
    tests/golden/tiny_llama.mim) through mimgpu.load_llama: its prompt and
    greedy logits stay within llama.cpp's distance from the float64 oracle
    (cmd/mim-run/main_test.go:218-267), and equal bit for bit those of the
    same weights bound from the GGUF bytes."""
    import os
    import mimgpu
    e, w = tiny
    V = e["config"]["vocab"]
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "tiny_llama.mim")
    ids = e["prompt_ids"]
    m = mimgpu.load_llama(ctx, path, a8=True, cache_f16=True, max_tokens=len(ids))
    s = m.session()
    got = s.run(ids, np.arange(len(ids)), all_rows=True)
    worst = np.abs(got - f32b64(e["prompt_logits"]).reshape(len(ids), V)).max()
    logits, pos = got[-1], len(ids)
    for i, nxt in enumerate(e["greedy"]):
        worst = max(worst, np.abs(logits - f32b64(e["greedy_logits"][i])).max())
        logits = s.run([nxt], [pos])[0]
        pos += 1
    assert worst <= e["llama_cpp_max_diff"] * 1.1
    m2 = _model(ctx, e, w, a8=1, cache_f16=1)
    s2 = m2.session()
    assert np.array_equal(s2.run(ids, np.arange(len(ids)), all_rows=True).view(np.uint32), got.view(np.uint32))
    s.free()
    m.free()
    s2.free()
    m2.free()


@pytest.mark.parametrize("shape,layers", [("8b", 2), ("70b", 1)])
def test_fused_norm_bit_identical(ctx, shape, layers):
    """One-token steps with each rms_norm inside the GEMV that reads it (the
    default) and as a kernel of its own: logits bit for bit and greedy ids
    identical, at the 8B and 70B layer dimensions."""
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    cfg = dict(bench.SHAPES[shape], layers=layers, vocab=4096)
    C, P = 64, 12
    m, weights = bench.build_model(ctx, cfg, C, P)
    ids = bench.prompt_ids(cfg["vocab"], P, seed=9)
    sess = []
    for norm in (True, False):
        s = m.session()
        s.set_fusions(norm=norm)
        s.run(ids, np.arange(P))
        sess.append(s)
    tok = 5
    for i in range(3):
        a, b = (s.run([tok], [P + i])[0] for s in sess)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), P + i
        tok = int(np.argmax(a))
    ga, gb = (s.generate(tok, P + 3, 16).tolist() for s in sess)
    assert ga == gb
    for s in sess:
        s.free()
    m.free()
    for _, t in weights.values():
        t.free()
