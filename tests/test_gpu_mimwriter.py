"""The benchmark model authored as a mim file (bench.write_mim ->
mimwriter.write_llama: the reference importer's layout and forward graph,
importer/llama.go:323-547) and loaded back through mimgpu.load_llama runs
bit for bit like the same weights bound directly: the prompt's logits and
16 greedy ids at two layers of the 8B shape."""
import numpy as np
import pytest

import bench

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    import mimgpu
    c = mimgpu.Context(0)
    yield c
    c.close()


def test_bench_model_through_a_mim_file(ctx, tmp_path):
    import mimfile
    import mimgpu
    cfg = dict(bench.CFG8B, layers=2, vocab=32000)
    P, C = 16, 64
    model, weights = bench.build_model(ctx, cfg, C, P)
    path = str(tmp_path / "bench8b_2l.mim")
    size = bench.write_mim(ctx, cfg, weights, path, C)
    with mimfile.MimFile(path) as f:
        f.verify_hashes()
        assert f.data_offset + f.data_length == size
        md = f.metadata()
        assert md["mim.context_length"] == C and md["llama.block_count"] == 2
        assert mimfile.GRAPH in f.sections
        for name in ("blk.1.ffn_down.weight", "output.weight", "blk.0.attn_norm.weight"):
            dt, t = weights[name]
            assert f.tensors[name].dtype == dt and bytes(f.data(name)) == ctx.download(t).tobytes()
    m2 = mimgpu.load_llama(ctx, path, max_tokens=P, context=C)
    ids = bench.prompt_ids(cfg["vocab"], P, seed=3)
    s1, s2 = model.session(), m2.session()
    a = s1.run(ids, np.arange(P))[0]
    b = s2.run(ids, np.arange(P))[0]
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    tok = int(np.argmax(a))
    assert s1.generate(tok, P, 16).tolist() == s2.generate(tok, P, 16).tolist()
    for o in (s1, s2, model, m2):
        o.free()
    for _, t in weights.values():
        t.free()


def test_qwen2_through_an_authored_file(ctx, tmp_path):
    """The tiny Qwen 2 written by mimwriter (biases as the third inputs of the
    q, k, v products, rotation of halves) and loaded by mimgpu.load_llama:
    the same prompt logits and greedy ids bit for bit as the same weights
    bound directly."""
    import os
    import mimgpu
    import mimwriter
    from conftest import GOLDEN, load_tiny
    e, w = load_tiny("qwen2")
    with open(os.path.join(GOLDEN, "tiny_qwen2.bin"), "rb") as f:
        blob = f.read()
    tensors = {t["name"]: (t["dtype"], tuple(t["shape"]), blob[t["offset"]:t["offset"] + t["nbytes"]])
               for t in e["tensors"]}
    cfg = e["config"]
    path = str(tmp_path / "qwen2.mim")
    mimwriter.write_llama(path, cfg, tensors, context=cfg["context"], metadata=mimwriter.llama_metadata(cfg, arch="qwen2"))
    ids = e["prompt_ids"]
    P = len(ids)
    m1 = mimgpu.Model(ctx, dict(cfg, a8=1, cache_f16=1, interleaved=0, max_tokens=P), w)
    m2 = mimgpu.load_llama(ctx, path, max_tokens=P)
    s1, s2 = m1.session(), m2.session()
    a = s1.run(ids, np.arange(P), all_rows=True)
    b = s2.run(ids, np.arange(P), all_rows=True)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    tok = int(np.argmax(a[-1]))
    assert s1.generate(tok, P, 8).tolist() == s2.generate(tok, P, 8).tolist()
    for o in (s1, s2, m1, m2):
        o.free()
