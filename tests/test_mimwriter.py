"""Authoring mim files (mimir-model_b200/mimwriter.py).

  * The reference importer's own file of the tiny Llama (testdata/compat/
    0.2-0.1/tiny-llama.mim of gsoultan/mimir-model: BuildLlama with
    dequant_matmul.v1 products and an f32 cache, context 64) is rebuilt from
    its tensors and metadata byte for byte: container layout, hashes,
    metadata section and the whole forward graph (importer/llama.go:323-547,
    importer/importer.go:115-160, writer.go, graph.go, metadata.go).
  * The a8 / f16-cache and three-slot graphs written for the same weights
    are the files whose SHA-256 tests/golden/mim_writer.json records, the
    ones the reference's own Python package validated and executed when the
    fixture was made (tests/golden/make_mim_writer_golden.py); the logits
    it computed for them are checked against the CPU restatement here.
  * The tiny Qwen 2's file (biases, rotation of head halves) was executed
    by the same package and meets the reference's own 2e-5 bar against its
    float64 logits, with the same greedy ids.
  * Round trips through this library's reader, every metadata type, and the
    writer's refusals.
"""
import hashlib
import json
import os

import numpy as np
import pytest

import mimfile
import mimwriter as W
from conftest import GOLDEN, f32b64, load_tiny

SRC = os.path.join(GOLDEN, "tiny_llama.mim")


def _source():
    """The fixture's tensors (without the importer-made kv positions), its
    metadata without the two keys the builder and importer add, its config."""
    f = mimfile.MimFile(SRC)
    md = f.metadata(typed=True)
    ctx = md.pop("mim.context_length")[1]
    md.pop("import.source_format")
    tensors = {n: (t.dtype, t.shape, bytes(f.data(n))) for n, t in f.tensors.items() if n != "mim.kv_positions"}
    cfg = mimfile.llama_config(f)
    f.close()
    return cfg, tensors, md, ctx


def test_rebuilds_the_importers_file_byte_for_byte():
    cfg, tensors, md, ctx = _source()
    out = W.write_llama(None, cfg, tensors, a8=False, cache_f16=False, context=ctx, metadata=md)
    with open(SRC, "rb") as f:
        want = f.read()
    assert len(out) == len(want)
    assert out == want


def test_tensor_insertion_order_does_not_change_the_file():
    cfg, tensors, md, ctx = _source()
    rev = dict(reversed(list(tensors.items())))
    a = W.write_llama(None, cfg, tensors, context=ctx, metadata=md)
    b = W.write_llama(None, cfg, rev, context=ctx, metadata=md)
    assert a == b


def _golden():
    with open(os.path.join(GOLDEN, "mim_writer.json")) as f:
        return json.load(f)


@pytest.mark.parametrize("case", ["a8_f16", "a8_f16_slots3"])
def test_authored_files_are_the_ones_the_reference_ran(case):
    g = _golden()[case]
    cfg, tensors, md, ctx = _source()
    out = W.write_llama(None, cfg, tensors, a8=True, cache_f16=True, context=ctx, slots=g["slots"], metadata=md)
    assert hashlib.sha256(out).hexdigest() == g["sha256"]
    assert len(out) == g["bytes"]


def test_reference_executor_logits_match_the_oracle():
    """The reference's Python executor ran the authored a8 / f16-cache file
    (its dequant_matmul_a8 is the f32 product there) and the three-slot file
    in slot 1; both gave the same logits, within 2e-5 of the largest logit of
    the CPU restatement's f32-product forward with an f16 cache."""
    import oracle as O
    g = _golden()
    e, w = load_tiny()
    ids = e["prompt_ids"]
    T = len(ids)
    single = f32b64(g["a8_f16"]["logits"]).reshape(T, -1)
    slot1 = f32b64(g["a8_f16_slots3"]["logits"]).reshape(T, -1)
    assert np.array_equal(single.view(np.uint32), slot1.view(np.uint32))
    ref = O.Llama(dict(e["config"], a8=0, cache_f16=1, interleaved=1), w)
    want = ref.forward(ids, np.arange(T), all_rows=True)
    assert np.abs(single - want).max() <= 2e-5 * np.abs(want).max()


def test_qwen2_file_meets_the_references_bar():
    """The tiny Qwen 2 (query/key/value biases, rotation of head halves) as
    this writer authors it is the file the reference's Python executor ran
    when the fixture was made; what it computed meets the reference's own
    bar (cmd/mim-run/main_test.go:179-216): every prompt logit within 2e-5
    of the largest float64 logit of testdata/qwen2/expected.json, and the
    same 8 greedy ids."""
    g = _golden()["qwen2_v1"]
    e, _ = load_tiny("qwen2")
    with open(os.path.join(GOLDEN, "tiny_qwen2.bin"), "rb") as f:
        blob = f.read()
    tensors = {t["name"]: (t["dtype"], tuple(t["shape"]), blob[t["offset"]:t["offset"] + t["nbytes"]])
               for t in e["tensors"]}
    cfg = e["config"]
    out = W.write_llama(None, cfg, tensors, a8=False, cache_f16=False, context=cfg["context"],
                        metadata=W.llama_metadata(cfg, arch="qwen2"))
    assert hashlib.sha256(out).hexdigest() == g["sha256"] and len(out) == g["bytes"]
    got, want = f32b64(g["logits"]), f32b64(e["prompt_logits"])
    assert np.abs(got - want).max() <= 2e-5 * np.abs(want).max()
    assert g["greedy"] == e["greedy"]
    # the graph carries the biases as third inputs of the q, k, v products
    # and rotates head halves
    assert b"attn_q.bias" in out and b"interleaved" in out


def test_round_trip_through_the_reader(tmp_path):
    cfg, tensors, md, ctx = _source()
    path = str(tmp_path / "t.mim")
    W.write_llama(path, cfg, tensors, a8=True, cache_f16=True, context=ctx, slots=2, metadata=md)
    with mimfile.MimFile(path) as f:
        f.verify_hashes()
        for n, (dt, shape, data) in tensors.items():
            t = f.tensors[n]
            assert (t.dtype, tuple(t.shape)) == (dt, tuple(shape)) and bytes(f.data(n)) == data
        got = f.metadata(typed=True)
        assert got["mim.context_length"] == (1, ctx) and got["mim.slots"] == (1, 2)
        assert got["import.source_format"] == (5, "gguf")
        for k, v in md.items():
            assert got[k] == v, k
        kv = np.frombuffer(f.data("mim.kv_positions"), "<i8")
        assert kv.tolist() == list(range(2 * ctx))
        assert mimfile.llama_config(f)["layers"] == cfg["layers"]


def test_every_metadata_type_round_trips(tmp_path):
    md = {"i": -5, "u": W.Uint(2 ** 63 + 7), "f": -0.25, "b": True, "s": "naïve", "y": b"\x00\x01\xff",
          "ii": [1, -2, 3], "ff": [0.5, -1.5], "ss": ["a", "", "ß"], "e": []}
    w = W.MimWriter()
    w.add_tensor("x", W.F32, (2,), np.array([1, 2], "<f4").tobytes())
    w.add_section(mimfile.METADATA, W.encode_metadata(md))
    path = str(tmp_path / "m.mim")
    w.write(path)
    with mimfile.MimFile(path) as f:
        f.verify_hashes()
        got = f.metadata(typed=True)
    assert got == {"i": (1, -5), "u": (2, 2 ** 63 + 7), "f": (3, -0.25), "b": (4, True), "s": (5, "naïve"),
                   "y": (6, b"\x00\x01\xff"), "ii": (7, [1, -2, 3]), "ff": (8, [0.5, -1.5]),
                   "ss": (9, ["a", "", "ß"]), "e": (7, [])}
    # typed entries go back unchanged
    assert W.encode_metadata(got) == W.encode_metadata(md)


def test_canonical_packing_of_large_and_small_tensors(tmp_path):
    w = W.MimWriter(data_alignment=4096)
    w.add_tensor("a", W.U8, (3,), b"abc")
    w.add_tensor("b", W.U8, (1 << 20,), bytes(1 << 20))
    w.add_tensor("c", W.U8, (5,), b"hello")
    path = str(tmp_path / "p.mim")
    w.write(path)
    with mimfile.MimFile(path) as f:
        assert [f.tensors[n].offset for n in "abc"] == [0, 4096, 4096 + (1 << 20)]
        assert f.data_offset % 4096 == 0 and bytes(f.data("c")) == b"hello"


def test_refusals():
    w = W.MimWriter()
    w.add_tensor("x", W.F32, (1,), bytes(4))
    with pytest.raises(mimfile.MimError, match="duplicate"):
        w.add_tensor("x", W.F32, (1,), bytes(4))
    with pytest.raises(mimfile.MimError, match="size-mismatch"):
        w.add_tensor("y", W.F32, (2,), bytes(4))
    with pytest.raises(mimfile.MimError, match="bad-name"):
        w.add_tensor("", W.F32, (1,), bytes(4))
    with pytest.raises(mimfile.MimError, match="duplicate"):
        w.add_section(mimfile.WEIGHTS, b"")
    with pytest.raises(mimfile.MimError, match="bad-alignment"):
        W.MimWriter(data_alignment=1000)
    cfg, tensors, md, ctx = _source()
    with pytest.raises(mimfile.MimError, match="cache would exceed"):
        W.write_llama(None, cfg, tensors, context=1 << 19, slots=3, metadata=md)
    with pytest.raises(mimfile.MimError, match="token_embd"):
        W.write_llama(None, cfg, {k: v for k, v in tensors.items() if k != "token_embd.weight"}, metadata=md)
    bad = dict(tensors)
    dt, shape, data = bad["blk.1.ffn_up.weight"]
    bad["blk.1.ffn_up.weight"] = (dt, (shape[0] // 2, shape[1]), data[:len(data) // 2])
    with pytest.raises(mimfile.MimError, match="ffn_up"):
        W.write_llama(None, cfg, bad, metadata=md)
