"""Makes tests/golden/mim_writer.json: mim files authored by this library's
writer (mimir-model_b200/mimwriter.py) for the tiny Llama of
tests/golden/tiny_llama.mim, loaded, validated and executed by the
reference's own Python package (python/mim of gsoultan/mimir-model:
container.open_file, executor.Program.load -> graph.validate, Session.run).

    python tests/golden/make_mim_writer_golden.py /path/to/mimir-model

Cases: the a8 graph with an f16 cache (dequant_matmul_a8.v2, attention.v2)
and the same with three slots, run in slot 1; and the tiny Qwen 2 of
tests/golden/tiny_qwen2.* (query/key/value biases, rotation of head
halves) with dequant_matmul.v1 products and an f32 cache, run through its
9-token prompt and its 8 greedy steps.  Recorded per case: the authored
file's SHA-256 and size (the tests check that the writer still writes
exactly that file) and the logits the executor returned (f32, base64; for
the Qwen 2 every prompt row, and the ids it picked).  The script asserts
that the three-slot file gives the single-slot logits bit for bit, and
that the Qwen 2 file meets the reference's own bar
(cmd/mim-run/main_test.go:179-216): every prompt and step logit within
2e-5 of the largest of the float64 logits in the reference's
testdata/qwen2/expected.json, and the same greedy ids.
"""
import base64
import hashlib
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "mimir-model_b200"))

import mimfile  # noqa: E402
import mimwriter  # noqa: E402


def main(ref: str):
    sys.path.insert(0, os.path.join(ref, "python"))
    from mim import container, executor, dtypes as MD, tensor as MT

    f = mimfile.MimFile(os.path.join(HERE, "tiny_llama.mim"))
    md = f.metadata(typed=True)
    ctx = md.pop("mim.context_length")[1]
    md.pop("import.source_format")
    cfg = mimfile.llama_config(f)
    tensors = {n: (t.dtype, t.shape, bytes(f.data(n))) for n, t in f.tensors.items() if n != "mim.kv_positions"}
    with open(os.path.join(HERE, "tiny_llama.json")) as fh:
        ids = json.load(fh)["prompt_ids"]
    T = len(ids)
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        for case, slots in (("a8_f16", 1), ("a8_f16_slots3", 3)):
            path = os.path.join(tmp, case + ".mim")
            mimwriter.write_llama(path, cfg, tensors, a8=True, cache_f16=True, context=ctx, slots=slots, metadata=md)
            with open(path, "rb") as fh:
                data = fh.read()
            s = executor.Program.load(container.open_file(path)).session()
            inp = {"tokens": MT.Tensor(MD.I32, [1, T], np.array([ids], np.int32)),
                   "positions": MT.Tensor(MD.I64, [1, T], np.arange(T, dtype=np.int64)[None])}
            if slots > 1:
                inp["slots"] = MT.Tensor(MD.I64, [1, T], np.ones((1, T), np.int64))
            logits = np.ascontiguousarray(np.asarray(s.run(inp)["logits"].arr, np.float32).reshape(T, -1))
            out[case] = dict(slots=slots, sha256=hashlib.sha256(data).hexdigest(), bytes=len(data),
                             logits=base64.b64encode(logits.tobytes()).decode())
    out["qwen2_v1"] = qwen2_case(container, executor, MD, MT)
    a = np.frombuffer(base64.b64decode(out["a8_f16"]["logits"]), np.float32)
    b = np.frombuffer(base64.b64decode(out["a8_f16_slots3"]["logits"]), np.float32)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), "slot 1 differs from the single-slot file"
    with open(os.path.join(HERE, "mim_writer.json"), "w") as fh:
        json.dump(out, fh, indent=1)
        fh.write("\n")


def near(got, want, tol=2e-5):
    return float(np.abs(got - want).max()) <= tol * float(np.abs(want).max())


def qwen2_case(container, executor, MD, MT):
    with open(os.path.join(HERE, "tiny_qwen2.json")) as fh:
        e = json.load(fh)
    blob = np.fromfile(os.path.join(HERE, "tiny_qwen2.bin"), np.uint8)
    tensors = {t["name"]: (t["dtype"], tuple(t["shape"]), blob[t["offset"]:t["offset"] + t["nbytes"]].tobytes())
               for t in e["tensors"]}
    cfg = e["config"]
    V, ids = cfg["vocab"], e["prompt_ids"]
    T = len(ids)
    md = mimwriter.llama_metadata(cfg, arch="qwen2")
    f32 = lambda s: np.frombuffer(base64.b64decode(s), np.float32)  # noqa: E731
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "qwen2.mim")
        mimwriter.write_llama(path, cfg, tensors, a8=False, cache_f16=False, context=cfg["context"], metadata=md)
        with open(path, "rb") as fh:
            data = fh.read()
        s = executor.Program.load(container.open_file(path)).session()

        def run(toks, p0):
            n = len(toks)
            r = s.run({"tokens": MT.Tensor(MD.I32, [1, n], np.array([toks], np.int32)),
                       "positions": MT.Tensor(MD.I64, [1, n], np.arange(p0, p0 + n, dtype=np.int64)[None])})
            return np.ascontiguousarray(np.asarray(r["logits"].arr, np.float32).reshape(n, V))

        prompt = run(ids, 0)
        assert near(prompt.ravel(), f32(e["prompt_logits"])), "prompt logits"
        logits, pos, picked = prompt[-1], T, []
        for i, want in enumerate(e["greedy"]):
            assert near(logits, f32(e["greedy_logits"][i])), f"step {i} logits"
            picked.append(int(np.argmax(logits)))
            assert picked[-1] == want, (i, picked[-1], want)
            logits = run([want], pos)[0]
            pos += 1
    return dict(slots=1, sha256=hashlib.sha256(data).hexdigest(), bytes=len(data),
                logits=base64.b64encode(prompt.tobytes()).decode(), greedy=picked)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_mim_writer_golden.py <path to the mimir-model checkout>")
    main(sys.argv[1])
