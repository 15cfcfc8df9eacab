"""Generates the golden fixtures under tests/golden/ from the reference's own
test data.  Run in a checkout that has the reference next to it:

    python tests/golden/make_golden.py /path/to/mimir-model

It reads, and never modifies:
  * testdata/quant_golden.json (quant_test.go:279-339): the decode golden
    vectors (bytes + exact f32 bits) for q8_0, q4_k and q6_k, and the q8_0
    encoder's input bits;
  * testdata/llama/tiny-q4km.gguf + expected.json (cmd/mim-run/main_test.go:
    179-267): the 2-layer tiny Llama whose prompt and greedy logits the
    float64 oracle wrote;
  * testdata/qwen2/tiny-q4km.gguf + expected.json: the tiny Qwen 2 of the
    same test (query/key/value biases, rotation of head halves), written as
    tiny_qwen2.bin / tiny_qwen2.json in the same way;
  * testdata/compat/0.2-0.1/tiny-llama.mim: the same tiny Llama as the
    reference's importer writes it (container 0.2: weights, metadata and
    graph sections), for the mim-file loader.

It writes quant_golden.json, tiny_llama.bin (the raw tensor bytes, byte for
byte as File.TensorData returns them), tiny_llama.json (tensor index,
hyperparameters and the expected logits/ids) and tiny_llama.mim (a byte
copy).  The gguf package (0.19) parses the GGUF container only; no
arithmetic of it is used.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

OUT = os.path.dirname(os.path.abspath(__file__))
DTYPE_IDS = {"F32": 1, "F16": 2, "Q8_0": 64, "Q4_K": 66, "Q6_K": 67}


def quant(ref: str):
    with open(os.path.join(ref, "testdata", "quant_golden.json")) as f:
        g = json.load(f)
    keep = {k: {kk: g[k][kk] for kk in ("bytes", "input_bits", "bits")} for k in ("q8_0", "q4_k", "q6_k")}
    with open(os.path.join(OUT, "quant_golden.json"), "w") as f:
        json.dump(keep, f)


def tiny_llama(ref: str, name: str = "llama"):
    import gguf

    d = os.path.join(ref, "testdata", name)
    with open(os.path.join(d, "expected.json")) as f:
        e = json.load(f)
    r = gguf.GGUFReader(os.path.join(d, e["model"]))
    arch = r.fields["general.architecture"].contents()
    meta = {k: r.fields[k].contents() for k in r.fields if k.startswith(arch + ".")}
    blob = bytearray()
    index = []
    for t in r.tensors:
        raw = bytes(np.asarray(t.data).tobytes())
        assert len(raw) == t.n_bytes, (t.name, len(raw), t.n_bytes)
        ne = [int(x) for x in t.shape]  # ggml order: ne0 (K) first
        shape = list(reversed(ne))      # mim order [N, K]
        off = len(blob)
        blob += raw
        blob += b"\0" * (-len(blob) % 256)
        index.append({"name": t.name, "dtype": DTYPE_IDS[t.tensor_type.name], "shape": shape,
                      "offset": off, "nbytes": len(raw)})
    with open(os.path.join(OUT, f"tiny_{name}.bin"), "wb") as f:
        f.write(blob)
    E = int(meta[f"{arch}.embedding_length"])
    H = int(meta[f"{arch}.attention.head_count"])
    cfg = {
        "arch": arch,
        "layers": int(meta[f"{arch}.block_count"]),
        "embed": E,
        "ffn": int(meta[f"{arch}.feed_forward_length"]),
        "heads": H,
        "kv_heads": int(meta.get(f"{arch}.attention.head_count_kv", H)),
        "head_dim": E // H,
        "rope_dims": int(meta.get(f"{arch}.rope.dimension_count", E // H)),
        "rope_theta": float(meta.get(f"{arch}.rope.freq_base", 10000.0)),
        "norm_eps": float(meta[f"{arch}.attention.layer_norm_rms_epsilon"]),
        "vocab": int(e["vocab"]),
        "context": 64,  # importFixture's LlamaOptions{Context: 64}
    }
    out = {"config": cfg, "tensors": index,
           "prompt_ids": e["prompt_ids"], "prompt_logits": e["prompt_logits"],
           "greedy": e["greedy"], "greedy_logits": e["greedy_logits"],
           "llama_cpp_max_diff": e["llama_cpp_max_diff"]}
    with open(os.path.join(OUT, f"tiny_{name}.json"), "w") as f:
        json.dump(out, f)


def mim_fixture(ref: str):
    src = os.path.join(ref, "testdata", "compat", "0.2-0.1", "tiny-llama.mim")
    with open(src, "rb") as f, open(os.path.join(OUT, "tiny_llama.mim"), "wb") as g:
        g.write(f.read())


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MIM_REFERENCE", "")
    if not ref or not os.path.isdir(ref):
        sys.exit("usage: make_golden.py <path to the mimir-model checkout>")
    quant(ref)
    tiny_llama(ref, "llama")
    tiny_llama(ref, "qwen2")
    mim_fixture(ref)
    print("wrote", sorted(os.listdir(OUT)))
