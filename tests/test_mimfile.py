"""The mim-file reader (mimir-model_b200/mimfile.py) against the reference's
container spec (spec/container.md v0.2, spec/metadata.md).

* A small valid file made by the writer below (the spec's canonical packing,
  sorted tensor table, metadata section) reads back exactly; single-fault
  mutations of it are rejected with the spec's error code, in the spirit of
  the reference's hostile corpus (hostile_test.go, spec/container.md §9.1).
* The reference importer's tiny Llama (tests/golden/tiny_llama.mim, a byte
  copy of testdata/compat/0.2-0.1/tiny-llama.mim) reads with the metadata
  and tensor bytes of the GGUF it came from (tests/golden/tiny_llama.*).
* Where the reference checkout is present, every file of its compat corpus
  reads the same through this reader and the reference's own Python reader.
"""
import hashlib
import json
import os
import struct
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "mimir-model_b200"))
import mimfile as M  # noqa: E402

GOLDEN = os.path.join(HERE, "golden")
REF = os.environ.get("MIM_REFERENCE", "/root/reference")


def _meta(entries):
    """spec/metadata.md: entries sorted by key; ints, strings, floats."""
    keys = sorted(entries)
    pool = bytearray()
    rows = []
    for k in keys:
        v = entries[k]
        ko, kb = len(pool), k.encode()
        pool += kb
        if isinstance(v, bool):
            rows.append(struct.pack("<IIB3xIQQ", ko, len(kb), 4, 0, int(v), 0))
        elif isinstance(v, int):
            rows.append(struct.pack("<IIB3xIQQ", ko, len(kb), 2, 0, v, 0))
        elif isinstance(v, float):
            rows.append(struct.pack("<IIB3xIQQ", ko, len(kb), 3, 0, struct.unpack("<Q", struct.pack("<d", v))[0], 0))
        else:
            vb = v.encode()
            vo = len(pool)
            pool += vb
            rows.append(struct.pack("<IIB3xIQQ", ko, len(kb), 5, len(vb), vo, 0))
    return b"MIMM" + struct.pack("<IQ", len(keys), len(pool)) + b"".join(rows) + bytes(pool)


def write_mim(tensors, meta=None, align=4096):
    """A canonical file: tensors [(name, dtype, shape, bytes)] packed in the
    given order, the table sorted by name, hashed sections."""
    data = bytearray()
    entries = []
    for name, dt, shape, raw in tensors:
        a = M.LARGE_ALIGN if len(raw) >= M.LARGE else M.TENSOR_ALIGN
        data += b"\0" * (-len(data) % a)
        entries.append((name.encode(), dt, shape, len(data), len(raw)))
        data += raw
    entries.sort(key=lambda e: e[0])
    pool = b"".join(e[0] for e in entries)
    md = _meta(meta) if meta is not None else None
    ns = 1 + (md is not None)
    ilen = 16 + 64 * ns + 96 * len(entries) + len(pool)
    ioff = 64
    moff = (ioff + ilen + 63) // 64 * 64
    doff = ((moff + (len(md) if md else 0)) + align - 1) // align * align
    flen = doff + len(data)
    index = struct.pack("<IIQ", ns, len(entries), len(pool))

    def sect(kind, flags, off, blob):
        return struct.pack("<IIQQB7x", kind, flags, off, len(blob), 1) + hashlib.sha256(blob).digest()

    index += sect(1, 1, doff, bytes(data))
    if md is not None:
        index += sect(2, 0, moff, md)
    no = 0
    for name, dt, shape, off, ln in entries:
        dims = list(shape) + [0] * (8 - len(shape))
        index += struct.pack("<IIIB3x8QQQ", no, len(name), dt, len(shape), *dims, off, ln)
        no += len(name)
    index += pool
    pre = b"MIM\0" + struct.pack("<HHII", 0, 2, 0x0A0B0C0D, align) + struct.pack("<QQQQQQ", ioff, ilen, doff,
                                                                                  len(data), flen, 0)
    out = bytearray(flen)
    out[0:64] = pre
    out[ioff:ioff + ilen] = index
    if md is not None:
        out[moff:moff + len(md)] = md
    out[doff:] = data
    return bytes(out), dict(ioff=ioff, ilen=ilen, doff=doff, ns=ns)


def _tensors():
    rng = np.random.default_rng(1)
    return [("b.weight", 1, (4, 8), rng.standard_normal(32).astype(np.float32).tobytes()),
            ("a.weight", 66, (2, 256), rng.integers(0, 256, 2 * 144, dtype=np.uint8).tobytes()),
            ("c.weight", 2, (3,), np.arange(3, dtype=np.float16).tobytes())]


def _open(tmp_path, blob):
    p = tmp_path / "m.mim"
    p.write_bytes(blob)
    return M.MimFile(str(p))


def test_valid_file_reads_back(tmp_path):
    ts = _tensors()
    blob, _ = write_mim(ts, {"general.architecture": "llama", "llama.block_count": 2, "x.eps": 1e-5, "b": True})
    with _open(tmp_path, blob) as f:
        f.verify_hashes()
        assert sorted(f.tensors) == ["a.weight", "b.weight", "c.weight"]
        for name, dt, shape, raw in ts:
            assert f.tensors[name].dtype == dt and f.tensors[name].shape == shape
            assert bytes(f.data(name)) == raw
        md = f.metadata()
        assert md == {"general.architecture": "llama", "llama.block_count": 2, "x.eps": 1e-5, "b": True}
        with pytest.raises(M.MimError) as e:
            f.data("nope")
        assert e.value.code == "not-found"


def _mutations(blob, lay):
    """(label, mutated file, expected code) for single faults."""
    b = bytearray(blob)
    ioff, doff = lay["ioff"], lay["doff"]
    t0 = ioff + 16 + 64 * lay["ns"]  # first tensor entry
    out = []

    def put(label, code, fn):
        x = bytearray(b)
        fn(x)
        out.append((label, bytes(x), code))

    out.append(("truncated-preamble", bytes(b[:40]), "truncated"))
    put("bad-magic", "bad-magic", lambda x: x.__setitem__(slice(0, 4), b"XIM\0"))
    put("big-endian", "big-endian", lambda x: x.__setitem__(slice(8, 12), bytes([0x0A, 0x0B, 0x0C, 0x0D])))
    put("bad-bom", "bad-byte-order-mark", lambda x: x.__setitem__(slice(8, 12), b"\1\2\3\4"))
    put("major-1", "unsupported-version", lambda x: x.__setitem__(slice(4, 6), b"\1\0"))
    put("alignment-1000", "bad-alignment", lambda x: x.__setitem__(slice(12, 16), struct.pack("<I", 1000)))
    out.append(("longer", bytes(b) + b"\0", "bad-length"))
    put("index-misaligned", "misaligned", lambda x: x.__setitem__(slice(16, 24), struct.pack("<Q", 65)))
    put("reserved", "reserved-non-zero", lambda x: x.__setitem__(56, 1))
    put("index-length", "bad-length", lambda x: x.__setitem__(slice(24, 32), struct.pack("<Q", lay["ilen"] + 8)))
    put("section-flag", "reserved-non-zero", lambda x: x.__setitem__(ioff + 16 + 4, 2))
    put("hash-alg", "bad-hash-algorithm", lambda x: x.__setitem__(ioff + 16 + 24, 7))
    put("weights-entry", "bad-length", lambda x: x.__setitem__(slice(ioff + 16 + 16, ioff + 16 + 24),
                                                                 struct.pack("<Q", 8)))
    put("bad-dtype", "bad-dtype", lambda x: x.__setitem__(slice(t0 + 8, t0 + 12), struct.pack("<I", 99)))
    put("rank-9", "bad-shape", lambda x: x.__setitem__(t0 + 12, 9))
    put("size-mismatch", "size-mismatch", lambda x: x.__setitem__(slice(t0 + 88, t0 + 96), struct.pack("<Q", 1)))
    return out


def test_hostile_single_faults(tmp_path):
    blob, lay = write_mim(_tensors(), {"general.name": "t"})
    for label, bad, code in _mutations(blob, lay):
        with pytest.raises(M.MimError) as e:
            _open(tmp_path, bad)
        assert e.value.code == code, (label, e.value)
    # table order: swap the first two names in the pool (a.weight <-> b.weight)
    x = bytearray(blob)
    pool = lay["ioff"] + lay["ilen"] - len(b"a.weightb.weightc.weight")
    x[pool:pool + 16] = b"b.weighta.weight"
    with pytest.raises(M.MimError) as e:
        _open(tmp_path, bytes(x))
    assert e.value.code in ("unsorted", "size-mismatch")
    # a tensor moved off its canonical position
    x = bytearray(blob)
    t0 = lay["ioff"] + 16 + 64 * lay["ns"]
    off = struct.unpack_from("<Q", x, t0 + 80)[0]
    struct.pack_into("<Q", x, t0 + 80, off + 64)
    with pytest.raises(M.MimError) as e:
        _open(tmp_path, bytes(x))
    assert e.value.code in ("non-canonical-layout", "out-of-bounds", "overlap")
    # no weights section
    x = bytearray(blob)
    struct.pack_into("<I", x, lay["ioff"] + 16, 6)
    with pytest.raises(M.MimError) as e:
        _open(tmp_path, bytes(x))
    assert e.value.code in ("unknown-required-section", "missing-section")


def test_tiny_llama_mim_matches_its_gguf():
    """The importer's file holds the GGUF's tensors byte for byte and the
    dimensions of its metadata (config of tests/golden/tiny_llama.json)."""
    with open(os.path.join(GOLDEN, "tiny_llama.json")) as fh:
        e = json.load(fh)
    blob = np.fromfile(os.path.join(GOLDEN, "tiny_llama.bin"), np.uint8)
    with M.MimFile(os.path.join(GOLDEN, "tiny_llama.mim")) as f:
        f.verify_hashes()
        cfg = M.llama_config(f)
        for k in ("layers", "embed", "ffn", "heads", "kv_heads", "head_dim", "rope_dims", "vocab", "context"):
            assert cfg[k] == e["config"][k], k
        assert cfg["rope_theta"] == e["config"]["rope_theta"]
        assert np.float32(cfg["norm_eps"]) == np.float32(e["config"]["norm_eps"])
        for t in e["tensors"]:
            mt = f.tensors[t["name"]]
            assert mt.dtype == t["dtype"] and list(mt.shape) == t["shape"]
            assert bytes(f.data(t["name"])) == blob[t["offset"]:t["offset"] + t["nbytes"]].tobytes()


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "python", "mim")), reason="no reference checkout")
def test_same_as_reference_reader_on_compat_corpus():
    sys.path.insert(0, os.path.join(REF, "python"))
    from mim.container import File  # the reference's own reader, as the checker

    root = os.path.join(REF, "testdata", "compat")
    n = 0
    for d in sorted(os.listdir(root)):
        for fn in sorted(os.listdir(os.path.join(root, d))):
            if not fn.endswith(".mim"):
                continue
            p = os.path.join(root, d, fn)
            rf = File.open(p)
            try:
                with M.MimFile(p) as f:
                    rt = {t.name: t for t in rf.tensors()}
                    assert sorted(rt) == sorted(f.tensors), p
                    for name, t in f.tensors.items():
                        assert rt[name].dtype.id == t.dtype and tuple(rt[name].shape) == t.shape, (p, name)
                        assert bytes(rf.tensor_data(rt[name])) == bytes(f.data(name)), (p, name)
                    rmd = rf.metadata()
                    md = f.metadata()
                    assert sorted(rmd) == sorted(md), p
                    for k, (typ, v) in rmd.items():
                        if typ in ("float", "floats"):
                            assert np.array_equal(np.float64(v), np.float64(md[k]), equal_nan=True), (p, k)
                        else:
                            assert md[k] == v, (p, k, typ)
                    n += 1
            finally:
                rf.close()
    assert n >= 3
