"""Writing mim files (the container of gsoultan/mimir-model): the container
(spec/container.md v0.2), the metadata section (spec/metadata.md), the
graph section (spec/graph.md v0.1) and the forward-pass graph of a
Llama-family model as the reference's importer builds it
(importer/llama.go:323-547, BuildLlama), so a model -- the benchmark's 8B
and 70B shapes included -- can be authored as a file that the reference's
interpreter and this library's `load_llama` both run.

Layout choices the spec leaves open follow the reference's writer, so that
the same tensors, metadata and options give the same bytes as a file the
reference's importer writes (the tests check this against the importer's
own tiny-Llama file):
  * tensors are packed in the order they are added, each at the canonical
    alignment (64 bytes, 4,096 from 1 MiB, spec/container.md §6), and listed
    in the index sorted by name with the name pool in that order
    (writer.go:96-223); the importer adds them sorted by name
    (importer/importer.go:115-160);
  * the weights section is entry 0 of the section table, the other sections
    follow in the order they were added, placed after the index at 64-byte
    boundaries, the weights at the next multiple of the data alignment;
  * metadata entries are sorted by key and the pool is filled in that order
    (metadata.go:54-148);
  * the graph's string pool and dims table grow in first-use order: the
    empty string, symbolic dimension names, value names and shapes in value
    order, then per op its attribute keys and payloads (graph.go:234-374).
"""
from __future__ import annotations

import hashlib
import os
import struct
from dataclasses import dataclass, field

try:
    from .mimfile import (DTYPES, FLAG_REQUIRED, GRAPH, INDEX_HEADER, LARGE, LARGE_ALIGN, MAX_ALIGN, MAX_NAME,
                          MAX_RANK, METADATA, MIN_ALIGN, PREAMBLE, SECTION_ENTRY, TENSOR_ALIGN, TENSOR_ENTRY,
                          WEIGHTS, MimError, _nbytes)
except ImportError:
    from mimfile import (DTYPES, FLAG_REQUIRED, GRAPH, INDEX_HEADER, LARGE, LARGE_ALIGN, MAX_ALIGN, MAX_NAME,
                         MAX_RANK, METADATA, MIN_ALIGN, PREAMBLE, SECTION_ENTRY, TENSOR_ALIGN, TENSOR_ENTRY,
                         WEIGHTS, MimError, _nbytes)

# dtype ids (spec/dtypes.md)
F32, F16, BF16, F64, I8, U8, I16, U16, I32, U32, I64, U64, BOOL, F8E4M3, F8E5M2 = range(1, 16)
Q8_0, Q4_0, Q4_K, Q6_K, MXFP4, AFFINE4_G64 = 64, 65, 66, 67, 68, 69
_FLOAT8 = (F8E4M3, F8E5M2)


def _up(n: int, a: int) -> int:
    return (n + a - 1) // a * a


# ---------------------------------------------------------------- metadata

class Uint(int):
    """A metadata integer stored as uint64 (type 2); a plain int is int64."""


def _meta_entry(v):
    """(type, plain value) of a metadata value (spec/metadata.md types 1-9)."""
    if isinstance(v, bool):
        return 4, v
    if isinstance(v, Uint):
        return 2, int(v)
    if isinstance(v, int):
        return 1, v
    if isinstance(v, float):
        return 3, v
    if isinstance(v, str):
        return 5, v
    if isinstance(v, (bytes, bytearray, memoryview)):
        return 6, bytes(v)
    if isinstance(v, (list, tuple)):
        if v and all(isinstance(x, str) for x in v):
            return 9, list(v)
        if v and all(isinstance(x, float) for x in v):
            return 8, list(v)
        if all(isinstance(x, int) and not isinstance(x, bool) for x in v):
            return 7, list(v)
    raise MimError("bad-metadata", f"unsupported value {type(v).__name__}")


def encode_metadata(md: dict) -> bytes:
    """The metadata section for {key: value}.  Values are Python values
    (int -> int64, Uint -> uint64, float, bool, str, bytes, lists of ints,
    floats or strs) or explicit (type, value) pairs as
    `MimFile.metadata(typed=True)` returns them."""
    entries, pool = [], bytearray()
    for key in sorted(md, key=lambda k: k.encode("utf-8")):
        kb = key.encode("utf-8")
        if not kb or len(kb) > 1024:
            raise MimError("bad-metadata", f"key {key!r}")
        v = md[key]
        if isinstance(v, tuple) and len(v) == 2 and type(v[0]) is int and 1 <= v[0] <= 9:
            typ, val = v
        else:
            typ, val = _meta_entry(v)
        koff = len(pool)
        pool += kb
        count = 0
        if typ == 1:
            payload = val & (2 ** 64 - 1)
        elif typ == 2:
            payload = val
        elif typ == 3:
            payload = struct.unpack("<Q", struct.pack("<d", val))[0]
        elif typ == 4:
            payload = 1 if val else 0
        elif typ in (5, 6):
            b = val.encode("utf-8") if typ == 5 else bytes(val)
            payload, count = len(pool), len(b)
            pool += b
        elif typ in (7, 8):
            pool += bytes(_up(len(pool), 8) - len(pool))
            payload, count = len(pool), len(val)
            pool += struct.pack(f"<{len(val)}{'q' if typ == 7 else 'd'}", *val)
        elif typ == 9:
            strs = [s.encode("utf-8") for s in val]
            tab, at = bytearray(), len(pool) + 8 * len(strs)
            for s in strs:
                tab += struct.pack("<II", at, len(s))
                at += len(s)
            payload, count = len(pool), len(strs)
            pool += tab + b"".join(strs)
        else:
            raise MimError("bad-metadata", f"{key}: type {typ}")
        entries.append(struct.pack("<IIB3xIQ8x", koff, len(kb), typ, count, payload))
    return b"MIMM" + struct.pack("<IQ", len(entries), len(pool)) + b"".join(entries) + bytes(pool)


# --------------------------------------------------------------- container

@dataclass
class _WTensor:
    name: str
    dtype: int
    shape: tuple
    data: object   # bytes, or a callable returning them (read twice: hash, then write)
    length: int
    offset: int = 0

    def bytes(self) -> bytes:
        if not callable(self.data):
            return self.data
        b = self.data()
        b = b if isinstance(b, bytes) else bytes(b)
        if len(b) != self.length:
            raise MimError("size-mismatch", f"tensor {self.name!r} gave {len(b)} bytes, needs {self.length}")
        return b


class MimWriter:
    """Tensors and sections in, a mim file out (spec/container.md)."""

    def __init__(self, data_alignment: int = 16384, hashes: bool = True):
        if data_alignment & (data_alignment - 1) or not MIN_ALIGN <= data_alignment <= MAX_ALIGN:
            raise MimError("bad-alignment", str(data_alignment))
        self.align, self.hashes = data_alignment, hashes
        self.tensors: list[_WTensor] = []
        self.sections: list[tuple[int, int, bytes]] = []
        self._names: set[str] = set()

    def add_tensor(self, name: str, dtype: int, shape, data) -> None:
        """data: the tensor's bytes, or a callable that returns them when the
        file is written (called twice with hashes on: once for the weights
        section's SHA-256, once to write), so large models need not sit in
        host memory whole."""
        nb = name.encode("utf-8")
        if not nb or len(nb) > MAX_NAME:
            raise MimError("bad-name", repr(name))
        if name in self._names:
            raise MimError("duplicate", f"tensor {name!r}")
        shape = tuple(int(d) for d in shape)
        if len(shape) > MAX_RANK:
            raise MimError("bad-shape", f"tensor {name!r} rank {len(shape)}")
        if dtype not in DTYPES:
            raise MimError("unsupported-dtype", f"tensor {name!r} dtype {dtype}")
        need = _nbytes(dtype, shape)
        if not callable(data):
            data = data if isinstance(data, bytes) else bytes(data)
            if need != len(data):
                raise MimError("size-mismatch", f"tensor {name!r} needs {need} bytes, got {len(data)}")
        self._names.add(name)
        self.tensors.append(_WTensor(name, dtype, shape, data, need))

    def add_section(self, kind: int, data: bytes, required: bool = False) -> None:
        if kind == WEIGHTS or any(k == kind for k, _, _ in self.sections):
            raise MimError("duplicate", f"section kind {kind}")
        self.sections.append((kind, FLAG_REQUIRED if required else 0, bytes(data)))

    def _pack(self) -> int:
        """Offsets of the canonical packing, in insertion order; the length."""
        end = 0
        for t in self.tensors:
            t.offset = _up(end, LARGE_ALIGN if t.length >= LARGE else TENSOR_ALIGN)
            end = t.offset + t.length
        return end

    def _weight_chunks(self):
        at = 0
        for t in self.tensors:
            if t.offset > at:
                yield bytes(t.offset - at)
            yield t.bytes()
            at = t.offset + t.length

    def chunks(self):
        """The file as a sequence of byte strings (the weights are not
        copied into one buffer)."""
        data_len = self._pack()
        order = sorted(self.tensors, key=lambda t: t.name.encode("utf-8"))
        pool, name_off = bytearray(), {}
        for t in order:
            name_off[t.name] = len(pool)
            pool += t.name.encode("utf-8")
        nsec = len(self.sections) + 1
        index_len = INDEX_HEADER + SECTION_ENTRY * nsec + TENSOR_ENTRY * len(order) + len(pool)
        pos, offs = _up(PREAMBLE + index_len, 64), []
        for _, _, d in self.sections:
            offs.append(pos)
            pos = _up(pos + len(d), 64)
        data_off = _up(pos, self.align)

        def entry(kind, flags, off, ln, digest):
            tail = struct.pack("<B7x", 1) + digest if self.hashes else bytes(40)
            return struct.pack("<IIQQ", kind, flags, off, ln) + tail

        wh = b""
        if self.hashes:
            h = hashlib.sha256()
            for c in self._weight_chunks():
                h.update(c)
            wh = h.digest()
        head = bytearray(b"MIM\0" + struct.pack("<HHII", 0, 2, 0x0A0B0C0D, self.align))
        head += struct.pack("<QQQQQQ", PREAMBLE, index_len, data_off, data_len, data_off + data_len, 0)
        head += struct.pack("<IIQ", nsec, len(order), len(pool))
        head += entry(WEIGHTS, FLAG_REQUIRED, data_off, data_len, wh)
        for (kind, flags, d), off in zip(self.sections, offs):
            head += entry(kind, flags, off, len(d), hashlib.sha256(d).digest() if self.hashes else b"")
        for t in order:
            dims = list(t.shape) + [0] * (MAX_RANK - len(t.shape))
            head += struct.pack("<IIIB3x8QQQ", name_off[t.name], len(t.name.encode("utf-8")), t.dtype,
                                len(t.shape), *dims, t.offset, t.length)
        head += pool
        yield bytes(head)
        at = len(head)
        for (_, _, d), off in zip(self.sections, offs):
            yield bytes(off - at)
            yield d
            at = off + len(d)
        yield bytes(data_off - at)
        yield from self._weight_chunks()

    def to_bytes(self) -> bytes:
        return b"".join(self.chunks())

    def write(self, path: str) -> None:
        """Writes the file through a temporary name in the same folder."""
        tmp = f"{path}.tmp{os.getpid()}"
        try:
            with open(tmp, "wb") as f:
                for c in self.chunks():
                    f.write(c)
            os.replace(tmp, path)
        finally:
            if os.path.exists(tmp):
                os.remove(tmp)


# ------------------------------------------------------------------- graph

# opcodes (spec/primitives.md §1) used by the builders here
OP = dict(cast=8, add=10, mul=11, or_=19, xor=20, cmplt=21, reshape=25, permute=27, scatter=31, const=32, call=34)
# value kinds and attribute types (spec/graph.md §3.4, §3.7)
INTERMEDIATE, INPUT, OUTPUT, WEIGHT, VARIABLE, CONST = range(6)
A_INT, A_INTS, A_FLOAT, A_STRING, A_DTYPE, A_SUBGRAPH = range(1, 7)
_ROWS = (1, 8, 16, 8, 32, 32, 4, 24, 32, 16, 8)  # row bytes of the 11 tables


@dataclass
class Value:
    name: str
    dtype: int
    shape: list            # sizes; d < 0 is symbolic dimension -1 - d
    kind: int = INTERMEDIATE
    ref: int = 0           # tensor index (weight, const, variable)
    zero: bool = False     # a variable that starts as zeros


@dataclass
class Op:
    opcode: int
    inputs: list
    outputs: list
    attrs: list = field(default_factory=list)  # (key, type, payload)


@dataclass
class Graph:
    symdims: list = field(default_factory=list)       # (name, bound)
    values: list = field(default_factory=list)        # Value
    subgraphs: list = field(default_factory=list)     # (ops, inputs, outputs); 0 is the main graph
    composites: list = field(default_factory=list)    # (name, version, subgraph)
    updates: list = field(default_factory=list)       # (variable, new value)
    primitive_version: int = 1
    stdlib_version: int = 1

    def encode(self) -> bytes:
        """The graph section (spec/graph.md): an 11-table directory after the
        16-byte header, every table 8-byte aligned."""
        t = _Tables()
        t.string("")
        for name, bound in self.symdims:
            t.tab[2] += struct.pack("<IIq", t.string(name), 0, bound)
        for v in self.values:
            if len(v.shape) > MAX_RANK:
                raise MimError("bad-shape", f"value {v.name!r} rank {len(v.shape)}")
            name = t.string(v.name)
            t.tab[4] += struct.pack("<IIIBBBxI12x", name, v.dtype, t.dims(v.shape), len(v.shape), v.kind,
                                    1 if v.zero else 0, v.ref)
        for ops, ins, outs in self.subgraphs:
            first = len(t.tab[5]) // 32
            for op in ops:
                a0 = len(t.tab[7]) // 24
                for key, typ, val in op.attrs:
                    k, count = t.string(key), 0
                    if typ == A_INT:
                        payload = val & (2 ** 64 - 1)
                    elif typ == A_INTS:
                        payload, count = t.dims(val), len(val)
                    elif typ == A_FLOAT:
                        payload = struct.unpack("<Q", struct.pack("<d", val))[0]
                    elif typ == A_STRING:
                        payload = t.string(val)
                    elif typ in (A_DTYPE, A_SUBGRAPH):
                        payload = val
                    else:
                        raise MimError("bad-graph", f"attribute {key!r} type {typ}")
                    t.tab[7] += struct.pack("<IB3xI4xQ", k, typ, count, payload)
                t.tab[5] += struct.pack("<H2xIIIIII4x", op.opcode, t.run(op.inputs), len(op.inputs),
                                        t.run(op.outputs), len(op.outputs), a0, len(op.attrs))
            t.tab[8] += struct.pack("<IIIIII8x", first, len(ops), t.run(ins), len(ins), t.run(outs), len(outs))
        for name, version, sub in self.composites:
            t.tab[9] += struct.pack("<IIII", t.string(name), version, sub, 0)
        for var, val in self.updates:
            t.tab[10] += struct.pack("<II", var, val)
        out = bytearray(b"MIMG" + struct.pack("<HHII", 0, 1, self.primitive_version, self.stdlib_version))
        out += bytes(16 * len(_ROWS))
        for i, tab in enumerate(t.tab):
            out += bytes(_up(len(out), 8) - len(out))
            struct.pack_into("<QQ", out, 16 + 16 * i, len(out), len(tab) // _ROWS[i])
            out += tab
        return bytes(out)


class _Tables:
    """The growing tables of one graph encoding: 0 string pool, 1 strings,
    2 symbolic dims, 3 dims, 4 values, 5 ops, 6 runs, 7 attrs, 8 subgraphs,
    9 composites, 10 updates."""

    def __init__(self):
        self.tab = [bytearray() for _ in _ROWS]
        self._str: dict[str, int] = {}

    def string(self, s: str) -> int:
        i = self._str.get(s)
        if i is None:
            b = s.encode("utf-8")
            if len(b) > MAX_NAME:
                raise MimError("bad-graph", f"string of {len(b)} bytes")
            i = self._str[s] = len(self.tab[1]) // 8
            self.tab[1] += struct.pack("<II", len(self.tab[0]), len(b))
            self.tab[0] += b
        return i

    def dims(self, ds) -> int:
        off = len(self.tab[3]) // 8
        self.tab[3] += struct.pack(f"<{len(ds)}q", *ds)
        return off

    def run(self, ids) -> int:
        off = len(self.tab[6]) // 4
        self.tab[6] += struct.pack(f"<{len(ids)}I", *ids)
        return off


# ------------------------------------------------------------------- Llama

MAX_LLAMA_CONTEXT = 1 << 20  # importer/llama.go:50: a typo cannot ask for an enormous cache


class _LlamaGraph:
    """The forward pass of importer/llama.go:323-547 (BuildLlama) for one
    block of tokens: inputs tokens i32[1, T] and positions i64[1, T] (and
    slots i64[1, T] with several sequences), output logits f32[1, T, V], the
    key-value cache as zero-initialised variables blk.N.cache_k / cache_v
    [1, Hkv, slots * C, D] that each layer scatters its new rows into before
    attending with the mask j <= p.  Values and ops are created in the order
    BuildLlama creates them, so the encoded section is the same."""

    def __init__(self, tensors: dict, a8: bool, cache: int):
        self.g = Graph(subgraphs=[([], [], [])])
        self.tensors = tensors        # name -> (dtype, shape)
        self.a8, self.cache = a8, cache
        self.stored_names: dict[int, str] = {}   # value id -> tensor name
        self.by_weight: dict[str, int] = {}

    @property
    def main(self):
        return self.g.subgraphs[0]

    def val(self, name, dt, *shape, kind=INTERMEDIATE) -> int:
        self.g.values.append(Value(name, dt, list(shape), kind))
        return len(self.g.values) - 1

    def op(self, opc, ins, out, *attrs) -> int:
        self.main[0].append(Op(OP[opc], list(ins), [out], list(attrs)))
        return out

    def call(self, name, ins, out, *attrs, version=1) -> int:
        return self.op("call", ins, out, ("name", A_STRING, name), ("version", A_INT, version), *attrs)

    def stored(self, name, kind) -> int:
        dt, shape = self.tensors[name]
        vid = self.val(name, dt, *shape, kind=kind)
        self.stored_names[vid] = name
        return vid

    def zeros(self, name, dt, *shape) -> int:
        self.g.values.append(Value(name, dt, list(shape), VARIABLE, 0, True))
        return len(self.g.values) - 1

    def weight(self, name, *shape) -> int:
        if name in self.by_weight:
            return self.by_weight[name]
        if name not in self.tensors:
            raise MimError("not-found", f"tensor {name!r} is missing")
        got = tuple(self.tensors[name][1])
        if got != tuple(shape):
            raise MimError("bad-shape", f"tensor {name!r} is {list(got)}, want {list(shape)}")
        vid = self.by_weight[name] = self.stored(name, WEIGHT)
        return vid

    def matmul(self, name, x, w, *shape, bias=None) -> int:
        """x times w^T: linear.v1 for f32 weights, dequant_matmul_a8 (v2 with
        blocks of 256 for Q4_K/Q6_K, v1 otherwise) with 8-bit activations,
        dequant_matmul.v1 without (importer/llama.go:243-268)."""
        out = self.val(name, F32, *shape)
        ins = [x, w] + ([bias] if bias is not None else [])
        dt = self.g.values[w].dtype
        if dt == F32:
            return self.call("linear", ins, out)
        if self.a8 and dt in (Q4_K, Q6_K):
            return self.call("dequant_matmul_a8", ins, out, ("block", A_INT, 256), version=2)
        if self.a8:
            return self.call("dequant_matmul_a8", ins, out)
        return self.call("dequant_matmul", ins, out)

    def f32_of(self, w) -> int:
        v = self.g.values[w]
        if v.dtype == F32:
            return w
        return self.op("cast", [w], self.val(v.name + ".f32", F32, *v.shape), ("to", A_DTYPE, F32))

    def build(self, c: dict) -> None:
        E, F, H, Hkv, D = c["embed"], c["ffn"], c["heads"], c["kv_heads"], c["head_dim"]
        slots, ctx = c["slots"], c["context"]
        C, V, T, sym = slots * ctx, c["vocab"], -1, -1
        self.g.symdims = [("T", C)]
        tokens = self.val("tokens", I32, 1, T, kind=INPUT)
        positions = self.val("positions", I64, 1, T, kind=INPUT)
        self.main[1].extend([tokens, positions])
        # mask: key j visible from the query at cache position p when j <= p
        # (and, with several slots, j >= the slot's first position)
        kpos = self.stored("mim.kv_positions", CONST)
        at, start = positions, None
        if slots > 1:
            sl = self.val("slots", I64, 1, T, kind=INPUT)
            self.main[1].append(sl)
            size = self.op("const", [], self.val("slot_size", I64, 1, 1), ("value", A_INT, ctx))
            start = self.op("mul", [sl, size], self.val("slot_start", I64, 1, T))
            at = self.op("add", [start, positions], self.val("slot_positions", I64, 1, T))
        qpos = self.op("reshape", [at], self.val("query_positions", I64, 1, 1, T, 1), ("shape", A_INTS, [1, 1, sym, 1]))
        hidden = self.op("cmplt", [qpos, kpos], self.val("mask.future", BOOL, 1, 1, T, C))
        if slots > 1:
            qstart = self.op("reshape", [start], self.val("query_slot_start", I64, 1, 1, T, 1),
                             ("shape", A_INTS, [1, 1, sym, 1]))
            before = self.op("cmplt", [kpos, qstart], self.val("mask.other_slots", BOOL, 1, 1, T, C))
            hidden = self.op("or_", [hidden, before], self.val("mask.hidden", BOOL, 1, 1, T, C))
        truth = self.op("const", [], self.val("true", BOOL, 1, 1, 1, 1), ("value", A_INT, 1))
        mask = self.op("xor", [hidden, truth], self.val("mask", BOOL, 1, 1, T, C))
        cache_idx = self.op("reshape", [at], self.val("cache_index", I64, T), ("shape", A_INTS, [sym]))

        table = self.stored("token_embd.weight", WEIGHT)
        edt = self.tensors["token_embd.weight"][0]
        if edt == F32 or DTYPES[edt][0] > 1 or edt in _FLOAT8:
            x = self.call("embedding", [table, tokens], self.val("embed", F32, 1, T, E))
        else:
            raw = self.call("embedding", [table, tokens], self.val("embed.raw", edt, 1, T, E))
            x = self.op("cast", [raw], self.val("embed", F32, 1, T, E), ("to", A_DTYPE, F32))
        eps = ("epsilon", A_FLOAT, float(c["norm_eps"]))
        qwen2 = c["arch"] == "qwen2"
        rope = (("theta", A_FLOAT, float(c["rope_theta"])), ("interleaved", A_INT, 0 if qwen2 else 1),
                ("rotary_dims", A_INT, c["rope_dims"]))
        cshape = (1, Hkv, C, D)
        for layer in range(c["layers"]):
            p = f"blk.{layer}."

            def w(name, *shape):
                return self.weight(p + name, *shape)

            attn_norm = w("attn_norm.weight", E)
            wq, wk, wv = w("attn_q.weight", E, E), w("attn_k.weight", Hkv * D, E), w("attn_v.weight", Hkv * D, E)
            wo, ffn_norm = w("attn_output.weight", E, E), w("ffn_norm.weight", E)
            wg, wu, wd = w("ffn_gate.weight", F, E), w("ffn_up.weight", F, E), w("ffn_down.weight", E, F)
            cache_k = self.zeros(p + "cache_k", self.cache, *cshape)
            cache_v = self.zeros(p + "cache_v", self.cache, *cshape)
            h = self.call("rms_norm", [x, self.f32_of(attn_norm)], self.val(p + "attn_in", F32, 1, T, E), eps)

            def heads(name, wt, n):
                bias = self.f32_of(w(f"attn_{name}.bias", n * D)) if qwen2 else None
                y = self.matmul(p + name, h, wt, 1, T, n * D, bias=bias)
                y = self.op("reshape", [y], self.val(p + name + ".heads", F32, 1, T, n, D),
                            ("shape", A_INTS, [1, sym, n, D]))
                return self.op("permute", [y], self.val(p + name + ".bhtd", F32, 1, n, T, D),
                               ("perm", A_INTS, [0, 2, 1, 3]))

            q, k, v = heads("q", wq, H), heads("k", wk, Hkv), heads("v", wv, Hkv)
            q = self.call("rope", [q, positions], self.val(p + "q.rope", F32, 1, H, T, D), *rope)
            k = self.call("rope", [k, positions], self.val(p + "k.rope", F32, 1, Hkv, T, D), *rope)
            version = 1
            if self.cache == F16:  # rounded to f16 on the way into the cache; attention.v2 reads them as they are
                k = self.op("cast", [k], self.val(p + "k.f16", F16, 1, Hkv, T, D), ("to", A_DTYPE, F16))
                v = self.op("cast", [v], self.val(p + "v.f16", F16, 1, Hkv, T, D), ("to", A_DTYPE, F16))
                version = 2
            axis = ("axis", A_INT, 2)
            new_k = self.op("scatter", [cache_k, cache_idx, k], self.val(p + "cache_k.next", self.cache, *cshape), axis)
            new_v = self.op("scatter", [cache_v, cache_idx, v], self.val(p + "cache_v.next", self.cache, *cshape), axis)
            self.g.updates += [(cache_k, new_k), (cache_v, new_v)]
            o = self.call("attention", [q, new_k, new_v, mask], self.val(p + "attn", F32, 1, H, T, D),
                          ("num_kv_heads", A_INT, Hkv), version=version)
            o = self.op("permute", [o], self.val(p + "attn.bthd", F32, 1, T, H, D), ("perm", A_INTS, [0, 2, 1, 3]))
            o = self.op("reshape", [o], self.val(p + "attn.merged", F32, 1, T, E), ("shape", A_INTS, [1, sym, E]))
            o = self.matmul(p + "attn_out", o, wo, 1, T, E)
            x = self.op("add", [x, o], self.val(p + "resid_attn", F32, 1, T, E))
            h = self.call("rms_norm", [x, self.f32_of(ffn_norm)], self.val(p + "ffn_in", F32, 1, T, E), eps)
            gate, up = self.matmul(p + "gate", h, wg, 1, T, F), self.matmul(p + "up", h, wu, 1, T, F)
            act = self.call("swiglu", [gate, up], self.val(p + "swiglu", F32, 1, T, F))
            down = self.matmul(p + "down", act, wd, 1, T, E)
            x = self.op("add", [x, down], self.val(p + "resid_ffn", F32, 1, T, E))
        out_norm = self.weight("output_norm.weight", E)
        head = self.weight("output.weight", V, E) if "output.weight" in self.tensors else table  # tied embeddings
        x = self.call("rms_norm", [x, self.f32_of(out_norm)], self.val("final_norm", F32, 1, T, E), eps)
        logits = self.matmul("logits", x, head, 1, T, V)
        self.g.values[logits].kind = OUTPUT
        self.main[2].append(logits)


def llama_metadata(cfg: dict, name: str = "", arch: str = "llama") -> dict:
    """The hyperparameter entries a Llama (or Qwen 2) GGUF carries, as the
    reference's GGUF importer keeps them (unsigned integers, float64): the
    keys importer/llama.go:104-162 (LlamaConfigOf) reads back."""
    md = {
        "general.architecture": arch,
        f"{arch}.block_count": Uint(cfg["layers"]),
        f"{arch}.embedding_length": Uint(cfg["embed"]),
        f"{arch}.feed_forward_length": Uint(cfg["ffn"]),
        f"{arch}.attention.head_count": Uint(cfg["heads"]),
        f"{arch}.attention.head_count_kv": Uint(cfg["kv_heads"]),
        f"{arch}.context_length": Uint(cfg.get("max_context", cfg.get("context", 4096))),
        f"{arch}.rope.dimension_count": Uint(cfg.get("rope_dims", cfg["embed"] // cfg["heads"])),
        f"{arch}.rope.freq_base": float(cfg.get("rope_theta", 10000.0)),
        f"{arch}.attention.layer_norm_rms_epsilon": float(cfg["norm_eps"]),
    }
    if name:
        md["general.name"] = name
    return md


def write_llama(path: str | None, cfg: dict, tensors: dict, *, a8: bool = True, cache_f16: bool = True,
                context: int | None = None, slots: int = 1, metadata: dict | None = None,
                source_format: str = "gguf", data_alignment: int = 16384):
    """A Llama model as a mim file with the reference importer's forward
    graph (BuildLlama, then Source.AddTo: importer/llama.go:323-547,
    importer/importer.go:115-160).

    cfg: layers, embed, ffn, heads, kv_heads, rope_dims, rope_theta, norm_eps
    (head_dim = embed / heads, the vocabulary from token_embd.weight).
    tensors: {GGUF name: (dtype, shape, bytes or a callable returning them)},
    every tensor of the file.
    metadata: the entries to keep (llama_metadata(cfg) when None); the
    builder adds mim.context_length (and mim.slots), the importer
    import.source_format.  a8 writes the quantized products as
    dequant_matmul_a8 (v2, blocks of 256, for Q4_K/Q6_K), cache_f16 an f16
    cache read by attention.v2.  Returns the bytes when path is None."""
    context = int(context or cfg.get("context", 4096))
    if metadata is None:
        metadata = llama_metadata(dict(cfg, context=context))
    arch = metadata.get("general.architecture", "llama")
    arch = arch[1] if isinstance(arch, tuple) else arch
    if arch not in ("llama", "qwen2"):
        raise MimError("unsupported", f"architecture {arch!r}: only llama and qwen2 graphs are built")
    E, H, Hkv = int(cfg["embed"]), int(cfg["heads"]), int(cfg["kv_heads"])
    if E % H or H % Hkv:
        raise MimError("bad-shape", f"embedding length {E}, {H} heads and {Hkv} key-value heads do not divide")
    D = E // H
    rope_dims = int(cfg.get("rope_dims", D))
    if rope_dims % 2 or rope_dims > D:
        raise MimError("bad-shape", f"rope dimension count {rope_dims} for head size {D}")
    slots = max(1, int(slots))
    if context > MAX_LLAMA_CONTEXT or slots > 1 << 10 or slots * context > MAX_LLAMA_CONTEXT:
        raise MimError("bad-shape", f"{slots} slots of {context} positions: the cache would exceed {MAX_LLAMA_CONTEXT}")
    emb = tensors.get("token_embd.weight")
    if emb is None or len(emb[1]) != 2 or int(emb[1][1]) != E:
        raise MimError("not-found", f"tensor token_embd.weight is missing or not [V, {E}]")
    if "mim.kv_positions" in tensors:
        raise MimError("duplicate", "tensor 'mim.kv_positions' already exists in the source")
    import numpy as np
    C = slots * context
    every = dict(tensors)
    every["mim.kv_positions"] = (I64, (1, 1, 1, C), np.arange(C, dtype="<i8").tobytes())
    b = _LlamaGraph({n: (int(t[0]), tuple(int(d) for d in t[1])) for n, t in every.items()}, a8,
                    F16 if cache_f16 else F32)
    b.build(dict(layers=int(cfg["layers"]), embed=E, ffn=int(cfg["ffn"]), heads=H, kv_heads=Hkv, head_dim=D,
                 rope_dims=rope_dims, rope_theta=float(cfg.get("rope_theta", 10000.0)),
                 norm_eps=float(cfg["norm_eps"]), vocab=int(emb[1][0]), context=context, slots=slots, arch=arch))
    order = sorted(every, key=lambda n: n.encode("utf-8"))
    index = {n: i for i, n in enumerate(order)}
    for vid, name in b.stored_names.items():
        b.g.values[vid].ref = index[name]
    w = MimWriter(data_alignment)
    for n in order:
        dt, shape, data = every[n]
        w.add_tensor(n, int(dt), shape, data)
    w.add_section(GRAPH, b.g.encode(), required=True)
    md = dict(metadata)
    md["mim.context_length"] = context
    if slots > 1:
        md["mim.slots"] = slots
    md["import.source_format"] = source_format
    w.add_section(METADATA, encode_metadata(md))
    if path is None:
        return w.to_bytes()
    w.write(path)
    return None
