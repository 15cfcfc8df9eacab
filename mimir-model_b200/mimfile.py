"""Reading mim files (the container of gsoultan/mimir-model), so a model file
written by the reference's tools runs on the GPU path unchanged.

Follows the reference's spec/container.md v0.2 (preamble, index, section
table, tensor table, canonical packing of the weights section; the checks in
the order the spec lists them, each failure classified with the spec's error
code) and spec/metadata.md (typed key-value entries).  The graph section is
not interpreted: `load_llama` recognises a Llama file by its metadata (the
keys the reference's importer writes, importer/llama.go) and runs the
device-resident Llama step of this library over its tensors, which keep the
GGUF names the step binds.

The file is mapped read-only and tensor bytes are handed out as memoryviews
of the mapping; nothing is copied before the upload.
"""
from __future__ import annotations

import hashlib
import mmap
import struct
from dataclasses import dataclass

PREAMBLE = 64
INDEX_HEADER = 16
SECTION_ENTRY = 64
TENSOR_ENTRY = 96
MAX_INDEX = 256 << 20
MAX_RANK = 8
MAX_NAME = 4096
MIN_ALIGN, MAX_ALIGN = 4096, 16 << 20
TENSOR_ALIGN, LARGE_ALIGN, LARGE = 64, 4096, 1 << 20
FLAG_REQUIRED = 1
WEIGHTS, METADATA, GRAPH, REPACK, TRAINING = 1, 2, 3, 4, 5
U64 = (1 << 64) - 1

# dtype id -> (block elements, block bytes), spec/dtypes.md
DTYPES = {1: (1, 4), 2: (1, 2), 3: (1, 2), 4: (1, 8), 5: (1, 1), 6: (1, 1), 7: (1, 2), 8: (1, 2), 9: (1, 4),
          10: (1, 4), 11: (1, 8), 12: (1, 8), 13: (1, 1), 14: (1, 1), 15: (1, 1),
          64: (32, 34), 65: (32, 18), 66: (256, 144), 67: (256, 210), 68: (32, 17), 69: (64, 36)}


class MimError(Exception):
    """A rejected file; `code` is the spec's error code (spec/container.md §9)."""

    def __init__(self, code: str, msg: str = ""):
        super().__init__(f"{code}: {msg}" if msg else code)
        self.code = code


@dataclass(frozen=True)
class Section:
    kind: int
    flags: int
    offset: int
    length: int
    hash_alg: int
    hash: bytes


@dataclass(frozen=True)
class Tensor:
    name: str
    dtype: int
    shape: tuple
    offset: int  # relative to the weights section
    length: int


def _in_bounds(off: int, ln: int, size: int) -> bool:
    return off <= size and ln <= size - off


def _pow2(v: int) -> bool:
    return v > 0 and v & (v - 1) == 0


def _nbytes(dtype: int, shape: tuple) -> int:
    be, bb = DTYPES[dtype]
    n = 1
    for d in shape:
        n *= d
        if n > U64:
            raise MimError("overflow", f"element count of {list(shape)}")
    if be > 1 and (len(shape) == 0 or shape[-1] % be):
        raise MimError("bad-shape", f"dtype {dtype} needs a last axis that is a multiple of {be}")
    b = n // be * bb
    if b > U64:
        raise MimError("overflow", f"byte size of {list(shape)}")
    return b


class MimFile:
    """A validated mim file: `tensors` (name -> Tensor), `sections`
    (kind -> Section), `metadata()` (key -> value), `data(name)`."""

    def __init__(self, path: str):
        self._fh = open(path, "rb")
        try:
            size = self._fh.seek(0, 2)
            self._mm = mmap.mmap(self._fh.fileno(), 0, access=mmap.ACCESS_READ) if size else b""
            self._b = memoryview(self._mm)
            self._parse(self._b, size)
        except Exception:
            self.close()
            raise

    def close(self):
        b, self._b = getattr(self, "_b", None), None
        if isinstance(b, memoryview):
            b.release()
        mm, self._mm = getattr(self, "_mm", None), None
        if isinstance(mm, mmap.mmap):
            try:
                mm.close()
            except BufferError:
                pass  # views handed out by data() are alive: the mapping goes with the last of them
        if getattr(self, "_fh", None):
            self._fh.close()
            self._fh = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # ------------------------------------------------------------ parsing
    def _parse(self, b: memoryview, size: int):
        if size < PREAMBLE:
            raise MimError("truncated", f"{size} bytes")
        magic = bytes(b[0:4])
        if magic not in (b"MIM\0", b"MMF\0"):
            raise MimError("bad-magic", repr(magic))
        major, minor, bom, align = struct.unpack_from("<HHII", b, 4)
        if bom == 0x0D0C0B0A:
            raise MimError("big-endian")
        if bom != 0x0A0B0C0D:
            raise MimError("bad-byte-order-mark", hex(bom))
        if major != 0:
            raise MimError("unsupported-version", f"major {major}")
        if not _pow2(align) or not MIN_ALIGN <= align <= MAX_ALIGN:
            raise MimError("bad-alignment", str(align))
        ioff, ilen, doff, dlen, flen, reserved = struct.unpack_from("<QQQQQQ", b, 16)
        if flen > size:
            raise MimError("truncated", f"file length {flen} > {size}")
        if flen < size:
            raise MimError("bad-length", f"file length {flen} < {size}")
        if ioff < PREAMBLE or ioff % 8:
            raise MimError("misaligned", f"index offset {ioff}")
        if ilen > MAX_INDEX:
            raise MimError("index-too-large", str(ilen))
        if not _in_bounds(ioff, ilen, size):
            raise MimError("out-of-bounds", "index")
        if doff % align:
            raise MimError("misaligned", f"data offset {doff}")
        if not _in_bounds(doff, dlen, size):
            raise MimError("out-of-bounds", "weights")
        if reserved:
            raise MimError("reserved-non-zero", "preamble")
        self.major, self.minor, self.data_alignment = major, minor, align
        self.data_offset, self.data_length = doff, dlen

        # index header
        if ilen < INDEX_HEADER:
            raise MimError("truncated", "index")
        ns, nt, pool = struct.unpack_from("<IIQ", b, ioff)
        if pool > MAX_INDEX or ilen != INDEX_HEADER + SECTION_ENTRY * ns + TENSOR_ENTRY * nt + pool:
            raise MimError("bad-length", "index")
        pool_off = ioff + INDEX_HEADER + SECTION_ENTRY * ns + TENSOR_ENTRY * nt

        # sections
        self.sections = {}
        regions = [(0, PREAMBLE), (ioff, ilen)]
        have_weights = False
        for i in range(ns):
            o = ioff + INDEX_HEADER + SECTION_ENTRY * i
            kind, flags, off, ln, alg = struct.unpack_from("<IIQQB", b, o)
            if flags & ~FLAG_REQUIRED:
                raise MimError("reserved-non-zero", f"section {i} flags")
            if any(b[o + 25:o + 32]):
                raise MimError("reserved-non-zero", f"section {i}")
            h = bytes(b[o + 32:o + 64])
            if alg == 0 and any(h):
                raise MimError("reserved-non-zero", f"section {i} hash")
            if alg not in (0, 1):
                raise MimError("bad-hash-algorithm", str(alg))
            if not _in_bounds(off, ln, size):
                raise MimError("out-of-bounds", f"section {i}")
            known = 1 <= kind <= 5
            if known and kind in self.sections:
                raise MimError("duplicate", f"section kind {kind}")
            if not known and flags & FLAG_REQUIRED:
                raise MimError("unknown-required-section", f"kind {kind}")
            if kind == WEIGHTS:
                if off != doff or ln != dlen:
                    raise MimError("bad-length", "weights section entry")
                have_weights = True
            elif off % 8:
                raise MimError("misaligned", f"section {i}")
            if kind != WEIGHTS:
                regions.append((off, ln))
            if known:
                self.sections[kind] = Section(kind, flags, off, ln, alg, h)
        if not have_weights:
            raise MimError("missing-section", "weights")
        regions.append((doff, dlen))
        regions.sort()
        end = 0
        for off, ln in regions:
            if off < end:
                raise MimError("overlap", f"region at {off}")
            end = max(end, off + ln)

        # tensors
        self.tensors = {}
        prev = None
        order = []
        for i in range(nt):
            o = ioff + INDEX_HEADER + SECTION_ENTRY * ns + TENSOR_ENTRY * i
            noff, nlen, dtype, rank = struct.unpack_from("<IIIB", b, o)
            if not _in_bounds(noff, nlen, pool):
                raise MimError("out-of-bounds", f"tensor {i} name")
            raw = bytes(b[pool_off + noff:pool_off + noff + nlen])
            try:
                name = raw.decode("utf-8")
            except UnicodeDecodeError:
                raise MimError("bad-name", repr(raw)) from None
            if not 0 < nlen <= MAX_NAME:
                raise MimError("bad-name", f"tensor {i}")
            if dtype not in DTYPES:
                raise MimError("bad-dtype", f"{name}: {dtype}")
            if rank > MAX_RANK:
                raise MimError("bad-shape", f"{name}: rank {rank}")
            if any(b[o + 13:o + 16]):
                raise MimError("reserved-non-zero", f"tensor {name}")
            dims = struct.unpack_from("<8Q", b, o + 16)
            if any(dims[rank:]):
                raise MimError("reserved-non-zero", f"tensor {name} dims")
            toff, tlen = struct.unpack_from("<QQ", b, o + 80)
            shape = tuple(dims[:rank])
            if tlen != _nbytes(dtype, shape):
                raise MimError("size-mismatch", name)
            a = LARGE_ALIGN if tlen >= LARGE else TENSOR_ALIGN
            if toff % a:
                raise MimError("misaligned", name)
            if not _in_bounds(toff, tlen, dlen):
                raise MimError("out-of-bounds", f"{name} data")
            if prev is not None:
                if raw == prev:
                    raise MimError("duplicate", name)
                if raw < prev:
                    raise MimError("unsorted", name)
            prev = raw
            t = Tensor(name, dtype, shape, toff, tlen)
            self.tensors[name] = t
            order.append(t)

        # canonical packing of the weights section
        end = 0
        for t in sorted(order, key=lambda t: (t.offset, t.length)):
            a = LARGE_ALIGN if t.length >= LARGE else TENSOR_ALIGN
            want = (end + a - 1) // a * a
            if t.offset < end and t.length:
                raise MimError("overlap", t.name)
            if t.length and t.offset != want:
                raise MimError("non-canonical-layout", t.name)
            end = max(end, t.offset + t.length)
        if end != dlen:
            raise MimError("non-canonical-layout", "weights section end")

    # ------------------------------------------------------------- access
    def data(self, name: str) -> memoryview:
        """The tensor's bytes (a view of the mapping)."""
        t = self.tensors.get(name)
        if t is None:
            raise MimError("not-found", name)
        o = self.data_offset + t.offset
        return self._b[o:o + t.length]

    def section_bytes(self, kind: int) -> memoryview | None:
        s = self.sections.get(kind)
        return None if s is None else self._b[s.offset:s.offset + s.length]

    def verify_hashes(self):
        """SHA-256 of every hashed section (spec/container.md §5.3)."""
        for s in self.sections.values():
            if s.hash_alg == 1 and hashlib.sha256(self._b[s.offset:s.offset + s.length]).digest() != s.hash:
                raise MimError("hash-mismatch", f"section kind {s.kind}")

    def metadata(self, typed: bool = False) -> dict:
        """The metadata section as {key: value} (spec/metadata.md); ints,
        uints, floats, bools, strings, bytes and arrays decoded.  typed:
        {key: (type, value)}, the entry's type kept (1 int64, 2 uint64, ...),
        as the writer takes them back."""
        m = self.section_bytes(METADATA)
        if m is None:
            return {}
        if len(m) < 16 or bytes(m[0:4]) not in (b"MIMM", b"MMFM"):
            raise MimError("bad-metadata", "header")
        count, pool = struct.unpack_from("<IQ", m, 4)
        if count > 1 << 24 or len(m) != 16 + 32 * count + pool:
            raise MimError("bad-metadata", "length")
        p0 = 16 + 32 * count
        out = {}

        def pool_bytes(off, ln):
            if not _in_bounds(off, ln, pool):
                raise MimError("bad-metadata", "pool bounds")
            return bytes(m[p0 + off:p0 + off + ln])

        for i in range(count):
            e = 16 + 32 * i
            koff, klen, typ = struct.unpack_from("<IIB", m, e)
            cnt, payload = struct.unpack_from("<IQ", m, e + 12)
            key = pool_bytes(koff, klen).decode("utf-8")
            if typ == 1:
                v = struct.unpack("<q", struct.pack("<Q", payload))[0]
            elif typ == 2:
                v = payload
            elif typ == 3:
                v = struct.unpack("<d", struct.pack("<Q", payload))[0]
            elif typ == 4:
                v = bool(payload)
            elif typ == 5:
                v = pool_bytes(payload, cnt).decode("utf-8")
            elif typ == 6:
                v = pool_bytes(payload, cnt)
            elif typ == 7:
                v = list(struct.unpack(f"<{cnt}q", pool_bytes(payload, 8 * cnt)))
            elif typ == 8:
                v = list(struct.unpack(f"<{cnt}d", pool_bytes(payload, 8 * cnt)))
            elif typ == 9:
                tab = struct.unpack(f"<{2 * cnt}I", pool_bytes(payload, 8 * cnt))
                v = [pool_bytes(tab[2 * j], tab[2 * j + 1]).decode("utf-8") for j in range(cnt)]
            else:
                raise MimError("bad-metadata", f"{key}: type {typ}")
            out[key] = (typ, v) if typed else v
        return out


def llama_config(f: MimFile) -> dict:
    """The dimensions of a llama- or qwen2-architecture file written by the
    reference's importer (metadata keys of importer/llama.go:104-162; the
    vocabulary from token_embd); "arch" names the architecture."""
    md = f.metadata()
    arch = md.get("general.architecture")
    if arch not in ("llama", "qwen2"):
        raise MimError("unsupported-dtype", f"architecture {arch!r} is not llama or qwen2")
    emb = f.tensors.get("token_embd.weight")
    if emb is None or len(emb.shape) != 2:
        raise MimError("not-found", "token_embd.weight")
    E = int(md[f"{arch}.embedding_length"])
    H = int(md[f"{arch}.attention.head_count"])
    cfg = dict(arch=arch, layers=int(md[f"{arch}.block_count"]), embed=E, ffn=int(md[f"{arch}.feed_forward_length"]),
               heads=H, kv_heads=int(md.get(f"{arch}.attention.head_count_kv", H)), head_dim=E // H,
               rope_dims=int(md.get(f"{arch}.rope.dimension_count", E // H)),
               rope_theta=float(md.get(f"{arch}.rope.freq_base", 10000.0)),
               norm_eps=float(md[f"{arch}.attention.layer_norm_rms_epsilon"]), vocab=int(emb.shape[0]),
               context=int(md.get("mim.context_length", md.get(f"{arch}.context_length", 4096))))
    return cfg
