"""Python binding of libmimgpu.so (include/mimgpu.h) through ctypes.

This is the host side that tests and bench.py drive.  It mirrors the
reference's operator interface: `Context.fast_paths` maps the same keys as
interp/fast.go:42-59 ("dequant_matmul.v1", "dequant_matmul_a8.v1", "dequant_matmul_a8.v2",
"rms_norm.v1", "rope.v1", "attention.v2", "swiglu.v1", "embedding.v1") to
callables taking (attrs, inputs) and returning (outputs, handled), raising
MimGPUError for the fast path's err.

There is no CPU fallback anywhere in this module: if the CUDA library is
missing or cannot be loaded, importing it raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmimgpu.so")

OK, ENOTHANDLED, EINVAL, ENOMEM, ECUDA, ENCCL, ETIMEOUT = range(7)
F32, F16, Q8_0, Q4_K, Q6_K = 1, 2, 64, 66, 67
BLOCK = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}

# Every symbol include/mimgpu.h declares, with (restype, argtypes).
P, I32, I64, D, SZ = C.c_void_p, C.c_int, C.c_int64, C.c_double, C.c_size_t
SIGNATURES = {
    "mimgpu_abi_version": (I32, []),
    "mimgpu_open": (I32, [I32, C.POINTER(P)]),
    "mimgpu_close": (None, [P]),
    "mimgpu_last_error": (C.c_char_p, [P]),
    "mimgpu_set_timeout_ms": (I32, [P, I64]),
    "mimgpu_stream_wait_value": (I32, [P, P, P, C.c_uint32]),
    "mimgpu_upload": (I32, [P, I32, I32, P, P, SZ, C.POINTER(P)]),
    "mimgpu_tensor_free": (None, [P]),
    "mimgpu_tensor_device_ptr": (P, [P]),
    "mimgpu_dequantize": (I32, [P, I32, P, SZ, P, I64]),
    "mimgpu_dequant_matmul": (I32, [P, P, I64, I64, P, P, P]),
    "mimgpu_dequant_matmul_a8": (I32, [P, I32, P, I64, I64, P, P, P]),
    "mimgpu_rms_norm": (I32, [P, P, I64, I64, P, D, P]),
    "mimgpu_rope": (I32, [P, P, I32, I32, I32, I32, P, I32, D, I32, I32, P]),
    "mimgpu_attention": (I32, [P, P, I32, I32, I32, I32, P, P, I32, I32, I32, P, P, D, I32, P]),
    "mimgpu_swiglu": (I32, [P, P, P, I64, P]),
    "mimgpu_embedding": (I32, [P, P, P, I64, P]),
    "mimgpu_dequant_matmul_a8_dev": (I32, [P, P, P, I64, I64, P, P, P]),
    "mimgpu_dequant_matmul_a8_block_dev": (I32, [P, P, I32, P, I64, I64, P, P, P]),
    "mimgpu_dequant_matmul_dev": (I32, [P, P, P, I64, I64, P, P, P]),
    "mimgpu_dequant_matmul_a8_static": (I32, [P, P, P, I64, I64, P, P, P]),
    "mimgpu_q8_new": (I32, [P, I64, I64, C.POINTER(P)]),
    "mimgpu_q8_free": (None, [P]),
    "mimgpu_q8_quantize_dev": (I32, [P, P, P, P]),
    "mimgpu_gemv_q8_dev": (I32, [P, P, P, P, P, P, P]),
    "mimgpu_gemv_q8_fused_dev": (I32, [P, P, P, P, I32, P, P]),
    "mimgpu_synth_tensor": (I32, [P, I32, C.c_uint64, I32, P, C.c_float, C.c_float, C.POINTER(P)]),
    "mimgpu_synth_rows": (I32, [P, I32, C.c_uint64, I32, P, I64, C.c_float, C.c_float, C.POINTER(P)]),
    "mimgpu_tensor_download": (I32, [P, P, SZ]),
    "mimgpu_tensor_nbytes": (SZ, [P]),
    "mimgpu_model_new": (I32, [P, P, C.POINTER(P)]),
    "mimgpu_model_set_weight": (I32, [P, C.c_char_p, P]),
    "mimgpu_model_free": (None, [P]),
    "mimgpu_session_new": (I32, [P, C.POINTER(P)]),
    "mimgpu_session_free": (None, [P]),
    "mimgpu_session_reset": (I32, [P]),
    "mimgpu_session_run": (I32, [P, P, P, I32, P, I32]),
    "mimgpu_session_generate": (I32, [P, I32, I64, I32, P]),
    "mimgpu_session_new_slots": (I32, [P, I32, C.POINTER(P)]),
    "mimgpu_session_run_slots": (I32, [P, P, P, P, I32, P]),
    "mimgpu_session_generate_slots": (I32, [P, P, P, I32, I32, P]),
    "mimgpu_session_stream": (P, [P]),
    "mimgpu_session_set_step_kernel": (I32, [P, I32]),
    "mimgpu_session_uses_step_kernel": (I32, [P]),
    "mimgpu_session_set_l2_prefetch": (I32, [P, I64]),
    "mimgpu_session_set_l2_prefetch_for": (I32, [P, I32, I32, I64]),
    "mimgpu_session_set_fusions": (I32, [P, C.c_uint]),
    "mimgpu_session_step_kernels": (I32, [P]),
    "mimgpu_session_trace_bytes": (SZ, [P]),
    "mimgpu_session_set_trace": (I32, [P, P, SZ]),
    "mimgpu_tp_unique_id": (I32, [P, SZ]),
    "mimgpu_tp_new": (I32, [P, P, SZ, I32, I32, C.POINTER(P)]),
    "mimgpu_tp_free": (None, [P]),
    "mimgpu_model_set_tp": (I32, [P, P]),
    "mimgpu_session_ipc_handle": (I32, [P, P, SZ]),
    "mimgpu_session_set_peers": (I32, [P, P, SZ, I32]),
}


class MimGPUError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"mimgpu error {code}: {msg}")
        self.code = code


_lib = None


def lib():
    """Loads libmimgpu.so; raises if it is missing (no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run mimir-model_b200/build.py (nvcc, sm_100a)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, np.float32)


class LlamaConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("layers", "embed", "ffn", "heads", "kv_heads", "head_dim", "rope_dims",
                                       "vocab", "context")] + [("rope_theta", C.c_double), ("norm_eps", C.c_double)] + \
               [(n, C.c_int) for n in ("a8", "cache_f16", "interleaved", "max_tokens")]


class Tensor:
    """A weight uploaded byte for byte into HBM (mimgpu_upload)."""

    def __init__(self, ctx: "Context", handle, dtype: int, shape):
        self.ctx, self.h, self.dtype, self.shape = ctx, handle, dtype, tuple(shape)

    @property
    def device_ptr(self) -> int:
        return lib().mimgpu_tensor_device_ptr(self.h)

    def free(self):
        if self.h:
            lib().mimgpu_tensor_free(self.h)
            self.h = None


class Context:
    def __init__(self, device: int = 0):
        h = P()
        rc = lib().mimgpu_open(device, C.byref(h))
        if rc != OK:
            raise MimGPUError(rc, f"cannot open CUDA device {device}")
        self.h = h
        self._tensors = []
        self.fast_paths = {
            "dequant_matmul.v1": self._fp_dequant_matmul,
            "dequant_matmul_a8.v1": self._fp_dequant_matmul_a8_v1,
            "dequant_matmul_a8.v2": self._fp_dequant_matmul_a8,
            "rms_norm.v1": self._fp_rms_norm,
            "rope.v1": self._fp_rope,
            "attention.v1": self._fp_attention,
            "attention.v2": self._fp_attention,
            "swiglu.v1": self._fp_swiglu,
            "embedding.v1": self._fp_embedding,
        }

    def close(self):
        for t in self._tensors:
            t.free()
        self._tensors = []
        if self.h:
            lib().mimgpu_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def _check(self, rc: int):
        if rc != OK:
            raise MimGPUError(rc, lib().mimgpu_last_error(self.h).decode())

    def call(self, rc: int) -> int:
        """Returns rc for OK/ENOTHANDLED, raises otherwise."""
        if rc not in (OK, ENOTHANDLED):
            self._check(rc)
        return rc

    def set_timeout_ms(self, ms: int):
        self._check(lib().mimgpu_set_timeout_ms(self.h, ms))

    # ---- weights
    def upload(self, dtype: int, shape, data) -> Tensor:
        raw = np.ascontiguousarray(data).view(np.uint8).ravel()
        shp = np.array(shape, np.int64)
        h = P()
        self._check(lib().mimgpu_upload(self.h, dtype, len(shape), _p(shp), _p(raw), raw.size, C.byref(h)))
        t = Tensor(self, h, dtype, shape)
        self._tensors.append(t)
        return t

    def synth(self, dtype: int, shape, seed: int, mean: float = 0.0, sigma: float = 0.02) -> Tensor:
        """Seeded random-init weights made on the device (benchmark inputs)."""
        shp = np.array(shape, np.int64)
        h = P()
        self._check(lib().mimgpu_synth_tensor(self.h, dtype, seed, len(shape), _p(shp), mean, sigma, C.byref(h)))
        t = Tensor(self, h, dtype, shape)
        self._tensors.append(t)
        return t

    def synth_rows(self, dtype: int, shape, row0: int, seed: int, mean: float = 0.0, sigma: float = 0.02) -> Tensor:
        """Rows [row0, row0 + shape[0]) of synth(dtype, full shape, seed): a shard."""
        shp = np.array(shape, np.int64)
        h = P()
        self._check(lib().mimgpu_synth_rows(self.h, dtype, seed, len(shape), _p(shp), row0, mean, sigma, C.byref(h)))
        t = Tensor(self, h, dtype, shape)
        self._tensors.append(t)
        return t

    def download(self, t: Tensor) -> np.ndarray:
        out = np.empty(lib().mimgpu_tensor_nbytes(t.h), np.uint8)
        self._check(lib().mimgpu_tensor_download(t.h, _p(out), out.size))
        return out

    # ---- per-op calls (host buffers)
    def dequantize(self, dtype: int, raw, n: int) -> np.ndarray:
        raw = np.ascontiguousarray(raw).view(np.uint8).ravel()
        out = np.empty(n, np.float32)
        self._check(lib().mimgpu_dequantize(self.h, dtype, _p(raw), raw.size, _p(out), n))
        return out

    def dequant_matmul(self, x, w: Tensor, bias=None, a8_block: int | None = None) -> np.ndarray:
        x = _f32(x)
        k = x.shape[-1]
        rows = x.size // k if k else 0
        y = np.empty(x.shape[:-1] + (w.shape[0],), np.float32)
        b = _f32(bias)
        if a8_block is None:
            rc = lib().mimgpu_dequant_matmul(self.h, _p(x), rows, k, w.h, _p(b), _p(y))
        else:
            rc = lib().mimgpu_dequant_matmul_a8(self.h, a8_block, _p(x), rows, k, w.h, _p(b), _p(y))
        self._check(rc)
        return y

    def rms_norm(self, x, scale, eps: float) -> np.ndarray:
        x = _f32(x)
        n = x.shape[-1]
        y = np.empty_like(x)
        self._check(lib().mimgpu_rms_norm(self.h, _p(x), x.size // n if n else 0, n, _p(_f32(scale)), eps, _p(y)))
        return y

    def rope(self, x, pos, theta: float, rotary: int | None = None, interleaved: bool = False) -> np.ndarray:
        x = _f32(x)
        B, H, T, Dd = x.shape
        pos = np.ascontiguousarray(pos, np.int64)
        y = np.empty_like(x)
        rc = lib().mimgpu_rope(self.h, _p(x), B, H, T, Dd, _p(pos), pos.shape[0], theta, rotary or Dd,
                               int(interleaved), _p(y))
        if self.call(rc) == ENOTHANDLED:
            return None
        return y

    def attention(self, q, k, v, mask=None, scale: float = 0.0, causal: bool = False) -> np.ndarray:
        q = _f32(q)
        B, Hq, Tq, Dd = q.shape
        kvdt = F16 if k.dtype == np.float16 else F32
        k, v = np.ascontiguousarray(k), np.ascontiguousarray(v)
        out = np.empty_like(q)
        ms = None
        if mask is not None:
            mask = np.ascontiguousarray(mask, np.uint8)
            ms = np.array(mask.shape, np.int32)
        rc = lib().mimgpu_attention(self.h, _p(q), B, Hq, Tq, Dd, _p(k), _p(v), kvdt, k.shape[1], k.shape[2],
                                    _p(mask), _p(ms), scale, int(causal), _p(out))
        if self.call(rc) == ENOTHANDLED:
            return None
        return out

    def swiglu(self, a, b) -> np.ndarray:
        a, b = _f32(a), _f32(b)
        y = np.empty_like(a)
        self._check(lib().mimgpu_swiglu(self.h, _p(a), _p(b), a.size, _p(y)))
        return y

    def embedding(self, table: Tensor, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        y = np.empty(ids.shape + (table.shape[1],), np.float32)
        self._check(lib().mimgpu_embedding(self.h, table.h, _p(ids), ids.size, _p(y)))
        return y

    # ---- fastFunc-shaped adapters: (attrs, inputs) -> (outputs, handled)
    def _fp_dequant_matmul(self, attrs, ins):
        x, w = ins[0], ins[1]
        return [self.dequant_matmul(x, w, ins[2] if len(ins) > 2 else None)], True

    def _fp_dequant_matmul_a8_v1(self, attrs, ins):
        # fastDequantMatmulA8 (interp/fast.go:225-230): no attributes, blocks of 32
        if attrs:
            return None, False
        x, w = ins[0], ins[1]
        return [self.dequant_matmul(x, w, ins[2] if len(ins) > 2 else None, a8_block=32)], True

    def _fp_dequant_matmul_a8(self, attrs, ins):
        x, w = ins[0], ins[1]
        return [self.dequant_matmul(x, w, ins[2] if len(ins) > 2 else None, a8_block=attrs.get("block", 32))], True

    def _fp_rms_norm(self, attrs, ins):
        if attrs.get("axis", -1) not in (-1, ins[0].ndim - 1):
            return None, False
        return [self.rms_norm(ins[0], ins[1] if len(ins) > 1 else None, attrs.get("epsilon", 1e-6))], True

    def _fp_rope(self, attrs, ins):
        if attrs.get("yarn_factor", 1.0) != 1.0:
            return None, False
        y = self.rope(ins[0], ins[1], attrs.get("theta", 10000.0), attrs.get("rotary_dims"),
                      bool(attrs.get("interleaved", False)))
        return ([y], True) if y is not None else (None, False)

    def _fp_attention(self, attrs, ins):
        if attrs.get("softcap", 0) > 0:
            return None, False
        mask = ins[3] if len(ins) > 3 else None
        if mask is not None and mask.dtype != np.bool_:
            return None, False
        y = self.attention(ins[0], ins[1], ins[2], mask, attrs.get("scale", 0.0), attrs.get("causal", False))
        return ([y], True) if y is not None else (None, False)

    def _fp_swiglu(self, attrs, ins):
        return [self.swiglu(ins[0], ins[1])], True

    def _fp_embedding(self, attrs, ins):
        return [self.embedding(ins[0], ins[1])], True


TP_ID_BYTES = 128  # NCCL_UNIQUE_ID_BYTES


def tp_unique_id() -> bytes:
    """A fresh tensor-parallel group id (made by rank 0, handed to the others)."""
    buf = C.create_string_buffer(TP_ID_BYTES)
    rc = lib().mimgpu_tp_unique_id(buf, TP_ID_BYTES)
    if rc != OK:
        raise MimGPUError(rc, "cannot make an NCCL group id")
    return buf.raw


class TensorParallel:
    """One rank of a tensor-parallel group (an NCCL communicator over the
    GPUs of one node).  Every rank binds it to its model with
    Model.set_tp before creating sessions."""

    def __init__(self, ctx: "Context", group_id: bytes, nranks: int, rank: int):
        h = P()
        ctx._check(lib().mimgpu_tp_new(ctx.h, group_id, len(group_id), nranks, rank, C.byref(h)))
        self.ctx, self.h, self.nranks, self.rank = ctx, h, nranks, rank

    def free(self):
        if self.h:
            lib().mimgpu_tp_free(self.h)
            self.h = None


def tp_rows(n: int, nranks: int, rank: int) -> tuple:
    """Rows [r0, r1) of an n-row matrix that a rank computes: equal slices
    (the vocabulary's last slice may be short)."""
    per = (n + nranks - 1) // nranks
    r0 = min(n, rank * per)
    return r0, min(n, r0 + per)


def load_llama(ctx: "Context", path: str, *, a8: bool = True, cache_f16: bool = True, max_tokens: int = 1,
               context: int | None = None) -> "Model":
    """A Llama mim file written by the reference's importer (importer/llama.go:
    tensors under their GGUF names, the dimensions in the metadata) as a
    device-resident model.  The file's graph section is not interpreted:
    the model runs the same Llama step as Model(ctx, cfg, weights), with
    8-bit activations (a8, dequant_matmul_a8.v2) or exact f32 products and an
    f16 or f32 key-value cache as asked.  Weight bytes go from the mapped
    file to HBM byte for byte."""
    try:
        from . import mimfile  # type: ignore
    except ImportError:
        import mimfile  # type: ignore
    with mimfile.MimFile(path) as f:
        cfg = mimfile.llama_config(f)
        if context:
            cfg["context"] = int(context)
        # llama rotates adjacent pairs, qwen2 the two halves of each head
        cfg.update(a8=int(a8), cache_f16=int(cache_f16), interleaved=int(cfg["arch"] == "llama"),
                   max_tokens=int(max_tokens))
        names = [n for n in f.tensors if n in ("token_embd.weight", "output.weight", "output_norm.weight")
                 or (n.startswith("blk.") and (n.endswith(".weight") or n.endswith(("attn_q.bias", "attn_k.bias",
                                                                                   "attn_v.bias"))))]
        # each tensor with the file's own shape (the model checks it against the dimensions)
        weights = {n: (f.tensors[n].dtype, ctx.upload(f.tensors[n].dtype, f.tensors[n].shape,
                                                      np.frombuffer(f.data(n), np.uint8))) for n in names}
        return Model(ctx, cfg, weights)


class Model:
    """The llama graph (importer/llama.go:317-547) as a device-resident decoder."""

    def __init__(self, ctx: Context, cfg: dict, weights: dict):
        c = LlamaConfig(**{k: int(cfg[k]) if k not in ("rope_theta", "norm_eps") else float(cfg[k])
                           for k, _ in LlamaConfig._fields_ if k in cfg})
        if c.max_tokens <= 0:
            c.max_tokens = 1
        self.ctx, self.vocab = ctx, c.vocab
        h = P()
        ctx._check(lib().mimgpu_model_new(ctx.h, C.byref(c), C.byref(h)))
        self.h = h
        self.weights = {}
        for name, (dt, arr) in weights.items():
            t = arr if isinstance(arr, Tensor) else ctx.upload(dt, _shape_of(name, cfg, dt, arr), arr)
            self.weights[name] = t
            ctx._check(lib().mimgpu_model_set_weight(h, name.encode(), t.h))

    def set_tp(self, tp: "TensorParallel | None"):
        """Binds a tensor-parallel group (before the first session)."""
        self.ctx._check(lib().mimgpu_model_set_tp(self.h, tp.h if tp is not None else None))
        self.tp = tp

    def session(self, slots: int = 1) -> "Session":
        """A session of `slots` independent sequences (batched decoding)."""
        h = P()
        self.ctx._check(lib().mimgpu_session_new_slots(self.h, int(slots), C.byref(h)))
        return Session(self, h)

    def free(self):
        if self.h:
            lib().mimgpu_model_free(self.h)
            self.h = None


def _shape_of(name: str, cfg: dict, dt: int, arr) -> tuple:
    E, F, V = cfg["embed"], cfg["ffn"], cfg["vocab"]
    kv = cfg["kv_heads"] * cfg["head_dim"]
    base = name.split(".", 2)[-1] if name.startswith("blk.") else name
    return {
        "token_embd.weight": (V, E), "output.weight": (V, E), "output_norm.weight": (E,),
        "attn_norm.weight": (E,), "ffn_norm.weight": (E,), "attn_q.weight": (E, E), "attn_k.weight": (kv, E),
        "attn_v.weight": (kv, E), "attn_output.weight": (E, E), "ffn_gate.weight": (F, E),
        "ffn_up.weight": (F, E), "ffn_down.weight": (E, F),
        "attn_q.bias": (E,), "attn_k.bias": (kv,), "attn_v.bias": (kv,),
    }[base]


class Session:
    def __init__(self, model: Model, h):
        self.m, self.h = model, h

    def reset(self):
        self.m.ctx._check(lib().mimgpu_session_reset(self.h))

    def run(self, tokens, positions, all_rows: bool = False) -> np.ndarray:
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(positions, np.int64)
        out = np.empty((t.size if all_rows else 1, self.m.vocab), np.float32)
        self.m.ctx._check(lib().mimgpu_session_run(self.h, _p(t), _p(p), t.size, _p(out), int(all_rows)))
        return out

    def ipc_handle(self) -> bytes:
        """This session's device arena as a CUDA IPC handle (tensor parallelism)."""
        buf = C.create_string_buffer(64)
        self.m.ctx._check(lib().mimgpu_session_ipc_handle(self.h, buf, 64))
        return buf.raw

    def set_peers(self, handles: list):
        """Maps every rank's arena (handles in rank order, this rank's included)
        so that decode steps exchange over peer memory."""
        blob = b"".join(handles)
        self.m.ctx._check(lib().mimgpu_session_set_peers(self.h, blob, 64, len(handles)))

    def run_slots(self, tokens, slots, positions) -> np.ndarray:
        """One run of rows of given sequences (mimgpu_session_run_slots): logits [rows, vocab]."""
        t = np.ascontiguousarray(tokens, np.int32)
        sl = np.ascontiguousarray(slots, np.int32)
        p = np.ascontiguousarray(positions, np.int64)
        out = np.empty((t.size, self.m.vocab), np.float32)
        self.m.ctx._check(lib().mimgpu_session_run_slots(self.h, _p(t), _p(sl), _p(p), t.size, _p(out)))
        return out

    def generate_slots(self, tokens, positions, steps: int) -> np.ndarray:
        """Greedy decode of sequences 0..len(tokens)-1 together: ids [steps, B]."""
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(positions, np.int64)
        ids = np.empty((steps, t.size), np.int32)
        self.m.ctx._check(lib().mimgpu_session_generate_slots(self.h, _p(t), _p(p), t.size, steps, _p(ids)))
        return ids

    def generate(self, token: int, pos: int, steps: int) -> np.ndarray:
        ids = np.empty(steps, np.int32)
        self.m.ctx._check(lib().mimgpu_session_generate(self.h, token, pos, steps, _p(ids)))
        return ids

    def set_step_kernel(self, on: bool):
        """One persistent kernel per decode step (opt-in, where the model
        qualifies) or the kernel-per-op path (the default); same bits."""
        self.m.ctx._check(lib().mimgpu_session_set_step_kernel(self.h, int(on)))

    def trace_bytes(self) -> int:
        return lib().mimgpu_session_trace_bytes(self.h)

    def set_trace(self, dev_ptr: int | None, nbytes: int = 0):
        """Binds a device buffer for the step kernel's phase timeline (profiling)."""
        self.m.ctx._check(lib().mimgpu_session_set_trace(self.h, dev_ptr, nbytes))

    @property
    def step_kernels(self) -> int:
        """Kernel launches per captured greedy decode step (0 before capture)."""
        return int(lib().mimgpu_session_step_kernels(self.h))

    def set_l2_prefetch(self, bytes_per_sm: int):
        """L2 prefetch of the next decode GEMV's weights (0 = off)."""
        self.m.ctx._check(lib().mimgpu_session_set_l2_prefetch(self.h, int(bytes_per_sm)))

    def set_fusions(self, norm: bool = True):
        """rms_norm of one-token steps inside the GEMVs that read it, or as a
        kernel of its own; the results are the same bits either way."""
        self.m.ctx._check(lib().mimgpu_session_set_fusions(self.h, 1 if norm else 0))

    def set_l2_prefetch_for(self, kind: int, distance: int, bytes_per_sm: int):
        """L2 prefetch of decode GEMV `kind` (0 q|k|v, 1 o, 2 gate|up, 3 down,
        4 head) by the GEMV `distance` (1 or 2) launches before it."""
        self.m.ctx._check(lib().mimgpu_session_set_l2_prefetch_for(self.h, int(kind), int(distance),
                                                                   int(bytes_per_sm)))

    @property
    def uses_step_kernel(self) -> bool:
        return bool(lib().mimgpu_session_uses_step_kernel(self.h))

    @property
    def stream(self) -> int:
        return lib().mimgpu_session_stream(self.h)

    def run_ptr(self, tok_ptr: int, pos_ptr: int, t: int, logits_ptr: int, all_rows: bool = False):
        """session_run on caller-owned host buffers (e.g. pinned memory)."""
        self.m.ctx._check(lib().mimgpu_session_run(self.h, tok_ptr, pos_ptr, t, logits_ptr, int(all_rows)))

    def free(self):
        if self.h:
            lib().mimgpu_session_free(self.h)
            self.h = None
