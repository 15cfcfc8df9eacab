#!/usr/bin/env python
"""Benchmark of the B200 decode hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mimgpu|reference]

Workload: the 8B-shape Q4_K_M llama decoder (32 layers, d_model 4096, 32/8
heads of 128, SwiGLU 14336, vocab 128256, RMSNorm eps 1e-5, RoPE theta
500000), random-init weights from seeded N(0, 0.02) (Q6_K for attn_v,
ffn_down and output, Q4_K elsewhere; f32 norms N(1, 0.02)), made on the
device.  A prompt of 128 seeded random ids is prefilled, then each timed
step is one greedy decode token at batch 1 through dequant_matmul_a8.v2
(block 256) and an f16 key-value cache.

Prints one JSON line: `value` is decode tok/s timed on the device with CUDA
events (weights and cache resident in HBM; 4.88 GB of weights stream per
token, far above the 126 MB L2, so no flush is needed); `e2e` is the same
rate through mimgpu_session_run with the token id and position copied in
from pinned host memory and the logits copied back every step;
`roofline` is the GEMV kernel alone over the real decode shapes.
--impl reference times the CPU restatement of the reference (oracle/) on
all host cores instead.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mimir-model_b200"))

METRIC = "Q4_K_M decode tok/s (8B, 70B TP 1–8 GPU); quant-GEMV HBM GB/s vs peak"
PUBLISHED_8B = 6.7  # the reference's published 8B-shape Q4_K_M decode (random weights, 4-core Xeon)
F32, Q4_K, Q6_K = 1, 66, 67
CFG8B = dict(layers=32, embed=4096, ffn=14336, heads=32, kv_heads=8, head_dim=128, rope_dims=128, vocab=128256,
             rope_theta=500000.0, norm_eps=1e-5)
CFG70B = dict(layers=80, embed=8192, ffn=28672, heads=64, kv_heads=8, head_dim=128, rope_dims=128, vocab=128256,
              rope_theta=500000.0, norm_eps=1e-5)
SHAPES = {"8b": CFG8B, "70b": CFG70B}
PROMPT = 128
GEMV_TRAFFIC_PER_ALGO_BYTE = (66_120_960 + 338_944) / 66_179_904
# DRAM bytes per algorithmic byte of step_kernel from one ncu capture of the
# same command (profiles/), or None until one exists
STEP_TRAFFIC_PER_ALGO_BYTE = None


def layout(cfg):
    """(name, dtype, shape, mean, sigma) of every weight, Q4_K_M."""
    E, F, V, KV = cfg["embed"], cfg["ffn"], cfg["vocab"], cfg["kv_heads"] * cfg["head_dim"]
    out = [("token_embd.weight", Q4_K, (V, E), 0.0, 0.02)]
    for l in range(cfg["layers"]):
        p = f"blk.{l}."
        out += [(p + "attn_norm.weight", F32, (E,), 1.0, 0.02), (p + "attn_q.weight", Q4_K, (E, E), 0.0, 0.02),
                (p + "attn_k.weight", Q4_K, (KV, E), 0.0, 0.02), (p + "attn_v.weight", Q6_K, (KV, E), 0.0, 0.02),
                (p + "attn_output.weight", Q4_K, (E, E), 0.0, 0.02), (p + "ffn_norm.weight", F32, (E,), 1.0, 0.02),
                (p + "ffn_gate.weight", Q4_K, (F, E), 0.0, 0.02), (p + "ffn_up.weight", Q4_K, (F, E), 0.0, 0.02),
                (p + "ffn_down.weight", Q6_K, (E, F), 0.0, 0.02)]
    out += [("output_norm.weight", F32, (E,), 1.0, 0.02), ("output.weight", Q6_K, (V, E), 0.0, 0.02)]
    return out


def nbytes(dt, shape):
    n = int(np.prod(shape))
    return n * 4 if dt == F32 else n // 256 * (144 if dt == Q4_K else 210)


def weight_bytes_per_token(cfg):
    """Algorithmic bytes per decode token: every weight once, one embedding row."""
    tot = 0
    for name, dt, shape, _, _ in layout(cfg):
        tot += nbytes(dt, shape[1:]) if name == "token_embd.weight" else nbytes(dt, shape)
    return tot


def l2_note(cfg, what: str) -> str:
    """The L2 statement of a bench line, with this shape's weight bytes."""
    return f"inputs larger than L2: {weight_bytes_per_token(cfg) / 1e9:.2f} GB of weights {what} vs 126 MB L2"


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def seed_of(name: str) -> int:
    h = 1469598103934665603
    for ch in name.encode():
        h = ((h ^ ch) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def prompt_ids(vocab, n=PROMPT, seed=20261201):
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.int32)


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device, self.p, self.lines = device, None, []

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "100", "-i", str(self.device)], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.p:
            time.sleep(0.2)
            self.p.terminate()
            out, _ = self.p.communicate(timeout=5)
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


# ----------------------------------------------------------------- GPU arm

def shard_rows(name, cfg, nranks, rank):
    """(first row, rows) of a weight a tensor-parallel rank holds: its rows of
    every split matrix, or the whole tensor (norms, the embedding table)."""
    E, F, V, KV = cfg["embed"], cfg["ffn"], cfg["vocab"], cfg["kv_heads"] * cfg["head_dim"]
    base = name.split(".", 2)[-1] if name.startswith("blk.") else name
    full = {"attn_q.weight": E, "attn_output.weight": E, "ffn_down.weight": E, "attn_k.weight": KV,
            "attn_v.weight": KV, "ffn_gate.weight": F, "ffn_up.weight": F, "output.weight": V}.get(base)
    if full is None or nranks == 1:
        return None
    per = (full + nranks - 1) // nranks
    r0 = min(full, rank * per)
    return r0, min(full, r0 + per) - r0


def build_model(ctx, cfg, context, max_tokens, tp=None):
    """The benchmark model, weights made on the device; tp = (ranks, rank)
    makes only this rank's rows of every split matrix (byte-identical to the
    same rows of the whole tensor)."""
    import mimgpu
    weights = {}
    for name, dt, shape, mean, sigma in layout(cfg):
        sh = shard_rows(name, cfg, *tp) if tp else None
        if sh:
            r0, rows = sh
            weights[name] = (dt, ctx.synth_rows(dt, (rows,) + tuple(shape[1:]), r0, seed_of(name), mean, sigma))
        else:
            weights[name] = (dt, ctx.synth(dt, shape, seed_of(name), mean, sigma))
    full = dict(cfg, context=context, a8=1, cache_f16=1, interleaved=1, max_tokens=max_tokens)
    return mimgpu.Model(ctx, full, weights), weights


def write_mim(ctx, cfg, weights, path, context):
    """The benchmark model as a mim file: every tensor under its GGUF name,
    the Llama hyperparameters as a GGUF carries them, and the reference
    importer's forward graph with dequant_matmul_a8.v2 products and an f16
    cache (mimwriter.write_llama), so the reference's interpreter and
    mimgpu.load_llama both run it.  Each tensor is read back from the device
    when the file is written.  Returns the file's size in bytes."""
    import mimwriter
    tensors = {name: (dt, t.shape, (lambda t=t: ctx.download(t).tobytes())) for name, (dt, t) in weights.items()}
    md = mimwriter.llama_metadata(dict(cfg, context=context), name=f"synthetic {cfg['layers']}-layer Q4_K_M "
                                  f"(seeded N(0,0.02) weights)")
    mimwriter.write_llama(path, cfg, tensors, a8=True, cache_f16=True, context=context, metadata=md)
    return os.path.getsize(path)


def gemv_roofline(ctx, cfg, weights, torch, reps=3):
    """The one-row GEMV alone over the decode step's own launch list -- per
    layer q|k|v (one fused launch), o, gate|up (one fused launch), down, then
    the head -- captured back to back in one CUDA graph (cold L2: each launch
    reads different weights) and timed with CUDA events on the launching
    stream around each replay.  Returns (bytes per launch, seconds per
    launch, launches)."""
    import mimgpu
    lib = mimgpu.lib()
    E, F = cfg["embed"], cfg["ffn"]
    st = torch.cuda.Stream()
    x_e = torch.randn(E, device="cuda", dtype=torch.float32)
    x_f = torch.randn(F, device="cuda", dtype=torch.float32)
    q8e, q8f = C.c_void_p(), C.c_void_p()
    ctx._check(lib.mimgpu_q8_new(ctx.h, 1, E, C.byref(q8e)))
    ctx._check(lib.mimgpu_q8_new(ctx.h, 1, F, C.byref(q8f)))
    ctx._check(lib.mimgpu_q8_quantize_dev(ctx.h, st.cuda_stream, x_e.data_ptr(), q8e))
    ctx._check(lib.mimgpu_q8_quantize_dev(ctx.h, st.cuda_stream, x_f.data_ptr(), q8f))
    y = torch.empty(4, max(cfg["vocab"], 2 * F), device="cuda", dtype=torch.float32)
    plan = []
    for l in range(cfg["layers"]):
        w = lambda n: weights[f"blk.{l}.{n}.weight"][1]
        plan.append(([w("attn_q"), w("attn_k"), w("attn_v")], q8e, x_e, E))
        plan.append(([w("attn_output")], q8e, x_e, E))
        plan.append(([w("ffn_gate"), w("ffn_up")], q8e, x_e, E))
        plan.append(([w("ffn_down")], q8f, x_f, F))
    plan.append(([weights["output.weight"][1]], q8e, x_e, E))
    args = []
    for ts, q8, x, K in plan:
        tarr = (C.c_void_p * len(ts))(*[t.h.value for t in ts])
        yarr = (C.c_void_p * len(ts))(*[y[i].data_ptr() for i in range(len(ts))])
        args.append((q8, x, len(ts), tarr, yarr))
    torch.cuda.synchronize()

    def enqueue():
        for q8, x, n, tarr, yarr in args:
            ctx._check(lib.mimgpu_gemv_q8_fused_dev(ctx.h, st.cuda_stream, q8, x.data_ptr(), n, tarr, yarr))

    with torch.cuda.stream(st):
        enqueue()  # warm-up: kernel attributes, tensor maps
    st.synchronize()
    # the launches back to back in one CUDA graph, so that host submission
    # does not gap them; one event pair around each replay
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st, capture_error_mode="thread_local"):
        enqueue()
    total_t = 0.0
    with torch.cuda.stream(st):
        g.replay()  # warm-up replay
        for rep in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            g.replay()
            b.record(st)
            b.synchronize()
            total_t += a.elapsed_time(b) / 1e3
    del g
    total_b, launches = 0, 0
    for ts, q8, x, K in plan:
        n = sum(t.shape[0] for t in ts)
        total_b += reps * (sum(nbytes(t.dtype, t.shape) for t in ts) + K + K // 256 * 4 + K // 32 * 2 + K // 16 * 2
                           + 4 * n)
        launches += reps
    lib.mimgpu_q8_free(q8e)
    lib.mimgpu_q8_free(q8f)
    return total_b / launches, total_t / launches, launches


PORT_NOTE = ("oracle/ C restatement of the reference's a8 decode path (gcc -O3 -march=x86-64-v3; the block sums of "
             "dotQ8KRef in AVX2 as the reference's dotQ4KQ8KAVX2/dotQ6KQ8KAVX2 compute them, bit-identical to the scalar "
             "checker; quantizer, attention and the f32 steps scalar C; a persistent worker pool over output rows)")


def cpu_baseline_sample(ctx, cfg, weights, prompt, budget_s=20.0):
    """The CPU restatement (oracle/, timed here as the reference's CPU path)
    on the same weights and the same prompt: decode steps until the budget."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    host = {name: (dt, ctx.download(t)) for name, (dt, t) in weights.items()}
    m = O.Llama(dict(cfg, context=prompt + 40, a8=1, cache_f16=1, interleaved=1, nthreads=O.threads()), host)
    ids = prompt_ids(cfg["vocab"], prompt)
    logits = m.forward(ids, np.arange(prompt))[0]
    tok, pos, steps, t0 = O.argmax(logits), prompt, 0, time.perf_counter()
    while True:
        logits = m.forward([tok], [pos])[0]
        tok, pos, steps = O.argmax(logits), pos + 1, steps + 1
        el = time.perf_counter() - t0
        if el > budget_s or steps >= 32:
            break
    del m, host
    return {"value": steps / el, "unit": "tok/s", "cores": O.threads(), "cpu": cpu_model(), "kind": "port",
            "sample": f"{steps} greedy decode tokens of the same model after the same {prompt}-token prompt, "
                      f"{el:.1f} s, all threads; {PORT_NOTE}"}


def run_gpu(args):
    import torch
    import mimgpu
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    cfg = dict(SHAPES[args.shape], layers=args.layers)
    prompt = args.prompt
    context = prompt + args.warmup + args.steps + 2 * args.e2e_steps + 8
    ctx = mimgpu.Context(local)
    # N > 1: tensor parallelism (one sequence over all ranks) for the 70B shape
    # or with --tp; otherwise N independent replicas, one sequence per GPU
    use_tp = world > 1 and (args.tp or args.shape == "70b")
    # a tensor-parallel rank makes and holds only its own rows of every split matrix
    if args.mim:
        if use_tp:
            raise SystemExit("--mim runs one GPU or replicas, not tensor parallelism")
        # the model from a mim file (written by --write-mim, or by the reference's importer)
        model = mimgpu.load_llama(ctx, args.mim, max_tokens=prompt, context=context)
        weights = {n: (t.dtype, t) for n, t in model.weights.items()}
    else:
        model, weights = build_model(ctx, cfg, context, prompt, (world, rank) if use_tp else None)
    tp = None
    if use_tp:
        # each rank computes its output rows of every matrix, bit-identical to one GPU
        gid = [mimgpu.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(gid, src=0)
        tp = mimgpu.TensorParallel(ctx, gid[0], world, rank)
        model.set_tp(tp)
    sess = model.session()
    if use_tp and args.p2p:
        # map every rank's arena: decode steps exchange over peer memory
        hs = [None] * world
        dist.all_gather_object(hs, sess.ipc_handle())
        sess.set_peers(hs)
    replicas = world if world > 1 and not use_tp else 1
    # replicas decode different sequences (a prompt of their own)
    ids = prompt_ids(cfg["vocab"], prompt, seed=20261201 + (rank if replicas > 1 else 0))
    logits = sess.run(ids, np.arange(prompt))[0]
    tok, pos = int(np.argmax(logits)), prompt
    # warm-up (also captures the decode graph)
    out = sess.generate(tok, pos, args.warmup)
    tok, pos = int(out[-1]), pos + args.warmup
    stream = torch.cuda.ExternalStream(sess.stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    with clocks:
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        out = sess.generate(tok, pos, args.steps)
        b.record(stream)
        torch.cuda.synchronize()
    dev_s = a.elapsed_time(b) / 1e3
    if dist:
        t = torch.tensor([dev_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_s = float(t.item())
    tok, pos = int(out[-1]), pos + args.steps
    # e2e through the public per-run call with pinned host buffers
    tok_h = torch.empty(1, dtype=torch.int32, pin_memory=True)
    pos_h = torch.empty(1, dtype=torch.int64, pin_memory=True)
    log_h = torch.empty(cfg["vocab"], dtype=torch.float32, pin_memory=True)
    log_np = log_h.numpy()
    for i in range(2):  # warm-up of the per-run path (graph capture)
        tok_h[0], pos_h[0] = tok, pos
        sess.run_ptr(tok_h.data_ptr(), pos_h.data_ptr(), 1, log_h.data_ptr())
        tok, pos = int(np.argmax(log_np)), pos + 1
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(args.e2e_steps):
        tok_h[0], pos_h[0] = tok, pos
        sess.run_ptr(tok_h.data_ptr(), pos_h.data_ptr(), 1, log_h.data_ptr())
        tok, pos = int(np.argmax(log_np)), pos + 1
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    wpt = weight_bytes_per_token(cfg)
    ms = dev_s / args.steps * 1e3
    value = replicas * args.steps / dev_s  # tokens of every sequence over the slowest rank's time
    peak, peak_kind = peaks()
    step_path = sess.uses_step_kernel
    if step_path:
        # the dominant kernel is the whole step: one step_kernel launch per token
        # (the one-thread advance kernel that follows it is inside the event
        # pair); algorithmic bytes = every weight once + the key/value rows read
        kv_avg = prompt + args.warmup + (args.steps + 1) / 2
        kv = 2 * cfg["layers"] * cfg["kv_heads"] * cfg["head_dim"] * 2 * kv_avg
        bpl, spl, nl = wpt + kv, dev_s / args.steps, args.steps
        kernel = "step_kernel (persistent decode step, k_step.cu; event time includes the advance kernel)"
        traffic = STEP_TRAFFIC_PER_ALGO_BYTE * bpl if STEP_TRAFFIC_PER_ALGO_BYTE else None
        launches = args.steps * 2
    else:
        # the kernel-per-op path: its dominant kernel, the one-row GEMV, alone over the decode shapes
        bpl, spl, nl = gemv_roofline(ctx, cfg, weights, torch)
        kernel = (f"gemv_row_kernel (one-row dequant_matmul_a8.v2 over the decode step's launch list: per layer "
                  f"q|k|v fused, o, gate|up fused, down; {cfg['layers']} layers + head)")
        traffic = GEMV_TRAFFIC_PER_ALGO_BYTE * bpl
        # the kernels of the captured one-token step, counted from its CUDA graph
        launches = args.steps * sess.step_kernels
    achieved = bpl / spl / 1e9
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "strong" if use_tp else "weak",
        "vs_baseline": round(value / PUBLISHED_8B, 2) if args.shape == "8b" else None, "dtype": "int8",
        "data": ("synthetic (seeded N(0,0.02) weights quantized Q4_K_M on the device; seeded random prompt ids)"
                 if not args.mim else f"weights from the mim file {os.path.basename(args.mim)}; seeded random prompt ids"),
        "config": {"workload": ("8B-shape Q4_K_M greedy decode, batch 1 (BASELINE config 3)" if args.shape == "8b"
                                else "70B-shape Q4_K_M greedy decode, batch 1 (BASELINE config 5)"),
                   "layers": cfg["layers"], "d_model": cfg["embed"], "heads": cfg["heads"],
                   "kv_heads": cfg["kv_heads"], "ffn": cfg["ffn"], "vocab": cfg["vocab"], "prompt": prompt,
                   "context_cache": context, "positions_timed": [prompt + args.warmup, pos - 1 - args.e2e_steps - 2],
                   "matmul": "dequant_matmul_a8.v2 block 256 (bit-exact dotQ8KRef)", "kv_cache": "f16",
                   "decode_path": ("one persistent step kernel per token" if step_path
                                   else f"CUDA graph of {sess.step_kernels} kernels per token (per layer: q|k|v "
                                        "GEMV with rms_norm, attention with RoPE and cache write, o GEMV, gate|up "
                                        "GEMV with rms_norm, SwiGLU, down GEMV; programmatic dependent launch)"),
                   "parallelism": (f"tp{world} (q|k|v by kv-head group, o / gate|up / down / head by output rows, "
                                   f"each rank holding its shard; attention, residual and SwiGLU exchanged by "
                                   f"{'peer-memory stores' if args.p2p else 'NCCL all-gathers'})") if use_tp
                   else (f"{world} independent replicas, one batch-1 sequence per GPU, no collective on the data "
                         f"path") if world > 1 else "1 GPU",
                   "l2": l2_note(cfg, "streamed per token")},
        "e2e": {"value": round(replicas * args.e2e_steps / e2e_s, 3), "unit": "tok/s",
                "h2d_bytes_per_step": 12, "d2h_bytes_per_step": 4 * cfg["vocab"],
                "api": "mimgpu_session_run (pinned host token/position in, logits out, host argmax)"},
        "step_roofline": {"bound": "hbm", "bytes_per_token": wpt, "achieved": round(wpt / (ms / 1e3) / 1e9, 1),
                          "peak": peak, "unit": "GB/s", "frac": round(wpt / (ms / 1e3) / 1e9 / peak, 4)},
        "roofline": {"kernel": kernel,
                     "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": round(traffic) if traffic else None,
                     "bytes_per_launch": round(bpl),
                     "us_per_launch": round(spl * 1e6, 3), "launches": nl, "peak_kind": peak_kind},
        "clocks": clocks.summary(),
        "gpu_launches": launches,
    }
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        try:
            line["cpu_baseline"] = cpu_baseline_sample(ctx, cfg, weights, prompt)
        except Exception as e:  # noqa: BLE001 - the baseline must not hide the GPU line
            line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    sess.free()  # releases the CUDA graphs that hold NCCL calls
    model.free()
    if tp is not None:
        tp.free()
    ctx.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------ GEMV-only sweep mode

def run_gemv(args):
    """Quant-GEMV HBM GB/s: y = W x through
    mimgpu_gemv_q8_dev for one shape `N,K,dtype[,rows]`, rotating over enough
    weight copies to exceed L2; the launches captured back to back in a CUDA
    graph, timed with CUDA events around each replay."""
    import torch
    import mimgpu
    lib = mimgpu.lib()
    parts = args.gemv.split(",")
    N, K = int(parts[0]), int(parts[1])
    dt = {"q4_k": Q4_K, "q6_k": Q6_K}[parts[2].lower()]
    rows = int(parts[3]) if len(parts) > 3 else 1
    torch.cuda.set_device(0)
    ctx = mimgpu.Context(0)
    wb = nbytes(dt, (N, K))
    copies = max(2, min(64, int(2 * 126e6 // wb) + 1)) if not args.gemv_hot else 1
    ws = [ctx.synth(dt, (N, K), 1000 + i) for i in range(copies)]
    st = torch.cuda.Stream()
    x = torch.randn(rows, K, device="cuda", dtype=torch.float32)
    y = torch.empty(rows, N, device="cuda", dtype=torch.float32)
    q8 = C.c_void_p()
    ctx._check(lib.mimgpu_q8_new(ctx.h, rows, K, C.byref(q8)))
    ctx._check(lib.mimgpu_q8_quantize_dev(ctx.h, st.cuda_stream, x.data_ptr(), q8))
    # the launches back to back in one CUDA graph (no host gaps between
    # them), each on the next weight copy so that L2 stays cold; one event
    # pair around each replay, the per-launch time is the replay's / n
    n = max(args.steps, copies)

    def enqueue():
        for i in range(n):
            ctx._check(lib.mimgpu_gemv_q8_dev(ctx.h, st.cuda_stream, q8, x.data_ptr(), ws[i % copies].h, None,
                                              y.data_ptr()))

    with torch.cuda.stream(st):
        for _ in range(max(1, args.warmup)):
            enqueue()
    st.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st, capture_error_mode="thread_local"):
        enqueue()
    ts = []
    with torch.cuda.stream(st):
        g.replay()
        for _ in range(5):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            g.replay()
            b.record(st)
            b.synchronize()
            ts.append(a.elapsed_time(b) / 1e3 / n)
    del g
    ts.sort()
    med = ts[len(ts) // 2]
    algo = wb + rows * (K + K // 256 * 4 + K // 32 * 2 + K // 16 * 2) + rows * N * 4
    peak, kind = peaks()
    print(json.dumps({"metric": "quant-GEMV HBM GB/s", "value": round(algo / med / 1e9, 1), "unit": "GB/s",
                      "shape": [N, K], "dtype": parts[2], "rows": rows, "us_median": round(med * 1e6, 3),
                      "us_min": round(ts[0] * 1e6, 3), "frac": round(algo / med / 1e9 / peak, 4),
                      "algorithmic_bytes": algo, "copies": copies, "launches": n, "peak_kind": kind,
                      "timing": "CUDA graph of the launches back to back, per launch = replay / launches",
                      "int8_tops": round(2 * N * K * rows / med / 1e12, 2)}), flush=True)
    lib.mimgpu_q8_free(q8)
    ctx.close()


# ------------------------------------------------- prefill mode (config 4)

def tensor_peak():
    """Dense int8 tensor peak in TOP/s: twice the measured bf16 cuBLAS burst
    (NVIDIA's dense int8 : bf16 ratio), or twice the fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return 2.0 * float(json.load(f)["bf16_tflops"]), "2 x measured bf16 burst"
    except (OSError, KeyError, ValueError):
        return 2.0 * 1590.0, "2 x fallback bf16"


def gemm_shape_time(ctx, lib, torch, st, N, K, dt, rows, reps):
    """Event time of one dequant_matmul_a8.v2 launch of [rows, K] x [N, K]^T
    (the tensor-core GEMM from 16 rows), rotating over weight copies larger
    than L2 together."""
    wb = nbytes(dt, (N, K))
    copies = max(2, min(16, int(2 * 126e6 // wb) + 1))
    ws = [ctx.synth(dt, (N, K), 4000 + i) for i in range(copies)]
    x = torch.randn(rows, K, device="cuda", dtype=torch.float32)
    y = torch.empty(rows, N, device="cuda", dtype=torch.float32)
    q8 = C.c_void_p()
    ctx._check(lib.mimgpu_q8_new(ctx.h, rows, K, C.byref(q8)))
    ctx._check(lib.mimgpu_q8_quantize_dev(ctx.h, st.cuda_stream, x.data_ptr(), q8))
    ts = []
    with torch.cuda.stream(st):
        for i in range(reps + 3):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            ctx._check(lib.mimgpu_gemv_q8_dev(ctx.h, st.cuda_stream, q8, x.data_ptr(), ws[i % copies].h, None,
                                              y.data_ptr()))
            b.record(st)
            b.synchronize()
            if i >= 3:
                ts.append(a.elapsed_time(b) / 1e3)
    lib.mimgpu_q8_free(q8)
    for w in ws:
        w.free()
    return statistics.median(ts)


def run_prefill(args):
    """Config 4: the 8B-shape prompt pass at T tokens (one sequence), timed on
    the device around mimgpu_session_run, and the tensor-core GEMM alone on
    the decoder's matrix shapes at M = T."""
    import torch
    import mimgpu
    lib = mimgpu.lib()
    torch.cuda.set_device(0)
    cfg = dict(SHAPES[args.shape], layers=args.layers)
    Ts = [int(t) for t in args.prefill.split(",")]
    ctx = mimgpu.Context(0)
    model, weights = build_model(ctx, cfg, max(Ts) + 8, max(Ts))
    sess = model.session()
    stream = torch.cuda.ExternalStream(sess.stream)
    E, F, KV = cfg["embed"], cfg["ffn"], cfg["kv_heads"] * cfg["head_dim"]
    params = sum(int(np.prod(shape)) for name, dt, shape, _, _ in layout(cfg)
                 if dt != F32 and name != "token_embd.weight")
    peak, peak_kind = tensor_peak()
    st = torch.cuda.Stream()
    for T in Ts:
        ids = prompt_ids(cfg["vocab"], T, seed=20261202)
        pos = np.arange(T)
        for _ in range(args.warmup):
            sess.run(ids, pos)
        torch.cuda.synchronize()
        dev, wall = [], []
        clocks = Clocks(0)
        with clocks:
            for _ in range(args.steps):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                t0 = time.perf_counter()
                a.record(stream)
                sess.run(ids, pos)
                b.record(stream)
                b.synchronize()
                wall.append(time.perf_counter() - t0)
                dev.append(a.elapsed_time(b) / 1e3)
        d, w = statistics.median(dev), statistics.median(wall)
        # the GEMM alone on the shapes of one layer (Q, K, V, O, gate, up, down) at M = T
        shapes = [(E, E, Q4_K), (KV, E, Q4_K), (KV, E, Q6_K), (E, E, Q4_K), (F, E, Q4_K), (F, E, Q4_K), (E, F, Q6_K)]
        g_t, g_ops = 0.0, 0.0
        per = {}
        for N, K, dt in shapes:
            t = gemm_shape_time(ctx, lib, torch, st, N, K, dt, T, 5)
            g_t += t
            g_ops += 2.0 * N * K * T
            per[f"{N}x{K} {'q4_k' if dt == Q4_K else 'q6_k'}"] = round(2.0 * N * K * T / t / 1e12, 1)
        useful = g_ops / g_t / 1e12
        executed = 3 * useful  # three int8 digit planes per weight
        print(json.dumps({
            "metric": "8B-shape Q4_K_M prefill tok/s (BASELINE config 4)", "value": round(T / d, 1),
            "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(d * 1e3, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic (seeded N(0,0.02) weights quantized Q4_K_M on the device; seeded "
                                     "random prompt ids)",
            "config": {"workload": f"8B-shape prompt pass, {T} tokens, logits of the last position",
                       "layers": cfg["layers"], "prompt": T,
                       "l2": l2_note(cfg, "per pass")},
            "e2e": {"value": round(T / w, 1), "unit": "tok/s", "h2d_bytes_per_step": 12 * T,
                    "d2h_bytes_per_step": 4 * cfg["vocab"], "api": "mimgpu_session_run (host ids/positions in, "
                                                                  "host logits out)"},
            "gemm": {"useful_int8_tops_per_shape": per, "layer_gemm_ms": round(g_t * 1e3, 3),
                     "layer_gemm_share_of_pass": round(g_t * cfg["layers"] / d, 3)},
            "roofline": {"kernel": "gemm_a8_tc_kernel (one layer's seven matrices at M = T)", "bound": "tensor",
                         "achieved": round(executed, 1), "peak": round(peak, 1), "unit": "TOP/s",
                         "frac": round(executed / peak, 4), "useful_tops": round(useful, 1),
                         "traffic": None, "peak_kind": peak_kind,
                         "note": "achieved counts the MMAs executed: three int8 planes per weight element"},
            "model_flops_tops": round(2.0 * params * T / d / 1e12, 1),
            "clocks": clocks.summary(),
        }), flush=True)
    sess.free()
    model.free()
    ctx.close()


# ------------------------------------------------ batched decode (config 4)

def run_batch(args):
    """Config 4's batched decode: B sequences in one session (one key-value
    cache each), each prefilled with its own prompt to ~1000 tokens of a
    1024-token cache, then greedy steps of all B sequences together, timed on
    the device; e2e through mimgpu_session_run_slots with host buffers."""
    import torch
    import mimgpu
    torch.cuda.set_device(0)
    cfg = dict(SHAPES[args.shape], layers=args.layers)
    B, C = args.batch, args.context
    prompt = C - args.warmup - args.steps - args.e2e_steps - 8
    ctx = mimgpu.Context(0)
    model, weights = build_model(ctx, cfg, C, max(B, prompt))
    sess = model.session(slots=B)
    t0 = time.perf_counter()
    first = []
    for b in range(B):
        ids = prompt_ids(cfg["vocab"], prompt, seed=20261203 + b)
        lg = sess.run_slots(ids, np.full(prompt, b), np.arange(prompt))
        first.append(int(np.argmax(lg[-1])))
    prefill_s = time.perf_counter() - t0
    pos = np.full(B, prompt, np.int64)
    out = sess.generate_slots(first, pos, args.warmup)  # warm-up (captures the batched graph)
    tok, pos = out[-1].copy(), pos + args.warmup
    stream = torch.cuda.ExternalStream(sess.stream)
    torch.cuda.synchronize()
    clocks = Clocks(0)
    with clocks:
        a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        out = sess.generate_slots(tok, pos, args.steps)
        b_.record(stream)
        torch.cuda.synchronize()
    dev_s = a.elapsed_time(b_) / 1e3
    tok, pos = out[-1].copy(), pos + args.steps
    # e2e: one run_slots per step, host argmax
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        lg = sess.run_slots(tok, np.arange(B), pos)
        tok, pos = lg.argmax(axis=1).astype(np.int32), pos + 1
    e2e_s = time.perf_counter() - t0
    value = B * args.steps / dev_s
    wpt = weight_bytes_per_token(cfg)
    peak, peak_kind = peaks()
    print(json.dumps({
        "metric": (f"8B-shape Q4_K_M batched decode tok/s (BASELINE config 4, batch {B})" if args.shape == "8b"
                   else f"70B-shape Q4_K_M batched decode tok/s (BASELINE config 5, batch {B})"),
        "value": round(value, 1),
        "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dev_s / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded N(0,0.02) weights quantized Q4_K_M on the device; seeded random prompt ids)",
        "config": {"workload": f"{args.shape.upper()}-shape greedy decode of {B} sequences together, {C}-token cache",
                   "layers": cfg["layers"], "batch": B, "context_cache": C, "prompt_per_sequence": prompt,
                   "prefill_s": round(prefill_s, 2),
                   "l2": l2_note(cfg, "streamed per step")},
        "e2e": {"value": round(B * args.e2e_steps / e2e_s, 1), "unit": "tok/s", "h2d_bytes_per_step": 16 * B,
                "d2h_bytes_per_step": 4 * cfg["vocab"] * B,
                "api": "mimgpu_session_run_slots (host ids/sequences/positions in, logits out, host argmax)"},
        "step_roofline": {"bound": "hbm", "bytes_per_step": wpt, "achieved": round(wpt / (dev_s / args.steps) / 1e9, 1),
                          "peak": peak, "unit": "GB/s", "frac": round(wpt / (dev_s / args.steps) / 1e9 / peak, 4),
                          "peak_kind": peak_kind},
        "clocks": clocks.summary(),
    }), flush=True)
    sess.free()
    model.free()
    ctx.close()


# ----------------------------------------------------------- reference arm

def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    cfg = CFG8B
    nt = O.threads()
    t0 = time.perf_counter()
    host = {}
    for name, dt, shape, mean, sigma in layout(cfg):
        if dt == F32:
            host[name] = (dt, O.gen_normal(seed_of(name), shape[0], mean, sigma))
        else:
            host[name] = (dt, O.gen_weight(dt, seed_of(name), shape[0], shape[1], sigma, nt))
    gen_s = time.perf_counter() - t0
    prompt = args.prompt
    context = prompt + args.warmup + args.steps + 8
    m = O.Llama(dict(cfg, context=context, a8=1, cache_f16=1, interleaved=1, nthreads=nt), host)
    ids = prompt_ids(cfg["vocab"], prompt)
    t0 = time.perf_counter()
    tok, pos = O.argmax(m.forward(ids, np.arange(prompt))[0]), prompt
    prefill_s = time.perf_counter() - t0
    for _ in range(args.warmup):
        tok, pos = O.argmax(m.forward([tok], [pos])[0]), pos + 1
    budget = args.reference_budget
    t0, steps = time.perf_counter(), 0
    for _ in range(args.steps):
        tok, pos = O.argmax(m.forward([tok], [pos])[0]), pos + 1
        steps += 1
        if time.perf_counter() - t0 > budget:
            break
    el = time.perf_counter() - t0
    value = steps / el
    sample = (f"{steps} greedy decode tokens (of {args.steps} asked; {budget:.0f} s budget) of the 8B-shape model "
              f"after the bench's {prompt}-token prompt (prefilled in {prefill_s:.0f} s); weights generated on the "
              f"host in {gen_s:.0f} s; {PORT_NOTE}")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "tok/s", "n_gpus": 0,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(el / steps * 1e3, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": round(value / PUBLISHED_8B, 3), "dtype": "int8",
        "data": "synthetic (seeded N(0,0.02) weights quantized Q4_K_M on the host; seeded random prompt ids)",
        "config": {"workload": "8B-shape Q4_K_M greedy decode, batch 1 (BASELINE config 3)", "prompt": prompt,
                   "implementation": "oracle/ C restatement of the Go reference path (go is not installed)"},
        "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "cores": nt, "cpu": cpu_model(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_write_mim(args):
    """--write-mim: the benchmark model of --shape / --layers, made on the
    device as the bench makes it, written as a mim file."""
    import mimgpu
    cfg = dict(SHAPES[args.shape], layers=args.layers)
    ctx = mimgpu.Context(int(os.environ.get("LOCAL_RANK", "0")))
    model, weights = build_model(ctx, cfg, args.context, 1)
    t0 = time.time()
    n = write_mim(ctx, cfg, weights, args.write_mim, args.context)
    print(json.dumps({"wrote": args.write_mim, "bytes": n, "shape": args.shape, "layers": args.layers,
                      "context": args.context, "seconds": round(time.time() - t0, 1)}), flush=True)
    model.free()
    for _, t in weights.values():
        t.free()
    ctx.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="mimgpu", choices=["mimgpu", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=64)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--reference-budget", type=float, default=120.0)
    ap.add_argument("--tp", action="store_true",
                    help="N > 1: tensor parallelism of one sequence (the default for --shape 70b; 8b runs replicas)")
    ap.add_argument("--p2p", action="store_true",
                    help="tensor parallelism: exchanges by peer-memory stores instead of NCCL all-gathers")
    ap.add_argument("--shape", default="8b", choices=sorted(SHAPES),
                    help="model shape: 8b (configs 3-4) or 70b (config 5)")
    ap.add_argument("--layers", type=int, default=0,
                    help="decoder layers (default: the shape's own; fewer only for profiling runs)")
    ap.add_argument("--prompt", type=int, default=PROMPT, help="prompt tokens before the timed decode steps")
    ap.add_argument("--gemv", default="", help="GEMV-only mode: N,K,q4_k|q6_k[,rows]")
    ap.add_argument("--gemv-hot", action="store_true", help="GEMV-only mode with one weight copy (L2-hot)")
    ap.add_argument("--prefill", default="", help="prefill mode (config 4): prompt lengths, e.g. 512,2048")
    ap.add_argument("--batch", type=int, default=0, help="batched decode mode (config 4): sequences, e.g. 32")
    ap.add_argument("--context", type=int, default=1024,
                    help="key-value cache per sequence in --batch mode, and the cache --write-mim records")
    ap.add_argument("--write-mim", default="", metavar="PATH",
                    help="write the --shape / --layers benchmark model as a mim file and exit")
    ap.add_argument("--mim", default="", metavar="PATH",
                    help="decode bench from a mim file (the --shape / --layers of the file) instead of weights "
                         "made on the device")
    args = ap.parse_args()
    if not args.layers:
        args.layers = SHAPES[args.shape]["layers"]
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.write_mim:
        run_write_mim(args)
    elif args.gemv:
        run_gemv(args)
    elif args.prefill:
        run_prefill(args)
    elif args.batch:
        run_batch(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
