"""The tensor-parallel row split, on the CPU with two gloo ranks (no GPU).

Each rank takes its rows of every split matrix exactly as bench.py's
shard_rows gives them to a GPU rank (q|k|v by kv-head group, o / gate|up /
down / head by output rows), makes them with the oracle's seeded generator
for that row range only, and computes its rows of the 8-bit product
(dotQ8KRef, gsoultan/mimir-model internal/kernels/q8k_test.go:35-117).  The
gathered shards must be the whole tensor byte for byte, and the gathered
outputs the one-rank product bit for bit: a row's dot product never crosses a
rank, which is what makes the GPU ranks' logits the one-GPU logits.
"""
import multiprocessing as mp
import os
import socket
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

CFG = dict(layers=1, embed=512, ffn=1024, heads=8, kv_heads=2, head_dim=64, vocab=1000)


def _rank(rank, world, port, q):
    try:
        sys.path.insert(0, ROOT)
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import torch
        import torch.distributed as dist
        import bench
        import oracle as O
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        cfg = dict(CFG)
        x = O.gen_normal(5, cfg["embed"]).reshape(1, -1)
        results = {}
        for name, dt, shape, _, sigma in bench.layout(cfg):
            sh = bench.shard_rows(name, cfg, world, rank)
            if sh is None or dt == O.F32 or shape[1] != cfg["embed"]:
                continue
            r0, rows = sh
            w = O.gen_weight_rows(dt, bench.seed_of(name), r0, rows, shape[1], sigma)
            y = O.dequant_matmul_a8(x, dt, w, rows)
            # every rank's shard and output rows to every rank (the exchange)
            parts_w, parts_y = [None] * world, [None] * world
            dist.all_gather_object(parts_w, w.tobytes())
            dist.all_gather_object(parts_y, y.tobytes())
            results[name] = (b"".join(parts_w), b"".join(parts_y))
        dist.destroy_process_group()
        q.put((rank, results))
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e)))


def test_row_split_over_two_gloo_ranks_is_the_whole_product():
    sys.path.insert(0, ROOT)
    import bench
    import oracle as O
    world = 2
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            r, res = q.get(timeout=300)
            got[r] = res
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert not isinstance(got[r], str), got[r]
    x = O.gen_normal(5, CFG["embed"]).reshape(1, -1)
    checked = 0
    for name, dt, shape, _, sigma in bench.layout(CFG):
        if name not in got[0]:
            continue
        whole_w = O.gen_weight(dt, bench.seed_of(name), shape[0], shape[1], sigma)
        whole_y = O.dequant_matmul_a8(x, dt, whole_w, shape[0])
        for r in range(world):
            w_bytes, y_bytes = got[r][name]
            assert w_bytes == whole_w.tobytes(), f"{name}: the shards are not the tensor"
            assert y_bytes == whole_y.tobytes(), f"{name}: the rank outputs are not the product"
        checked += 1
    # q, k, v, o, gate, up (and the head): every split matrix of K = embed
    assert checked >= 6
