"""One rank of the tensor-parallel GPU test (run in a spawned process): builds
the synthetic 8B-layer-shape model on its GPU, joins the group, and returns
the prompt logits and greedy ids."""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def model_cfg(shape: str = "8b"):
    """Two layers of the 8B shape, or one of the 70B shape (E 8192, F 28672,
    64 / 8 heads), vocabulary 32000."""
    if shape == "70b":
        return dict(layers=1, embed=8192, ffn=28672, heads=64, kv_heads=8, head_dim=128, rope_dims=128,
                    vocab=32000, rope_theta=500000.0, norm_eps=1e-5)
    return dict(layers=2, embed=4096, ffn=14336, heads=32, kv_heads=8, head_dim=128, rope_dims=128, vocab=32000,
                rope_theta=500000.0, norm_eps=1e-5)


def decode(device: int, group_id: bytes | None, nranks: int, rank: int, steps: int = 32, exchange=None,
           shape: str = "8b"):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "mimir-model_b200"))
    import bench
    import mimgpu
    cfg = model_cfg(shape)
    ctx = mimgpu.Context(device)
    # a rank of a group holds only its rows of every split matrix
    model, _ = bench.build_model(ctx, cfg, 128, 16, (nranks, rank) if group_id is not None else None)
    tp = None
    if group_id is not None:
        tp = mimgpu.TensorParallel(ctx, group_id, nranks, rank)
        model.set_tp(tp)
    s = model.session()
    if exchange is not None:  # map every rank's arena: decode steps exchange over peer memory
        s.set_peers(exchange(s.ipc_handle()))
    prompt = np.random.default_rng(3).integers(0, cfg["vocab"], 16).astype(np.int32)
    logits = s.run(prompt, np.arange(16), all_rows=True)
    ids = s.generate(int(np.argmax(logits[-1])), 16, steps)
    s.free()
    model.free()
    if tp is not None:
        tp.free()
    ctx.close()
    return logits, ids


def rank_main(rank: int, nranks: int, group_id: bytes, port: int, p2p: bool, q, shape: str = "8b"):
    import torch.distributed as dist
    from datetime import timedelta
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=nranks,
                                timeout=timedelta(seconds=120))

        def exchange(handle):
            out = [None] * nranks
            dist.all_gather_object(out, handle)
            return out

        q.put((rank, decode(rank, group_id, nranks, rank, exchange=exchange if p2p else None, shape=shape)))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)))
