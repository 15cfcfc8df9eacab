"""Tensor parallelism across 2 GPUs of one node (needs >= 2 GPUs; skipped
otherwise): every rank holds and reads only its rows of each matrix (q|k|v by
kv-head group, o / gate|up / down / head by output rows), computes complete
block-ordered dot products and exchanges the attention output, the residual
and the SwiGLU output, so the prompt logits and 32 greedy ids of 8B- and
70B-shaped layers are bit-identical to one GPU."""
import multiprocessing as mp
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


_ONE = {}


def _one_gpu(shape):
    import tp_worker
    if shape not in _ONE:
        _ONE[shape] = tp_worker.decode(0, None, 1, 0, shape=shape)
    return _ONE[shape]


@pytest.mark.skipif("_gpus() < 2")
@pytest.mark.parametrize("shape,p2p", [("8b", False), ("8b", True), ("70b", True)],
                         ids=["8b-nccl", "8b-peer-memory", "70b-peer-memory"])
def test_tp2_bit_identical_to_one_gpu(shape, p2p):
    """Prompt (16 tokens: NCCL all-gathers) and 32 greedy steps (NCCL, or
    peer-memory exchanges inside the kernels) on 2 ranks, each holding only
    its shard of every split matrix."""
    import socket
    import tp_worker
    import mimgpu
    want_logits, want_ids = _one_gpu(shape)
    gid = mimgpu.tp_unique_id()
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=tp_worker.rank_main, args=(r, 2, gid, port, p2p, q, shape)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(2):
            r, res = q.get(timeout=600)
            got[r] = res
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(2):
        assert not isinstance(got[r], str), got[r]
        logits, ids = got[r]
        assert np.array_equal(logits.view(np.uint32), want_logits.view(np.uint32)), f"rank {r} logits"
        assert ids.tolist() == want_ids.tolist(), f"rank {r} ids"
