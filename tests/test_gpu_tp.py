"""Tensor parallelism across 2 GPUs of one node (needs >= 2 GPUs; skipped
otherwise): every rank computes complete block-ordered dot products over its
output rows and all-gathers the activations it needs, so the prompt logits
and 32 greedy ids of a 2-layer 8B-shape model are bit-identical to one GPU."""
import multiprocessing as mp
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.fixture(scope="module")
def one_gpu():
    import tp_worker
    return tp_worker.decode(0, None, 1, 0)


@pytest.mark.skipif("_gpus() < 2")
@pytest.mark.parametrize("p2p", [False, True], ids=["nccl", "peer-memory"])
def test_tp2_bit_identical_to_one_gpu(one_gpu, p2p):
    """Prompt (16 tokens: NCCL all-gathers) and 32 greedy steps (NCCL, or
    peer-memory exchanges inside the kernels) on 2 ranks."""
    import socket
    import tp_worker
    import mimgpu
    want_logits, want_ids = one_gpu
    gid = mimgpu.tp_unique_id()
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=tp_worker.rank_main, args=(r, 2, gid, port, p2p, q)) for r in range(2)]
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
