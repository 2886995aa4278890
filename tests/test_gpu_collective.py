"""Multi-GPU: the NVLS multimem gradient SUM against NCCL's all_reduce(SUM).

Runs as two child processes (one per GPU, NCCL process group) when the
machine has at least two GPUs; skipped otherwise.  Each rank fills the
symmetric buffer with its own seeded gradient, sums it twice in a row through
pbg_nvls_allreduce_sum_f32 and compares with NCCL on the same data (two ranks:
a + b is exact in either order, so the results must be equal).
"""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue):
    import datetime
    import sys

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "ai-game-learning_b200"))
    from pbg_b200.distributed import NVLSFlatSum

    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=device)
    try:
        n = 4 * world * 262_147
        flat = NVLSFlatSum(n, device)
        results = []
        for call in range(2):
            g = torch.Generator(device=device).manual_seed(100 * call + rank)
            data = torch.randn(n, generator=g, device=device)
            flat.buffer.copy_(data)
            ref = data.clone()
            dist.all_reduce(ref, op=dist.ReduceOp.SUM)
            flat.sum_()
            torch.cuda.synchronize(device)
            flat.check()
            results.append(bool(torch.equal(flat.buffer, ref)))
        queue.put((rank, results))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nvls_sum_matches_nccl_on_two_ranks():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
        assert p.exitcode == 0
    got = dict(queue.get() for _ in range(2))
    assert got[0] == [True, True] and got[1] == [True, True]
