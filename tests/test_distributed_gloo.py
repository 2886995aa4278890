"""DistributedSUM semantics on two CPU ranks (gloo), as replica.py:321-379 defines them.

The GPU path runs the same calls over NCCL; these tests cover the host logic
without a GPU: the SUM of flat [K,N] gradients, zeroing of a lane inactive on
every rank, the packed one-all-reduce agreement (active lanes, failures, step
budget), asymmetric active lanes raising on every rank, and the global
decision-mass normaliser used by the loss's global-Z variant.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, scenario, queue):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "ai-game-learning_b200"))
    from pbg_b200.distributed import DistributedSUM

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        d = DistributedSUM()
        if scenario == "sum":
            grads = torch.arange(12, dtype=torch.float32).reshape(2, 6) * (rank + 1)
            out = d.sum_gradients(grads.clone(), torch.tensor([True, True]))
            queue.put((rank, "sum", out.tolist()))
            # lane 1 inactive on every rank: its rows are zeroed before the SUM
            out = d.sum_gradients(grads.clone(), torch.tensor([True, False]))
            queue.put((rank, "sum_inactive", out.tolist()))
            failures, steps = d.agree(torch.tensor([True, False]), torch.tensor([False, rank == 1]), 5 * rank + 1)
            queue.put((rank, "agree", (failures.tolist(), steps)))
            failed = d.agree_failures(torch.tensor([rank == 1, False]))
            queue.put((rank, "fail", failed.tolist()))
            queue.put((rank, "steps", d.maximum_steps(3 + rank, "cpu")))
            z = d.global_sum(torch.tensor([0.5 * (rank + 1)], dtype=torch.float64))
            queue.put((rank, "z", float(z[0])))
        elif scenario == "disagree":
            try:
                d.agree_active(torch.tensor([True, rank == 0]))
                queue.put((rank, "disagree", "no error"))
            except RuntimeError as exc:
                queue.put((rank, "disagree", str(exc)))
            try:
                d.sum_gradients(torch.ones(2, 3), torch.tensor([rank == 0, True]))
                queue.put((rank, "sum_disagree", "no error"))
            except RuntimeError as exc:
                queue.put((rank, "sum_disagree", str(exc)))
    finally:
        dist.destroy_process_group()


def _run(scenario):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, scenario, queue)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    out = {}
    while not queue.empty():
        rank, key, value = queue.get()
        out[(rank, key)] = value
    return out


def test_gradient_sum_agreement_and_budget():
    out = _run("sum")
    base = [[float(i) for i in range(6)], [float(i) for i in range(6, 12)]]
    want = [[3 * v for v in row] for row in base]
    assert out[(0, "sum")] == want and out[(1, "sum")] == want
    want_inactive = [want[0], [0.0] * 6]
    assert out[(0, "sum_inactive")] == want_inactive and out[(1, "sum_inactive")] == want_inactive
    # one packed MAX all-reduce: failures from any rank, the larger step budget
    assert out[(0, "agree")] == ([False, True], 6) and out[(1, "agree")] == ([False, True], 6)
    assert out[(0, "fail")] == [True, False] == out[(1, "fail")]
    assert out[(0, "steps")] == 4 == out[(1, "steps")]
    assert out[(0, "z")] == pytest.approx(1.5) and out[(1, "z")] == pytest.approx(1.5)


def test_active_lane_disagreement_raises_on_every_rank():
    out = _run("disagree")
    for key in ("disagree", "sum_disagree"):
        assert "asymmetric" in out[(0, key)] and "asymmetric" in out[(1, key)]
