"""Multi-GPU: the NVLS multimem gradient SUM against NCCL's all_reduce(SUM).

Runs as child processes (one per GPU, NCCL process group) at 2, 4 and 8 ranks,
each case skipped when the machine has fewer GPUs.  Each rank fills the
symmetric buffer with its own seeded gradient, sums it twice in a row through
pbg_nvls_allreduce_sum_f32 and compares with NCCL on the same data and with a
float64 sum of every rank's input, then sums a third gradient as four buckets
launched back to back on a side stream (``NVLSFlatSum.sum_range_``).  At two ranks a + b is exact in either
order, so the NVLS result must equal NCCL's bit for bit; at 4 and 8 ranks the
switch and NCCL add in different orders, so both are held to the float64 sum
within fp32 rounding of a W-term sum (rtol 4e-6 plus an absolute term scaled
by the sum of magnitudes).  A third call runs after the error word is set by
hand: the sticky error keeps the kernel off the buffer.
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
            inputs = [torch.randn(n, generator=torch.Generator(device=device).manual_seed(100 * call + r),
                                  device=device) for r in range(world)]
            data = inputs[rank]
            flat.buffer.copy_(data)
            ref = data.clone()
            dist.all_reduce(ref, op=dist.ReduceOp.SUM)
            flat.sum_()
            torch.cuda.synchronize(device)
            flat.check()
            exact = torch.stack(inputs).double().sum(0)
            scale = torch.stack(inputs).double().abs().sum(0)
            bound = 4e-6 * exact.abs() + 2.0 * world * 2.0 ** -24 * scale
            nvls_err = (flat.buffer.double() - exact).abs()
            nccl_err = (ref.double() - exact).abs()
            results.append({
                "equal_nccl": bool(torch.equal(flat.buffer, ref)),
                "nvls_ok": bool((nvls_err <= bound).all()),
                "nccl_ok": bool((nccl_err <= bound).all()),
                "nvls_max_err": float(nvls_err.max()),
            })
        # four buckets summed one after another on a side stream (the bench's overlapped step)
        inputs = [torch.randn(n, generator=torch.Generator(device=device).manual_seed(300 + r), device=device)
                  for r in range(world)]
        flat.buffer.copy_(inputs[rank])
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        q = n // 4 // (4 * world) * (4 * world)  # bucket bounds are multiples of 4 * world
        for k in range(4):
            flat.sum_range_(k * q, q if k < 3 else n - 3 * q, side)
        torch.cuda.current_stream(device).wait_stream(side)
        torch.cuda.synchronize(device)
        flat.check()
        exact = torch.stack(inputs).double().sum(0)
        scale = torch.stack(inputs).double().abs().sum(0)
        bound = 4e-6 * exact.abs() + 2.0 * world * 2.0 ** -24 * scale
        two_term = world != 2 or bool(torch.equal(flat.buffer, inputs[0] + inputs[1]))  # a + b: exact in fp32
        results.append({"equal_nccl": two_term, "nvls_ok": bool(((flat.buffer.double() - exact).abs() <= bound).all()),
                        "nccl_ok": True, "nvls_max_err": float((flat.buffer.double() - exact).abs().max())})
        # a set error word keeps every later launch off the buffer and the pads
        before = flat.buffer.clone()
        flat.error.fill_(1)
        flat.sum_()
        torch.cuda.synchronize(device)
        untouched = bool(torch.equal(flat.buffer, before))
        raised = False
        try:
            flat.raise_if_failed()
        except RuntimeError:
            raised = True
        flat.reset()
        queue.put((rank, results, untouched, raised))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_nvls_sum_matches_nccl_and_float64(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    try:
        for p in procs:
            p.start()
        for p in procs:
            p.join(240)
        codes = [p.exitcode for p in procs]
    finally:
        # a worker that did not finish is stopped and reaped before the test reports
        for p in procs:
            if p.is_alive():
                p.terminate()
        for p in procs:
            p.join(30)
    assert codes == [0] * world, f"worker exit codes {codes}"
    got = {}
    for _ in range(world):
        rank, results, untouched, raised = queue.get(timeout=30)
        got[rank] = (results, untouched, raised)
    for rank in range(world):
        results, untouched, raised = got[rank]
        for r in results:
            assert r["nvls_ok"] and r["nccl_ok"], r
            if world == 2:
                assert r["equal_nccl"], r
        assert untouched and raised
