"""Time the flat-gradient SUM: libpbgb200's NVLS multimem kernel vs NCCL, over buffer sizes.

    torchrun --nproc-per-node N ai-game-learning_b200/collective_sweep.py

One process per GPU; each size is timed over 20 back-to-back calls with CUDA events, max over
ranks, after 3 warm-up calls.  Rank 0 prints one line per size.
"""
import datetime, os, sys, torch, torch.distributed as dist
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from pbg_b200.distributed import NVLSFlatSum
world, rank = int(os.environ["WORLD_SIZE"]), int(os.environ["RANK"])
torch.cuda.set_device(rank); dev = torch.device("cuda", rank)
dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
for n in (8192, 262144, 1048576, 4194304, 16777216):
    f = NVLSFlatSum(n, dev); f.buffer.normal_()
    s = torch.cuda.current_stream()
    for _ in range(3): f.sum_(s)
    torch.cuda.synchronize(); dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(s)
    for _ in range(20): f.sum_(s)
    b.record(s); torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / 20 * 1000], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX); f.check()
    x = torch.zeros(n, device=dev)
    for _ in range(3): dist.all_reduce(x)
    torch.cuda.synchronize(); dist.barrier(); a.record(s)
    for _ in range(20): dist.all_reduce(x)
    b.record(s); torch.cuda.synchronize()
    u = torch.tensor([a.elapsed_time(b) / 20 * 1000], device=dev, dtype=torch.float64)
    dist.all_reduce(u, op=dist.ReduceOp.MAX)
    if rank == 0: print(f"n={n} bytes={4*n} nvls_us={float(t[0]):.1f} nccl_us={float(u[0]):.1f}", flush=True)
    del f; torch.cuda.synchronize(); dist.barrier()
dist.destroy_process_group()
