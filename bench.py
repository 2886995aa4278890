"""Benchmark: learner decisions/s of the fused PPO loss backward (+ gradient SUM).

Workload (the configuration the headline metric is quoted
on): per rank 4,194,304 synthetic decisions x 8 actions, generated on the
device with seed 0 + rank -- logits bf16 N(0,1), legal masks Bernoulli(0.7)
with the lowest index forced legal in empty rows, the taken action drawn
from the legal set with the counter RNG (LEARNER purpose), old log pi from
logits + N(0,0.1), advantages N(0,1), decision-mass weights U(0,1).  One
step = the fused masked log-softmax / clipped-ratio / entropy / dlogits
kernel over all rows and (N > 1) the SUM all-reduce of a flat fp32 gradient
buffer of --params parameters (libpbgb200's NVLS multimem kernel on symmetric
memory from 4 ranks; NCCL at 2 ranks or when the fabric has no multicast).  With
--buckets B > 1 the rows run as B chunks and the SUM as B buckets on a
second stream, bucket k starting when chunk k is done, so the SUM overlaps the
remaining loss (default 1: loss, then SUM; on a 2-GPU B200 box four buckets
took 153 us per step against 120 us serial, each SUM call carrying ~16 us of
launch and cross-rank barriers).  Weak scaling: each rank owns its own rows.

``--impl reference`` times the CPU restatement of the same loss on the same
rows (the reference has no CPU execution path) on all host threads.  The
reference's own PyTorch CUDA loss program, when the driver installed it under
baseline/_ref, is timed inside the b200 arm on the same box and reported as
``reference_torch_cuda`` (the comparator the north star names), with the
speed-up of ``value`` and of ``e2e`` over it.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "ai-game-learning_b200"))

METRIC = "learner decisions/sec (fused PPO loss backward + flat-gradient SUM all-reduce)"
UNIT = "decisions/s"
BYTES_PER_ROW = lambda A: 5 * A + 16  # bf16 logits in + u8 mask + i32 action + 3 f32 + bf16 dlogits out


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--rows", type=int, default=4_194_304)
    p.add_argument("--actions", type=int, default=8)
    p.add_argument("--params", type=int, default=4_194_304)
    p.add_argument("--e2e-steps", type=int, default=10)
    p.add_argument("--profile-hands", type=int, default=4096,
                   help="--profile-forward rollout_with_model: hands of the profiled rollout; learner_step_cfg2: "
                        "H / 4 preflop and H / 16 postflop presentations")
    p.add_argument("--engine-compare", action="store_true",
                   help="time the reference's own training iteration (pbg.runtime.TrainingSession from baseline/_ref) "
                        "unmodified and with pbg_b200.engine.install(learner=True), each in a fresh process, and "
                        "print one JSON line (player nodes/s and learner presentations/s of both)")
    p.add_argument("--engine-arm", choices=("reference", "reference_eager", "b200", "b200_eager"), default=None,
                   help=argparse.SUPPRESS)
    p.add_argument("--engine-roots", type=int, default=4096)
    p.add_argument("--engine-iterations", type=int, default=6)
    p.add_argument("--learner-scaling", nargs="?", const="cfg1", choices=("cfg1", "cfg2"), default=None,
                   help="time a learner step data-parallel instead: every rank a step over its own presentations "
                        "(cfg1: 16,384 for the MLP; cfg2: 1,024 preflop + 256 postflop for the attention "
                        "network), the SUM of the real flat gradient (NCCL), then AdamW; one JSON line")
    p.add_argument("--allreduce", choices=("auto", "nvls", "nccl"), default="auto",
                   help="gradient SUM at N > 1: auto = libpbgb200's NVLS kernel from 4 ranks, NCCL below")
    p.add_argument("--comm-sms", type=int, default=16,
                   help="N > 1 with buckets: SMs reserved for the gradient SUM (the loss kernel runs on the rest)")
    p.add_argument("--buckets", type=int, default=1,
                   help="N > 1: the rows' loss runs as this many chunks, and the gradient SUM as as many buckets "
                        "on a second stream, bucket k starting when chunk k's loss is done")
    p.add_argument("--component", default=None,
                   help="run one entry of the components object (its name there) and print it as one JSON line")
    p.add_argument("--profile-forward", choices=("preflop", "postflop", "attention", "folded", "posterior",
                                                 "readout", "reach", "showdown", "optimizer", "poker_loss",
                                                 "rollout_with_model", "completion", "rollout", "learner_step",
                                                 "learner_step_cfg2"),
                   default=None,
                   help="run one eager forward of that component (attention: one attention-core launch at the "
                        "postflop sequence length, 48 x 2,406 tokens x 8 heads; folded: the removal queries and "
                        "the beta eigendecomposition of components.folded_statistics; posterior: one call of "
                        "components.posterior_sampler; readout: one launch of components.loss_readout; reach: "
                        "one launch of components.reach_update; showdown / optimizer: one call of "
                        "components.showdown / components.optimizer_step; poker_loss: one launch of the "
                        "sampled batch of components.poker_loss; rollout_with_model: one whole rollout of "
                        "--profile-hands hands of components.rollout_with_model) "
                        "between cudaProfilerStart/Stop (for ncu "
                        "--profile-from-start off) after two warm-up runs, print nothing else, exit")
    return p.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ----------------------------------------------------------- inputs


def make_inputs(rows, A, seed, device):
    import torch
    from pbg_b200.rng import DrawPurpose, logical_categorical, logical_rng_keys

    g = torch.Generator(device=device).manual_seed(seed)
    logits = torch.randn((rows, A), generator=g, device=device).to(torch.bfloat16)
    mask = torch.rand((rows, A), generator=g, device=device) < 0.7
    empty = ~mask.any(1)
    mask[:, 0] |= empty
    uniform = mask.float()
    keys = logical_rng_keys(seed=seed, iteration=0, root=torch.arange(rows, device=device),
                            path=torch.zeros(rows, dtype=torch.int64, device=device), draw=0,
                            purpose=DrawPurpose.LEARNER)
    action = logical_categorical(uniform, keys).to(torch.int32)
    pert = logits.float() + 0.1 * torch.randn((rows, A), generator=g, device=device)
    old = torch.log_softmax(pert.masked_fill(~mask, -torch.inf), -1).gather(1, action.long()[:, None])[:, 0]
    adv = torch.randn(rows, generator=g, device=device)
    weight = torch.rand(rows, generator=g, device=device)
    del uniform, keys, pert
    return logits.contiguous(), mask.contiguous(), action.contiguous(), old.contiguous(), adv, weight


# ----------------------------------------------------------- clocks


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during timing."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------- peaks


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def committed_traffic(rows):
    """DRAM bytes per launch of the loss kernel from the committed ncu summary."""

    path = os.path.join(ROOT, "profiles", "ppo_bf16x8_loss_4M.txt")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("dram_bytes_per_row:"):
                    return float(line.split(":")[1]) * rows
    except OSError:
        pass
    return None


# ----------------------------------------------------------- CPU legs


def cpu_loss_rate(inputs_host, seconds=3.0, threads=None):
    """Oracle loss passes over host rows on all threads for ~`seconds` wall."""

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O

    logits, mask, action, old, adv, weight = inputs_host
    N = logits.shape[0]
    threads = threads or os.cpu_count() or 1
    chunks = np.array_split(np.arange(N), threads)
    O.lib()

    def run(idx):
        lo, hi = int(idx[0]), int(idx[-1]) + 1
        O.ppo_categorical(logits[lo:hi], mask[lo:hi], action[lo:hi], old[lo:hi], adv[lo:hi], weight[lo:hi],
                          inv_count=1.0 / N)
        return hi - lo

    rows = 0
    start = time.perf_counter()
    with cf.ThreadPoolExecutor(threads) as pool:
        while True:
            rows += sum(pool.map(run, chunks))
            if time.perf_counter() - start >= seconds:
                break
    wall = time.perf_counter() - start
    return rows / wall, threads, rows, wall


def host_sample(rows, A, seed):
    """A CPU copy of the device workload generator's distribution (numpy)."""

    import numpy as np

    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((rows, A)).astype(np.float32)
    # bf16 rounding, as the device inputs carry
    logits = (logits.view(np.uint32) + 0x8000 & 0xFFFF0000).view(np.float32)
    mask = rng.random((rows, A)) < 0.7
    mask[~mask.any(1), 0] = True
    cum = np.cumsum(mask, 1)
    pick = (rng.random(rows) * cum[:, -1]).astype(np.int64)
    action = (cum <= pick[:, None]).sum(1).astype(np.int32)
    pert = np.where(mask, logits + 0.1 * rng.standard_normal((rows, A)).astype(np.float32), -np.inf)
    mx = pert.max(1)
    lse = np.log(np.exp(pert - mx[:, None]).sum(1)) + mx
    old = (pert[np.arange(rows), action] - lse).astype(np.float32)
    adv = rng.standard_normal(rows).astype(np.float32)
    weight = rng.random(rows).astype(np.float32)
    return logits, mask.astype(np.uint8), action, old, adv, weight


def reference_arm(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    sample = host_sample(args.rows, args.actions, 0)
    for _ in range(args.warmup):
        cpu_loss_rate(sample, seconds=0.0)
    rates = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        rate, threads, rows, wall = cpu_loss_rate(sample, seconds=0.0)
        rates.append(rate)
    elapsed = time.perf_counter() - t0
    value = args.steps * sample[0].shape[0] / elapsed
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * elapsed / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic",
        "config": {"workload": "cfg5 loss microbench: 4,194,304 decisions x 8 actions per step, fused PPO "
                               "loss backward, CPU restatement (oracle port)",
                   "rows_per_step": sample[0].shape[0], "actions": args.actions, "same_rows_as_b200_arm": True},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{sample[0].shape[0]} rows x {args.actions} actions per step, all host threads"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------- poker learner objective


def _poker_loss_inputs(device, S, W, E, M=2, seed=11):
    """A seeded learner batch on the device: raw fields with the model head's value ranges
    (softmax omega, sigmoid mu / iota, softplus + 0.02 scale), a reference copy perturbed as
    after one update, legal sets shaped as the game's (check/call always, fold when facing a bet
    with probability 0.7, raise ticks one contiguous range ending at the all-in, none in 10% of
    rows), legal taken actions, old log pi near the current one, N(0,1) advantages, posteriors
    with 30% zeros (Rao-Blackwell), values and targets N(0,1)."""

    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    T = E - 2
    raw = {"type_logits": torch.randn(S, W, 3, device=device, generator=g) * 1.5,
           "omega": torch.softmax(torch.randn(S, W, M, device=device, generator=g), -1),
           "mu": torch.sigmoid(torch.randn(S, W, M, device=device, generator=g)),
           "s": torch.nn.functional.softplus(torch.randn(S, W, M, device=device, generator=g)) + 0.02,
           "iota": torch.sigmoid(torch.randn(S, W, device=device, generator=g))}
    ref = {k: v.clone() for k, v in raw.items()}
    ref["type_logits"] += 0.3 * torch.randn(S, W, 3, device=device, generator=g)
    ref["mu"] = (ref["mu"] + 0.1 * torch.randn(S, W, M, device=device, generator=g)).clamp(0, 1)
    mask = torch.zeros(S, E, dtype=torch.bool, device=device)
    mask[:, 1] = True
    mask[:, 0] = torch.rand(S, device=device, generator=g) < 0.7
    lo = torch.randint(0, T, (S,), device=device, generator=g)
    ticks = torch.arange(T, device=device)
    raise_ok = (torch.rand(S, device=device, generator=g) >= 0.1)[:, None] & (ticks[None] >= lo[:, None])
    mask[:, 2:] = raise_ok
    legal_count = mask.sum(1)
    pick = (torch.rand(S, device=device, generator=g) * legal_count).long()
    action = (mask.cumsum(1) <= pick[:, None]).sum(1).to(torch.int32)
    old = -1.5 + 0.5 * torch.randn(S, W, device=device, generator=g)
    adv = torch.randn(S, W, device=device, generator=g)
    post = torch.rand(S, W, device=device, generator=g) * (torch.rand(S, W, device=device, generator=g) > 0.3)
    value = torch.randn(S, W, device=device, generator=g)
    old_value = value + 0.3 * torch.randn(S, W, device=device, generator=g)
    target = torch.randn(S, W, device=device, generator=g)
    controls = torch.tensor([[0.2, math.log(1.5), 0.5, 0.2, 0.01, 0.05, 0.0, 0.0, 1e-8, 1.0]], device=device)
    return dict(raw=raw, ref=ref, mask=mask, action=action, old=old, adv=adv, post=post if W > 1 else None,
                value=value, old_value=old_value, target=target, controls=controls)


def _events_ms(device, fn, reps):
    """Mean CUDA-event time (ms) of `fn` after two warm-up calls.  With PROFILE_ONE_FORWARD: one call
    between cudaProfilerStart/Stop after the warm-ups (no timing)."""

    import torch

    if PROFILE_ONE_FORWARD:
        fn()
        fn()
        torch.cuda.synchronize(device)
        torch.cuda.profiler.start()
        fn()
        torch.cuda.synchronize(device)
        torch.cuda.profiler.stop()
        return float("nan")
    for _ in range(2):
        fn()
    torch.cuda.synchronize(device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize(device)
    return a.elapsed_time(b) / reps


def _reference_pbg():
    """The reference package installed by the driver under baseline/_ref (None when absent)."""

    path = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(path, "pbg")):
        return None
    if path not in sys.path:
        sys.path.append(path)
    try:
        import pbg.core.learner  # noqa: F401
        import pbg.games.poker.queued.policy  # noqa: F401
    except Exception:  # the reference's own import failed on this box
        return None
    return path


def _reference_poker_loss_ms(device, d, reps):
    """The reference's own loss program on the same batch: pbg.core.learner.LearnerOperation.forward_loss
    with pbg's PokerPolicyOperator.learner, then (total * weight).sum().backward() (training.py:403)."""

    import torch
    from pbg.core.contracts import mode_schema
    from pbg.core.learner import LearnerOperation, LossConfig, ModelEvaluation, SequentialLearnerBatch
    from pbg.games.poker.queued.policy import PokerLegality, PokerPolicyOperator

    S, E = d["mask"].shape
    W = d["raw"]["type_logits"].shape[1]
    op = PokerPolicyOperator()
    legality = PokerLegality(torch.arange(E, dtype=torch.int32, device=device)[None].expand(S, -1).contiguous(),
                             d["mask"])

    def policy(input_type, model_input, raw_rows, act, private, owner, reference):
        return op.learner(raw_rows, legality, act, private, owner, reference)

    fields = {"model_input": torch.zeros(S, 1, device=device), "owner": torch.zeros(S, dtype=torch.int32, device=device),
              "action": d["action"], "old_log_policy": d["old"], "advantage_target": d["adv"],
              "old_value": d["old_value"], "value_target": d["target"]}
    if W == 1:
        fields["sampled_private_state"] = torch.zeros(S, 2, dtype=torch.int32, device=device)
    else:
        fields["posterior"] = d["post"]
    from types import MappingProxyType

    batch = SequentialLearnerBatch("post", torch.arange(S, device=device), MappingProxyType(fields))
    learner = LearnerOperation(mode_schema("self_play", "sequential", "sampled" if W == 1 else "rao_blackwell"),
                               LossConfig(), None, policy)
    leaves = {k: v.detach().clone().requires_grad_() for k, v in d["raw"].items()}
    value = d["value"].detach().clone().requires_grad_()
    weight = torch.ones(1, device=device)

    def step():
        for t in (*leaves.values(), value):
            t.grad = None
        res = learner.forward_loss(batch, iteration=0, lane_count=1, loss_controls=d["controls"],
                                   evaluation=ModelEvaluation(leaves, value), reference_raw=d["ref"])
        (res.total * weight).sum().backward()

    return _events_ms(device, step, reps)


def poker_loss_component(device, reps=10):
    """The fused poker learner objective (pbg_poker_learner_objective) on a sampled cfg2-size batch and a
    Rao-Blackwell batch over all 1,326 hands, beside the reference's own PyTorch CUDA loss program on the
    same batches when the driver installed it."""

    import torch
    from pbg_b200.learner import PokerLearnerObjective

    out = {}
    obj = PokerLearnerObjective(device)
    for name, S, W in (("sampled", 65_536, 1), ("rao_blackwell", 512, 1326)):
        d = _poker_loss_inputs(device, S, W, 202)
        lw = torch.ones(1, device=device)

        def run():
            obj(d["raw"], d["mask"], d["action"], d["old"], d["adv"], d["value"], d["old_value"], d["target"],
                d["controls"], lw, posterior=d["post"], reference_raw=d["ref"])

        ms = _events_ms(device, run, reps)
        if PROFILE_ONE_FORWARD:
            return {}
        rows = S * W
        # bytes: raw + reference fields (2 x 40 B at M = 2), gradient out (40 B), old/adv/post/value/targets
        # and the value gradient (7 x 4 B), the mask row and action shared by a sigma row's columns
        bytes_per_row = 40 + 40 + 40 + 28 + (202 + 4) / W
        entry = {"workload": f"HU 100bb R13 (E = 202 events, M = 2), {S} sigma rows x {W} private column(s), "
                             "reference KL, clipped value, one lane",
                 "ms": ms, "sigma_rows_per_s": S / (ms / 1e3), "policy_rows_per_s": rows / (ms / 1e3),
                 "hbm_gbs": rows * bytes_per_row / (ms / 1e3) / 1e9, "bytes_per_policy_row": bytes_per_row,
                 "bound": "SFU / FP32 issue (2 x (T+1) logistic edges per component per row, forward and backward)",
                 "kernel": "learner_objective_kernel", "gpu_launches": 1 if W == 1 else 2}
        if _reference_pbg() is not None:
            try:
                ref_ms = _reference_poker_loss_ms(device, d, max(2, reps // 2))
                entry["reference_torch_cuda_ms"] = ref_ms
                entry["speedup_vs_reference_torch_cuda"] = ref_ms / ms
            except torch.OutOfMemoryError:
                entry["reference_torch_cuda_ms"] = "out of memory"
        out[name] = entry
        del d
        torch.cuda.empty_cache()
    return out


def learner_step_component(device, rows=16_384, reps=20):
    """The learner step the metric counts, at cfg1: HU 8bb R4 (E = 18, K = 16 class rows, M = 2), the fp32
    preflop-class MLP (two hidden layers of 256, pbg_b200.mlp), `rows` sampled learner presentations:
    forward, fused poker objective, backward and AdamW, replayed from a CUDA graph.  Beside it, when the
    driver installed the reference, the same network in torch through the reference's own loss program
    (LearnerOperation.forward_loss with its PokerPolicyOperator.learner), autograd and torch AdamW."""

    import torch
    from pbg_b200.mlp import MLPLearnerStep, PreflopMLP
    from pbg_b200.poker import NLHEGeometry

    geometry = NLHEGeometry(2, 8.0, 4)
    model = PreflopMLP(geometry, device=device, seed=0)
    step = MLPLearnerStep(model)
    batch = _mlp_batch(device, geometry, rows)
    if PROFILE_ONE_FORWARD:  # one eager learner step between cudaProfilerStart/Stop
        _device_ms(device, lambda: step(batch))
        return {}
    for _ in range(3):
        step(batch)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step(batch)
    ms = _device_ms(device, graph.replay, reps)
    flops = 3 * 2 * rows * (model.inp * model.hidden + model.hidden ** 2 + model.hidden * model.out)
    out = {"workload": f"cfg1 learner step: HU 8bb R4, fp32 MLP {model.inp}-256-256-{model.out} "
                       f"({model.numel} parameters), {rows} sampled presentations, forward + fused objective + "
                       "backward + AdamW (one CUDA graph)",
           "ms": ms, "presentations_per_s": rows / (ms / 1e3), "gemm_tflops": flops / (ms / 1e3) / 1e12,
           "parameters": model.numel, "kernels": "cuBLAS sgemm x 8, mlp bias/heads/bias-gradient kernels, "
                                                 "learner_objective_kernel, adam"}
    if _reference_pbg() is not None:
        try:
            ref_ms = _reference_mlp_step_ms(device, model, geometry, batch, reps=max(3, reps // 4))
            out["reference_torch_cuda_ms"] = ref_ms
            out["reference_presentations_per_s"] = rows / (ref_ms / 1e3)
            out["speedup_vs_reference_torch_cuda"] = ref_ms / ms
        except Exception as exc:  # noqa: BLE001 - reported, not fatal
            out["reference_torch_cuda_ms"] = f"failed: {str(exc)[:200]}"
    return out


def _cfg2_model(device):
    """The cfg2 queued model: HU 100bb R13, d_model 128, 2 layers, 4 heads, class embedding 32, hidden 512,
    M = 2 (random weights)."""

    from pbg_b200.poker import NLHEGeometry
    from pbg_b200.preflop import PreflopConfig
    from pbg_b200.queued_model import QueuedPokerModel, parameter_shapes

    geo = NLHEGeometry(2, 100.0, 13)
    cfg = PreflopConfig(d_model=128, n_heads=4, layers=2, m_raise=2, k_act=5, max_players=2,
                        class_embedding_dim=32, ffn_hidden=512, max_history_tokens=geo.history_tokens)
    params = _random_params(parameter_shapes(cfg, 13), seed=29)
    return QueuedPokerModel(geo, cfg, params, device), geo, cfg, params


def _cfg2_learner_batches(device, model, pre_rows, post_rows, seed=41):
    """Learner batches of retained rows from a seeded rollout of the cfg2 geometry: the preflop rows of
    the roots and the heads-up postflop rows (post_2) of later steps, played by a fixed raw policy that
    mostly calls; each row's legal set from the state machine with a legal taken action, the dealt
    private hands as the sampled private state, the actor as owner, seeded old log policy, advantage,
    values and targets."""

    import torch
    from pbg_b200.family_rollout import FamilyRollout

    roll = FamilyRollout(model, seed=seed, iteration=3)
    hands = max(pre_rows, 4 * post_rows)
    arena, log_reach = roll.roots(hands, device=device)
    raw = roll._raw_buffers(hands, device)
    raw["type_logits"][..., 1] = 2.0  # mostly check/call, so that hands reach the flop
    machine = roll.machine
    found = {"pre": [], "post_2": []}
    need = {"pre": pre_rows, "post_2": post_rows}
    for _ in range(64):
        state = arena.state
        code = torch.where(state.terminal, -1, machine.input_type(state))
        for kind, value in (("pre", 0), ("post_2", 1)):
            have = sum(int(r.numel()) for r in found[kind][0::3]) if found[kind] else 0
            if have < need[kind]:
                rows = torch.nonzero(code == value).flatten()[: need[kind] - have]
                if rows.numel():
                    model_input, sub = roll._family_rows(arena, kind, rows, log_reach)
                    found[kind] += [rows, model_input, sub]
        if all((sum(int(r.numel()) for r in found[k][0::3]) if found[k] else 0) >= need[k] for k in need):
            break
        roll.stepper.step(arena, raw)
        roll.stepper.reach_update(arena, raw, log_reach)
    g = torch.Generator(device=device).manual_seed(seed)
    batches = []
    for kind in ("pre", "post_2"):
        parts = found[kind]
        model_input = torch.cat(parts[1::3])
        subs = parts[2::3]
        private = torch.cat([s.combo_ids for s in subs]).to(torch.int32)
        owner = torch.cat([s.to_act for s in subs]).to(torch.int64)
        mask = torch.cat([machine.legality(s).mask for s in subs])
        S = model_input.shape[0]
        pick = (torch.rand(S, device=device, generator=g) * mask.sum(1)).long()
        action = (mask.cumsum(1) <= pick[:, None]).sum(1).to(torch.int32)
        value = torch.randn(S, 1, device=device, generator=g)
        batches.append({"input_type": kind, "model_input": model_input, "sampled_private_state": private,
                        "owner": owner, "mask": mask, "action": action,
                        "old_log_policy": -1.5 + 0.5 * torch.randn(S, 1, device=device, generator=g),
                        "advantage_target": torch.randn(S, 1, device=device, generator=g),
                        "old_value": value + 0.3 * torch.randn(S, 1, device=device, generator=g),
                        "value_target": torch.randn(S, 1, device=device, generator=g),
                        "controls": torch.tensor([[0.2, math.log(1.5), 0.5, 0.2, 0.01, 0.05, 0.0, 0.0, 1e-8, 1.0]],
                                                 device=device),
                        "lane_weight": torch.ones(1, device=device)})
    return batches


def _reference_cfg2_step_ms(device, cfg, params, batches, reps):
    """The same learner step on the reference's PyTorch CUDA path: pbg's own QueuedPokerModel (SDPA
    attention) with the same weights, its learner_operation and LearnerOperation.forward_loss under bf16
    autocast (training.py:381-403), pbg's PokerPolicyOperator.learner, autograd, torch AdamW."""

    import dataclasses
    from types import MappingProxyType

    import torch
    from pbg.core.contracts import mode_schema
    from pbg.core.learner import LearnerOperation, LossConfig, SequentialLearnerBatch
    from pbg.games.poker.model.preflop import PokerModelConfig
    from pbg.games.poker.queued.hooks import NLHEGeometry as RefGeometry
    from pbg.games.poker.queued.model import QueuedPokerModel as RefModel
    from pbg.games.poker.queued.policy import PokerLegality, PokerPolicyOperator

    model = RefModel(RefGeometry(2, 100.0, 13), PokerModelConfig(**dataclasses.asdict(cfg))).to(device)
    with torch.no_grad():
        for name, param in model.named_parameters():
            param.copy_(params[name].to(device))
    opt = torch.optim.AdamW(list(model.parameters()), lr=3e-4, weight_decay=0.0)
    op = PokerPolicyOperator()
    prepared = []
    for b in batches:
        S, E = b["mask"].shape
        legality = PokerLegality(torch.arange(E, dtype=torch.int32, device=device)[None].expand(S, -1).contiguous(),
                                 b["mask"])

        def policy(input_type, model_input, raw_rows, act, private, owner, reference, legality=legality):
            return op.learner(raw_rows, legality, act, private, owner, reference)

        fields = {k: b[k] for k in ("model_input", "owner", "action", "old_log_policy", "advantage_target",
                                    "old_value", "value_target", "sampled_private_state")}
        physical = SequentialLearnerBatch(b["input_type"], torch.arange(S, device=device), MappingProxyType(fields))
        learner = LearnerOperation(mode_schema("self_play", "sequential", "sampled"), LossConfig(), None, policy)
        prepared.append((b, physical, learner))

    def step():
        opt.zero_grad(set_to_none=True)
        for b, physical, learner in prepared:
            with torch.autocast("cuda", dtype=torch.bfloat16):
                evaluation = model.learner_operation(b["input_type"], b["model_input"], b["sampled_private_state"],
                                                     b["owner"])
                result = learner.forward_loss(physical, iteration=0, lane_count=1, loss_controls=b["controls"],
                                              evaluation=evaluation)
            (result.total * b["lane_weight"]).sum().backward()
        opt.step()

    return _events_ms(device, step, reps)


def learner_step_cfg2_component(device, pre_rows=1024, post_rows=256, reps=3):
    """The learner step the metric counts, at cfg2: HU 100bb R13 with the cfg2 attention network (d_model
    128, 2 layers, 4 heads), `pre_rows` preflop and `post_rows` heads-up postflop learner presentations
    (sampled private rows) from a seeded rollout: the training forward on this build's kernels, the fused
    poker objective, the backward (pbg_b200.model_train) and AdamW.  Beside it, when the driver installed
    the reference, the same step on the reference's own PyTorch CUDA path with the same weights."""

    import torch
    from pbg_b200.model_train import ModelLearnerStep

    model, geo, cfg, params = _cfg2_model(device)
    batches = _cfg2_learner_batches(device, model, pre_rows, post_rows)
    step = ModelLearnerStep(model)
    if PROFILE_ONE_FORWARD:
        _device_ms(device, lambda: step(batches), 1)
        return {}
    step(batches)  # warm-up (bindings, first launches)
    ms = _events_ms(device, lambda: step(batches), reps)
    per_family = {}
    for b in batches:
        per_family[b["input_type"]] = _events_ms(device, lambda b=b: step.gradient([b]), reps)
    rows = sum(b["model_input"].shape[0] for b in batches)
    out = {"workload": f"cfg2 learner step: HU 100bb R13, cfg2 network (d_model 128, 2 layers, 4 heads, "
                       f"{step.flat.numel} parameters), {pre_rows} preflop + {post_rows} postflop (post_2) "
                       "sampled presentations, training forward + fused objective + backward + AdamW",
           "ms": ms, "presentations_per_s": rows / (ms / 1e3), "parameters": step.flat.numel,
           "forward_backward_ms_by_family": per_family,
           "kernels": "linear_tcgen05_kernel, attention_kernel (with log-sum-exp), layernorm, incidence_combine; "
                      "backward: attention_dq_kernel + attention_dkv_kernel (fused), gelu / layernorm / "
                      "incidence-combine backward kernels, cuBLAS bf16 GEMMs for the maps' dX and dW; "
                      "learner_objective_kernel, adam"}
    if _reference_pbg() is not None:
        try:
            ref_ms = _reference_cfg2_step_ms(device, cfg, params, batches, reps=reps)
            out["reference_torch_cuda_ms"] = ref_ms
            out["reference_presentations_per_s"] = rows / (ref_ms / 1e3)
            out["speedup_vs_reference_torch_cuda"] = ref_ms / ms
        except Exception as exc:  # noqa: BLE001 - reported, not fatal
            out["reference_torch_cuda_ms"] = f"failed: {str(exc)[:300]}"
    return out


def learner_scaling(args, device, world, rank, rows=16_384):
    """cfg1 learner step, data parallel: each rank runs forward, objective and backward over its own
    `rows` presentations (CUDA graph), the flat gradient (172,720 fp32) is SUM-all-reduced with NCCL,
    then AdamW (CUDA graph).  Weak scaling; the step is timed with CUDA events, max over ranks."""

    import torch
    import torch.distributed as dist
    from pbg_b200.mlp import MLPLearnerStep, PreflopMLP
    from pbg_b200.poker import NLHEGeometry

    geometry = NLHEGeometry(2, 8.0, 4)
    model = PreflopMLP(geometry, device=device, seed=0)  # the same initial weights on every rank
    step = MLPLearnerStep(model)
    batch = _mlp_batch(device, geometry, rows, seed=5 + rank)
    for _ in range(3):
        step(batch)
    torch.cuda.synchronize(device)
    g_grad, g_adam = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_grad):
        step.gradient(batch)
    with torch.cuda.graph(g_adam):
        step.adam.step()

    def one():
        g_grad.replay()
        if world > 1:
            dist.all_reduce(step.adam.grad)
        g_adam.replay()

    for _ in range(max(3, args.warmup)):
        one()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        one()
    b.record()
    torch.cuda.synchronize(device)
    ms = a.elapsed_time(b) / args.steps
    t = torch.tensor([ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
    del g_grad, g_adam
    if rank == 0:
        ms = float(t)
        print(json.dumps({"metric": "learner presentations/s (cfg1 learner step, data parallel)",
                          "value": world * rows / (ms / 1e3), "unit": "presentations/s", "n_gpus": world,
                          "steps": args.steps, "ms_per_step": ms, "scaling": "weak",
                          "config": {"workload": f"HU 8bb R4, fp32 MLP ({model.numel} parameters), {rows} "
                                                 "presentations per rank per step, NCCL SUM of the flat gradient"}}))


def learner_scaling_cfg2(args, device, world, rank, pre_rows=1024, post_rows=256):
    """cfg2 learner step, data parallel: each rank runs the training forward, fused objective and backward
    of the attention network over its own presentations (`pre_rows` preflop + `post_rows` postflop from a
    rollout seeded by the rank), the flat gradient (4,226,931 fp32) is SUM-all-reduced with NCCL, then
    AdamW.  Weak scaling; timed with CUDA events, max over ranks."""

    import torch
    import torch.distributed as dist
    from pbg_b200.model_train import ModelLearnerStep

    model, _, _, _ = _cfg2_model(device)  # the same initial weights on every rank
    batches = _cfg2_learner_batches(device, model, pre_rows, post_rows, seed=41 + rank)
    step = ModelLearnerStep(model)

    def one():
        step.gradient(batches)
        if world > 1:
            dist.all_reduce(step.adam.grad)
        step.adam.step()

    for _ in range(max(3, args.warmup)):
        one()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    steps = min(args.steps, 10)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        one()
    b.record()
    torch.cuda.synchronize(device)
    ms = a.elapsed_time(b) / steps
    t = torch.tensor([ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
    if rank == 0:
        ms = float(t)
        rows = pre_rows + post_rows
        print(json.dumps({"metric": "learner presentations/s (cfg2 learner step, data parallel)",
                          "value": world * rows / (ms / 1e3), "unit": "presentations/s", "n_gpus": world,
                          "steps": steps, "ms_per_step": ms, "scaling": "weak",
                          "config": {"workload": f"HU 100bb R13, cfg2 attention network ({step.flat.numel} "
                                                 f"parameters), {pre_rows} preflop + {post_rows} postflop "
                                                 "presentations per rank per step, NCCL SUM of the flat gradient"}}))


def _mlp_batch(device, geometry, S, seed=5):
    import torch

    d = _poker_loss_inputs(device, S, 1, geometry.events, seed=seed)
    g = torch.Generator(device=device).manual_seed(seed + 1)
    return {"model_input": torch.randn(S, geometry.preflop_model_input_width, device=device, generator=g),
            "sampled_class": torch.randint(0, geometry.private_classes, (S,), device=device, generator=g),
            "mask": d["mask"], "action": d["action"], "old_log_policy": d["old"], "advantage_target": d["adv"],
            "old_value": d["old_value"], "value_target": d["target"], "controls": d["controls"],
            "lane_weight": torch.ones(1, device=device)}


def _reference_mlp_step_ms(device, model, geometry, batch, reps):
    """The same learner step on the reference's PyTorch CUDA path: torch modules for the network (the
    reference heads' activations), pbg's LearnerOperation.forward_loss with pbg's
    PokerPolicyOperator.learner, (total * weight).sum().backward() (training.py:403), torch AdamW."""

    import torch
    from types import MappingProxyType

    from pbg.core.contracts import mode_schema
    from pbg.core.learner import LearnerOperation, LossConfig, ModelEvaluation, SequentialLearnerBatch
    from pbg.games.poker.queued.policy import PokerLegality, PokerPolicyOperator

    S = batch["model_input"].shape[0]
    E = geometry.events
    K, R, M = model.K, model.row, model.M
    params = {k: v.detach().clone().requires_grad_() for k, v in model.params.items()}
    opt = torch.optim.AdamW(list(params.values()), lr=3e-4, weight_decay=0.0)
    op = PokerPolicyOperator()
    legality = PokerLegality(torch.arange(E, dtype=torch.int32, device=device)[None].expand(S, -1).contiguous(),
                             batch["mask"])

    def policy(input_type, model_input, raw_rows, act, private, owner, reference):
        return op.learner(raw_rows, legality, act, private, owner, reference)

    fields = {"model_input": batch["model_input"], "owner": torch.zeros(S, dtype=torch.int32, device=device),
              "action": batch["action"], "old_log_policy": batch["old_log_policy"],
              "advantage_target": batch["advantage_target"], "old_value": batch["old_value"],
              "value_target": batch["value_target"],
              "sampled_private_state": torch.zeros(S, 2, dtype=torch.int32, device=device)}
    ref_batch = SequentialLearnerBatch("pre", torch.arange(S, device=device), MappingProxyType(fields))
    learner = LearnerOperation(mode_schema("self_play", "sequential", "sampled"), LossConfig(), None, policy)
    rows = torch.arange(S, device=device)
    cls = batch["sampled_class"].long()

    def step():
        opt.zero_grad(set_to_none=True)
        x = batch["model_input"]
        h1 = torch.relu(torch.nn.functional.linear(x, params["w1"], params["b1"]))
        h2 = torch.relu(torch.nn.functional.linear(h1, params["w2"], params["b2"]))
        z = torch.nn.functional.linear(h2, params["w3"], params["b3"])
        r = z[:, :K * R].reshape(S, K, R)[rows, cls]
        raw = {"type_logits": r[:, None, :3], "omega": torch.softmax(r[:, 3:3 + M], -1)[:, None],
               "mu": torch.sigmoid(r[:, 3 + M:3 + 2 * M])[:, None],
               "s": (torch.nn.functional.softplus(r[:, 3 + 2 * M:3 + 3 * M]) + model.s_min)[:, None],
               "iota": torch.sigmoid(r[:, 3 + 3 * M])[:, None]}
        value = z[rows, K * R + cls][:, None]
        res = learner.forward_loss(ref_batch, iteration=0, lane_count=1, loss_controls=batch["controls"],
                                   evaluation=ModelEvaluation(raw, value))
        (res.total * batch["lane_weight"]).sum().backward()
        opt.step()

    return _events_ms(device, step, reps)


def reference_torch_loss_component(device, inputs, reps=5):
    """The reference's own PyTorch CUDA loss program on the cfg5 rows: pbg.core.learner.LearnerOperation
    .forward_loss (sampled, sequential, unmodified, from baseline/_ref) over the same 4,194,304 x 8 bf16
    logits, masks, actions, old log pi and advantages, with a categorical policy operation (masked
    log-softmax selected log pi and entropy in torch, the math of the reference's game-neutral fixture
    tests/categorical_policy_fixture.py), then (total * weight).sum().backward() for d logits."""

    import torch
    from types import MappingProxyType

    from pbg.core.contracts import mode_schema
    from pbg.core.learner import (EntropyLossConfig, LearnerOperation, LossConfig, ModelEvaluation,
                                  PolicyEvaluation, SequentialLearnerBatch, ValueLossConfig)

    logits, mask, action, old, adv, weight = inputs
    N, A = logits.shape
    legal = mask.bool()

    def policy(input_type, model_input, raw, act, private, owner, reference):
        x = raw["logits"].reshape(N, A).float().masked_fill(~legal, -torch.inf)
        logp = torch.log_softmax(x, -1)
        sel = logp.gather(1, act.long()[:, None]).squeeze(1)
        prob = logp.exp()
        ent = -(prob * torch.where(legal, logp, torch.zeros_like(logp))).sum(-1)
        return PolicyEvaluation(sel, ent, torch.zeros_like(sel))

    fields = MappingProxyType({
        "model_input": torch.zeros(N, 1, device=device), "owner": torch.zeros(N, dtype=torch.int32, device=device),
        "sampled_private_state": torch.zeros(N, 2, dtype=torch.int32, device=device), "action": action,
        "old_log_policy": old[:, None], "old_value": torch.zeros(N, 1, device=device),
        "value_target": torch.zeros(N, 1, device=device), "advantage_target": adv[:, None]})
    batch = SequentialLearnerBatch("pre", torch.arange(N, device=device), fields)
    cfg = LossConfig(policy_clip=0.2, value=ValueLossConfig(coefficient=0.0),
                     entropy=EntropyLossConfig(coefficient=0.01))
    learner = LearnerOperation(mode_schema("self_play", "sequential", "sampled"), cfg, None, policy,
                               precision="bf16")
    leaf = logits.detach().clone().requires_grad_()
    value = torch.zeros(N, 1, device=device)
    controls = learner.controls((cfg,), 0, device)

    def step():
        leaf.grad = None
        res = learner.forward_loss(batch, iteration=0, lane_count=1, loss_controls=controls,
                                   evaluation=ModelEvaluation({"logits": leaf[:, None, :]}, value))
        res.total.sum().backward()

    ms = _events_ms(device, step, reps)
    del leaf
    torch.cuda.empty_cache()
    return {"workload": "cfg5 rows (4,194,304 x 8, bf16 logits): the reference's LearnerOperation.forward_loss "
                        "+ backward on the device, inputs resident",
            "ms_per_step": ms, "value": N / (ms / 1e3), "unit": UNIT, "source": "baseline/_ref (pbg, unmodified)"}


# ----------------------------------------------------------- the reference's engine, with and without the drop-ins

ENGINE_CONFIG = """kind: nlhe_run_v1
scientific:
  mode: {{training_regime: self_play, rollout_mode: sequential, private_estimator: sampled}}
  game: {{players: 2, stack_bb: 8.0, rank_count: 4}}
  model:
    d_model: 64
    n_heads: 4
    layers: 2
    raises: {{components: 2, minimum_scale: 0.02}}
    class_embedding_dim: 8
    ffn_hidden: 128
    folder_beta_rank: 0
    folder_line_dim: 8
    epsilon: 1.0e-8
  objective:
    policy_clip: 0.2
    value: {{kind: mse, coefficient: 0.5}}
    entropy: {{kind: constant, coefficient: 0.01}}
  optimizer: {{kind: adamw, learning_rate: 0.0003, beta1: 0.9, beta2: 0.999, epsilon: 1.0e-8, weight_decay: 0.0,
              grad_clip: 1.0}}
  schedule: {{batch_size: 1024, epochs: 1}}
  lambda: 0.95
run:
  seed: 0
  reproducibility: strict
  utility: raw_bb
  workload: {{roots: {roots}}}
  execution:
    device: cuda:0
    precision: fp32
    attention: sdpa
    memory: {{reserve_bytes: 67108864}}
    microbatch: auto
    tensor_program: {{mode: {program}}}
  iterations: {iterations}
  checkpoint_every: 100000
  output_dir: {out}
"""


def engine_arm(args):
    """One arm of --engine-compare in this process: a TrainingSession of the config above, timed per iteration
    (CUDA-synchronised wall clock: an iteration is host-scheduled work spanning many kernels)."""

    import tempfile

    import torch

    sys.path.append(os.path.join(ROOT, "baseline", "_ref"))
    if args.engine_arm.startswith("b200"):
        from pbg_b200 import engine

        engine.install(learner=True)
    from pbg.config import load_config
    from pbg.runtime import TrainingSession

    out = tempfile.mkdtemp(prefix="engine-")
    path = os.path.join(out, "cfg.yaml")
    program = "eager" if args.engine_arm.endswith("_eager") else "captured"
    with open(path, "w") as f:
        f.write(ENGINE_CONFIG.format(roots=args.engine_roots, iterations=args.engine_iterations, program=program,
                                     out=out))
    session = TrainingSession(load_config(path), benchmark_telemetry=True)
    rows = []
    for _ in range(args.engine_iterations):
        torch.cuda.synchronize()
        t = time.perf_counter()
        result = session.step()
        torch.cuda.synchronize()
        wall = time.perf_counter() - t
        lanes = [lane for lane in getattr(result, "results", (result,)) if lane is not None]
        rows.append({"seconds": wall, "player_nodes": sum(int(lane.player_nodes) for lane in lanes),
                     "presentations": sum(int(lane.learner.statistical_presentations) for lane in lanes)})
        tele = getattr(lanes[0], "telemetry", None) if lanes else None
        if tele is not None:
            rows[-1]["telemetry"] = {"rollout_seconds": tele.rollout_seconds,
                                     "model_inference_seconds": tele.model_inference_seconds,
                                     "target_propagation_seconds": tele.target_propagation_seconds,
                                     "host_synchronizations": tele.host_synchronizations,
                                     "phases": {k: dict(v) for k, v in tele.phase_measurements.items()}}
    print(json.dumps({"arm": args.engine_arm, "program": program, "iterations": rows}), flush=True)


def engine_compare(args):
    """Both arms in fresh processes; steady state = every iteration after the first two (compilation and
    capture happen in the first iterations of the reference's captured tensor programs)."""

    env = dict(os.environ, TORCH_CUDA_ARCH_LIST=os.environ.get("TORCH_CUDA_ARCH_LIST", "10.0"))
    arms = {}
    for arm in ("reference", "b200"):
        proc = subprocess.run([sys.executable, os.path.abspath(__file__), "--engine-arm", arm, "--engine-roots",
                               str(args.engine_roots), "--engine-iterations", str(args.engine_iterations)],
                              capture_output=True, text=True, env=env, timeout=1500)
        lines = [line for line in proc.stdout.splitlines() if line.startswith("{")]
        if proc.returncode != 0 or not lines:
            arms[arm] = {"error": proc.stderr[-2000:]}
            continue
        data = json.loads(lines[-1])
        steady = data["iterations"][2:] or data["iterations"]
        seconds = sum(r["seconds"] for r in steady)
        data["player_nodes_per_s"] = sum(r["player_nodes"] for r in steady) / seconds
        data["learner_presentations_per_s"] = sum(r["presentations"] for r in steady) / seconds
        data["seconds_per_iteration"] = seconds / len(steady)
        arms[arm] = data
    line = {"metric": "reference training iteration: player nodes/s and learner presentations/s",
            "workload": f"pbg.runtime.TrainingSession, HU 8bb R4 self-play, sampled, {args.engine_roots} roots per "
                        "iteration, transformer d64 / 2 layers, batch 1024, fp32; steady state after 2 iterations",
            "reference": arms.get("reference"), "reference_eager": arms.get("reference_eager"),
            "b200": arms.get("b200")}
    ref, b200 = arms.get("reference", {}), arms.get("b200", {})
    if "player_nodes_per_s" in ref and "player_nodes_per_s" in b200:
        line["speedup_player_nodes"] = b200["player_nodes_per_s"] / ref["player_nodes_per_s"]
        line["speedup_presentations"] = b200["learner_presentations_per_s"] / ref["learner_presentations_per_s"]
    eager = arms.get("reference_eager", {})
    if "player_nodes_per_s" in eager and "player_nodes_per_s" in b200:
        line["speedup_vs_reference_eager"] = b200["player_nodes_per_s"] / eager["player_nodes_per_s"]
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------- rollout component


ROLLOUT_BYTES_HU = 64 * 2 + 40 + 16 + 8 + 16 + 25 + 110 + 100  # state r+w, raw row, address, outputs, history


def rollout_component(device, hands=65_536, seed=0):
    """Fused rollout step over a full self-play rollout (HU 100bb, 13 ranks, cfg2's 65,536 hands).

    A fixed seeded raw policy row per hand (the model is not on this path yet) drives every step.
    The same rollout runs once untimed to count the decisions each step makes (it is deterministic),
    then again timed with CUDA events around every step, each step replayed from a CUDA graph.
    """

    import torch
    from pbg_b200.poker import NLHEGeometry
    from pbg_b200.rollout import RolloutStep

    geometry = NLHEGeometry(2, 100.0, 13)
    stepper = RolloutStep(geometry, seed=seed, iteration=0)
    g = torch.Generator(device=device).manual_seed(seed + 7)
    raw = {"type_logits": torch.randn((hands, 1, 3), generator=g, device=device),
           "omega": torch.softmax(torch.randn((hands, 1, 2), generator=g, device=device), -1),
           "mu": torch.rand((hands, 1, 2), generator=g, device=device),
           "s": torch.rand((hands, 1, 2), generator=g, device=device) * 0.3 + 0.02,
           "iota": torch.rand((hands, 1), generator=g, device=device) * 0.2}
    counts = []
    arena = stepper.roots(hands, device=device)
    if PROFILE_ONE_FORWARD:  # one eager rollout to terminal, every step a profiled launch
        torch.cuda.profiler.start()
    for _ in range(400):
        active = int((~arena.state.terminal).sum())
        if active == 0:
            break
        counts.append(active)
        stepper.step(arena, raw)
    if PROFILE_ONE_FORWARD:
        torch.cuda.synchronize(device)
        torch.cuda.profiler.stop()
        return {}
    arena = stepper.roots(hands, device=device)
    stream = torch.cuda.current_stream(device)
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in counts]
    torch.cuda.synchronize(device)
    # one step over fixed arena buffers, replayed from a CUDA graph (no host gaps between steps)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        stepper.step(arena, raw)
    torch.cuda.synchronize(device)
    for a, b in events:
        a.record(stream)
        graph.replay()
        b.record(stream)
    torch.cuda.synchronize(device)
    assert bool(arena.state.terminal.all())
    times = [a.elapsed_time(b) for a, b in events]
    total_ms = sum(times)
    decisions = sum(counts)
    peak, _ = measured_peak()
    achieved = ROLLOUT_BYTES_HU * decisions / (total_ms / 1000.0) / 1e9
    return {"workload": "fused rollout step, HU 100bb R13, 65,536 hands to terminal, raw policy at the actor row",
            "decisions": decisions, "steps": len(counts), "ms": total_ms,
            "decisions_per_s": decisions / (total_ms / 1000.0),
            "first_step_us": 1000.0 * times[0], "step_us": [round(1000.0 * t, 1) for t in times],
            "live_hands": counts,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "bytes_per_decision": ROLLOUT_BYTES_HU,
                         "kernel": "rollout_step_kernel"},
            "gpu_launches": len(counts)}


def targets_component(device, lanes=256, depth=8, branching=2, p_train=2, width=8, reps=20):
    """Layered lambda-return targets over a seeded full binary forest (RB, branched: the widest mode).

    The forest is re-seeded from pristine work arenas before every pass (a device copy outside the
    timed region); each pass is ONE cooperative launch over all layers, timed with CUDA events that
    are queued behind a device-side sleep (so they bracket the kernel, not the host's launch latency).
    """

    import torch
    from pbg_b200.targets import INT32_MAX, LayeredTargets, synthetic_tree_plan

    args, info = synthetic_tree_plan(lanes, depth, branching, p_train, width, device=device, seed=5)
    bound = LayeredTargets(*args)
    live = [args[3][0], args[4][0], args[5][0], args[6][0], args[7][0]]  # work0, work1, trace, cost, delta
    pristine = [x.clone() for x in live]
    stream = torch.cuda.current_stream(device)
    times = []
    # every timed launch is queued behind a device-side sleep, so the events bracket the kernel
    # rather than the host's launch latency
    for rep in range(reps + 3):
        for dst, src in zip(live, pristine):
            dst.copy_(src)
        torch.cuda._sleep(1_000_000)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        failure = bound.launch()
        b.record(stream)
        torch.cuda.synchronize(device)
        if rep >= 3:
            times.append(a.elapsed_time(b))
    if not bool((failure == INT32_MAX).all()):
        raise RuntimeError("layered targets reported a failed lane on the synthetic forest")
    ms = sorted(times)[len(times) // 2]
    # the fixed cost of one inter-layer grid barrier: the same launch over 1 and over 65 empty layers
    empty = []
    for layers in (1, 65):
        plan = list(args)
        plan[0] = torch.zeros(layers + 1, dtype=torch.int32)
        hollow = LayeredTargets(*plan)
        samples = []
        for rep in range(13):
            torch.cuda._sleep(1_000_000)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            hollow.launch()
            b.record(stream)
            torch.cuda.synchronize(device)
            if rep >= 3:
                samples.append(a.elapsed_time(b))
        empty.append(sorted(samples)[len(samples) // 2])
    barrier_us = 1000.0 * (empty[1] - empty[0]) / 64
    peak, _ = measured_peak()
    achieved = info["algorithmic_bytes"] / (ms / 1000.0) / 1e9
    return {"workload": f"layered targets, {lanes} lanes x full binary tree of depth {depth}, "
                        f"{info['estimator']} {info['rollout']}, P={p_train}, width {width}",
            "nodes": info["nodes"], "layers": depth, "us_per_pass": 1000.0 * ms,
            "grid_barrier_us": barrier_us, "empty_launch_us": 1000.0 * empty[0],
            "nodes_per_s": info["nodes"] / (ms / 1000.0),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "bytes_per_node": info["bytes_per_node"],
                         "kernel": "layered_targets_kernel"},
            "gpu_launches": 1}


def model_linear_component(device, rows=524_288, reps=10):
    """The model's dense maps on the tensor cores (pbg_linear_bf16) at d_model 256, hidden 1024:
    attention in-projection (256 -> 768), FFN w1 with fused GELU (256 -> 1024), FFN w2 (1024 -> 256),
    over `rows` token rows (about 600 preflop sequences of cfg2's 876 tokens).  Each launch is queued
    behind a device-side sleep; inputs are larger than L2."""

    import torch
    from pbg_b200.model import linear, pipeline_error

    _, peak_kind = measured_peak()
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tflops_peak = float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        tflops_peak = 1590.0
    g = torch.Generator(device=device).manual_seed(11)
    out = {}
    for name, k, n, act in (("w_qkv", 256, 768, None), ("ffn_w1_gelu", 256, 1024, "gelu"),
                            ("ffn_w2", 1024, 256, None)):
        x = (torch.randn((rows, k), generator=g, device=device) / 2).to(torch.bfloat16)
        w = (torch.randn((n, k), generator=g, device=device) / k ** 0.5).to(torch.bfloat16)
        b = torch.randn((n,), generator=g, device=device) * 0.1
        y = torch.empty((rows, n), dtype=torch.bfloat16, device=device)
        times = []
        for rep in range(reps + 3):
            torch.cuda._sleep(1_000_000)
            a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            linear(x, w, b, act, out=y)
            e.record()
            torch.cuda.synchronize(device)
            if rep >= 3:
                times.append(a.elapsed_time(e))
        if pipeline_error(device):
            raise RuntimeError("linear layer pipeline wait ran out")
        ms = sorted(times)[len(times) // 2]
        flops = 2.0 * rows * n * k
        nbytes = 2.0 * (rows * k + n * k + rows * n) + 4.0 * n
        out[name] = {"m": rows, "k": k, "n": n, "us": 1000.0 * ms, "tflops": flops / ms / 1e9,
                     "frac_tensor": flops / ms / 1e9 / tflops_peak, "gbs": nbytes / ms / 1e6}
        del x, w, y
    return {"workload": f"tcgen05 linear layers over {rows} bf16 token rows (d_model 256, hidden 1024)",
            "layers": out, "peak_tflops": tflops_peak, "peak_kind": peak_kind, "kernel": "linear_tcgen05_kernel",
            "gpu_launches": 3}


def model_attention_component(device, batch=600, length=876, heads=8, reps=10):
    """The model's reach-biased self-attention core (pbg_attention_bf16) at cfg2's preflop sequence
    length: `batch` sequences x `length` tokens x `heads` heads of width 32, fp32 key bias and key mask.
    Each launch queued behind a device-side sleep."""

    import math

    import torch
    from pbg_b200.model import attention, pipeline_error

    g = torch.Generator(device=device).manual_seed(13)
    qkv = torch.randn((batch, length, 3 * heads * 32), generator=g, device=device).to(torch.bfloat16)
    bias = torch.randn((batch, length), generator=g, device=device)
    mask = torch.rand((batch, length), generator=g, device=device) > 0.1
    q_scale = torch.full((heads,), 1.0 / math.sqrt(32), device=device)
    times = []
    for rep in range(reps + 3):
        torch.cuda._sleep(1_000_000)
        a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        attention(qkv, heads, q_scale, bias, mask)
        e.record()
        torch.cuda.synchronize(device)
        if rep >= 3:
            times.append(a.elapsed_time(e))
    if pipeline_error(device):
        raise RuntimeError("attention pipeline wait ran out")
    ms = sorted(times)[len(times) // 2]
    flops = 4.0 * batch * heads * length * length * 32
    exps = float(batch * heads * length * length)
    return {"workload": f"reach-biased attention core, {batch} sequences x {length} tokens x {heads} heads (width 32)",
            "us": 1000.0 * ms, "tflops": flops / ms / 1e9, "exp_per_s": exps / (ms / 1000.0),
            "bound": "SFU/latency (softmax); the tensor pipe does 2 MMAs of 128x128x32 and 8 of 128x32x16 per key block",
            "kernel": "attention_kernel", "gpu_launches": 1}


def profile_attention(device, batch=48, length=2406, heads=8):
    """Two warm-up launches of the attention core at the postflop sequence length, then one between
    cudaProfilerStart/Stop (qkv 177 MB: larger than L2)."""

    import math

    import torch
    from pbg_b200.model import attention

    g = torch.Generator(device=device).manual_seed(14)
    qkv = torch.randn((batch, length, 3 * heads * 32), generator=g, device=device).to(torch.bfloat16)
    bias = torch.randn((batch, length), generator=g, device=device)
    mask = torch.rand((batch, length), generator=g, device=device) > 0.1
    q_scale = torch.full((heads,), 1.0 / math.sqrt(32), device=device)
    for _ in range(2):
        attention(qkv, heads, q_scale, bias, mask)
    torch.cuda.synchronize(device)
    torch.cuda.profiler.start()
    attention(qkv, heads, q_scale, bias, mask)
    torch.cuda.synchronize(device)
    torch.cuda.profiler.stop()


def preflop_forward_component(device, batch=256, players=2, history=16, reps=5):
    """The preflop policy/value network forward (pbg_b200.preflop, the reference's default
    PokerModelConfig: d_model 256, 8 heads, 6 layers, hidden 1024, R13 -> 169 class rows per seat)
    for `batch` heads-up decisions with `history` public-history tokens; random weights of that
    architecture, synthetic public batch.  Timed with CUDA events (host orchestration included)."""

    import torch
    from pbg_b200.preflop import PreflopConfig, PreflopModel, parameter_shapes

    cfg = PreflopConfig()
    model = PreflopModel(cfg, 13, _random_params(parameter_shapes(cfg, 13)), device)
    pub = _synthetic_pub(device, batch, players, history, street=0)
    d = torch.Generator(device=device).manual_seed(19)
    ranges = torch.rand((batch, players, 169), generator=d, device=device)
    ms, eager_ms = _time_forward(device, lambda: model.forward(pub, ranges), reps)
    tokens = players * 169 + 1 + 4 * players + 1 + 4 + 1 + 2 + 5 + history + 1 + cfg.k_act
    return {"workload": f"preflop policy/value forward, default PokerModelConfig, R13 heads-up, {batch} decisions, "
                        f"{tokens} tokens each", "ms": ms, "eager_ms": eager_ms, "launch": "CUDA graph replay",
            "decisions_per_s": batch / (ms / 1000.0),
            "class_rows_per_s": batch * 169 / (ms / 1000.0), "token_rows_per_s": batch * tokens / (ms / 1000.0),
            "kernels": ["linear_tcgen05_kernel", "attention_kernel", "layernorm_kernel"]}


def postflop_forward_component(device, batch=24, players=2, history=16, reps=5):
    """The compact postflop policy/value network forward (pbg_b200.postflop, default PokerModelConfig,
    R13) for `batch` heads-up flop decisions: 1,176 board-compatible combo rows per live seat, evaluator
    summary with hand log ratios and rank-16 beta eigenpairs; random weights of that architecture,
    synthetic public batch.  Timed with CUDA events over CUDA-graph replay (and eagerly)."""

    import torch
    from pbg_b200.postflop import PostflopMasks, PostflopModel, input_errors, parameter_shapes
    from pbg_b200.preflop import PreflopConfig

    cfg = PreflopConfig()
    model = PostflopModel(cfg, 13, _random_params(parameter_shapes(cfg, 13)), device)
    pub = _synthetic_pub(device, batch, players, history, street=1)
    g = torch.Generator().manual_seed(20)
    hands = 1326
    combos = torch.combinations(torch.arange(52), 2)
    board = torch.stack([torch.randperm(52, generator=g)[:3] for _ in range(batch)])
    pub["board"] = torch.cat((board, torch.full((batch, 2), -1, dtype=torch.long)), 1).to(device)
    compat = ~(combos[None, :, :, None] == board[:, None, None, :]).any(-1).any(-1)
    compact = 1176
    vector = torch.randn((batch, 52, 16), generator=g)
    summary = {"hand_log_ratio": torch.randn((batch, hands), generator=g).to(device) * 0.3,
               "beta_eigenvalue": torch.randn((batch, 16), generator=g).to(device),
               "beta_eigenvector": (vector / vector.norm(dim=1, keepdim=True)).to(device)}
    masks = PostflopMasks(compatibility=compat.to(device), evaluator_summary=summary, compact_size=compact)
    ranges = torch.rand((batch, players, hands), generator=g).to(device)
    ms, eager_ms = _time_forward(device, lambda: model.forward(pub, ranges, None, masks), reps)
    if input_errors(device):
        raise RuntimeError("postflop bench inputs failed the encoder's checks")
    tokens = players * compact + 1 + 1 + 4 * players + 1 + 4 + 1 + 2 + 5 + 3 + 5 + history + cfg.k_act
    return {"workload": f"postflop policy/value forward, default PokerModelConfig, R13 heads-up flop, {batch} "
                        f"decisions, {players} x {compact} compact combo rows, {tokens} tokens each", "ms": ms,
            "eager_ms": eager_ms, "launch": "CUDA graph replay", "decisions_per_s": batch / (ms / 1000.0),
            "combo_rows_per_s": batch * players * compact / (ms / 1000.0),
            "token_rows_per_s": batch * tokens / (ms / 1000.0),
            "kernels": ["linear_tcgen05_kernel", "attention_kernel", "layernorm_kernel"]}


def _random_params(shapes: dict, seed: int = 17) -> dict:
    """Random weights of the given architecture: N(0, 1/fan_in) maps, N(0, 0.05) vectors, unit LayerNorm
    gains, temperatures 1 (theta = log(expm1(0.5)))."""

    import torch

    g = torch.Generator().manual_seed(seed)
    params = {}
    for name, shape in shapes.items():
        scale = (1.0 / shape[1] ** 0.5) if len(shape) == 2 and "embedding" not in name else 0.05
        params[name] = torch.randn(shape, generator=g) * scale
        if name.endswith("theta"):
            params[name] = torch.full(shape, -0.4328)
        if (name.startswith("layer_norms") or "norm.weight" in name) and name.endswith("weight"):
            params[name] = torch.ones(shape)
    return params


def _synthetic_pub(device, batch: int, players: int, history: int, street: int) -> dict:
    """A seeded public batch (PokerPublicBatch fields, preflop.py:104-170) of the given shape."""

    import torch

    d = torch.Generator(device=device).manual_seed(18)
    r = lambda *shape: torch.rand(shape, generator=d, device=device)  # noqa: E731
    return {"street": torch.full((batch,), street, dtype=torch.long, device=device),
           "pot": r(batch) * 3, "stacks": r(batch, players) * 100, "committed": r(batch, players),
           "to_act": torch.randint(0, players, (batch,), generator=d, device=device),
           "legality_summary": r(batch, 4), "n_ticks": torch.full((batch,), 200.0, device=device),
           "raise_grid_bounds": r(batch, 2), "status": torch.zeros((batch, players), dtype=torch.long, device=device),
           "seat_mask": torch.ones((batch, players), dtype=torch.bool, device=device),
           "button": torch.randint(0, players, (batch,), generator=d, device=device),
           "committed_street": r(batch, players), "call_amount": r(batch), "current_bet": r(batch),
           "min_raise_to": r(batch), "max_raise_to": r(batch) * 100, "last_full_raise": torch.ones(batch, device=device),
           "history": {"actor": torch.randint(-1, players, (batch, history), generator=d, device=device),
                       "street": torch.zeros((batch, history), dtype=torch.long, device=device),
                       "action": torch.randint(0, 3, (batch, history), generator=d, device=device),
                       "amount": r(batch, history), "pot_before": r(batch, history), "call_amount": r(batch, history),
                       "current_bet": r(batch, history), "min_raise_to": r(batch, history),
                       "max_raise_to": r(batch, history), "mask": r(batch, history) < 0.8}}


PROFILE_ONE_FORWARD = False


def _time_forward(device, forward, reps: int):
    """Median CUDA-event time (ms) of a forward replayed from a CUDA graph, and of the eager forward.
    With PROFILE_ONE_FORWARD: two warm-up forwards, then one between cudaProfilerStart/Stop (no timing)."""

    import torch

    if PROFILE_ONE_FORWARD:
        forward()
        forward()
        torch.cuda.synchronize(device)
        torch.cuda.profiler.start()
        forward()
        torch.cuda.synchronize(device)
        torch.cuda.profiler.stop()
        return float("nan"), float("nan")

    def timed(fn):
        times = []
        for rep in range(reps + 2):
            torch.cuda.synchronize(device)
            a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            e.record()
            torch.cuda.synchronize(device)
            if rep >= 2:
                times.append(a.elapsed_time(e))
        return sorted(times)[len(times) // 2]

    eager_ms = timed(forward)
    # the same forward captured once in a CUDA graph (every launch is on the current stream and
    # nothing reads the device from the host), replayed without Python in between
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        forward()
    torch.cuda.current_stream(device).wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        forward()
    ms = timed(graph.replay)
    del graph
    return ms, eager_ms


def rollout_with_model_component(device, hands=65_536):
    """Family-scheduled rollout with the policy network in the loop (pbg_b200.family_rollout): HU 100bb
    R13 (cfg2), `hands` roots played to the end; every step groups the live hands by partition (preflop
    classes / postflop combos), encodes their retained rows, evaluates QueuedPokerModel with cfg2's
    architecture (d_model 128, 2 layers, 4 heads, class embedding 32, hidden 512, M = 2; random weights)
    and runs the fused rollout step and reach update.  Player decisions per second of the whole loop
    (host grouping included), the metric of pbg.benchmark's player_nodes_per_second."""

    import time

    import torch
    from pbg_b200.family_rollout import FamilyRollout
    from pbg_b200.poker import NLHEGeometry
    from pbg_b200.preflop import PreflopConfig
    from pbg_b200.queued_model import QueuedPokerModel, parameter_shapes

    geo = NLHEGeometry(2, 100.0, 13)
    cfg = PreflopConfig(d_model=128, n_heads=4, layers=2, m_raise=2, k_act=5, max_players=2,
                        class_embedding_dim=32, ffn_hidden=512, max_history_tokens=geo.history_tokens)
    model = QueuedPokerModel(geo, cfg, _random_params(parameter_shapes(cfg, 13), seed=29), device)

    def play():
        roll = FamilyRollout(model, seed=41, iteration=3)
        arena, log_reach = roll.roots(hands, device=device)
        total, steps = 0, 0
        while True:
            n = roll.step(arena, log_reach)
            if n == 0:
                break
            total, steps = total + n, steps + 1
        return total, steps, roll.families

    small = hands
    hands = min(hands, 1024)
    play()  # warm-up on a small arena (bindings, first launches)
    hands = small
    if PROFILE_ONE_FORWARD:  # one whole rollout between cudaProfilerStart/Stop
        torch.cuda.synchronize(device)
        torch.cuda.profiler.start()
        play()
        torch.cuda.synchronize(device)
        torch.cuda.profiler.stop()
        return {}
    torch.cuda.synchronize(device)
    t = time.perf_counter()
    decisions, steps, families = play()
    torch.cuda.synchronize(device)
    seconds = time.perf_counter() - t
    return {"workload": f"family-scheduled rollout with the model in the loop, HU 100bb R13, {hands} hands to the "
                        "end, cfg2 architecture (d_model 128, 2 layers, 4 heads), random weights",
            "decisions": decisions, "steps": steps, "families": families, "seconds": seconds,
            "decisions_per_s": decisions / seconds,
            "kernels": ["direct_model_input_kernel", "linear_tcgen05_kernel", "attention_kernel", "rollout_step_kernel",
                        "reach_kernel"]}


def _device_ms(device, fn, reps: int = 10) -> float:
    """Median CUDA-event time (ms) of fn, each call queued behind a device-side sleep."""

    import torch

    if PROFILE_ONE_FORWARD:
        fn()
        fn()
        torch.cuda.synchronize(device)
        torch.cuda.profiler.start()
        fn()
        torch.cuda.synchronize(device)
        torch.cuda.profiler.stop()
        return float("nan")
    times = []
    for rep in range(reps + 2):
        torch.cuda._sleep(1_000_000)
        a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        e.record()
        torch.cuda.synchronize(device)
        if rep >= 2:
            times.append(a.elapsed_time(e))
    return sorted(times)[len(times) // 2]


def readout_component(device, rows=4_194_304, hidden=128, reps=10):
    """The loss backward fused with the readout's weight gradient (pbg_ppo_readout_backward) on the cfg5
    rows (4,194,304 x 8, bf16 logits) with bf16 hidden rows of width `hidden`: one launch writes dlogits,
    dweight [8, hidden] and dbias.  Algorithmic bytes per row: 56 (the loss) + 2 * hidden (the hidden row),
    against the measured HBM copy bandwidth; each launch is queued behind a device-side sleep."""

    import torch
    from pbg_b200.loss import FusedPPOReadoutBackward, LossConfig

    logits, mask, action, old, adv, weight = make_inputs(rows, 8, 0, device)
    g = torch.Generator(device=device).manual_seed(5)
    h = torch.randn((rows, hidden), generator=g, device=device).to(torch.bfloat16)
    op = FusedPPOReadoutBackward(rows, hidden, device, LossConfig())
    dl = torch.empty_like(logits)
    ms = _device_ms(device, lambda: op(logits, mask, action, old, adv, weight, h, dl), reps)
    if PROFILE_ONE_FORWARD:
        return {}
    peak, kind = measured_peak()
    per_row = 56 + 2 * hidden
    gbs = per_row * rows / (ms / 1000.0) / 1e9
    return {"workload": f"cfg5 rows ({rows} x 8, bf16) with the readout's weight gradient, hidden width {hidden}",
            "us": 1000.0 * ms, "decisions_per_s": rows / (ms / 1000.0),
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                         "bytes_per_row": per_row, "peak_kind": kind},
            "kernel": "ppo_readout_bulk_kernel", "gpu_launches": 1}


def optimizer_component(device, params=4_226_931, reps=10):
    """The flat-buffer Adam step (pbg_b200.optim.FlatAdam, two launches: norm with the finalise in its last
    block, then apply) over the
    cfg2 architecture's 4,226,931 fp32 parameters (16,907,724 B, model_storage_bytes / 4).  Algorithmic
    bytes per parameter: 4 (gradient read by the norm pass) + 16 read + 16 written by the apply; each step
    queued behind a device-side sleep."""

    import torch
    from pbg_b200.optim import FlatAdam

    g = torch.Generator(device=device).manual_seed(9)
    master = torch.randn(params, generator=g, device=device)
    opt = FlatAdam(master, lr=1e-3, decay=0.01, clip=1.0)
    grad = torch.randn(params, generator=g, device=device) * 1e-3

    def step():
        opt.grad.copy_(grad)
        opt.step()

    ms = _device_ms(device, step, reps)
    copy_ms = _device_ms(device, lambda: opt.grad.copy_(grad), reps)
    peak, kind = measured_peak()
    step_ms = ms - copy_ms
    gbs = 36 * params / (step_ms / 1000.0) / 1e9
    return {"workload": f"flat AdamW step over {params} fp32 parameters (cfg2 architecture)", "us": 1000.0 * step_ms,
            "note": "timed as (gradient refill + step) minus the refill alone; the 68 MB working set fits in the "
                    "126 MB L2, so part of the traffic is L2 hits",
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                         "bytes_per_param": 36, "peak_kind": kind},
            "kernels": ["adam_norm_kernel", "adam_apply4_kernel"], "gpu_launches": 2}


def showdown_component(device, hands=1_048_576, players=6, reps=10):
    """Sampled settlement's showdown (poker_gpu_evaluator.evaluate_showdowns, the contract-v2 call
    signature): `hands` 6-max R13 showdowns, every seat at stratum 0 except ~20 % folded (-1), seeded
    distinct cards per hand; one launch per call, queued behind a device-side sleep."""

    import numpy as np
    import torch
    import poker_gpu_evaluator as poker

    rng = np.random.default_rng(12)
    deal = np.argsort(rng.random((hands, 52), dtype=np.float32), axis=1)[:, : 5 + 2 * players]
    board = torch.from_numpy(deal[:, :5].astype(np.uint8)).to(device)
    lo = np.minimum(deal[:, 5::2], deal[:, 6::2])
    hi = np.maximum(deal[:, 5::2], deal[:, 6::2])
    combo = torch.from_numpy((lo * (103 - lo) // 2 + hi - lo - 1).astype(np.int32)).to(device)
    level = np.where(rng.random((hands, players)) < 0.2, -1, 0).astype(np.int32)
    level[:, 0] = 0
    base = -rng.integers(1, 16, (hands, players)).astype(np.float32)
    amount = np.zeros((hands, players), np.float32)
    amount[:, 0] = -base.sum(1)
    level, base, amount = (torch.from_numpy(x).to(device) for x in (level, base, amount))
    ev = poker.bind(13)
    ms = _device_ms(device, lambda: ev.evaluate_showdowns(board_cards=board, combo_ids=combo, stratum_level=level,
                                                          payoff_baseline=base, stratum_amount=amount), reps)
    return {"workload": f"{hands} {players}-max R13 showdowns (one stratum, ~20 % of seats folded)",
            "us": 1000.0 * ms, "hands_per_s": hands / (ms / 1000.0),
            "seat_hands_per_s": hands * players / (ms / 1000.0),
            "bound": "integer issue (7-card evaluation per contending seat)", "kernel": "showdown_kernel",
            "gpu_launches": 1}


def completion_component(device, leaves=4096, players=6, samples=(256, 1024), reps=5):
    """Rao-Blackwell leaf completion (poker_gpu_evaluator.complete, the contract-v2 call of
    RBCompletionBinding, hooks.py:2472-2477) at cfg3's geometry: `leaves` 6-max R13 leaf rows of
    [6, 1326] fp32 range weights (preflop / flop / turn / river boards in turn, three strata, ~20 % of
    seats folded), each sample count in `samples`.  One launch per call, queued behind a device-side
    sleep.  The HBM floor per leaf is the range read plus the p_hat and v_hat writes; the CPU figure is
    the C restatement (oracle) on one core over a few leaves of the same workload."""

    import numpy as np
    import torch
    import poker_gpu_evaluator as poker

    H = 1326
    rng = np.random.default_rng(31)
    board = np.full((leaves, 5), 255, np.uint8)
    shown = np.array([0, 3, 4, 5])[np.arange(leaves) % 4]
    cards = np.argsort(rng.random((leaves, 52), dtype=np.float32), axis=1)[:, :5]
    board = np.where(np.arange(5)[None, :] < shown[:, None], cards, 255).astype(np.uint8)
    w = np.exp(rng.normal(0.0, 1.5, (leaves, players, H))).astype(np.float32)
    level = np.where(rng.random((leaves, players)) < 0.2, -1, rng.integers(0, 3, (leaves, players))).astype(np.int32)
    level[:, :2] = np.maximum(level[:, :2], 0)
    base = -rng.integers(1, 40, (leaves, players)).astype(np.float32) * 0.5
    pot = -base.sum(1)
    amount = np.stack([pot * 0.6, pot * 0.3, pot * 0.1], 1).astype(np.float32)
    seed = rng.integers(0, 2**62, leaves, dtype=np.int64)
    t = {k: torch.from_numpy(v).to(device) for k, v in
         dict(board_cards=board, range_weights=w, stratum_level=level, payoff_baseline=base, stratum_amount=amount,
              seed=seed).items()}
    ev = poker.bind(13)
    if PROFILE_ONE_FORWARD:
        _device_ms(device, lambda: ev.complete(**t, n_samples=samples[0], validate=False))
        return {}
    peak, peak_kind = measured_peak()
    algo = leaves * (players * H * 4 * 3 + 5 + players * 12 + 3 * 4 + 8 + 4)
    out = {"workload": f"{leaves} {players}-max R13 leaves ([{players}, {H}] range weights; boards preflop / "
                       "flop / turn / river in turn; 3 strata; ~20 % of seats folded)",
           "kernel": "rb_complete_kernel", "gpu_launches": 1, "algorithmic_bytes": algo,
           "bound": "instruction issue and shared-memory latency (per sample: 6 seat draws with "
                    "inclusion-exclusion masses, the runout, 7-card evaluations) above the HBM floor"}
    for n in samples:
        ms = _device_ms(device, lambda: ev.complete(**t, n_samples=n, validate=False), reps)
        gbs = algo / (ms / 1000.0) / 1e9
        out[f"n{n}"] = {"us": 1000.0 * ms, "leaves_per_s": leaves / (ms / 1000.0),
                        "samples_per_s": leaves * n / (ms / 1000.0), "hbm_gbs": gbs, "peak_gbs": peak,
                        "frac": gbs / peak, "peak_kind": peak_kind}
    try:
        import time
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O

        k = 4
        t0 = time.perf_counter()
        O.rb_complete(13, board[:k], w[:k], level[:k], base[:k], amount[:k], samples[0], seed[:k])
        dt = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": k / dt, "unit": "leaves/s", "cores": 1, "kind": "port",
                               "sample": f"{k} leaves at n_samples={samples[0]} through the C restatement"}
    except Exception as exc:  # the oracle is optional on a box without a C compiler
        out["cpu_baseline"] = {"unavailable": str(exc)[:200]}
    return out


def reach_component(device, hands=16_384, seed=0, reps=10):
    """The reach update after a preflop decision (pbg_reach_update, hooks.py:1641-1703): `hands` HU 100bb
    R13 hands after their first step, a seeded raw policy for every private row; per hand the 169 class
    rows' log pi of the taken action (closed-form policy) and the [2, 1326] log-reach rows read and
    written.  Each call queued behind a device-side sleep (the update is applied repeatedly in place)."""

    import torch
    from pbg_b200.poker import NLHEGeometry
    from pbg_b200.rollout import RolloutStep

    geometry = NLHEGeometry(2, 100.0, 13)
    stepper = RolloutStep(geometry, seed=seed, iteration=0)
    H, M = geometry.private_hands, 2
    g = torch.Generator(device=device).manual_seed(seed + 3)
    raw = {"type_logits": torch.randn((hands, H, 3), generator=g, device=device),
           "omega": torch.softmax(torch.randn((hands, H, M), generator=g, device=device), -1),
           "mu": torch.rand((hands, H, M), generator=g, device=device),
           "s": torch.rand((hands, H, M), generator=g, device=device) * 0.3 + 0.02,
           "iota": torch.rand((hands, H), generator=g, device=device) * 0.2}
    arena = stepper.roots(hands, device=device)
    stepper.step(arena, raw)
    log_reach = torch.zeros((hands, 2, H), dtype=torch.float32, device=device)
    ms = _device_ms(device, lambda: stepper.reach_update(arena, raw, log_reach), reps)
    per_hand = 169 * (3 + 3 * M + 1) * 4 + 2 * 4 * 2 * H
    peak, kind = measured_peak()
    gbs = per_hand * hands / (ms / 1000.0) / 1e9
    return {"workload": f"reach update after the first (preflop) decision, HU 100bb R13, {hands} hands",
            "us": 1000.0 * ms, "hands_per_s": hands / (ms / 1000.0),
            "policy_rows_per_s": 169 * hands / (ms / 1000.0),
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                         "bytes_per_hand": per_hand, "peak_kind": kind},
            "kernel": "reach_kernel", "gpu_launches": 1}


def folded_component(device, rows=64):
    """Multiway folded statistics (queued/folded.py): 6-max R13, four folded seats (all tight), flop
    boards, `rows` decisions; the finite-difference removal queries (1 + 52 + 1326 per decision) in
    one launch of pbg_folded_phi_queries, and the whole folded_statistics call (normalisation, queries,
    assembly, torch.linalg.eigh of the 52 x 52 beta matrices, card masses)."""

    import torch
    from pbg_b200.folded import folded_statistics, phi_queries
    from pbg_b200.poker import NLHEGeometry, PokerStateMachine

    geo = NLHEGeometry(6, 100.0, 13)
    combo = PokerStateMachine(geo).combo_cards(torch.arange(geo.private_hands, dtype=torch.int32, device=device))
    g = torch.Generator(device=device).manual_seed(23)
    status = torch.zeros((rows, 6), dtype=torch.int8, device=device)
    status[:, 2:] = 1
    board = torch.full((rows, 5), 255, dtype=torch.uint8, device=device)
    board[:, :3] = torch.tensor([3, 17, 40], dtype=torch.uint8, device=device)
    weights = torch.rand((rows, 6, geo.private_hands), generator=g, device=device)
    folder = status.eq(1)
    raw = weights * folder[..., None]
    clash = ((combo.long()[None, :, :, None] == board.long()[:, None, None, :]) & (board != 255)[:, None, None, :]).any(-1).any(-1)
    raw = raw.masked_fill(clash[:, None], 0.0)
    prob = raw / raw.sum(-1, keepdim=True).clamp_min(1e-38)
    base = torch.full((rows,), 49.0, device=device)
    if PROFILE_ONE_FORWARD:
        from pbg_b200.folded import symmetric_eigh

        beta = torch.randn((rows, 52, 52), generator=g, device=device)
        _device_ms(device, lambda: (phi_queries(prob, folder, folder, base, 52), symmetric_eigh(beta + beta.mT)))
        return {}
    queries_ms = _device_ms(device, lambda: phi_queries(prob, folder, folder, base, 52))
    whole_ms = _device_ms(device, lambda: folded_statistics(geo, board_cards=board, range_weights=weights, status=status,
                                                            combo_cards=combo, beta_rank=52, line_dim=0), reps=5)
    queries = 1 + 52 + 1326
    return {"workload": f"folded statistics, 6-max R13, 4 tight folders, flop, {rows} decisions x {queries} removal "
                        "queries", "phi_queries_ms": queries_ms, "folded_statistics_ms": whole_ms,
            "queries_per_s": rows * queries / (queries_ms / 1000.0), "decisions_per_s": rows / (whole_ms / 1000.0),
            "bound": "FP32 issue (per-query hand sums over shared memory)", "kernel": "folded_phi_kernel",
            "gpu_launches": 1}


def branching_component(device, n_alias=65536, n_nodes=200000):
    """Branched learner sampling metadata: the Walker alias table over `n_alias` weights
    (alias_table.cu) and the decision log mass of an `n_nodes`-node forest (branching_metadata.cu),
    each launch sequence queued behind a device-side sleep."""

    import numpy as np
    import torch
    from pbg_b200.branching import build_alias_table, decision_log_mass

    logw = torch.linspace(-40.0, 0.0, n_alias, dtype=torch.float64, device=device)
    w = torch.softmax(logw, 0) * n_alias
    prob, alias = torch.empty_like(w), torch.empty(n_alias, dtype=torch.int32, device=device)
    alias_ms = _device_ms(device, lambda: build_alias_table(w.clone(), prob, alias))
    rng = np.random.default_rng(5)
    parent = np.full(n_nodes, -1, dtype=np.int32)
    degree = np.zeros(n_nodes, dtype=np.int32)
    nxt = 1
    for node in range(n_nodes):
        kids = min(int(rng.integers(1, 6)), n_nodes - nxt)
        parent[nxt: nxt + kids] = node
        degree[node] = kids
        nxt += kids
        if nxt >= n_nodes:
            break
    pp, dd = torch.from_numpy(parent).to(device), torch.from_numpy(degree).to(device)
    fail = torch.zeros(1, dtype=torch.int32, device=device)
    mass_ms = _device_ms(device, lambda: decision_log_mass(pp, dd, fail))
    return {"workload": f"alias table over {n_alias} weights; decision log mass of a {n_nodes}-node forest",
            "alias_table_ms": alias_ms, "decision_log_mass_ms": mass_ms,
            "kernels": ["alias_classify_kernel", "alias_block_scan_kernel", "alias_scatter_kernel", "alias_pair_kernel",
                        "decision_log_mass_kernel"], "gpu_launches": 6}


def posterior_component(device, parents=4096, rows=16384, reps=10):
    """Collision-conditioned posterior profiles (rb_sampling.py): 6-max R13 (1326 private hands), `parents`
    parent rows of [6, 1326] fp32 range weights (board-conflicting hands masked; flop/turn/river boards),
    `rows` fresh child rows, up to 256 attempts each.  One call = the CDF pass + the sampling pass, each
    call queued behind a device-side sleep."""

    import numpy as np
    import torch
    from pbg_b200.poker import NLHEGeometry
    from pbg_b200.rb_sampling import CollisionConditionedProfileSampler

    geo = NLHEGeometry(6, 100.0, 13)
    g = torch.Generator(device=device).manual_seed(21)
    w = torch.rand((parents, 6, geo.private_hands), generator=g, device=device)
    board = torch.full((parents, 5), 255, dtype=torch.uint8, device=device)
    rng = np.random.default_rng(21)
    cards = np.stack([rng.permutation(52)[:5] for _ in range(parents)])
    shown = np.array([3, 4, 5])[np.arange(parents) % 3]
    host = np.where(np.arange(5)[None, :] < shown[:, None], cards, 255).astype(np.uint8)
    board.copy_(torch.from_numpy(host))
    inherited = torch.randint(0, geo.private_hands, (parents, 6), generator=g, device=device, dtype=torch.int32)
    source = torch.randint(0, parents, (rows,), generator=g, device=device)
    ordinal = torch.ones(rows, dtype=torch.int64, device=device)
    active = torch.ones(rows, dtype=torch.bool, device=device)
    root = torch.randint(0, 2**62, (rows,), generator=g, device=device)
    path = torch.randint(0, 2**62, (rows,), generator=g, device=device)
    sampler = CollisionConditionedProfileSampler(geo)
    if PROFILE_ONE_FORWARD:
        _device_ms(device, lambda: sampler.sample_children(
            range_weights=w, board_cards=board, inherited_profile=inherited, source=source, ordinal=ordinal,
            active=active, root=root, path=path, seed=1, iteration=0, retry_epoch=0))
        return {}
    times = []
    for rep in range(reps + 3):
        torch.cuda._sleep(1_000_000)
        a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        sampler.sample_children(range_weights=w, board_cards=board, inherited_profile=inherited, source=source,
                                ordinal=ordinal, active=active, root=root, path=path, seed=1, iteration=rep,
                                retry_epoch=0)
        e.record()
        torch.cuda.synchronize(device)
        if rep >= 3:
            times.append(a.elapsed_time(e))
    ms = sorted(times)[len(times) // 2]
    counts = sampler.last_observation.attempt_count.float()
    peak, _ = measured_peak()
    cdf_bytes = parents * 6 * geo.private_hands * 8  # weights read + CDF written, fp32
    return {"workload": f"collision-conditioned posterior, 6-max R13, {parents} parents x 6 x 1326, {rows} child rows",
            "us_per_call": 1000.0 * ms, "rows_per_s": rows / (ms / 1000.0),
            "mean_attempts": float(counts.mean()), "exhausted": int(sampler.last_observation.exhausted.sum()),
            "cdf_pass_bytes": cdf_bytes, "cdf_pass_gbs_upper": cdf_bytes / (ms / 1000.0) / 1e9, "peak_gbs": peak,
            "kernels": ["posterior_cdf_kernel", "posterior_sample_kernel"], "gpu_launches": 4}


# ----------------------------------------------------------- device arm


COMPONENTS = {"rollout_step": rollout_component, "layered_targets": targets_component,
              "model_linear": model_linear_component, "model_attention": model_attention_component,
              "preflop_forward": preflop_forward_component, "postflop_forward": postflop_forward_component,
              "posterior_sampler": posterior_component, "loss_readout": readout_component,
              "poker_loss": poker_loss_component, "optimizer_step": optimizer_component,
              "showdown": showdown_component, "rb_completion": completion_component,
              "learner_step_cfg1": learner_step_component, "learner_step_cfg2": learner_step_cfg2_component,
              "reach_update": reach_component, "folded_statistics": folded_component,
              "branched_sampling": branching_component, "rollout_with_model": rollout_with_model_component}


def main():
    args = parse()
    if args.engine_arm:
        engine_arm(args)
        return
    if args.engine_compare:
        engine_compare(args)
        return
    if args.impl == "reference":
        reference_arm(args)
        return
    import torch
    import torch.distributed as dist
    from pbg_b200.loss import FusedPPOBackward, LossConfig

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if args.profile_forward == "attention":
        profile_attention(device)
        return
    if args.component:  # one component's entry, printed alone
        print(json.dumps({args.component: COMPONENTS[args.component](device)}), flush=True)
        return
    if args.profile_forward:
        global PROFILE_ONE_FORWARD
        PROFILE_ONE_FORWARD = True
        name = {"folded": "folded_component", "posterior": "posterior_component",
                "readout": "readout_component", "reach": "reach_component", "showdown": "showdown_component",
                "optimizer": "optimizer_component", "poker_loss": "poker_loss_component",
                "rollout_with_model": "rollout_with_model_component", "completion": "completion_component",
                "rollout": "rollout_component", "learner_step": "learner_step_component",
                "learner_step_cfg2": "learner_step_cfg2_component"}.get(
            args.profile_forward, f"{args.profile_forward}_forward_component")
        if name == "rollout_with_model_component":
            rollout_with_model_component(device, hands=args.profile_hands)
        elif name == "learner_step_cfg2_component":  # --profile-hands H: H / 4 preflop + H / 16 postflop rows
            learner_step_cfg2_component(device, pre_rows=args.profile_hands // 4, post_rows=args.profile_hands // 16)
        else:
            globals()[name](device)
        return
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    if args.learner_scaling == "cfg2":
        learner_scaling_cfg2(args, device, world, rank)
        if world > 1:
            dist.destroy_process_group()
        return
    if args.learner_scaling:
        learner_scaling(args, device, world, rank)
        if world > 1:
            dist.destroy_process_group()
        return
    N, A = args.rows, args.actions
    inputs = make_inputs(N, A, seed=rank, device=device)
    logits, mask, action, old, adv, weight = inputs
    op = FusedPPOBackward(N, A, device, LossConfig(policy_clip=0.2, negative_advantage_ratio_cap=None,
                                                   entropy_coefficient=0.01))
    dlogits = torch.empty_like(logits)
    stream = torch.cuda.current_stream(device)
    flat = None
    allreduce_kind = "none (single rank)"
    if world > 1:
        # from 4 ranks up the flat gradient lives in symmetric memory and is summed through
        # NVLink SHARP by libpbgb200's multimem kernel (1.5x NCCL at 8 ranks); at 2 ranks a
        # multimem SUM moves more NVLink bytes than NCCL's ring, and NCCL is kept, as it is
        # when the fabric exposes no multicast object
        from pbg_b200.distributed import NVLSFlatSum

        try:
            if args.allreduce == "nccl" or (args.allreduce == "auto" and world < 4):
                raise RuntimeError("NCCL ring (two ranks, or requested)")
            flat = NVLSFlatSum(args.params, device)
            grad = flat.buffer
            allreduce_kind = "NVLS multimem SUM (libpbgb200)"
        except RuntimeError:
            grad = torch.empty(args.params, device=device)
            allreduce_kind = "NCCL SUM"
        grad.copy_(torch.randn(args.params, device=device) * 1e-3)
    else:
        grad = torch.randn(args.params, device=device) * 1e-3
    bound = op.bind(logits, mask, action, old, adv, weight, dlogits)
    bound.launch(stream)  # one-time device set-up happens outside any capture
    torch.cuda.synchronize(device)
    # The loss kernel alone, replayed from a CUDA graph over fixed buffers (host launch cost never gaps
    # the device): the whole step at N = 1, and the roofline timing at every N.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        bound.launch()
    torch.cuda.synchronize(device)
    # N > 1: the loss runs as `buckets` row chunks and the flat gradient SUM as as many buckets on a
    # second stream, bucket k starting when chunk k is done (the way a backward hands finished gradient
    # buckets to the collective while it still computes), so the SUM overlaps the remaining loss.
    buckets = max(1, args.buckets) if world > 1 else 1
    if world > 1 and (N % buckets or args.params % (4 * world * buckets)):
        buckets = 1
    chunk_ops, chunk_binds = [], []
    rows_b, params_b = N // buckets, args.params // buckets
    # the persistent loss kernel holds every register of an SM, so nothing shares an SM it runs on:
    # with buckets the SUM gets `comm_sms` SMs of its own and the loss chunks the rest
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    comm_ctas = max(1, min(args.comm_sms, sms // 2)) if buckets > 1 else 0
    loss_ctas = sms - comm_ctas if buckets > 1 else 0
    if buckets > 1:
        for k in range(buckets):
            lo, hi = k * rows_b, (k + 1) * rows_b
            chunk = FusedPPOBackward(rows_b, A, device, op.config)
            chunk.set_controls(inv_count=1.0 / N)
            chunk_ops.append(chunk)
            chunk_binds.append(chunk.bind(logits[lo:hi], mask[lo:hi], action[lo:hi], old[lo:hi], adv[lo:hi],
                                          weight[lo:hi], dlogits[lo:hi], max_ctas=loss_ctas))
            chunk_binds[-1].launch(stream)
    comm = torch.cuda.Stream(device) if world > 1 else None
    done = [torch.cuda.Event() for _ in range(buckets)]

    def overlapped_step():
        main = torch.cuda.current_stream(device)
        comm.wait_stream(main)
        for k in range(buckets):
            if buckets > 1:
                chunk_binds[k].launch(main)
            else:
                bound.launch(main)
            done[k].record(main)
            comm.wait_event(done[k])
            if flat is not None:
                flat.sum_range_(k * params_b, params_b, comm, max_ctas=comm_ctas)
            else:
                with torch.cuda.stream(comm):
                    dist.all_reduce(grad[k * params_b:(k + 1) * params_b], op=dist.ReduceOp.SUM)
        main.wait_stream(comm)

    step_graph = None
    if flat is not None:
        overlapped_step()  # warm once outside capture
        torch.cuda.synchronize(device)
        step_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(step_graph):
            overlapped_step()
    sum_graph = None
    if flat is not None:
        sum_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(sum_graph):
            flat.sum_()
    torch.cuda.synchronize(device)

    def step(events=None):
        if world == 1:
            graph.replay()
        elif step_graph is not None:
            step_graph.replay()
        else:
            overlapped_step()

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        time.sleep(0.3)
        torch.cuda.synchronize(device)
        start.record(stream)
        for i in range(args.steps):
            step()
        end.record(stream)
        torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    for chunk, rows in ([(c, rows_b) for c in chunk_ops] if buckets > 1 else [(op, N)]):
        if float(chunk.stats[7]) != rows:
            raise RuntimeError("loss kernel reported a failed launch (stats rows != rows)")
    if flat is not None:
        flat.check()
    elapsed_ms = start.elapsed_time(end)
    # the loss kernel alone over all rows (its own events per launch, on the launching stream): the roofline
    kernel_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                     for _ in range(args.steps)]
    torch.cuda.synchronize(device)
    for a, b in kernel_events:
        a.record(stream)
        graph.replay()
        b.record(stream)
    torch.cuda.synchronize(device)
    if float(op.stats[7]) != N:
        raise RuntimeError("loss kernel reported a failed launch (stats rows != N)")
    kernel_ms = sum(a.elapsed_time(b) for a, b in kernel_events) / args.steps
    if world > 1:
        t = torch.tensor([elapsed_ms, kernel_ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms, kernel_ms = float(t[0]), float(t[1])
    ms_per_step = elapsed_ms / args.steps
    value = world * N / (ms_per_step / 1000.0)

    # the gradient SUM alone, NVLS kernel vs NCCL on the same bytes (max over ranks)
    allreduce = None
    if world > 1:
        def time_reduce(fn, reps=20):
            for _ in range(3):
                fn()
            torch.cuda.synchronize(device)
            dist.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(reps):
                fn()
            b.record(stream)
            torch.cuda.synchronize(device)
            t = torch.tensor([a.elapsed_time(b) / reps], device=device, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t[0]) * 1000.0

        nbytes = 4 * args.params
        bus = lambda us: 2.0 * (world - 1) / world * nbytes / (us * 1e-6) / 1e9
        scratch = torch.zeros(args.params, device=device)
        nccl_us = time_reduce(lambda: dist.all_reduce(scratch, op=dist.ReduceOp.SUM))
        allreduce = {"bytes": nbytes, "nccl_us": nccl_us, "nccl_busbw_gbs": bus(nccl_us)}
        if sum_graph is not None:
            nvls_us = time_reduce(sum_graph.replay)
            allreduce.update({"nvls_us": nvls_us, "nvls_busbw_gbs": bus(nvls_us)})
        del scratch

    # end to end through the public API: pinned host inputs -> device -> loss -> stats back
    host = [t.cpu().pin_memory() for t in inputs]
    stats_host = torch.empty(8, dtype=torch.float64).pin_memory()
    dev_in = [torch.empty_like(t) for t in inputs]
    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = stats_host.numel() * stats_host.element_size()

    e2e_bound = op.bind(*dev_in, dlogits)

    def e2e_step():
        for d, h in zip(dev_in, host):
            d.copy_(h, non_blocking=True)
        e2e_bound.launch(stream)
        if world > 1:
            if flat is not None:
                flat.sum_(stream)
            else:
                dist.all_reduce(grad, op=dist.ReduceOp.SUM)
        stats_host.copy_(op.stats, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = e0.elapsed_time(e1) / args.e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t[0])
    e2e_value = world * N / (e2e_ms / 1000.0)

    peak, peak_kind = measured_peak()
    algo_bytes = BYTES_PER_ROW(A) * N
    achieved = algo_bytes / (kernel_ms / 1000.0) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "cfg5 loss microbench: 4,194,304 decisions x 8 actions per rank, fused PPO "
                               "loss backward + flat fp32 gradient SUM all-reduce",
                   "rows_per_rank": N, "actions": A, "grad_params": args.params,
                   "allreduce": allreduce_kind,
                   "l2": "inputs larger than L2 (235 MB per pass)", "parallelism": f"dp{world}",
                   "buckets": buckets, "comm_sms": comm_ctas,
                   "launch": ("CUDA graph replay (loss kernel)" if world == 1 else
                              f"{buckets} loss chunks on the main stream, {buckets} gradient-SUM buckets on a second "
                              "stream, bucket k after chunk k" + (" (one CUDA graph)" if step_graph is not None
                                                                   else " (eager, NCCL)"))},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": committed_traffic(N),
                     "kernel": "ppo_bf16x8_bulk_kernel", "kernel_ms": kernel_ms, "peak_kind": peak_kind,
                     "algorithmic_bytes": algo_bytes},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": args.steps * (1 if world == 1 else buckets * (2 if flat is not None else 1)),
        "clocks": clocks.summary(),
    }
    if rank == 0:
        line["components"] = {}
        if world == 1:  # single-GPU kernels of the path, measured once, outside the scaling runs
            line["components"] = {name: fn(device) for name, fn in COMPONENTS.items()}
        if allreduce is not None:
            line["components"]["gradient_sum"] = allreduce
    if rank == 0 and world == 1 and _reference_pbg() is not None:
        ref = reference_torch_loss_component(device, inputs)
        ref["speedup_value"] = value / ref["value"]
        ref["speedup_e2e"] = e2e_value / ref["value"]
        line["reference_torch_cuda"] = ref
    if rank == 0 and world == 1:
        sample = host_sample(1 << 21, A, 0)
        rate, threads, rows, wall = cpu_loss_rate(sample, seconds=3.0)
        line["cpu_baseline"] = {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
                                "sample": f"{rows} rows ({rows // sample[0].shape[0]} passes over a "
                                          f"{sample[0].shape[0]}-row sample) in {wall:.1f} s on {threads} threads"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        del step_graph, sum_graph, flat, grad
        torch.cuda.synchronize(device)
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
