"""One training iteration of the reference's own engine, optionally routed to libpbgb200.

    python tests/engine_dropin_run.py <out_dir> <reference|b200|b200_learner> [roots] [iterations] [program]
                                      [sampled|rao_blackwell|branched_rao_blackwell] [players stack_bb ranks]

Test infrastructure for tests/test_gpu_engine_dropin.py (run in a fresh process
so that the two engines never share imported state).  It loads the reference
package installed under baseline/_ref, builds a heads-up 8bb 4-rank
self-play run (sampled private estimator, or Rao-Blackwell with evaluator
completion of 64 samples per leaf; sequential rollout, a small transformer), and runs ``pbg.runtime.TrainingSession.step`` once; with
``b200`` it first calls ``pbg_b200.engine.install()`` so that the state
machine, the composite policy and the layered targets of that same engine run
on this build's kernels (``b200_learner``: the learner's loss program too).  The learner's tensor program runs eagerly in both
(``tensor_program: eager``).  Writes <out_dir>/<arm>.pt with the model
state before and after the optimizer step, the flat gradient rows each
optimizer transition received, the loss metrics and the node counts.
"""

from __future__ import annotations

import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "ai-game-learning_b200"))
sys.path.append(os.path.join(ROOT, "baseline", "_ref"))

CONFIG = """kind: nlhe_run_v1
scientific:
  mode: {{training_regime: self_play, rollout_mode: sequential, private_estimator: {estimator}}}{completion}
  game: {{players: {players}, stack_bb: {stack}, rank_count: {ranks}}}
  model:
    d_model: 32
    n_heads: 4
    layers: 1
    raises: {{components: 2, minimum_scale: 0.02}}
    class_embedding_dim: 8
    ffn_hidden: 64
    folder_beta_rank: {beta_rank}
    folder_line_dim: 8
    epsilon: 1.0e-8
  objective:
    policy_clip: 0.2
    value: {{kind: mse, coefficient: 0.5}}
    entropy: {{kind: constant, coefficient: 0.01}}
  optimizer: {{kind: adamw, learning_rate: 0.0003, beta1: 0.9, beta2: 0.999, epsilon: 1.0e-8, weight_decay: 0.0,
              grad_clip: 1.0}}
  schedule: {{batch_size: 16, epochs: 1}}
  lambda: 0.95
run:
  seed: 20261202
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
  checkpoint_every: 1000
  output_dir: {out}
"""


BRANCHED = """kind: nlhe_run_v1
scientific:
  mode: {{training_regime: self_play, rollout_mode: branched.fixed, private_estimator: rao_blackwell}}
  game: {{players: {players}, stack_bb: {stack}, rank_count: {ranks}}}
  model:
    d_model: 32
    n_heads: 4
    layers: 1
    raises: {{components: 2, minimum_scale: 0.02}}
    class_embedding_dim: 8
    ffn_hidden: 64
    folder_beta_rank: {beta_rank}
    folder_line_dim: 8
    epsilon: 1.0e-8
  objective:
    policy_clip: 0.2
    value: {{kind: mse, coefficient: 0.5}}
    entropy: {{kind: constant, coefficient: 0.01}}
    branching: {{trace_coefficient: 0.1, cost_coefficient: 0.1, trace_epsilon: 1.0e-6}}
  optimizer: {{kind: adamw, learning_rate: 0.0003, beta1: 0.9, beta2: 0.999, epsilon: 1.0e-8, weight_decay: 0.0,
              grad_clip: 1.0}}
  schedule: {{batch_size: 16, epochs: 1}}
  lambda: 0.95
  branching:
    fixed_beta: {{player: 1.5, chance: 1.25}}
    beta_max: 3
    minimum_tree_size: 16
    cost_safeguard: {{gamma_deviance_max: 0.2, p95_underprediction_max: 1.5, consecutive_iterations: 4}}
  completion: {{samples: 16}}
run:
  seed: 20261202
  reproducibility: strict
  utility: raw_bb
  workload: {{roots: {roots}, tree_nodes: 512}}
  execution:
    device: cuda:0
    precision: fp32
    attention: sdpa
    memory: {{reserve_bytes: 67108864}}
    microbatch: auto
    tensor_program: {{mode: {program}}}
  iterations: {iterations}
  checkpoint_every: 1000
  output_dir: {out}
"""


def main() -> None:
    out, arm = sys.argv[1], sys.argv[2]
    roots = int(sys.argv[3]) if len(sys.argv) > 3 else 16
    iterations = int(sys.argv[4]) if len(sys.argv) > 4 else 1
    program = sys.argv[5] if len(sys.argv) > 5 else "eager"
    estimator = sys.argv[6] if len(sys.argv) > 6 else "sampled"
    players = int(sys.argv[7]) if len(sys.argv) > 7 else 2
    stack = float(sys.argv[8]) if len(sys.argv) > 8 else 8.0
    ranks = int(sys.argv[9]) if len(sys.argv) > 9 else 4
    completion = "\n  completion: {samples: 64}" if estimator == "rao_blackwell" else ""
    import torch

    handle = None
    if arm in ("b200", "b200_learner"):
        from pbg_b200 import engine

        handle = engine.install(learner=arm == "b200_learner")
    from pbg.config import load_config
    from pbg.runtime import TrainingSession

    os.makedirs(out, exist_ok=True)
    path = os.path.join(out, f"{arm}.yaml")
    with open(path, "w") as f:
        template = BRANCHED if estimator == "branched_rao_blackwell" else CONFIG
        f.write(template.format(roots=roots, iterations=iterations, program=program, estimator=estimator,
                              completion=completion, players=players, stack=stack, ranks=ranks,
                              beta_rank=0 if players == 2 else 4, out=os.path.join(out, f"run_{arm}")))
    # record the flat gradient rows each optimizer transition receives (pbg/core/optimization.py:394-399)
    from pbg.core import optimization

    gradients = []
    original_step = optimization.DenseAdam.step_device

    def recording_step(self, active):
        gradients.append(self.gradient_rows.detach().float().cpu().clone())
        return original_step(self, active)

    optimization.DenseAdam.step_device = recording_step
    torch.manual_seed(0)
    session = TrainingSession(load_config(path))
    module = session.modules.lane_module(0)
    state0 = {k: v.detach().cpu().clone() for k, v in module.state_dict().items()}
    # the flat gradient's layout: trainable parameters in module order (optimization.py:109-147)
    layout = [(name, p.numel()) for name, p in module.named_parameters() if p.requires_grad]
    walls = []
    results = []
    for _ in range(iterations):
        torch.cuda.synchronize()
        t = time.perf_counter()
        results.append(session.step())
        torch.cuda.synchronize()
        walls.append(time.perf_counter() - t)
    state = {k: v.detach().cpu().clone() for k, v in session.modules.lane_module(0).state_dict().items()}
    fused_calls = 0
    if handle is not None:
        from pbg_b200 import ops

        fused_calls = ops.CALLS["poker_learner_objective"]
    lanes = []
    for result in results:
        for lane in getattr(result, "results", (result,)):
            if lane is None:
                continue
            lanes.append({name: getattr(lane, name) for name in ("player_nodes", "leaves", "target_layers",
                                                                  "executed_edges")})
            lanes[-1]["losses"] = [dict(loss) for loss in lane.learner.losses]
            lanes[-1]["presentations"] = lane.learner.statistical_presentations
    torch.save({"state0": state0, "state": state, "lanes": lanes, "walls": walls, "gradients": gradients, "layout": layout, "fused_calls": fused_calls,
                "installed": None if handle is None else [f"{getattr(m, '__name__', m)}.{n}" for m, n, _ in handle.replaced]},
               os.path.join(out, f"{arm}.pt"))
    print(json.dumps({"arm": arm, "walls": walls, "lanes": lanes}, default=str)[:4000])


if __name__ == "__main__":
    main()
