"""Route an imported reference package (pbg) to libpbgb200 for the hot path.

The reference builds its game operations from a few classes and loaders:

* ``PokerStateMachine(geometry)`` in the sequential and branched hooks
  (pbg/games/poker/queued/hooks.py:1305, 2210; branching.py:185), the root
  payload (operations.py:394, 593) and the queued model (model.py:197-299);
* ``PokerPolicyOperator()`` in the operations bundle and the hooks
  (operations.py:149, hooks.py:1310, 2211);
* ``layered_target_cuda()``, the layered-targets extension loader that the
  target executor calls (pbg/core/targets.py:24, 634);
* ``LearnerOperation.forward_loss`` (pbg/core/learner.py:1824-2159), the
  learner's loss program.

``install()`` replaces exactly those names in the imported modules with this
build's drop-ins, so every rollout step (legality, chip accounting, keyed
chance, histories, leaves, model-input rows), every policy evaluation
(sampling, selected log pi, the learner's differentiable policy operation) and
every layered-target pass of the reference's own engine runs on the sm_100a
kernels, while the engine, storage, scheduling and the showdown and
completion bindings stay the reference's (the evaluator they call,
``poker_gpu_evaluator``, is this build's module: sampled showdowns and
Rao-Blackwell leaf completion on the device).
With ``learner=True`` the loss program of every learner whose policy
operation is the poker one (``PokerLearnerPolicy``, hooks.py:2200-2246)
becomes one launch of ``pbg_poker_learner_objective``: the adapter selects the
sampled private rows and the reference raw fields exactly as the reference
does (learner.py:1885-1962), rebuilds the legal events from the retained model
input as the policy operation does (hooks.py:2226-2246), and returns the
reference's ``LossResult`` whose ``total`` backpropagates into the model.
Other learners keep the reference's program.  ``uninstall(handle)`` restores
the originals.

The kernels the learner's tensor program reaches (legality and the fused
objective) are torch custom operators (pbg_b200.ops), so the reference's
compiled and CUDA-graph-captured tensor programs (``tensor_program: captured``,
its default) keep working with the drop-ins.
"""

from __future__ import annotations

import importlib
from dataclasses import dataclass

from .poker import NLHEGeometry, PokerStateMachine
from .policy import PokerPolicyOperator


def _geometry(geometry) -> NLHEGeometry:
    if isinstance(geometry, NLHEGeometry):
        return geometry
    return NLHEGeometry(int(geometry.players), float(geometry.stack_bb), int(geometry.rank_count))


class EngineStateMachine(PokerStateMachine):
    """The device state machine constructed from the reference's NLHEGeometry (hooks.py:72-192)."""

    def __init__(self, geometry) -> None:
        super().__init__(_geometry(geometry))
        self.reference_geometry = geometry

    def combo_cards(self, combo_ids):
        """hooks.py:1128-1143.  The reference also builds host-side tables with it (the Rao-Blackwell
        target algebra, operations.py:593-595, passes a CPU arange): those ids are decoded by the
        same kernel on the current CUDA device and the cards returned where the ids live."""

        if combo_ids.is_cuda:
            return super().combo_cards(combo_ids)
        import torch

        return super().combo_cards(combo_ids.to(torch.device("cuda", torch.cuda.current_device()))).to(
            combo_ids.device)


class EnginePolicyOperator(PokerPolicyOperator):
    """The device composite policy with the reference constructor's keyword (policy.py:139-142)."""


_TARGETS = (
    ("pbg.games.poker.queued.hooks", "PokerStateMachine", "machine"),
    ("pbg.games.poker.queued.operations", "PokerStateMachine", "machine"),
    ("pbg.games.poker.queued.model", "PokerStateMachine", "machine"),
    ("pbg.games.poker.queued.branching", "PokerStateMachine", "machine"),
    ("pbg.games.poker.queued.hooks", "PokerPolicyOperator", "policy"),
    ("pbg.games.poker.queued.operations", "PokerPolicyOperator", "policy"),
    ("pbg.core.targets", "layered_target_cuda", "targets"),
)


def _fused_forward_loss(original):
    """A LearnerOperation.forward_loss that runs the poker objective as one fused launch."""

    import torch
    from pbg.core.contracts import PrivateEstimator
    from pbg.core.learner import LossResult, _select_sampled_private
    from pbg.games.poker.queued.hooks import PokerLearnerPolicy

    from .learner import poker_learner_loss

    def forward_loss(self, batch, *, iteration, reference_operation=None, reference_cache=None, lane_count=1,
                     loss_controls=None, evaluation=None, reference_raw=None):
        policy = self.policy_operation
        if (not isinstance(policy, PokerLearnerPolicy) or evaluation is None or reference_operation is not None
                or reference_cache is not None):
            return original(self, batch, iteration=iteration, reference_operation=reference_operation,
                            reference_cache=reference_cache, lane_count=lane_count, loss_controls=loss_controls,
                            evaluation=evaluation, reference_raw=reference_raw)
        if loss_controls is None:
            loss_controls = self.controls((self.loss,), iteration, batch.sigma_index.device)
        sigma, action = batch.sigma_fields, batch.action_fields
        rows, action_rows = batch.rows, batch.action_rows
        sampled = self.mode.private_estimator is PrivateEstimator.SAMPLED
        private = sigma["sampled_private_state"] if sampled else sigma["owner"][:, None]
        if sampled:  # learner.py:1890-1910: the owner's sampled combo row
            raw = {k: _select_sampled_private(v, private, sigma["owner"]) for k, v in evaluation.policy_raw.items()}
            value = _select_sampled_private(evaluation.value, private, sigma["owner"]).reshape(rows, 1)
            old = action["old_log_policy"].reshape(action_rows, -1)[:, :1]
            adv = action["advantage_target"].reshape(action_rows, -1)[:, :1]
            old_value = sigma["old_value"].reshape(rows, -1)[:, :1]
            target = sigma["value_target"].reshape(rows, -1)[:, :1]
            posterior = None
            ref = None if reference_raw is None else dict(reference_raw)
        else:
            raw, value = dict(evaluation.policy_raw), evaluation.value
            old, adv = action["old_log_policy"], action["advantage_target"]
            old_value, target, posterior = sigma["old_value"], sigma["value_target"], action["posterior"]
            ref = None if reference_raw is None else dict(reference_raw)
        width = raw["type_logits"].shape[1] if raw["type_logits"].ndim == 3 else 1
        if raw["type_logits"].ndim == 2:
            raw = {k: v.unsqueeze(1) for k, v in raw.items()}
            ref = None if ref is None else {k: v.unsqueeze(1) for k, v in ref.items()}
        # hooks.py:2226-2246: legality from the public state of the retained row
        combos = torch.zeros((rows, policy.machine.geometry.players), dtype=torch.int32,
                             device=sigma["model_input"].device)
        state = policy.machine.state_from_model_input(batch.input_type, sigma["model_input"], combos)
        mask = policy.machine.legality(state).mask
        heads = {}
        if "trace_target" in sigma or "cost_target" in sigma:
            heads = dict(trace_pred=evaluation.public_heads["trace"], cost_pred=evaluation.public_heads["cost"],
                         trace_target=sigma["trace_target"], cost_target=sigma["cost_target"])
        ptr = None if action_rows == rows and not heads else batch.action_ptr
        result = poker_learner_loss(None, raw, value.reshape(rows, width), mask=mask, action=action["action"],
                                    old_log_policy=old.reshape(action_rows, width),
                                    advantage_target=adv.reshape(action_rows, width),
                                    old_value=old_value.reshape(rows, width), value_target=target.reshape(rows, width),
                                    controls=loss_controls, posterior=posterior, action_ptr=ptr, reference_raw=ref,
                                    **heads)
        return LossResult(*(getattr(result, name) for name in LossResult.__dataclass_fields__))

    return forward_loss


@dataclass
class Installed:
    """What ``install`` replaced: (module, name, original value)."""

    replaced: list


def install(*, machine: bool = True, policy: bool = True, targets: bool = True, learner: bool = False
            ) -> Installed:
    """Replace the reference's hot-path constructors with this build's; returns a restore handle."""

    from .targets import layered_target_cuda

    drop_ins = {"machine": EngineStateMachine, "policy": EnginePolicyOperator, "targets": layered_target_cuda}
    wanted = {"machine": machine, "policy": policy, "targets": targets}
    replaced = []
    for module_name, name, kind in _TARGETS:
        if not wanted[kind]:
            continue
        module = importlib.import_module(module_name)
        if not hasattr(module, name):
            raise AttributeError(f"{module_name} has no {name}: the reference layout changed")
        replaced.append((module, name, getattr(module, name)))
        setattr(module, name, drop_ins[kind])
    if learner:
        from pbg.core.learner import LearnerOperation

        replaced.append((LearnerOperation, "forward_loss", LearnerOperation.forward_loss))
        LearnerOperation.forward_loss = _fused_forward_loss(LearnerOperation.forward_loss)
    return Installed(replaced)


def uninstall(handle: Installed) -> None:
    for module, name, original in reversed(handle.replaced):
        setattr(module, name, original)
    handle.replaced.clear()


__all__ = ["EnginePolicyOperator", "EngineStateMachine", "Installed", "install", "uninstall"]
