"""Route an imported reference package (pbg) to libpbgb200 for the hot path.

The reference builds its game operations from a few classes and loaders:

* ``PokerStateMachine(geometry)`` in the sequential and branched hooks
  (pbg/games/poker/queued/hooks.py:1305, 2210; branching.py:185), the root
  payload (operations.py:394, 593) and the queued model (model.py:197-299);
* ``PokerPolicyOperator()`` in the operations bundle and the hooks
  (operations.py:149, hooks.py:1310, 2211);
* ``layered_target_cuda()``, the layered-targets extension loader that the
  target executor calls (pbg/core/targets.py:24, 634).

``install()`` replaces exactly those names in the imported modules with this
build's drop-ins, so every rollout step (legality, chip accounting, keyed
chance, histories, leaves, model-input rows), every policy evaluation
(sampling, selected log pi, the learner's differentiable policy operation) and
every layered-target pass of the reference's own engine runs on the sm_100a
kernels, while the engine, storage, scheduling and the showdown binding
(``poker_gpu_evaluator``, already this build's module) stay the reference's.
``uninstall(handle)`` restores the originals.

The learner's tensor program must run eagerly
(``run.execution.tensor_program.mode: eager``): the reference compiles that
program with ``torch.compile(fullgraph=True)``, which cannot trace a call into
a shared library.
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

    def rb_leaf(self, *args, **kwargs):
        """hooks.py:1218-1271: Rao-Blackwell leaves go to the external evaluator's completion, which
        this build does not provide; sampled settlement (``sampled_leaf``) is on the device."""

        raise NotImplementedError("Rao-Blackwell leaf completion is not part of this build")


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


@dataclass
class Installed:
    """What ``install`` replaced: (module, name, original value)."""

    replaced: list


def install(*, machine: bool = True, policy: bool = True, targets: bool = True) -> Installed:
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
    return Installed(replaced)


def uninstall(handle: Installed) -> None:
    for module, name, original in reversed(handle.replaced):
        setattr(module, name, original)
    handle.replaced.clear()


__all__ = ["EnginePolicyOperator", "EngineStateMachine", "Installed", "install", "uninstall"]
