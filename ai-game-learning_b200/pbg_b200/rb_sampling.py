"""Collision-conditioned posterior profiles (pbg/games/poker/queued/rb_sampling.py).

``CollisionConditionedProfileSampler.sample_children`` keeps the reference's
keyword arguments, result (one generating profile per child row, int32
``[G, P]``) and ``last_observation``; the whole bounded attempt envelope runs
in ``pbg_posterior_sample_children`` (a CDF pass over the parents and one warp
per child row with lanes over attempts).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from ._native import call, lib, ptr, stream
from .poker import NLHEGeometry

POSTERIOR_MAX_ATTEMPTS = 256


class PosteriorSamplingError(RuntimeError):
    """A posterior-profile request violated the bounded CUDA contract."""


@dataclass(frozen=True)
class RejectionObservation:
    """Device-resident rejection-tail telemetry for one sampler call."""

    attempt_count: Tensor
    exhausted: Tensor
    minimum_failing_address: Tensor


class CollisionConditionedProfileSampler:
    """Exact all-or-reject posterior sampler with logical CUDA addresses (rb_sampling.py:58-84)."""

    def __init__(self, geometry: NLHEGeometry, *, max_attempts: int = POSTERIOR_MAX_ATTEMPTS) -> None:
        if isinstance(max_attempts, bool) or not isinstance(max_attempts, int) or max_attempts <= 0:
            raise ValueError("max_attempts must be a positive integer")
        self.geometry = geometry
        self.max_attempts = max_attempts
        self.last_observation: RejectionObservation | None = None

    def sample_children(self, *, range_weights: Tensor, board_cards: Tensor, inherited_profile: Tensor,
                        source: Tensor, ordinal: Tensor, active: Tensor, root: Tensor, path: Tensor, seed: int,
                        iteration: int, retry_epoch: Tensor | int) -> Tensor:
        device = range_weights.device
        players, hands = self.geometry.players, self.geometry.private_hands
        if device.type != "cuda":
            raise PosteriorSamplingError("branched RB sampling requires CUDA")
        if (range_weights.dtype != torch.float32 or range_weights.ndim != 3
                or range_weights.shape[1:] != (players, hands)
                or board_cards.shape != (range_weights.shape[0], 5) or board_cards.dtype != torch.uint8
                or inherited_profile.shape != (range_weights.shape[0], players)
                or inherited_profile.dtype != torch.int32):
            raise PosteriorSamplingError("posterior parents require FP32 [B,P,H], uint8 [B,5], and int32 [B,P]")
        edges = source.numel()
        if any(value.device != device or value.shape != (edges,) for value in (source, ordinal, active, root, path)):
            raise PosteriorSamplingError("posterior child descriptors must be device-local [G]")
        if active.dtype != torch.bool:
            raise PosteriorSamplingError("posterior active mask must be bool")
        parents = range_weights.shape[0]
        if edges and bool(((source < 0) | (source >= parents) | (ordinal < 0)).any()):
            raise PosteriorSamplingError("posterior source or child ordinal is invalid")
        epoch_rows, epoch_scalar = None, 0
        if torch.is_tensor(retry_epoch):
            if retry_epoch.numel() == 1:
                epoch_scalar = int(retry_epoch.reshape(()).item())
            elif retry_epoch.numel() == edges:
                epoch_rows = retry_epoch.reshape(edges).to(device=device, dtype=torch.int64).contiguous()
            else:
                raise PosteriorSamplingError("retry_epoch must be a scalar or hold one value per child row")
        else:
            epoch_scalar = int(retry_epoch)
        g = self.geometry.c
        work = torch.empty(int(lib().pbg_posterior_workspace_floats(g, parents)), dtype=torch.float32, device=device)
        profile = torch.empty((edges, players), dtype=torch.int32, device=device)
        count = torch.empty(edges, dtype=torch.int32, device=device)
        exhausted = torch.empty(edges, dtype=torch.bool, device=device)
        worst = torch.empty((), dtype=torch.int64, device=device)
        status = torch.zeros(1, dtype=torch.int32, device=device)
        i64 = lambda t: t.to(torch.int64).contiguous()  # noqa: E731
        call("pbg_posterior_sample_children", g, parents, ptr(range_weights.contiguous()),
             ptr(board_cards.contiguous()), ptr(inherited_profile.contiguous()), edges, ptr(i64(source)),
             ptr(i64(ordinal)), ptr(active.contiguous()), ptr(i64(root)), ptr(i64(path)), int(seed),
             int(iteration), ptr(epoch_rows), epoch_scalar, self.max_attempts, ptr(work), ptr(profile), ptr(count),
             ptr(exhausted), ptr(worst), ptr(status), stream(device))
        if int(status.item()):
            raise PosteriorSamplingError("posterior seat has no board-legal mass")
        self.last_observation = RejectionObservation(count, exhausted, worst)
        return profile


__all__ = ["POSTERIOR_MAX_ATTEMPTS", "CollisionConditionedProfileSampler", "PosteriorSamplingError",
           "RejectionObservation"]
