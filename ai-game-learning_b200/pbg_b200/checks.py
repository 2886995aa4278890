"""Device-side input checks that never fault the CUDA context.

The reference validates device tensors with ``accelerator_assert``
(pbg/games/poker/model/primitives.py:15-21) and ``torch._assert_async``, which
end the CUDA context when they fire.  Here a failed check sets its bit in a
per-device flag word without reading the device; ``input_errors`` reads it and
``raise_input_errors`` raises the reference's ValueError on the host.
"""

from __future__ import annotations

import torch
from torch import Tensor

_MESSAGES: list[str] = []
_FLAGS: dict = {}


def _assert(condition: Tensor, message: str) -> None:
    """primitives.py:15-21 (accelerator_assert): a ValueError on the host; on CUDA the check's bit in
    the device's flag word, set without a device read."""

    if condition.device.type != "cuda":
        if not bool(condition):
            raise ValueError(message)
        return
    if message not in _MESSAGES:
        _MESSAGES.append(message)
    index = _MESSAGES.index(message)
    flags = _FLAGS.get(condition.device)
    if flags is None:
        flags = _FLAGS[condition.device] = torch.zeros(64, dtype=torch.bool, device=condition.device)
    flags[index: index + 1].logical_or_(~condition.reshape(1))


def input_errors(device, reset: bool = True) -> list[str]:
    """The messages of the device-side input checks that failed since the last reset (reads the device)."""

    flags = _FLAGS.get(torch.device(device))
    if flags is None:
        return []
    failed = [_MESSAGES[i] for i in torch.nonzero(flags[: len(_MESSAGES)]).flatten().tolist()]
    if reset:
        flags.zero_()
    return failed


def raise_input_errors(device) -> None:
    """Raise ValueError, as the reference's checks do, when a device-side input check failed."""

    failed = input_errors(device)
    if failed:
        raise ValueError("; ".join(failed))


__all__ = ["input_errors", "raise_input_errors"]
