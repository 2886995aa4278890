"""The fp32 preflop-class MLP of cfg1 and one learner step over it.

The reference has no MLP: its preflop model is a transformer over class-row
tokens (pbg/games/poker/model/preflop.py).  cfg1 names a preflop-class MLP
(two hidden layers of 256, fp32), which the reference admits behind its
``ModelOperation`` protocol (pbg/core/learner.py:324-350; the reference runs
such non-production models in its own tests, tests/model_support.py): one
retained preflop row in, the raw composite-policy fields and the value of each
of the K private class rows out, with the reference heads' activations
(pbg/games/poker/model/heads.py:28-62).  Its parity is therefore to a PyTorch
restatement of the same network.

``MLPLearnerStep`` is the learner step the metric counts (learner
presentations through forward, loss and backward, then the optimizer):
dense maps on cuBLAS (plain fp32 GEMMs), the bias/ReLU epilogues, the heads
and their backward, the bias gradients (``csrc/mlp.cu``), the fused poker
objective (``pbg_poker_learner_objective``) and the flat AdamW transition
(``pbg_adam_step``) from this library.  Parameters and gradients are single
flat fp32 buffers (the reference's DenseGradientOwner layout,
optimization.py:106-169), so the gradient SUM across ranks is one buffer.
"""

from __future__ import annotations

import math

import torch
from torch import Tensor

from . import _native as N
from ._native import call, ptr, stream
from .learner import PokerLearnerObjective
from .optim import FlatAdam
from .poker import NLHEGeometry


WGRAD_CHUNK = 512  # rows per partial weight gradient


def _weight_gradient(dy: Tensor, x: Tensor, out: Tensor) -> None:
    """out = dy^T x over S rows.  The output is small and the reduction long, so the rows are cut into
    chunks of WGRAD_CHUNK whose partial products run as one batched GEMM (enough tiles for every SM),
    then summed over the chunks (a fixed-order reduction); the remainder rows are added last."""

    S = dy.shape[0]
    chunks = S // WGRAD_CHUNK
    if chunks < 2:
        torch.mm(dy.t(), x, out=out)
        return
    rows = chunks * WGRAD_CHUNK
    parts = torch.bmm(dy[:rows].view(chunks, WGRAD_CHUNK, -1).transpose(1, 2), x[:rows].view(chunks, WGRAD_CHUNK, -1))
    torch.sum(parts, 0, out=out)
    if rows < S:
        out.addmm_(dy[rows:].t(), x[rows:])


class PreflopMLP:
    """x [S, W_pre] -> ReLU(x W1^T + b1) -> ReLU(. W2^T + b2) -> . W3^T + b3 -> heads of the sampled row."""

    def __init__(self, geometry: NLHEGeometry, *, hidden: int = 256, mixtures: int = 2, s_min: float = 0.02,
                 seed: int = 0, device="cuda") -> None:
        self.geometry = geometry
        self.K = geometry.private_classes
        self.M = int(mixtures)
        self.row = 4 + 3 * self.M
        self.out = self.K * self.row + self.K
        self.inp = geometry.preflop_model_input_width
        self.hidden = int(hidden)
        self.s_min = float(s_min)
        self.device = torch.device(device)
        self.shapes = [("w1", (hidden, self.inp)), ("b1", (hidden,)), ("w2", (hidden, hidden)), ("b2", (hidden,)),
                       ("w3", (self.out, hidden)), ("b3", (self.out,))]
        self.numel = sum(math.prod(shape) for _, shape in self.shapes)
        g = torch.Generator().manual_seed(seed)
        parts = []
        for name, shape in self.shapes:  # torch.nn.Linear's default initialisation
            fan_in = shape[1] if name.startswith("w") else dict(self.shapes)["w" + name[1]][1]
            bound = 1.0 / math.sqrt(fan_in)
            parts.append((torch.rand(shape, generator=g) * 2 - 1).mul_(bound).reshape(-1))
        self.master = torch.cat(parts).to(self.device).contiguous()
        self.params = self.views(self.master)
        self._status = torch.zeros(1, dtype=torch.int32, device=self.device)

    def views(self, flat: Tensor) -> dict:
        out, offset = {}, 0
        for name, shape in self.shapes:
            n = math.prod(shape)
            out[name] = flat[offset:offset + n].view(shape)
            offset += n
        return out

    def forward(self, x: Tensor, sampled_class: Tensor):
        """Raw fields of the sampled class row ([S,1,...]), its value [S,1] and the backward cache."""

        if x.dtype != torch.float32 or x.ndim != 2 or x.shape[1] != self.inp or not x.is_cuda:
            raise ValueError(f"model input must be CUDA fp32 [S, {self.inp}]")
        S = x.shape[0]
        p = self.params
        dev = x.device
        x = x.contiguous()
        cls = sampled_class.to(torch.int32).contiguous()
        h1 = torch.mm(x, p["w1"].t())
        call("pbg_mlp_bias_relu", S, self.hidden, ptr(h1), ptr(p["b1"]), stream(dev))
        h2 = torch.mm(h1, p["w2"].t())
        call("pbg_mlp_bias_relu", S, self.hidden, ptr(h2), ptr(p["b2"]), stream(dev))
        z = torch.mm(h2, p["w3"].t())
        M = self.M
        raw = {"type_logits": torch.empty((S, 1, 3), device=dev), "omega": torch.empty((S, 1, M), device=dev),
               "mu": torch.empty((S, 1, M), device=dev), "s": torch.empty((S, 1, M), device=dev),
               "iota": torch.empty((S, 1), device=dev)}
        value = torch.empty((S, 1), device=dev)
        call("pbg_mlp_heads", S, self.K, M, self.s_min, ptr(z), self.out, ptr(p["b3"]), ptr(cls),
             ptr(raw["type_logits"]), ptr(raw["omega"]), ptr(raw["mu"]), ptr(raw["s"]), ptr(raw["iota"]),
             ptr(value), ptr(self._status), stream(dev))
        return raw, value, (x, h1, h2, z, cls, raw)

    def check(self) -> None:
        """Raise if a forward saw a class id outside [0, K) (one device read)."""

        if int(self._status.item()):
            self._status.zero_()
            raise ValueError(f"sampled class ids must lie in [0, {self.K})")

    def backward(self, cache, d_raw: dict, d_value: Tensor, grad: Tensor) -> None:
        """Gradient of the objective with respect to every parameter, written into the flat ``grad``."""

        x, h1, h2, z, cls, raw = cache
        S = x.shape[0]
        dev = x.device
        p = self.params
        g = self.views(grad)
        dz = torch.empty((S, self.out), device=dev)
        f = lambda t: t.detach().float().contiguous()  # noqa: E731
        call("pbg_mlp_heads_backward", S, self.K, self.M, ptr(z), self.out, ptr(p["b3"]), ptr(cls),
             ptr(raw["omega"]), ptr(raw["mu"]), ptr(raw["iota"]), ptr(f(d_raw["type_logits"])),
             ptr(f(d_raw["omega"])), ptr(f(d_raw["mu"])), ptr(f(d_raw["s"])), ptr(f(d_raw["iota"])),
             ptr(f(d_value)), ptr(dz), self.out, stream(dev))
        partial = torch.empty(int(N.lib().pbg_mlp_bias_partials(S, max(self.out, self.hidden))), device=dev)
        call("pbg_mlp_relu_backward_bias", S, self.out, ptr(dz), None, ptr(g["b3"]), ptr(partial), partial.numel(),
             stream(dev))
        _weight_gradient(dz, h2, g["w3"])
        dh2 = torch.mm(dz, p["w3"])
        call("pbg_mlp_relu_backward_bias", S, self.hidden, ptr(dh2), ptr(h2), ptr(g["b2"]), ptr(partial),
             partial.numel(), stream(dev))
        _weight_gradient(dh2, h1, g["w2"])
        dh1 = torch.mm(dh2, p["w2"])
        call("pbg_mlp_relu_backward_bias", S, self.hidden, ptr(dh1), ptr(h1), ptr(g["b1"]), ptr(partial),
             partial.numel(), stream(dev))
        _weight_gradient(dh1, x, g["w1"])


class MLPLearnerStep:
    """Forward, fused objective, backward and AdamW of the cfg1 MLP over one learner batch (sampled rows)."""

    def __init__(self, model: PreflopMLP, *, lr: float = 3e-4, beta1: float = 0.9, beta2: float = 0.999,
                 epsilon: float = 1e-8, weight_decay: float = 0.0, grad_clip: float = 1.0) -> None:
        self.model = model
        self.objective = PokerLearnerObjective(model.device)
        self.adam = FlatAdam(model.master, lr=lr, beta1=beta1, beta2=beta2, epsilon=epsilon, decay=weight_decay,
                             clip=grad_clip)

    def gradient(self, batch: dict):
        """Forward, objective and backward: the flat gradient lands in ``self.adam.grad``."""

        m = self.model
        raw, value, cache = m.forward(batch["model_input"], batch["sampled_class"])
        result, grads = self.objective(raw, batch["mask"], batch["action"], batch["old_log_policy"],
                                       batch["advantage_target"], value, batch["old_value"], batch["value_target"],
                                       batch["controls"], batch["lane_weight"])
        m.backward(cache, grads, grads["value"], self.adam.grad)
        return result

    def __call__(self, batch: dict):
        result = self.gradient(batch)
        self.adam.step()
        return result


__all__ = ["MLPLearnerStep", "PreflopMLP"]
