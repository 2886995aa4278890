"""The allocation-free PPO loss entry point against the regular one.

pbg_ppo_categorical_backward_noalloc serves callers that cannot allocate
device memory (hosts that own all device memory through their own pool,
bindings that cannot pass a scratch buffer): its per-block statistics live in
an array built into the library.  It must give the same gradients and loss
statistics as pbg_ppo_categorical_backward with caller scratch, on
consecutive calls that reuse the built-in array.  This file sorts last so
that a run stopping at the first failure has run every other test first.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _inputs(N, A, seed, dtype):
    g = torch.Generator(device=DEV).manual_seed(seed)
    logits = torch.randn((N, A), generator=g, device=DEV).to(dtype)
    mask = torch.rand((N, A), generator=g, device=DEV) < 0.7
    mask[:, 0] |= ~mask.any(1)
    cum = mask.cumsum(1)
    pick = (torch.rand(N, generator=g, device=DEV) * cum[:, -1]).long()
    action = (cum <= pick[:, None]).sum(1).to(torch.int32)
    old = torch.log_softmax((logits.float() + 0.3 * torch.randn((N, A), generator=g, device=DEV))
                            .masked_fill(~mask, -torch.inf), -1).gather(1, action.long()[:, None])[:, 0]
    adv = torch.randn(N, generator=g, device=DEV)
    weight = torch.rand(N, generator=g, device=DEV)
    return logits.contiguous(), mask.contiguous(), action.contiguous(), old.contiguous(), adv, weight


@pytest.mark.parametrize("A,dtype", [(8, torch.bfloat16), (5, torch.float32)])
def test_noalloc_loss_matches_caller_scratch_on_consecutive_calls(A, dtype):
    from pbg_b200._native import call, lib, ptr, stream

    L = lib()
    controls = torch.tensor([0.2, float(np.log(2.0)), 0.01, 1.0, 1.0 / 300_000], dtype=torch.float32, device=DEV)
    for call_index, (N, seed) in enumerate(((300_000, 1), (123_457, 2))):
        logits, mask, action, old, adv, weight = _inputs(N, A, seed, dtype)
        code = 1 if dtype == torch.bfloat16 else 0
        partials = torch.zeros(int(L.pbg_ppo_partials_size(N, A)), dtype=torch.float64, device=DEV)
        ref_d = torch.empty_like(logits)
        ref_s = torch.zeros(8, dtype=torch.float64, device=DEV)
        call("pbg_ppo_categorical_backward", N, A, code, ptr(logits), ptr(mask), ptr(action), ptr(old), ptr(adv),
             ptr(weight), ptr(controls), ptr(ref_d), ptr(partials), ptr(ref_s), stream())
        got_d = torch.full_like(logits, float("nan"))
        got_s = torch.full((8,), float("nan"), dtype=torch.float64, device=DEV)
        call("pbg_ppo_categorical_backward_noalloc", N, A, code, ptr(logits), ptr(mask), ptr(action), ptr(old),
             ptr(adv), ptr(weight), ptr(controls), ptr(got_d), ptr(got_s), stream())
        torch.cuda.synchronize()
        scale = float(ref_d.float().abs().max())
        torch.testing.assert_close(got_d.float(), ref_d.float(), rtol=1e-5, atol=1e-5 * scale,
                                   msg=f"dlogits differ on call {call_index}")
        torch.testing.assert_close(got_s, ref_s, rtol=1e-5, atol=1e-9 * N, msg=f"statistics differ on call {call_index}")
        assert int(got_s[7]) == N


def test_noalloc_rejects_bad_arguments():
    from pbg_b200._native import lib

    L = lib()
    rc = L.pbg_ppo_categorical_backward_noalloc(16, 40, 0, None, None, None, None, None, None, None, None, None,
                                                None)
    assert rc == -1
    assert b"A in [1,32]" in L.pbg_last_error()
