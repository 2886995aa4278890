"""Loss backward fused with the readout's weight gradient (pbg_ppo_readout_backward).

The logits come from a readout x = h W^T + b (pbg/core/tensor_ops.py:25-38); autograd forms the
weight and bias gradients from the loss's dlogits (pbg/core/learner.py:2021-2077).  The fused pass must
write the same dlogits as the plain loss backward (same arithmetic per row: bit-identical) and
dweight = dlogits^T h, dbias = sum dlogits against a float64 torch restatement over the kernel's own
bf16 dlogits, within rtol 1e-5 of the sum of the terms' magnitudes (the fp32 tolerance).
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _inputs(N, d, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    logits = torch.randn((N, 8), generator=g, device=DEV).to(torch.bfloat16)
    mask = torch.rand((N, 8), generator=g, device=DEV) < 0.7
    mask[:, 0] |= ~mask.any(1)
    cum = mask.cumsum(1)
    pick = (torch.rand(N, generator=g, device=DEV) * cum[:, -1]).long()
    action = (cum <= pick[:, None]).sum(1).to(torch.int32)
    old = torch.log_softmax((logits.float() + 0.1 * torch.randn((N, 8), generator=g, device=DEV))
                            .masked_fill(~mask, -torch.inf), -1).gather(1, action.long()[:, None])[:, 0]
    adv = torch.randn(N, generator=g, device=DEV)
    weight = torch.rand(N, generator=g, device=DEV)
    hidden = torch.randn((N, d), generator=g, device=DEV).to(torch.bfloat16)
    return logits, mask, action, old.contiguous(), adv, weight, hidden


def _check_readout(dl, hidden, dweight, dbias):
    d64, h64 = dl.double(), hidden.double()
    ref_w = d64.T @ h64
    mag_w = d64.abs().T @ h64.abs()
    assert torch.all((dweight.double() - ref_w).abs() <= 1e-5 * mag_w + 1e-30), "dweight differs"
    ref_b, mag_b = d64.sum(0), d64.abs().sum(0)
    assert torch.all((dbias.double() - ref_b).abs() <= 1e-5 * mag_b + 1e-30), "dbias differs"


@pytest.mark.parametrize("N,d", [(4999, 64), (5000, 128), (300_001, 128), (70_000, 256), (453, 256), (33, 128)])
def test_readout_backward_matches_loss_and_torch(N, d):
    from pbg_b200.loss import FusedPPOBackward, FusedPPOReadoutBackward, LossConfig

    cfg = LossConfig(0.2, 1.5, 0.01)
    logits, mask, action, old, adv, weight, hidden = _inputs(N, d, 7 + d)
    plain = FusedPPOBackward(N, 8, DEV, cfg)
    want_d, want_s = plain(logits, mask, action, old, adv, weight)
    want_s = want_s.clone()
    fused = FusedPPOReadoutBackward(N, d, DEV, cfg)
    for call in range(2):  # the second call reuses the cleared scratch
        dl, dweight, dbias, stats = fused(logits, mask, action, old, adv, weight, hidden)
        torch.cuda.synchronize()
        assert torch.equal(dl, want_d), f"dlogits differ from the loss backward (call {call})"
        s, w = stats.cpu().numpy(), want_s.cpu().numpy()
        np.testing.assert_allclose(s[[0, 1, 2, 3, 6, 7]], w[[0, 1, 2, 3, 6, 7]], rtol=1e-5, atol=1e-9 * N)
        assert s[4] == w[4] and s[5] == w[5] and s[7] == N
        _check_readout(dl, hidden, dweight, dbias)


@pytest.mark.parametrize("d", [128, 256])
def test_readout_backward_unaligned_row_streams(d):
    """Per-row streams that are not 16-byte aligned take the direct-load kernel; same results."""

    from pbg_b200.loss import FusedPPOBackward, FusedPPOReadoutBackward, LossConfig

    N = 20_001
    logits, mask, action, old, adv, weight, hidden = _inputs(N + 1, d, 3)
    logits, mask, hidden = logits[:N].contiguous(), mask[:N].contiguous(), hidden[:N].contiguous()
    action, old, adv, weight = action[1:], old[1:], adv[1:], weight[1:]  # 4-byte offsets
    assert action.data_ptr() % 16 != 0
    want_d, want_s = FusedPPOBackward(N, 8, DEV, LossConfig())(logits, mask, action, old, adv, weight)
    dl, dweight, dbias, stats = FusedPPOReadoutBackward(N, d, DEV)(logits, mask, action, old, adv, weight, hidden)
    torch.cuda.synchronize()
    assert torch.equal(dl, want_d)
    np.testing.assert_allclose(stats.cpu().numpy()[[0, 6, 7]], want_s.cpu().numpy()[[0, 6, 7]], rtol=1e-5)
    _check_readout(dl, hidden, dweight, dbias)


def test_readout_backward_matches_the_oracle():
    """Against the CPU restatement (double precision, from the un-rounded gradient): the kernel sums the
    bf16 dlogits it writes, so the bar is the bf16 one, 2e-2 of the sum of the terms' magnitudes."""

    import math

    import oracle as O
    from pbg_b200.loss import FusedPPOReadoutBackward, LossConfig

    N, d = 5000, 128
    logits, mask, action, old, adv, weight, hidden = _inputs(N, d, 21)
    dl, dweight, dbias, stats = FusedPPOReadoutBackward(N, d, DEV, LossConfig(0.2, 1.5, 0.01))(
        logits, mask, action, old, adv, weight, hidden)
    torch.cuda.synchronize()
    host = lambda t: t.detach().cpu().numpy()  # noqa: E731
    ref_d, ref_w, ref_b, ref_s = O.ppo_readout(host(logits.float()), host(mask), host(action), host(old), host(adv),
                                               host(weight), host(hidden.float()), log_cap=math.log(1.5))
    mag_w = np.abs(ref_d).astype(np.float64).T @ np.abs(host(hidden.float())).astype(np.float64)
    assert np.all(np.abs(host(dweight) - ref_w) <= 2e-2 * mag_w + 1e-30)
    assert np.all(np.abs(host(dbias) - ref_b) <= 2e-2 * np.abs(ref_d).sum(0) + 1e-30)
    np.testing.assert_allclose(host(stats)[[0, 6, 7]], ref_s[[0, 6, 7]], rtol=1e-4, atol=1e-9 * N)


def test_readout_backward_empty_batch_and_bad_arguments():
    from pbg_b200._native import lib, ptr
    from pbg_b200.loss import FusedPPOReadoutBackward

    fused = FusedPPOReadoutBackward(0, 128, DEV)
    fused.dweight.fill_(7.0)
    empty = torch.empty((0, 8), dtype=torch.bfloat16, device=DEV)
    e = torch.empty(0, device=DEV)
    dl, dweight, dbias, stats = fused(empty, torch.empty((0, 8), dtype=torch.bool, device=DEV),
                                      torch.empty(0, dtype=torch.int32, device=DEV), e, e, e,
                                      torch.empty((0, 128), dtype=torch.bfloat16, device=DEV))
    torch.cuda.synchronize()
    assert torch.count_nonzero(dweight) == 0 and torch.count_nonzero(dbias) == 0 and float(stats[7]) == 0.0

    L = lib()
    assert L.pbg_ppo_readout_partials_size(100, 8, 96) == -1
    out = torch.zeros(16, device=DEV)
    rc = L.pbg_ppo_readout_backward(16, 8, None, None, None, None, None, None, ptr(out), None, 96, None, ptr(out),
                                    ptr(out), ptr(out), ptr(out), None)
    assert rc == -1 and b"hidden width" in L.pbg_last_error()
    rc = L.pbg_ppo_readout_backward(16, 4, None, None, None, None, None, None, ptr(out), None, 128, None, ptr(out),
                                    ptr(out), ptr(out), ptr(out), None)
    assert rc == -1 and b"A == 8" in L.pbg_last_error()
