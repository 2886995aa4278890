"""tcgen05 linear layer against a plain PyTorch fp32 reference of the same map.

Tolerance: bf16 output rounding (2^-8 relative) plus fp32 accumulation-order
differences: rtol 2e-2, atol 2e-2 on O(1) values.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _ref(x, w, b, act):
    y = x.float() @ w.float().t()
    if b is not None:
        y = y + b
    if act == "gelu":
        y = torch.nn.functional.gelu(y)
    return y


@pytest.mark.parametrize("m,k,n,act,bias", [
    (128, 64, 128, None, True),
    (1000, 256, 768, None, True),      # M tail, three 256-wide column tiles
    (777, 256, 1024, "gelu", True),    # FFN w1 shape
    (4096, 1024, 256, None, True),     # FFN w2 shape
    (300, 128, 384, None, False),      # 128-wide tiles, no bias
    (5000, 512, 640, "gelu", True),    # 128-wide tiles
    (1, 64, 128, "gelu", True),        # one row
    (33, 256, 128, "gelu", True),      # rows past M in the first 32-row block
])
def test_linear_matches_fp32_reference(m, k, n, act, bias):
    from pbg_b200.model import linear, pipeline_error

    g = torch.Generator(device=DEV).manual_seed(m * 7 + n)
    x = (torch.randn((m, k), generator=g, device=DEV) / 2).to(torch.bfloat16)
    w = (torch.randn((n, k), generator=g, device=DEV) / k ** 0.5).to(torch.bfloat16)
    b = torch.randn((n,), generator=g, device=DEV) * 0.1 if bias else None
    y = linear(x, w, b, act)
    torch.cuda.synchronize()
    assert pipeline_error(DEV) == 0
    torch.testing.assert_close(y.float(), _ref(x, w, b, act), rtol=2e-2, atol=2e-2)


def test_linear_batched_shape_and_ffn():
    from pbg_b200.model import FFN, Linear, pipeline_error

    g = torch.Generator(device=DEV).manual_seed(3)
    d, hidden = 256, 1024
    x = (torch.randn((4, 93, d), generator=g, device=DEV) / 2).to(torch.bfloat16)
    w1 = Linear((torch.randn((hidden, d), generator=g, device=DEV) / d ** 0.5), torch.randn(hidden, device=DEV) * 0.1)
    w2 = Linear((torch.randn((d, hidden), generator=g, device=DEV) / hidden ** 0.5), torch.randn(d, device=DEV) * 0.1)
    y = FFN(w1, w2)(x)
    torch.cuda.synchronize()
    assert pipeline_error(DEV) == 0
    assert y.shape == (4, 93, d)
    h = torch.nn.functional.gelu(x.float() @ w1.weight.float().t() + w1.bias).to(torch.bfloat16)
    ref = h.float() @ w2.weight.float().t() + w2.bias
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2)


def test_linear_rejects_unsupported_shapes():
    from pbg_b200._native import NativeError
    from pbg_b200.model import linear

    x = torch.zeros((8, 100), dtype=torch.bfloat16, device=DEV)
    w = torch.zeros((64, 100), dtype=torch.bfloat16, device=DEV)
    with pytest.raises(NativeError):
        linear(x, w)  # K not a multiple of 64
    with pytest.raises(NativeError):
        linear(torch.zeros((8, 64), dtype=torch.bfloat16, device=DEV),
               torch.zeros((192, 64), dtype=torch.bfloat16, device=DEV))  # N not a multiple of 128
    with pytest.raises(NativeError):
        linear(x.float(), w)


def test_gelu_epilogue_matches_torch_gelu_to_bf16_rounding():
    # identity weights: the layer evaluates GELU(x + b) directly; the epilogue's erf
    # (Abramowitz & Stegun 7.1.26, |error| <= 1.5e-7) stays within one bf16 ulp (plus 1e-6
    # absolute in the far negative tail, where GELU itself is below 1e-5)
    from pbg_b200.model import linear

    n = 128
    x = torch.linspace(-8, 8, 4096 * n, device=DEV).reshape(4096, n).to(torch.bfloat16)
    w = torch.eye(n, device=DEV, dtype=torch.bfloat16)
    b = torch.zeros(n, device=DEV)
    y = linear(x, w, b, "gelu").float()
    ref = torch.nn.functional.gelu(x.float())
    ulp = ref.abs().clamp_min(1e-30) * 2.0 ** -8
    assert bool(((y - ref).abs() <= ulp + 1e-6).all())
    # a bf16 rounding may only flip where the erf's absolute error is relatively small
    body = ref.abs() >= 1e-2
    flips = (y[body] != ref[body].to(torch.bfloat16).float()).float().mean().item()
    assert flips < 0.01
