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
    (128, 64, 64, None, True),
    (1000, 256, 768, None, True),      # M tail, three 256-wide column tiles
    (777, 256, 1024, "gelu", True),    # FFN w1 shape
    (4096, 1024, 256, None, True),     # FFN w2 shape
    (300, 128, 96, None, False),       # 96-wide tile, no bias
    (5000, 512, 160, "gelu", True),    # 160-wide tile
    (1, 64, 32, "gelu", True),         # one row
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
        linear(x, w)
    with pytest.raises(NativeError):
        linear(x.float(), w)
