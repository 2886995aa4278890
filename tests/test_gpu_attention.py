"""tcgen05 attention core against a plain PyTorch fp32 reference of the same map.

softmax((q / temperature) . k / sqrt(32) + key_bias, masked keys excluded) . v per head,
from the same bf16 qkv; bf16 output: rtol/atol 2e-2.
"""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _reference(qkv, heads, q_scale, bias, mask):
    b, l, _ = qkv.shape
    x = qkv.float().reshape(b, l, 3, heads, 32)
    q, k, v = x[:, :, 0].transpose(1, 2), x[:, :, 1].transpose(1, 2), x[:, :, 2].transpose(1, 2)
    logits = torch.einsum("bhqd,bhkd->bhqk", q, k) * q_scale[None, :, None, None]
    if bias is not None:
        logits = logits + bias[:, None, None, :]
    if mask is not None:
        logits = logits.masked_fill(~mask[:, None, None, :], -math.inf)
    p = torch.nan_to_num(torch.softmax(logits, -1), nan=0.0)
    return torch.einsum("bhqk,bhkd->bhqd", p, v).transpose(1, 2).reshape(b, l, heads * 32)


@pytest.mark.parametrize("batch,length,heads,biased,masked", [
    (2, 5, 8, True, True),
    (3, 128, 8, True, False),
    (2, 300, 4, False, True),
    (2, 876, 8, True, True),     # cfg2's preflop sequence length
    (1, 257, 1, False, False),
])
def test_attention_matches_fp32_reference(batch, length, heads, biased, masked):
    from pbg_b200.model import attention, pipeline_error

    g = torch.Generator(device=DEV).manual_seed(batch * 1000 + length)
    qkv = torch.randn((batch, length, 3 * heads * 32), generator=g, device=DEV).to(torch.bfloat16)
    temperature = torch.nn.functional.softplus(torch.randn(heads, generator=g, device=DEV)) + 0.5
    q_scale = 1.0 / (temperature * math.sqrt(32))
    bias = torch.log(torch.rand((batch, length), generator=g, device=DEV).clamp_min(1e-6)) if biased else None
    mask = (torch.rand((batch, length), generator=g, device=DEV) > 0.3) if masked else None
    if mask is not None:
        mask[:, 0] = True
    out = attention(qkv, heads, q_scale, bias, mask)
    torch.cuda.synchronize()
    assert pipeline_error(DEV) == 0
    torch.testing.assert_close(out.float(), _reference(qkv, heads, q_scale, bias, mask), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("length,heads", [(2406, 8), (384, 8), (640, 2)])
def test_attention_rising_bias_moves_the_shift(length, heads):
    # a key bias rising along the sequence makes the running maximum grow block after block (the
    # shift of the accumulated output moves whenever it grows by more than 2^8); leading keys absent
    from pbg_b200.model import attention, pipeline_error

    batch = 2
    g = torch.Generator(device=DEV).manual_seed(length)
    qkv = torch.randn((batch, length, 3 * heads * 32), generator=g, device=DEV).to(torch.bfloat16)
    q_scale = torch.full((heads,), 1.0 / math.sqrt(32), device=DEV)
    bias = torch.linspace(-60.0, 20.0, length, device=DEV)[None].expand(batch, -1).contiguous()
    bias = bias + torch.randn((batch, length), generator=g, device=DEV)
    mask = torch.rand((batch, length), generator=g, device=DEV) > 0.2
    mask[0, :100] = False
    out = attention(qkv, heads, q_scale, bias, mask)
    torch.cuda.synchronize()
    assert pipeline_error(DEV) == 0
    torch.testing.assert_close(out.float(), _reference(qkv, heads, q_scale, bias, mask), rtol=2e-2, atol=2e-2)


def test_attention_all_keys_masked_gives_zero():
    from pbg_b200.model import attention

    qkv = torch.randn((1, 40, 3 * 64), device=DEV).to(torch.bfloat16)
    mask = torch.zeros((1, 40), dtype=torch.bool, device=DEV)
    out = attention(qkv, 2, torch.ones(2, device=DEV), None, mask)
    assert not out.float().abs().any()


def test_mha_forward_biased_composes_projections():
    from pbg_b200.model import MHA, Linear

    d, heads = 256, 8
    g = torch.Generator(device=DEV).manual_seed(4)
    w_qkv = Linear(torch.randn((3 * d, d), generator=g, device=DEV) / 16, torch.randn(3 * d, generator=g, device=DEV) * 0.1)
    w_o = Linear(torch.randn((d, d), generator=g, device=DEV) / 16, torch.randn(d, generator=g, device=DEV) * 0.1)
    theta = torch.full((heads,), math.log(math.expm1(0.5)), device=DEV)  # temperature 1 (the reference's init)
    mha = MHA(w_qkv, w_o, theta, heads)
    x = torch.randn((2, 200, d), generator=g, device=DEV).to(torch.bfloat16)
    bias = torch.randn((2, 200), generator=g, device=DEV)
    mask = torch.rand((2, 200), generator=g, device=DEV) > 0.2
    y = mha.forward_biased(x, bias, mask)
    qkv = (x.float() @ w_qkv.weight.float().t() + w_qkv.bias).to(torch.bfloat16)
    merged = _reference(qkv, heads, torch.full((heads,), 1 / math.sqrt(32), device=DEV), bias, mask).to(torch.bfloat16)
    ref = merged.float() @ w_o.weight.float().t() + w_o.bias
    torch.testing.assert_close(y.float(), ref, rtol=3e-2, atol=3e-2)
