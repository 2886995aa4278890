"""The fused epilogue of the tensor-core map (pbg_linear_ex), the batched-row LayerNorm
(pbg_layernorm_rows) and the incidence combine pass (pbg_incidence_combine) against plain torch
fp32 references of the same operations (pbg/games/poker/model/incidence.py:30-84, primitives.py FFN /
MHA maps, tensor_ops.py LayerNorm).  Tolerances: bf16 operands and outputs 2e-2; fp32 outputs of bf16
operands 1e-2 relative to the output scale; the combine pass is fp32 elementwise (its seat sums in
seat order, torch's reduction order differs: 1e-5), its bf16 copies within one bf16 rounding.
"""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _bf(x):
    return x.to(torch.bfloat16)


@pytest.mark.parametrize("m,n,k", [(300, 256, 256), (1000, 128, 384), (77, 256, 768)])
@pytest.mark.parametrize("mode", ["scale_f32", "residual_f32", "residual_gelu_bf16", "strided", "grouped_residual"])
def test_linear_ex_matches_torch(m, n, k, mode):
    from pbg_b200.model import linear_ex, pipeline_error

    g = torch.Generator(device=DEV).manual_seed(m + n + k)
    w = _bf(torch.randn((n, k), generator=g, device=DEV) / k ** 0.5)
    bias = torch.randn(n, generator=g, device=DEV) * 0.1
    wide = _bf(torch.randn((m, k + 64), generator=g, device=DEV))
    x = wide[:, 32: 32 + k] if mode == "strided" else wide[:, :k].contiguous()
    acc = x.float() @ w.float().T
    scale = torch.rand(m, generator=g, device=DEV)
    residual = torch.randn((m, n), generator=g, device=DEV)
    if mode == "scale_f32":
        y = linear_ex(x, w, None, row_scale=scale, out_dtype=torch.float32)
        want = acc * scale[:, None]
    elif mode == "residual_f32":
        y = linear_ex(x, w, bias, residual=residual, out_dtype=torch.float32)
        want = acc + bias + residual
    elif mode == "residual_gelu_bf16":
        y = linear_ex(x, w, bias, "gelu", residual=residual)
        want = F.gelu(acc + bias + residual)
    elif mode == "grouped_residual":  # one residual row per group of rows (a factored FFN's context)
        group = {300: 5, 1000: 8, 77: 7}[m]
        ctx = torch.randn((m // group, n), generator=g, device=DEV)
        y = linear_ex(x, w, bias, "gelu", residual=ctx, residual_group=group)
        want = F.gelu(acc + bias + ctx.repeat_interleave(group, 0))
    else:  # strided operand, fp32 residual slice, output into a column slice of a wider bf16 buffer
        out_wide = torch.zeros((m, n + 128), dtype=torch.bfloat16, device=DEV)
        res_wide = torch.randn((m, n + 64), generator=g, device=DEV)
        y = linear_ex(x, w, bias, residual=res_wide[:, 64:], out=out_wide[:, 128:])
        want = acc + bias + res_wide[:, 64:]
        assert torch.count_nonzero(out_wide[:, :128]) == 0
    torch.cuda.synchronize()
    assert pipeline_error(DEV) == 0
    tol = 2e-2 if y.dtype == torch.bfloat16 else 1e-2
    scale_ref = float(want.abs().max())
    assert float((y.float() - want).abs().max()) <= tol * max(1.0, scale_ref)


def test_layernorm_rows_matches_torch():
    from pbg_b200._native import call, ptr, rows_ptr, stream

    g = torch.Generator(device=DEV).manual_seed(5)
    batch, length, d, group = 7, 53, 256, 40
    x = torch.randn((batch, length, d), generator=g, device=DEV) * 3 + 1
    gain = torch.rand(d, generator=g, device=DEV) + 0.5
    bias = torch.randn(d, generator=g, device=DEV)
    out = torch.zeros((batch * group, 3 * d), dtype=torch.bfloat16, device=DEV)
    view = out[:, d: 2 * d]
    call("pbg_layernorm_rows", batch * group, d, group, ptr(x), 0, length * d, d, ptr(gain), ptr(bias), 1e-5,
         rows_ptr(view), 1, group * view.stride(0), view.stride(0), stream(DEV))
    want = F.layer_norm(x[:, :group], (d,), gain, bias, 1e-5).reshape(-1, d)
    torch.testing.assert_close(view.float(), want, rtol=2e-2, atol=2e-2)
    assert torch.count_nonzero(out[:, :d]) == 0 and torch.count_nonzero(out[:, 2 * d:]) == 0


@pytest.mark.parametrize("players", [2, 3, 9])
def test_incidence_combine_matches_reference_terms(players):
    from pbg_b200._native import call, ptr, stream

    g = torch.Generator(device=DEV).manual_seed(players)
    batch, rows, d, length, width = 3, 45, 128, 60, 640
    source = torch.randn((batch, players, rows, d), generator=g, device=DEV)
    overlap = torch.randn((batch, players, rows, d), generator=g, device=DEV)
    scale = torch.rand((batch, rows), generator=g, device=DEV)
    inc = torch.zeros((batch * players * rows, 3 * d), dtype=torch.bfloat16, device=DEV)
    other_card = torch.empty((batch, players, rows, d), device=DEV)
    ffn = torch.zeros((batch, length + players * rows, width), dtype=torch.bfloat16, device=DEV)
    call("pbg_incidence_combine", batch, players, rows, d, ptr(source), ptr(overlap), ptr(scale), ptr(inc), 3 * d,
         d, 2 * d, ptr(other_card), ptr(ffn), ffn.shape[1] * width, width, 2 * d, 3 * d, stream(DEV))
    same = source * scale[:, None, :, None]
    oe = same.sum(1, keepdim=True) - same
    oc = overlap.sum(1, keepdim=True) - overlap - 2.0 * oe
    own = overlap - 2.0 * same
    torch.testing.assert_close(other_card, oc, rtol=1e-5, atol=1e-5)
    inc4 = inc.view(batch, players, rows, 3 * d)
    ulp = dict(rtol=2 ** -7, atol=1e-5)  # one bf16 ulp: a rounding flip of an fp32 value differing in its last bits
    torch.testing.assert_close(inc4[..., d: 2 * d].float(), _bf(oe).float(), **ulp)
    torch.testing.assert_close(inc4[..., 2 * d:].float(), _bf(own).float(), **ulp)
    assert torch.count_nonzero(inc4[..., :d]) == 0
    f = ffn[:, : players * rows].view(batch, players, rows, width)
    torch.testing.assert_close(f[..., 2 * d: 3 * d].float(), _bf(oc * oc).float(), **ulp)
    torch.testing.assert_close(f[..., 3 * d: 4 * d].float(), _bf(oc * oe).float(), **ulp)
    assert torch.count_nonzero(ffn[:, players * rows:]) == 0
    assert torch.count_nonzero(f[..., : 2 * d]) == 0 and torch.count_nonzero(f[..., 4 * d:]) == 0


def test_scatter_rows_places_each_block():
    from pbg_b200._native import call, ptr, rows_ptr, stream

    g = torch.Generator(device=DEV).manual_seed(9)
    batch, group, length, d, width = 5, 37, 50, 256, 1024
    src = torch.randn((batch * group, d), generator=g, device=DEV).to(torch.bfloat16)
    dst = torch.zeros((batch * length, width), dtype=torch.bfloat16, device=DEV)
    call("pbg_scatter_rows_bf16", batch * group, d, group, ptr(src), rows_ptr(dst[:, 256: 256 + d]), length * width,
         width, stream(DEV))
    view = dst.view(batch, length, width)
    assert torch.equal(view[:, :group, 256: 256 + d], src.view(batch, group, d))
    assert torch.count_nonzero(view[:, group:]) == 0
    assert torch.count_nonzero(view[:, :, :256]) == 0 and torch.count_nonzero(view[:, :, 256 + d:]) == 0


@pytest.mark.parametrize("d,x_bf16,y_bf16", [(256, False, True), (128, False, True), (512, False, True),
                                             (200, False, True), (256, True, True), (256, False, False),
                                             (96, True, False)])
def test_layernorm_paths_match_torch(d, x_bf16, y_bf16):
    # the vectorised path (fp32 in, bf16 out, width a multiple of 128) and the general one
    from pbg_b200._native import call, ptr, stream

    g = torch.Generator(device=DEV).manual_seed(d)
    rows = 1000
    x = torch.randn((rows, d), generator=g, device=DEV) * 2 + 0.5
    if x_bf16:
        x = x.to(torch.bfloat16)
    gain = torch.rand(d, generator=g, device=DEV) + 0.5
    bias = torch.randn(d, generator=g, device=DEV)
    y = torch.empty((rows, d), dtype=torch.bfloat16 if y_bf16 else torch.float32, device=DEV)
    call("pbg_layernorm", rows, d, ptr(x), int(x_bf16), ptr(gain), ptr(bias), 1e-5, ptr(y), int(y_bf16), d,
         stream(DEV))
    want = F.layer_norm(x.float(), (d,), gain, bias, 1e-5)
    tol = 2e-2 if y_bf16 else 1e-5
    torch.testing.assert_close(y.float(), want, rtol=tol, atol=tol)
