"""RMSNorm and the val Linear as library ops (model.py:31-42, 65, 81) against float64 torch.

rms_norm: y = round_x(x / sqrt(mean(x^2) + eps)) * weight and its gradients (dx, dweight), fp32 and
bf16 inputs; within 1e-5 relative for fp32 inputs (fp32 arithmetic) and 1e-2 for bf16 inputs.
linear: y = x W^T with bf16 tensor-core products (1e-2) or fp32 products (1e-5), dx and dW.
Edge cases: a single row, rows not a multiple of the CTA's eight, widths not a multiple of 32.
block_scalars: the block's learned scalars (model.py:72, 75, 84) and their gradients, bit-identical
to autograd of the reference's fp32 expressions, on and beyond the clamp bounds.
"""
import pytest
import torch

import unifiedlm_c_b200._lib as L
from unifiedlm_c_b200.block import block_scalars
from unifiedlm_c_b200.norm import linear, rms_norm

pytestmark = pytest.mark.gpu


def rel(a, b):
    b = b.double().cpu()
    return float((a.detach().double().cpu() - b).norm() / b.norm().clamp(min=1e-30))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(1, 1, 768), (3, 37, 288), (16, 1024, 768), (2, 5, 50)],
                         ids=lambda s: "x".join(map(str, s)))
def test_rms_norm_matches_reference(shape, dtype):
    g = torch.Generator().manual_seed(sum(shape))
    x = (torch.randn(*shape, generator=g) * 3).to(dtype)
    w = 1 + 0.1 * torch.randn(shape[-1], generator=g)
    dy = torch.randn(*shape, generator=g)
    xr = x.double().requires_grad_(True)
    wr = w.double().requires_grad_(True)
    xh = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-5)
    if dtype == torch.bfloat16:
        xh = xh + (xh.detach().to(torch.bfloat16).double() - xh.detach())  # the type_as rounding
    yr = xh * wr
    (yr * dy.double()).sum().backward()
    xd = x.cuda().requires_grad_(True)
    wd = w.cuda().requires_grad_(True)
    y = rms_norm(xd, wd, 1e-5)
    assert y.dtype == torch.float32
    (y * dy.cuda()).sum().backward()
    torch.cuda.synchronize()
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    errs = {"y": rel(y, yr), "dx": rel(xd.grad.float(), xr.grad), "dw": rel(wd.grad, wr.grad)}
    assert max(errs.values()) < tol, errs
    assert xd.grad.dtype == dtype
    assert L.device_error() == 0


@pytest.mark.parametrize("precision", ["bf16", "fp32"])
@pytest.mark.parametrize("shape", [(16, 1024, 768, 768), (2, 200, 64, 64), (1, 3, 40, 24), (4, 512, 288, 288)],
                         ids=lambda s: "x".join(map(str, s)))
def test_linear_matches_reference(shape, precision):
    B, T, K, N = shape
    g = torch.Generator().manual_seed(B * T + K)
    x = torch.randn(B, T, K, generator=g)
    W = torch.randn(N, K, generator=g) / K ** 0.5
    dy = torch.randn(B, T, N, generator=g)
    xr, Wr = x.double().requires_grad_(True), W.double().requires_grad_(True)
    yr = xr @ Wr.t()
    (yr * dy.double()).sum().backward()
    xd, Wd = x.cuda().requires_grad_(True), W.cuda().requires_grad_(True)
    y = linear(xd, Wd, precision=precision)
    (y * dy.cuda()).sum().backward()
    torch.cuda.synchronize()
    tol = 1e-2 if precision == "bf16" else 1e-5
    errs = {"y": rel(y, yr), "dx": rel(xd.grad, xr.grad), "dW": rel(Wd.grad, Wr.grad)}
    assert max(errs.values()) < tol, errs
    assert L.device_error() == 0


@pytest.mark.parametrize("log_eps", [-11.0, -10.0, 0.3, 10.0, 10.5])
@pytest.mark.parametrize("M", [1, 2048, 3000])
def test_block_scalars_match_autograd(M, log_eps):
    """w = exp(clamp(log_w, -7, 12)), eps = exp(clamp(log_eps, -10, 10)), g = -exp(log_rate) and
    their gradients equal, bit for bit, PyTorch's evaluation of the same fp32 expressions (clamp
    passes the gradient on its bounds and blocks it beyond them)."""
    gen = torch.Generator().manual_seed(M)
    lw = torch.randn(M, generator=gen) * 6 + 2
    lw[: min(M, 4)] = torch.tensor([-7.0, 12.0, -7.5, 12.5])[: min(M, 4)]
    le = torch.tensor(log_eps)
    lr = torch.tensor(-8.3)
    dw = torch.randn(M, generator=gen)
    deps, dg = torch.randn((), generator=gen), torch.randn((), generator=gen)
    outs = []
    for fused in (True, False):
        p = [t.clone().cuda().requires_grad_(True) for t in (lw, le, lr)]
        if fused:
            w, eps, g = block_scalars(*p)
        else:
            w, eps, g = p[0].clamp(-7.0, 12.0).exp(), p[1].clamp(-10.0, 10.0).exp(), -p[2].exp()
        ((w * dw.cuda()).sum() + eps * deps.cuda() + g * dg.cuda()).backward()
        outs.append([t.detach().cpu() for t in (w, eps, g)] + [t.grad.cpu() for t in p])
    for a, b in zip(*outs):
        assert a.shape == b.shape and a.dtype == b.dtype
        assert torch.equal(a, b), (a, b)
    assert L.device_error() == 0
