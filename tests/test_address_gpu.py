"""The fused addressing prologue (conv -> key GEMM -> relu^2 -> normalise) and its backward against
the float64 oracle (oracle.memory.prologue, model.py:61-62, 70-72, 79). Bars as elsewhere: 1e-2
relative with bf16 products, 1e-5 in fp32 mode. The largest shape (4096 rows) runs the key-weight
gradient as a split-K product."""
import math

import pytest
import torch

import unifiedlm_c_b200._lib as L
from oracle import memory as O
from unifiedlm_c_b200.prologue import address

pytestmark = pytest.mark.gpu
TOL = {"bf16": 1e-2, "fp32": 1e-5}


def rel(a, b):
    return float((a.detach().double().cpu() - b).norm() / b.norm().clamp(min=1e-30))


@pytest.mark.parametrize("precision", ["bf16", "fp32"])
@pytest.mark.parametrize("shape", [(2, 200, 64, 140), (1, 40, 32, 48), (2, 256, 768, 2048), (4, 1024, 768, 2048)],
                         ids=lambda s: "x".join(map(str, s)))
def test_address_matches_oracle(precision, shape):
    B, T, D, M = shape
    g = torch.Generator().manual_seed(0)
    h = torch.randn(B, T, D, generator=g, dtype=torch.float64)
    conv = torch.randn(D, 1, 4, generator=g, dtype=torch.float64) * 0.5
    kw = torch.randn(M, D, generator=g, dtype=torch.float64) / math.sqrt(D)
    kb = torch.randn(M, generator=g, dtype=torch.float64) * 0.5
    log_eps = torch.tensor(0.3, dtype=torch.float64)
    dr = torch.randn(B, T, M, generator=g, dtype=torch.float64)

    leaves = [t.clone().requires_grad_(True) for t in (h, conv, kw, kb, log_eps)]
    r_ref = O.prologue(*leaves)
    (r_ref * dr).sum().backward()
    refs = [t.grad for t in leaves]

    dev = [t.float().cuda().requires_grad_(True) for t in (h, conv, kw, kb, log_eps)]
    eps = dev[4].clamp(-10, 10).exp()
    r = address(dev[0], dev[1], dev[2], dev[3], eps, precision=precision)
    (r * dr.float().cuda()).sum().backward()
    torch.cuda.synchronize()
    errs = {"r": rel(r, r_ref.detach())}
    errs.update({n: rel(d.grad, rf) for n, d, rf in zip(("dh", "dconv", "dkey_w", "dkey_b", "dlog_eps"), dev, refs)})
    assert max(errs.values()) < TOL[precision], errs
    assert L.device_error() == 0
