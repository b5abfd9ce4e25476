"""addressed_memory (the prologue and the fast memory with the addresses left unnormalised between
them) against the float64 oracle composition oracle.memory.prologue -> memory_dense
(model.py:79-83, kernel.py:199-238), with the gradients of all eight inputs. Bars as elsewhere:
1e-2 relative with bf16 products, 1e-5 in fp32 mode, for every tensor output and gradient.

The two scalar gradients are sums that cancel: dg = sum over (b, t, s) of (t - s) D[t, s]
dL/dD[t, s] (oracle.memory.decay_grad_terms) and dlog_eps = -eps sum over (b, t, m) of
dr r / den. On these inputs the sums are 1/30 to 1/5000 of the absolute sums of their terms, so
the operand rounding (2^-9 relative in bf16, 2^-24 in fp32) is amplified by that factor. Each
scalar passes at the relative bar (3e-2 for bf16 as in test_memory_gpu.py, 1e-5 for fp32) or at
the summation error bound: |error| < SUM_TOL * (absolute sum of the oracle's terms).

The shapes reach every scan variant: the TMA scans with the recompute backward (T <= 1024), the
TMA scans with a saved c (T <= 2048) and the two-pass scans (longer T)."""
import math

import pytest
import torch

import unifiedlm_c_b200._lib as L
from oracle import memory as O
from unifiedlm_c_b200.block import addressed_memory
from unifiedlm_c_b200.prologue import address_fwd_raw

pytestmark = pytest.mark.gpu
TOL = {"bf16": 1e-2, "fp32": 1e-5}
DG_TOL = {"bf16": 3e-2, "fp32": 1e-5}
SUM_TOL = {"bf16": 1e-4, "fp32": 5e-8}
NAMES = ("dh", "dconv", "dkey_w", "dkey_b", "dlog_eps", "dv", "dg", "dw")


def rel(a, b):
    b = b.double().cpu()
    return float((a.detach().double().cpu() - b).norm() / b.norm().clamp(min=1e-30))


def make(B, T, D, M, seed=0):
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(B, T, D, generator=g, dtype=torch.float64)
    conv = torch.randn(D, 1, 4, generator=g, dtype=torch.float64) * 0.5
    kw = torch.randn(M, D, generator=g, dtype=torch.float64) / math.sqrt(D)
    kb = torch.randn(M, generator=g, dtype=torch.float64) * 0.5
    log_eps = torch.tensor(0.3, dtype=torch.float64)
    v = torch.randn(B, T, D, generator=g, dtype=torch.float64)
    lg = torch.tensor(math.log(0.97), dtype=torch.float64)
    w = torch.exp(torch.randn(M, generator=g, dtype=torch.float64))
    dq = torch.randn(B, T, M, generator=g, dtype=torch.float64)
    df = torch.randn(B, T, D, generator=g, dtype=torch.float64)
    return (h, conv, kw, kb, log_eps, v, lg, w), dq, df


@pytest.mark.parametrize("precision", ["bf16", "fp32"])
@pytest.mark.parametrize("shape", [(1, 40, 32, 48), (2, 200, 64, 140), (2, 256, 768, 2048), (1, 1500, 64, 96),
                                   (1, 2500, 32, 40)], ids=lambda s: "x".join(map(str, s)))
def test_addressed_memory_matches_oracle(precision, shape):
    inputs, dq, df = make(*shape)
    leaves = [t.clone().requires_grad_(True) for t in inputs]
    h, conv, kw, kb, log_eps, v, lg, w = leaves
    r = O.prologue(h, conv, kw, kb, log_eps)
    r.retain_grad()
    q_ref, f_ref = O.memory_dense(r, v, lg, w)
    ((q_ref * dq).sum() + (f_ref * df).sum()).backward()
    refs = [t.grad for t in leaves]
    # absolute sum of the terms of dlog_eps: eps * dr r / den, den = eps + sum z = eps / (1 - sum r)
    eps_ref = O.null_mass(log_eps).detach()
    den_ref = eps_ref / (1.0 - r.detach().sum(-1, keepdim=True))
    eps_terms = float((eps_ref * r.grad * r.detach() / den_ref).abs().sum())
    g_terms = float(O.decay_grad_terms(r, v, lg, w, dq, df).abs().sum())

    dev = [t.float().cuda().requires_grad_(True) for t in inputs]
    h, conv, kw, kb, log_eps, v, lg, w = dev
    eps = log_eps.clamp(-10, 10).exp()
    q, fast = addressed_memory(h, conv, kw, kb, eps, v, lg, w, precision=precision)
    ((q * dq.float().cuda()).sum() + (fast * df.float().cuda()).sum()).backward()
    torch.cuda.synchronize()
    errs = {"q": rel(q, q_ref.detach()), "fast": rel(fast, f_ref.detach())}
    errs.update({n: rel(d.grad, rf) for n, d, rf in zip(NAMES, dev, refs)})
    for name, idx, terms in (("dg", 6, g_terms), ("dlog_eps", 4, eps_terms)):
        rel_err = errs.pop(name)
        abs_err = abs(float(dev[idx].grad) - float(refs[idx]))
        assert rel_err < DG_TOL[precision] or abs_err < SUM_TOL[precision] * terms, (name, rel_err, abs_err, terms)
    assert max(errs.values()) < TOL[precision], errs
    assert L.device_error() == 0


@pytest.mark.parametrize("precision", ["bf16", "fp32"])
def test_unnormalised_form_matches_normalised(precision):
    """The key product's row sums (epilogue partials) give the same den as the normalising pass,
    and z / den the same addresses."""
    (h, conv, kw, kb, log_eps, *_), _, _ = make(2, 300, 256, 520, seed=1)
    prec = L.ULM_PREC_FP32 if precision == "fp32" else L.ULM_PREC_BF16
    args = (h.float().cuda(), conv.float().cuda(), kw.float().cuda(), kb.float().cuda(),
            log_eps.exp().float().cuda().reshape(()), prec)
    r, den, _, _ = address_fwd_raw(*args, normalize=True)
    z, den_z, _, _ = address_fwd_raw(*args, normalize=False)
    torch.cuda.synchronize()
    assert rel(den_z, den) < 1e-6
    assert rel(z / den_z.reshape(2, 300, 1), r) < 1e-6
    assert L.device_error() == 0
