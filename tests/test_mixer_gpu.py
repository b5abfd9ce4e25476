"""block_mixer: UnifiedBlock.forward's mixing span with the `mu` combine fused into the fast read's
tensor-core tiles (y = x + mu(q w) + fast, model.py:79-85) and its gradient fused into the dq
product, against the float64 oracle composition (oracle.memory.prologue -> memory_dense -> combine),
with the gradients of all ten inputs. Bars as in test_block_gpu.py: 1e-2 relative with bf16
products and 1e-5 in fp32 mode for every tensor, the two cancelling scalars (dg, dlog_eps) at the
relative bar or the summation bound. The prior-mass gradient dw is the sum of two nearly opposite
parts (the combine's direct q . (dy mu) and the slot statistics' -(dy mu) w . q / c, equal where
n << w: d(q w)/dw = r n / (w + n)^2), so its bar is relative to the norm of |part 1| + |part 2|
(the summation bound with the same 1e-2 / 1e-5 factor). The model-level tests (test_model_gpu.py)
run this op too."""
import math

import pytest
import torch

import unifiedlm_c_b200._lib as L
from oracle import memory as O
from unifiedlm_c_b200.block import block_mixer

pytestmark = pytest.mark.gpu
TOL = {"bf16": 1e-2, "fp32": 1e-5}
DG_TOL = {"bf16": 3e-2, "fp32": 1e-5}
SUM_TOL = {"bf16": 1e-4, "fp32": 5e-8}
NAMES = ("dx", "dh", "dconv", "dkey_w", "dkey_b", "dlog_eps", "dv", "dg", "dw", "dmu")


def rel(a, b):
    b = b.double().cpu()
    return float((a.detach().double().cpu() - b).norm() / b.norm().clamp(min=1e-30))


def make(B, T, D, M, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, D, generator=g, dtype=torch.float64)
    h = torch.randn(B, T, D, generator=g, dtype=torch.float64)
    conv = torch.randn(D, 1, 4, generator=g, dtype=torch.float64) * 0.5
    kw = torch.randn(M, D, generator=g, dtype=torch.float64) / math.sqrt(D)
    kb = torch.randn(M, generator=g, dtype=torch.float64) * 0.5
    log_eps = torch.tensor(0.3, dtype=torch.float64)
    v = torch.randn(B, T, D, generator=g, dtype=torch.float64)
    lg = torch.tensor(math.log(0.97), dtype=torch.float64)
    w = torch.exp(torch.randn(M, generator=g, dtype=torch.float64))
    mu = torch.randn(D, M, generator=g, dtype=torch.float64) * 0.3
    dy = torch.randn(B, T, D, generator=g, dtype=torch.float64)
    return (x, h, conv, kw, kb, log_eps, v, lg, w, mu), dy


def oracle_mixer(x, h, conv, kw, kb, log_eps, v, lg, w, mu):
    r = O.prologue(h, conv, kw, kb, log_eps)
    r.retain_grad()
    q, fast = O.memory_dense(r, v, lg, w)
    return x + (q * w) @ mu.t() + fast, r


@pytest.mark.parametrize("precision", ["bf16", "fp32"])
@pytest.mark.parametrize("shape", [(1, 40, 32, 48), (2, 200, 64, 140), (2, 256, 768, 2048), (1, 1500, 64, 96),
                                   (1, 2500, 32, 40)], ids=lambda s: "x".join(map(str, s)))
def test_mixer_matches_oracle(precision, shape):
    inputs, dy = make(*shape)
    leaves = [t.clone().requires_grad_(True) for t in inputs]
    y_ref, r = oracle_mixer(*leaves)
    (y_ref * dy).sum().backward()
    refs = [t.grad for t in leaves]
    x, h, conv, kw, kb, log_eps, v, lg, w, mu = leaves
    eps_ref = O.null_mass(log_eps).detach()
    den_ref = eps_ref / (1.0 - r.detach().sum(-1, keepdim=True))
    eps_terms = float((eps_ref * r.grad * r.detach() / den_ref).abs().sum())
    # the decay's terms: the combine does not depend on g, so dL/dfast = dy and dL/dq = (dy mu) w
    dq = (dy @ mu.detach()) * w.detach()
    g_terms = float(O.decay_grad_terms(r, v, lg, w, dq, dy).abs().sum())
    # dw's two parts: the combine's direct share and the rest (through c = w + n)
    q_ref, _ = O.memory_dense(r.detach(), v.detach(), lg.detach(), w.detach())
    dw_comb = (q_ref * (dy @ mu.detach())).sum((0, 1))
    dw_scale = float((dw_comb.abs() + (w.grad - dw_comb).abs()).norm())

    dev = [t.float().cuda().requires_grad_(True) for t in inputs]
    x, h, conv, kw, kb, log_eps, v, lg, w, mu = dev
    y = block_mixer(x, h, conv, kw, kb, log_eps.clamp(-10, 10).exp(), v, lg, w, mu, precision=precision)
    (y * dy.float().cuda()).sum().backward()
    torch.cuda.synchronize()
    errs = {"y": rel(y, y_ref.detach())}
    errs.update({n: rel(d.grad, rf) for n, d, rf in zip(NAMES, dev, refs)})
    for name, idx, terms in (("dg", 7, g_terms), ("dlog_eps", 5, eps_terms)):
        rel_err = errs.pop(name)
        abs_err = abs(float(dev[idx].grad) - float(refs[idx]))
        assert rel_err < DG_TOL[precision] or abs_err < SUM_TOL[precision] * terms, (name, rel_err, abs_err, terms)
    dw_err = float((dev[8].grad.double().cpu() - refs[8]).norm())
    errs["dw"] = min(errs["dw"], dw_err / dw_scale)
    assert max(errs.values()) < TOL[precision], errs
    assert L.device_error() == 0


def test_mixer_bf16_activations_and_split_grad():
    """bf16 x, h and v (autocast-style activations) at a shape whose dmu product runs split-K."""
    inputs, dy = make(4, 1024, 768, 2048, seed=2)
    x64, h64, conv, kw, kb, log_eps, v64, lg, w, mu = inputs
    xb, hb, vb = (t.to(torch.bfloat16) for t in (x64, h64, v64))
    leaves = [t.clone().requires_grad_(True) for t in (xb.double(), hb.double(), conv, kw, kb, log_eps, vb.double(),
                                                        lg, w, mu)]
    y_ref, _ = oracle_mixer(*leaves)
    (y_ref * dy).sum().backward()
    dev = [t.cuda().requires_grad_(True) for t in (xb, hb)] + \
          [t.float().cuda().requires_grad_(True) for t in (conv, kw, kb, log_eps)] + \
          [vb.cuda().requires_grad_(True)] + [t.float().cuda().requires_grad_(True) for t in (lg, w, mu)]
    x, h, conv_, kw_, kb_, le, v, lg_, w_, mu_ = dev
    y = block_mixer(x, h, conv_, kw_, kb_, le.clamp(-10, 10).exp(), v, lg_, w_, mu_)
    assert y.dtype == torch.bfloat16
    (y.float() * dy.float().cuda()).sum().backward()
    torch.cuda.synchronize()
    errs = {"y": rel(y, y_ref.detach())}
    for n, d, lf in zip(NAMES, dev, leaves):
        if n not in ("dg", "dlog_eps"):
            errs[n] = rel(d.grad.float(), lf.grad)
    assert max(errs.values()) < 1e-2, errs
    assert L.device_error() == 0
