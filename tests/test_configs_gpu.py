"""Parity at the shapes of BASELINE configs 2 and 3 (reduced batch so the float64 oracle finishes in
seconds): the 15M model's loss and every parameter gradient (dim 288, 6 layers, M 768, vocab 32000,
T 256, Zipf(1.1) tokens with BOS=1, prior 4, lam 0.95), and the 42M operator sweep (D 512, M 1024,
T up to 2048, lam in {0.9, 0.99, 0.999}, relu²-normalised addresses from a Gaussian K u + b with
eps = 1), forward and backward. Bars: 1e-2 relative with bf16 products, 1e-5 in fp32 mode; the
operator-level decay gradient at 3e-2 relative or the summation bound 1e-4 x sum |terms| (a sum of
B*T*T terms that cancel, see test_block_gpu.py)."""
import math

import numpy as np
import pytest
import torch

import unifiedlm_c_b200._lib as L
from oracle import memory as O
from unifiedlm_c_b200.kernel import unified_memory
from unifiedlm_c_b200.model import ModelArgs, UnifiedLM
from test_model_gpu import rel_errors

pytestmark = pytest.mark.gpu
TOL = {"bf16": 1e-2, "fp32": 1e-5}


def zipf_tokens(B, T, V, seed):
    """Zipf(s=1.1) ranks rejected to < V, rank -> id, BOS=1 first in every row."""
    rng = np.random.default_rng(seed)
    out = np.empty((B, T), dtype=np.int64)
    for b in range(B):
        row = []
        while len(row) < T - 1:
            draw = rng.zipf(1.1, size=4 * T)
            row.extend(int(x) - 1 for x in draw if x <= V)
        out[b, 0] = 1
        out[b, 1:] = row[:T - 1]
    return torch.from_numpy(out)


@pytest.mark.parametrize("precision", ["bf16", "fp32"])
def test_config2_model(precision):
    torch.manual_seed(0)
    args = ModelArgs(dim=288, n_layers=6, hidden_dim=768, vocab_size=32000, max_seq_len=256)
    model = UnifiedLM(args)
    with torch.no_grad():
        for layer in model.layers:
            layer.log_rate.fill_(math.log(-math.log(0.95)))
            layer.conv.weight.normal_(std=0.5)
            layer.key.bias.normal_(std=0.3)
            layer.val.weight.normal_(std=1.0 / math.sqrt(288))
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    model = model.cuda().train()
    tokens = zipf_tokens(2, 256, 32000, seed=1)
    errs = rel_errors(model, sd, tokens, precision)
    assert max(errs.values()) < TOL[precision], errs
    assert L.device_error() == 0


def config3_inputs(B, T, D, M, lam, seed):
    g = torch.Generator().manual_seed(seed)
    u = torch.randn(B, T, D, generator=g, dtype=torch.float64)
    K = torch.randn(M, D, generator=g, dtype=torch.float64) / math.sqrt(D)
    b = torch.randn(M, generator=g, dtype=torch.float64) * 0.5
    r = O.address(u, K, b, torch.tensor(0.0, dtype=torch.float64))  # eps = exp(0) = 1
    v = torch.randn(B, T, D, generator=g, dtype=torch.float64)
    lg = torch.tensor(math.log(lam), dtype=torch.float64)
    w = torch.full((M,), 4.0, dtype=torch.float64)
    dq = torch.randn(B, T, M, generator=g, dtype=torch.float64) * 0.1
    df = torch.randn(B, T, D, generator=g, dtype=torch.float64)
    return r, v, lg, w, dq, df


@pytest.mark.parametrize("T", [512, 1024, 2048])
@pytest.mark.parametrize("lam", [0.9, 0.99, 0.999])
def test_config3_operator_sweep(T, lam):
    B, D, M = 2, 512, 1024
    r, v, lg, w, dq, df = config3_inputs(B, T, D, M, lam, seed=T)
    leaves = [t.clone().requires_grad_(True) for t in (r, v, lg, w)]
    q_ref, f_ref = O.memory_dense(*leaves)
    ((q_ref * dq).sum() + (f_ref * df).sum()).backward()
    refs = [t.grad for t in leaves]
    dev = [t.float().cuda().requires_grad_(True) for t in (r, v, lg, w)]
    q, fast = unified_memory(dev[0], dev[1].to(torch.bfloat16), dev[2], dev[3], precision="bf16")
    ((q * dq.float().cuda()).sum() + (fast.float() * df.float().cuda()).sum()).backward()
    torch.cuda.synchronize()

    def rel(a, b_):
        return float((a.detach().double().cpu() - b_).norm() / b_.norm().clamp(min=1e-30))

    errs = {"q": rel(q, q_ref.detach()), "fast": rel(fast, f_ref.detach())}
    errs.update({n: rel(d.grad, rf) for n, d, rf in zip(("dr", "dv", "dg", "dw"), dev, refs)})
    # the decay gradient: relative bar or the summation bound over its (t - s) D dL/dD terms
    dg_rel = errs.pop("dg")
    g_terms = float(O.decay_grad_terms(r, v, lg, w, dq, df).abs().sum())
    dg_abs = abs(float(dev[2].grad) - float(refs[2]))
    assert dg_rel < 3e-2 or dg_abs < 1e-4 * g_terms, (dg_rel, dg_abs, g_terms)
    assert max(errs.values()) < TOL["bf16"], errs
    assert L.device_error() == 0


@pytest.mark.parametrize("T", [512, 1024])
def test_config3_operator_fp32(T):
    """Config 3 in the fp32 mode (1e-5 for every output, dg included) at lam 0.99; T = 2048 in fp32
    runs in the chunk-carry form (test_chunk_gpu.py)."""
    B, D, M = 1, 512, 1024
    r, v, lg, w, dq, df = config3_inputs(B, T, D, M, 0.99, seed=T + 7)
    leaves = [t.clone().requires_grad_(True) for t in (r, v, lg, w)]
    q_ref, f_ref = O.memory_dense(*leaves)
    ((q_ref * dq).sum() + (f_ref * df).sum()).backward()
    dev = [t.float().cuda().requires_grad_(True) for t in (r, v, lg, w)]
    q, fast = unified_memory(*dev, precision="fp32")
    ((q * dq.float().cuda()).sum() + (fast * df.float().cuda()).sum()).backward()
    torch.cuda.synchronize()

    def rel(a, b_):
        return float((a.detach().double().cpu() - b_).norm() / b_.norm().clamp(min=1e-30))

    errs = {"q": rel(q, q_ref.detach()), "fast": rel(fast, f_ref.detach())}
    errs.update({n: rel(d.grad, lf.grad) for n, d, lf in zip(("dr", "dv", "dg", "dw"), dev, leaves)})
    assert max(errs.values()) < TOL["fp32"], errs
    assert L.device_error() == 0
