"""The chunk-carry decomposition of the fast read, checked in float64 on the CPU.

The library's long-sequence form splits the sequence into chunks of C positions: a carry product
walks the chunks keeping the (M x D) state in the tensor cores' accumulator and writes one state
per chunk boundary, the inter-chunk read is a product against that state with a per-row decay,
and the intra-chunk part is the whole-sequence machinery on C-long pieces. The backward needs one
more carry (the reverse state of q dO^T) and three position-weighted dot products for d/dg.

This file restates that decomposition step by step, exactly as the kernels split the work, and
checks it against the oracle's float64 autograd of the reference's function (kernel.py:1-15,
test_all.py:54-61). It runs no GPU code.
"""
import pytest
import torch

from oracle import memory as O


def chunk_carry_forward(q, k, v, g, C):
    """(fast, H): H[:, n] = state entering chunk n (H[:, 0] = 0), H_end = state after the last."""
    B, T, M = q.shape
    D = v.shape[-1]
    NT = T // C
    lam = torch.exp(g)
    i = torch.arange(T) % C
    vhat = v * lam ** (C - 1 - i)[None, :, None]          # the carry's B operand, per-chunk decay
    H = torch.zeros(B, NT + 1, M, D, dtype=q.dtype)
    for n in range(NT):                                   # carry product: acc = lam^C acc + k^T vhat
        sl = slice(n * C, (n + 1) * C)
        H[:, n + 1] = lam ** C * H[:, n] + k[:, sl].transpose(1, 2) @ vhat[:, sl]
    fast = torch.empty(B, T, D, dtype=q.dtype)
    tt = torch.arange(C)
    Dc = (tt[:, None] >= tt[None, :]).to(q.dtype) * lam ** (tt[:, None] - tt[None, :]).clamp(min=0)
    for n in range(NT):
        sl = slice(n * C, (n + 1) * C)
        F = lam ** (tt + 1)[None, :, None] * (q[:, sl] @ H[:, n])        # inter read, row decay
        P = Dc * (q[:, sl] @ k[:, sl].transpose(1, 2))                     # intra scores
        fast[:, sl] = F + P @ v[:, sl]
    return fast, H


def chunk_carry_backward(q, k, v, g, dO, H, C):
    """(dq_fast, dk_fast, dv, dg_fast): the fast read's gradients by the chunk-carry products."""
    B, T, M = q.shape
    NT = T // C
    lam = torch.exp(g)
    tt = torch.arange(C)
    lag = (tt[:, None] - tt[None, :]).clamp(min=0).to(q.dtype)
    Dc = (tt[:, None] >= tt[None, :]).to(q.dtype) * lam ** lag
    i = torch.arange(T) % C
    dOhat = dO * lam ** i[None, :, None]                  # the reverse carry's B operand
    R = torch.zeros(B, NT, M, dO.shape[-1], dtype=q.dtype)  # R[:, n]: state from chunks > n
    for n in range(NT - 1, 0, -1):
        sl = slice(n * C, (n + 1) * C)
        R[:, n - 1] = lam ** C * R[:, n] + q[:, sl].transpose(1, 2) @ dOhat[:, sl]
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    dg = torch.zeros((), dtype=q.dtype)
    for n in range(NT):
        sl = slice(n * C, (n + 1) * C)
        qn, kn, vn, don = q[:, sl], k[:, sl], v[:, sl], dO[:, sl]
        P = Dc * (qn @ kn.transpose(1, 2))
        acc = don @ vn.transpose(1, 2)                    # dS before the decay
        dS = Dc * acc
        dg = dg + (lag * P * acc).sum()                   # intra share (score-gradient epilogue)
        dq_inter = lam ** (tt + 1)[None, :, None] * (don @ H[:, n].transpose(1, 2))
        dk_inter = lam ** (C - tt)[None, :, None] * (vn @ R[:, n].transpose(1, 2))
        dv_inter = lam ** (C - tt)[None, :, None] * (kn @ R[:, n])
        dg = dg + ((tt + 1)[None, :, None] * qn * dq_inter).sum()          # term A
        dg = dg + ((C - 1 - tt)[None, :, None] * kn * dk_inter).sum()      # term C
        if n < NT - 1:
            dg = dg + C * lam ** (C + 1) * (R[:, n] * H[:, n]).sum()       # term B
        dq[:, sl] = dS @ kn + dq_inter
        dk[:, sl] = dS.transpose(1, 2) @ qn + dk_inter
        dv[:, sl] = P.transpose(1, 2) @ don + dv_inter
    return dq, dk, dv, dg


def fast_read_dense(q, k, v, g):
    T = q.shape[1]
    return ((q @ k.transpose(1, 2)) * O.decay_matrix(T, g)) @ v


@pytest.mark.parametrize("B,T,M,D,C,lam", [(2, 256, 24, 16, 64, 0.95), (1, 192, 40, 8, 64, 0.9),
                                           (2, 512, 16, 12, 128, 0.999), (1, 64, 8, 8, 64, 0.8)])
def test_chunk_carry_matches_dense_fast_read(B, T, M, D, C, lam):
    torch.manual_seed(0)
    q = torch.rand(B, T, M, dtype=torch.float64)
    k = torch.rand(B, T, M, dtype=torch.float64)
    v = torch.randn(B, T, D, dtype=torch.float64)
    dO = torch.randn(B, T, D, dtype=torch.float64)
    g = torch.tensor(lam, dtype=torch.float64).log()
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v, g)]
    ref = fast_read_dense(*leaves)
    (ref * dO).sum().backward()

    fast, H = chunk_carry_forward(q, k, v, g, C)
    assert torch.allclose(fast, ref.detach(), rtol=1e-10, atol=1e-10)
    # the end state is the decode state's fast part: S = sum_s lam^(T-1-s) k_s v_s^T
    w_end = torch.exp(g) ** (T - 1 - torch.arange(T, dtype=torch.float64))
    S_end = k.transpose(1, 2) @ (v * w_end[None, :, None])
    assert torch.allclose(H[:, -1], S_end, rtol=1e-10, atol=1e-10)

    dq, dk, dv, dg = chunk_carry_backward(q, k, v, g, dO, H[:, :-1], C)
    for got, leaf in zip((dq, dk, dv), leaves[:3]):
        assert torch.allclose(got, leaf.grad, rtol=1e-9, atol=1e-9)
    assert abs(float(dg) - float(leaves[3].grad)) <= 1e-9 * max(1.0, abs(float(leaves[3].grad)))
