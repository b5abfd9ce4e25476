"""UnifiedBlock's address -> fast-memory span as one differentiable call (model.py:79-83).

    r = normalize(relu(conv(h) K^T + b)^2),   (q, fast) = unified_memory(r, v, g, w)

`addressed_memory(h, conv_weight, key_weight, key_bias, eps, v, g, w, precision)` returns the same
(q, fast) as `unified_memory(address(h, ...), v, g, w)` with the same gradients, but the addresses
never exist in normalised form: the key product leaves z = relu(.)^2 and one row sum per column
block (the epilogue), a small kernel forms den = eps + sum, and every reader of r (the forward
and backward scans, the address backward) applies 1 / den to the rows it loads. That removes a
read-modify-write pass over the (B,T,M) fp32 addresses per block.

The pair is the `torch.library` ops `ulm::addressed_memory_fwd` / `ulm::addressed_memory_bwd`
(libulm_b200.so: ulm_address_fwd with normalize = 0, ulm_memory_fwd / ulm_memory_bwd with den,
ulm_address_bwd with normalized = 0).
"""
from typing import Optional

import torch

from .kernel import PRECISION, memory_bwd_raw, memory_fwd_fake, memory_fwd_raw
from .prologue import address_bwd_fake, address_bwd_raw, address_fwd_fake, address_fwd_raw

_OUT = tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
             torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]


@torch.library.custom_op("ulm::addressed_memory_fwd", mutates_args=())
def addressed_memory_fwd(h: torch.Tensor, conv_w: torch.Tensor, key_w: torch.Tensor, key_b: torch.Tensor,
                         eps: torch.Tensor, v: torch.Tensor, g: torch.Tensor, w: torch.Tensor, precision: int) -> _OUT:
    """Returns (q, fast, z, den, u_op, kw_op, c, qop, kop, vop, P); all but the first two are saved
    for the backward."""
    z, den, u_op, kw = address_fwd_raw(h, conv_w, key_w, key_b, eps, precision, normalize=False)
    q, fast, c, qop, kop, vop, P = memory_fwd_raw(z, den, v, g, w, precision)
    return q, fast, z, den, u_op, kw, c, qop, kop, vop, P


@addressed_memory_fwd.register_fake
def _fwd_fake(h, conv_w, key_w, key_b, eps, v, g, w, precision):
    z, den, u_op, kw = address_fwd_fake(h, key_w, precision)
    q, fast, c, qop, kop, vop, P = memory_fwd_fake(z, v, precision)
    return q, fast, z, den, u_op, kw, c, qop, kop, vop, P


@torch.library.custom_op("ulm::addressed_memory_bwd", mutates_args=())
def addressed_memory_bwd(dq_out: Optional[torch.Tensor], dfast: torch.Tensor, h: torch.Tensor, conv_w: torch.Tensor,
                         g: torch.Tensor, w: torch.Tensor, q: torch.Tensor, z: torch.Tensor, den: torch.Tensor,
                         u_op: torch.Tensor, kw: torch.Tensor, c: torch.Tensor, qop: torch.Tensor, kop: torch.Tensor,
                         vop: torch.Tensor, P: torch.Tensor, precision: int
                         ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                                    torch.Tensor, torch.Tensor, torch.Tensor]:
    """Returns (dh fp32, dconv_w, dkey_w, dkey_b, deps, dv, dg, dw)."""
    dr, dv, dg, dw = memory_bwd_raw(dq_out, dfast, z, den, g, w, q, c, qop, kop, vop, P, precision)
    dh, dconv, dkw, dkb, deps = address_bwd_raw(dr, z, den, u_op, kw, h, conv_w, precision, normalized=False)
    return dh, dconv, dkw, dkb, deps, dv, dg, dw


@addressed_memory_bwd.register_fake
def _bwd_fake(dq_out, dfast, h, conv_w, g, w, q, z, den, u_op, kw, c, qop, kop, vop, P, precision):
    dh, dconv, dkw, dkb, deps = address_bwd_fake(h, z, conv_w)
    M = z.shape[-1]
    return (dh, dconv, dkw, dkb, deps, dfast.new_empty(dfast.shape), z.new_empty((), dtype=torch.float32),
            z.new_empty(M, dtype=torch.float32))


def _setup(ctx, inputs, output):
    h, conv_w, key_w, key_b, eps, v, g, w, precision = inputs
    q, fast, z, den, u_op, kw, c, qop, kop, vop, P = output
    ctx.save_for_backward(h, conv_w, g, w, q, z, den, u_op, kw, c, qop, kop, vop, P)
    ctx.precision = precision
    ctx.dtypes = (h.dtype, conv_w.dtype, key_w.dtype, key_b.dtype, eps.dtype, v.dtype)
    ctx.v_dim = v.shape[-1]
    ctx.g_shape = g.shape
    ctx.mark_non_differentiable(z, den, u_op, kw, c, qop, kop, vop, P)


def _backward(ctx, dq_out, dfast, *unused):
    h, conv_w, g, w, q, z, den, u_op, kw, c, qop, kop, vop, P = ctx.saved_tensors
    hd, cd, kd, bd, ed, vd = ctx.dtypes
    if dfast is None:
        dfast = torch.zeros(q.shape[0], q.shape[1], ctx.v_dim, device=q.device, dtype=vd)
    dh, dconv, dkw, dkb, deps, dv, dg, dw = addressed_memory_bwd(
        None if dq_out is None else dq_out.float().contiguous(), dfast.contiguous(), h, conv_w, g, w, q, z, den,
        u_op, kw, c, qop, kop, vop, P, ctx.precision)
    return (dh.to(hd), dconv.to(cd), dkw.to(kd), dkb.to(bd), deps.to(ed), dv.to(vd), dg.reshape(ctx.g_shape), dw,
            None)


torch.library.register_autograd("ulm::addressed_memory_fwd", _backward, setup_context=_setup)


def addressed_memory(h, conv_weight, key_weight, key_bias, eps, v, g, w, precision="bf16"):
    """(q fp32 (B,T,M), fast (B,T,D) in v's dtype) = unified_memory(address(h, conv_weight,
    key_weight, key_bias, eps), v, g, w): h (B,T,D), conv_weight (D,1,K), key_weight (M,D),
    key_bias (M,), eps 0-d, v (B,T,D), g 0-d log decay, w (M,)."""
    for t in (h, v, g, w):
        if not t.is_cuda:
            raise RuntimeError("addressed_memory runs on CUDA tensors only (no CPU path)")
    out_dtype = v.dtype
    hh = h if h.dtype in (torch.float32, torch.bfloat16) else h.float()
    vv = v if v.dtype in (torch.float32, torch.bfloat16) else v.float()
    q, fast, *_ = torch.ops.ulm.addressed_memory_fwd(hh.contiguous(), conv_weight, key_weight, key_bias,
                                                     eps.float().reshape(()), vv.contiguous(), g.float().reshape(()),
                                                     w.float().contiguous(), PRECISION[precision])
    return q, fast.to(out_dtype)
