"""UnifiedBlock's address -> fast-memory span as one differentiable call (model.py:79-83).

    r = normalize(relu(conv(h) K^T + b)^2),   (q, fast) = unified_memory(r, v, g, w)

`addressed_memory(h, conv_weight, key_weight, key_bias, eps, v, g, w, precision)` returns the same
(q, fast) as `unified_memory(address(h, ...), v, g, w)` with the same gradients, but the addresses
never exist in normalised form: the key product leaves z = relu(.)^2 and one row sum per column
block (the epilogue), a small kernel forms den = eps + sum, and every reader of r (the forward
and backward scans, the address backward) applies 1 / den to the rows it loads. That removes a
read-modify-write pass over the (B,T,M) fp32 addresses per block.

The pair is the `torch.library` ops `ulm::addressed_memory_fwd` / `ulm::addressed_memory_bwd`
(libulm_b200.so: ulm_address_fwd with normalize = 0 and ulm_memory_fwd with den; the backward is
one call, ulm_addressed_memory_bwd = ulm_memory_bwd with den followed by ulm_address_bwd with
normalized = 0).
"""
from typing import Optional

import torch

from . import _lib as L
from .kernel import (PRECISION, _op_dtype, _require_cuda, bwd_work_buffer, combine_fwd_fake, combine_fwd_raw,
                     memory_fwd_fake, memory_fwd_raw, operand_copy, operand_ld, operand_or_input, unaliased)
from .prologue import address_bwd_fake, address_fwd_fake, address_fwd_raw
from .norm import (_linear_fwd_fake, _rms_norm_fwd_fake, linear_bwd_raw, linear_fwd_raw, rms_norm_bwd_raw,
                   rms_norm_fwd_raw)

_OUT = tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
             torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]


@torch.library.custom_op("ulm::addressed_memory_fwd", mutates_args=())
def addressed_memory_fwd(h: torch.Tensor, conv_w: torch.Tensor, key_w: torch.Tensor, key_b: torch.Tensor,
                         eps: torch.Tensor, v: torch.Tensor, g: torch.Tensor, w: torch.Tensor, precision: int) -> _OUT:
    """Returns (q, fast, z, den, u_op, kw_op, c, qop, kop, vop, P); all but the first two are saved
    for the backward."""
    z, den, u_op, kw = address_fwd_raw(h, conv_w, key_w, key_b, eps, precision, normalize=False)
    q, fast, c, qop, kop, vop, P = memory_fwd_raw(z, den, v, g, w, precision)
    return q, fast, z, den, u_op, kw, c, qop, kop, unaliased(vop, v), P


@addressed_memory_fwd.register_fake
def _fwd_fake(h, conv_w, key_w, key_b, eps, v, g, w, precision):
    z, den, u_op, kw = address_fwd_fake(h, key_w, precision)
    q, fast, c, qop, kop, vop, P = memory_fwd_fake(z, v, precision)
    return q, fast, z, den, u_op, kw, c, qop, kop, vop, P


def _block_bwd_buffers(dfast_like, z, h, conv_w, v_dtype, precision, combine):
    """Outputs and work buffers of the fused block backward (ulm_addressed_memory_bwd / ulm_mixer_bwd)."""
    B, T, M = z.shape
    D = h.shape[-1]
    K = conv_w.shape[-1]
    dev = z.device
    opt = _op_dtype(precision)
    lib = L.lib()
    f32 = dict(device=dev, dtype=torch.float32)
    bufs = dict(
        dr=torch.empty(B, T, M, **f32), dv=torch.empty(B, T, D, device=dev, dtype=v_dtype),
        dg=torch.empty((), **f32), dw=torch.empty(M, **f32), doop=operand_copy(dfast_like, opt),
        dS=bwd_work_buffer(B, T, M, D, precision, dev), dqf=torch.empty(B, T, M, **f32),
        dk=torch.empty(B, T, M, **f32),
        partial=torch.empty(int(lib.ulm_memory_stats_bwd_scratch(B, T, M)), device=dev, dtype=torch.uint8),
        dh=torch.empty(B, T, D, **f32), dconv=torch.empty(D, K, **f32), dkw=torch.empty(M, D, **f32),
        dkb=torch.empty(M, **f32), deps=torch.empty((), **f32),
        work=torch.empty(int(lib.ulm_address_bwd_work_bytes(B, T, D, M, precision)), device=dev, dtype=torch.uint8),
        cw=conv_w.detach().reshape(D, K).float().contiguous())
    if combine:
        bufs["dmu"] = torch.empty(D, M, **f32)
        bufs["mw"] = torch.empty(D, operand_ld(M), device=dev, dtype=opt)
        bufs["gpart"] = torch.empty(int(lib.ulm_combine_grad_scratch(B, T, M, D)), device=dev, dtype=torch.uint8)
    return bufs


def addressed_memory_bwd_raw(dq_out, dfast, h, conv_w, g, w, q, z, den, u_op, kw, c, qop, kop, vop, P, precision):
    """ulm_addressed_memory_bwd on fresh buffers: (dh fp32, dconv_w, dkey_w, dkey_b, deps, dv, dg, dw)."""
    _require_cuda(dfast, z, g, w, q, c, den, h)
    B, T, M = z.shape
    D = dfast.shape[-1]
    K = conv_w.shape[-1]
    o = _block_bwd_buffers(dfast, z, h, conv_w, dfast.dtype, precision, combine=False)
    p = L.ptr
    with torch.cuda.device(z.device):
        L.check(L.lib().ulm_addressed_memory_bwd(
            p(dq_out), p(dfast), L.dtype_code(dfast.dtype), p(z), p(den), p(g), p(w), p(q),
            p(c) if c.numel() else None, p(qop), p(kop), p(vop), p(P), p(o["doop"]), p(o["dS"]), p(o["dqf"]),
            p(o["dk"]), p(o["partial"]), p(o["dr"]), p(o["dv"]), p(o["dg"]), p(o["dw"]), p(u_op), u_op.shape[1],
            p(h), L.dtype_code(h.dtype), p(o["cw"]), K, p(kw), kw.shape[1], p(o["dh"]), p(o["dconv"]), p(o["dkw"]),
            p(o["dkb"]), p(o["deps"]), p(o["work"]), B, T, M, D, precision, L.stream_of(z)))
    return (o["dh"], o["dconv"].reshape(D, 1, K), o["dkw"], o["dkb"], o["deps"], o["dv"], o["dg"], o["dw"])


def mixer_bwd_raw(dy, h, conv_w, g, w, mu, z, den, u_op, kw, q, c, qop, kop, vop, P, v_dtype, precision):
    """ulm_mixer_bwd on fresh buffers: (dh fp32, dconv_w, dkey_w, dkey_b, deps, dv, dg, dw, dmu)."""
    _require_cuda(dy, z, g, w, mu, den, h)
    B, T, M = z.shape
    D = dy.shape[-1]
    K = conv_w.shape[-1]
    o = _block_bwd_buffers(dy, z, h, conv_w, v_dtype, precision, combine=True)
    p = L.ptr
    with torch.cuda.device(z.device):
        L.check(L.lib().ulm_mixer_bwd(
            p(dy), L.dtype_code(dy.dtype), p(z), p(den), p(g), p(w), p(mu), p(q) if q.numel() else None,
            p(c) if c.numel() else None, p(qop), p(kop), p(vop), p(P), p(o["doop"]), p(o["dS"]), p(o["mw"]),
            p(o["dqf"]), p(o["dk"]), p(o["partial"]), p(o["gpart"]), p(o["dr"]), p(o["dv"]), L.dtype_code(v_dtype),
            p(o["dg"]), p(o["dw"]), p(o["dmu"]), p(u_op), u_op.shape[1], p(h), L.dtype_code(h.dtype), p(o["cw"]), K,
            p(kw), kw.shape[1], p(o["dh"]), p(o["dconv"]), p(o["dkw"]), p(o["dkb"]), p(o["deps"]), p(o["work"]), B, T,
            M, D, precision, L.stream_of(z)))
    return (o["dh"], o["dconv"].reshape(D, 1, K), o["dkw"], o["dkb"], o["deps"], o["dv"], o["dg"], o["dw"],
            o["dmu"])


@torch.library.custom_op("ulm::addressed_memory_bwd", mutates_args=())
def addressed_memory_bwd(dq_out: Optional[torch.Tensor], dfast: torch.Tensor, h: torch.Tensor, conv_w: torch.Tensor,
                         g: torch.Tensor, w: torch.Tensor, q: torch.Tensor, z: torch.Tensor, den: torch.Tensor,
                         u_op: torch.Tensor, kw: torch.Tensor, c: torch.Tensor, qop: torch.Tensor, kop: torch.Tensor,
                         vop: torch.Tensor, P: torch.Tensor, precision: int
                         ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                                    torch.Tensor, torch.Tensor, torch.Tensor]:
    """Returns (dh fp32, dconv_w, dkey_w, dkey_b, deps, dv, dg, dw)."""
    return addressed_memory_bwd_raw(dq_out, dfast, h, conv_w, g, w, q, z, den, u_op, kw, c, qop, kop, vop, P,
                                    precision)


@addressed_memory_bwd.register_fake
def _bwd_fake(dq_out, dfast, h, conv_w, g, w, q, z, den, u_op, kw, c, qop, kop, vop, P, precision):
    dh, dconv, dkw, dkb, deps = address_bwd_fake(h, z, conv_w)
    M = z.shape[-1]
    return (dh, dconv, dkw, dkb, deps, dfast.new_empty(dfast.shape), z.new_empty((), dtype=torch.float32),
            z.new_empty(M, dtype=torch.float32))


def _setup(ctx, inputs, output):
    h, conv_w, key_w, key_b, eps, v, g, w, precision = inputs
    q, fast, z, den, u_op, kw, c, qop, kop, vop, P = output
    ctx.save_for_backward(h, conv_w, g, w, q, z, den, u_op, kw, c, qop, kop, operand_or_input(vop, v), P)
    ctx.precision = precision
    ctx.dtypes = (h.dtype, conv_w.dtype, key_w.dtype, key_b.dtype, eps.dtype, v.dtype)
    ctx.v_dim = v.shape[-1]
    ctx.g_shape = g.shape
    ctx.mark_non_differentiable(z, den, u_op, kw, c, qop, kop, vop, P)
    ctx.set_materialize_grads(False)  # no zero tensors for the outputs nothing differentiates


def _backward(ctx, dq_out, dfast, *unused):
    if dq_out is None and dfast is None:
        return (None,) * 9
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


def mixer_fwd_raw(x, h, conv_w, key_w, key_b, eps, v, g, w, mu, precision):
    """The mixing span's forward without autograd (y = x + mu(q w) + fast, model.py:79-85) for
    inference: returns (y, z, den, kop, vop), the output and what a decode prefill reads."""
    z, den, u_op, kw = address_fwd_raw(h, conv_w, key_w, key_b, eps, precision, normalize=False)
    y, q, c, qop, kop, vop, P = combine_fwd_raw(z, den, v, g, w, mu, x, precision)
    return y, z, den, kop, vop


# ---- the whole mixing span of UnifiedBlock.forward with the combine fused (model.py:79-85) -------

_MIX_OUT = tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                 torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]


@torch.library.custom_op("ulm::mixer_fwd", mutates_args=())
def mixer_fwd(x: torch.Tensor, h: torch.Tensor, conv_w: torch.Tensor, key_w: torch.Tensor, key_b: torch.Tensor,
              eps: torch.Tensor, v: torch.Tensor, g: torch.Tensor, w: torch.Tensor, mu: torch.Tensor,
              precision: int) -> _MIX_OUT:
    """Returns (y, z, den, u_op, kw_op, q, c, qop, kop, vop, P); all but y are saved for the backward."""
    z, den, u_op, kw = address_fwd_raw(h, conv_w, key_w, key_b, eps, precision, normalize=False)
    y, q, c, qop, kop, vop, P = combine_fwd_raw(z, den, v, g, w, mu, x, precision)
    return y, z, den, u_op, kw, q, c, qop, kop, unaliased(vop, v), P


@mixer_fwd.register_fake
def _mixer_fwd_fake(x, h, conv_w, key_w, key_b, eps, v, g, w, mu, precision):
    z, den, u_op, kw = address_fwd_fake(h, key_w, precision)
    y, q, c, qop, kop, vop, P = combine_fwd_fake(z, v, x, precision)
    return y, z, den, u_op, kw, q, c, qop, kop, vop, P


@torch.library.custom_op("ulm::mixer_bwd", mutates_args=())
def mixer_bwd(dy: torch.Tensor, h: torch.Tensor, conv_w: torch.Tensor, g: torch.Tensor, w: torch.Tensor,
              mu: torch.Tensor, z: torch.Tensor, den: torch.Tensor, u_op: torch.Tensor, kw: torch.Tensor,
              q: torch.Tensor, c: torch.Tensor, qop: torch.Tensor, kop: torch.Tensor, vop: torch.Tensor,
              P: torch.Tensor, v_dtype: torch.dtype, precision: int
              ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                         torch.Tensor, torch.Tensor, torch.Tensor]:
    """Returns (dh fp32, dconv_w, dkey_w, dkey_b, deps, dv, dg, dw, dmu)."""
    return mixer_bwd_raw(dy, h, conv_w, g, w, mu, z, den, u_op, kw, q, c, qop, kop, vop, P, v_dtype, precision)


@mixer_bwd.register_fake
def _mixer_bwd_fake(dy, h, conv_w, g, w, mu, z, den, u_op, kw, q, c, qop, kop, vop, P, v_dtype, precision):
    dh, dconv, dkw, dkb, deps = address_bwd_fake(h, z, conv_w)
    M = z.shape[-1]
    return (dh, dconv, dkw, dkb, deps, dy.new_empty(dy.shape, dtype=v_dtype), z.new_empty((), dtype=torch.float32),
            z.new_empty(M, dtype=torch.float32), z.new_empty(mu.shape, dtype=torch.float32))


def _mix_setup(ctx, inputs, output):
    x, h, conv_w, key_w, key_b, eps, v, g, w, mu, precision = inputs
    y, z, den, u_op, kw, q, c, qop, kop, vop, P = output
    ctx.save_for_backward(h, conv_w, g, w, mu, z, den, u_op, kw, q, c, qop, kop, operand_or_input(vop, v), P)
    ctx.precision = precision
    ctx.dtypes = (x.dtype, h.dtype, conv_w.dtype, key_w.dtype, key_b.dtype, eps.dtype, v.dtype, mu.dtype)
    ctx.g_shape = g.shape
    ctx.mark_non_differentiable(z, den, u_op, kw, q, c, qop, kop, vop, P)
    ctx.set_materialize_grads(False)  # no zero tensors for the saved outputs


def _mix_backward(ctx, dy, *unused):
    if dy is None:
        return (None,) * 11
    h, conv_w, g, w, mu, z, den, u_op, kw, q, c, qop, kop, vop, P = ctx.saved_tensors
    xd, hd, cd, kd, bd, ed, vd, md = ctx.dtypes
    dh, dconv, dkw, dkb, deps, dv, dg, dw, dmu = mixer_bwd(dy.contiguous(), h, conv_w, g, w, mu, z, den, u_op, kw, q,
                                                           c, qop, kop, vop, P, vd, ctx.precision)
    return (dy, dh.to(hd), dconv.to(cd), dkw.to(kd), dkb.to(bd), deps.to(ed), dv, dg.reshape(ctx.g_shape), dw,
            dmu.to(md), None)


torch.library.register_autograd("ulm::mixer_fwd", _mix_backward, setup_context=_mix_setup)


def block_mixer(x, h, conv_weight, key_weight, key_bias, eps, v, g, w, mu_weight, precision="bf16"):
    """UnifiedBlock.forward's output without dropout (model.py:79-85):
    y = x + mu((q w)) + fast, (q, fast) = unified_memory(address(h, ...), v, g, w), in x's dtype,
    with the combine's product accumulated in the fast read's tiles and its gradient in the dq
    product's. mu_weight: the `mu` Linear's weight (D, M)."""
    for t in (x, h, v, g, w, mu_weight):
        if not t.is_cuda:
            raise RuntimeError("block_mixer runs on CUDA tensors only (no CPU path)")
    xx = x if x.dtype in (torch.float32, torch.bfloat16) else x.float()
    hh = h if h.dtype in (torch.float32, torch.bfloat16) else h.float()
    vv = v if v.dtype in (torch.float32, torch.bfloat16) else v.float()
    y, *_ = torch.ops.ulm.mixer_fwd(xx.contiguous(), hh.contiguous(), conv_weight, key_weight, key_bias,
                                    eps.float().reshape(()), vv.contiguous(), g.float().reshape(()),
                                    w.float().contiguous(), mu_weight.float().contiguous(), PRECISION[precision])
    return y.to(x.dtype)


# ---- UnifiedBlock.forward as one op (model.py:76-85 without dropout) -----------------------------
# x feeds both the norm and the residual, h both the val projection and the mixer; as one op the
# backward adds those gradients where they are produced (the val product's epilogue adds the
# mixer's dh, the norm backward adds the residual's dy as it writes dx) instead of in separate sums.

_BLOCK_OUT = tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                   torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                   torch.Tensor, torch.Tensor]


@torch.library.custom_op("ulm::block_fwd", mutates_args=())
def block_fwd(x: torch.Tensor, norm_w: torch.Tensor, conv_w: torch.Tensor, key_w: torch.Tensor, key_b: torch.Tensor,
              eps: torch.Tensor, val_w: torch.Tensor, g: torch.Tensor, w: torch.Tensor, mu: torch.Tensor,
              norm_eps: float, precision: int) -> _BLOCK_OUT:
    """Returns (y, h, rstd, v, x_op, wv_op, z, den, u_op, kw, q, c, qop, kop, vop, P); all but y are
    saved for the backward (v in bf16 for bf16 products, as the reference's autocast gives it)."""
    h, rstd = rms_norm_fwd_raw(x, norm_w, norm_eps)
    v, x_op, wv_op = linear_fwd_raw(h, val_w, precision, precision == PRECISION["bf16"])
    z, den, u_op, kw = address_fwd_raw(h, conv_w, key_w, key_b, eps, precision, normalize=False)
    y, q, c, qop, kop, vop, P = combine_fwd_raw(z, den, v, g, w, mu, x, precision)
    return y, h, rstd, v, x_op, wv_op, z, den, u_op, kw, q, c, qop, kop, unaliased(vop, v), P


@block_fwd.register_fake
def _block_fwd_fake(x, norm_w, conv_w, key_w, key_b, eps, val_w, g, w, mu, norm_eps, precision):
    h, rstd = _rms_norm_fwd_fake(x, norm_w, norm_eps)
    v, x_op, wv_op = _linear_fwd_fake(h, val_w, precision, precision == PRECISION["bf16"])
    z, den, u_op, kw = address_fwd_fake(h, key_w, precision)
    y, q, c, qop, kop, vop, P = combine_fwd_fake(z, v, x, precision)
    return y, h, rstd, v, x_op, wv_op, z, den, u_op, kw, q, c, qop, kop, vop, P


@torch.library.custom_op("ulm::block_bwd", mutates_args=())
def block_bwd(dy: torch.Tensor, x: torch.Tensor, norm_w: torch.Tensor, rstd: torch.Tensor, h: torch.Tensor,
              conv_w: torch.Tensor, g: torch.Tensor, w: torch.Tensor, mu: torch.Tensor, z: torch.Tensor,
              den: torch.Tensor, u_op: torch.Tensor, kw: torch.Tensor, q: torch.Tensor, c: torch.Tensor,
              qop: torch.Tensor, kop: torch.Tensor, vop: torch.Tensor, P: torch.Tensor, x_op: torch.Tensor,
              wv_op: torch.Tensor, v_dtype: torch.dtype, precision: int
              ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                         torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Returns (dx fp32, dnorm_w, dconv_w, dkey_w, dkey_b, deps, dval_w, dg, dw, dmu), fp32."""
    D = x.shape[-1]
    dh_mix, dconv, dkw, dkb, deps, dv, dg, dw, dmu = mixer_bwd_raw(dy, h, conv_w, g, w, mu, z, den, u_op, kw, q, c,
                                                                   qop, kop, vop, P, v_dtype, precision)
    # dh = dv W_v + the mixer's dh (added in the product's epilogue)
    dh, dval = linear_bwd_raw(dv.reshape(-1, D), x_op, wv_op, D, precision, dx_add=dh_mix.reshape(-1, D))
    # dx = the norm's backward + the residual's dy (added as dx is written)
    dx, dnorm = rms_norm_bwd_raw(dh.reshape(x.shape), x, norm_w, rstd, dx_add=dy.float().contiguous())
    return dx, dnorm, dconv, dkw, dkb, deps, dval, dg, dw, dmu


@block_bwd.register_fake
def _block_bwd_fake(dy, x, norm_w, rstd, h, conv_w, g, w, mu, z, den, u_op, kw, q, c, qop, kop, vop, P, x_op, wv_op,
                    v_dtype, precision):
    dh, dconv, dkw, dkb, deps = address_bwd_fake(h, z, conv_w)
    M, D = z.shape[-1], x.shape[-1]
    f32 = torch.float32
    return (x.new_empty(x.shape, dtype=f32), x.new_empty(D, dtype=f32), dconv, dkw, dkb, deps,
            x.new_empty(wv_op.shape[0], D, dtype=f32), z.new_empty((), dtype=f32), z.new_empty(M, dtype=f32),
            z.new_empty(mu.shape, dtype=f32))


def _blk_setup(ctx, inputs, output):
    x, norm_w, conv_w, key_w, key_b, eps, val_w, g, w, mu, norm_eps, precision = inputs
    y, h, rstd, v, x_op, wv_op, z, den, u_op, kw, q, c, qop, kop, vop, P = output
    ctx.save_for_backward(x, norm_w, rstd, h, conv_w, g, w, mu, z, den, u_op, kw, q, c, qop, kop,
                          operand_or_input(vop, v), P, x_op, wv_op)
    ctx.precision = precision
    ctx.v_dtype = v.dtype
    ctx.dtypes = (x.dtype, norm_w.dtype, conv_w.dtype, key_w.dtype, key_b.dtype, eps.dtype, val_w.dtype, mu.dtype)
    ctx.g_shape = g.shape
    ctx.mark_non_differentiable(h, rstd, v, x_op, wv_op, z, den, u_op, kw, q, c, qop, kop, vop, P)
    ctx.set_materialize_grads(False)


def _blk_backward(ctx, dy, *unused):
    if dy is None:
        return (None,) * 12
    (x, norm_w, rstd, h, conv_w, g, w, mu, z, den, u_op, kw, q, c, qop, kop, vop, P, x_op,
     wv_op) = ctx.saved_tensors
    xd, nd, cd, kd, bd, ed, vwd, md = ctx.dtypes
    dx, dnorm, dconv, dkw, dkb, deps, dval, dg, dw, dmu = block_bwd(
        dy.contiguous(), x, norm_w, rstd, h, conv_w, g, w, mu, z, den, u_op, kw, q, c, qop, kop, vop, P, x_op, wv_op,
        ctx.v_dtype, ctx.precision)
    return (dx.to(xd), dnorm.to(nd), dconv.to(cd), dkw.to(kd), dkb.to(bd), deps.to(ed), dval.to(vwd),
            dg.reshape(ctx.g_shape), dw, dmu.to(md), None, None)


torch.library.register_autograd("ulm::block_fwd", _blk_backward, setup_context=_blk_setup)


def unified_block(x, norm_weight, norm_eps, conv_weight, key_weight, key_bias, eps, val_weight, g, w, mu_weight,
                  precision="bf16"):
    """UnifiedBlock.forward without dropout (model.py:76-85): h = RMSNorm(x), v = val(h) (bf16 for
    bf16 products), y = x + mu(q w) + fast with (q, fast) = unified_memory(address(h, ...), v, g, w),
    in x's dtype."""
    for t in (x, norm_weight, val_weight, g, w, mu_weight):
        if not t.is_cuda:
            raise RuntimeError("unified_block runs on CUDA tensors only (no CPU path)")
    xx = x if x.dtype in (torch.float32, torch.bfloat16) else x.float()
    nw = norm_weight if norm_weight.dtype in (torch.float32, torch.bfloat16) else norm_weight.float()
    y, *_ = torch.ops.ulm.block_fwd(xx.contiguous(), nw.contiguous(), conv_weight, key_weight, key_bias,
                                    eps.float().reshape(()), val_weight.float().contiguous(), g.float().reshape(()),
                                    w.float().contiguous(), mu_weight.float().contiguous(), float(norm_eps),
                                    PRECISION[precision])
    return y.to(x.dtype)


# ---- the block's learned scalars (model.py:72, 75, 84) ---------------------------------------------

@torch.library.custom_op("ulm::block_scalars_fwd", mutates_args=())
def block_scalars_fwd(log_w: torch.Tensor, log_eps: torch.Tensor, log_rate: torch.Tensor
                      ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(w (M,), eps (), g ()) fp32 from fp32 log parameters in one launch (ulm_block_scalars_fwd)."""
    w = torch.empty_like(log_w)
    eps = log_eps.new_empty(())
    g = log_rate.new_empty(())
    with torch.cuda.device(log_w.device):
        L.check(L.lib().ulm_block_scalars_fwd(L.ptr(log_w), L.ptr(log_eps), L.ptr(log_rate), L.ptr(w), L.ptr(eps),
                                              L.ptr(g), log_w.numel(), L.stream_of(log_w)))
    return w, eps, g


@block_scalars_fwd.register_fake
def _block_scalars_fwd_fake(log_w, log_eps, log_rate):
    return log_w.new_empty(log_w.shape), log_eps.new_empty(()), log_rate.new_empty(())


@torch.library.custom_op("ulm::block_scalars_bwd", mutates_args=())
def block_scalars_bwd(log_w: torch.Tensor, log_eps: torch.Tensor, w: torch.Tensor, eps: torch.Tensor,
                      g: torch.Tensor, dw: torch.Tensor, deps: torch.Tensor, dg: torch.Tensor
                      ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(dlog_w, dlog_eps, dlog_rate) in one launch (ulm_block_scalars_bwd)."""
    dlw = torch.empty_like(log_w)
    dle = log_eps.new_empty(())
    dlr = g.new_empty(())
    with torch.cuda.device(log_w.device):
        L.check(L.lib().ulm_block_scalars_bwd(L.ptr(log_w), L.ptr(log_eps), L.ptr(w), L.ptr(eps), L.ptr(g),
                                              L.ptr(dw), L.ptr(deps), L.ptr(dg), L.ptr(dlw), L.ptr(dle), L.ptr(dlr),
                                              log_w.numel(), L.stream_of(log_w)))
    return dlw, dle, dlr


@block_scalars_bwd.register_fake
def _block_scalars_bwd_fake(log_w, log_eps, w, eps, g, dw, deps, dg):
    return log_w.new_empty(log_w.shape), log_eps.new_empty(()), g.new_empty(())


def _bs_setup(ctx, inputs, output):
    log_w, log_eps, _ = inputs
    w, eps, g = output
    ctx.save_for_backward(log_w, log_eps, w, eps, g)


def _bs_backward(ctx, dw, deps, dg):
    log_w, log_eps, w, eps, g = ctx.saved_tensors
    dw = torch.zeros_like(w) if dw is None else dw.float().contiguous()
    deps = torch.zeros_like(eps) if deps is None else deps.float().reshape(())
    dg = torch.zeros_like(g) if dg is None else dg.float().reshape(())
    return block_scalars_bwd(log_w, log_eps, w, eps, g, dw, deps, dg)


torch.library.register_autograd("ulm::block_scalars_fwd", _bs_backward, setup_context=_bs_setup)


def block_scalars(log_w, log_eps, log_rate):
    """UnifiedBlock's learned scalars as the reference evaluates them (model.py:72, 75, 84):
    w = exp(clamp(log_w, -7, 12)), eps = exp(clamp(log_eps, -10, 10)), g = -exp(log_rate), in
    fp32, with the same gradients as autograd of those expressions; one launch each way instead of
    one per elementwise step."""
    for t in (log_w, log_eps, log_rate):
        if not t.is_cuda:
            raise RuntimeError("block_scalars runs on CUDA tensors only (no CPU path)")
    return torch.ops.ulm.block_scalars_fwd(log_w.float().contiguous(), log_eps.float().reshape(()),
                                           log_rate.float().reshape(()))
