"""The addressing prologue of UnifiedBlock on sm_100a: h -> r (model.py:61-62, 70-72, 79).

    u = causal depthwise conv(h),  z = relu(u K^T + b)^2,  r = z / (eps + sum_m z)

`address(h, conv_weight, key_weight, key_bias, eps, precision)` returns r (fp32, (B,T,M)) and is
differentiable in h, the conv weight (D,1,K), the key weight (M,D), the key bias (M,) and eps (0-d);
eps = exp(clamp(log_eps, -10, 10)) stays a torch expression in the caller so autograd applies the
clamp exactly as the reference does. The work runs in libulm_b200.so (ulm_address_fwd / _bwd) through
the `torch.library` ops `ulm::address_fwd` and `ulm::address_bwd`.
"""
import torch

from . import _lib as L
from .kernel import PRECISION, operand_ld


def _op_dtype(precision):
    return torch.float32 if precision == L.ULM_PREC_FP32 else torch.bfloat16


def _weight_op(key_w, precision):
    M, D = key_w.shape
    ld = operand_ld(D)
    kw = torch.empty(M, ld, device=key_w.device, dtype=_op_dtype(precision))
    kw[:, :D].copy_(key_w.detach())
    if ld > D:
        kw[:, D:].zero_()
    return kw


def address_fwd_raw(h, conv_w, key_w, key_b, eps, precision, normalize=True):
    """ulm_address_fwd on fresh buffers: (r, den, u_op, kw_op); with normalize=False the first
    output holds z = r * den (the row sums come from the key product's epilogue)."""
    B, T, D = h.shape
    M = key_w.shape[0]
    K = conv_w.shape[-1]
    dev = h.device
    r = torch.empty(B, T, M, device=dev, dtype=torch.float32)
    den = torch.empty(B * T, device=dev, dtype=torch.float32)
    u_op = torch.empty(B * T, operand_ld(D), device=dev, dtype=_op_dtype(precision))
    kw = _weight_op(key_w, precision)
    cw = conv_w.detach().reshape(D, K).float().contiguous()
    kb = key_b.detach().float().contiguous()
    lib = L.lib()
    work = None if normalize else torch.empty(int(lib.ulm_address_fwd_work_bytes(B, T, M)), device=dev,
                                              dtype=torch.uint8)
    with torch.cuda.device(dev):
        L.check(lib.ulm_address_fwd(L.ptr(h), L.dtype_code(h.dtype), L.ptr(cw), K, L.ptr(kw), kw.shape[1],
                                    L.ptr(kb), L.ptr(eps), L.ptr(r), L.ptr(den), 1 if normalize else 0, L.ptr(work),
                                    L.ptr(u_op), u_op.shape[1], B, T, D, M, precision, L.stream_of(h)))
    return r, den, u_op, kw


def address_fwd_fake(h, key_w, precision):
    B, T, D = h.shape
    M = key_w.shape[0]
    opt = _op_dtype(precision)
    return (h.new_empty(B, T, M, dtype=torch.float32), h.new_empty(B * T, dtype=torch.float32),
            h.new_empty(B * T, operand_ld(D), dtype=opt), h.new_empty(M, operand_ld(D), dtype=opt))


def address_bwd_raw(dr, r, den, u_op, kw, h, conv_w, precision, normalized=True):
    """ulm_address_bwd on fresh buffers: (dh fp32, dconv_w (D,1,K), dkey_w (M,D), dkey_b (M,),
    deps 0-d); r and den as address_fwd_raw returned them with the same normalize flag."""
    B, T, D = h.shape
    M = r.shape[-1]
    K = conv_w.shape[-1]
    dev = h.device
    dh = torch.empty(B, T, D, device=dev, dtype=torch.float32)
    dconv = torch.empty(D, K, device=dev, dtype=torch.float32)
    dkw = torch.empty(M, D, device=dev, dtype=torch.float32)
    dkb = torch.empty(M, device=dev, dtype=torch.float32)
    deps = torch.empty((), device=dev, dtype=torch.float32)
    work = torch.empty(int(L.lib().ulm_address_bwd_work_bytes(B, T, D, M, precision)), device=dev, dtype=torch.uint8)
    cw = conv_w.detach().reshape(D, K).float().contiguous()
    drc = dr.float().contiguous()
    with torch.cuda.device(dev):
        L.check(L.lib().ulm_address_bwd(L.ptr(drc), L.ptr(r), L.ptr(den), 1 if normalized else 0, L.ptr(u_op),
                                        u_op.shape[1], L.ptr(h), L.dtype_code(h.dtype), L.ptr(cw), K, L.ptr(kw),
                                        kw.shape[1], L.ptr(dh), L.ptr(dconv), L.ptr(dkw), L.ptr(dkb), L.ptr(deps),
                                        L.ptr(work), B, T, D, M, precision, L.stream_of(h)))
    return dh, dconv.reshape(D, 1, K), dkw, dkb, deps


def address_bwd_fake(h, r, conv_w):
    B, T, D = h.shape
    M = r.shape[-1]
    K = conv_w.shape[-1]
    return (h.new_empty(B, T, D, dtype=torch.float32), h.new_empty(D, 1, K, dtype=torch.float32),
            h.new_empty(M, D, dtype=torch.float32), h.new_empty(M, dtype=torch.float32),
            h.new_empty((), dtype=torch.float32))


@torch.library.custom_op("ulm::address_fwd", mutates_args=())
def address_fwd(h: torch.Tensor, conv_w: torch.Tensor, key_w: torch.Tensor, key_b: torch.Tensor, eps: torch.Tensor,
                precision: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Returns (r, den, u_op, kw_op); the last three are saved for the backward."""
    return address_fwd_raw(h, conv_w, key_w, key_b, eps, precision)


@address_fwd.register_fake
def _address_fwd_fake(h, conv_w, key_w, key_b, eps, precision):
    return address_fwd_fake(h, key_w, precision)


@torch.library.custom_op("ulm::address_bwd", mutates_args=())
def address_bwd(dr: torch.Tensor, r: torch.Tensor, den: torch.Tensor, u_op: torch.Tensor, kw: torch.Tensor,
                h: torch.Tensor, conv_w: torch.Tensor, precision: int
                ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Returns (dh fp32, dconv_w (D,1,K), dkey_w (M,D), dkey_b (M,), deps 0-d)."""
    return address_bwd_raw(dr, r, den, u_op, kw, h, conv_w, precision)


@address_bwd.register_fake
def _address_bwd_fake(dr, r, den, u_op, kw, h, conv_w, precision):
    return address_bwd_fake(h, r, conv_w)


def _setup(ctx, inputs, output):
    h, conv_w, key_w, key_b, eps, precision = inputs
    r, den, u_op, kw = output
    ctx.save_for_backward(r, den, u_op, kw, h, conv_w)
    ctx.precision = precision
    ctx.dtypes = (h.dtype, conv_w.dtype, key_w.dtype, key_b.dtype, eps.dtype)
    ctx.mark_non_differentiable(den, u_op, kw)
    ctx.set_materialize_grads(False)  # no zero tensors for the outputs nothing differentiates


def _backward(ctx, dr, *unused):
    if dr is None:
        return None, None, None, None, None, None
    r, den, u_op, kw, h, conv_w = ctx.saved_tensors
    dh, dconv, dkw, dkb, deps = address_bwd(dr, r, den, u_op, kw, h, conv_w, ctx.precision)
    hd, cd, kd, bd, ed = ctx.dtypes
    return dh.to(hd), dconv.to(cd), dkw.to(kd), dkb.to(bd), deps.to(ed), None


torch.library.register_autograd("ulm::address_fwd", _backward, setup_context=_setup)


def address(h, conv_weight, key_weight, key_bias, eps, precision="bf16"):
    """r = relu(conv(h) K^T + b)^2 / (eps + sum): UnifiedBlock.code(conv(h)) (model.py:70-72, 79)."""
    if not h.is_cuda:
        raise RuntimeError("address runs on CUDA tensors only (no CPU path)")
    hh = h if h.dtype in (torch.float32, torch.bfloat16) else h.float()
    r, *_ = torch.ops.ulm.address_fwd(hh.contiguous(), conv_weight, key_weight, key_bias,
                                      eps.float().reshape(()), PRECISION[precision])
    return r
