"""RMSNorm and Linear of UnifiedBlock's input side as library ops (model.py:31-42, 65, 81).

`rms_norm(x, weight, eps)` = x / sqrt(mean(x^2) + eps) in fp32, rounded to x's type, times weight
(the reference's RMSNorm.forward); `linear(x, weight, precision)` = x W^T in x's type with bf16
tensor-core products and fp32 accumulation ("bf16") or fp32 products ("fp32"). Both are
`torch.library` custom ops with fake kernels and autograd (libulm_b200.so: ulm_rms_norm_fwd / _bwd,
ulm_linear_fwd / _bwd), launched on the current CUDA stream. No CPU path.
"""
import torch

from . import _lib as L
from .kernel import PRECISION, _op_dtype, _require_cuda, operand_ld


def rms_norm_fwd_raw(x, weight, eps):
    """ulm_rms_norm_fwd on fresh buffers: (y in promote(x, weight) type, rstd (rows,) fp32)."""
    _require_cuda(x, weight)
    D = x.shape[-1]
    rows = x.numel() // max(D, 1)
    y = torch.empty(x.shape, device=x.device, dtype=torch.promote_types(x.dtype, weight.dtype))
    rstd = torch.empty(rows, device=x.device, dtype=torch.float32)
    with torch.cuda.device(x.device):
        L.check(L.lib().ulm_rms_norm_fwd(L.ptr(x), L.dtype_code(x.dtype), L.ptr(weight), L.ptr(y),
                                         L.dtype_code(y.dtype), L.ptr(rstd), rows, D, float(eps), L.stream_of(x)))
    return y, rstd


@torch.library.custom_op("ulm::rms_norm_fwd", mutates_args=())
def rms_norm_fwd(x: torch.Tensor, weight: torch.Tensor, eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns (y, rstd); y in promote(x, weight) type, rstd (rows,) fp32 saved for the backward."""
    return rms_norm_fwd_raw(x, weight, eps)


@rms_norm_fwd.register_fake
def _rms_norm_fwd_fake(x, weight, eps):
    D = x.shape[-1]
    rows = x.numel() // max(D, 1)
    return (x.new_empty(x.shape, dtype=torch.promote_types(x.dtype, weight.dtype)),
            x.new_empty(rows, dtype=torch.float32))


def rms_norm_bwd_raw(dy, x, weight, rstd, dx_add=None):
    """ulm_rms_norm_bwd on fresh buffers: (dx fp32 (+ dx_add fp32 when given), dweight fp32)."""
    D = x.shape[-1]
    rows = x.numel() // max(D, 1)
    dx = torch.empty(x.shape, device=x.device, dtype=torch.float32)
    dw = torch.empty(D, device=x.device, dtype=torch.float32)
    work = torch.empty(int(L.lib().ulm_rms_norm_bwd_work_bytes(rows, D)), device=x.device, dtype=torch.uint8)
    with torch.cuda.device(x.device):
        L.check(L.lib().ulm_rms_norm_bwd(L.ptr(dy), L.dtype_code(dy.dtype), L.ptr(x), L.dtype_code(x.dtype),
                                         L.ptr(weight), L.ptr(rstd), L.ptr(dx), L.ptr(dx_add), L.ptr(dw),
                                         L.ptr(work), rows, D, L.stream_of(x)))
    return dx, dw


@torch.library.custom_op("ulm::rms_norm_bwd", mutates_args=())
def rms_norm_bwd(dy: torch.Tensor, x: torch.Tensor, weight: torch.Tensor, rstd: torch.Tensor
                 ) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns (dx fp32, dweight fp32)."""
    return rms_norm_bwd_raw(dy, x, weight, rstd)


@rms_norm_bwd.register_fake
def _rms_norm_bwd_fake(dy, x, weight, rstd):
    return x.new_empty(x.shape, dtype=torch.float32), x.new_empty(x.shape[-1], dtype=torch.float32)


def _rn_setup(ctx, inputs, output):
    x, weight, eps = inputs
    ctx.save_for_backward(x, weight, output[1])
    ctx.dtypes = (x.dtype, weight.dtype)
    ctx.mark_non_differentiable(output[1])
    ctx.set_materialize_grads(False)


def _rn_backward(ctx, dy, _drstd):
    if dy is None:
        return None, None, None
    x, weight, rstd = ctx.saved_tensors
    dx, dw = rms_norm_bwd(dy.contiguous(), x, weight, rstd)
    return dx.to(ctx.dtypes[0]), dw.to(ctx.dtypes[1]), None


torch.library.register_autograd("ulm::rms_norm_fwd", _rn_backward, setup_context=_rn_setup)


def rms_norm(x, weight, eps):
    """RMSNorm (model.py:31-42): x (..., D) fp32 or bf16, weight (D,) fp32 or bf16."""
    xx = x if x.dtype in (torch.float32, torch.bfloat16) else x.float()
    w = weight if weight.dtype in (torch.float32, torch.bfloat16) else weight.float()
    y, _ = torch.ops.ulm.rms_norm_fwd(xx.contiguous(), w.contiguous(), float(eps))
    return y


# ---- Linear --------------------------------------------------------------------------------------

def linear_fwd_raw(x, weight, precision, out_bf16):
    """ulm_linear_fwd on fresh buffers: (y, x_op, w_op)."""
    _require_cuda(x, weight)
    K = x.shape[-1]
    N = x.numel() // max(K, 1)
    Nout = weight.shape[0]
    opt = _op_dtype(precision)
    y = torch.empty(*x.shape[:-1], Nout, device=x.device, dtype=torch.bfloat16 if out_bf16 else x.dtype)
    x_op = torch.empty(N, operand_ld(K), device=x.device, dtype=opt)
    w_op = torch.empty(Nout, operand_ld(K), device=x.device, dtype=opt)
    with torch.cuda.device(x.device):
        L.check(L.lib().ulm_linear_fwd(L.ptr(x), L.dtype_code(x.dtype), L.ptr(weight), L.ptr(x_op), L.ptr(w_op),
                                       L.ptr(y), L.dtype_code(y.dtype), N, K, Nout, precision, L.stream_of(x)))
    return y, x_op, w_op


@torch.library.custom_op("ulm::linear_fwd", mutates_args=())
def linear_fwd(x: torch.Tensor, weight: torch.Tensor, precision: int, out_bf16: bool
               ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Returns (y, x_op, w_op); y in x's type or bf16 (out_bf16); the operand copies are saved for
    the backward."""
    return linear_fwd_raw(x, weight, precision, out_bf16)


@linear_fwd.register_fake
def _linear_fwd_fake(x, weight, precision, out_bf16):
    K = x.shape[-1]
    N = x.numel() // max(K, 1)
    opt = _op_dtype(precision)
    return (x.new_empty(*x.shape[:-1], weight.shape[0], dtype=torch.bfloat16 if out_bf16 else x.dtype),
            x.new_empty(N, operand_ld(K), dtype=opt),
            x.new_empty(weight.shape[0], operand_ld(K), dtype=opt))


def linear_bwd_raw(dy, x_op, w_op, K, precision, dx_add=None):
    """ulm_linear_bwd on fresh buffers: (dx fp32 (N, K) (+ dx_add fp32 (N, K) when given), dweight
    fp32 (Nout, K))."""
    Nout = w_op.shape[0]
    N = x_op.shape[0]
    dx = torch.empty(N, K, device=dy.device, dtype=torch.float32)
    dw = torch.empty(Nout, K, device=dy.device, dtype=torch.float32)
    work = torch.empty(int(L.lib().ulm_linear_bwd_work_bytes(N, K, Nout, precision)), device=dy.device,
                       dtype=torch.uint8)
    with torch.cuda.device(dy.device):
        L.check(L.lib().ulm_linear_bwd(L.ptr(dy), L.dtype_code(dy.dtype), L.ptr(x_op), L.ptr(w_op), L.ptr(dx),
                                       L.ptr(dx_add), L.ptr(dw), L.ptr(work), N, K, Nout, precision,
                                       L.stream_of(dy)))
    return dx, dw


@torch.library.custom_op("ulm::linear_bwd", mutates_args=())
def linear_bwd(dy: torch.Tensor, x_op: torch.Tensor, w_op: torch.Tensor, K: int, precision: int
               ) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns (dx fp32 (N, K), dweight fp32 (Nout, K))."""
    return linear_bwd_raw(dy, x_op, w_op, K, precision)


@linear_bwd.register_fake
def _linear_bwd_fake(dy, x_op, w_op, K, precision):
    return (dy.new_empty(x_op.shape[0], K, dtype=torch.float32),
            dy.new_empty(w_op.shape[0], K, dtype=torch.float32))


def _lin_setup(ctx, inputs, output):
    x, weight, precision, out_bf16 = inputs
    ctx.save_for_backward(output[1], output[2])
    ctx.meta = (x.shape, x.dtype, weight.dtype, precision)
    ctx.mark_non_differentiable(output[1], output[2])
    ctx.set_materialize_grads(False)


def _lin_backward(ctx, dy, _dx_op, _dw_op):
    if dy is None:
        return None, None, None, None
    x_op, w_op = ctx.saved_tensors
    shape, xdt, wdt, precision = ctx.meta
    dx, dw = linear_bwd(dy.reshape(-1, dy.shape[-1]).contiguous(), x_op, w_op, shape[-1], precision)
    return dx.reshape(shape).to(xdt), dw.to(wdt), None, None


torch.library.register_autograd("ulm::linear_fwd", _lin_backward, setup_context=_lin_setup)


def linear(x, weight, precision="bf16", out_dtype=None):
    """x W^T without bias (nn.Linear's forward for UnifiedBlock.val): x (..., K) fp32 or bf16,
    weight (Nout, K); the result has x's type, or bf16 with out_dtype=torch.bfloat16 (the type
    autocast gives it, and the one the fast memory's tensor-core operands use)."""
    xx = x if x.dtype in (torch.float32, torch.bfloat16) else x.float()
    bf16 = out_dtype == torch.bfloat16
    y, _, _ = torch.ops.ulm.linear_fwd(xx.contiguous(), weight.float().contiguous(), PRECISION[precision], bf16)
    want = torch.bfloat16 if bf16 else x.dtype
    return y if y.dtype == want else y.to(want)
