"""UnifiedLM's output Linear with its cross-entropy loss, fused on sm_100a (model.py:153-157).

`lm_head_loss(h, weight, targets, precision)` equals
`F.cross_entropy((h @ weight.T).view(-1, V), targets.view(-1), ignore_index=-1)` with the same
gradients for h and weight, but the (N, V) logits are never materialised: the forward product's
epilogue keeps each row's running max and sum of exponentials per column block and the target's
logit; the backward recomputes the product with an epilogue that writes dlogits = (softmax - onehot)
* dloss / count (operand type), followed by dh = dlogits W and dW = dlogits^T h. The work runs in
libulm_b200.so (ulm_lm_head_loss_fwd / _bwd) through the `torch.library` ops `ulm::lm_head_fwd` and
`ulm::lm_head_bwd`.
"""
import torch

from . import _lib as L
from .kernel import PRECISION, _op_dtype, operand_ld


def _weight_op(weight, opt):
    V, D = weight.shape
    if weight.dtype == opt and operand_ld(D) == D and weight.is_contiguous():
        return weight.detach()
    w = torch.empty(V, operand_ld(D), device=weight.device, dtype=opt)
    w[:, :D] = weight.detach()
    return w


@torch.library.custom_op("ulm::lm_head_fwd", mutates_args=())
def lm_head_fwd(h: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor, precision: int
                ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """h (N, D), weight (V, D), targets (N,) int64. Returns (loss 0-d, lse, count, h_op, w_op, work);
    all but the loss are saved for the backward."""
    N, D = h.shape
    V = weight.shape[0]
    dev = h.device
    opt = _op_dtype(precision)
    lib = L.lib()
    h_op = torch.empty(N, operand_ld(D), device=dev, dtype=opt)
    h_op[:, :D] = h.detach()
    w_op = _weight_op(weight, opt)
    if w_op.data_ptr() == weight.data_ptr():
        w_op = w_op.clone()  # outputs of the op may not alias its inputs
    lse = torch.empty(N, device=dev, dtype=torch.float32)
    loss = torch.empty((), device=dev, dtype=torch.float32)
    count = torch.empty((), device=dev, dtype=torch.float32)
    work = torch.empty(int(lib.ulm_lm_head_work_bytes(N, V, D, precision)), device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        L.check(lib.ulm_lm_head_loss_fwd(L.ptr(h_op), h_op.shape[1], L.ptr(w_op), w_op.shape[1], L.ptr(targets),
                                         L.ptr(lse), L.ptr(loss), L.ptr(count), L.ptr(work), N, V, D, precision,
                                         L.stream_of(h)))
    return loss, lse, count, h_op, w_op, work


@lm_head_fwd.register_fake
def _lm_head_fwd_fake(h, weight, targets, precision):
    N, D = h.shape
    V = weight.shape[0]
    opt = _op_dtype(precision)
    nbytes = int(L.lib().ulm_lm_head_work_bytes(N, V, D, precision))
    return (h.new_empty((), dtype=torch.float32), h.new_empty(N, dtype=torch.float32),
            h.new_empty((), dtype=torch.float32), h.new_empty(N, operand_ld(D), dtype=opt),
            h.new_empty(V, operand_ld(D), dtype=opt), h.new_empty(nbytes, dtype=torch.uint8))


@torch.library.custom_op("ulm::lm_head_bwd", mutates_args=("work",))
def lm_head_bwd(dloss: torch.Tensor, count: torch.Tensor, h_op: torch.Tensor, w_op: torch.Tensor,
                targets: torch.Tensor, lse: torch.Tensor, work: torch.Tensor, D: int, precision: int
                ) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns (dh (N, D) fp32, dW (V, D) fp32)."""
    N = h_op.shape[0]
    V = w_op.shape[0]
    dev = h_op.device
    dh = torch.empty(N, D, device=dev, dtype=torch.float32)
    dw = torch.empty(V, D, device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        L.check(L.lib().ulm_lm_head_loss_bwd(L.ptr(dloss), L.ptr(count), L.ptr(h_op), h_op.shape[1], L.ptr(w_op),
                                             w_op.shape[1], L.ptr(targets), L.ptr(lse), L.ptr(dh), L.ptr(dw),
                                             L.ptr(work), N, V, D, precision, L.stream_of(h_op)))
    return dh, dw


@lm_head_bwd.register_fake
def _lm_head_bwd_fake(dloss, count, h_op, w_op, targets, lse, work, D, precision):
    return (h_op.new_empty(h_op.shape[0], D, dtype=torch.float32),
            h_op.new_empty(w_op.shape[0], D, dtype=torch.float32))


def _setup(ctx, inputs, output):
    h, weight, targets, precision = inputs
    loss, lse, count, h_op, w_op, work = output
    ctx.save_for_backward(count, h_op, w_op, targets, lse, work)
    ctx.precision = precision
    ctx.D = h.shape[1]
    ctx.dtypes = (h.dtype, weight.dtype)
    ctx.mark_non_differentiable(lse, count, h_op, w_op, work)
    ctx.set_materialize_grads(False)  # no zero tensors for the outputs nothing differentiates


def _backward(ctx, dloss, *unused):
    if dloss is None:
        return None, None, None, None
    count, h_op, w_op, targets, lse, work = ctx.saved_tensors
    dh, dw = lm_head_bwd(dloss.float().reshape(()).contiguous(), count, h_op, w_op, targets, lse, work, ctx.D,
                         ctx.precision)
    hd, wd = ctx.dtypes
    return dh.to(hd), dw.to(wd), None, None


torch.library.register_autograd("ulm::lm_head_fwd", _backward, setup_context=_setup)


def lm_head_loss(h, weight, targets, precision="bf16"):
    """Mean cross entropy of h @ weight.T against targets (ignore_index -1): h (..., D) on the GPU,
    weight (V, D), targets (...) integer."""
    if not h.is_cuda:
        raise RuntimeError("lm_head_loss runs on CUDA tensors only (no CPU path)")
    D = h.shape[-1]
    hh = h.reshape(-1, D)
    hh = hh if hh.dtype in (torch.float32, torch.bfloat16) else hh.float()
    tg = targets.reshape(-1).to(torch.int64).contiguous()
    loss, *_ = torch.ops.ulm.lm_head_fwd(hh.contiguous(), weight, tg, PRECISION[precision])
    return loss
