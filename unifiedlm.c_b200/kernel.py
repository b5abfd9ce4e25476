"""Drop-in replacement of the reference's kernel.py: UnifiedBlock's fast memory on sm_100a.

unified_memory(r, v, g, w) -> (q, fast), for every batch row and position t (kernel.py:1-15):

    k_t    = r_{t-1}                                     (k_0 = 0, write address)
    c_t    = w + sum_{s<=t} lam^(t-s) k_s                (slot evidence mass, lam = exp(g))
    q_t    = r_t / c_t
    fast_t = sum_{s<=t} lam^(t-s) (q_t . k_s) v_s

Same names, argument meaning, dtypes and gradients as the reference (kernel.py:199-238): r any float
(computed in fp32), v (B,T,D), g a 0-d tensor (log decay), w (M,); q is fp32, fast has v's dtype;
the backward returns (dr fp32, dv in dfast's dtype, dg 0-d, dw (M,) fp32).

The work runs in libulm_b200.so (include/ulm_b200.h) on the current CUDA stream, through two
`torch.library` custom ops (`ulm::memory_fwd`, `ulm::memory_bwd`) with fake kernels, so the call is
traceable by torch.compile. `precision="bf16"` (default) contracts bf16 operands on the tensor
cores with fp32 accumulation like the reference; `precision="fp32"` contracts in fp32 for 1e-5
parity. There is no CPU path: CPU tensors or a missing library raise.
"""
from typing import Optional

import torch

from . import _lib as L

CHUNK = 64  # the reference's chunk length (kernel.py:20); here the form and chunk length of the fast
            # read's products follow ulm_memory_chunk_len (whole sequences up to a few thousand tokens)

PRECISION = {"bf16": L.ULM_PREC_BF16, "fp32": L.ULM_PREC_FP32}


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("unified_memory runs on CUDA tensors only (no CPU path)")


def operand_ld(n):
    return (n + 7) // 8 * 8


def _op_dtype(precision):
    return torch.float32 if precision == L.ULM_PREC_FP32 else torch.bfloat16


def serves_as_operand(x, opt):
    """Whether a (B,T,D) array can be its own tensor-core operand copy: the operand type, a row
    stride that needs no padding, contiguous (and, checked by operand_copy on real tensors, a
    16-byte aligned start; the fake kernels assume it, as every fresh allocation is)."""
    return x.dtype == opt and operand_ld(x.shape[-1]) == x.shape[-1] and x.is_contiguous()


def operand_copy(x, opt):
    """Buffer for the tensor-core operand copy of a (B,T,D) array: x itself when it serves as one
    (the library then skips the copy), else a new one."""
    B, T, D = x.shape
    if serves_as_operand(x, opt) and x.data_ptr() % 16 == 0:
        return x
    return torch.empty(B, T, operand_ld(D), device=x.device, dtype=opt)


def operand_copy_fake(x, opt):
    """The fake-tensor counterpart of unaliased(operand_copy(x, opt), x)."""
    B, T, D = x.shape
    return x.new_empty(0, dtype=x.dtype) if serves_as_operand(x, opt) else x.new_empty(B, T, operand_ld(D), dtype=opt)


def saved_buffer(B, T, M, D, precision, device):
    """The fast read's saved buffer (ulm_memory_saved_bytes): the decayed scores in the
    whole-sequence form, the chunk-boundary states and intra-chunk scores in the chunk-carry form."""
    n = int(L.lib().ulm_memory_saved_bytes(B, T, M, D, precision))
    return torch.empty(n, device=device, dtype=torch.uint8)


def bwd_work_buffer(B, T, M, D, precision, device):
    """The operator backward's work buffer (ulm_memory_bwd_work_bytes)."""
    n = int(L.lib().ulm_memory_bwd_work_bytes(B, T, M, D, precision))
    return torch.empty(n, device=device, dtype=torch.uint8)


def memory_fwd_raw(r, den, v, g, w, precision):
    """ulm_memory_fwd on fresh buffers: (q, fast, c, qop, kop, vop, P). den None: r holds the
    addresses; else r holds z and den the row denominators (r = z / den)."""
    _require_cuda(r, v, g, w, den)
    B, T, M = r.shape
    D = v.shape[-1]
    dev = r.device
    opt = _op_dtype(precision)
    q = torch.empty(B, T, M, device=dev, dtype=torch.float32)
    # the backward rebuilds c from r on the TMA scan path; an empty placeholder stands in for it
    c = torch.empty_like(q) if L.lib().ulm_memory_needs_c(T, M) else q.new_empty(0)
    fast = torch.empty(B, T, D, device=dev, dtype=v.dtype)
    qop = torch.empty(B, T, operand_ld(M), device=dev, dtype=opt)
    kop = torch.empty_like(qop)
    vop = operand_copy(v, opt)
    P = saved_buffer(B, T, M, D, precision, dev)
    with torch.cuda.device(dev):
        L.check(L.lib().ulm_memory_fwd(L.ptr(r), L.ptr(den), L.ptr(v), L.dtype_code(v.dtype), L.ptr(g), L.ptr(w),
                                       L.ptr(q), L.ptr(fast), L.ptr(c) if c.numel() else None, L.ptr(qop),
                                       L.ptr(kop), L.ptr(vop), L.ptr(P),
                                       B, T, M, D, precision, L.stream_of(r)))
    return q, fast, c, qop, kop, vop, P


def memory_fwd_fake(r, v, precision):
    B, T, M = r.shape
    D = v.shape[-1]
    opt = _op_dtype(precision)
    c_shape = (B, T, M) if L.lib().ulm_memory_needs_c(T, M) else (0,)
    return (r.new_empty(B, T, M, dtype=torch.float32), v.new_empty(B, T, D), r.new_empty(c_shape, dtype=torch.float32),
            r.new_empty(B, T, operand_ld(M), dtype=opt), r.new_empty(B, T, operand_ld(M), dtype=opt),
            operand_copy_fake(v, opt),
            r.new_empty(int(L.lib().ulm_memory_saved_bytes(B, T, M, D, precision)), dtype=torch.uint8))


def memory_bwd_raw(dq_out, dfast, r, den, g, w, q, c, qop, kop, vop, P, precision):
    """ulm_memory_bwd on fresh buffers: (dr, dv, dg, dw); dr is the gradient of the normalised
    addresses whether r holds them or z (with den)."""
    _require_cuda(dfast, r, g, w, q, c, den)
    B, T, M = r.shape
    D = dfast.shape[-1]
    dev = r.device
    opt = _op_dtype(precision)
    dr = torch.empty(B, T, M, device=dev, dtype=torch.float32)
    dv = torch.empty(B, T, D, device=dev, dtype=dfast.dtype)
    dg = torch.empty((), device=dev, dtype=torch.float32)
    dw = torch.empty(M, device=dev, dtype=torch.float32)
    doop = operand_copy(dfast, opt)
    dS = bwd_work_buffer(B, T, M, D, precision, dev)
    dqf = torch.empty(B, T, M, device=dev, dtype=torch.float32)
    dk = torch.empty_like(dqf)
    partial = torch.empty(int(L.lib().ulm_memory_stats_bwd_scratch(B, T, M)), device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        L.check(L.lib().ulm_memory_bwd(L.ptr(dq_out), L.ptr(dfast), L.dtype_code(dfast.dtype), L.ptr(r), L.ptr(den),
                                       L.ptr(g), L.ptr(w), L.ptr(q), L.ptr(c) if c.numel() else None, L.ptr(qop),
                                       L.ptr(kop), L.ptr(vop), L.ptr(P),
                                       L.ptr(doop), L.ptr(dS), L.ptr(dqf), L.ptr(dk), L.ptr(partial), L.ptr(dr),
                                       L.ptr(dv), L.ptr(dg), L.ptr(dw), B, T, M, D, precision, L.stream_of(r)))
    return dr, dv, dg, dw


@torch.library.custom_op("ulm::memory_fwd", mutates_args=())
def memory_fwd(r: torch.Tensor, v: torch.Tensor, g: torch.Tensor, w: torch.Tensor, precision: int
               ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                          torch.Tensor]:
    """Returns (q, fast, c, qop, kop, vop, P); the last five are saved for the backward (vop is
    empty when v itself serves as the operand copy)."""
    q, fast, c, qop, kop, vop, P = memory_fwd_raw(r, None, v, g, w, precision)
    return q, fast, c, qop, kop, unaliased(vop, v), P


def unaliased(op, x):
    """An op's output must not alias its input: an empty placeholder when the operand copy is x."""
    return x.new_empty(0) if op.data_ptr() == x.data_ptr() else op


def operand_or_input(op, x):
    """The operand copy saved for a backward: the placeholder stands for the input x itself."""
    return x if op.numel() == 0 else op


@memory_fwd.register_fake
def _memory_fwd_fake(r, v, g, w, precision):
    return memory_fwd_fake(r, v, precision)


@torch.library.custom_op("ulm::memory_bwd", mutates_args=())
def memory_bwd(dq_out: Optional[torch.Tensor], dfast: torch.Tensor, r: torch.Tensor, g: torch.Tensor,
               w: torch.Tensor, q: torch.Tensor, c: torch.Tensor, qop: torch.Tensor, kop: torch.Tensor,
               vop: torch.Tensor, P: torch.Tensor, precision: int
               ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Returns (dr, dv, dg, dw) (kernel.py:216-233)."""
    return memory_bwd_raw(dq_out, dfast, r, None, g, w, q, c, qop, kop, vop, P, precision)


@memory_bwd.register_fake
def _memory_bwd_fake(dq_out, dfast, r, g, w, q, c, qop, kop, vop, P, precision):
    B, T, M = r.shape
    return (r.new_empty(B, T, M, dtype=torch.float32), dfast.new_empty(dfast.shape),
            r.new_empty((), dtype=torch.float32), r.new_empty(M, dtype=torch.float32))


def _setup_context(ctx, inputs, output):
    r, v, g, w, precision = inputs
    q, fast, c, qop, kop, vop, P = output
    ctx.save_for_backward(r, g, w, q, c, qop, kop, operand_or_input(vop, v), P)
    ctx.precision = precision
    ctx.v_dtype = v.dtype
    ctx.v_dim = v.shape[-1]
    ctx.g_shape = g.shape
    ctx.mark_non_differentiable(c, qop, kop, vop, P)
    ctx.set_materialize_grads(False)  # no zero tensors for the outputs nothing differentiates


def _backward(ctx, dq_out, dfast, *unused):
    if dq_out is None and dfast is None:
        return None, None, None, None, None
    r, g, w, q, c, qop, kop, vop, P = ctx.saved_tensors
    if dfast is None:
        dfast = torch.zeros(q.shape[0], q.shape[1], ctx.v_dim, device=q.device, dtype=ctx.v_dtype)
    dr, dv, dg, dw = memory_bwd(None if dq_out is None else dq_out.float().contiguous(), dfast.contiguous(),
                                r, g, w, q, c, qop, kop, vop, P, ctx.precision)
    return dr, dv.to(ctx.v_dtype), dg.reshape(ctx.g_shape), dw, None


torch.library.register_autograd("ulm::memory_fwd", _backward, setup_context=_setup_context)


def unified_memory(r, v, g, w, precision="bf16"):
    """r: (B,T,M) read addresses, v: (B,T,D) values, g: scalar log decay, w: (M,) prior mass.
    Returns (q fp32 (B,T,M), fast (B,T,D) in v's dtype)."""
    prec = PRECISION[precision]
    out_dtype = v.dtype
    vv = v if v.dtype in (torch.float32, torch.bfloat16) else v.float()
    g1 = g.float().reshape(())
    q, fast, *_ = torch.ops.ulm.memory_fwd(r.float().contiguous(), vv.contiguous(), g1,
                                           w.float().contiguous(), prec)
    return q, fast.to(out_dtype)


def combine_fwd_raw(r, den, v, g, w, mu, x, precision):
    """ulm_memory_combine_fwd on fresh buffers: y = x + mu(q w) + fast, plus the tensors saved for
    the backward (q, c, qop, kop, vop, P); q and c are empty when the backward rebuilds them."""
    _require_cuda(r, v, g, w, mu, x, den)
    B, T, M = r.shape
    D = v.shape[-1]
    dev = r.device
    opt = _op_dtype(precision)
    lib = L.lib()
    keep = bool(lib.ulm_memory_needs_c(T, M))
    q = torch.empty(B, T, M, device=dev, dtype=torch.float32) if keep else r.new_empty(0)
    c = torch.empty(B, T, M, device=dev, dtype=torch.float32) if keep else r.new_empty(0)
    y = torch.empty(B, T, D, device=dev, dtype=x.dtype)
    qop = torch.empty(B, T, operand_ld(M), device=dev, dtype=opt)
    kop = torch.empty_like(qop)
    vop = operand_copy(v, opt)
    P = saved_buffer(B, T, M, D, precision, dev)
    wmu = torch.empty(M, operand_ld(D), device=dev, dtype=opt)
    with torch.cuda.device(dev):
        L.check(lib.ulm_memory_combine_fwd(
            L.ptr(r), L.ptr(den), L.ptr(v), L.dtype_code(v.dtype), L.ptr(g), L.ptr(w), L.ptr(mu), L.ptr(x),
            L.dtype_code(x.dtype), L.ptr(y), L.ptr(q) if keep else None, L.ptr(c) if keep else None, L.ptr(qop),
            L.ptr(kop), L.ptr(vop), L.ptr(P), L.ptr(wmu), B, T, M, D, precision, L.stream_of(r)))
    return y, q, c, qop, kop, vop, P


def combine_fwd_fake(r, v, x, precision):
    B, T, M = r.shape
    D = v.shape[-1]
    opt = _op_dtype(precision)
    keep = (B, T, M) if L.lib().ulm_memory_needs_c(T, M) else (0,)
    return (x.new_empty(B, T, D), r.new_empty(keep, dtype=torch.float32), r.new_empty(keep, dtype=torch.float32),
            r.new_empty(B, T, operand_ld(M), dtype=opt), r.new_empty(B, T, operand_ld(M), dtype=opt),
            operand_copy_fake(v, opt),
            r.new_empty(int(L.lib().ulm_memory_saved_bytes(B, T, M, D, precision)), dtype=torch.uint8))


def combine_bwd_raw(dy, r, den, g, w, mu, q, c, qop, kop, vop, P, v_dtype, precision):
    """ulm_memory_combine_bwd on fresh buffers: (dr, dv, dg, dw, dmu)."""
    _require_cuda(dy, r, g, w, mu, den)
    B, T, M = r.shape
    D = dy.shape[-1]
    dev = r.device
    opt = _op_dtype(precision)
    lib = L.lib()
    dr = torch.empty(B, T, M, device=dev, dtype=torch.float32)
    dv = torch.empty(B, T, D, device=dev, dtype=v_dtype)
    dg = torch.empty((), device=dev, dtype=torch.float32)
    dw = torch.empty(M, device=dev, dtype=torch.float32)
    dmu = torch.empty(D, M, device=dev, dtype=torch.float32)
    doop = operand_copy(dy, opt)
    dS = bwd_work_buffer(B, T, M, D, precision, dev)
    mw = torch.empty(D, operand_ld(M), device=dev, dtype=opt)
    dqf = torch.empty(B, T, M, device=dev, dtype=torch.float32)
    dk = torch.empty_like(dqf)
    partial = torch.empty(int(lib.ulm_memory_stats_bwd_scratch(B, T, M)), device=dev, dtype=torch.uint8)
    gpart = torch.empty(int(lib.ulm_combine_grad_scratch(B, T, M, D)), device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        L.check(lib.ulm_memory_combine_bwd(
            L.ptr(dy), L.dtype_code(dy.dtype), L.ptr(r), L.ptr(den), L.ptr(g), L.ptr(w), L.ptr(mu),
            L.ptr(q) if q.numel() else None, L.ptr(c) if c.numel() else None, L.ptr(qop), L.ptr(kop), L.ptr(vop),
            L.ptr(P), L.ptr(doop), L.ptr(dS), L.ptr(mw), L.ptr(dqf), L.ptr(dk), L.ptr(partial), L.ptr(gpart),
            L.ptr(dr), L.ptr(dv), L.dtype_code(v_dtype), L.ptr(dg), L.ptr(dw), L.ptr(dmu), B, T, M, D, precision,
            L.stream_of(r)))
    return dr, dv, dg, dw, dmu
