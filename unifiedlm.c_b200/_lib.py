"""ctypes binding of the C ABI in include/ulm_b200.h (libulm_b200.so, built in-tree).

There is no fallback: if the library is missing or a call fails, the caller gets an exception.
"""
import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libulm_b200.so")

ULM_OK, ULM_ERR_INVALID, ULM_ERR_CUDA, ULM_ERR_UNSUPPORTED, ULM_ERR_DEVICE = range(5)
ULM_F32, ULM_BF16 = 0, 1
ULM_PREC_BF16, ULM_PREC_FP32 = 0, 1

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int

# name -> (restype, argtypes); kept in the order of include/ulm_b200.h
SIGNATURES = {
    "ulm_last_error": (ctypes.c_char_p, []),
    "ulm_version": (_I, []),
    "ulm_device_error": (_I, [ctypes.POINTER(_I)]),
    "ulm_memory_stats_fwd": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _P]),
    "ulm_memory_stats_bwd": (_I, [_P] * 12 + [_I64, _I64, _I64, _P]),
    "ulm_memory_stats_bwd_scratch": (_I64, [_I64, _I64, _I64]),
    "ulm_memory_stats_bwd_noalloc": (_I, [_P] * 11 + [_I64, _I64, _I64, _P]),
    "ulm_memory_needs_c": (_I, [_I64, _I64]),
    "ulm_block_scalars_fwd": (_I, [_P] * 6 + [_I64, _P]),
    "ulm_block_scalars_bwd": (_I, [_P] * 11 + [_I64, _P]),
    "ulm_decayed_scores": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I, _P]),
    "ulm_causal_apply": (_I, [_P, _I64, _P, _I64, _P, _I64, _I, _I, _I64, _I64, _I64, _I, _P]),
    "ulm_operand_ld": (_I64, [_I64]),
    "ulm_set_gemm_pairs": (_I, [_I]),
    "ulm_set_epilogue_mode": (_I, [_I]),
    "ulm_set_scan_mode": (_I, [_I]),
    "ulm_set_pdl": (_I, [_I]),
    "ulm_set_chunk_mode": (_I, [_I]),
    "ulm_memory_chunk_len": (_I, [_I64, _I64, _I64, _I]),
    "ulm_memory_saved_bytes": (_I64, [_I64, _I64, _I64, _I64, _I]),
    "ulm_memory_bwd_work_bytes": (_I64, [_I64, _I64, _I64, _I64, _I]),
    "ulm_memory_fwd": (_I, [_P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I, _P]),
    "ulm_memory_bwd": (_I, [_P, _P, _I] + [_P] * 19 + [_I64, _I64, _I64, _I64, _I, _P]),
    "ulm_memory_combine_fwd": (_I, [_P, _P, _P, _I, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P, _P,
                                    _I64, _I64, _I64, _I64, _I, _P]),
    "ulm_memory_combine_bwd": (_I, [_P, _I] + [_P] * 20 + [_I, _P, _P, _P, _I64, _I64, _I64, _I64, _I, _P]),
    "ulm_combine_grad_scratch": (_I64, [_I64, _I64, _I64, _I64]),
    "ulm_address_fwd": (_I, [_P, _I, _P, _I64, _P, _I64, _P, _P, _P, _P, _I, _P, _P, _I64, _I64, _I64, _I64, _I64,
                             _I, _P]),
    "ulm_address_fwd_work_bytes": (_I64, [_I64, _I64, _I64]),
    "ulm_address_bwd": (_I, [_P, _P, _P, _I, _P, _I64, _P, _I, _P, _I64, _P, _I64, _P, _P, _P, _P, _P, _P,
                             _I64, _I64, _I64, _I64, _I, _P]),
    "ulm_address_bwd_work_bytes": (_I64, [_I64, _I64, _I64, _I64, _I]),
    "ulm_addressed_memory_bwd": (_I, [_P, _P, _I] + [_P] * 19 + [_P, _I64, _P, _I, _P, _I64, _P, _I64] + [_P] * 6 +
                                 [_I64] * 4 + [_I, _P]),
    "ulm_mixer_bwd": (_I, [_P, _I] + [_P] * 20 + [_I, _P, _P, _P] + [_P, _I64, _P, _I, _P, _I64, _P, _I64] +
                      [_P] * 6 + [_I64] * 4 + [_I, _P]),
    "ulm_rms_norm_fwd": (_I, [_P, _I, _P, _P, _I, _P, _I64, _I64, ctypes.c_float, _P]),
    "ulm_rms_norm_bwd": (_I, [_P, _I, _P, _I, _P, _P, _P, _P, _P, _P, _I64, _I64, _P]),
    "ulm_rms_norm_bwd_work_bytes": (_I64, [_I64, _I64]),
    "ulm_linear_fwd": (_I, [_P, _I, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I, _P]),
    "ulm_linear_bwd": (_I, [_P, _I, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I, _P]),
    "ulm_linear_bwd_work_bytes": (_I64, [_I64, _I64, _I64, _I]),
    "ulm_lm_head_loss_fwd": (_I, [_P, _I64, _P, _I64, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I, _P]),
    "ulm_lm_head_loss_bwd": (_I, [_P, _P, _P, _I64, _P, _I64, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I, _P]),
    "ulm_lm_head_work_bytes": (_I64, [_I64, _I64, _I64, _I]),
    "ulm_decode_prepare_block": (_I, [_P, _P, _P, _P, _I, _I64, _I64, _P]),
    "ulm_decode_reset_block": (_I, [_P] * 6 + [_I64] * 4 + [_P]),
    "ulm_decode_block_step": (_I, [_P] * 7 + [_I] + [_P] * 8 + [_I64] * 4 + [ctypes.c_float, _P]),
    "ulm_decode_block_work_bytes": (_I64, [_I64, _I64, _I64]),
    "ulm_decode_embed": (_I, [_P, _P, _I, _P, _I64, _I64, _P]),
    "ulm_decode_head": (_I, [_P, _P, _P, _P, _I, _P, _P, _P, _I64, _I64, _I64, ctypes.c_float, _P]),
    "ulm_decode_sample": (_I, [_P, _I64, _I64, ctypes.c_float, ctypes.c_float, _P, _P, _P, _I, _P, _I64, _P]),
    "ulm_decode_head_work_bytes": (_I64, [_I64, _I64]),
    "ulm_decode_prefill_block": (_I, [_P] * 7 + [_I] + [_P] * 7 + [_I64] * 5 + [_I, _P]),
    "ulm_decode_prefill_work_bytes": (_I64, [_I64, _I64, _I64, _I]),
}

_lib = None


def lib():
    """The loaded library with argument types declared. Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; "
                               f"g.build()'` (nvcc, sm_100a)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


class UlmError(RuntimeError):
    pass


def check(rc):
    if rc != ULM_OK:
        msg = lib().ulm_last_error().decode(errors="replace")
        raise UlmError(f"libulm_b200 status {rc}: {msg}")


def ptr(t):
    """Device (or host) address of a tensor, or NULL for None."""
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def dtype_code(dtype):
    if dtype == torch.float32:
        return ULM_F32
    if dtype == torch.bfloat16:
        return ULM_BF16
    raise UlmError(f"unsupported element type {dtype}")


def device_error():
    """Synchronise and read/clear the device-side error flag (0 = none)."""
    site = _I(0)
    check(lib().ulm_device_error(ctypes.byref(site)))
    return site.value
