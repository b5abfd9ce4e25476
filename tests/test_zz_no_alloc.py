"""The statistics backward that allocates nothing (ulm_memory_stats_bwd_noalloc).

It exists for hosts that cannot give this library device memory when they call it, such as a
serving runtime that reserves all of HBM for its own pool at start-up, or a plugin host that owns
every device allocation. Instead of caller scratch it uses a fixed block compiled into the library.
This file is collected last so that a run stopping at its first failure has run every other test;
it also passes on its own in a fresh process.
"""
import ctypes

import pytest
import torch

import unifiedlm_c_b200._lib as L
from unifiedlm_c_b200.kernel import operand_ld

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def inputs(B, T, M, seed, dev=DEV):
    g_ = torch.Generator(device=dev).manual_seed(seed)
    mk = lambda: torch.randn(B, T, M, device=dev, generator=g_)  # noqa: E731
    r = torch.rand(B, T, M, device=dev, generator=g_) / max(M, 1)
    q = torch.rand(B, T, M, device=dev, generator=g_) / max(M, 1)
    c = 1.0 + torch.rand(B, T, M, device=dev, generator=g_)
    w = torch.full((M,), 4.0, device=dev)
    g = torch.tensor([-0.02], device=dev)
    return dict(dqf=mk(), dq_out=mk(), dk=mk(), q=q, c=c, r=r, w=w, g=g)


def run(lib, x, B, T, M, noalloc, dev=DEV):
    # outputs start as nan so that a result the call does not write shows up
    dr = torch.full((B, T, M), float("nan"), device=dev)
    dw = torch.full((M,), float("nan"), device=dev)
    dg = torch.full((1,), float("nan"), device=dev)
    args = [L.ptr(x[k]) for k in ("dqf", "dq_out", "dk", "q", "c", "r", "w", "g")] + [L.ptr(dr), L.ptr(dw), L.ptr(dg)]
    with torch.cuda.device(dev):
        st = L.stream_of(dr)
        if noalloc:
            L.check(lib.ulm_memory_stats_bwd_noalloc(*args, B, T, M, st))
        else:
            part = torch.empty(int(lib.ulm_memory_stats_bwd_scratch(B, T, M)), device=dev, dtype=torch.uint8)
            L.check(lib.ulm_memory_stats_bwd(*args, L.ptr(part), B, T, M, st))
        torch.cuda.synchronize()
    return dr, dw, dg


def rel(a, b):
    return float((a - b).norm() / b.norm().clamp(min=1e-30))


def test_noalloc_matches_stats_bwd_twice_in_a_row():
    lib = L.lib()
    for (B, T, M, seed) in ((4, 300, 256, 1), (16, 1024, 2048, 2)):   # two calls, the second reuses the block
        x = inputs(B, T, M, seed)
        ref = run(lib, x, B, T, M, noalloc=False)
        got = run(lib, x, B, T, M, noalloc=True)
        for a, b in zip(got, ref):
            assert rel(a, b) < 1e-6
    assert L.device_error() == 0


def test_noalloc_rejects_sizes_beyond_its_block():
    lib = L.lib()
    dummy = ctypes.c_void_p(16)
    rc = lib.ulm_memory_stats_bwd_noalloc(*([dummy] * 11), 64, 16, 8192, None)
    assert rc == L.ULM_ERR_INVALID
    assert b"scratch" in lib.ulm_last_error()


def test_noalloc_empty_extent_zeroes_dw_dg_like_stats_bwd():
    # T = 0 with a B x M far beyond the block: nothing to compute, dw and dg are zeroed, as the
    # allocating call does for the same arguments
    lib = L.lib()
    B, T, M = 512, 0, 4096
    x = inputs(B, T, M, 3)
    got = run(lib, x, B, T, M, noalloc=True)
    ref = run(lib, x, B, T, M, noalloc=False)
    for a, b in zip(got[1:], ref[1:]):
        assert torch.equal(a, b)
        assert torch.count_nonzero(a) == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two visible GPUs")
def test_noalloc_second_device_after_first():
    # the block's address is looked up per context: a call on cuda:1 after cuda:0 uses cuda:1's
    lib = L.lib()
    B, T, M = 4, 300, 256
    for dev in ("cuda:0", "cuda:1", "cuda:0"):
        x = inputs(B, T, M, 4, dev=dev)
        ref = run(lib, x, B, T, M, noalloc=False, dev=dev)
        got = run(lib, x, B, T, M, noalloc=True, dev=dev)
        for a, b in zip(got, ref):
            assert rel(a, b) < 1e-6
    assert L.device_error() == 0
