"""Parity of the sm_100a fast-memory operator with the float64 CPU oracle.

bf16 precision (tensor-core products, bf16 operands, fp32 accumulation): relative error of q,
fast, dr, dv and dw below 1e-2, the reference kernel's bar (test_all.py:140-166). The decay
gradient dg is a single scalar that, on random inputs, is a sum of ~1e5 terms cancelling to about
1/500 of their absolute sum; rounding the operands to bf16 alone (any kernel that takes bf16
operands, the reference's included) moves it by ~1e-2 relative, which is the operator-level dlam
error the reference publishes (up to 1.7e-2, docs/kernel.md:32). Its operator-level bound is
therefore 3e-2; the model-level test (test_model_gpu.py) holds every parameter gradient, log_rate
included, to 1e-2.
fp32 precision: every output below 1e-5, the 1e-5 parity mode.
Relative error = ||x - x_ref|| / ||x_ref|| over the whole tensor.
"""
import ctypes
import os

import pytest
import torch

import unifiedlm_c_b200._lib as L
from oracle import memory as O
from unifiedlm_c_b200.kernel import unified_memory, operand_ld

pytestmark = pytest.mark.gpu

TOL = {"bf16": 1e-2, "fp32": 1e-5}
DG_TOL = {"bf16": 3e-2, "fp32": 1e-5}
DEV = "cuda:0"


def check(errs, precision):
    dg = errs.pop("dg")
    assert dg < DG_TOL[precision], ("dg", dg, errs)
    assert max(errs.values()) < TOL[precision], errs


def make_inputs(B, T, M, D, lam=0.95, seed=0):
    g_ = torch.Generator().manual_seed(seed)
    a = torch.randn(B, T, M, generator=g_, dtype=torch.float64) + 0.3
    z = torch.relu(a).square()
    r = z / (1.0 + z.sum(-1, keepdim=True))
    v = torch.randn(B, T, D, generator=g_, dtype=torch.float64)
    g = torch.tensor(float(torch.log(torch.tensor(lam))), dtype=torch.float64)
    w = torch.exp(torch.randn(M, generator=g_, dtype=torch.float64))
    dq_out = torch.randn(B, T, M, generator=g_, dtype=torch.float64)
    dfast = torch.randn(B, T, D, generator=g_, dtype=torch.float64)
    return r, v, g, w, dq_out, dfast


def rel(x, ref):
    ref = ref.double().cpu()
    return float((x.detach().double().cpu() - ref).norm() / ref.norm().clamp(min=1e-30))


def run_gpu(r, v, g, w, dq_out, dfast, precision, v_dtype=torch.float32, use_dq=True):
    leaves = [r.float().to(DEV), v.to(v_dtype).to(DEV), g.float().to(DEV), w.float().to(DEV)]
    for t in leaves:
        t.requires_grad_(True)
    q, fast = unified_memory(*leaves, precision=precision)
    loss = (fast.float() * dfast.float().to(DEV)).sum()
    if use_dq:
        loss = loss + (q * dq_out.float().to(DEV)).sum()
    loss.backward()
    torch.cuda.synchronize()
    return q, fast, [t.grad for t in leaves]


SHAPES = [
    (1, 40, 48, 32),      # tiny, partial tiles everywhere
    (2, 200, 140, 64),    # the reference's kernel test shape (T not a multiple of 64, M of 8)
    (2, 70, 20, 24),      # the golden fixture's shape
    (8, 512, 256, 64),    # BASELINE config 1 (260K op)
    (2, 384, 1024, 512),  # 42M op shape, short T
]


@pytest.mark.parametrize("precision", ["bf16", "fp32"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_memory_matches_oracle(shape, precision):
    r, v, g, w, dq_out, dfast = make_inputs(*shape)
    q, fast, grads = run_gpu(r, v, g, w, dq_out, dfast, precision)
    q_ref, fast_ref = O.memory_dense(r, v, g, w)
    refs = O.memory_grads(r, v, g, w, dq_out, dfast, form="dense")
    errs = {"q": rel(q, q_ref), "fast": rel(fast, fast_ref)}
    errs.update({n: rel(gr, rf) for n, gr, rf in zip(("dr", "dv", "dg", "dw"), grads, refs)})
    check(errs, precision)
    assert L.device_error() == 0


@pytest.mark.parametrize("lam", [0.9, 0.99, 0.999])
def test_decay_sweep_bf16(lam):
    r, v, g, w, dq_out, dfast = make_inputs(2, 512, 512, 128, lam=lam, seed=1)
    q, fast, grads = run_gpu(r, v, g, w, dq_out, dfast, "bf16")
    q_ref, fast_ref = O.memory_dense(r, v, g, w)
    refs = O.memory_grads(r, v, g, w, dq_out, dfast, form="dense")
    errs = {"q": rel(q, q_ref), "fast": rel(fast, fast_ref)}
    errs.update({n: rel(gr, rf) for n, gr, rf in zip(("dr", "dv", "dg", "dw"), grads, refs)})
    check(errs, "bf16")


def test_golden_fixture(golden_dir):
    f = torch.load(os.path.join(golden_dir, "memory_op.pt"), weights_only=False)
    for precision in ("bf16", "fp32"):
        q, fast, grads = run_gpu(f["r"], f["v"], f["g"], f["w"], f["dq_out"], f["dfast"], precision)
        errs = {"q": rel(q, f["q"]), "fast": rel(fast, f["fast"])}
        errs.update({n: rel(gr, f[n]) for n, gr in zip(("dr", "dv", "dg", "dw"), grads)})
        check(errs, precision)


@pytest.mark.parametrize("shape", [(0, 16, 32, 24), (2, 0, 32, 24), (2, 16, 0, 24), (2, 16, 8, 0)],
                         ids=["no_rows", "no_positions", "no_slots", "no_channels"])
def test_empty_extents(shape):
    """Empty batches and sequences (and the degenerate no-slot / no-channel shapes) give outputs and
    gradients of the right shapes: zero where the sums are empty, the oracle's values elsewhere."""
    r, v, g, w, dq_out, dfast = make_inputs(*shape)
    q, fast, grads = run_gpu(r, v, g, w, dq_out, dfast, "fp32")
    q_ref, fast_ref = O.memory_dense(r, v, g, w)
    refs = O.memory_grads(r, v, g, w, dq_out, dfast, form="dense")
    assert q.shape == q_ref.shape and fast.shape == fast_ref.shape
    for gr, rf in zip(grads, refs):
        assert gr.shape == rf.shape
    for x, ref in [(q.detach(), q_ref), (fast.detach(), fast_ref)] + list(zip(grads, refs)):
        if ref.numel() and float(ref.abs().max()) == 0.0:
            assert float(x.abs().max()) == 0.0
        elif ref.numel():
            assert rel(x, ref) < 1e-5
    assert L.device_error() == 0


def test_without_q_gradient_and_bf16_values():
    r, v, g, w, dq_out, dfast = make_inputs(2, 200, 140, 64, seed=3)
    q, fast, grads = run_gpu(r, v, g, w, dq_out, dfast, "bf16", v_dtype=torch.bfloat16, use_dq=False)
    assert fast.dtype == torch.bfloat16 and grads[1].dtype == torch.bfloat16
    refs = O.memory_grads(r, v.bfloat16().double(), g, w, None, dfast, form="dense")
    _, fast_ref = O.memory_dense(r, v.bfloat16().double(), g, w)
    assert rel(fast, fast_ref) < 1e-2
    errs = {n: rel(gr, rf) for n, gr, rf in zip(("dr", "dv", "dg", "dw"), grads, refs)}
    check(errs, "bf16")


def test_products_against_torch():
    """ulm_decayed_scores / ulm_causal_apply through the C ABI against torch fp32 math."""
    torch.manual_seed(0)
    B, T, K, V = 3, 300, 200, 96
    lib = L.lib()
    a = torch.randn(B, T, K, device=DEV)
    b = torch.randn(B, T, K, device=DEV)
    c = torch.randn(B, T, V, device=DEV)
    g = torch.tensor([-0.03], device=DEV)
    t = torch.arange(T, device=DEV, dtype=torch.float32)
    Dm = torch.where(t[:, None] >= t[None, :], torch.exp(g * (t[:, None] - t[None, :])), torch.zeros(()))
    ld_k, ld_t, ld_v = operand_ld(K), operand_ld(T), operand_ld(V)
    a16 = torch.zeros(B, T, ld_k, device=DEV, dtype=torch.bfloat16)
    b16 = torch.zeros_like(a16)
    c16 = torch.zeros(B, T, ld_v, device=DEV, dtype=torch.bfloat16)
    a16[..., :K], b16[..., :K], c16[..., :V] = a, b, c
    P = torch.zeros(B, T, ld_t, device=DEV, dtype=torch.bfloat16)
    st = L.stream_of(a)
    L.check(lib.ulm_decayed_scores(L.ptr(a16), ld_k, L.ptr(b16), ld_k, L.ptr(P), ld_t, L.ptr(g), B, T, K,
                                   L.ULM_PREC_BF16, st))
    ref_P = (a16[..., :K].float() @ b16[..., :K].float().transpose(1, 2)) * Dm
    assert rel(P[..., :T].float(), ref_P) < 5e-3
    for transpose in (0, 1):
        o = torch.empty(B, T, V, device=DEV)
        L.check(lib.ulm_causal_apply(L.ptr(P), ld_t, L.ptr(c16), ld_v, L.ptr(o), V, L.ULM_F32, transpose, B, T, V,
                                     L.ULM_PREC_BF16, st))
        Pf = P[..., :T].float()
        ref = (Pf.transpose(1, 2) if transpose else Pf) @ c16[..., :V].float()
        assert rel(o, ref) < 1e-4, transpose
    torch.cuda.synchronize()
    assert L.device_error() == 0


def test_full_size_properties():
    """At the 110M shape (B=16, T=1024, M=2048, D=768): linearity of fast in v, exact causality,
    determinism, and one batch row against the oracle."""
    B, T, M, D = 16, 1024, 2048, 768
    torch.manual_seed(0)
    a = torch.randn(B, T, M, device=DEV) + 0.3
    z = torch.relu(a).square()
    r = z / (1.0 + z.sum(-1, keepdim=True))
    v1 = torch.randn(B, T, D, device=DEV)
    v2 = torch.randn(B, T, D, device=DEV)
    g = torch.tensor(-0.05, device=DEV)
    w = torch.full((M,), 4.0, device=DEV)
    q, f1 = unified_memory(r, v1, g, w)
    _, f2 = unified_memory(r, v2, g, w)
    _, f12 = unified_memory(r, v1 + v2, g, w)
    assert rel(f12, f1 + f2) < 1e-2
    _, f1b = unified_memory(r, v1, g, w)
    assert torch.equal(f1, f1b)  # deterministic
    v3 = v1.clone()
    v3[:, 700:] = torch.randn(B, T - 700, D, device=DEV)
    _, f3 = unified_memory(r, v3, g, w)
    assert torch.equal(f3[:, :700], f1[:, :700])  # nothing leaks backwards in time
    q_ref, fast_ref = O.memory_dense(r[:1].double().cpu(), v1[:1].double().cpu(), g.double().cpu(),
                                     w.double().cpu())
    assert rel(q[:1], q_ref) < 1e-5 and rel(f1[:1], fast_ref) < 1e-2
    assert L.device_error() == 0


@pytest.mark.parametrize("T", [37, 1500, 2500, 4200])
def test_stats_kernels_through_c_abi(T):
    """ulm_memory_stats_fwd / ulm_memory_stats_bwd (the reference's K1 / K5 interface, with the dg
    identity) against the oracle, on both the register-resident and the two-pass scan paths."""
    B, M, D = (2 if T < 4096 else 1), 40, 16   # T > 4096 runs the two-pass fallback scans
    r, v, g, w, dq_out, dfast = make_inputs(B, T, M, D, lam=0.99, seed=7)
    k, c_ref, q_ref = O.memory_stats(r, g, w)
    Dm = O.decay_matrix(T, g)
    dS = (dfast @ v.transpose(1, 2)) * Dm
    dqf_ref, dk_ref = dS @ k, dS.transpose(1, 2) @ q_ref
    dr_ref, _, dg_ref, dw_ref = O.memory_grads(r, v, g, w, dq_out, dfast, form="dense")
    lib = L.lib()
    cu = lambda x: x.float().to(DEV).contiguous()  # noqa: E731
    rr, gg, ww = cu(r), cu(g).reshape(1), cu(w)
    q = torch.empty(B, T, M, device=DEV)
    c = torch.empty_like(q)
    qop = torch.empty(B, T, operand_ld(M), device=DEV)
    kop = torch.empty_like(qop)
    st = L.stream_of(q)
    L.check(lib.ulm_memory_stats_fwd(L.ptr(rr), L.ptr(ww), L.ptr(gg), L.ptr(q), L.ptr(c), L.ptr(qop), L.ptr(kop),
                                     L.ULM_F32, operand_ld(M), B, T, M, st))
    torch.cuda.synchronize()
    assert rel(q, q_ref) < 1e-5 and rel(c, c_ref) < 1e-5
    assert torch.equal(qop[..., :M], q)
    assert torch.equal(kop[:, 1:, :M], rr[:, :-1]) and not kop[:, 0, :M].any()
    dr = torch.empty_like(q)
    dw = torch.empty(M, device=DEV)
    dg = torch.empty(1, device=DEV)
    part = torch.empty(int(lib.ulm_memory_stats_bwd_scratch(B, T, M)), device=DEV, dtype=torch.uint8)
    dqf_d, dqo_d, dk_d = cu(dqf_ref), cu(dq_out), cu(dk_ref)  # keep the device copies alive across the call
    L.check(lib.ulm_memory_stats_bwd(L.ptr(dqf_d), L.ptr(dqo_d), L.ptr(dk_d), L.ptr(q), L.ptr(c),
                                     L.ptr(rr), L.ptr(ww), L.ptr(gg), L.ptr(dr), L.ptr(dw), L.ptr(dg), L.ptr(part),
                                     B, T, M, st))
    torch.cuda.synchronize()
    assert rel(dr, dr_ref) < 1e-5 and rel(dw, dw_ref) < 1e-5, (rel(dr, dr_ref), rel(dw, dw_ref))
    assert rel(dg, dg_ref.reshape(1)) < 1e-4, rel(dg, dg_ref.reshape(1))
    # without the saved q and c: rebuilt from r where the TMA scans apply, refused elsewhere
    dr2, dw2, dg2 = torch.empty_like(dr), torch.empty_like(dw), torch.empty_like(dg)
    rc = lib.ulm_memory_stats_bwd(L.ptr(dqf_d), L.ptr(dqo_d), L.ptr(dk_d), None, None, L.ptr(rr), L.ptr(ww),
                                  L.ptr(gg), L.ptr(dr2), L.ptr(dw2), L.ptr(dg2), L.ptr(part), B, T, M, st)
    if lib.ulm_memory_needs_c(T, M):
        assert rc == L.ULM_ERR_INVALID
    else:
        L.check(rc)
        torch.cuda.synchronize()
        assert rel(dr2, dr) < 1e-6 and rel(dw2, dw) < 1e-6 and rel(dg2, dg) < 1e-6
    assert L.device_error() == 0


@pytest.mark.parametrize("kind", ["scores", "read", "read_t"])
def test_pair_and_single_cta_products_agree(kind):
    """The 2-SM (CTA pair) and single-CTA tensor-core kernels compute the same products."""
    torch.manual_seed(1)
    B, T, K, V = 2, 640, 384, 512
    lib = L.lib()
    ldk, ldt, ldv = operand_ld(K), operand_ld(T), operand_ld(V)
    a = torch.randn(B, T, ldk, device=DEV).bfloat16()
    b = torch.randn(B, T, ldk, device=DEV).bfloat16()
    c = torch.randn(B, T, ldv, device=DEV).bfloat16()
    g = torch.tensor([-0.01], device=DEV)
    outs = []
    for pairs in (1, 0):
        old = lib.ulm_set_gemm_pairs(pairs)
        try:
            P = torch.zeros(B, T, ldt, device=DEV, dtype=torch.bfloat16)
            st = L.stream_of(P)
            L.check(lib.ulm_decayed_scores(L.ptr(a), ldk, L.ptr(b), ldk, L.ptr(P), ldt, L.ptr(g), B, T, K,
                                           L.ULM_PREC_BF16, st))
            if kind == "scores":
                outs.append(P[..., :T].float())
            else:
                o = torch.empty(B, T, V, device=DEV)
                L.check(lib.ulm_causal_apply(L.ptr(P), ldt, L.ptr(c), ldv, L.ptr(o), V, L.ULM_F32,
                                             1 if kind == "read_t" else 0, B, T, V, L.ULM_PREC_BF16, st))
                outs.append(o)
            torch.cuda.synchronize()
        finally:
            lib.ulm_set_gemm_pairs(old)
    assert rel(outs[0], outs[1].double().cpu()) < 1e-6
    t = torch.arange(T, device=DEV, dtype=torch.float32)
    Dm = torch.where(t[:, None] >= t[None, :], torch.exp(g * (t[:, None] - t[None, :])), torch.zeros(()))
    ref = (a[..., :K].float() @ b[..., :K].float().transpose(1, 2)) * Dm
    if kind == "scores":
        assert rel(outs[0], ref.double().cpu()) < 5e-3
    assert L.device_error() == 0


@pytest.mark.parametrize("shape", [(3, 1000, 200), (16, 1024, 2048), (5, 300, 68), (1, 128, 36)],
                         ids=lambda s: "x".join(map(str, s)))
def test_scan_modes_agree(shape):
    """The persistent pipelined scans (ulm_set_scan_mode(1), the default) and the one-cluster-per-item
    scans compute the same q, c, operand copies, dr, dw and dg, with and without dq_out. The
    pipelined kernels give each thread two slots of half a warp's rows and join the two halves'
    partial sums with lam^8, the per-item kernels chain a warp's 16 rows directly, so the fp32 results
    agree to rounding: within 1e-5 of the array's largest magnitude (measured differences are ~1e-7
    relative), and the bf16 copy of q within one bf16 step where the fp32 q values straddle a
    rounding boundary."""
    B, T, M = shape
    gen = torch.Generator().manual_seed(B * T + M)
    a = torch.randn(B, T, M, generator=gen) + 0.3
    z = torch.relu(a).square()
    r = (z / (1.0 + z.sum(-1, keepdim=True))).to(DEV)
    w = torch.exp(torch.randn(M, generator=gen)).to(DEV)
    g = torch.tensor([-0.03], device=DEV)
    dqf = torch.randn(B, T, M, generator=gen).to(DEV)
    dqo = torch.randn(B, T, M, generator=gen).to(DEV)
    dk = torch.randn(B, T, M, generator=gen).to(DEV)
    lib = L.lib()
    ldo = operand_ld(M)
    st = L.stream_of(r)
    part = torch.empty(int(lib.ulm_memory_stats_bwd_scratch(B, T, M)), device=DEV, dtype=torch.uint8)
    res = {}
    for mode in (0, 1):
        old = lib.ulm_set_scan_mode(mode)
        try:
            q, c = torch.empty(B, T, M, device=DEV), torch.empty(B, T, M, device=DEV)
            qop = torch.empty(B, T, ldo, device=DEV, dtype=torch.bfloat16)
            kop = torch.empty_like(qop)
            L.check(lib.ulm_memory_stats_fwd(L.ptr(r), L.ptr(w), L.ptr(g), L.ptr(q), L.ptr(c), L.ptr(qop), L.ptr(kop),
                                             L.ULM_BF16, ldo, B, T, M, st))
            outs = [q, c, qop[..., :M].float(), kop[..., :M].float()]
            for dq_out in (dqo, None):
                dr, dw, dg = torch.empty(B, T, M, device=DEV), torch.empty(M, device=DEV), torch.empty(1, device=DEV)
                L.check(lib.ulm_memory_stats_bwd(L.ptr(dqf), L.ptr(dq_out) if dq_out is not None else None, L.ptr(dk),
                                                 None, None, L.ptr(r), L.ptr(w), L.ptr(g), L.ptr(dr), L.ptr(dw),
                                                 L.ptr(dg), L.ptr(part), B, T, M, st))
                torch.cuda.synchronize()
                outs += [dr.clone(), dw.clone(), dg.clone()]
            res[mode] = outs
        finally:
            lib.ulm_set_scan_mode(old)
    names = ["q", "c", "qop", "kop", "dr", "dw", "dg", "dr0", "dw0", "dg0"]
    for name, x0, x1 in zip(names, res[0], res[1]):
        if name.startswith("dg"):
            assert abs(float(x0) - float(x1)) <= 1e-5 * abs(float(x0)) + 1e-12, (name, float(x0), float(x1))
        elif name == "kop":  # r shifted by one position: no scan arithmetic
            assert torch.equal(x0, x1)
        elif name == "qop":
            assert ((x0 - x1).abs() <= x0.abs() * 2.0 ** -7).all(), (name, float((x0 - x1).abs().max()))
        else:
            err = float((x0 - x1).abs().max())
            assert err <= 1e-5 * float(x0.abs().max()) + 1e-30, (name, err, float(x0.abs().max()))
    assert L.device_error() == 0
