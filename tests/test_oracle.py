"""The CPU oracle pinned against the reference's own outputs (tests/golden/, made by
tests/golden/make_golden.py from the reference's test_all.py / model.py / run.c), plus the
reference's self-consistency checks (test_all.py:100-137) restated on the oracle."""
import os

import torch

from oracle import memory as O

TOL = 1e-8


def load(golden_dir, name):
    return torch.load(os.path.join(golden_dir, name), weights_only=False)


def test_memory_op_matches_reference_chunked_and_dense(golden_dir):
    f = load(golden_dir, "memory_op.pt")
    for fn in (lambda: O.memory_chunked(f["r"], f["v"], f["g"], f["w"], 64),
               lambda: O.memory_dense(f["r"], f["v"], f["g"], f["w"])):
        q, fast = fn()
        assert (q - f["q"]).abs().max() < 1e-12
        assert (fast - f["fast"]).abs().max() < 1e-12
        assert (q - f["q_dense"]).abs().max() < 1e-12
        assert (fast - f["fast_dense"]).abs().max() < 1e-12


def test_memory_grads_match_reference(golden_dir):
    f = load(golden_dir, "memory_op.pt")
    for form in ("chunked", "dense"):
        dr, dv, dg, dw = O.memory_grads(f["r"], f["v"], f["g"], f["w"], f["dq_out"], f["dfast"], form=form)
        for got, ref in ((dr, f["dr"]), (dv, f["dv"]), (dg, f["dg"]), (dw, f["dw"])):
            assert ((got - ref).norm() / ref.norm()) < 1e-10, form


def test_stats_match_chunked_q(golden_dir):
    f = load(golden_dir, "memory_op.pt")
    k, c, q = O.memory_stats(f["r"], f["g"], f["w"])
    assert (q - f["q"]).abs().max() < 1e-12
    assert (k[:, 1:] - f["r"][:, :-1]).abs().max() == 0 and k[:, 0].abs().max() == 0


def _params(sd):
    return {k: v.clone() for k, v in sd.items()}


def test_model_forward_and_grads_match_reference(golden_dir):
    f = load(golden_dir, "model_tiny.pt")
    p = {k: v.clone().requires_grad_(True) for k, v in f["state_dict"].items()}
    # the classifier is tied to the embedding in the reference: one parameter, gradient summed
    p["output.weight"] = p["tok_embeddings.weight"]
    logits, loss = O.lm_forward(p, f["tokens"], f["tokens"], form="chunked", chunk=64)
    assert (logits - f["logits"]).abs().max() < 1e-10
    # the reference computes its cross-entropy in fp32 (test_all.py:74)
    assert abs(loss.item() - f["loss"].item()) / abs(f["loss"].item()) < 1e-6
    loss.backward()
    for name, ref in f["grads"].items():
        got = p[name].grad
        assert ((got - ref).norm() / ref.norm().clamp(min=1e-30)) < 1e-5, name


def test_forward_recurrent_matches_reference(golden_dir):
    f = load(golden_dir, "model_tiny.pt")
    p = _params(f["state_dict"])
    n = f["recurrent_len"]
    rec = O.lm_forward_recurrent(p, f["tokens"][:, :n])
    assert (rec - f["recurrent_logits"]).abs().max() < 1e-10


def test_greedy_decode_matches_reference_runc(golden_dir):
    f = load(golden_dir, "runc_tiny.pt")
    p = _params(f["state_dict"])
    ids = O.greedy_decode(p, steps=len(f["ids"]))
    assert ids == f["ids"].tolist()


# --- the reference's own consistency tests, on the oracle (test_all.py:100-137) ---------------

def tiny_params(seed=0, dim=32, n_layers=3, hidden=48, vocab=97):
    g = torch.Generator().manual_seed(seed)
    p = {"tok_embeddings.weight": torch.randn(vocab, dim, generator=g, dtype=torch.float64) * 0.02,
         "norm.weight": torch.ones(dim, dtype=torch.float64)}
    p["output.weight"] = p["tok_embeddings.weight"]
    for i in range(n_layers):
        pre = f"layers.{i}."
        p[pre + "norm.weight"] = torch.ones(dim, dtype=torch.float64)
        p[pre + "conv.weight"] = torch.randn(dim, 1, 4, generator=g, dtype=torch.float64) * 0.5
        p[pre + "key.weight"] = torch.randn(hidden, dim, generator=g, dtype=torch.float64) * 0.02
        p[pre + "key.bias"] = torch.randn(hidden, generator=g, dtype=torch.float64) * 0.5
        p[pre + "mu.weight"] = torch.randn(dim, hidden, generator=g, dtype=torch.float64) * 0.02
        p[pre + "val.weight"] = torch.randn(dim, dim, generator=g, dtype=torch.float64) * 0.2
        p[pre + "log_eps"] = torch.zeros((), dtype=torch.float64)
        p[pre + "log_rate"] = torch.tensor(torch.log(torch.tensor(0.05)).item(), dtype=torch.float64)
        p[pre + "log_w"] = torch.randn(hidden, generator=g, dtype=torch.float64)
    return p


def test_chunked_equals_dense():
    p = tiny_params()
    x = torch.randint(0, 97, (3, 40), generator=torch.Generator().manual_seed(1))
    a, _ = O.lm_forward(p, x, form="chunked", chunk=7)
    b, _ = O.lm_forward(p, x, form="dense")
    assert (a - b).abs().max() < TOL


def test_parallel_equals_recurrent():
    p = tiny_params()
    x = torch.randint(0, 97, (3, 40), generator=torch.Generator().manual_seed(2))
    a, _ = O.lm_forward(p, x, form="chunked", chunk=16)
    assert (a - O.lm_forward_recurrent(p, x)).abs().max() < TOL


def test_causality():
    p = tiny_params()
    g = torch.Generator().manual_seed(3)
    x = torch.randint(0, 97, (3, 40), generator=g)
    x2 = x.clone()
    x2[:, 25:] = torch.randint(0, 97, (3, 15), generator=g)
    a, _ = O.lm_forward(p, x, form="chunked", chunk=7)
    b, _ = O.lm_forward(p, x2, form="chunked", chunk=7)
    assert (a[:, :25] - b[:, :25]).abs().max() < TOL


def test_gradients_finite():
    p = {k: v.clone().requires_grad_(True) for k, v in tiny_params().items()}
    p["output.weight"] = p["tok_embeddings.weight"]
    x = torch.randint(0, 97, (3, 40), generator=torch.Generator().manual_seed(4))
    _, loss = O.lm_forward(p, x, x, form="chunked", chunk=7)
    loss.backward()
    for name, t in p.items():
        assert t.grad is not None and torch.isfinite(t.grad).all(), name


def test_sampler_restatement_matches_runc_fixture(golden_dir):
    """oracle.sampler (run.c's sample() restated) on the oracle's recurrent model reproduces the
    token ids the reference's run.c printed with sampling on (temperature > 0, top-p and plain
    multinomial, fixed seeds)."""
    from oracle import sampler as S
    base = torch.load(os.path.join(golden_dir, "runc_tiny.pt"), weights_only=False)
    runs = torch.load(os.path.join(golden_dir, "runc_sampled.pt"), weights_only=False)["runs"]
    params = {k: v.double() for k, v in base["state_dict"].items()}
    for run in runs:
        ids, margin = S.sampled_decode(params, run["steps"], run["temperature"], run["topp"], run["seed"])
        assert ids == run["ids"].tolist(), (run["temperature"], run["topp"], run["seed"], margin)


def test_xorshift_matches_published_sequence():
    """The generator's first outputs from seed 42 (xorshift64* with the (12, 25, 27) shifts)."""
    from oracle import sampler as S
    st, outs = 42, []
    for _ in range(3):
        st, u = S.xorshift_next(st)
        outs.append(u)
    # recomputed independently with Python's arbitrary-precision integers
    ref, s = [], 42
    for _ in range(3):
        s ^= s >> 12
        s ^= (s << 25) % (1 << 64)
        s ^= s >> 27
        ref.append((s * 0x2545F4914F6CDD1D % (1 << 64)) >> 32)
    assert outs == ref
