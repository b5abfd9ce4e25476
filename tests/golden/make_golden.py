"""Generate the golden fixtures in this folder from the reference implementation itself.

Run where the reference checkout is present (its directory in ULM_REFERENCE_DIR, else a `reference`
directory beside this repository):

    python tests/golden/make_golden.py

It imports the reference's own `model.py` / `test_all.py` (pure-PyTorch float64 forms) and runs
the reference's C decoder built by `make -C oracle` (oracle/_ref/run), and writes small `.pt`
fixtures. The tests load only the fixtures; nothing at test time reads the reference checkout.

Fixtures:
  memory_op.pt  : the fast-memory operator on a ragged shape (T=70 over chunk 64): inputs r, v,
                  g, w and upstream gradients; outputs q, fast from the reference's chunkwise
                  form (test_all.chunked_mix, chunk 64) and quadratic form (test_all.dense_mix);
                  gradients dr, dv, dg, dw by float64 autograd through chunked_mix.
  model_tiny.pt : a reference tiny_model (test_all.tiny_model) state_dict in float64, tokens,
                  reference_forward(chunked(64)) logits and loss, every parameter gradient, and
                  forward_recurrent logits.
  runc_tiny.pt  : the model of test_all.test_runc (fp32), and the greedy token ids that the
                  reference's run.c prints for it from BOS, read through a vocabulary whose
                  pieces are "|<id>" so the text maps back to ids.
  runc_sampled.pt: run.c's sampled token ids for the same model from BOS (temperature > 0, top-p
                  and plain multinomial, fixed seeds). `python make_golden.py --sampled` writes only
                  this file (it needs runc_tiny.pt and oracle/_ref/run, not the reference's Python).
"""
import os
import subprocess
import sys
import tempfile

import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("ULM_REFERENCE_DIR") or os.path.normpath(os.path.join(REPO, os.pardir, "reference"))


def load_reference():
    sys.path.insert(0, REF)
    import model as ref_model  # noqa: E402
    import test_all as ref_tests  # noqa: E402
    return ref_model, ref_tests


def memory_op_fixture(ref_model, ref_tests):
    torch.manual_seed(1234)
    B, T, M, D = 2, 70, 20, 24          # D >= M so mu = [I; 0] exposes q * w directly
    args = ref_model.ModelArgs(dim=D, n_layers=1, hidden_dim=M, vocab_size=16, max_seq_len=T)
    block = ref_model.UnifiedBlock(args).double()
    with torch.no_grad():
        block.log_rate.fill_(torch.log(torch.tensor(0.08)).item())   # lam = exp(-0.08)
        block.log_w.normal_(std=1.0)
    a = torch.randn(B, T, M, dtype=torch.float64) + 0.3
    z = F.relu(a).square()
    r0 = (z / (1.0 + z.sum(-1, keepdim=True))).detach()
    v0 = torch.randn(B, T, D, dtype=torch.float64)
    dq_out = torch.randn(B, T, M, dtype=torch.float64)
    dfast = torch.randn(B, T, D, dtype=torch.float64)
    x = torch.zeros(B, T, D, dtype=torch.float64)

    # a twin block sharing log_rate / log_w: mu = 0 on `block` exposes fast alone, mu = [I; 0]
    # on `twin` (with v = 0) exposes q * w alone
    twin = ref_model.UnifiedBlock(args).double()
    twin.log_rate, twin.log_w, twin.log_eps = block.log_rate, block.log_w, block.log_eps
    with torch.no_grad():
        block.mu.weight.zero_()
        twin.mu.weight.copy_(torch.eye(D, M, dtype=torch.float64))

    def run(form):
        r = r0.clone().requires_grad_(True)
        v = v0.clone().requires_grad_(True)
        k = F.pad(r, (0, 0, 1, 0))[:, :-1]
        mix = (lambda *a_: ref_tests.chunked_mix(*a_, 64)) if form == "chunked" else ref_tests.dense_mix
        fast = mix(block, x, r, k, v)
        qw = mix(twin, x, r, k, torch.zeros_like(v))[..., :M]
        q = qw / block._w()
        return r, v, q, fast

    block.zero_grad()
    r, v, q, fast = run("chunked")
    loss = (q * dq_out).sum() + (fast * dfast).sum()
    loss.backward()
    g = -block.log_rate.exp()
    w = block._w()
    out = {
        "r": r0, "v": v0, "g": g.detach().clone(), "w": w.detach().clone(),
        "dq_out": dq_out, "dfast": dfast,
        "q": q.detach(), "fast": fast.detach(),
        "dr": r.grad.detach(), "dv": v.grad.detach(),
        "dg": (block.log_rate.grad / g).detach(), "dw": (block.log_w.grad / w).detach(),
    }
    with torch.no_grad():
        _, _, qd, fd = run("dense")
    out["q_dense"], out["fast_dense"] = qd.detach(), fd.detach()
    return out


def model_fixture(ref_tests):
    model = ref_tests.tiny_model(seed=3, dim=32, n_layers=2, hidden_dim=48, vocab_size=97,
                                 max_seq_len=140).double().train()
    g = torch.Generator().manual_seed(5)
    tokens = torch.randint(0, 97, (2, 140), generator=g)
    logits, loss = ref_tests.reference_forward(model, tokens, tokens, ref_tests.chunked(64))
    loss.backward()
    grads = {n: p.grad.detach().clone() for n, p in model.named_parameters()}
    with torch.no_grad():
        rec = model.forward_recurrent(tokens[:, :40])
    sd = {n: t.detach().clone() for n, t in model.state_dict().items()}
    return {"state_dict": sd, "tokens": tokens, "logits": logits.detach(), "loss": loss.detach(),
            "grads": grads, "recurrent_logits": rec, "recurrent_len": 40}


def runc_fixture(ref_model):
    import importlib.util
    spec = importlib.util.spec_from_file_location("ulm_export", os.path.join(REPO, "unifiedlm.c_b200", "export.py"))
    ulm_export = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ulm_export)
    write_model_bin, write_tokenizer_bin = ulm_export.write_model_bin, ulm_export.write_tokenizer_bin
    seq = 64
    steps = 40
    binary = os.path.join(REPO, "oracle", "_ref", "run")
    # the model of test_all.test_runc with an untied classifier: with tied embeddings and fresh
    # blocks the greedy token after BOS is BOS again and run.c stops at once (the reference's test
    # feeds a text prompt instead); take the first seed whose greedy run from BOS is long
    for seed in range(100):
        torch.manual_seed(seed)
        model = ref_model.UnifiedLM(ref_model.ModelArgs(dim=32, n_layers=2, hidden_dim=48, vocab_size=512,
                                                        max_seq_len=seq)).eval()
        with torch.no_grad():
            for layer in model.layers:
                layer.val.weight.normal_(std=0.2)
                layer.conv.weight.normal_(std=0.5)
            model.output.weight = torch.nn.Parameter(torch.randn(512, 32) * 0.5)
        sd = {n: t.detach().clone() for n, t in model.state_dict().items()}
        with tempfile.TemporaryDirectory() as tmp:
            mpath, tpath = os.path.join(tmp, "model.bin"), os.path.join(tmp, "tok.bin")
            write_model_bin(sd, mpath, seq)
            write_tokenizer_bin(tpath, [f"|{i}" for i in range(512)])
            text = subprocess.run([binary, mpath, "-z", tpath, "-t", "0", "-n", str(steps)],
                                  capture_output=True, text=True, check=True).stdout
        ids = [int(p) for p in text.strip().split("|") if p]
        if len(ids) >= 30:
            break
    # the reference's own token-by-token PyTorch form must agree (test_all.py:169-193)
    toks = [1]
    with torch.no_grad():
        for _ in range(len(ids)):
            toks.append(int(model.forward_recurrent(torch.tensor([toks]))[0, -1].argmax()))
    assert toks[1:] == ids, (toks[1:], ids)
    return {"state_dict": sd, "max_seq_len": seq, "steps": steps, "seed": seed, "ids": torch.tensor(ids)}


SAMPLED_RUNS = [(1.0, 0.9, 42), (0.8, 0.9, 7), (1.0, 1.0, 3), (0.7, 0.0, 11)]  # (temperature, topp, seed)


def runc_sampled_fixture():
    import importlib.util
    spec = importlib.util.spec_from_file_location("ulm_export", os.path.join(REPO, "unifiedlm.c_b200", "export.py"))
    ulm_export = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ulm_export)
    base = torch.load(os.path.join(HERE, "runc_tiny.pt"), weights_only=False)
    binary = os.path.join(REPO, "oracle", "_ref", "run")
    steps = 48
    runs = []
    with tempfile.TemporaryDirectory() as tmp:
        mpath, tpath = os.path.join(tmp, "model.bin"), os.path.join(tmp, "tok.bin")
        ulm_export.write_model_bin(base["state_dict"], mpath, base["max_seq_len"])
        ulm_export.write_tokenizer_bin(tpath, [f"|{i}" for i in range(512)])
        for temperature, topp, seed in SAMPLED_RUNS:
            text = subprocess.run([binary, mpath, "-z", tpath, "-t", str(temperature), "-p", str(topp), "-s",
                                   str(seed), "-n", str(steps)], capture_output=True, text=True, check=True).stdout
            ids = [int(p) for p in text.strip().split("|") if p]
            runs.append({"temperature": temperature, "topp": topp, "seed": seed, "steps": steps,
                         "ids": torch.tensor(ids)})
    return {"runs": runs}


def main():
    import sys
    if "--sampled" in sys.argv:
        torch.save(runc_sampled_fixture(), os.path.join(HERE, "runc_sampled.pt"))
        return
    ref_model, ref_tests = load_reference()
    torch.save(memory_op_fixture(ref_model, ref_tests), os.path.join(HERE, "memory_op.pt"))
    torch.save(model_fixture(ref_tests), os.path.join(HERE, "model_tiny.pt"))
    torch.save(runc_fixture(ref_model), os.path.join(HERE, "runc_tiny.pt"))
    torch.save(runc_sampled_fixture(), os.path.join(HERE, "runc_sampled.pt"))
    for f in sorted(os.listdir(HERE)):
        print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
