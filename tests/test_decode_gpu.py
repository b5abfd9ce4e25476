"""Batched recurrent decode (ulm_decode_*) against the reference's run.c and the float64 oracle.

* fp32 mode greedy tokens identical to the reference's run.c (fixture from the reference's own
  binary, and a live run of oracle/_ref/run when it was built).
* per-step logits against the oracle's forward_recurrent (model.py:164-175): fp32 mode within
  1e-4 relative, bf16 weights within 2e-2.
"""
import math
import os
import subprocess
import tempfile

import pytest
import torch

import unifiedlm_c_b200._lib as L
from oracle import memory as O
from unifiedlm_c_b200 import export
from unifiedlm_c_b200.decode import BatchedDecoder

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
RUNC = os.path.join(ROOT, "oracle", "_ref", "run")


def load(golden_dir, name):
    return torch.load(os.path.join(golden_dir, name), weights_only=False)


@pytest.mark.parametrize("use_graph", [True, False])
def test_greedy_tokens_match_reference_runc(golden_dir, use_graph):
    f = load(golden_dir, "runc_tiny.pt")
    ids = f["ids"].tolist()
    assert len(ids) >= 30
    dec = BatchedDecoder(f["state_dict"], batch=3, precision="fp32", use_graph=use_graph)
    out = dec.generate(torch.ones(3, 1, dtype=torch.long), steps=f["steps"])
    for row in out.tolist():
        assert row[:len(ids)] == ids
        assert len(ids) == f["steps"] or row[len(ids)] == 1  # run.c stops at a predicted BOS


def rand_params(seed, dim, n_layers, hidden, vocab):
    g = torch.Generator().manual_seed(seed)
    p = {"tok_embeddings.weight": torch.randn(vocab, dim, generator=g) * 0.3, "norm.weight": 1 + 0.1 * torch.randn(dim, generator=g)}
    p["output.weight"] = torch.randn(vocab, dim, generator=g) * 0.3   # untied: greedy runs do not stick at BOS
    for i in range(n_layers):
        pre = f"layers.{i}."
        p[pre + "norm.weight"] = 1 + 0.1 * torch.randn(dim, generator=g)
        p[pre + "conv.weight"] = torch.randn(dim, 1, 4, generator=g) * 0.5
        p[pre + "key.weight"] = torch.randn(hidden, dim, generator=g) / math.sqrt(dim)
        p[pre + "key.bias"] = torch.randn(hidden, generator=g) * 0.3
        p[pre + "mu.weight"] = torch.randn(dim, hidden, generator=g) * 0.05
        p[pre + "val.weight"] = torch.randn(dim, dim, generator=g) / math.sqrt(dim)
        p[pre + "log_eps"] = torch.tensor(0.0)
        p[pre + "log_rate"] = torch.tensor(math.log(-math.log(0.95)))
        p[pre + "log_w"] = torch.randn(hidden, generator=g) * 0.5 + math.log(4.0)
    return p


@pytest.mark.parametrize("precision,tol", [("fp32", 1e-4), ("bf16", 2e-2)])
@pytest.mark.parametrize("shape", [(32, 2, 48, 97), (768, 2, 2048, 512)], ids=["tiny", "110M-block"])
def test_logits_match_oracle_recurrent(precision, tol, shape):
    dim, n_layers, hidden, vocab = shape
    p = rand_params(0, dim, n_layers, hidden, vocab)
    B, T = 3, 10
    tokens = torch.randint(0, vocab, (B, T), generator=torch.Generator().manual_seed(1))
    ref = O.lm_forward_recurrent({k: v.double() for k, v in p.items()}, tokens)
    dec = BatchedDecoder(p, batch=B, precision=precision)
    dec.prepare_graph()
    for t in range(T):
        dec.feed(tokens[:, t])
        got = dec.logits.double().cpu()
        err = float((got - ref[:, t]).norm() / ref[:, t].norm())
        assert err < tol, (t, err)


def test_live_runc_token_identity(tmp_path):
    """Export a model, decode it with the reference's run.c (built by `make -C oracle`) and with the
    batched decoder in fp32 mode; the greedy tokens must be the same."""
    if not os.path.exists(RUNC):
        pytest.skip("oracle/_ref/run not built (needs the reference checkout)")
    steps = 64
    mpath, tpath = str(tmp_path / "m.bin"), str(tmp_path / "tok.bin")
    export.write_tokenizer_bin(tpath, [f"|{i}" for i in range(512)])
    for seed in range(3, 50):  # first seed whose greedy run from BOS is long
        p = rand_params(seed, 64, 3, 128, 512)
        export.write_model_bin(p, mpath, max_seq_len=steps)
        text = subprocess.run([RUNC, mpath, "-z", tpath, "-t", "0", "-n", str(steps)], capture_output=True,
                              text=True, check=True).stdout
        ids = [int(x) for x in text.strip().split("|") if x]
        if len(ids) >= 48:
            break
    assert len(ids) >= 48
    dec = BatchedDecoder(p, batch=2, precision="fp32")
    out = dec.generate(torch.ones(2, 1, dtype=torch.long), steps=steps)
    assert out[0, :len(ids)].tolist() == ids and out[1, :len(ids)].tolist() == ids


@pytest.mark.parametrize("use_graph", [True, False])
def test_sampled_tokens_match_reference_runc(golden_dir, use_graph):
    """Sampling on the device (temperature > 0, top-p and plain multinomial) reproduces the token ids
    the reference's run.c printed for the same model and seeds (fixture runc_sampled.pt)."""
    base = load(golden_dir, "runc_tiny.pt")
    for run in load(golden_dir, "runc_sampled.pt")["runs"]:
        ids = run["ids"].tolist()
        dec = BatchedDecoder(base["state_dict"], batch=2, precision="fp32", use_graph=use_graph,
                             temperature=run["temperature"], topp=run["topp"], seed=[run["seed"], run["seed"]])
        out = dec.generate(torch.ones(2, 1, dtype=torch.long), steps=run["steps"])
        for row in out.tolist():
            assert row[:len(ids)] == ids, (run["temperature"], run["topp"], run["seed"])


@pytest.mark.parametrize("topp", [0.9, 0.5, 1.0])
@pytest.mark.parametrize("scale", [0.3, 3.0, 30.0], ids=["flat", "medium", "peaked"])
def test_device_sampler_matches_oracle(topp, scale):
    """ulm_decode_sample on random logits (V = 32000, 64 sequences, own seeds) against run.c's
    sampler restated in oracle.sampler with exact (float64) running sums: same tokens and advanced
    states, except where the decisive comparison is within 2e-6 of its boundary (the device's
    parallel sums differ in the last bits; run.c's sequential float32 sums drift further on flat
    distributions, where tens of thousands of terms are summed)."""
    import numpy as np
    import unifiedlm_c_b200._lib as L
    from oracle import sampler as S
    B, V, D = 64, 32000, 8
    g = torch.Generator().manual_seed(int(scale * 10) + int(topp * 100))
    logits = torch.randn(B, V, generator=g) * scale
    seeds = [int(x) for x in torch.randint(1, 2**62, (B,), generator=g)]
    rng = torch.tensor(seeds, dtype=torch.int64, device="cuda")
    emb = torch.randn(V, D, device="cuda")
    x = torch.empty(B, D, device="cuda")
    nxt = torch.empty(B, dtype=torch.int32, device="cuda")
    lg = logits.cuda()
    temperature = 0.8
    L.check(L.lib().ulm_decode_sample(L.ptr(lg), B, V, temperature, topp, L.ptr(rng), L.ptr(nxt), L.ptr(emb),
                                      L.ULM_F32, L.ptr(x), D, None))
    torch.cuda.synchronize()
    got, states = nxt.cpu().tolist(), [s & S.MASK64 for s in rng.cpu().tolist()]
    checked = 0
    for b in range(B):
        tok, st, margin = S.sample(logits[b].numpy(), temperature, topp, seeds[b], acc=np.float64)
        assert states[b] == st
        if margin > 2e-6:
            assert got[b] == tok, (b, got[b], tok, margin)
            checked += 1
    assert checked >= B // 2  # flat distributions put many cumulative boundaries near any coin
    assert torch.equal(x.cpu(), emb.cpu()[torch.tensor(got)])
    assert L.device_error() == 0


def test_decoder_from_model_bin(golden_dir, tmp_path):
    """BatchedDecoder.from_model_bin over run.c's checkpoint file gives run.c's greedy tokens."""
    f = load(golden_dir, "runc_tiny.pt")
    path = str(tmp_path / "m.bin")
    export.write_model_bin(f["state_dict"], path, f["max_seq_len"])
    dec = BatchedDecoder.from_model_bin(path, batch=2, precision="fp32")
    out = dec.generate(torch.ones(2, 1, dtype=torch.long), steps=f["steps"])
    ids = f["ids"].tolist()
    assert out[0, :len(ids)].tolist() == ids and out[1, :len(ids)].tolist() == ids


def test_live_runc_sampled_identity(tmp_path):
    """Sampled decode (temperature 1, top-p 0.9, seed 5) of an exported model against a live run of
    the reference's run.c."""
    if not os.path.exists(RUNC):
        pytest.skip("oracle/_ref/run not built (needs the reference checkout)")
    steps = 48
    mpath, tpath = str(tmp_path / "m.bin"), str(tmp_path / "tok.bin")
    export.write_tokenizer_bin(tpath, [f"|{i}" for i in range(512)])
    p = rand_params(9, 64, 3, 128, 512)
    export.write_model_bin(p, mpath, max_seq_len=steps)
    text = subprocess.run([RUNC, mpath, "-z", tpath, "-t", "1.0", "-p", "0.9", "-s", "5", "-n", str(steps)],
                          capture_output=True, text=True, check=True).stdout
    ids = [int(x) for x in text.strip().split("|") if x]
    dec = BatchedDecoder.from_model_bin(mpath, batch=1, precision="fp32", temperature=1.0, topp=0.9, seed=5)
    out = dec.generate(torch.ones(1, 1, dtype=torch.long), steps=steps)
    assert out[0, :len(ids)].tolist() == ids


@pytest.mark.parametrize("precision,P", [("fp32", 37), ("fp32", 512), ("bf16", 300), ("bf16", 1024)])
def test_prefill_matches_token_by_token(precision, P):
    """BatchedDecoder.prefill (the prompt in one parallel pass, the state from one carry product per
    block) against feeding the prompt token by token: the last position's logits within 1e-4 (fp32)
    or 2e-2 (bf16 products against bf16-weight steps), and in fp32 mode the greedy continuation
    identical. P = 512 (fp32, chunks of 64) and 1024 (bf16, chunks of 256 set for the test) run the
    blocks' fast read in the chunk-carry form."""
    lib = L.lib()
    lib.ulm_set_chunk_mode(256 if (precision, P) == ("bf16", 1024) else -1)
    try:
        _prefill_case(precision, P)
    finally:
        lib.ulm_set_chunk_mode(-1)


def _prefill_case(precision, P):
    p = rand_params(7, 64, 3, 128, 512)
    B, steps = 3, 24
    prompt = torch.randint(0, 512, (B, P), generator=torch.Generator().manual_seed(P))
    a = BatchedDecoder(p, batch=B, precision=precision)
    a.prepare_graph()
    for t in range(P):
        nt = a.feed(prompt[:, t])
    ref_logits = a.logits.double().cpu()
    ref = [nt.clone()] + [a.step_greedy().clone() for _ in range(steps)]
    b = BatchedDecoder(p, batch=B, precision=precision)
    b.prepare_graph()
    nt = b.prefill(prompt)
    err = float((b.logits.double().cpu() - ref_logits).norm() / ref_logits.norm())
    assert err < (1e-4 if precision == "fp32" else 2e-2), err
    got = [nt.clone()] + [b.step_greedy().clone() for _ in range(steps)]
    if precision == "fp32":
        assert torch.equal(torch.stack(got), torch.stack(ref))


def test_model_step_and_forward_recurrent_use_the_decoder():
    """UnifiedBlock.init_state / step and UnifiedLM.forward_recurrent (model.py:88-111, 164-175) on
    the library's decode kernels, against the oracle's token-by-token form in float64."""
    from unifiedlm_c_b200.model import ModelArgs, UnifiedLM
    p = rand_params(3, 32, 2, 48, 97)
    args = ModelArgs(dim=32, n_layers=2, hidden_dim=48, vocab_size=97, max_seq_len=64)
    model = UnifiedLM(args)
    model.load_state_dict(p, strict=False)
    with torch.no_grad():
        model.output.weight.copy_(p["output.weight"])  # tied: the embedding follows
    tied = {k: v for k, v in p.items()}
    tied["tok_embeddings.weight"] = p["output.weight"]
    model = model.cuda()
    tokens = torch.randint(0, 97, (2, 12), generator=torch.Generator().manual_seed(2))
    ref = O.lm_forward_recurrent({k: v.double() for k, v in tied.items()}, tokens)
    got = model.forward_recurrent(tokens.cuda()).double().cpu()
    assert float((got - ref).norm() / ref.norm()) < 1e-4
    # the block API: one block's steps against the oracle's step
    blk = model.layers[0]
    s = blk.init_state(2, "cuda")
    so = O.block_init_state({k[len("layers.0."):]: v.double() for k, v in tied.items() if k.startswith("layers.0.")},
                            2)
    x = torch.randn(2, 32, generator=torch.Generator().manual_seed(4))
    pb = {k[len("layers.0."):]: v.double() for k, v in tied.items() if k.startswith("layers.0.")}
    for _ in range(5):
        y = blk.step(x.cuda(), s)
        yo = O.block_step(pb, x.double(), so)
        assert float((y.double().cpu() - yo).norm() / yo.norm()) < 1e-5
        x = yo.float()


def test_live_runc_token_identity_c5_shape(tmp_path):
    """BASELINE config 5's model shape (dim 768, M 2048, 12 blocks, vocab 32000), fp32 mode: 32
    greedy tokens from BOS identical to the reference's run.c on the same model.bin."""
    if not os.path.exists(RUNC):
        pytest.skip("oracle/_ref/run not built (needs the reference checkout)")
    steps = 32
    mpath, tpath = str(tmp_path / "m.bin"), str(tmp_path / "tok.bin")
    export.write_tokenizer_bin(tpath, [f"|{i}" for i in range(32000)])
    ids = []
    for seed in range(11, 16):  # first seed whose greedy run from BOS does not stop early at BOS
        p = rand_params(seed, 768, 12, 2048, 32000)
        export.write_model_bin(p, mpath, max_seq_len=steps)
        text = subprocess.run([RUNC, mpath, "-z", tpath, "-t", "0", "-n", str(steps)], capture_output=True,
                              text=True, check=True, timeout=300).stdout
        ids = [int(x) for x in text.strip().split("|") if x]
        if len(ids) >= 24:
            break
    assert len(ids) >= 24
    dec = BatchedDecoder(p, batch=2, precision="fp32")
    out = dec.generate(torch.ones(2, 1, dtype=torch.long), steps=steps)
    assert out[0, :len(ids)].tolist() == ids and out[1, :len(ids)].tolist() == ids
