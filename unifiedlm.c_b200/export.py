"""`model.bin` version 1: the fp32 checkpoint format the C decoder reads.

Layout (export.py:1-13, 37-81 and run.c:140-186 of the reference):

* a 256-byte header: uint32 magic 0x554C4D65 ("ULMe"), int32 version 1, then seven int32
  `dim, n_layers, hidden_dim, vocab_size, max_seq_len, conv_size, shared_classifier`, zero padded;
* fp32 token embedding table (vocab, dim);
* per block: norm (dim), conv (dim, conv_size) oldest -> newest, key weight (hidden, dim),
  key bias (hidden), mu (dim, hidden), val (dim, dim), then the derived scalars in the form the
  decoder uses them: w = exp(clamp(log_w, -7, 12)) (hidden), lam = exp(-exp(log_rate)) (1),
  eps = exp(clamp(log_eps, -10, 10)) (1);
* final norm (dim), and the classifier (vocab, dim) only when it is not tied to the embedding.

The layout has to match byte for byte so that checkpoints written here run in the reference's
`run.c` and the other way round.
"""
import struct

import numpy as np
import torch

MAGIC = 0x554C4D65
VERSION = 1
HEADER_BYTES = 256
CONFIG_FIELDS = ("dim", "n_layers", "hidden_dim", "vocab_size", "max_seq_len", "conv_size",
                 "shared_classifier")


def _f32(t):
    return t.detach().cpu().reshape(-1).to(torch.float32).numpy()


def write_model_bin(params, path, max_seq_len):
    """Write a UnifiedLM state_dict-like mapping as model.bin v1."""
    emb = params["tok_embeddings.weight"]
    head = params["output.weight"]
    vocab, dim = emb.shape
    n_layers = 1 + max(int(k.split(".")[1]) for k in params if k.startswith("layers."))
    hidden = params["layers.0.key.weight"].shape[0]
    conv_size = params["layers.0.conv.weight"].shape[-1]
    shared = bool(emb.data_ptr() == head.data_ptr() or torch.equal(emb, head))
    with open(path, "wb") as f:
        f.write(struct.pack("<Ii", MAGIC, VERSION))
        f.write(struct.pack("<7i", dim, n_layers, hidden, vocab, max_seq_len, conv_size, int(shared)))
        f.write(b"\0" * (HEADER_BYTES - f.tell()))
        parts = [_f32(emb)]
        for i in range(n_layers):
            p = lambda n: params[f"layers.{i}.{n}"]  # noqa: E731
            parts += [_f32(p("norm.weight")), _f32(p("conv.weight")[:, 0, :]), _f32(p("key.weight")),
                      _f32(p("key.bias")), _f32(p("mu.weight")), _f32(p("val.weight")),
                      _f32(torch.exp(torch.clamp(p("log_w"), -7.0, 12.0))),
                      _f32(torch.exp(-torch.exp(p("log_rate")))),
                      _f32(torch.exp(torch.clamp(p("log_eps"), -10.0, 10.0)))]
        parts.append(_f32(params["norm.weight"]))
        if not shared:
            parts.append(_f32(head))
        for a in parts:
            f.write(a.astype("<f4").tobytes())


def read_model_bin(path):
    """Read model.bin v1. Returns (config dict, tensors dict) with the per-block derived scalars
    under `layers.{i}.w`, `.lam`, `.eps` and the conv weight as (dim, conv_size)."""
    raw = open(path, "rb").read()
    magic, version = struct.unpack_from("<Ii", raw, 0)
    if magic != MAGIC:
        raise ValueError(f"bad checkpoint magic 0x{magic:08x}")
    if version != VERSION:
        raise ValueError(f"need an fp32 checkpoint (version 1), got {version}")
    cfg = dict(zip(CONFIG_FIELDS, struct.unpack_from("<7i", raw, 8)))
    data = np.frombuffer(raw, dtype="<f4", offset=HEADER_BYTES)
    d, m, V, K = cfg["dim"], cfg["hidden_dim"], cfg["vocab_size"], cfg["conv_size"]
    out, pos = {}, 0

    def take(name, *shape):
        nonlocal pos
        n = int(np.prod(shape))
        if pos + n > data.size:
            raise ValueError(f"checkpoint truncated at {name}")
        out[name] = torch.from_numpy(data[pos:pos + n].copy()).reshape(shape)
        pos += n

    take("tok_embeddings.weight", V, d)
    for i in range(cfg["n_layers"]):
        pre = f"layers.{i}."
        take(pre + "norm.weight", d)
        take(pre + "conv", d, K)
        take(pre + "key.weight", m, d)
        take(pre + "key.bias", m)
        take(pre + "mu.weight", d, m)
        take(pre + "val.weight", d, d)
        take(pre + "w", m)
        take(pre + "lam", 1)
        take(pre + "eps", 1)
    take("norm.weight", d)
    if cfg["shared_classifier"]:
        out["output.weight"] = out["tok_embeddings.weight"]
    else:
        take("output.weight", V, d)
    return cfg, out


def write_tokenizer_bin(path, pieces, scores=None):
    """Write a vocabulary in the llama2.c tokenizer.bin layout read by run.c (run.c:286-307):
    int32 max_token_length, then per token float32 score, int32 byte length, the bytes."""
    enc = [p.encode("utf-8") for p in pieces]
    scores = scores if scores is not None else [0.0] * len(enc)
    with open(path, "wb") as f:
        f.write(struct.pack("<i", max(len(b) for b in enc)))
        for b, s in zip(enc, scores):
            f.write(struct.pack("<fi", float(s), len(b)))
            f.write(b)
