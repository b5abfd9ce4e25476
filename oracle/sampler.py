"""TEST INFRASTRUCTURE ONLY — a CPU restatement of the reference run.c sampler, used by tests/ to
check the device sampler (ulm_decode_sample). Nothing in the library imports this module.

run.c's sample() (run.c:527-534) with its helpers, in float32 with sequential sums, as run.c
computes them:
  * temperature 0: first index of the largest logit (sample_argmax, run.c:460-470);
  * otherwise logits / temperature, softmax (run.c:66-75), a coin from the xorshift64* generator
    (random_u32 / random_f32, run.c:516-525), then either the first index whose running cdf exceeds
    the coin (sample_mult, run.c:472-479, when topp <= 0 or >= 1) or top-p sampling
    (sample_topp, run.c:487-514): candidates p >= (1 - topp) / (n - 1), sorted by descending p
    (ties here by ascending index), the shortest prefix whose running sum exceeds topp, and the first
    entry of that prefix whose running sum exceeds coin * (prefix sum).
"""
import numpy as np

MASK64 = (1 << 64) - 1


def xorshift_next(state):
    """One step of the 64-bit xorshift* generator: (new state, 32-bit output)."""
    state ^= state >> 12
    state ^= (state << 25) & MASK64
    state ^= state >> 27
    state &= MASK64
    return state, ((state * 0x2545F4914F6CDD1D) & MASK64) >> 32


def random_f32(state):
    state, u = xorshift_next(state)
    return state, np.float32((u >> 8) / 16777216.0)


def softmax_f32(x, acc=np.float32):
    """run.c's softmax in float32; the normaliser is a sequential float32 sum as in run.c, or the
    exact (float64) sum with acc=np.float64."""
    x = np.asarray(x, dtype=np.float32)
    e = np.exp(x - x.max()).astype(np.float32)
    if acc is np.float32:
        total = np.float32(0.0)
        for v in e:  # sequential, as run.c
            total = np.float32(total + v)
    else:
        total = np.float32(np.sum(e, dtype=np.float64))
    return (e / total).astype(np.float32)


def sample(logits, temperature, topp, state, acc=np.float32):
    """Returns (token, new state, margin): margin is the distance of the decisive comparison from its
    boundary (a tie-break-free check for tests comparing against a parallel implementation).
    acc: the type of the running sums; float32 (sequential) is run.c's arithmetic, float64 the exact
    sums a parallel implementation is compared against."""
    logits = np.asarray(logits, dtype=np.float32)
    if temperature == 0.0:
        return int(np.argmax(logits)), state, float("inf")
    p = softmax_f32(logits / np.float32(temperature), acc)
    state, coin = random_f32(state)
    if topp <= 0.0 or topp >= 1.0:
        cdf = np.cumsum(p, dtype=acc)  # sequential accumulation
        hit = np.nonzero(coin < cdf)[0]
        i = int(hit[0]) if hit.size else p.size - 1
        lo = cdf[i - 1] if i > 0 else acc(0.0)
        return i, state, float(min(abs(coin - lo), abs(cdf[i] - coin)))
    n = p.size
    cutoff = np.float32((np.float32(1.0) - np.float32(topp)) / np.float32(n - 1))
    idx = np.nonzero(p >= cutoff)[0]
    order = idx[np.lexsort((idx, -p[idx]))]  # descending p, ascending index on ties
    cum = np.cumsum(p[order], dtype=acc)
    above = np.nonzero(cum > np.float32(topp))[0]
    last = int(above[0]) if above.size else order.size - 1
    margin = float(abs(cum[last] - np.float32(topp)))
    r = acc(coin) * cum[last] if acc is not np.float32 else np.float32(coin * cum[last])
    cdf = cum[:last + 1]
    hit = np.nonzero(r < cdf)[0]
    j = int(hit[0]) if hit.size else last
    lo = cdf[j - 1] if j > 0 else acc(0.0)
    margin = min(margin, float(abs(r - lo)), float(abs(cdf[j] - r)))
    return int(order[j]), state, margin


def sampled_decode(params, steps, temperature, topp, seed, bos=1):
    """run.c's generate() with an empty prompt (run.c:542-571) and the sampler above on the float64
    recurrent model of oracle.memory (logits rounded to float32, as run.c holds them): returns the
    ids and the smallest decision margin seen."""
    import torch

    from . import memory as O
    L = O.n_layers_of(params)
    blocks = [O.block_params(params, i) for i in range(L)]
    states = [O.block_init_state(p, 1) for p in blocks]
    token, out, state, margin = bos, [], seed & MASK64, float("inf")
    with torch.no_grad():
        for _ in range(steps):
            h = params["tok_embeddings.weight"][torch.tensor([token])]
            for p, s in zip(blocks, states):
                h = O.block_step(p, h, s)
            logits = (O.rmsnorm(h, params["norm.weight"]) @ params["output.weight"].t())[0]
            nxt, state, m = sample(logits.float().numpy(), temperature, topp, state)
            margin = min(margin, m)
            if nxt == bos:
                break
            out.append(nxt)
            token = nxt
    return out, margin
