"""Benchmark of the fast-memory path at the 110M shape.

One step = the fast-memory path of every one of the 12 UnifiedBlocks, forward and backward, on
16 sequences x 1024 tokens per GPU (dim D=768, slots M=2048): the addressing prologue
(conv -> key GEMM -> relu^2 -> normalise, model.py:70-72, 79), the fast-memory operator
(unified_memory, kernel.py:199-238), then the operator's backward and the prologue's backward, which
yield the path's parameter gradients (key weight and bias, conv, eps, prior mass w, decay). At N>1
those gradients are all-reduced over NCCL (data parallel, 16 sequences per GPU). Inputs are seeded
synthetic normalised hidden states and values, resident in HBM and larger than L2, so no L2 flush is
needed between steps. Metric: tokens per second through all 12 blocks, whole job.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--precision bf16|fp32]

Under torchrun each rank drives one GPU; the step time is the max over ranks of the CUDA-event time.
`--impl reference` times the reference's CPU algorithm for the same path (the chunked pure-PyTorch
form of test_all.py:28-51 with the model.py prologue, restated in oracle/memory.py) on this host's
cores.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from __graft_entry__ import load_package  # noqa: E402

WORKLOAD = dict(B=16, T=1024, M=2048, D=768, L=12, lam=0.95, prior=4.0)
METRIC = "fast-memory fwd+bwd tokens/s (110M shape)"
PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")


def peaks():
    try:
        p = json.load(open(PEAKS_FILE))
        return {"bf16_tflops": p["bf16_tflops"], "hbm_gbs": p["hbm_gbs"], "source": "measured"}
    except Exception:
        return {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0, "source": "fallback"}


def make_inputs(B, T, M, D, L, lam, prior, device, seed=0):
    """Seeded synthetic inputs of one step and per-block weights (the reference's init scales).

    Every block gets its own h, v, dq_out and dfast (lists of L tensors, 235 MB per block at the
    110M shape), as in a model where each block's inputs come from its neighbours: no block reads
    what an earlier block left in L2."""
    import math
    gen = torch.Generator(device=device).manual_seed(seed)
    rn = lambda *s_: torch.randn(*s_, device=device, generator=gen)  # noqa: E731
    hs, vs, dqs, dfs = [], [], [], []
    for _ in range(L):
        h = rn(B, T, D)
        hs.append(h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-5))
        # dtypes as under the reference's bf16 autocast: the residual stream and h = norm(x) stay
        # fp32, v = val(h) is bf16, so fast and its gradient are bf16; q and its gradient are fp32
        vs.append(rn(B, T, D).to(torch.bfloat16))
        dqs.append(rn(B, T, M) * 1e-3)
        dfs.append((rn(B, T, D) * 1e-3).to(torch.bfloat16))
    blocks = []
    for _ in range(L):
        blocks.append({"conv": rn(D, 1, 4) * 0.5, "key_w": rn(M, D) / math.sqrt(D), "key_b": rn(M) * 0.1,
                       "eps": torch.ones((), device=device),
                       "g": torch.tensor(math.log(lam), device=device), "w": torch.full((M,), prior, device=device)})
    return hs, vs, dqs, dfs, blocks


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.PIPE, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path:
            return None
        err = self.proc.stderr.read() if self.proc.stderr else ""
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(parts)
            except Exception:
                pass
        raw = open(self.path).read()
        os.unlink(self.path)
        if not rows:
            return {"error": (err or raw)[-300:]}
        sm = [float(p[1]) for p in rows if p[1].replace(".", "").isdigit()]
        mx = [float(p[2]) for p in rows if p[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for p in rows for n, val in zip(names, p[5:9]) if val.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_reference_seconds(T, M, D, lam, prior, reps, threads):
    """Seconds for one sequence x one block of the reference's CPU form of the path (prologue +
    chunked fast memory, forward and backward, fp32): the median of `reps` timed samples after one
    untimed one."""
    import math
    from oracle import memory as O
    torch.set_num_threads(threads)
    g_ = torch.Generator().manual_seed(0)
    h = torch.randn(1, T, D, generator=g_)
    v = torch.randn(1, T, D, generator=g_)
    conv = (torch.randn(D, 1, 4, generator=g_) * 0.5).requires_grad_(True)
    kw = (torch.randn(M, D, generator=g_) / math.sqrt(D)).requires_grad_(True)
    kb = (torch.randn(M, generator=g_) * 0.1).requires_grad_(True)
    log_eps = torch.zeros((), requires_grad=True)
    g = torch.tensor(math.log(lam), requires_grad=True)
    w = torch.full((M,), prior, requires_grad=True)
    dq_out = torch.randn(1, T, M, generator=g_)
    dfast = torch.randn(1, T, D, generator=g_)

    def once():
        r = O.prologue(h, conv, kw, kb, log_eps)
        q, fast = O.memory_chunked(r, v, g, w, 64)
        ((q * dq_out).sum() + (fast * dfast).sum()).backward()

    once()  # warm-up
    secs = []
    for _ in range(reps):
        t0 = time.perf_counter()
        once()
        secs.append(time.perf_counter() - t0)
    return statistics.median(secs)


def workload_config(W):
    """The workload both arms name in their JSON line."""
    return {"workload": f"fast-memory path fwd+bwd (addressing prologue + unified_memory) x {W['L']} blocks "
                        f"(110M shape), {W['B']} seq x {W['T']} tok per GPU",
            "B_per_gpu": W["B"], "T": W["T"], "M": W["M"], "D": W["D"], "layers": W["L"], "lam": W["lam"]}


def run_reference(args, rank):
    if rank != 0:
        return
    W = WORKLOAD
    threads = os.cpu_count() or 1
    reps = 3
    # warm-up W samples, then K timed steps; one step = the median of 3 samples of 1 sequence
    # through 1 block
    for _ in range(max(args.warmup, 0)):
        cpu_reference_seconds(W["T"], W["M"], W["D"], W["lam"], W["prior"], 1, threads)
    secs = [cpu_reference_seconds(W["T"], W["M"], W["D"], W["lam"], W["prior"], reps, threads)
            for _ in range(args.steps)]
    per_sample = statistics.median(secs)
    value = W["T"] / (W["L"] * per_sample)
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": per_sample * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic", "impl": "reference",
            "config": dict(workload_config(W), parallelism=f"dp{args.gpus}",
                           sample="median of 3 samples of 1 sequence x 1 block per timed step on the host "
                                  "cores, the median over the steps scaled to the workload's tokens"),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": f"1 seq x 1 block (T={W['T']}, M={W['M']}, D={W['D']}) fwd+bwd, "
                                       "prologue + chunked pure-PyTorch form (model.py:70-79, test_all.py:28-51 "
                                       "restated), fp32"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "decode": runc_decode_baseline()}
    print(json.dumps(line), flush=True)


# DRAM bytes (read + write) of the six fast-memory products of one block at the 110M shape, summed
# over one-kernel ncu captures of `bench.py --profile-block` (dram__bytes_read.sum +
# dram__bytes_write.sum per launch)
PRODUCTS_DRAM_BYTES = 801400000

DECODE = dict(D=768, L=12, M=2048, V=32000, batches=(1, 16, 64, 256), prompt=1024, steps=256, warmup=3)


def decode_params(D, L, M, V, device, seed=0):
    """Seeded random UnifiedLM weights at the 110M shape (untied classifier), on the device."""
    import math
    gen = torch.Generator(device=device).manual_seed(seed)
    rn = lambda *s: torch.randn(*s, device=device, generator=gen)  # noqa: E731
    p = {"tok_embeddings.weight": rn(V, D) * 0.3, "norm.weight": 1 + 0.1 * rn(D), "output.weight": rn(V, D) * 0.3}
    for i in range(L):
        pre = f"layers.{i}."
        p[pre + "norm.weight"] = 1 + 0.1 * rn(D)
        p[pre + "conv.weight"] = rn(D, 1, 4) * 0.5
        p[pre + "key.weight"] = rn(M, D) / math.sqrt(D)
        p[pre + "key.bias"] = rn(M) * 0.3
        p[pre + "mu.weight"] = rn(D, M) * 0.05
        p[pre + "val.weight"] = rn(D, D) / math.sqrt(D)
        p[pre + "log_eps"] = torch.zeros((), device=device)
        p[pre + "log_rate"] = torch.tensor(math.log(-math.log(0.95)), device=device)
        p[pre + "log_w"] = rn(M) * 0.5 + math.log(4.0)
    return p


def bench_decode(dev, pk):
    """batched greedy decode at the 110M shape, per batch size and weight
    precision: a 1024-token prompt fed in one parallel pass (BatchedDecoder.prefill: the blocks'
    training-form forward, then each block's state from one carry product), then 256 greedy steps
    (one CUDA graph per step). bf16 weights with fp32 state, and the fp32 mode (run.c's arithmetic).
    CUDA events around the prefill and around the steps."""
    from unifiedlm_c_b200.decode import BatchedDecoder
    C = DECODE
    params = decode_params(C["D"], C["L"], C["M"], C["V"], dev)
    gen = torch.Generator(device=dev).manual_seed(5)
    out = {}
    for prec in ("bf16", "fp32"):
        rows = {}
        for B in C["batches"]:
            dec = BatchedDecoder(params, batch=B, precision=prec, device=dev)
            dec.prepare_graph()
            prompt = torch.randint(0, C["V"], (B, C["prompt"]), device=dev, generator=gen)
            prompt[:, 0] = 1
            dec.prefill(prompt)  # warm-up (first-call set-up)
            for _ in range(C["warmup"]):
                dec.step_greedy()
            dec.reset()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            torch.cuda.synchronize()
            ev[0].record()
            dec.prefill(prompt)
            ev[1].record()
            for _ in range(C["steps"]):
                dec.step_greedy()
            ev[2].record()
            torch.cuda.synchronize()
            t_pre = ev[0].elapsed_time(ev[1]) / 1e3
            t_step = ev[1].elapsed_time(ev[2]) / 1e3 / C["steps"]
            state_bytes = 8 * C["D"] * C["M"] * C["L"] * B  # U read + write, fp32
            rows[B] = {"tokens_per_s": round(B / t_step, 1), "ms_per_step": round(t_step * 1e3, 4),
                       "state_gbs": round(state_bytes / t_step / 1e9, 1),
                       "prefill_ms": round(t_pre * 1e3, 3), "prefill_tokens_per_s": round(B * C["prompt"] / t_pre, 1)}
            del dec
            torch.cuda.empty_cache()
        out[prec] = rows
    top = out["bf16"][max(C["batches"])]
    return {"metric": "batched greedy decode tokens/s (110M shape)", "value": top["tokens_per_s"],
            "unit": "tokens/s", "batch": max(C["batches"]), "precision": "bf16 weights, fp32 state",
            "workload": f"{C['prompt']}-token prompt (parallel prefill), then {C['steps']} greedy steps per sequence",
            "roofline": {"bound": "hbm", "achieved": top["state_gbs"], "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(top["state_gbs"] / pk["hbm_gbs"], 4),
                         "bytes": "8*D*M*L*B per step (fp32 state read + write)",
                         "kernel": "decode_state_kernel (plus per-step GEMMs and head)"},
            "by_batch": out["bf16"], "fp32_mode_by_batch": out["fp32"]}


def bench_mixer(dev, W, blocks, precision, steps=5, warmup=3):
    """UnifiedBlock's mixing span (address + fast memory + mu(q w) + residual, model.py:79-85) fwd+bwd
    over the 12 blocks at the 110M shape, through autograd, in two forms: the fused combine
    (block.block_mixer: mu(q w) in the fast read's tiles, its gradient in the dq product) and the
    reference's structure on top of the same fast memory (addressed_memory, then a bf16 Linear for
    mu and the residual in PyTorch). bf16 activations, fp32 parameters, as under autocast."""
    import math
    import torch.nn.functional as F
    from unifiedlm_c_b200.block import addressed_memory, block_mixer
    B, T, M, D, L = W["B"], W["T"], W["M"], W["D"], W["L"]
    gen = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(B, T, D, device=dev, generator=gen).to(torch.bfloat16)
    h = (torch.randn(B, T, D, device=dev, generator=gen)).to(torch.bfloat16)
    v = torch.randn(B, T, D, device=dev, generator=gen).to(torch.bfloat16)
    dy = (torch.randn(B, T, D, device=dev, generator=gen) * 1e-3).to(torch.bfloat16)
    params = []
    for blk in blocks:
        p = {k: blk[k].detach().clone().requires_grad_(True) for k in ("conv", "key_w", "key_b", "g", "w")}
        p["eps"] = blk["eps"].detach().clone().requires_grad_(True)
        p["mu"] = (torch.randn(D, M, device=dev, generator=gen) * 0.02 / math.sqrt(L)).requires_grad_(True)
        params.append(p)
    xs = x.clone().requires_grad_(True)

    def step(fused):
        for p in params:
            if fused:
                y = block_mixer(xs, h, p["conv"], p["key_w"], p["key_b"], p["eps"], v, p["g"], p["w"], p["mu"],
                                precision=precision)
            else:
                q, fast = addressed_memory(h, p["conv"], p["key_w"], p["key_b"], p["eps"], v, p["g"], p["w"],
                                           precision=precision)
                y = xs + (F.linear((q * p["w"]).to(torch.bfloat16), p["mu"].to(torch.bfloat16)) + fast.to(xs.dtype))
            y.backward(dy)

    out = {}
    for fused in (True, False):
        for _ in range(warmup):
            step(fused)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(steps):
            step(fused)
        e1.record()
        torch.cuda.synchronize()
        secs = e0.elapsed_time(e1) / 1e3 / steps
        out["fused" if fused else "unfused"] = {"tokens_per_s": round(B * T / secs, 1), "ms_per_step": round(secs * 1e3, 3)}
    return {"metric": "block mixing span fwd+bwd tokens/s (110M shape, 12 blocks)",
            "value": out["fused"]["tokens_per_s"], "unit": "tokens/s",
            "workload": "address + fast memory + mu(q w) + residual per block, autograd, bf16 activations",
            "fused": out["fused"], "unfused_torch_combine": out["unfused"],
            "speedup": round(out["fused"]["tokens_per_s"] / out["unfused"]["tokens_per_s"], 3)}


def bench_head(dev, W, steps=5, warmup=3):
    """Output Linear + cross entropy fwd+bwd at the 110M shape (16 x 1024 rows, V 32000, D 768):
    the fused head (head.lm_head_loss, no logits written) and the reference's form under bf16
    autocast (bf16 Linear, then F.cross_entropy), both through autograd."""
    import torch.nn.functional as F
    from unifiedlm_c_b200.head import lm_head_loss
    B, T, D, V = W["B"], W["T"], W["D"], 32000
    gen = torch.Generator(device=dev).manual_seed(11)
    h = torch.randn(B * T, D, device=dev, generator=gen).requires_grad_(True)
    Wt = (torch.randn(V, D, device=dev, generator=gen) * 0.02).requires_grad_(True)
    tgt = torch.randint(0, V, (B * T,), device=dev, generator=gen)

    def step(fused):
        if fused:
            loss = lm_head_loss(h, Wt, tgt)
        else:
            with torch.autocast("cuda", dtype=torch.bfloat16):
                logits = F.linear(h, Wt)
            loss = F.cross_entropy(logits.float(), tgt, ignore_index=-1)
        loss.backward()

    out = {}
    for fused in (True, False):
        for _ in range(warmup):
            step(fused)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(steps):
            step(fused)
        e1.record()
        torch.cuda.synchronize()
        secs = e0.elapsed_time(e1) / 1e3 / steps
        out["fused" if fused else "torch_autocast"] = {"tokens_per_s": round(B * T / secs, 1),
                                                       "ms_per_step": round(secs * 1e3, 3)}
    return {"metric": "LM head + cross entropy fwd+bwd tokens/s (110M shape, V 32000)",
            "value": out["fused"]["tokens_per_s"], "unit": "tokens/s", "fused": out["fused"],
            "torch_autocast": out["torch_autocast"],
            "speedup": round(out["fused"]["tokens_per_s"] / out["torch_autocast"]["tokens_per_s"], 3)}


def zipf_tokens(B, T, V, seed):
    """Zipf(s=1.1) ranks rejected to < V, rank -> id, BOS=1 first in every row (4)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    out = np.empty((B, T), dtype=np.int64)
    for b in range(B):
        row = []
        while len(row) < T - 1:
            draw = rng.zipf(1.1, size=4 * T)
            row.extend(int(x) - 1 for x in draw if x <= V)
        out[b, 0] = 1
        out[b, 1:] = row[:T - 1]
    return torch.from_numpy(out)


MODELS = {
    "c4": dict(dim=768, n_layers=12, hidden_dim=2048, vocab_size=32000, max_seq_len=1024, batch=16),
    "c2": dict(dim=288, n_layers=6, hidden_dim=768, vocab_size=32000, max_seq_len=256, batch=64),
}


def bench_model(dev, name, steps, warmup, world, rank, bucket_mb=25):
    """One UnifiedLM training step per iteration at a BASELINE model config (c4: 110M, 16 x 1024
    tokens per GPU; c2: 15M, 64 x 256): token ids copied from pinned host memory, forward with the
    fused head, backward, the mean of every parameter gradient over ranks (DDP: bucketed NCCL
    all-reduces overlapping the backward), fused AdamW, and the loss read back to the host. bf16
    tensor-core products, fp32 parameters and statistics. Synthetic Zipf(1.1) token ids with BOS=1;
    random init with prior 4 and lam 0.95 (the same seed on every rank). Device time over the K steps
    (CUDA events), max over ranks."""
    import math
    from unifiedlm_c_b200.model import ModelArgs, UnifiedLM
    cfg = dict(MODELS[name])
    B = cfg.pop("batch")
    torch.manual_seed(1234)
    model = UnifiedLM(ModelArgs(**cfg))
    with torch.no_grad():
        for layer in model.layers:
            layer.log_rate.fill_(math.log(-math.log(0.95)))
    model = model.to(dev).train()
    model.fused_head = True
    model.set_precision("bf16")
    params = [p for p in model.parameters()]
    n_params = sum(p.numel() for p in params)
    opt = model.configure_optimizers(0.1, 6e-4, (0.9, 0.95), "cuda")
    net = model
    if world > 1:
        # the reference's data parallelism (train.py:182-183): DDP's gradient buckets, each
        # all-reduced over NCCL as soon as the backward has produced it, overlapping the rest of the
        # backward; the buckets are the gradients' own storage (no packing copies). The step's
        # autograd graph is the same every iteration, so DDP runs in its static-graph mode (same
        # averaged gradients; at two GPUs config 4 took 16.5 ms per step against 17.4 without it)
        from torch.nn.parallel import DistributedDataParallel
        net = DistributedDataParallel(model, device_ids=[dev.index], gradient_as_bucket_view=True,
                                      bucket_cap_mb=bucket_mb, static_graph=True)
    T = cfg["max_seq_len"]
    host = [zipf_tokens(B, T + 1, cfg["vocab_size"], seed=1000 * rank + i).pin_memory() for i in range(4)]
    dtok = torch.empty(B, T + 1, dtype=torch.int64, device=dev)
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()

    def step(i):
        dtok.copy_(host[i % len(host)], non_blocking=True)
        net(dtok[:, :-1], dtok[:, 1:])
        model.last_loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)  # as train.py:287
        loss_host.copy_(model.last_loss.detach(), non_blocking=True)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        step(i)
    e1.record()
    torch.cuda.synchronize()
    secs = torch.tensor(e0.elapsed_time(e1) / 1e3, device=dev)
    if world > 1:
        dist.all_reduce(secs, op=dist.ReduceOp.MAX)
    secs = float(secs)
    out = {"metric": f"UnifiedLM training step tokens/s ({name}: dim {cfg['dim']}, {cfg['n_layers']} layers, "
                     f"M {cfg['hidden_dim']}, V {cfg['vocab_size']}, {B} x {T} per GPU)",
           "value": round(world * B * T * steps / secs, 1), "unit": "tokens/s", "n_gpus": world,
           "ms_per_step": round(secs / steps * 1e3, 3), "steps": steps, "warmup": warmup,
           "params": n_params, "grad_allreduce_bytes": 4 * n_params if world > 1 else 0,
           "h2d_bytes_per_step": B * (T + 1) * 8, "d2h_bytes_per_step": 4,
           "loss": round(float(loss_host), 4),
           "step": "token ids H2D from pinned memory, forward (fused head), backward with DDP's bucketed NCCL "
                   "all-reduce of all fp32 gradients overlapping it (N>1, static-graph mode), fused AdamW, loss "
                   "D2H; device time (CUDA events), max over ranks",
           "ddp_bucket_mb": bucket_mb if world > 1 else None, "ddp_static_graph": world > 1}
    del model, opt, net
    torch.cuda.empty_cache()
    return out


def bench_config3(dev, reps=5, warmup=2):
    """the fast-memory operator at D 512, M 1024, B 32, T in {512, 1024, 2048},
    lam in {0.9, 0.99, 0.999}, bf16 products with fp32 statistics, forward and backward timed
    separately (CUDA events, mean of `reps` launches after `warmup`). Addresses r are relu²-normalised
    from a Gaussian K u + b with eps 1; v bf16. The automatic choice is the whole-sequence form up to
    T = 2048; both forms are also timed at T = 2048 and at T = 8192, where the chunk-carry form wins."""
    import math
    import unifiedlm_c_b200._lib as L_
    from unifiedlm_c_b200.kernel import PRECISION, memory_bwd_raw, memory_fwd_raw, operand_or_input
    B, D, M = 32, 512, 1024  # BASELINE config 3 (T = 8192 extends it with 8 rows, same tokens per call)
    prec = PRECISION["bf16"]
    lib = L_.lib()
    gen = torch.Generator(device=dev).manual_seed(3)
    Kw = torch.randn(M, D, device=dev, generator=gen) / math.sqrt(D)
    bias = torch.randn(M, device=dev, generator=gen) * 0.5
    w = torch.full((M,), 4.0, device=dev)
    out = []

    def timed(fn):
        for _ in range(warmup):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3 / reps

    # (T, batch rows, lam values, chunk modes): the sweep in the automatic form choice, then both
    # forms at T = 2048 and at T = 8192 (same tokens per call) where the chunk-carry form takes over
    cases = [(T, B, (0.9, 0.99, 0.999), [-1]) for T in (512, 1024, 2048)]
    cases += [(2048, B, (0.99,), [1024]), (8192, 8, (0.99,), [-1, 0])]
    for T, Bc, lams, modes_T in cases:
        u = torch.randn(Bc, T, D, device=dev, generator=gen)
        z = torch.relu(u @ Kw.t() + bias).square()
        r = z / (1.0 + z.sum(-1, keepdim=True))
        del u, z
        v = torch.randn(Bc, T, D, device=dev, generator=gen).to(torch.bfloat16)
        dq = torch.randn(Bc, T, M, device=dev, generator=gen) * 1e-3
        df = (torch.randn(Bc, T, D, device=dev, generator=gen) * 1e-3).to(torch.bfloat16)
        for lam in lams:
            g = torch.tensor(math.log(lam), device=dev)
            for mode in modes_T:
                lib.ulm_set_chunk_mode(mode)
                C = int(lib.ulm_memory_chunk_len(T, M, D, prec))
                saved = memory_fwd_raw(r, None, v, g, w, prec)
                q, fast, c, qop, kop, vop, P = saved
                vop = operand_or_input(vop, v)
                t_f = timed(lambda: memory_fwd_raw(r, None, v, g, w, prec))
                t_b = timed(lambda: memory_bwd_raw(dq, df, r, None, g, w, q, c, qop, kop, vop, P, prec))
                out.append({"T": T, "B": Bc, "lam": lam, "form": f"chunk {C}" if C else "whole sequence",
                            "choice": "automatic" if mode == -1 else "forced",
                            "fwd_ms": round(t_f * 1e3, 3), "bwd_ms": round(t_b * 1e3, 3),
                            "fwd_tokens_per_s": round(Bc * T / t_f, 1), "bwd_tokens_per_s": round(Bc * T / t_b, 1)})
                del saved, q, fast, c, qop, kop, vop, P
        lib.ulm_set_chunk_mode(-1)
        del r, v, dq, df
        torch.cuda.empty_cache()
    return {"metric": "fast-memory operator fwd / bwd tokens/s (42M op sweep, D 512, M 1024, B 32)",
            "unit": "tokens/s", "precision": "bf16 products, fp32 statistics", "sweep": out}


def chunk_sweep(dev, reps=4, warmup=2):
    """fwd and bwd ms of unified_memory per form of the fast read (ulm_set_chunk_mode: 0 = the
    whole-sequence form, C = chunks of C) at D 512 / M 1024 and D 768 / M 2048, T in {2048, 4096,
    8192}, B = 65536 / T rows, bf16, lam 0.99; CUDA events, mean of `reps` calls after `warmup`."""
    import math
    import unifiedlm_c_b200._lib as L_
    from unifiedlm_c_b200.kernel import PRECISION, memory_bwd_raw, memory_fwd_raw, operand_or_input
    lib = L_.lib()
    prec = PRECISION["bf16"]

    def timed(fn):
        for _ in range(warmup):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    for D, M in ((512, 1024), (768, 2048)):
        for T in (2048, 4096, 8192):
            B = 65536 // T
            gen = torch.Generator(device=dev).manual_seed(1)
            z = torch.relu(torch.randn(B, T, M, device=dev, generator=gen)).square()
            r = z / (1.0 + z.sum(-1, keepdim=True))
            del z
            v = torch.randn(B, T, D, device=dev, generator=gen).to(torch.bfloat16)
            dq = torch.randn(B, T, M, device=dev, generator=gen) * 1e-3
            df = (torch.randn(B, T, D, device=dev, generator=gen) * 1e-3).to(torch.bfloat16)
            g = torch.tensor(math.log(0.99), device=dev)
            w = torch.full((M,), 4.0, device=dev)
            res = {}
            for mode in (0, 256, 512, 1024):
                lib.ulm_set_chunk_mode(mode)
                q, fast, c, qop, kop, vop, P = memory_fwd_raw(r, None, v, g, w, prec)
                vop = operand_or_input(vop, v)
                t_f = timed(lambda: memory_fwd_raw(r, None, v, g, w, prec))
                t_b = timed(lambda: memory_bwd_raw(dq, df, r, None, g, w, q, c, qop, kop, vop, P, prec))
                res["whole" if mode == 0 else f"chunk {mode}"] = {"fwd_ms": round(t_f, 3), "bwd_ms": round(t_b, 3)}
                del q, fast, c, qop, kop, vop, P
                torch.cuda.empty_cache()
            lib.ulm_set_chunk_mode(-1)
            print(json.dumps({"D": D, "M": M, "T": T, "B": B, "automatic": int(lib.ulm_memory_chunk_len(T, M, D, prec)),
                              "ms": res}), flush=True)
            del r, v, dq, df
            torch.cuda.empty_cache()


def runc_decode_baseline(steps=32):
    """The reference's own C decoder (run.c, built with its runomp flags into oracle/_ref/run_omp),
    greedy, at the 110M shape with seeded random weights, all host cores. Returns tokens/s or None."""
    binary = os.path.join(ROOT, "oracle", "_ref", "run_omp")
    if not os.path.exists(binary):
        return None
    load_package()
    from unifiedlm_c_b200 import export
    C = DECODE
    params = {k: v.cpu() for k, v in decode_params(C["D"], C["L"], C["M"], C["V"], "cpu").items()}
    with tempfile.TemporaryDirectory() as tmp:
        mpath, tpath = os.path.join(tmp, "model.bin"), os.path.join(tmp, "tok.bin")
        export.write_model_bin(params, mpath, max_seq_len=steps)
        export.write_tokenizer_bin(tpath, [f"|{i}" for i in range(C["V"])])
        env = dict(os.environ, OMP_NUM_THREADS=str(os.cpu_count() or 1))
        res = subprocess.run([binary, mpath, "-z", tpath, "-t", "0", "-n", str(steps)], capture_output=True,
                             text=True, env=env, timeout=600)
    for line in res.stderr.splitlines():
        if "achieved tok/s" in line:
            return {"value": float(line.split(":")[1]), "unit": "tokens/s", "cores": os.cpu_count() or 1,
                    "kind": "reference", "sample": f"run.c (runomp flags) greedy, batch 1, {steps} steps, "
                                                  "110M shape, seeded random weights"}
    return None


def timed_products(ulm_lib, L_, tensors, W, prec):
    """CUDA-event time of each tensor-core product launch of one block's fwd+bwd (the dominant
    kernel family), with its algorithmic flops. Returns (flops, seconds) summed over launches."""
    B, T, M, D = W["B"], W["T"], W["M"], W["D"]
    qop, kop, vop, P, doop, dS, dqf, dk, dv, fast, g = tensors
    ldm, ldd, ldt = L_.lib().ulm_operand_ld(M), L_.lib().ulm_operand_ld(D), L_.lib().ulm_operand_ld(T)
    st = torch.cuda.current_stream()
    sp = L_.stream_of(qop)
    pairs = T * (T + 1) // 2  # (t, s) pairs with s <= t
    lib = L_.lib()
    calls = [
        (2 * B * pairs * M, lambda: lib.ulm_decayed_scores(L_.ptr(qop), ldm, L_.ptr(kop), ldm, L_.ptr(P), ldt,
                                                           L_.ptr(g), B, T, M, prec, sp)),
        (2 * B * pairs * D, lambda: lib.ulm_causal_apply(L_.ptr(P), ldt, L_.ptr(vop), ldd, L_.ptr(fast), D,
                                                         L_.dtype_code(fast.dtype), 0, B, T, D, prec, sp)),
        (2 * B * pairs * D, lambda: lib.ulm_decayed_scores(L_.ptr(doop), ldd, L_.ptr(vop), ldd, L_.ptr(dS), ldt,
                                                           L_.ptr(g), B, T, D, prec, sp)),
        (2 * B * pairs * M, lambda: lib.ulm_causal_apply(L_.ptr(dS), ldt, L_.ptr(kop), ldm, L_.ptr(dqf), M,
                                                         L_.ULM_F32, 0, B, T, M, prec, sp)),
        (2 * B * pairs * M, lambda: lib.ulm_causal_apply(L_.ptr(dS), ldt, L_.ptr(qop), ldm, L_.ptr(dk), M,
                                                         L_.ULM_F32, 1, B, T, M, prec, sp)),
        (2 * B * pairs * D, lambda: lib.ulm_causal_apply(L_.ptr(P), ldt, L_.ptr(doop), ldd, L_.ptr(dv), D,
                                                         L_.dtype_code(dv.dtype), 1, B, T, D, prec, sp)),
    ]
    # compulsory DRAM bytes of each launch: its operands read once, its output written once (the
    # causal score matrices P and dS hold T (T + 1) / 2 entries per row)
    tri = B * pairs * P.element_size()
    btm, btd = B * T * M, B * T * D
    nbytes = [btm * qop.element_size() + btm * kop.element_size() + tri,
              tri + btd * vop.element_size() + btd * fast.element_size(),
              btd * doop.element_size() + btd * vop.element_size() + 2 * tri,
              tri + btm * kop.element_size() + btm * dqf.element_size(),
              tri + btm * qop.element_size() + btm * dk.element_size(),
              tri + btd * doop.element_size() + btd * dv.element_size()]
    calls = [(fl, fn, nb) for (fl, fn), nb in zip(calls, nbytes)]
    flops, secs = 0, 0.0
    per = []
    for fl, fn, nb in calls:
        L_.check(fn())  # warm
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        reps = 5
        torch.cuda.synchronize()
        ev[0].record(st)
        for _ in range(reps):
            L_.check(fn())
        ev[1].record(st)
        torch.cuda.synchronize()
        s = ev[0].elapsed_time(ev[1]) / 1e3 / reps
        per.append((fl, s, nb))
        flops += fl
        secs += s
    return flops, secs, per


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--precision", default="bf16", choices=["bf16", "fp32"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--grad-segments", type=int, default=1,
                    help="with N>1 ranks: all-reduce the gradients in this many runs of blocks, each started "
                         "as soon as its backward is issued (default 1: one all-reduce after the backward)")
    ap.add_argument("--no-decode", action="store_true", help="skip the batched-decode measurement")
    ap.add_argument("--no-mixer", action="store_true", help="skip the fused-combine measurement")
    ap.add_argument("--no-head", action="store_true", help="skip the fused LM-head measurement")
    ap.add_argument("--no-model", action="store_true", help="skip the UnifiedLM training-step measurements (c4, c2)")
    ap.add_argument("--no-config3", action="store_true", help="skip the config-3 operator sweep")
    ap.add_argument("--model-steps", type=int, default=10, help="timed UnifiedLM training steps (after 3 warm-up)")
    ap.add_argument("--nccl-max-ctas", type=int, default=0,
                    help="with N>1 ranks: at most this many CTAs per NCCL collective (0: NCCL's choice)")
    ap.add_argument("--ddp-bucket-mb", type=int, default=25, help="DDP gradient bucket size of the model steps")
    ap.add_argument("--profile-step", action="store_true",
                    help="run one warm-up step and one step, no timing or report (for ncu launch lists)")
    ap.add_argument("--profile-block", action="store_true",
                    help="run one block of the step (fwd + bwd) twice, no timing or report (for ncu captures "
                         "of single kernels on a small case)")
    ap.add_argument("--profile-decode", action="store_true",
                    help="run a few decode steps at the 110M shape (batch --profile-batch), no report (for ncu)")
    ap.add_argument("--profile-batch", type=int, default=16, help="batch of --profile-decode")
    ap.add_argument("--chunk-sweep", action="store_true",
                    help="time the fast read's two forms (whole sequence; chunks of 256 / 512 / 1024) fwd + bwd at the "
                         "42M and 110M widths for T in {2048, 4096, 8192}, 65536 tokens per call; prints one JSON "
                         "line per shape")
    ap.add_argument("--profile-model", action="store_true",
                    help="run two UnifiedLM training steps at config 4 (110M), no report (for ncu launch lists)")
    ap.add_argument("--profile-chunk", action="store_true",
                    help="run the config-3 operator at T=2048 (chunk-carry form), B=8, fwd + bwd twice, no report "
                         "(for ncu captures of the carry products)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    load_package()
    import unifiedlm_c_b200._lib as L_
    from unifiedlm_c_b200.kernel import memory_fwd, operand_copy, operand_or_input, PRECISION
    from unifiedlm_c_b200.prologue import address_fwd
    from unifiedlm_c_b200.block import addressed_memory_fwd, addressed_memory_bwd

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.profile_decode:
        from unifiedlm_c_b200.decode import BatchedDecoder
        C = DECODE
        Bp = args.profile_batch
        dec = BatchedDecoder(decode_params(C["D"], C["L"], C["M"], C["V"], dev), batch=Bp, precision="bf16",
                             device=dev, use_graph=False)
        dec.reset()
        dec.feed(torch.ones(Bp, dtype=torch.int32, device=dev))
        for _ in range(2):
            dec.step_greedy()
        torch.cuda.synchronize()
        return
    if args.chunk_sweep:
        chunk_sweep(dev)
        return
    if args.profile_model:
        bench_model(dev, "c4", 1, 1, 1, 0)
        return
    if args.profile_chunk:
        import math
        from unifiedlm_c_b200.kernel import unified_memory
        B, T, D, M = 8, 2048, 512, 1024
        gen = torch.Generator(device=dev).manual_seed(3)
        z = torch.relu(torch.randn(B, T, M, device=dev, generator=gen)).square()
        r = (z / (1.0 + z.sum(-1, keepdim=True))).requires_grad_(True)
        v = torch.randn(B, T, D, device=dev, generator=gen).to(torch.bfloat16).requires_grad_(True)
        g = torch.tensor(math.log(0.99), device=dev, requires_grad=True)
        w = torch.full((M,), 4.0, device=dev, requires_grad=True)
        for _ in range(2):
            q, fast = unified_memory(r, v, g, w)
            (q.sum() + fast.float().sum()).backward()
        torch.cuda.synchronize()
        return
    if world > 1:
        from datetime import timedelta
        opts = None
        if args.nccl_max_ctas > 0:
            # cap the SMs NCCL's kernels take, so a collective that overlaps the backward leaves the
            # persistent one-CTA-per-SM kernels most of the machine
            opts = dist.ProcessGroupNCCL.Options()
            opts.config.max_ctas = args.nccl_max_ctas
            opts.config.min_ctas = min(args.nccl_max_ctas, 2)
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120), pg_options=opts)
    W = dict(WORKLOAD, L=1) if args.profile_block else WORKLOAD
    prec = PRECISION[args.precision]
    hs, vs, dqs, dfs, blocks = make_inputs(W["B"], W["T"], W["M"], W["D"], W["L"], W["lam"], W["prior"], dev,
                                           seed=rank)
    from unifiedlm_c_b200.dp import GradBucket
    M_, D_ = W["M"], W["D"]
    # the path's parameter gradients in one flat bucket, DP-averaged every step: by default one NCCL
    # all-reduce after the last backward. With --grad-segments S the bucket is cut into S runs of
    # blocks, each packed and its all-reduce started as soon as the backward reaches its first
    # block, so the exchange overlaps the rest of the backward (DDP's gradient buckets)
    segs = args.grad_segments if world > 1 else 1
    if W["L"] % segs:
        raise SystemExit(f"--grad-segments {segs} does not divide the {W['L']} blocks")
    grad_shapes = [(M_, D_), (M_,), (D_, 1, 4), (), (M_,), ()] * W["L"]
    bucket = GradBucket(grad_shapes, device=dev, segments=segs)

    def step(hs_, vs_, dqs_, dfs_, before_bwd=None, bk=None, after_segment=None):
        """One training step of the path, in a model's order: every block's forward (block i on
        hs_[i], vs_[i]), then the backward from the last block to the first (on dqs_[i], dfs_[i]),
        the gradients packed into bucket `bk` (default `bucket`) segment by segment. `before_bwd`
        runs between the two phases (the e2e loop makes the stream wait there for the gradient
        inputs, which it copies last); `after_segment(s)` runs once segment s is packed (and, with N
        ranks, its all-reduce started)."""
        bk = bucket if bk is None else bk
        per_seg = len(blocks) // bk.segments
        saved = []
        for blk, h_, v_ in zip(blocks, hs_, vs_):
            saved.append(addressed_memory_fwd(h_, blk["conv"], blk["key_w"], blk["key_b"], blk["eps"], v_,
                                              blk["g"], blk["w"], prec))
        if before_bwd is not None:
            before_bwd()
        grads = [None] * len(blocks)
        for i in reversed(range(len(blocks))):
            blk = blocks[i]
            q, fast, z, den, u_op, kw, c, qop, kop, vop, P = saved[i]
            saved[i] = None
            dh, dconv, dkw, dkb, deps, dv, dg, dw = addressed_memory_bwd(
                dqs_[i], dfs_[i], hs_[i], blk["conv"], blk["g"], blk["w"], q, z, den, u_op, kw, c, qop, kop,
                operand_or_input(vop, vs_[i]), P, prec)
            grads[i] = [dkw, dkb, dconv, deps, dw, dg]
            if i % per_seg == 0:
                bk.pack_segment(i // per_seg, [t for g6 in grads[i:i + per_seg] for t in g6])
                bk.start_segment(i // per_seg)
                if after_segment is not None:
                    after_segment(i // per_seg)
        bk.finish(average=True)
        return bk.flat

    if args.profile_step or args.profile_block:
        step(hs, vs, dqs, dfs)
        step(hs, vs, dqs, dfs)
        torch.cuda.synchronize()
        if world > 1:
            dist.destroy_process_group()
        return
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # the sampler starts with the warm-up so that short timed regions still see >= 1 sample under load
    with ClockSampler(local) as clocks:
        for _ in range(args.warmup):
            step(hs, vs, dqs, dfs)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        ev0.record()
        for _ in range(args.steps):
            step(hs, vs, dqs, dfs)
        ev1.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    secs = torch.tensor(ev0.elapsed_time(ev1) / 1e3, device=dev)
    if world > 1:
        dist.all_reduce(secs, op=dist.ReduceOp.MAX)
    secs = float(secs)
    tokens = world * W["B"] * W["T"] * args.steps
    value = tokens / secs
    if L_.device_error() != 0:
        raise RuntimeError("a kernel reported a device-side error during the bench")

    # e2e: every step's inputs copied from pinned host memory and its parameter gradients read back,
    # pipelined as a training loop with a prefetching loader does it: the host-to-device copy of
    # step i+1 runs on its own stream during step i (two device input slots), and the gradients are
    # read back on another stream into one of two pinned host buffers (two device buckets). On one
    # GPU each block's gradients are read back as soon as its backward has packed them, so only the
    # first block's 6 MB remain after the last step; with N ranks the read follows the all-reduce,
    # on rank 0 only (after the all-reduce every rank holds the same averaged gradients, so one copy
    # is the job's result; N reads of it would only add host traffic). The timed region spans the
    # first copy to the last read, the maximum over ranks. The inputs copied are the step's
    # ends, as a model's would be: the first block's h and v and the last block's upstream
    # gradients dq_out and dfast; the other blocks read their own device-resident inputs, which in
    # a model their neighbouring blocks write.
    host = [t.cpu().pin_memory() for t in (hs[0], vs[0], dqs[-1], dfs[-1])]
    slots_in = [[torch.empty_like(t, device=dev) for t in host] for _ in range(2)]

    def slot_inputs(k):
        h_, v_, dq_, df_ = slots_in[k]
        return [h_] + hs[1:], [v_] + vs[1:], dqs[:-1] + [dq_], dfs[:-1] + [df_]
    out_buckets = [GradBucket(grad_shapes, device=dev, segments=W["L"] if world == 1 else segs) for _ in range(2)]
    host_out = [torch.empty(bucket.flat.shape, dtype=bucket.flat.dtype).pin_memory() for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = host_out[0].numel() * host_out[0].element_size()
    main_s = torch.cuda.current_stream(dev)
    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def e2e_run(n, start_ev=None):
        # per slot: the forward inputs (h, v) and the gradient inputs (dq_out, dfast) have arrived
        in_ready = [torch.cuda.Event() for _ in range(2)]
        grad_ready = [torch.cuda.Event() for _ in range(2)]
        in_free = [None, None]    # the step that last read the slot has finished
        out_free = [None, None]   # the read of the bucket's previous result has finished

        def copy_in(i):
            k = i % 2
            with torch.cuda.stream(h2d_s):
                if start_ev is not None and i == 0:
                    h2d_s.wait_event(start_ev)
                if in_free[k] is not None:
                    h2d_s.wait_event(in_free[k])
                for j, (d_, h_) in enumerate(zip(slots_in[k], host)):
                    d_.copy_(h_, non_blocking=True)
                    if j == 1:
                        in_ready[k].record(h2d_s)
                grad_ready[k].record(h2d_s)

        def read_back(src, dst):
            ready = torch.cuda.Event()
            ready.record(main_s)
            with torch.cuda.stream(d2h_s):
                d2h_s.wait_event(ready)
                dst.copy_(src, non_blocking=True)

        copy_in(0)
        for i in range(n):
            k = i % 2
            bk = out_buckets[k]
            main_s.wait_event(in_ready[k])
            if out_free[k] is not None:  # the read of step i-2's gradients (done during step i-1)
                main_s.wait_event(out_free[k])
            if i + 1 < n:
                copy_in(i + 1)
            per_segment = None
            if world == 1:
                def per_segment(s_, bk=bk, dst=host_out[k]):
                    a, b = bk.offsets[s_ * bk.per_segment], bk.offsets[(s_ + 1) * bk.per_segment]
                    read_back(bk.segment(s_), dst[a:b])
            out = step(*slot_inputs(k), before_bwd=lambda k=k: main_s.wait_event(grad_ready[k]), bk=bk,
                       after_segment=per_segment)
            ev = torch.cuda.Event()
            ev.record(main_s)
            in_free[k] = ev
            if world > 1 and rank == 0:
                read_back(out, host_out[k])
            done = torch.cuda.Event()
            done.record(d2h_s)
            out_free[k] = done
        main_s.wait_stream(d2h_s)
        main_s.wait_stream(h2d_s)

    e2e_run(2)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # at least 20 steps: the first step's copy-in (235 MB, nothing to overlap it with) is the loop's
    # one-time fill and stays inside the timed region, spread over more steps as in a training run
    e2e_steps = max(20, args.steps)
    e0.record(main_s)
    e2e_run(e2e_steps, start_ev=e0)
    e1.record(main_s)
    torch.cuda.synchronize()
    e2e_secs = torch.tensor(e0.elapsed_time(e1) / 1e3, device=dev)
    if world > 1:
        dist.all_reduce(e2e_secs, op=dist.ReduceOp.MAX)
    e2e_value = world * W["B"] * W["T"] * e2e_steps / float(e2e_secs)
    del slots_in, out_buckets, host_out, host

    # roofline of the dominant kernel family (tensor-core products), CUDA events per launch
    blk0 = blocks[0]
    g, w = blk0["g"], blk0["w"]
    h, v, dfast = hs[0], vs[0], dfs[0]
    r, _, _, _ = address_fwd(h, blk0["conv"], blk0["key_w"], blk0["key_b"], blk0["eps"], prec)
    q, fast, c, qop, kop, vop, P = memory_fwd(r, v, g, w, prec)
    vop = operand_or_input(vop, v)
    ldd, ldt = L_.lib().ulm_operand_ld(W["D"]), L_.lib().ulm_operand_ld(W["T"])
    opt = qop.dtype
    doop = torch.zeros(W["B"], W["T"], ldd, device=dev, dtype=opt)
    doop[..., :W["D"]] = dfast.to(opt)
    dS = torch.empty(W["B"], W["T"], ldt, device=dev, dtype=opt)
    dqf = torch.empty(W["B"], W["T"], W["M"], device=dev)
    dk = torch.empty_like(dqf)
    # outputs in the step's types: fast and dv in v's / dfast's type, dq and dk fp32
    dvb = torch.empty(W["B"], W["T"], W["D"], device=dev, dtype=dfast.dtype)
    fastb = torch.empty(W["B"], W["T"], W["D"], device=dev, dtype=v.dtype)
    flops, psecs, per = timed_products(None, L_, (qop, kop, vop, P, doop, dS, dqf, dk, dvb, fastb, g), W, prec)
    pk = peaks()
    achieved = flops / psecs / 1e12
    # each product's own roofline time: the slower of its flops at the tensor peak and its compulsory
    # bytes at the copy peak (dq and dk write fp32 T x M gradients, so their bytes bound them)
    floors = [max(f / (pk["bf16_tflops"] * 1e12), nb / (pk["hbm_gbs"] * 1e9)) for f, _, nb in per]
    roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": round(achieved / pk["bf16_tflops"], 4), "traffic": PRODUCTS_DRAM_BYTES,
                "traffic_note": "dram__bytes_read.sum + dram__bytes_write.sum of the six products of one block, "
                                "from one-kernel ncu captures of bench.py --profile-block",
                "algorithmic_flops_per_block": flops,
                "kernel": "tc2_gemm_kernel (6 causal products per block fwd+bwd)",
                "peak_source": pk["source"],
                "per_launch_ms": [round(s * 1e3, 4) for _, s, _ in per],
                "per_launch_tflops": [round(f / s / 1e12, 1) for f, s, _ in per],
                "per_launch_compulsory_mb": [round(nb / 1e6, 1) for _, _, nb in per],
                "per_launch_floor_ms": [round(t * 1e3, 4) for t in floors],
                "floor_frac": round(sum(floors) / psecs, 4),
                "floor_note": "per product max(flops / bf16 peak, compulsory bytes / hbm peak); floor_frac = "
                              "sum of those times / sum of the measured launch times"}

    models = None
    if not args.no_model:
        models = {name: bench_model(dev, name, args.model_steps, 3, world, rank, args.ddp_bucket_mb)
                  for name in ("c4", "c2")}
        if L_.device_error() != 0:
            raise RuntimeError("a kernel reported a device-side error during the model steps")
    config3 = None
    if world == 1 and not args.no_config3:
        config3 = bench_config3(dev)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        s = cpu_reference_seconds(W["T"], W["M"], W["D"], W["lam"], W["prior"], 15, threads)
        cpu = {"value": W["T"] / (W["L"] * s), "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": f"1 seq x 1 block (T={W['T']}, M={W['M']}, D={W['D']}) fwd+bwd, median of 15, prologue + chunked "
                         "pure-PyTorch form (model.py:70-79, test_all.py:28-51 restated in oracle/memory.py), "
                         "fp32, scaled to 12 blocks"}

    mixer = None
    if world == 1 and not args.no_mixer:
        mixer = bench_mixer(dev, W, blocks, args.precision)
    head = None
    if world == 1 and not args.no_head:
        head = bench_head(dev, W)

    decode = None
    if not args.no_decode:
        decode = bench_decode(dev, pk)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            decode["cpu_baseline"] = runc_decode_baseline()

    # kernels of ours per step, per block: prologue fwd 3 (conv, key GEMM, den); operator fwd 3
    # (stats scan, scores, read) + the conversion of v to the operand type when v is not already
    # one; operator bwd 7 (scores grad, dq, dk, dv, stats scan, dw, dg) + the conversion of dfast
    # likewise; prologue bwd 9 (address backward, db column sums + their sum, deps, dK GEMM, dK sum,
    # du GEMM, conv bwd, dconv sum)
    opt_dtype = torch.float32 if args.precision == "fp32" else torch.bfloat16
    converts = sum(int(operand_copy(x, opt_dtype) is not x) for x in (v, dfast))
    launches = args.steps * W["L"] * (3 + 3 + 7 + 9 + converts)
    line = {"metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(secs / args.steps * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": args.precision, "data": "synthetic",
            "config": dict(workload_config(W), parallelism=f"dp{world}", grad_allreduce_segments=segs,
                           l2="every block reads its own inputs (235 MB per block); r is 134 MB; no flush"),
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "d2h_ranks": 1, "steps": e2e_steps,
                    "h2d_gbs_per_rank": round(h2d * e2e_steps / float(e2e_secs) / 1e9, 1),
                    "h2d_gbs_all_ranks": round(world * h2d * e2e_steps / float(e2e_secs) / 1e9, 1),
                    "copies": "pinned host buffers; H2D of step i+1 during step i on its own stream "
                              "(double-buffered; forward inputs first, the step waits for the gradient inputs "
                              "before its backward); the gradients read back on another stream, per block as "
                              "the backward packs them on one GPU, after the all-reduce and by rank 0 alone "
                              "with N ranks (every rank holds the same averaged gradients); timed from the first "
                              "copy (the loop's unoverlapped fill) to the last read over max(20, steps) steps, max "
                              "over ranks"},
            "roofline": roofline, "cpu_baseline": cpu, "clocks": clocks.summary(), "gpu_launches": launches,
            "mixer": mixer, "head": head, "decode": decode, "model_step": models, "config3": config3}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
