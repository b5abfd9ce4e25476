"""Batched greedy decode on the GPU: UnifiedLM.forward_recurrent / run.c generate for B sequences.

The reference decodes one sequence at a time, token by token, either in Python
(UnifiedLM.forward_recurrent, model.py:164-175) or in C (run.c forward, run.c:193-265). Here a
`BatchedDecoder` keeps the constant-size state of every block for B sequences on the device
(U (B,D,M) fp32, c and r_prev (B,M), the conv window (B,D,conv_size-1)) and advances all of them
one token per step through libulm_b200.so (ulm_decode_* in include/ulm_b200.h). A step has no
allocation and no host synchronisation, so it is captured once in a CUDA graph and replayed.

precision "fp32": fp32 weights and FMA contractions, run.c's order in the state update (the mode
for token identity with run.c). "bf16": bf16 weights on the tensor cores, fp32 state.

Sampling: temperature 0 is run.c's greedy pick; temperature > 0 samples on the device as run.c's
sample() does (softmax of logits / temperature, a coin from a xorshift64* state per sequence, then
multinomial or top-p), with sequence b seeded by seed + b (or seeds[b]), so sequence 0 follows
run.c run with `-s seed`. `BatchedDecoder.from_model_bin` loads run.c's model.bin directly.
"""
import math

import torch

from . import _lib as L


def rmsnorm_rows(x, weight, eps):
    """RMSNorm of the residual stream rows in fp32, as the decode step applies it:
    weight * (x / sqrt(mean(x^2) + eps))."""
    return weight * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps))


class BatchedDecoder:
    def __init__(self, params, batch, precision="fp32", device="cuda", norm_eps=1e-5, use_graph=True,
                 temperature=0.0, topp=0.9, seed=0):
        """params: a UnifiedLM state_dict-like mapping (reference parameter names), or the tensors
        of a model.bin (export.read_model_bin: per block `conv` (D,K) and the derived `w`, `lam`,
        `eps`, used exactly as run.c uses them)."""
        self.B = int(batch)
        self.dev = torch.device(device)
        self.prec = precision
        self.wdt = torch.float32 if precision == "fp32" else torch.bfloat16
        self.wcode = L.dtype_code(self.wdt)
        self.norm_eps = float(norm_eps)
        f32 = lambda t: t.detach().to(self.dev, torch.float32).contiguous()  # noqa: E731
        wt = lambda t: t.detach().to(self.dev, self.wdt).contiguous()  # noqa: E731
        self.L = 1 + max(int(k.split(".")[1]) for k in params if k.startswith("layers."))
        emb = params["tok_embeddings.weight"]
        self.V, self.D = emb.shape
        self.M = params["layers.0.key.weight"].shape[0]
        derived = "layers.0.lam" in params  # model.bin layout
        self.K = params["layers.0.conv" if derived else "layers.0.conv.weight"].shape[-1]
        if self.M % 4:
            raise ValueError("the batched decoder needs hidden_dim % 4 == 0")
        self.emb = wt(emb)
        head = params.get("output.weight", emb)
        self.cls = self.emb if head.data_ptr() == emb.data_ptr() or torch.equal(head, emb) else wt(head)
        self.final_norm = f32(params["norm.weight"])
        lib = L.lib()
        B, D, M = self.B, self.D, self.M
        self.layers = []
        for i in range(self.L):
            p = lambda n: params[f"layers.{i}.{n}"]  # noqa: E731
            lay = {
                "norm": f32(p("norm.weight")), "key_w": wt(p("key.weight")), "key_b": f32(p("key.bias")),
                "val_w": wt(p("val.weight")), "mu": f32(p("mu.weight")),
            }
            if derived:
                lay.update(conv=f32(p("conv")), w=f32(p("w")), lam=f32(p("lam").reshape(1)),
                           eps=f32(p("eps").reshape(1)))
            else:
                lay.update(conv=f32(p("conv.weight")[:, 0, :]),
                           w=f32(torch.exp(torch.clamp(p("log_w").double(), -7.0, 12.0))),
                           lam=f32(torch.exp(-torch.exp(p("log_rate").double())).reshape(1)),
                           eps=f32(torch.exp(torch.clamp(p("log_eps").double(), -10.0, 10.0)).reshape(1)))
            lay["g"] = torch.log(lay["lam"]).reshape(())  # log decay, for the parallel prefill's products
            lay["prior"] = torch.empty(D, M, device=self.dev, dtype=self.wdt)
            lay["U"] = torch.empty(B, D, M, device=self.dev)
            lay["c"] = torch.empty(B, M, device=self.dev)
            lay["r_prev"] = torch.empty(B, M, device=self.dev)
            lay["buf"] = torch.empty(B, D, max(self.K - 1, 1), device=self.dev)
            self.layers.append(lay)
        self.x = torch.zeros(B, D, device=self.dev)
        self.logits = torch.empty(B, self.V, device=self.dev)
        self.next_token = torch.zeros(B, device=self.dev, dtype=torch.int32)
        self.tokens_in = torch.zeros(B, device=self.dev, dtype=torch.int32)
        self.work = torch.empty(int(lib.ulm_decode_block_work_bytes(B, D, M)), device=self.dev, dtype=torch.uint8)
        self.head_work = torch.empty(int(lib.ulm_decode_head_work_bytes(B, D)), device=self.dev, dtype=torch.uint8)
        with torch.cuda.device(self.dev):
            st = L.stream_of(self.x)
            for lay in self.layers:
                L.check(lib.ulm_decode_prepare_block(L.ptr(lay["mu"]), L.ptr(lay["w"]), L.ptr(lay["lam"]),
                                                     L.ptr(lay["prior"]), self.wcode, D, M, st))
        self.temperature = float(temperature)
        self.topp = float(topp)
        seeds = list(seed) if isinstance(seed, (list, tuple)) else [int(seed) + b for b in range(B)]
        if len(seeds) != B:
            raise ValueError("one seed per sequence")
        # one 64-bit xorshift state per sequence (stored as int64 with the same bits)
        to_i64 = lambda u: u - (1 << 64) if u >= (1 << 63) else u  # noqa: E731
        self.rng = torch.tensor([to_i64(s_ & 0xFFFFFFFFFFFFFFFF) for s_ in seeds], dtype=torch.int64,
                                device=self.dev)
        self.graphs = {}
        self.use_graph = use_graph

    @classmethod
    def from_model_bin(cls, path, batch, precision="fp32", device="cuda", **kw):
        """A decoder over run.c's checkpoint file (model.bin v1, export.py:37-81)."""
        from .export import read_model_bin
        cfg, tensors = read_model_bin(path)
        return cls(tensors, batch, precision=precision, device=device, **kw)

    # -------------------------------------------------------------------------------------------
    def reset(self):
        """Fresh state for every sequence (UnifiedBlock.init_state / run.c reset_state)."""
        lib = L.lib()
        with torch.cuda.device(self.dev):
            st = L.stream_of(self.x)
            for lay in self.layers:
                L.check(lib.ulm_decode_reset_block(L.ptr(lay["mu"]), L.ptr(lay["w"]), L.ptr(lay["U"]),
                                                   L.ptr(lay["c"]), L.ptr(lay["r_prev"]), L.ptr(lay["buf"]),
                                                   self.B, self.D, self.M, self.K, st))

    def _layers_and_head(self, sample=False):
        lib = L.lib()
        st = L.stream_of(self.x)
        B, D, M = self.B, self.D, self.M
        for lay in self.layers:
            L.check(lib.ulm_decode_block_step(
                L.ptr(self.x), L.ptr(lay["norm"]), L.ptr(lay["conv"]), L.ptr(lay["key_w"]), L.ptr(lay["key_b"]),
                L.ptr(lay["val_w"]), L.ptr(lay["prior"]), self.wcode, L.ptr(lay["w"]), L.ptr(lay["lam"]),
                L.ptr(lay["eps"]), L.ptr(lay["U"]), L.ptr(lay["c"]), L.ptr(lay["r_prev"]), L.ptr(lay["buf"]),
                L.ptr(self.work), B, D, M, self.K, self.norm_eps, st))
        L.check(lib.ulm_decode_head(L.ptr(self.x), L.ptr(self.final_norm), L.ptr(self.cls), L.ptr(self.emb),
                                    self.wcode, L.ptr(self.logits), L.ptr(self.next_token), L.ptr(self.head_work),
                                    B, D, self.V, self.norm_eps, st))
        if sample:
            L.check(lib.ulm_decode_sample(L.ptr(self.logits), B, self.V, self.temperature, self.topp,
                                          L.ptr(self.rng), L.ptr(self.next_token), L.ptr(self.emb), self.wcode,
                                          L.ptr(self.x), D, st))

    def _run_step(self, sample=False):
        """One token for every sequence; with `sample` the next token is drawn (temperature > 0)
        instead of the greedy pick, advancing each sequence's random state."""
        sample = bool(sample and self.temperature > 0.0)
        if not self.use_graph:
            self._layers_and_head(sample)
            return
        if sample not in self.graphs:
            rng0 = self.rng.clone()
            side = torch.cuda.Stream(self.dev)
            side.wait_stream(torch.cuda.current_stream(self.dev))
            with torch.cuda.stream(side):  # warm-up outside capture (first-call set-up in the library)
                self._layers_and_head(sample)
            torch.cuda.current_stream(self.dev).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self._layers_and_head(sample)
            self.graphs[sample] = graph
            self.rng.copy_(rng0)  # the warm-up must not consume random draws
            return "captured"
        self.graphs[sample].replay()

    def feed(self, tokens, sample=False):
        """Advance every sequence by one token (int tensor (B,) on any device). Returns the next
        tokens (int32 (B,) on the device: greedy, or drawn when `sample` and temperature > 0);
        self.logits holds the logits."""
        self.tokens_in.copy_(tokens.to(self.tokens_in.dtype), non_blocking=True)
        L.check(L.lib().ulm_decode_embed(L.ptr(self.tokens_in), L.ptr(self.emb), self.wcode, L.ptr(self.x),
                                         self.B, self.D, L.stream_of(self.x)))
        self._run_step(sample)
        return self.next_token

    def step_greedy(self):
        """Advance every sequence by its own last greedy token (x already holds its embedding)."""
        self._run_step()
        return self.next_token

    def step_sample(self):
        """Advance every sequence by its own last token and draw the next one (temperature > 0;
        greedy at temperature 0)."""
        self._run_step(sample=True)
        return self.next_token

    def prepare_graph(self):
        """Capture the step graphs (each runs the step on scratch state), then reset."""
        if self.use_graph:
            for sample in ((False, True) if self.temperature > 0.0 else (False,)):
                if sample not in self.graphs:
                    self.reset()
                    self._run_step(sample)
        self.reset()

    @torch.no_grad()
    def generate(self, prompt, steps, bos=1, stop_at_bos=False):
        """Continuation of `prompt` (B, P) ints, as run.c generate(): the prompt is fed token by
        token, then each step feeds the previous token; the token after the last prompt token and
        all later ones are drawn by the sampler (greedy at temperature 0; random draws only there,
        as run.c calls sample() only past the prompt). Returns (B, steps) int64 on the host: the
        token produced after each fed token (positions inside the prompt report the greedy guess)."""
        self.prepare_graph()
        prompt = prompt.to(self.dev)
        out = []
        P = prompt.shape[1]
        for t in range(P):
            out.append(self.feed(prompt[:, t], sample=(t == P - 1)).clone())
        for _ in range(steps - P):
            nt = self.step_sample()
            out.append(nt.clone())
        return torch.stack(out, 1).long().cpu()

    @torch.no_grad()
    def prefill(self, prompt):
        """Feed a whole prompt (B, P) ints in one parallel pass instead of P steps: every block runs
        its training-form forward over the P positions (the addressing prologue, the fast memory and
        the combine, libulm_b200.so) and its state is then set to what P token-by-token steps leave
        (ulm_decode_prefill_block: U = w mu + sum_s lam^(P-1-s) v_s k_s^T from one carry product,
        c, r_prev and the conv window). The last position's logits go through the decode head.
        Returns the next tokens (greedy, int32 (B,) on the device); self.logits holds the logits."""
        from .block import mixer_fwd_raw
        prompt = prompt.to(self.dev)
        B, P = prompt.shape
        if B != self.B:
            raise ValueError(f"prompt batch {B} != decoder batch {self.B}")
        lib = L.lib()
        prec = L.ULM_PREC_FP32 if self.prec == "fp32" else L.ULM_PREC_BF16
        st = L.stream_of(self.x)
        x = self.emb[prompt.long()].float()
        work = torch.empty(int(lib.ulm_decode_prefill_work_bytes(B, P, self.D, prec)), device=self.dev,
                           dtype=torch.uint8)
        for lay in self.layers:
            h = rmsnorm_rows(x, lay["norm"], self.norm_eps)
            v = (h.to(self.wdt) @ lay["val_w"].t()).to(self.wdt if self.prec == "bf16" else torch.float32)
            y, z, den, kop, vop = mixer_fwd_raw(x, h, lay["conv"][:, None, :], lay["key_w"], lay["key_b"],
                                                lay["eps"].reshape(()), v, lay["g"], lay["w"], lay["mu"], prec)
            with torch.cuda.device(self.dev):
                L.check(lib.ulm_decode_prefill_block(
                    L.ptr(kop), L.ptr(vop), L.ptr(lay["g"]), L.ptr(lay["lam"]), L.ptr(z), L.ptr(den), L.ptr(h),
                    L.dtype_code(h.dtype), L.ptr(lay["mu"]), L.ptr(lay["w"]), L.ptr(work), L.ptr(lay["U"]),
                    L.ptr(lay["c"]), L.ptr(lay["r_prev"]), L.ptr(lay["buf"]), B, P, self.D, self.M, self.K, prec,
                    st))
            x = y
        self.x.copy_(x[:, -1])
        with torch.cuda.device(self.dev):
            L.check(lib.ulm_decode_head(L.ptr(self.x), L.ptr(self.final_norm), L.ptr(self.cls), L.ptr(self.emb),
                                        self.wcode, L.ptr(self.logits), L.ptr(self.next_token),
                                        L.ptr(self.head_work), B, self.D, self.V, self.norm_eps, st))
        return self.next_token

    def state_bytes(self):
        return self.L * self.B * (self.D * self.M + 2 * self.M + self.D * max(self.K - 1, 1)) * 4
