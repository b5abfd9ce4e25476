"""Batched greedy decode on the GPU: UnifiedLM.forward_recurrent / run.c generate for B sequences.

The reference decodes one sequence at a time, token by token, either in Python
(UnifiedLM.forward_recurrent, model.py:164-175) or in C (run.c forward, run.c:193-265). Here a
`BatchedDecoder` keeps the constant-size state of every block for B sequences on the device
(U (B,D,M) fp32, c and r_prev (B,M), the conv window (B,D,conv_size-1)) and advances all of them
one token per step through libulm_b200.so (ulm_decode_* in include/ulm_b200.h). A step has no
allocation and no host synchronisation, so it is captured once in a CUDA graph and replayed.

precision "fp32": fp32 weights and FMA contractions, run.c's order in the state update (the mode
for token identity with run.c). "bf16": bf16 weights on the tensor cores, fp32 state.
"""
import math

import torch

from . import _lib as L


class BatchedDecoder:
    def __init__(self, params, batch, precision="fp32", device="cuda", norm_eps=1e-5, use_graph=True):
        """params: a UnifiedLM state_dict-like mapping (reference parameter names)."""
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
        self.K = params["layers.0.conv.weight"].shape[-1]
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
                "norm": f32(p("norm.weight")), "conv": f32(p("conv.weight")[:, 0, :]),
                "key_w": wt(p("key.weight")), "key_b": f32(p("key.bias")), "val_w": wt(p("val.weight")),
                "mu": f32(p("mu.weight")),
                "w": f32(torch.exp(torch.clamp(p("log_w").double(), -7.0, 12.0))),
                "lam": f32(torch.exp(-torch.exp(p("log_rate").double())).reshape(1)),
                "eps": f32(torch.exp(torch.clamp(p("log_eps").double(), -10.0, 10.0)).reshape(1)),
            }
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
        self.graph = None
        self.use_graph = use_graph

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

    def _layers_and_head(self):
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

    def _run_step(self):
        if not self.use_graph:
            self._layers_and_head()
            return
        if self.graph is None:
            side = torch.cuda.Stream(self.dev)
            side.wait_stream(torch.cuda.current_stream(self.dev))
            with torch.cuda.stream(side):  # warm-up outside capture (first-call set-up in the library)
                self._layers_and_head()
            torch.cuda.current_stream(self.dev).wait_stream(side)
            # the warm-up advanced the state: restore it after capture by the caller's reset/replay order
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self._layers_and_head()
            return "captured"
        self.graph.replay()

    def feed(self, tokens):
        """Advance every sequence by one token (int tensor (B,) on any device). Returns the greedy
        next tokens (int32 (B,) on the device); self.logits holds the logits."""
        self.tokens_in.copy_(tokens.to(self.tokens_in.dtype), non_blocking=True)
        L.check(L.lib().ulm_decode_embed(L.ptr(self.tokens_in), L.ptr(self.emb), self.wcode, L.ptr(self.x),
                                         self.B, self.D, L.stream_of(self.x)))
        self._run_step()
        return self.next_token

    def step_greedy(self):
        """Advance every sequence by its own last greedy token (x already holds its embedding)."""
        self._run_step()
        return self.next_token

    def prepare_graph(self):
        """Capture the step graph (runs the step twice on scratch state), then reset."""
        if self.use_graph and self.graph is None:
            self.reset()
            self._run_step()
        self.reset()

    @torch.no_grad()
    def generate(self, prompt, steps, bos=1, stop_at_bos=False):
        """Greedy continuation of `prompt` (B, P) ints, as run.c generate() with temperature 0:
        the prompt is fed token by token, then each step feeds the previous greedy token.
        Returns (B, steps) int64 on the host: the tokens produced after each fed token (positions
        inside the prompt report the greedy guess there)."""
        self.prepare_graph()
        prompt = prompt.to(self.dev)
        out = []
        P = prompt.shape[1]
        for t in range(P):
            nt = self.feed(prompt[:, t])
            out.append(nt.clone())
        for _ in range(steps - P):
            nt = self.step_greedy()
            out.append(nt.clone())
        return torch.stack(out, 1).long().cpu()

    def state_bytes(self):
        return self.L * self.B * (self.D * self.M + 2 * self.M + self.D * max(self.K - 1, 1)) * 4
