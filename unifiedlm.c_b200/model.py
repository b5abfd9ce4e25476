"""Drop-in replacement of the reference's model.py with the fast memory on sm_100a.

ModelArgs, RMSNorm, UnifiedBlock and UnifiedLM keep the reference's constructor arguments,
parameter names, shapes and initialisation (model.py:13-204), so state_dicts, checkpoints and the
model.bin exporter interoperate unchanged. UnifiedBlock.forward routes the addressing prologue, the
fast read and the `mu` combine with the residual to `block.block_mixer` (libulm_b200.so; the same
result as `x + mu(q w) + fast` with `q, fast = kernel.unified_memory(prologue.address(...))`,
without materialising the normalised addresses or q); with dropout active in training the combine
runs as the reference's separate Linear. The val projection and RMSNorm stay PyTorch (cuBLAS).
`step` / `init_state` / `forward_recurrent` keep the reference's token-by-token semantics
(model.py:88-111, 164-175) for small-batch use, and `decode.py` holds the batched CUDA decoder.

The block's precision follows `UnifiedBlock.precision` ("bf16" tensor-core products, default; or
"fp32" for the 1e-5 parity mode), set for a whole model by `UnifiedLM.set_precision`.
"""
import inspect
import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .block import addressed_memory, block_mixer
from .head import lm_head_loss
from .kernel import CHUNK


@dataclass
class ModelArgs:
    dim: int = 288
    n_layers: int = 12          # number of UnifiedBlocks
    hidden_dim: int = 712       # memory slots per block
    vocab_size: int = 32000
    max_seq_len: int = 256
    norm_eps: float = 1e-5
    dropout: float = 0.0
    conv_size: int = 4          # causal depthwise conv on the address path
    prior: float = 4.0          # initial prior mass w of every slot, in tokens


def _hi(x):
    """Slot statistics in fp32 even under bf16/fp16 autocast (model.py:26-28)."""
    return x.float() if x.dtype in (torch.float16, torch.bfloat16) else x


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = _hi(x)
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).type_as(x) * self.weight


class UnifiedBlock(nn.Module):
    """One associative memory whose slots hold running posterior means (model.py:45-111):

        address  r_t = normalize(relu(K u_t + b)^2),  u_t = causal depthwise conv(RMSNorm(x_t))
        write    key r_{t-1}, value v_t = W_v h_t
        read     y_t = sum_a r_t,a (w_a mu_a + sum_{s<=t} lam^(t-s) r_{s-1,a} v_s)
                                 / (w_a      + sum_{s<=t} lam^(t-s) r_{s-1,a})
    """

    def __init__(self, args: ModelArgs):
        super().__init__()
        d, m = args.dim, args.hidden_dim
        self.norm = RMSNorm(d, eps=args.norm_eps)
        self.conv = nn.Conv1d(d, d, args.conv_size, groups=d, padding=args.conv_size - 1, bias=False)
        self.key = nn.Linear(d, m, bias=True)
        self.mu = nn.Linear(m, d, bias=False)
        self.log_eps = nn.Parameter(torch.zeros(()))
        self.val = nn.Linear(d, d, bias=False)
        self.log_rate = nn.Parameter(torch.tensor(math.log(1.0 / (4 * args.max_seq_len))))
        self.log_w = nn.Parameter(torch.full((m,), math.log(args.prior)))
        self.dropout = nn.Dropout(args.dropout)
        self.precision = "bf16"

    def code(self, u):
        z = F.relu(_hi(self.key(u))).square()
        return z / (self.log_eps.clamp(-10, 10).exp() + z.sum(-1, keepdim=True))

    def _w(self):
        return self.log_w.clamp(-7.0, 12.0).exp()

    def forward(self, x):
        h = self.norm(x)
        eps = self.log_eps.clamp(-10, 10).exp()
        v = self.val(h)
        w = self._w()
        g = -self.log_rate.exp()
        if self.dropout.p == 0.0 or not self.training:
            # conv + code(u) + the fast memory + mu(q w) + residual in one call pair on the GPU
            # (model.py:79-85): the combine accumulates in the fast read's tensor-core tiles
            return block_mixer(x, h, self.conv.weight, self.key.weight, self.key.bias, eps, v, g, w,
                               self.mu.weight, precision=self.precision)
        # with dropout on the mixed output the combine stays a separate product
        q, fast = addressed_memory(h, self.conv.weight, self.key.weight, self.key.bias, eps, v, g, w,
                                   precision=self.precision)
        return x + self.dropout(self.mu((q * w).type_as(x)) + fast.type_as(x))

    # ---- token-by-token form (the reference for run.c) ----
    def init_state(self, batch: int, device):
        d, m = self.mu.out_features, self.mu.in_features
        dt = self.mu.weight.dtype
        return {"buf": torch.zeros(batch, d, self.conv.kernel_size[0] - 1, device=device, dtype=dt),
                "U": (self.mu.weight * self._w()).expand(batch, d, m).clone(),
                "c": self._w().expand(batch, m).clone(),
                "r_prev": torch.zeros(batch, m, device=device, dtype=dt)}

    @torch.no_grad()
    def step(self, x, s):
        """x: (B,d), one position. Write (key r_{t-1}, value v_t), then read."""
        h = self.norm(x)
        win = torch.cat([s["buf"], h[:, :, None]], dim=-1)
        u = (win * self.conv.weight[:, 0, :]).sum(-1)
        s["buf"] = win[:, :, 1:]
        r = self.code(u)
        lam = torch.exp(-self.log_rate.exp())
        v = self.val(h)
        w = self._w()
        s["U"] = lam * s["U"] + (1 - lam) * self.mu.weight * w + v[:, :, None] * s["r_prev"][:, None, :]
        s["c"] = lam * s["c"] + (1 - lam) * w + s["r_prev"]
        y = (s["U"] @ (r / s["c"])[:, :, None]).squeeze(-1)
        s["r_prev"] = r
        return x + y.to(x.dtype)


class UnifiedLM(nn.Module):
    last_loss: Optional[torch.Tensor]

    def __init__(self, params: ModelArgs):
        super().__init__()
        self.params = params
        self.tok_embeddings = nn.Embedding(params.vocab_size, params.dim)
        self.dropout = nn.Dropout(params.dropout)
        self.layers = nn.ModuleList([UnifiedBlock(params) for _ in range(params.n_layers)])
        self.norm = RMSNorm(params.dim, eps=params.norm_eps)
        self.output = nn.Linear(params.dim, params.vocab_size, bias=False)
        self.tok_embeddings.weight = self.output.weight
        self.apply(self._init_weights)
        for pn, p in self.named_parameters():
            if pn.endswith("mu.weight"):
                nn.init.normal_(p, mean=0.0, std=0.02 / math.sqrt(params.n_layers))
            elif pn.endswith("val.weight"):
                nn.init.zeros_(p)
            elif pn.endswith("conv.weight"):
                with torch.no_grad():
                    p.zero_()
                    p[:, 0, -1] = 1.0
        self.last_loss = None
        # True: forward(tokens, targets) computes last_loss with the fused head and returns None
        # instead of the logits (training loops that only read last_loss, as train.py does)
        self.fused_head = False

    def _init_weights(self, module):
        if isinstance(module, nn.Linear):
            nn.init.normal_(module.weight, mean=0.0, std=0.02)
            if module.bias is not None:
                nn.init.zeros_(module.bias)
        elif isinstance(module, nn.Embedding):
            nn.init.normal_(module.weight, mean=0.0, std=0.02)

    def set_precision(self, precision: str):
        for layer in self.layers:
            layer.precision = precision
        return self

    def forward(self, tokens: torch.Tensor, targets: Optional[torch.Tensor] = None) -> torch.Tensor:
        h = self.dropout(self.tok_embeddings(tokens))
        for layer in self.layers:
            h = layer(h)
        h = self.norm(h)
        if targets is not None and self.fused_head:
            # output Linear + cross entropy in one pass that never writes the (B, T, V) logits
            # (head.lm_head_loss); the logits are not returned in this mode
            prec = self.layers[0].precision if len(self.layers) else "bf16"
            self.last_loss = lm_head_loss(h, self.output.weight, targets, precision=prec)
            return None
        if targets is not None:
            logits = self.output(h)
            self.last_loss = F.cross_entropy(logits.view(-1, logits.size(-1)), targets.view(-1), ignore_index=-1)
        else:
            logits = self.output(h[:, [-1], :])
            self.last_loss = None
        return logits

    @torch.no_grad()
    def forward_recurrent(self, tokens: torch.Tensor) -> torch.Tensor:
        B, T = tokens.shape
        states = [layer.init_state(B, tokens.device) for layer in self.layers]
        out = []
        for t in range(T):
            h = self.tok_embeddings(tokens[:, t])
            for layer, s in zip(self.layers, states):
                h = layer.step(h, s)
            out.append(self.output(self.norm(h)))
        return torch.stack(out, dim=1)

    def configure_optimizers(self, weight_decay, learning_rate, betas, device_type):
        param_dict = {pn: p for pn, p in self.named_parameters() if p.requires_grad}
        decay_params = [p for n, p in param_dict.items() if p.dim() >= 2]
        nodecay_params = [p for n, p in param_dict.items() if p.dim() < 2]
        groups = [{"params": decay_params, "weight_decay": weight_decay},
                  {"params": nodecay_params, "weight_decay": 0.0}]
        fused = "fused" in inspect.signature(torch.optim.AdamW).parameters and device_type == "cuda"
        return torch.optim.AdamW(groups, lr=learning_rate, betas=betas, **(dict(fused=True) if fused else {}))

    def estimate_mfu(self, fwdbwd_per_iter, dt):
        """Model flops utilisation against the A100 bf16 peak, counted as the reference does
        (model.py:196-204)."""
        N = sum(p.numel() for p in self.parameters())
        cfg = self.params
        T, m, d = cfg.max_seq_len, cfg.hidden_dim, cfg.dim
        mix = min(CHUNK, T) * (2 * m + d) + 2 * m * d
        flops_per_token = 6 * N + 6 * cfg.n_layers * mix
        return flops_per_token * T * fwdbwd_per_iter / dt / 312e12
