"""Drop-in replacement of the reference's model.py with the fast memory on sm_100a.

The classes keep the reference's constructor arguments, parameter names, shapes and initial values
(ModelArgs model.py:13-23, RMSNorm :31-42, UnifiedBlock :45-111, UnifiedLM :114-204), so
state_dicts, checkpoints and the model.bin exporter interoperate unchanged; the computation runs in
libulm_b200.so:

* UnifiedBlock.forward (model.py:77-85): RMSNorm, the val projection and the whole mixing span
  (conv -> key -> relu^2 code -> fast memory -> mu(q w) + residual) as one library op
  (`block.unified_block`, whose backward adds the residual's and the two paths' gradients inside its
  kernels); with dropout active in training they run as separate ops (`norm.rms_norm`,
  `norm.linear`, `block.addressed_memory`) so the dropout mask can sit before the residual.
* UnifiedBlock.init_state / step (model.py:88-111) and UnifiedLM.forward_recurrent (:164-175): the
  batched decode kernels (ulm_decode_*), the same state dict (buf, U, c, r_prev) kept in fp32.
* UnifiedLM.forward with `fused_head`: output Linear + cross entropy without the logits
  (`head.lm_head_loss`).

`UnifiedBlock.precision` ("bf16" tensor-core products, default; "fp32" for the 1e-5 parity mode) is
set for a whole model by `UnifiedLM.set_precision`.
"""
import inspect
import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib as L
from .block import addressed_memory, block_scalars, unified_block
from .head import lm_head_loss
from .kernel import CHUNK
from .norm import linear, rms_norm


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


class RMSNorm(nn.Module):
    """x / rms(x) * weight with fp32 statistics (model.py:31-42), one library kernel each way."""

    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        return rms_norm(x, self.weight, self.eps)


def _fp32(t):
    return t.detach().float().contiguous()


class UnifiedBlock(nn.Module):
    """One associative memory whose slots hold running posterior means (model.py:45-111):

        address  r_t = normalize(relu(K u_t + b)^2),  u_t = causal depthwise conv(RMSNorm(x_t))
        write    key r_{t-1}, value v_t = W_v h_t
        read     y_t = sum_a r_t,a (w_a mu_a + sum_{s<=t} lam^(t-s) r_{s-1,a} v_s)
                                 / (w_a      + sum_{s<=t} lam^(t-s) r_{s-1,a})
    """

    def __init__(self, args: ModelArgs):
        super().__init__()
        dim, slots, width = args.dim, args.hidden_dim, args.conv_size
        # parameters in the reference's order and with its names: norm, conv, key, mu, log_eps, val,
        # log_rate (initial forgetting 1 / (4 max_seq_len)), log_w (initial prior mass)
        self.norm = RMSNorm(dim, eps=args.norm_eps)
        self.conv = nn.Conv1d(dim, dim, width, groups=dim, padding=width - 1, bias=False)
        self.key = nn.Linear(dim, slots)
        self.mu = nn.Linear(slots, dim, bias=False)
        self.log_eps = nn.Parameter(torch.tensor(0.0))
        self.val = nn.Linear(dim, dim, bias=False)
        self.log_rate = nn.Parameter(torch.tensor(-math.log(4.0 * args.max_seq_len)))
        self.log_w = nn.Parameter(torch.full((slots,), math.log(args.prior)))
        self.dropout = nn.Dropout(args.dropout)
        self.precision = "bf16"
        self._decode = None  # decode-form weights, rebuilt when a parameter changes

    # the learned scalars' transforms (model.py:72, 74-75, 84)
    def _w(self):
        return torch.exp(self.log_w.clamp(-7.0, 12.0))

    def _eps(self):
        return torch.exp(self.log_eps.clamp(-10.0, 10.0))

    def _g(self):
        return -torch.exp(self.log_rate)

    def code(self, u):
        """relu(K u + b)^2 normalised with the learnable null mass (model.py:70-72), fp32."""
        a = self.key(u)
        z = F.relu(a.float() if a.dtype in (torch.float16, torch.bfloat16) else a).square()
        return z / (self._eps() + z.sum(-1, keepdim=True))

    def forward(self, x):
        # the same values and gradients as _w(), _g(), _eps(), in one launch each way
        w, eps, g = block_scalars(self.log_w, self.log_eps, self.log_rate)
        if self.dropout.p == 0.0 or not self.training:
            # norm, val, addressing, fast memory and combine as one op (v in bf16 with the
            # tensor-core products, as under the reference's bf16 autocast)
            return unified_block(x, self.norm.weight, self.norm.eps, self.conv.weight, self.key.weight,
                                 self.key.bias, eps, self.val.weight, g, w, self.mu.weight, precision=self.precision)
        h = self.norm(x)
        v = linear(h, self.val.weight, precision=self.precision,
                   out_dtype=torch.bfloat16 if self.precision == "bf16" else None)
        q, fast = addressed_memory(h, self.conv.weight, self.key.weight, self.key.bias, eps, v, g, w,
                                   precision=self.precision)
        return x + self.dropout(self.mu((q * w).type_as(x)) + fast.type_as(x))

    # ---- token-by-token form: the library's batched decode kernels -----------------------------
    def _decode_weights(self):
        """The block's weights in the decode kernels' layout (ulm_decode_block_step): fp32, or bf16
        matrices when the module holds bf16 weights; rebuilt after any parameter update."""
        params = (self.norm.weight, self.conv.weight, self.key.weight, self.key.bias, self.val.weight,
                  self.mu.weight, self.log_w, self.log_rate, self.log_eps)
        stamp = tuple((p.data_ptr(), p._version) for p in params)
        if self._decode is not None and self._decode[0] == stamp:
            return self._decode[1]
        wdt = torch.bfloat16 if self.mu.weight.dtype == torch.bfloat16 else torch.float32
        dev = self.mu.weight.device
        with torch.no_grad():
            lam = torch.exp(-torch.exp(self.log_rate.detach().double())).float().reshape(1)
            pack = {"norm": _fp32(self.norm.weight), "conv": _fp32(self.conv.weight[:, 0, :]),
                    "key_w": self.key.weight.detach().to(wdt).contiguous(), "key_b": _fp32(self.key.bias),
                    "val_w": self.val.weight.detach().to(wdt).contiguous(), "mu": _fp32(self.mu.weight),
                    "w": torch.exp(self.log_w.detach().double().clamp(-7.0, 12.0)).float(), "lam": lam,
                    "eps": torch.exp(self.log_eps.detach().double().clamp(-10.0, 10.0)).float().reshape(1),
                    "prior": torch.empty(self.mu.out_features, self.mu.in_features, device=dev, dtype=wdt),
                    "wcode": L.dtype_code(wdt)}
            D, M = self.mu.out_features, self.mu.in_features
            with torch.cuda.device(dev):
                L.check(L.lib().ulm_decode_prepare_block(L.ptr(pack["mu"]), L.ptr(pack["w"]), L.ptr(pack["lam"]),
                                                         L.ptr(pack["prior"]), pack["wcode"], D, M,
                                                         L.stream_of(pack["mu"])))
        self._decode = (stamp, pack)
        return pack

    def init_state(self, batch: int, device):
        """Fresh recurrent state for `batch` sequences (model.py:88-94): buf (B, d, conv_size-1) the
        conv window, U (B, d, m) = mu * w the slot contents, c (B, m) = w the evidence mass, r_prev
        (B, m) = 0; fp32 on the device, as run.c keeps it."""
        D, M, K = self.mu.out_features, self.mu.in_features, self.conv.kernel_size[0]
        f = dict(device=device, dtype=torch.float32)
        s = {"buf": torch.empty(batch, D, max(K - 1, 1), **f), "U": torch.empty(batch, D, M, **f),
             "c": torch.empty(batch, M, **f), "r_prev": torch.empty(batch, M, **f)}
        pk = self._decode_weights()
        with torch.cuda.device(s["U"].device):
            L.check(L.lib().ulm_decode_reset_block(L.ptr(pk["mu"]), L.ptr(pk["w"]), L.ptr(s["U"]), L.ptr(s["c"]),
                                                   L.ptr(s["r_prev"]), L.ptr(s["buf"]), batch, D, M, K,
                                                   L.stream_of(s["U"])))
        return s

    @torch.no_grad()
    def step(self, x, s):
        """x: (B, d), one position: write (key r_{t-1}, value v_t), then read (model.py:96-111),
        advancing the state s in place. Returns x + y in x's dtype."""
        B, D = x.shape
        M, K = self.mu.in_features, self.conv.kernel_size[0]
        pk = self._decode_weights()
        xf = x.detach().float().contiguous().clone()
        work = torch.empty(int(L.lib().ulm_decode_block_work_bytes(B, D, M)), device=xf.device, dtype=torch.uint8)
        with torch.cuda.device(xf.device):
            L.check(L.lib().ulm_decode_block_step(
                L.ptr(xf), L.ptr(pk["norm"]), L.ptr(pk["conv"]), L.ptr(pk["key_w"]), L.ptr(pk["key_b"]),
                L.ptr(pk["val_w"]), L.ptr(pk["prior"]), pk["wcode"], L.ptr(pk["w"]), L.ptr(pk["lam"]),
                L.ptr(pk["eps"]), L.ptr(s["U"]), L.ptr(s["c"]), L.ptr(s["r_prev"]), L.ptr(s["buf"]), L.ptr(work),
                B, D, M, K, float(self.norm.eps), L.stream_of(xf)))
        return xf.to(x.dtype)


class UnifiedLM(nn.Module):
    """Token embedding, n_layers UnifiedBlocks, final RMSNorm and an output Linear tied to the
    embedding (model.py:114-204)."""

    last_loss: Optional[torch.Tensor]

    def __init__(self, params: ModelArgs):
        super().__init__()
        self.params = params
        self.tok_embeddings = nn.Embedding(params.vocab_size, params.dim)
        self.dropout = nn.Dropout(params.dropout)
        self.layers = nn.ModuleList(UnifiedBlock(params) for _ in range(params.n_layers))
        self.norm = RMSNorm(params.dim, eps=params.norm_eps)
        self.output = nn.Linear(params.dim, params.vocab_size, bias=False)
        self.tok_embeddings.weight = self.output.weight
        self._reset_parameters()
        self.last_loss = None
        # True: forward(tokens, targets) computes last_loss with the fused head and returns None
        # instead of the logits (training loops that only read last_loss, as train.py does)
        self.fused_head = False

    @torch.no_grad()
    def _reset_parameters(self):
        """The reference's initial values (model.py:131-147): N(0, 0.02) for every Linear and the
        embedding with zero biases; mu N(0, 0.02 / sqrt(n_layers)) (GPT-2 residual scaling); val zero
        (an empty fast store); the conv the identity (u_t = h_t)."""
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                nn.init.normal_(m.weight, mean=0.0, std=0.02)
                if getattr(m, "bias", None) is not None:
                    nn.init.zeros_(m.bias)
        for blk in self.layers:
            nn.init.normal_(blk.mu.weight, mean=0.0, std=0.02 / math.sqrt(self.params.n_layers))
            nn.init.zeros_(blk.val.weight)
            blk.conv.weight.zero_()
            blk.conv.weight[:, 0, -1] = 1.0

    def set_precision(self, precision: str):
        for layer in self.layers:
            layer.precision = precision
        return self

    def forward(self, tokens: torch.Tensor, targets: Optional[torch.Tensor] = None) -> torch.Tensor:
        h = self.dropout(self.tok_embeddings(tokens))
        for layer in self.layers:
            h = layer(h)
        h = self.norm(h)
        if targets is None:
            self.last_loss = None
            return self.output(h[:, [-1], :])
        if self.fused_head:
            # output Linear + cross entropy in one pass that never writes the (B, T, V) logits
            prec = self.layers[0].precision if len(self.layers) else "bf16"
            self.last_loss = lm_head_loss(h, self.output.weight, targets, precision=prec)
            return None
        logits = self.output(h)
        self.last_loss = F.cross_entropy(logits.view(-1, logits.size(-1)), targets.view(-1), ignore_index=-1)
        return logits

    @torch.no_grad()
    def forward_recurrent(self, tokens: torch.Tensor) -> torch.Tensor:
        """Token-by-token inference with constant state per block (model.py:164-175): the logits after
        every position (B, T, V), from the batched decoder (run.c's computation for B sequences; fp32
        weights give run.c's arithmetic, bf16 weights the bf16 decode mode)."""
        from .decode import BatchedDecoder
        B, T = tokens.shape
        prec = "bf16" if self.output.weight.dtype == torch.bfloat16 else "fp32"
        dec = BatchedDecoder(self.state_dict(), batch=B, precision=prec, device=tokens.device,
                             norm_eps=self.params.norm_eps)
        dec.prepare_graph()
        out = torch.empty(B, T, self.params.vocab_size, device=tokens.device, dtype=torch.float32)
        for t in range(T):
            dec.feed(tokens[:, t])
            out[:, t] = dec.logits
        return out

    def configure_optimizers(self, weight_decay, learning_rate, betas, device_type):
        """AdamW with weight decay on the matrices and embeddings only (parameters of two or more
        dimensions), fused on CUDA (model.py:177-193)."""
        params = [p for p in self.parameters() if p.requires_grad]
        groups = [{"params": [p for p in params if p.dim() >= 2], "weight_decay": weight_decay},
                  {"params": [p for p in params if p.dim() < 2], "weight_decay": 0.0}]
        extra = {}
        if device_type == "cuda" and "fused" in inspect.signature(torch.optim.AdamW).parameters:
            extra["fused"] = True
        return torch.optim.AdamW(groups, lr=learning_rate, betas=betas, **extra)

    def estimate_mfu(self, fwdbwd_per_iter, dt):
        """Model flops utilisation in units of the A100's 312 TFLOP/s bf16 peak, with the
        reference's count (model.py:196-204): 6 flops per parameter and token plus, per block, the
        chunked mixing's min(CHUNK, T)(2m + d) + 2 m d, times 6."""
        cfg = self.params
        mix = min(CHUNK, cfg.max_seq_len) * (2 * cfg.hidden_dim + cfg.dim) + 2 * cfg.hidden_dim * cfg.dim
        n_params = sum(p.numel() for p in self.parameters())
        per_token = 6 * n_params + 6 * cfg.n_layers * mix
        return per_token * cfg.max_seq_len * fwdbwd_per_iter / dt / 312e12
