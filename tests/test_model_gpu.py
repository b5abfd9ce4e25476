"""Model-level parity, the reference's test_kernel (test_all.py:140-166) restated: loss and every
parameter gradient of UnifiedLM.forward against the float64 oracle. Relative error per parameter =
||g - g_ref|| / ||g_ref||, max over layers. Bars: 1e-2 with bf16 products, 1e-5 in fp32 mode."""
import math
import os

import pytest
import torch

from oracle import memory as O
from unifiedlm_c_b200.model import ModelArgs, UnifiedLM

pytestmark = pytest.mark.gpu
TOL = {"bf16": 1e-2, "fp32": 1e-5}


@pytest.fixture(autouse=True)
def no_tf32():
    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old


def rel_errors(model, params_ref, tokens, precision):
    """Run our model on cuda:0 and the oracle in float64; return {name: rel error}."""
    model.set_precision(precision)
    x = tokens.cuda()
    model(x, x)
    model.last_loss.backward()
    p = {k: v.detach().double().cpu().clone().requires_grad_(True) for k, v in params_ref.items()}
    p["output.weight"] = p["tok_embeddings.weight"]
    _, loss = O.lm_forward(p, tokens, tokens, form="chunked", chunk=64)
    loss.backward()
    out = {"loss": abs(model.last_loss.item() - loss.item()) / abs(loss.item())}
    for name, prm in model.named_parameters():
        ref = p[name].grad
        key = name.split(".", 2)[-1] if name.startswith("layers.") else name
        err = float((prm.grad.double().cpu() - ref).norm() / ref.norm().clamp(min=1e-30))
        out[key] = max(out.get(key, 0.0), err)
    return out


@pytest.mark.parametrize("precision", ["bf16", "fp32"])
def test_reference_golden_model(golden_dir, precision):
    f = torch.load(os.path.join(golden_dir, "model_tiny.pt"), weights_only=False)
    sd = f["state_dict"]
    args = ModelArgs(dim=32, n_layers=2, hidden_dim=48, vocab_size=97, max_seq_len=140)
    model = UnifiedLM(args).cuda().train()
    model.load_state_dict({k: v.float() for k, v in sd.items()})
    model.set_precision(precision)
    x = f["tokens"].cuda()
    logits = model(x, x)
    model.last_loss.backward()
    ref_loss = f["loss"].item()
    errs = {"logits": float((logits.double().cpu() - f["logits"]).norm() / f["logits"].norm()),
            "loss": abs(model.last_loss.item() - ref_loss) / abs(ref_loss)}
    for name, prm in model.named_parameters():
        ref = f["grads"][name]
        errs[name] = float((prm.grad.double().cpu() - ref).norm() / ref.norm().clamp(min=1e-30))
    assert max(errs.values()) < TOL[precision], errs


@pytest.mark.parametrize("precision", ["bf16", "fp32"])
def test_kernel_config(precision):
    """dim 64, 2 layers, M 140, T 200 (partial last chunk), B 2, vocab 512, as test_all.test_kernel."""
    torch.manual_seed(0)
    args = ModelArgs(dim=64, n_layers=2, hidden_dim=140, vocab_size=512, max_seq_len=200)
    model = UnifiedLM(args)
    with torch.no_grad():
        for layer in model.layers:
            layer.conv.weight.normal_(std=0.5)
            layer.key.bias.normal_(std=0.5)
            layer.val.weight.normal_(std=0.2)
            layer.log_rate.fill_(math.log(0.05))
            layer.log_w.normal_(std=1.0)
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    model = model.cuda().train()
    tokens = torch.randint(0, 512, (2, 200), generator=torch.Generator().manual_seed(1))
    errs = rel_errors(model, sd, tokens, precision)
    assert max(errs.values()) < TOL[precision], errs


@pytest.mark.parametrize("precision", ["bf16", "fp32"])
def test_config4_dims_model(precision):
    """BASELINE config 4's widths (dim 768, M 2048, vocab 32000, T 1024) with 2 blocks and one
    sequence: the loss and every parameter gradient against the float64 oracle. bf16 at 1e-2. The
    fp32 mode is held to 3e-5 at these widths: the reference's own algorithm computed in plain fp32
    (the oracle's restatement in float32 on the CPU) is 1.3e-4 from float64 here (the embedding,
    9.6e-5 for key.weight), since the relu^2 normalisation's backward (dr minus its z-weighted
    mean) cancels and amplifies fp32 rounding; this library's fp32 mode measures 1.6e-5 at most
    (the embedding) and below 1e-5 for the loss and every block parameter but key.weight (1.3e-5).
    The 1e-5 bar holds at the smaller model configs (test_kernel_config, config 2)."""
    torch.manual_seed(0)
    args = ModelArgs(dim=768, n_layers=2, hidden_dim=2048, vocab_size=32000, max_seq_len=1024)
    model = UnifiedLM(args)
    with torch.no_grad():
        for layer in model.layers:
            layer.log_rate.fill_(math.log(-math.log(0.95)))
            layer.conv.weight.normal_(std=0.5)
            layer.key.bias.normal_(std=0.3)
            layer.val.weight.normal_(std=1.0 / math.sqrt(768))
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    model = model.cuda().train()
    tokens = torch.randint(0, 32000, (1, 1024), generator=torch.Generator().manual_seed(3))
    tokens[:, 0] = 1
    errs = rel_errors(model, sd, tokens, precision)
    assert max(errs.values()) < (TOL["bf16"] if precision == "bf16" else 3e-5), errs


@pytest.mark.parametrize("backend", ["aot_eager", "inductor"])
def test_torch_compile_fullgraph(backend):
    """The drop-in traces under torch.compile(fullgraph=True) (train.py:177-180 compiles the model):
    the library ops are torch.library custom ops with fake kernels and registered autograd, so the
    whole forward and backward is one graph; loss and gradients equal eager mode."""
    torch.manual_seed(0)
    args = ModelArgs(dim=64, n_layers=2, hidden_dim=128, vocab_size=512, max_seq_len=128)
    eager = UnifiedLM(args).cuda().train()
    with torch.no_grad():
        for layer in eager.layers:
            layer.val.weight.normal_(std=0.1)
            layer.conv.weight.normal_(std=0.5)
    compiled_model = UnifiedLM(args).cuda().train()
    compiled_model.load_state_dict(eager.state_dict())
    tokens = torch.randint(0, 512, (2, 128), generator=torch.Generator().manual_seed(1)).cuda()
    eager(tokens, tokens)
    eager.last_loss.backward()
    torch._dynamo.reset()
    step = torch.compile(lambda x: (compiled_model(x, x), compiled_model.last_loss)[1], fullgraph=True,
                         backend=backend)
    loss = step(tokens)
    loss.backward()
    torch.cuda.synchronize()
    assert abs(loss.item() - eager.last_loss.item()) <= 1e-5 * abs(eager.last_loss.item())
    for (n, a), (_, b) in zip(eager.named_parameters(), compiled_model.named_parameters()):
        err = float((a.grad - b.grad).norm() / a.grad.norm().clamp(min=1e-30))
        assert err < 1e-5, (n, err)
