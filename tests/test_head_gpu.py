"""The fused LM head + cross entropy (head.lm_head_loss, model.py:153-157) against
F.cross_entropy(h W^T, targets, ignore_index=-1) in float64 on the CPU: loss, dh and dW within
1e-2 relative with bf16 operands (the logits stay fp32 in the accumulator) and 1e-5 in fp32 mode,
with ignored targets; and the whole model with the fused head against the oracle."""
import pytest
import torch
import torch.nn.functional as F

import unifiedlm_c_b200._lib as L
from unifiedlm_c_b200.head import lm_head_loss

pytestmark = pytest.mark.gpu
TOL = {"bf16": 1e-2, "fp32": 1e-5}


def rel(a, b):
    b = b.double().cpu()
    return float((a.detach().double().cpu() - b).norm() / b.norm().clamp(min=1e-30))


@pytest.mark.parametrize("precision", ["bf16", "fp32"])
@pytest.mark.parametrize("shape", [(300, 97, 32), (1024, 32000, 288), (2048, 512, 768)],
                         ids=lambda s: "x".join(map(str, s)))
def test_head_loss_matches_reference(precision, shape):
    N, V, D = shape
    g = torch.Generator().manual_seed(N + V)
    h = torch.randn(N, D, generator=g, dtype=torch.float64)
    W = torch.randn(V, D, generator=g, dtype=torch.float64) * (1.0 / D ** 0.5)
    t = torch.randint(0, V, (N,), generator=g)
    t[::7] = -1  # ignored rows
    hr, Wr = h.clone().requires_grad_(True), W.clone().requires_grad_(True)
    ref = F.cross_entropy(hr @ Wr.t(), t, ignore_index=-1)
    ref.backward()
    hd, Wd = h.float().cuda().requires_grad_(True), W.float().cuda().requires_grad_(True)
    loss = lm_head_loss(hd, Wd, t.cuda(), precision=precision)
    loss.backward()
    torch.cuda.synchronize()
    errs = {"loss": abs(float(loss) - float(ref)) / abs(float(ref)), "dh": rel(hd.grad, hr.grad),
            "dW": rel(Wd.grad, Wr.grad)}
    assert max(errs.values()) < TOL[precision], errs
    assert L.device_error() == 0


@pytest.mark.parametrize("precision", ["bf16", "fp32"])
def test_model_with_fused_head(precision):
    """The drop-in model with fused_head = True: loss and every parameter gradient against the
    float64 oracle (the test_kernel configuration of test_model_gpu.py)."""
    import math

    from test_model_gpu import rel_errors
    from unifiedlm_c_b200.model import ModelArgs, UnifiedLM
    torch.manual_seed(0)
    model = UnifiedLM(ModelArgs(dim=64, n_layers=2, hidden_dim=140, vocab_size=512, max_seq_len=200))
    with torch.no_grad():
        for layer in model.layers:
            layer.conv.weight.normal_(std=0.5)
            layer.key.bias.normal_(std=0.5)
            layer.val.weight.normal_(std=0.2)
            layer.log_rate.fill_(math.log(0.05))
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    model = model.cuda().train()
    model.fused_head = True
    tokens = torch.randint(0, 512, (2, 200), generator=torch.Generator().manual_seed(1))
    errs = rel_errors(model, sd, tokens, precision)
    assert max(errs.values()) < TOL[precision], errs
    assert L.device_error() == 0
