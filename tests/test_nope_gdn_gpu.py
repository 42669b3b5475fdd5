"""The NoPE-GDN model around the fused-gate op (GPU): the layer agrees with the same layer whose
gates are evaluated in torch around plain ``cuda_kda``, and a small model trains (finite
gradients everywhere, loss going down over a few steps)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from kda_testutil import rel_err
from mlx_vit_b200 import cuda_kda
from mlx_vit_b200.nope_gdn import GatedDeltaLayer, NoPEGDNVideo

pytestmark = pytest.mark.gpu


def unfused_forward(layer, x):
    """The layer's forward with g and beta evaluated in torch (nope_gdn_mlx.py:802-816)."""
    B, L, _ = x.shape
    H, D = layer.H, layer.D
    bf = torch.bfloat16
    # SiLU + L2 norm over the whole (B, L, H*D) row, then the head reshape (:797-799, :818-821)
    q = F.silu(layer.q_conv1d(layer.q_proj(x)))
    k = F.silu(layer.k_conv1d(layer.k_proj(x)))
    v = F.silu(layer.v_conv1d(layer.v_proj(x))).view(B, L, H, D)
    q = (F.normalize(q.float(), dim=-1) * layer.scale).to(bf).view(B, L, H, D)
    k = F.normalize(k.float(), dim=-1).to(bf).view(B, L, H, D)
    f = layer.f_proj_2(layer.f_proj_1(x)).view(B, L, H, D).to(bf)
    g = -torch.exp(layer.A_log).view(1, 1, H, 1) * F.softplus(f.float() + layer.dt_bias.view(H, D))
    beta = torch.sigmoid(layer.b_proj(x).to(bf).float())
    o, _ = cuda_kda(q, k, v.to(bf).contiguous(), g, beta, None, layer.chunk)
    gate = layer.g_proj_2(layer.g_proj_1(x)).view(B, L, H, D)
    return layer.o_proj(layer.o_norm(o, gate).reshape(B, L, H * D))


def test_layer_fused_gates_equal_unfused(cuda):
    torch.manual_seed(0)
    layer = GatedDeltaLayer(256, 4, 64).to(cuda)
    # mild decays (A = 1.5): this checks the layer's wiring; strong-decay parity of the gate
    # gradients (df amplified by A) is the op-level tests' subject
    with torch.no_grad():
        layer.A_log.fill_(float(np.log(1.5)))
    x = torch.randn(2, 200, 256, device=cuda)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y1, _ = layer(x)
    g1 = torch.autograd.grad(y1.float().square().sum(), list(layer.parameters()))
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y2 = unfused_forward(layer, x)
    g2 = torch.autograd.grad(y2.float().square().sum(), list(layer.parameters()))
    assert rel_err(y1.detach().float().cpu().numpy(), y2.detach().float().cpu().numpy()) <= 2e-2
    errs = {}
    for (n, _), a, b in zip(layer.named_parameters(), g1, g2):
        assert torch.isfinite(a).all(), n
        errs[n] = rel_err(a.float().cpu().numpy(), b.float().cpu().numpy())
    # A_log and dt_bias gradients are sums over (B, T) of bf16 dg with cancellation, so two
    # bf16 paths differ in them by more (15-30 % here, depending on the seed's cancellation); the
    # op-level tests pin them against the oracle with the dg bound carried through the chain
    # rule.  Every other gradient: 5e-2.
    # f_proj_1 / f_proj_2 receive df = dg (-A) sigmoid(x) summed over every token: the same
    # bf16-dg noise, which the fused path's own bf16 roundings (conv, norms) move by a few %.
    loose = {"A_log": 0.35, "dt_bias": 0.35, "f_proj_1.weight": 0.1, "f_proj_2.weight": 0.1}
    bad = {n: e for n, e in errs.items() if e > loose.get(n, 5e-2)}
    assert not bad, bad


def test_small_model_trains(cuda):
    torch.manual_seed(1)
    model = NoPEGDNVideo(img_size=64, frames=8, dim=128, depth=2, heads=2, num_classes=10).to(cuda)
    clips = torch.rand(2, 8, 64, 64, 3, device=cuda)
    labels = torch.tensor([3, 7], device=cuda)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
    losses = []
    for _ in range(6):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = F.cross_entropy(model(clips).float(), labels)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        for n, p in model.named_parameters():
            assert p.grad is not None and torch.isfinite(p.grad).all(), n
        opt.step()
        losses.append(loss.item())
    assert losses[-1] < losses[0], losses
