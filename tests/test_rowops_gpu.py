"""GPU parity of the fused row kernels (kda_l2norm_silu_*, kda_conv_silu_*, kda_gated_rmsnorm_*)
against fp32 torch restatements of the reference's lines on the same bf16 inputs: forward and
every gradient, max|delta|/max|ref| <= 2e-2 (bf16 I/O).

The q / k prologue is ``l2_normalize(nn.silu(q), axis=-1) * scale`` on the (B, L, H*D)
projection, BEFORE the reshape to heads (nope_gdn_mlx.py:797-799, reshape :818-821), so the
norm spans all H*D channels of a token; the output norm is ``RMSNormGated(D)`` on the
(B, L, H, D) output, per head (:340-371, :880-885)."""
import pytest
import torch
import torch.nn.functional as F

from kda_testutil import rel_err
from mlx_vit_b200.rowops import gated_rmsnorm, l2norm_silu

pytestmark = pytest.mark.gpu
TOL = 2e-2


def np_(x):
    return x.detach().float().cpu().numpy()


@pytest.mark.parametrize("H,D", [(12, 64), (5, 64), (3, 128), (1, 64)])
@pytest.mark.parametrize("scale", [1.0, 0.125])
def test_l2norm_silu_over_all_heads(cuda, H, D, scale):
    torch.manual_seed(H * D)
    x = (torch.randn(3, 37, H * D, device=cuda) * 2).to(torch.bfloat16)
    x[0, 0] = 0  # a zero row: the norm clamps at 1e-12
    dy = torch.randn_like(x)
    xa = x.clone().requires_grad_(True)
    y = l2norm_silu(xa, scale)
    y.backward(dy)
    xr = x.float().requires_grad_(True)
    yr = F.normalize(F.silu(xr), dim=-1, eps=1e-12) * scale   # (B, L, H*D), nope_gdn_mlx.py:797
    yr.backward(dy.float())
    assert torch.isfinite(y).all() and torch.isfinite(xa.grad).all()
    assert rel_err(np_(y), np_(yr)) <= TOL
    assert rel_err(np_(xa.grad), np_(xr.grad)) <= TOL


def test_l2norm_silu_norm_spans_the_row(cuda):
    """Doubling one head's input changes every head's output: the norm is shared by the row."""
    x = torch.randn(2, 5, 4 * 64, device=cuda).to(torch.bfloat16)
    x2 = x.clone()
    x2[..., :64] *= 4
    y, y2 = l2norm_silu(x), l2norm_silu(x2)
    assert not torch.allclose(y[..., 64:].float(), y2[..., 64:].float())
    n = y.float().norm(dim=-1)
    assert torch.allclose(n, torch.ones_like(n), atol=1e-2)


@pytest.mark.parametrize("D", [64, 128])
def test_gated_rmsnorm(cuda, D):
    torch.manual_seed(D + 1)
    o = torch.randn(2, 50, 3, D, device=cuda).to(torch.bfloat16)
    g = torch.randn_like(o)
    w = torch.randn(D, device=cuda) * 0.5 + 1
    dy = torch.randn_like(o)
    oa, ga, wa = o.clone().requires_grad_(True), g.clone().requires_grad_(True), w.clone().requires_grad_(True)
    y = gated_rmsnorm(oa, ga, wa, 1e-5)
    y.backward(dy)
    orf, grf, wrf = o.float().requires_grad_(True), g.float().requires_grad_(True), w.clone().requires_grad_(True)
    yr = orf * torch.rsqrt(orf.pow(2).mean(-1, keepdim=True) + 1e-5) * wrf * torch.sigmoid(grf)
    yr.backward(dy.float())
    assert rel_err(np_(y), np_(yr)) <= TOL
    for a, b in ((oa.grad, orf.grad), (ga.grad, grf.grad), (wa.grad, wrf.grad)):
        assert rel_err(np_(a), np_(b)) <= TOL


def test_rowops_reject_bad_input(cuda):
    with pytest.raises(ValueError):
        l2norm_silu(torch.randn(4, 44, device=cuda).to(torch.bfloat16))
    with pytest.raises(ValueError):
        l2norm_silu(torch.randn(4, 64, device=cuda))


@pytest.mark.parametrize("H,D", [(3, 64), (3, 128), (12, 64)])
@pytest.mark.parametrize("norm", [False, True])
def test_conv_silu(cuda, H, D, norm):
    """Causal depthwise conv (kernel 4) + SiLU (+ L2 norm over the H*D row, scale) against
    F.conv1d in fp32 (nope_gdn_mlx.py:793-799)."""
    from mlx_vit_b200.rowops import conv_silu
    torch.manual_seed(D + norm + H)
    B, T = 2, 131
    C = H * D
    x = torch.randn(B, T, C, device=cuda).to(torch.bfloat16)
    w = torch.empty(C, 1, 4, device=cuda).uniform_(-0.5, 0.5)
    b = torch.randn(C, device=cuda) * 0.1
    dy = torch.randn_like(x)
    scale = 0.125 if norm else 1.0
    xa, wa, ba = x.clone().requires_grad_(True), w.clone().requires_grad_(True), b.clone().requires_grad_(True)
    y = conv_silu(xa, wa, ba, H, D, norm, scale)
    y.backward(dy)
    xr, wr, br = x.float().requires_grad_(True), w.clone().requires_grad_(True), b.clone().requires_grad_(True)
    z = F.conv1d(F.pad(xr.transpose(1, 2), (3, 0)), wr, br, groups=C).transpose(1, 2)
    yr = F.silu(z)
    if norm:
        yr = F.normalize(yr, dim=-1, eps=1e-12) * scale  # over all C = H*D channels
    yr.backward(dy.float())
    assert rel_err(np_(y), np_(yr)) <= TOL
    for a, r in ((xa.grad, xr.grad), (wa.grad, wr.grad), (ba.grad, br.grad)):
        assert torch.isfinite(a).all()
        assert rel_err(np_(a), np_(r)) <= TOL
