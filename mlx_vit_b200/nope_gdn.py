"""The NoPE-GDN video model around ``cuda_kda_gated``: the end-to-end use of the op in training.

A PyTorch restatement of the reference layer stack for the full-model training configuration:
``GatedDeltaLayer`` (nope_gdn_mlx.py:652-885: q/k/v projections, short causal depthwise
convolutions, SiLU + L2 norm (q scaled by D^-1/2), the low-rank decay gate
g = -e^{A_log} softplus(f_proj_2(f_proj_1(x)) + dt_bias) and the write gate beta = sigmoid(b_proj(x)),
the recurrence, the low-rank output gate with gated RMSNorm, and the output projection), the
pre-norm block with a GELU MLP (``HybridBlock``, :4009-4090), a tubelet embedding and a
classification head.  The recurrence and both gates run in the library's fused kernels
(``cuda_kda_gated``), the q / k prologue (SiLU + L2 norm) and the output's gated RMSNorm in its
one-pass row kernels (``rowops``); everything else is PyTorch (cuBLAS GEMMs, elementwise kernels).

Parameters follow the reference's initialisation where it sets one: A ~ U[1, 16] as A_log,
dt_bias = 0, RMSNorm weight 1, conv weights ~ U(+-1/sqrt(K)) with zero bias.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from .kda import cuda_kda_gated
from .rowops import conv_silu, gated_rmsnorm


class ShortCausalConv1d(nn.Module):
    """Depthwise causal convolution over time (nope_gdn_mlx.py:400-431): kernel K, K-1 zeros in front."""

    def __init__(self, channels: int, kernel_size: int = 4):
        super().__init__()
        s = 1.0 / math.sqrt(kernel_size)
        self.weight = nn.Parameter(torch.empty(channels, 1, kernel_size).uniform_(-s, s))
        self.bias = nn.Parameter(torch.zeros(channels))
        self.k = kernel_size

    def forward(self, x):  # (B, L, C)
        y = F.conv1d(F.pad(x.transpose(1, 2), (self.k - 1, 0)), self.weight.to(x.dtype),
                     self.bias.to(x.dtype), groups=x.shape[-1])
        return y.transpose(1, 2)


class RMSNormGated(nn.Module):
    """out = RMSNorm(x) * weight * sigmoid(gate), normalised over the last dim (:340-371)."""

    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps
        self.fused = True  # the library's one-pass kernel (kda_gated_rmsnorm_*); False: torch ops

    def forward(self, x, gate):
        if self.fused and x.is_cuda and x.shape[-1] in (64, 128):
            return gated_rmsnorm(x.to(torch.bfloat16), gate.to(torch.bfloat16), self.weight, self.eps)
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight
        return (y * torch.sigmoid(gate.float())).to(x.dtype)


class GatedDeltaLayer(nn.Module):
    """Channel-wise KDA layer (the reference's ``GatedDeltaLayer`` with channel_wise_decay=True)."""

    def __init__(self, hidden: int, num_heads: int, head_dim: int = 64, chunk_size: int = 64,
                 decay_low_rank: int | None = None, allow_neg_eigval: bool = False):
        super().__init__()
        H, D = num_heads, head_dim
        self.H, self.D, self.chunk = H, D, chunk_size
        self.allow_neg = allow_neg_eigval
        self.scale = D ** -0.5
        tot = H * D
        self.q_proj = nn.Linear(hidden, tot, bias=False)
        self.k_proj = nn.Linear(hidden, tot, bias=False)
        self.v_proj = nn.Linear(hidden, tot, bias=False)
        r = decay_low_rank or D
        self.f_proj_1 = nn.Linear(hidden, r, bias=False)
        self.f_proj_2 = nn.Linear(r, tot, bias=False)
        self.A_log = nn.Parameter(torch.log(torch.empty(H).uniform_(1.0, 16.0)))
        self.dt_bias = nn.Parameter(torch.zeros(tot))
        self.b_proj = nn.Linear(hidden, H, bias=False)
        self.q_conv1d = ShortCausalConv1d(tot)
        self.k_conv1d = ShortCausalConv1d(tot)
        self.v_conv1d = ShortCausalConv1d(tot)
        self.g_proj_1 = nn.Linear(hidden, D, bias=False)
        self.g_proj_2 = nn.Linear(D, tot, bias=True)
        self.o_norm = RMSNormGated(D)
        self.o_proj = nn.Linear(tot, hidden, bias=False)
        self.fused_rows = True  # conv + SiLU (+ L2 norm) in the library's fused kernels; False: torch ops

    def forward(self, x, state=None):
        B, L, _ = x.shape
        H, D = self.H, self.D
        bf = torch.bfloat16
        if self.fused_rows:  # conv + SiLU (+ L2 norm) in one pass each: kda_conv_silu_*
            cv = lambda conv, t, norm, sc: conv_silu(t.to(bf), conv.weight, conv.bias, H, D, norm, sc)
            q = cv(self.q_conv1d, self.q_proj(x), True, self.scale).view(B, L, H, D)
            k = cv(self.k_conv1d, self.k_proj(x), True, 1.0).view(B, L, H, D)
            v = cv(self.v_conv1d, self.v_proj(x), False, 1.0).view(B, L, H, D)
        else:
            # the L2 norm spans the whole H*D row, before the head reshape (nope_gdn_mlx.py:797-799)
            v = F.silu(self.v_conv1d(self.v_proj(x))).view(B, L, H, D)
            qr = self.q_conv1d(self.q_proj(x))
            kr = self.k_conv1d(self.k_proj(x))
            q = (F.normalize(F.silu(qr).float(), dim=-1) * self.scale).to(bf).view(B, L, H, D)
            k = F.normalize(F.silu(kr).float(), dim=-1).to(bf).view(B, L, H, D)
        f = self.f_proj_2(self.f_proj_1(x)).view(B, L, H, D).to(bf)
        b = self.b_proj(x).to(bf)
        o, new_state = cuda_kda_gated(q, k, v.to(bf).contiguous(), f.contiguous(), self.A_log,
                                      self.dt_bias, b.contiguous(), state, chunk_size=self.chunk,
                                      allow_neg_eigval=self.allow_neg)
        gate = self.g_proj_2(self.g_proj_1(x)).view(B, L, H, D)
        o = self.o_norm(o, gate).reshape(B, L, H * D)
        return self.o_proj(o), new_state


class KDABlock(nn.Module):
    """Pre-norm block: x + layer(LN(x)), x + MLP(LN(x)) (``HybridBlock`` with block_type "gdn")."""

    def __init__(self, dim: int, heads: int, mlp_ratio: float = 4.0, chunk_size: int = 64):
        super().__init__()
        self.norm1 = nn.LayerNorm(dim, eps=1e-6)
        self.layer = GatedDeltaLayer(dim, heads, dim // heads, chunk_size)
        self.norm2 = nn.LayerNorm(dim, eps=1e-6)
        h = int(dim * mlp_ratio)
        self.mlp = nn.Sequential(nn.Linear(dim, h), nn.GELU(), nn.Linear(h, dim))

    def forward(self, x):
        y, _ = self.layer(self.norm1(x))
        x = x + y
        return x + self.mlp(self.norm2(x))


class NoPEGDNVideo(nn.Module):
    """Tubelet embedding (no positional embedding), ``depth`` KDA blocks, final norm, mean pool,
    linear head.  Input clips are channels-last (B, T, H, W, C) as the reference's loaders give."""

    def __init__(self, img_size=224, frames=16, tubelet=(2, 16, 16), in_ch=3, dim=768, depth=12,
                 heads=12, mlp_ratio=4.0, num_classes=400, chunk_size=64):
        super().__init__()
        self.embed = nn.Conv3d(in_ch, dim, kernel_size=tubelet, stride=tubelet)
        self.blocks = nn.ModuleList(KDABlock(dim, heads, mlp_ratio, chunk_size) for _ in range(depth))
        self.norm = nn.LayerNorm(dim, eps=1e-6)
        self.head = nn.Linear(dim, num_classes)
        self.tokens = (frames // tubelet[0]) * (img_size // tubelet[1]) * (img_size // tubelet[2])

    def forward(self, clips):  # (B, T, H, W, C)
        x = self.embed(clips.permute(0, 4, 1, 2, 3))  # (B, dim, T', H', W')
        x = x.flatten(2).transpose(1, 2)  # (B, T'H'W', dim), time-major tokens
        for blk in self.blocks:
            x = blk(x)
        return self.head(self.norm(x).mean(1))
