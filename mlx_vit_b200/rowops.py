"""Fused row operations of the GDN layer around the recurrence (bf16), with autograd:
``l2norm_silu`` is the q / k prologue y = l2norm(silu(x)) * scale over the last dimension, which
in the layer is a token's whole H*D channel row (nope_gdn_mlx.py:797-799, l2_normalize :76-79,
normalised before the head reshape at :818-821); ``conv_silu`` fuses the short causal
convolution in front of it; ``gated_rmsnorm`` is the output's y = rmsnorm(o) * w * sigmoid(gate)
over each head's D = 64 or 128 channels (RMSNormGated(D), :340-371).  One CUDA pass each way
(``kda_l2norm_silu_*``, ``kda_conv_silu_*``, ``kda_gated_rmsnorm_*`` in include/kda_b200.h); no
CPU path."""
from __future__ import annotations

import ctypes

import torch

from . import _lib


def _ptr(x):
    return ctypes.c_void_p(x.data_ptr())


def _stream(x):
    return ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)


def _check_rows(*xs):
    for x in xs:
        if not x.is_cuda or x.dtype != torch.bfloat16:
            raise ValueError("fused row ops take bf16 CUDA tensors")
    D = xs[0].shape[-1]
    if D not in (64, 128):
        raise ValueError(f"fused row ops need D = 64 or 128, got {D}")
    return xs[0].numel() // D, D


def _check_wide(*xs):
    for x in xs:
        if not x.is_cuda or x.dtype != torch.bfloat16:
            raise ValueError("fused row ops take bf16 CUDA tensors")
    n = xs[0].shape[-1]
    if n % 8 or n > 8192:
        raise ValueError(f"l2norm_silu needs a row length that is a multiple of 8 and at most 8192, got {n}")
    return xs[0].numel() // n, n


class L2NormSiLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, scale):
        x = x.contiguous()
        rows, D = _check_wide(x)
        y = torch.empty_like(x)
        with torch.cuda.device(x.device):
            _lib.check(_lib.lib().kda_l2norm_silu_fwd(rows, D, _ptr(x), _ptr(y), float(scale), _stream(x)),
                       "kda_l2norm_silu_fwd")
        ctx.save_for_backward(x)
        ctx.scale = scale
        return y

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        dy = dy.to(torch.bfloat16).contiguous()
        rows, D = _check_wide(x, dy)
        dx = torch.empty_like(x)
        with torch.cuda.device(x.device):
            _lib.check(_lib.lib().kda_l2norm_silu_bwd(rows, D, _ptr(x), _ptr(dy), _ptr(dx), float(ctx.scale),
                                                      _stream(x)), "kda_l2norm_silu_bwd")
        return dx, None


class GatedRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, o, gate, w, eps):
        o, gate = o.contiguous(), gate.contiguous()
        rows, D = _check_rows(o, gate)
        w32 = w.to(torch.float32).contiguous()
        y = torch.empty_like(o)
        with torch.cuda.device(o.device):
            _lib.check(_lib.lib().kda_gated_rmsnorm_fwd(rows, D, _ptr(o), _ptr(gate), _ptr(w32), _ptr(y),
                                                        float(eps), _stream(o)), "kda_gated_rmsnorm_fwd")
        ctx.save_for_backward(o, gate, w32)
        ctx.eps, ctx.w_dtype = eps, w.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        o, gate, w32 = ctx.saved_tensors
        dy = dy.to(torch.bfloat16).contiguous()
        rows, D = _check_rows(o, gate, dy)
        do, dg = torch.empty_like(o), torch.empty_like(gate)
        dw = torch.empty(D, dtype=torch.float32, device=o.device)
        with torch.cuda.device(o.device):
            _lib.check(_lib.lib().kda_gated_rmsnorm_bwd(rows, D, _ptr(o), _ptr(gate), _ptr(w32), _ptr(dy), _ptr(do),
                                                        _ptr(dg), _ptr(dw), float(ctx.eps), _stream(o)),
                       "kda_gated_rmsnorm_bwd")
        return do, dg, dw.to(ctx.w_dtype), None


class ConvSiLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, H, D, norm, scale):
        x = x.contiguous()
        if not x.is_cuda or x.dtype != torch.bfloat16 or x.shape[-1] != H * D or (H * D) % 8 or H * D > 2048:
            raise ValueError("conv_silu takes a bf16 CUDA tensor [B, T, H*D] with H*D a multiple of 8, "
                             "at most 2048")
        B, T = x.shape[0], x.shape[1]
        w32 = w.reshape(H * D, 4).to(torch.float32).contiguous()
        b32 = b.to(torch.float32).contiguous()
        y = torch.empty_like(x)
        with torch.cuda.device(x.device):
            _lib.check(_lib.lib().kda_conv_silu_fwd(B, T, H, D, _ptr(x), _ptr(w32), _ptr(b32), _ptr(y), int(norm),
                                                    float(scale), _stream(x)), "kda_conv_silu_fwd")
        ctx.save_for_backward(x, w32, b32)
        ctx.meta = (H, D, norm, scale, w.shape, w.dtype, b.dtype)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w32, b32 = ctx.saved_tensors
        H, D, norm, scale, wshape, wdt, bdt = ctx.meta
        dy = dy.to(torch.bfloat16).contiguous()
        B, T = x.shape[0], x.shape[1]
        dx = torch.empty_like(x)
        dw = torch.empty_like(w32)
        db = torch.empty_like(b32)
        dz = torch.empty(x.shape, dtype=torch.float32, device=x.device)
        with torch.cuda.device(x.device):
            _lib.check(_lib.lib().kda_conv_silu_bwd(B, T, H, D, _ptr(x), _ptr(w32), _ptr(b32), _ptr(dy), _ptr(dx),
                                                    _ptr(dw), _ptr(db), int(norm), float(scale), _ptr(dz),
                                                    _stream(x)), "kda_conv_silu_bwd")
        return dx, dw.reshape(wshape).to(wdt), db.to(bdt), None, None, None, None


def conv_silu(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, heads: int, head_dim: int,
              norm: bool = False, scale: float = 1.0) -> torch.Tensor:
    """silu(causal depthwise conv4(x)) over time for x [B, T, H*D] (bf16); with ``norm`` also the
    L2 norm over each token's whole H*D row and ``scale`` (nope_gdn_mlx.py:793-799).  ``weight``
    is the conv's [C, 1, 4] (or [C, 4]) tensor."""
    return ConvSiLU.apply(x, weight, bias, heads, head_dim, norm, scale)


def l2norm_silu(x: torch.Tensor, scale: float = 1.0) -> torch.Tensor:
    """y = silu(x) / max(||silu(x)||, 1e-12) * scale over the last dim (bf16 in and out; the layer
    passes rows of H*D channels, as the reference normalises before its head reshape)."""
    return L2NormSiLU.apply(x, scale)


def gated_rmsnorm(o: torch.Tensor, gate: torch.Tensor, w: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """y = o * rsqrt(mean(o^2) + eps) * w * sigmoid(gate) over the last dim (bf16 in and out)."""
    return GatedRMSNorm.apply(o, gate, w, eps)
