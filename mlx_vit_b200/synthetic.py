"""Seeded synthetic KDA inputs with the distributions the benchmark configurations name.

q and k ~ N(0,1), then L2-normalised over the head dimension per (b, t, h); v ~ N(0,1);
beta = sigmoid(N(0,1)); per-channel log-decay g = -softplus(N(0,1)) (so g <= 0, the
precondition of the chunkwise form, nope_gdn_mlx.py:625); the initial state is zero or
N(0, state_std^2); the upstream gradients dO ~ N(0,1) and dS_T ~ N(0,1).

The draws come from numpy's PCG64 generator in a fixed order (q, k, v, g, beta, state, dO,
dS_T), so the same seed gives bit-identical float32 arrays on every machine.  All arrays are
returned as float32 numpy arrays in the reference layout: q, k, v, g, dO are (B, T, H, D),
beta is (B, T, H), state and dS_T are (B, H, Dv, Dk) (rows = value dim, as in
nope_gdn_mlx.py:632).
"""
from __future__ import annotations

import numpy as np


def _l2n(x: np.ndarray) -> np.ndarray:
    n = np.sqrt((x.astype(np.float64) ** 2).sum(-1, keepdims=True))
    return (x / np.maximum(n, 1e-12)).astype(np.float32)


def _softplus(x: np.ndarray) -> np.ndarray:
    x64 = x.astype(np.float64)
    return (np.log1p(np.exp(-np.abs(x64))) + np.maximum(x64, 0.0)).astype(np.float32)


def make_inputs(B: int, T: int, H: int, D: int, seed: int = 0, state_std: float = 0.0,
                with_grads: bool = True) -> dict:
    rng = np.random.default_rng(seed)
    f = np.float32
    q = _l2n(rng.standard_normal((B, T, H, D), dtype=f))
    k = _l2n(rng.standard_normal((B, T, H, D), dtype=f))
    v = rng.standard_normal((B, T, H, D), dtype=f)
    g = -_softplus(rng.standard_normal((B, T, H, D), dtype=f))
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((B, T, H), dtype=f).astype(np.float64)))).astype(f)
    state = (rng.standard_normal((B, H, D, D), dtype=f) * f(state_std)).astype(f) if state_std > 0 \
        else np.zeros((B, H, D, D), f)
    out = dict(q=q, k=k, v=v, g=g, beta=beta, state=state)
    if with_grads:
        out["do"] = rng.standard_normal((B, T, H, D), dtype=f)
        out["dst"] = rng.standard_normal((B, H, D, D), dtype=f)
    return out


def make_inputs_torch(B: int, T: int, H: int, D: int, seed: int, device, dtype, state_std=0.1):
    """Device-side generator with the same distributions (not bit-identical to
    ``make_inputs``).  Used where the inputs are too large to build on the host quickly."""
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    f32 = torch.float32
    rn = lambda *s: torch.randn(*s, generator=gen, device=device, dtype=f32)
    q = torch.nn.functional.normalize(rn(B, T, H, D), dim=-1)
    k = torch.nn.functional.normalize(rn(B, T, H, D), dim=-1)
    v = rn(B, T, H, D)
    g = -torch.nn.functional.softplus(rn(B, T, H, D))
    beta = torch.sigmoid(rn(B, T, H))
    state = rn(B, H, D, D) * state_std
    do = rn(B, T, H, D)
    dst = rn(B, H, D, D)
    return dict(q=q.to(dtype), k=k.to(dtype), v=v.to(dtype), g=g, beta=beta.to(dtype),
                state=state, do=do.to(dtype), dst=dst)
