"""Strided input views read in place (KdaDesc strides): q, k, v as slices of one fused
projection [B, T, 3, H, D], g and beta as slices of wider tensors, dO as a slice -- the layout a
layer that computes q, k, v with one matmul hands over.  Every kernel family must give exactly
what it gives on dense copies of the same values (same kernels, same arithmetic)."""
import ctypes

import numpy as np
import pytest
import torch

from mlx_vit_b200 import _lib, cuda_kda, kda_forward
from mlx_vit_b200.kda import _desc, _in_place_ok
from mlx_vit_b200.synthetic import make_inputs

pytestmark = pytest.mark.gpu


def strided_views(inp, dev, dtype):
    B, T, H, D = inp["q"].shape
    qkv = torch.empty(B, T, 3, H, D, device=dev, dtype=dtype)
    for i, n in enumerate("qkv"):
        qkv[:, :, i] = torch.from_numpy(inp[n]).to(dev).to(dtype)
    gw = torch.zeros(B, T, H, 2 * D, device=dev)
    gw[..., :D] = torch.from_numpy(inp["g"]).to(dev)
    bw = torch.zeros(B, T, 2 * H, device=dev, dtype=dtype)
    bw[..., H:] = torch.from_numpy(inp["beta"]).to(dev).to(dtype)
    dow = torch.zeros(B, T + 3, H, D, device=dev, dtype=dtype)
    dow[:, 3:] = torch.from_numpy(inp["do"]).to(dev).to(dtype)
    return dict(q=qkv[:, :, 0], k=qkv[:, :, 1], v=qkv[:, :, 2], g=gw[..., :D], beta=bw[..., H:],
                do=dow[:, 3:], state=torch.from_numpy(inp["state"]).to(dev),
                dst=torch.from_numpy(inp["dst"]).to(dev))


def fwd_bwd(t, grad=True):
    leaves = {n: t[n] for n in ("q", "k", "v", "g", "beta", "state")}
    if not grad:
        with torch.no_grad():
            o, S = cuda_kda(*(leaves[n] for n in ("q", "k", "v", "g", "beta", "state")))
        return [o, S]
    req = {n: x.requires_grad_(True) for n, x in leaves.items()}
    o, S = cuda_kda(*(req[n] for n in ("q", "k", "v", "g", "beta", "state")))
    gs = torch.autograd.grad([o, S], [req[n] for n in ("q", "k", "v", "g", "beta", "state")],
                             [t["do"], t["dst"]])
    return [o, S] + list(gs)


@pytest.mark.parametrize("dtype,D,T,grad", [
    (torch.bfloat16, 64, 300, True),    # tensor-core forward + backward
    (torch.float32, 32, 100, True),     # fp32 generic kernels
    (torch.bfloat16, 128, 200, False),  # D = 128 tensor-core forward
    (torch.float32, 64, 9, False),      # token-by-token kernel (T <= 16, no gradient)
])
def test_strided_views_equal_dense(cuda, dtype, D, T, grad):
    inp = make_inputs(2, T, 3, D, seed=D + T, state_std=0.1)
    sv = strided_views(inp, cuda, dtype)
    for n in ("q", "k", "v", "g", "do"):
        assert not sv[n].is_contiguous() and _in_place_ok(sv[n]), n
    dense = {n: x.contiguous() for n, x in sv.items()}
    a = fwd_bwd({n: x.detach().clone() if n in ("state", "dst") else x for n, x in sv.items()}, grad)
    b = fwd_bwd(dense, grad)
    for i, (x, y) in enumerate(zip(a, b)):
        assert torch.equal(x, y), i


def test_descriptor_carries_the_view_strides(cuda):
    inp = make_inputs(2, 70, 3, 64, seed=1, state_std=0.1)
    sv = strided_views(inp, cuda, torch.bfloat16)
    d = _desc(sv["q"], sv["beta"], 64, 0, sv["k"], sv["v"], sv["g"], sv["do"])
    H, D = 3, 64
    assert (d.q.b, d.q.t, d.q.h) == (70 * 3 * H * D, 3 * H * D, D)
    assert (d.g.b, d.g.t, d.g.h) == (70 * H * 2 * D, H * 2 * D, 2 * D)
    assert (d.beta.b, d.beta.t, d.beta.h) == (70 * 2 * H, 2 * H, 1)
    assert (d.dO.t, d.dO.h) == (H * D, D)
    dd = _desc(sv["q"].contiguous(), sv["beta"].contiguous(), 64, 0)
    assert (dd.q.b, dd.q.t, dd.q.h) == (0, 0, 0)


def test_tma_unaligned_strides_rejected_then_copied(cuda):
    """A time stride that is not a whole number of 16-byte units cannot be TMA-read: the C ABI
    refuses it with KDA_ERR_MISALIGNED, and the Python op copies such a view instead."""
    inp = make_inputs(1, 64, 2, 64, seed=2, state_std=0.1, with_grads=False)
    bf = torch.bfloat16
    wide = torch.zeros(1, 64, 2 * 64 + 4, device=cuda, dtype=bf)  # t stride 132 elements = 264 B
    wide[..., :128] = torch.from_numpy(inp["q"]).to(cuda).to(bf).reshape(1, 64, 128)
    q = wide[..., :128].unflatten(-1, (2, 64))
    assert not _in_place_ok(q)
    k, v = (torch.from_numpy(inp[n]).to(cuda).to(bf) for n in "kv")
    g, beta = torch.from_numpy(inp["g"]).to(cuda), torch.from_numpy(inp["beta"]).to(cuda).to(bf)
    L = _lib.lib()
    d = _desc(q, beta, 64, 0, k, v, g)
    o = torch.empty(q.shape, dtype=bf, device=cuda)
    S = torch.empty(1, 2, 64, 64, device=cuda)
    nws = L.kda_workspace_bytes(ctypes.byref(d), 0)
    ws = torch.empty(max(nws, 16), dtype=torch.uint8, device=cuda)
    P = lambda x: ctypes.c_void_p(x.data_ptr())
    st = L.kda_fwd(ctypes.byref(d), P(q), P(k), P(v), P(g), P(beta), None, P(o), P(S), None, P(ws), nws,
                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _lib.STATUS_CODE["KDA_ERR_MISALIGNED"]
    with torch.no_grad():
        o1, S1 = cuda_kda(q, k, v, g, beta)
        o2, S2 = cuda_kda(q.contiguous(), k, v, g, beta)
    assert torch.equal(o1, o2) and torch.equal(S1, S2)
