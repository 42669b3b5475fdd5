"""GPU: kda_bwd_noalloc, the backward entry point that allocates nothing.

It exists for callers that cannot call cudaMalloc, for example a host that owns all device
memory through its own pool, or one that must not trigger the device synchronisation an
allocation can cause.  Instead of a caller-provided workspace it uses a static device array
inside the library.  These tests check, through the C ABI, that two calls in a row give the
same gradients as the regular kda_bwd with its own workspace, and that a problem too large for
the static array is refused with a clear status.  This file is collected last so that a run
stopping at its first failure has already run every other test."""
import ctypes

import numpy as np
import pytest
import torch

from kda_testutil import rel_err, TOL_BF16
from mlx_vit_b200 import _lib, kda_forward, kda_backward
from mlx_vit_b200.kda import _desc, _ptr
from mlx_vit_b200.synthetic import make_inputs

pytestmark = pytest.mark.gpu


def _inputs(dev, B=2, T=200, H=3, D=64):
    inp = make_inputs(B, T, H, D, seed=31, state_std=0.1)
    t = {}
    for k in ("q", "k", "v", "beta", "do"):
        t[k] = torch.from_numpy(inp[k]).to(dev).to(torch.bfloat16)
    for k in ("g", "state", "dst"):
        t[k] = torch.from_numpy(inp[k]).to(dev)
    return t


def _noalloc(t, saved, chunk=64):
    L = _lib.lib()
    q = t["q"]
    B, T, H, D = q.shape
    desc = _desc(q, t["beta"], chunk, 0)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(q), torch.empty_like(q)
    dg = torch.empty((B, T, H, D), dtype=torch.float32, device=q.device)
    db = torch.empty_like(t["beta"])
    ds0 = torch.empty((B, H, D, D), dtype=torch.float32, device=q.device)
    st = L.kda_bwd_noalloc(ctypes.byref(desc), _ptr(q), _ptr(t["k"]), _ptr(t["v"]), _ptr(t["g"]),
                           _ptr(t["beta"]), _ptr(t["state"]), _ptr(saved), _ptr(t["do"]),
                           _ptr(t["dst"]), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(dg), _ptr(db),
                           _ptr(ds0), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(st, "kda_bwd_noalloc")
    return dq, dk, dv, dg, db, ds0


def test_noalloc_matches_kda_bwd_two_calls(cuda):
    t = _inputs(cuda)
    _, _, saved = kda_forward(t["q"], t["k"], t["v"], t["g"], t["beta"], t["state"], 64, save_states=True)
    ref = kda_backward(t["q"], t["k"], t["v"], t["g"], t["beta"], t["state"], saved, t["do"], t["dst"], 64)
    names = ("dq", "dk", "dv", "dg", "dbeta", "dstate0")
    for call in range(2):  # the second call sees the first call's leftovers in the shared scratch
        got = _noalloc(t, saved)
        torch.cuda.synchronize()
        for n, a, r in zip(names, got, ref):
            e = rel_err(a.float().cpu().numpy(), r.float().cpu().numpy())
            assert e <= TOL_BF16, (call, n, e)
            assert np.isfinite(a.float().cpu().numpy()).all(), (call, n)


def test_noalloc_refuses_problems_beyond_its_scratch(cuda):
    L = _lib.lib()
    # 8 x 64 x 1024 chunks need ~4.3 GB of workspace, far above the static scratch; the call
    # must be refused before any pointer is touched
    desc = _lib.KdaDesc(8, 64 * 1024, 64, 64, 64, 64, _lib.KDA_BF16, _lib.KDA_BF16, 0, 0)
    assert L.kda_workspace_bytes(ctypes.byref(desc), 1) > _lib.KDA_NOALLOC_SCRATCH_BYTES
    z = ctypes.c_void_p(0)
    st = L.kda_bwd_noalloc(ctypes.byref(desc), *([z] * 15), z)
    assert st == -8
    assert b"scratch" in L.kda_strerror(st)
