"""GPU parity of the D = 128 tensor-core forward (the streaming-inference configuration: bf16
q/k/v, chunk 64, no saved states) through the C ABI, against the CPU oracle in float64 on the
same bf16-rounded inputs, plus the D = 128 training path (generic fp32 kernels).  Tolerance
max|delta|/max|ref| <= 2e-2 (bf16 I/O)."""
import numpy as np
import pytest
import torch

from kda_testutil import rel_err, TOL_BF16
from mlx_vit_b200 import _lib, cuda_kda, kda_forward
from mlx_vit_b200.synthetic import make_inputs
from oracle import kda_oracle as O

pytestmark = pytest.mark.gpu


def bf16_inputs(inp):
    r = dict(inp)
    for k in ("q", "k", "v", "beta"):
        r[k] = torch.from_numpy(inp[k]).to(torch.bfloat16).float().numpy()
    return r


def run(inp, dev, state=True):
    t = {k: torch.from_numpy(inp[k]).to(dev) for k in ("q", "k", "v", "g", "beta", "state")}
    for k in ("q", "k", "v", "beta"):
        t[k] = t[k].to(torch.bfloat16)
    with torch.no_grad():
        o, S = cuda_kda(t["q"], t["k"], t["v"], t["g"], t["beta"], t["state"] if state else None)
    return o.float().cpu().numpy(), S.cpu().numpy()


@pytest.mark.parametrize("B,T,H", [(1, 64, 2), (2, 200, 3), (1, 1, 1), (1, 130, 4), (1, 400, 2)])
def test_d128_forward_matches_oracle(cuda, B, T, H):
    inp = make_inputs(B, T, H, 128, seed=T + 10 * H + B, state_std=0.1, with_grads=False)
    ref_o, ref_S = O.compiled_forward(**{k: v for k, v in bf16_inputs(inp).items()}, dtype=np.float64)
    o, S = run(inp, cuda)
    assert np.isfinite(o).all() and np.isfinite(S).all()
    assert rel_err(o, ref_o) <= TOL_BF16, rel_err(o, ref_o)
    assert rel_err(S, ref_S) <= TOL_BF16, rel_err(S, ref_S)


@pytest.mark.parametrize("scale", [8.0, 16.0])
def test_d128_strong_and_mixed_decay(cuda, scale):
    """Per-head decay scales 1 and `scale` in one launch: factored and exact (big-chunk) decay
    handling side by side."""
    inp = make_inputs(1, 300, 2, 128, seed=int(scale), state_std=0.1, with_grads=False)
    inp["g"] = (inp["g"] * np.array([1.0, scale], np.float32).reshape(1, 1, 2, 1)).astype(np.float32)
    ref_o, ref_S = O.compiled_forward(**bf16_inputs(inp), dtype=np.float64)
    o, S = run(inp, cuda)
    assert rel_err(o, ref_o) <= TOL_BF16, rel_err(o, ref_o)
    assert rel_err(S, ref_S) <= TOL_BF16, rel_err(S, ref_S)


def test_d128_streaming_segments_equal_one_pass(cuda):
    """Four segments with the state carried equal one pass over the whole sequence (the
    streaming-inference use), and agree with the fp32 generic kernels."""
    from mlx_vit_b200.synthetic import make_inputs_torch
    t = make_inputs_torch(1, 1024, 2, 128, seed=3, device=cuda, dtype=torch.bfloat16)
    q, k, v, g, beta, st = (t[n] for n in ("q", "k", "v", "g", "beta", "state"))
    with torch.no_grad():
        o1, S1 = cuda_kda(q, k, v, g, beta, st)
        s, outs = st, []
        for i in range(4):
            sl = slice(256 * i, 256 * (i + 1))
            o, s = cuda_kda(q[:, sl].contiguous(), k[:, sl].contiguous(), v[:, sl].contiguous(),
                            g[:, sl].contiguous(), beta[:, sl].contiguous(), s)
            outs.append(o)
        o4 = torch.cat(outs, 1)
        og, Sg = cuda_kda(q, k, v, g, beta, st, force_generic=True)
    assert rel_err(o4.float().cpu().numpy(), o1.float().cpu().numpy()) <= 1e-2
    assert rel_err(s.cpu().numpy(), S1.cpu().numpy()) <= 1e-2
    assert rel_err(o1.float().cpu().numpy(), og.float().cpu().numpy()) <= TOL_BF16
    assert rel_err(S1.cpu().numpy(), Sg.cpu().numpy()) <= TOL_BF16


def test_d128_no_device_wait_timed_out(cuda):
    assert _lib.lib().kda_device_status(0) == 0


def test_d128_gradients_match_oracle(cuda):
    """D = 128 with gradients runs the fp32 generic kernels at an internal chunk of 16 (the
    backward's working set at chunk 64 does not fit shared memory); outputs and every gradient
    against the oracle at the bf16 bound."""
    inp = make_inputs(1, 100, 2, 128, seed=2, state_std=0.1)
    bf = torch.bfloat16
    lv = {}
    for k in ("q", "k", "v", "g", "beta", "state"):
        x = torch.from_numpy(inp[k]).to(cuda)
        lv[k] = (x.to(bf) if k in ("q", "k", "v", "beta") else x).requires_grad_(True)
    o, S = cuda_kda(lv["q"], lv["k"], lv["v"], lv["g"], lv["beta"], lv["state"])
    torch.autograd.backward([o, S], [torch.from_numpy(inp["do"]).to(cuda).to(bf),
                                     torch.from_numpy(inp["dst"]).to(cuda)])
    got = dict(o=o, S_T=S, dq=lv["q"].grad, dk=lv["k"].grad, dv=lv["v"].grad, dg=lv["g"].grad,
               dbeta=lv["beta"].grad, dstate0=lv["state"].grad)
    r = bf16_inputs(inp)
    r["do"] = torch.from_numpy(inp["do"]).to(bf).float().numpy()
    ref = O.fwd_bwd(r, dtype=np.float64)
    for k, x in got.items():
        x = x.detach().float().cpu().numpy()
        assert np.isfinite(x).all(), k
        assert rel_err(x, ref[k]) <= TOL_BF16, (k, rel_err(x, ref[k]))
