"""GPU parity of the token-by-token forward (kda_fwd_recurrent) against the oracle: fp32 I/O at
1e-4 relative, bf16 I/O at 2e-2 (oracle in float64 on the same bf16-rounded inputs); a decode
loop of single tokens equals one chunked pass; cuda_kda routes short no-grad calls to it."""
import numpy as np
import pytest
import torch

from kda_testutil import rel_err, TOL_FP32, TOL_BF16
from mlx_vit_b200 import _lib, cuda_kda, kda_recurrent
from mlx_vit_b200.synthetic import make_inputs
from oracle import kda_oracle as O

pytestmark = pytest.mark.gpu


def dev_inputs(inp, dev, dtype):
    t = {k: torch.from_numpy(inp[k]).to(dev) for k in ("q", "k", "v", "g", "beta", "state")}
    for k in ("q", "k", "v", "beta"):
        t[k] = t[k].to(dtype)
    return t


@pytest.mark.parametrize("D", [16, 32, 64, 128])
@pytest.mark.parametrize("T", [1, 5, 16, 40])
def test_recurrent_fp32_matches_oracle(cuda, D, T):
    inp = make_inputs(2, T, 3, D, seed=D + T, state_std=0.1, with_grads=False)
    ref_o, ref_S = O.compiled_forward(**inp, dtype=np.float64)
    t = dev_inputs(inp, cuda, torch.float32)
    o, S = kda_recurrent(t["q"], t["k"], t["v"], t["g"], t["beta"], t["state"])
    assert rel_err(o.cpu().numpy(), ref_o) <= TOL_FP32
    assert rel_err(S.cpu().numpy(), ref_S) <= TOL_FP32


@pytest.mark.parametrize("D", [64, 128])
def test_recurrent_bf16_matches_oracle(cuda, D):
    inp = make_inputs(1, 12, 4, D, seed=D, state_std=0.1, with_grads=False)
    r = dict(inp)
    for k in ("q", "k", "v", "beta"):
        r[k] = torch.from_numpy(inp[k]).to(torch.bfloat16).float().numpy()
    ref_o, ref_S = O.compiled_forward(**r, dtype=np.float64)
    t = dev_inputs(inp, cuda, torch.bfloat16)
    o, S = kda_recurrent(t["q"], t["k"], t["v"], t["g"], t["beta"], t["state"])
    assert rel_err(o.float().cpu().numpy(), ref_o) <= TOL_BF16
    assert rel_err(S.cpu().numpy(), ref_S) <= TOL_BF16


def test_decode_loop_equals_chunked_pass(cuda):
    """Decoding token by token with the state carried (cuda_kda routes T = 1 without gradients
    to the step kernel) reproduces one chunked pass over the whole sequence."""
    inp = make_inputs(1, 100, 2, 64, seed=5, state_std=0.1, with_grads=False)
    t = dev_inputs(inp, cuda, torch.float32)
    c0 = _lib.lib().kda_launch_counter()
    with torch.no_grad():
        o_full, S_full = cuda_kda(t["q"], t["k"], t["v"], t["g"], t["beta"], t["state"])
        s, outs = t["state"], []
        for i in range(100):
            sl = slice(i, i + 1)
            o, s = cuda_kda(t["q"][:, sl], t["k"][:, sl], t["v"][:, sl], t["g"][:, sl], t["beta"][:, sl], s)
            outs.append(o)
    torch.cuda.synchronize()
    # one launch per decoded token (the chunked pass is a single generic launch here)
    assert _lib.lib().kda_launch_counter() - c0 == 100 + 1
    assert rel_err(torch.cat(outs, 1).cpu().numpy(), o_full.cpu().numpy()) <= TOL_FP32
    assert rel_err(s.cpu().numpy(), S_full.cpu().numpy()) <= TOL_FP32


def test_recurrent_rejects_unsupported_dim(cuda):
    inp = make_inputs(1, 4, 1, 48, seed=1, state_std=0.0, with_grads=False)
    t = dev_inputs(inp, cuda, torch.float32)
    with pytest.raises(Exception):
        kda_recurrent(t["q"], t["k"], t["v"], t["g"], t["beta"])


def test_low_level_wrappers_take_strided_and_bf16_operands(cuda):
    """The public low-level calls (kda_recurrent, kda_forward, kda_backward) accept what
    cuda_kda accepts: a strided time slice of a B = 2 batch and a bf16 g / state are made dense
    float32 before the kernel reads them, and give the dense float32 answer."""
    import torch
    from mlx_vit_b200 import kda_recurrent, kda_forward, kda_backward
    from mlx_vit_b200.synthetic import make_inputs
    inp = make_inputs(2, 40, 2, 64, seed=12, state_std=0.1)
    t = {k: torch.from_numpy(v).to(cuda) for k, v in inp.items()}
    sl = slice(5, 9)
    view = {k: (t[k][:, sl] if t[k].dim() >= 3 and k not in ("state", "dst") else t[k]) for k in t}
    assert not view["q"].is_contiguous()
    dense = {k: x.contiguous() for k, x in view.items()}
    o1, S1 = kda_recurrent(view["q"], view["k"], view["v"], view["g"].to(torch.bfloat16),
                           view["beta"], view["state"].to(torch.bfloat16))
    o2, S2 = kda_recurrent(dense["q"], dense["k"], dense["v"],
                           dense["g"].to(torch.bfloat16).float(), dense["beta"],
                           dense["state"].to(torch.bfloat16).float())
    assert torch.equal(o1, o2) and torch.equal(S1, S2)
    bf = torch.bfloat16
    qv, kv, vv = (x.to(bf)[:, :, :] for x in (t["q"], t["k"], t["v"]))
    args = (qv[:, 1:], kv[:, 1:], vv[:, 1:], t["g"][:, 1:].to(bf), t["beta"][:, 1:].to(bf), t["state"])
    o, S, cs = kda_forward(*args, 64, save_states=True)
    ref_o, ref_S, ref_cs = kda_forward(*(x.contiguous() if x is not None else None for x in args[:3]),
                                       args[3].float().contiguous(), args[4].contiguous(), args[5], 64,
                                       save_states=True)
    assert torch.equal(o, ref_o) and torch.equal(S, ref_S)
    do = t["do"][:, 1:].to(bf)
    g1 = kda_backward(*args, cs, do, None, 64)
    g2 = kda_backward(*(x.contiguous() for x in args[:3]), args[3].float().contiguous(),
                      args[4].contiguous(), args[5], ref_cs, do.contiguous(), None, 64)
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)
