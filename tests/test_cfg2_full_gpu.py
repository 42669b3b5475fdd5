"""GPU parity at the benchmarked shapes: B8 H12 T1568 D64 chunk 64 (configs 1 and 2).

At this size the persistent chunk kernels (one CTA per SM) each walk about 16 of the 2400
chunks, so the paths that only run when a CTA owns several chunks -- the next-chunk TMA
prefetch, the mbarrier phase flip and the wait on the previous chunk's bulk stores -- are
exercised exactly as the benchmark runs them.  The whole batch runs on the GPU; the oracle (the
restated ``compiled`` path and its step backward, float64 on the same bf16-rounded inputs) runs
on a fixed sample of 8 (b, h) sequences spread over b and h, which are independent of the
others (the reference folds heads into the batch, nope_gdn_mlx.py:833-838).
Tolerance: max|delta| / max|ref| <= 2e-2 per output and gradient, per sampled sequence."""
import numpy as np
import pytest
import torch

from kda_testutil import rel_err, TOL_BF16
from mlx_vit_b200 import cuda_kda, cuda_kda_gated
from mlx_vit_b200.synthetic import make_inputs
from oracle import kda_oracle as O

pytestmark = pytest.mark.gpu

B, T, H, D = 8, 1568, 12, 64
PAIRS = [(0, 0), (1, 5), (2, 11), (3, 3), (4, 8), (5, 1), (6, 10), (7, 6)]
GRAD_KEYS = ("q", "k", "v", "g", "beta", "state")


def bf16_round(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16).float().numpy()


def sample(inp):
    """The sampled (b, h) sequences as a batch of P single-head sequences."""
    out = {}
    for k, x in inp.items():
        if x.ndim == 4 and x.shape[1] == T:      # (B, T, H, D)
            out[k] = np.stack([x[b, :, h] for b, h in PAIRS])[:, :, None]
        elif x.ndim == 3:                        # (B, T, H)
            out[k] = np.stack([x[b, :, h] for b, h in PAIRS])[:, :, None]
        else:                                    # (B, H, D, D)
            out[k] = np.stack([x[b, h] for b, h in PAIRS])[:, None]
    return out


def unsample(x, kind):
    """The same sequences picked out of a full GPU result (numpy)."""
    if kind == "state":
        return np.stack([x[b, h] for b, h in PAIRS])[:, None]
    return np.stack([x[b, :, h] for b, h in PAIRS])[:, :, None]


def chunk_count_exceeds_persistent_grid():
    n_sm = torch.cuda.get_device_properties(0).multi_processor_count
    assert B * H * ((T + 63) // 64) > 2 * n_sm


def test_cfg2_fwd_bwd_full_shape(cuda):
    chunk_count_exceeds_persistent_grid()
    inp = make_inputs(B, T, H, D, seed=2024, state_std=0.1)
    bf = torch.bfloat16
    leaves = {}
    for k in GRAD_KEYS:
        x = torch.from_numpy(inp[k]).to(cuda)
        leaves[k] = (x.to(bf) if k in ("q", "k", "v", "beta") else x).requires_grad_(True)
    do = torch.from_numpy(inp["do"]).to(cuda).to(bf)
    dst = torch.from_numpy(inp["dst"]).to(cuda)
    o, S = cuda_kda(leaves["q"], leaves["k"], leaves["v"], leaves["g"], leaves["beta"],
                    leaves["state"], chunk_size=64)
    torch.autograd.backward([o, S], [do, dst])
    got = dict(o=o, S_T=S, dq=leaves["q"].grad, dk=leaves["k"].grad, dv=leaves["v"].grad,
               dg=leaves["g"].grad, dbeta=leaves["beta"].grad, dstate0=leaves["state"].grad)
    got = {k: v.detach().float().cpu().numpy() for k, v in got.items()}
    r = sample(inp)
    for k in ("q", "k", "v", "beta", "do"):
        r[k] = bf16_round(r[k])
    ref = O.fwd_bwd(r, dtype=np.float64)
    for k, x in got.items():
        assert np.isfinite(x).all(), k
        kind = "state" if k in ("S_T", "dstate0") else "seq"
        mine = unsample(x, kind)
        for i in range(len(PAIRS)):
            e = rel_err(mine[i], ref[k][i])
            assert e <= TOL_BF16, (k, PAIRS[i], e)


def test_cfg1_inference_forward_full_shape(cuda):
    """Config 1: forward only (no saved record), zero initial state, output and final state."""
    chunk_count_exceeds_persistent_grid()
    inp = make_inputs(B, T, H, D, seed=77, state_std=0.0, with_grads=False)
    bf = torch.bfloat16
    t = {k: torch.from_numpy(v).to(cuda) for k, v in inp.items()}
    with torch.no_grad():
        o, S = cuda_kda(t["q"].to(bf), t["k"].to(bf), t["v"].to(bf), t["g"], t["beta"].to(bf), None)
    assert o.dtype == bf and S.dtype == torch.float32
    r = sample(inp)
    for k in ("q", "k", "v", "beta"):
        r[k] = bf16_round(r[k])
    o_ref, S_ref = O.compiled_forward(r["q"], r["k"], r["v"], r["g"], r["beta"], None,
                                      dtype=np.float64)
    mo = unsample(o.float().cpu().numpy(), "seq")
    ms = unsample(S.cpu().numpy(), "state")
    for i in range(len(PAIRS)):
        assert rel_err(mo[i], o_ref[i]) <= TOL_BF16, ("o", PAIRS[i], rel_err(mo[i], o_ref[i]))
        assert rel_err(ms[i], S_ref[i]) <= TOL_BF16, ("S_T", PAIRS[i], rel_err(ms[i], S_ref[i]))


def test_cfg2_gated_reference_init_full_shape(cuda):
    """The fused-gate entry points at the benchmarked shape with the reference's gate init
    (A = e^{A_log} uniform in [1, 16], nope_gdn_mlx.py:748-751), so most chunks are "big"
    (exact diagonal blocks) and mix with mild ones across heads.  Recurrence outputs and the
    write-gate gradient against the oracle at 2e-2 on the sampled sequences; df against the
    oracle with the bf16 dg bound carried through the gate (A * 2e-2 * max|dg|); dA_log and
    ddt_bias checked for internal consistency with df over the whole batch."""
    chunk_count_exceeds_persistent_grid()
    rng = np.random.default_rng(31)
    f32 = np.float32
    inp = make_inputs(B, T, H, D, seed=31, state_std=0.1)
    f = rng.standard_normal((B, T, H, D), dtype=f32)
    bl = rng.standard_normal((B, T, H), dtype=f32)
    A_log = np.log(rng.uniform(1.0, 16.0, H)).astype(f32)
    dtb = (rng.standard_normal(H * D) * 0.3).astype(f32)
    bf = torch.bfloat16
    lv = {}
    for k in ("q", "k", "v"):
        lv[k] = torch.from_numpy(inp[k]).to(cuda).to(bf).requires_grad_(True)
    lv["f"] = torch.from_numpy(f).to(cuda).to(bf).requires_grad_(True)
    lv["b"] = torch.from_numpy(bl).to(cuda).to(bf).requires_grad_(True)
    lv["A_log"] = torch.from_numpy(A_log).to(cuda).requires_grad_(True)
    lv["dt_bias"] = torch.from_numpy(dtb).to(cuda).requires_grad_(True)
    lv["state"] = torch.from_numpy(inp["state"]).to(cuda).requires_grad_(True)
    o, S = cuda_kda_gated(lv["q"], lv["k"], lv["v"], lv["f"], lv["A_log"], lv["dt_bias"], lv["b"],
                          lv["state"])
    do = torch.from_numpy(inp["do"]).to(cuda).to(bf)
    dst = torch.from_numpy(inp["dst"]).to(cuda)
    torch.autograd.backward([o, S], [do, dst])
    got = dict(o=o, S_T=S, dq=lv["q"].grad, dk=lv["k"].grad, dv=lv["v"].grad, df=lv["f"].grad,
               db=lv["b"].grad, dstate0=lv["state"].grad, dA_log=lv["A_log"].grad,
               ddt_bias=lv["dt_bias"].grad)
    got = {k: v.detach().float().cpu().numpy() for k, v in got.items()}
    for k, x in got.items():
        assert np.isfinite(x).all(), k

    full = dict(inp, f=f, b=bl)
    r = sample(full)
    for k in ("q", "k", "v", "f", "b", "do"):
        r[k] = bf16_round(r[k])
    hs = np.array([h for _, h in PAIRS])
    # each sampled sequence has its own head's gate parameters
    x = r["f"].astype(np.float64) + dtb.reshape(H, D)[hs][:, None, None, :]
    A = np.exp(A_log.astype(np.float64))[hs][:, None, None, None]
    sp = O.softplus(x)
    g = -A * sp
    sig = 1.0 / (1.0 + np.exp(-x))
    beta = 1.0 / (1.0 + np.exp(-r["b"].astype(np.float64)))
    ref = O.fwd_bwd(dict(q=r["q"], k=r["k"], v=r["v"], g=g, beta=beta, state=r["state"],
                         do=r["do"], dst=r["dst"]), dtype=np.float64)
    df_ref = ref["dg"] * (-A) * sig
    db_ref = ref["dbeta"] * beta * (1.0 - beta)
    for k in ("o", "S_T", "dq", "dk", "dv", "dstate0", "db"):
        kind = "state" if k in ("S_T", "dstate0") else "seq"
        mine = unsample(got[k], kind)
        want = db_ref if k == "db" else ref[k]
        for i in range(len(PAIRS)):
            e = rel_err(mine[i], want[i])
            assert e <= TOL_BF16, (k, PAIRS[i], e)
    mine_df = unsample(got["df"], "seq")
    for i in range(len(PAIRS)):
        bound = A[i, 0, 0, 0] * TOL_BF16 * np.abs(ref["dg"][i]).max()
        assert np.abs(mine_df[i] - df_ref[i]).max() <= bound, (PAIRS[i],)
    # parameter gradients: sums of the kernel's own df over (b, t), up to df's bf16 rounding
    dfa = got["df"].astype(np.float64)
    rt = 2.0 ** -8
    assert (np.abs(got["ddt_bias"] - dfa.sum(axis=(0, 1)).reshape(-1)) <=
            rt * np.abs(dfa).sum(axis=(0, 1)).reshape(-1) + 1e-6).all()
    xf = bf16_round(f).astype(np.float64) + dtb.reshape(H, D)
    term = dfa * O.softplus(xf) * (1.0 + np.exp(-xf))
    assert (np.abs(got["dA_log"] - term.sum(axis=(0, 1, 3))) <=
            rt * np.abs(term).sum(axis=(0, 1, 3)) + 1e-6).all()


def test_cfg2_no_device_wait_timed_out(cuda):
    from mlx_vit_b200 import _lib
    assert _lib.lib().kda_device_status(0) == 0
