"""CPU checks of the oracle's gate restatement (nope_gdn_mlx.py:83-86, 802-816) and its
chain rule, against torch float64 autograd as an independent implementation."""
import numpy as np
import torch

from oracle import kda_oracle as O


def _case(seed=0, B=2, T=5, H=3, D=8):
    rng = np.random.default_rng(seed)
    f = rng.standard_normal((B, T, H, D)) * 3.0
    A_log = np.log(rng.uniform(1.0, 16.0, H))
    dtb = rng.standard_normal(H * D) * 0.5
    b = rng.standard_normal((B, T, H)) * 2.0
    dg = rng.standard_normal((B, T, H, D))
    dbeta = rng.standard_normal((B, T, H))
    return f, A_log, dtb, b, dg, dbeta


def test_softplus_is_stable_and_exact():
    x = np.array([-800.0, -30.0, -1.0, 0.0, 1e-8, 2.5, 40.0, 800.0])
    ref = torch.nn.functional.softplus(torch.from_numpy(x)).numpy()  # x above 20 returns x
    got = O.softplus(x)
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, ref, rtol=1e-15, atol=1e-16)


def test_gates_and_vjp_match_torch_autograd():
    for neg in (False, True):
        f, A_log, dtb, b, dg, dbeta = _case(seed=int(neg))
        g, beta = O.gates(f, A_log, dtb, b, allow_neg_eigval=neg)
        tf, tA, tdtb, tb = (torch.tensor(x, dtype=torch.float64, requires_grad=True)
                            for x in (f, A_log, dtb, b))
        H, D = f.shape[2], f.shape[3]
        tg = -torch.exp(tA).reshape(1, 1, H, 1) * torch.nn.functional.softplus(
            tf + tdtb.reshape(H, D), threshold=1e9)
        tbeta = (2.0 if neg else 1.0) * torch.sigmoid(tb)
        np.testing.assert_allclose(g, tg.detach().numpy(), rtol=1e-13)
        np.testing.assert_allclose(beta, tbeta.detach().numpy(), rtol=1e-13)
        ((tg * torch.from_numpy(dg)).sum() + (tbeta * torch.from_numpy(dbeta)).sum()).backward()
        df, dA, ddtb, db = O.gates_vjp(f, A_log, dtb, b, dg, dbeta, allow_neg_eigval=neg)
        for got, ref in ((df, tf.grad), (dA, tA.grad), (ddtb, tdtb.grad), (db, tb.grad)):
            np.testing.assert_allclose(got, ref.numpy(), rtol=1e-12, atol=1e-14)
