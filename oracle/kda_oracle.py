"""CPU oracle for the chunkwise KDA (Kimi Delta Attention) recurrence -- TEST INFRASTRUCTURE.

This module is a numpy restatement of the reference's KDA oracle paths.  It is the checker,
never the product: only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline / ``--impl reference`` leg import it.  The CUDA path in ``mlx_vit_b200`` never
calls into this file.

Pinning: the restatement is checked (tests/test_oracle.py) against golden vectors produced
by executing the reference's own source (``GatedDeltaLayer._loop_compiled_kda`` and
``GatedDeltaLayer._kda_python_backward_full`` from nope_gdn_mlx.py) on a torch-backed MLX
emulator in float64 (tests/golden/make_golden.py).  MLX itself is not installable here, so
the MLX primitive semantics (exp, matmul, broadcasting) are emulated; the reference's
algorithm code is run unmodified.

Conventions (nope_gdn_mlx.py:616-638, 890-917):
  * inputs q, k, v, g: (B, T, H, D); beta: (B, T, H); state: (B, H, Dv, Dk) or None (zeros)
  * the state is stored [value dim, key dim]; the decay exp(g_t) scales its columns
  * per step: S <- S * exp(g_t)[None, :];  S <- S (I - b k k^T) + b v k^T;  o_t = S q_t
    (output uses the post-update state)
  * q, k, v, beta are cast to the compute dtype, g is used as given (float32 in the
    reference), the state is float32; output is returned in q's dtype.
"""
from __future__ import annotations

import numpy as np


def compiled_forward(q, k, v, g, beta, state=None, dtype=np.float32, return_u=False):
    """Restates ``_loop_compiled_kda`` (nope_gdn_mlx.py:890-917) with the fused step
    ``_kda_step_fused`` (:616-638), including its O(D^3) ``state @ (I - b k k^T)`` form.

    Returns (o, S_T) and, if ``return_u``, u_t = beta_t (v_t - S'_t k_t) for every step
    (the quantity the reference's Metal forward saves for its step backward).
    """
    B, T, H, D = q.shape
    Dv = v.shape[-1]
    q32, k32, v32, b32 = (x.astype(dtype) for x in (q, k, v, beta))
    g = g.astype(dtype)
    S = np.zeros((B, H, Dv, D), dtype) if state is None else state.astype(dtype).copy()
    I = np.eye(D, dtype=dtype)
    outs = np.empty((B, T, H, Dv), dtype)
    us = np.empty((B, T, H, Dv), dtype) if return_u else None
    for t in range(T):
        decay = np.exp(g[:, t])                                    # (B, H, D)
        S = S * decay[..., None, :]                                # column-wise scale
        bt = b32[:, t][..., None, None]                            # (B, H, 1, 1)
        kt, vt = k32[:, t], v32[:, t]
        if return_u:
            us[:, t] = b32[:, t][..., None] * (vt - np.einsum("bhij,bhj->bhi", S, kt))
        k_outer = kt[..., :, None] @ kt[..., None, :]
        S = S @ (I - bt * k_outer)
        S = S + bt * (vt[..., :, None] @ kt[..., None, :])
        outs[:, t] = (S @ q32[:, t][..., :, None])[..., 0]
    o = outs.astype(q.dtype)
    return (o, S, us) if return_u else (o, S)


def step_backward(q, k, v, g, beta, state, do, dstate_final, dtype=np.float32):
    """Restates the reference's hand-derived step backward
    ``GatedDeltaLayer._kda_python_backward_full`` (nope_gdn_mlx.py:3184-3295): a forward
    replay that materialises every S_t, then the reverse-time loop
        gS += do_t q_t^T;  dq_t = S'^T do_t + k_t (u_t . do_t);  du = gS k_t;
        dk_t = gS^T u_t - S'^T (beta_t du);  dbeta_t = du . (v_t - S' k_t);  dv_t = beta_t du;
        dS' = gS - (beta_t du) k_t^T;  dg_t = colsum(dS' * S');  gS = dS' * exp(g_t).
    These gradients equal autograd through ``_loop_compiled_kda`` (checked against the golden
    vectors).  Returns (dq, dk, dv, dg, dbeta, dstate0) in ``dtype``.
    """
    B, T, H, D = q.shape
    Dv = v.shape[-1]
    q, k, v, g, beta, do = (x.astype(dtype) for x in (q, k, v, g, beta, do))
    S0 = np.zeros((B, H, Dv, D), dtype) if state is None else state.astype(dtype)
    # forward replay (S_list[t] = state after step t-1's update)
    S_list = [S0]
    S = S0
    us = np.empty((B, T, H, Dv), dtype)
    for t in range(T):
        Sp = S * np.exp(g[:, t])[..., None, :]
        u = beta[:, t][..., None] * (v[:, t] - np.einsum("bhij,bhj->bhi", Sp, k[:, t]))
        us[:, t] = u
        S = Sp + u[..., :, None] * k[:, t][..., None, :]
        S_list.append(S)
    gS = dstate_final.astype(dtype).copy()
    dq = np.empty_like(q); dk = np.empty_like(k); dv = np.empty((B, T, H, Dv), dtype)
    dg = np.empty_like(g); dbeta = np.empty_like(beta)
    for t in range(T - 1, -1, -1):
        qt, kt, vt, ut, dot = q[:, t], k[:, t], v[:, t], us[:, t], do[:, t]
        St = S_list[t + 1]
        Sp = St - ut[..., :, None] * kt[..., None, :]
        gS = gS + dot[..., :, None] * qt[..., None, :]
        ud = (ut * dot).sum(-1, keepdims=True)
        dq[:, t] = np.einsum("bhlj,bhl->bhj", Sp, dot) + kt * ud
        du = np.einsum("bhij,bhj->bhi", gS, kt)
        dk_outer = np.einsum("bhij,bhi->bhj", gS, ut)
        w = vt - np.einsum("bhij,bhj->bhi", Sp, kt)
        dbeta[:, t] = (du * w).sum(-1)
        dw = beta[:, t][..., None] * du
        dv[:, t] = dw
        dSp = gS - dw[..., :, None] * kt[..., None, :]
        dk[:, t] = dk_outer - np.einsum("bhlj,bhl->bhj", Sp, dw)
        dg[:, t] = (dSp * Sp).sum(-2)
        gS = dSp * np.exp(g[:, t])[..., None, :]
    return dq, dk, dv, dg, dbeta, gS


def fwd_bwd(inp: dict, dtype=np.float64):
    """Oracle forward + VJP on an input dict from ``mlx_vit_b200.synthetic.make_inputs``.

    Returns dict(o, S_T, dq, dk, dv, dg, dbeta, dstate0) in ``dtype``.
    """
    o, S_T = compiled_forward(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"],
                              inp["state"], dtype=dtype)
    dq, dk, dv, dg, db, ds0 = step_backward(inp["q"], inp["k"], inp["v"], inp["g"],
                                            inp["beta"], inp["state"], inp["do"],
                                            inp["dst"], dtype=dtype)
    return dict(o=o.astype(dtype), S_T=S_T, dq=dq, dk=dk, dv=dv, dg=dg, dbeta=db, dstate0=ds0)


def chunkwise_forward(q, k, v, g, beta, state=None, chunk=64, dtype=np.float64):
    """Restates the chunkwise WY forward ``_chunkwise_kda_forward`` (nope_gdn_mlx.py:2318-2456)
    on the (B, T, H, D) layout: pad T to a multiple of ``chunk`` with g = 0, beta = 0,
    q = k = v = 0 (:2355-2361); per chunk gamma = cumsum(g) (:576), K_proj = e^gamma k,
    K_back = e^(gamma_C - gamma) k, Q' = e^gamma q (:577-580, :2399);
    M[s,t] = sum_d k_s k_t e^min(gamma_t - gamma_s, 0), M_oq[s,t] = sum_d k_s q_t e^min(..)
    (kernel 3, :1301-1336); IA = I + beta_row * M^T strict-lower (:585-597);
    U = solve(IA, beta (V - K_proj S^T)) (:600-603 + kernel 1);
    O = Q' S^T + (M_oq^T * tril) U;  S' = e^gamma_C * S + U^T K_back (:606-613).
    The chunkwise kernels in ``mlx_vit_b200/csrc`` implement this same algebra.
    Returns (o, S_T, chunk_states) with chunk_states[b, h, c] = state entering chunk c.
    """
    B, T, H, D = q.shape
    Dv = v.shape[-1]
    C = chunk
    nc = (T + C - 1) // C
    Tp = nc * C

    def pad(x):
        w = [(0, 0)] * x.ndim
        w[1] = (0, Tp - T)
        return np.pad(x.astype(dtype), w)
    q, k, v, g, beta = (pad(x) for x in (q, k, v, g, beta))
    S = np.zeros((B, H, Dv, D), dtype) if state is None else state.astype(dtype).copy()
    o = np.zeros((B, Tp, H, Dv), dtype)
    states = np.zeros((B, H, nc, Dv, D), dtype)
    tril_strict = np.tril(np.ones((C, C), bool), -1)
    tril_incl = np.tril(np.ones((C, C), bool), 0)
    for c in range(nc):
        sl = slice(c * C, (c + 1) * C)
        # (B, H, C, D) views
        qc, kc, vc, gc = (x[:, sl].transpose(0, 2, 1, 3) for x in (q, k, v, g))
        bc = beta[:, sl].transpose(0, 2, 1)                        # (B, H, C)
        states[:, :, c] = S
        gam = np.cumsum(gc, axis=2)
        eg = np.exp(gam)
        Kp, Qp = eg * kc, eg * qc
        Kb = np.exp(gam[:, :, -1:, :] - gam) * kc
        # E[t, s, d] = exp(min(gamma_t - gamma_s, 0))
        E = np.exp(np.minimum(gam[:, :, :, None, :] - gam[:, :, None, :, :], 0.0))
        Mkk = np.einsum("bhtd,bhsd,bhtsd->bhts", kc, kc, E)           # [t, s]
        Mqk = np.einsum("bhtd,bhsd,bhtsd->bhts", qc, kc, E)
        A = np.where(tril_strict, bc[..., :, None] * Mkk, 0.0)
        P = np.where(tril_incl, Mqk, 0.0)
        R = bc[..., None] * (vc - Kp @ np.swapaxes(S, -1, -2))
        U = np.linalg.solve(np.eye(C) + A, R)
        O = Qp @ np.swapaxes(S, -1, -2) + P @ U
        S = np.exp(gam[:, :, -1, :])[..., None, :] * S + np.swapaxes(U, -1, -2) @ Kb
        o[:, sl] = O.transpose(0, 2, 1, 3)
    return o[:, :T], S, states


def softplus(x):
    """Stable softplus log(1 + e^x) = log1p(e^-|x|) + max(x, 0) (nope_gdn_mlx.py:83-86)."""
    return np.log1p(np.exp(-np.abs(x))) + np.maximum(x, 0.0)


def _sigmoid(x):
    return 0.5 * (1.0 + np.tanh(0.5 * x))


def gates(f, A_log, dt_bias, b, allow_neg_eigval=False, dtype=np.float64):
    """Decay and write gates of the channel-wise layer (nope_gdn_mlx.py:802-816):
    g = -exp(A_log[h]) * softplus(f + dt_bias[h, :]),  beta = s * sigmoid(b), s = 2 if
    allow_neg_eigval else 1.  f: (B, T, H, D); A_log: (H,); dt_bias: (H*D,); b: (B, T, H)."""
    B, T, H, D = f.shape
    x = f.astype(dtype) + dt_bias.astype(dtype).reshape(H, D)
    g = -np.exp(A_log.astype(dtype)).reshape(1, 1, H, 1) * softplus(x)
    beta = (2.0 if allow_neg_eigval else 1.0) * _sigmoid(b.astype(dtype))
    return g, beta


def gates_vjp(f, A_log, dt_bias, b, dg, dbeta, allow_neg_eigval=False, dtype=np.float64):
    """Chain rule through ``gates``: returns (df, dA_log, ddt_bias, db).

    d g / d x = -exp(A_log) * sigmoid(x) (softplus' = sigmoid), d g / d A_log = g,
    d beta / d b = beta * (1 - beta / s)."""
    B, T, H, D = f.shape
    x = f.astype(dtype) + dt_bias.astype(dtype).reshape(H, D)
    A = np.exp(A_log.astype(dtype)).reshape(1, 1, H, 1)
    g = -A * softplus(x)
    df = dg.astype(dtype) * (-A) * _sigmoid(x)
    dA_log = (dg.astype(dtype) * g).sum(axis=(0, 1, 3))
    ddt_bias = df.sum(axis=(0, 1)).reshape(H * D)
    s = 2.0 if allow_neg_eigval else 1.0
    beta = s * _sigmoid(b.astype(dtype))
    db = dbeta.astype(dtype) * beta * (1.0 - beta / s)
    return df, dA_log, ddt_bias, db
