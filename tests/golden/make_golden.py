"""Generate the golden KDA fixtures by running the reference's own source.

This script runs only where the reference checkout is present (it is not needed, and not
run, on the GPU box or by the test-suite).  It

1. installs the torch-backed ``mlx`` emulator (``mlx_emul.py``) with ``mx.float32``
   mapped to float64,
2. imports the reference module ``nope_gdn_mlx.py`` unmodified,
3. runs ``GatedDeltaLayer._loop_compiled_kda`` (nope_gdn_mlx.py:890-917, the ``compiled``
   path, one ``_kda_step_fused`` step per token, :616-638) on seeded float32 inputs from
   ``mlx_vit_b200.synthetic.make_inputs`` and takes gradients of
   ``sum(o * dO) + sum(S_T * dS_T)`` with autograd (what MLX autograd computes for that path),
4. cross-checks those gradients against the reference's hand-written step backward
   ``GatedDeltaLayer._kda_python_backward_full`` (:3184-3295) executed on the same inputs,
5. writes ``<case>.npz`` with the float32-rounded golden outputs and gradients, plus
   ``manifest.json`` with the shapes, seeds, input checksums and cross-check errors.

Inputs are not stored: the tests rebuild them from the seed and compare the checksum.

Usage:  python tests/golden/make_golden.py /path/to/reference
        (or with the reference checkout's directory in KDA_REFERENCE_DIR)
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import mlx_emul  # noqa: E402
from mlx_vit_b200.synthetic import make_inputs  # noqa: E402

# name: (B, T, H, D, chunk, seed, state_std)
CASES = {
    # the reference's own verify shape (nope_gdn_mlx.py:4838, B=1 L=16 H=2 D=16 chunk=8)
    "verify_b1t16h2d16": (1, 16, 2, 16, 8, 0, 0.0),
    # ragged T (not a multiple of the chunk), nonzero initial state
    "ragged_b2t100h2d32": (2, 100, 2, 32, 32, 1, 0.1),
    # one partial chunk only
    "short_b1t5h1d64": (1, 5, 1, 64, 64, 2, 0.1),
    # B=2 H=4 T=256 D=64 chunk=64, zero initial state
    "cfg0_b2t256h4d64": (2, 256, 4, 64, 64, 0, 0.0),
    # config-2 distributions (state ~ N(0, 0.1^2)), small T, ragged last chunk
    "cfg2small_b1t200h2d64": (1, 200, 2, 64, 64, 3, 0.1),
}


def checksum(arrs: dict) -> str:
    h = hashlib.sha256()
    for k in sorted(arrs):
        h.update(k.encode())
        h.update(np.ascontiguousarray(arrs[k]).tobytes())
    return h.hexdigest()[:16]


def run_case(ref, B, T, H, D, seed, state_std):
    G = ref.GatedDeltaLayer
    inp = make_inputs(B, T, H, D, seed=seed, state_std=state_std)
    t64 = {k: torch.from_numpy(v).to(torch.float64) for k, v in inp.items()}
    leaves = {k: t64[k].clone().requires_grad_(True) for k in ("q", "k", "v", "g", "beta", "state")}
    o, S_T = G._loop_compiled_kda(None, leaves["q"], leaves["k"], leaves["v"], leaves["g"],
                                  leaves["beta"], leaves["state"])
    loss = (o * t64["do"]).sum() + (S_T * t64["dst"]).sum()
    loss.backward()
    grads = {k: leaves[k].grad.detach() for k in leaves}

    # cross-check: the reference's hand-written step backward, run on the (B*H, L, D) fold
    def fold(x):  # (B, T, H, D) -> (B*H, T, D)
        return x.permute(0, 2, 1, 3).reshape(B * H, T, D)
    qf, kf, vf, gf = (fold(t64[n]) for n in ("q", "k", "v", "g"))
    bf = t64["beta"].permute(0, 2, 1).reshape(B * H, T)
    S = t64["state"].reshape(B * H, D, D).clone()
    us = []
    for t in range(T):  # u_t = beta_t (v_t - S' k_t), the quantity the Metal forward saves
        Sp = S * torch.exp(gf[:, t])[:, None, :]
        u = bf[:, t, None] * (vf[:, t] - torch.einsum("bij,bj->bi", Sp, kf[:, t]))
        S = Sp + u[:, :, None] * kf[:, t, None, :]
        us.append(u)
    u = torch.stack(us, 1)
    dq, dk, dv, dg, dbeta, dS0 = G._kda_python_backward_full(
        qf, kf, vf, gf, bf, u, S, t64["state"].reshape(B * H, D, D), fold(t64["do"]),
        t64["dst"].reshape(B * H, D, D))

    def unfold(x):
        return x.reshape(B, H, T, D).permute(0, 2, 1, 3)
    hand = dict(q=unfold(dq), k=unfold(dk), v=unfold(dv), g=unfold(dg),
                beta=dbeta.reshape(B, H, T).permute(0, 2, 1), state=dS0.reshape(B, H, D, D))
    xerr = {}
    for n in hand:
        ref_g = grads[n]
        xerr[n] = float((hand[n] - ref_g).abs().max() / max(ref_g.abs().max().item(), 1e-30))
    out = dict(o=o.detach(), S_T=S_T.detach(), dq=grads["q"], dk=grads["k"], dv=grads["v"],
               dg=grads["g"], dbeta=grads["beta"], dstate0=grads["state"])
    out = {k: v.numpy().astype(np.float32) for k, v in out.items()}
    return inp, out, xerr


def main():
    ref_dir = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KDA_REFERENCE_DIR")
    if not ref_dir:
        sys.exit("usage: make_golden.py /path/to/reference (the checkout holding nope_gdn_mlx.py)")
    mlx_emul.install(torch.float64)
    spec = importlib.util.spec_from_file_location("nope_gdn_mlx", os.path.join(ref_dir, "nope_gdn_mlx.py"))
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    manifest = {"generator": "tests/golden/make_golden.py",
                "reference_functions": ["GatedDeltaLayer._loop_compiled_kda (nope_gdn_mlx.py:890-917)",
                                        "_kda_step_fused (nope_gdn_mlx.py:616-638)",
                                        "GatedDeltaLayer._kda_python_backward_full (nope_gdn_mlx.py:3184-3295)"],
                "precision": "float64 (mx.float32 emulated as float64), stored as float32",
                "cases": {}}
    for name, (B, T, H, D, C, seed, sstd) in CASES.items():
        inp, out, xerr = run_case(ref, B, T, H, D, seed, sstd)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
        manifest["cases"][name] = dict(B=B, T=T, H=H, D=D, chunk=C, seed=seed, state_std=sstd,
                                       input_checksum=checksum(inp),
                                       hand_backward_vs_autograd_rel=xerr)
        print(name, "hand-vs-autograd rel err:", {k: f"{v:.1e}" for k, v in xerr.items()})
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)


if __name__ == "__main__":
    main()
