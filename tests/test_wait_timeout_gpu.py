"""The device-side bounded-wait failure path, made to run without faulting anything: with the
test-only flag KDA_FLAG_DEBUG_WAIT_TIMEOUT the forward's state scan first waits a few polls on
an mbarrier that nothing completes, before it issues any copy or holds tensor memory.  The wait
gives up, the kernel records KDA_ERR_TIMEOUT in the device status word and returns; the host
reads the status through kda_device_status, and the context stays usable."""
import numpy as np
import pytest
import torch

from kda_testutil import rel_err, TOL_BF16
from mlx_vit_b200 import _lib, kda_forward
from mlx_vit_b200.synthetic import make_inputs
from oracle import kda_oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports_timeout(cuda):
    L = _lib.lib()
    assert L.kda_device_status(1) == 0
    inp = make_inputs(1, 130, 2, 64, seed=3, state_std=0.1, with_grads=False)
    bf = torch.bfloat16
    t = {k: torch.from_numpy(v).to(cuda) for k, v in inp.items()}
    args = (t["q"].to(bf), t["k"].to(bf), t["v"].to(bf), t["g"], t["beta"].to(bf), t["state"])
    kda_forward(*args, 64, flags=_lib.KDA_FLAG_DEBUG_WAIT_TIMEOUT)
    assert L.kda_device_status(1) == _lib.STATUS_CODE["KDA_ERR_TIMEOUT"]
    assert L.kda_device_status(0) == 0  # the read with reset cleared it
    # the context is intact: the same call without the hook computes the right answer
    o, S, _ = kda_forward(*args, 64)
    r = dict(inp)
    for k in ("q", "k", "v", "beta"):
        r[k] = torch.from_numpy(inp[k]).to(bf).float().numpy()
    o_ref, S_ref = O.compiled_forward(r["q"], r["k"], r["v"], r["g"], r["beta"], r["state"],
                                      dtype=np.float64)
    assert rel_err(o.float().cpu().numpy(), o_ref) <= TOL_BF16
    assert rel_err(S.cpu().numpy(), S_ref) <= TOL_BF16
    assert L.kda_device_status(0) == 0
