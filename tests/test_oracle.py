"""CPU: the oracle restatement against the golden vectors made by running the reference's own
source (tests/golden/make_golden.py), and the chunkwise algebra against the recurrence."""
import numpy as np
import pytest

from kda_testutil import manifest, golden, rel_err, OUT_KEYS
from mlx_vit_b200.synthetic import make_inputs
from oracle import kda_oracle as O

import sys, os
sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
from make_golden import checksum  # noqa: E402

CASES = manifest()["cases"]


@pytest.mark.parametrize("name", sorted(CASES))
def test_inputs_reproduce(name):
    c = CASES[name]
    inp = make_inputs(c["B"], c["T"], c["H"], c["D"], seed=c["seed"], state_std=c["state_std"])
    assert checksum(inp) == c["input_checksum"]


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_golden(name):
    c = CASES[name]
    inp = make_inputs(c["B"], c["T"], c["H"], c["D"], seed=c["seed"], state_std=c["state_std"])
    gold = golden(name)
    r = O.fwd_bwd(inp, dtype=np.float64)
    for k in OUT_KEYS:
        assert rel_err(r[k], gold[k]) < 1e-6, (name, k)
    # the reference's hand backward agreed with autograd when the fixtures were made
    for k, e in c["hand_backward_vs_autograd_rel"].items():
        assert e < 1e-12, (name, k, e)


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_fp32_within_north_star_tolerance(name):
    c = CASES[name]
    inp = make_inputs(c["B"], c["T"], c["H"], c["D"], seed=c["seed"], state_std=c["state_std"])
    gold = golden(name)
    r = O.fwd_bwd(inp, dtype=np.float32)
    for k in OUT_KEYS:
        assert rel_err(r[k], gold[k]) < 1e-5, (name, k)


@pytest.mark.parametrize("name", sorted(CASES))
def test_chunkwise_algebra_equals_recurrence(name):
    c = CASES[name]
    inp = make_inputs(c["B"], c["T"], c["H"], c["D"], seed=c["seed"], state_std=c["state_std"])
    gold = golden(name)
    for chunk in sorted({c["chunk"], 16, 64}):
        o, S, states = O.chunkwise_forward(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"],
                                           inp["state"], chunk=chunk)
        assert rel_err(o, gold["o"]) < 1e-6
        assert rel_err(S, gold["S_T"]) < 1e-6
        np.testing.assert_array_equal(states[:, :, 0], inp["state"])


def test_chunkwise_handles_strong_decay():
    # gamma spans far beyond exp's range inside a chunk: the clipped-difference form stays finite
    inp = make_inputs(1, 96, 1, 16, seed=5, state_std=0.1)
    inp["g"] = inp["g"] * 40.0
    o_ref, S_ref = O.compiled_forward(**{k: inp[k] for k in ("q", "k", "v", "g", "beta", "state")},
                                      dtype=np.float64)
    o, S, _ = O.chunkwise_forward(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], inp["state"], chunk=64)
    assert np.isfinite(o).all() and rel_err(o, o_ref) < 1e-6 and rel_err(S, S_ref) < 1e-9
