"""CPU: the seeded synthetic weights reproduce the reference's own seed-0
initialisation of the tiny configuration (checksums recorded from the
reference model by tests/golden/make_golden.py)."""

import os

import numpy as np

from utttcompanion_b200.workloads import CONFIG_TINY, reference_init_state_dict

from conftest import GOLDEN


def test_reference_init_order_reproduced_for_config_1():
    g = np.load(os.path.join(GOLDEN, "init_cfg1.npz"))
    sd = reference_init_state_dict(CONFIG_TINY, seed=0)
    names = [str(n) for n in g["names"]]
    assert sorted(sd) == names
    for i, n in enumerate(names):
        t = sd[n].double()
        assert abs(float(t.sum()) - g["sums"][i]) <= 1e-6 * max(1.0, abs(g["sums"][i])), n
        assert abs(float(t.square().sum()) - g["sq"][i]) <= 1e-6 * max(1.0, g["sq"][i]), n
        k = min(4, t.numel())
        np.testing.assert_array_equal(t.reshape(-1)[:k].numpy(), g["first"][i][:k])
