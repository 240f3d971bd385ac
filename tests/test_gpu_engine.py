"""GPU: the device-side scheduling kernels of the packed decode batch (uttt_engine_admit,
uttt_engine_step) against their host restatement (engine_rules.HostTable) on random picks
with stop ids mixed in, stop-free and with stop rules: every row field after every step must
agree exactly."""

import numpy as np
import pytest
import torch

from engine_rules import ASSISTANT_ID, USER_ID, HostTable
from utttcompanion_b200.model import DecodeTable

pytestmark = pytest.mark.gpu


def _fields(t):
    if isinstance(t, HostTable):
        return {k: np.array(getattr(t, k), np.int64) for k in
                ("tokens", "pos", "slots", "state", "produced", "max_new", "eos", "status", "ring")}
    return {k: getattr(t, k).cpu().numpy().astype(np.int64) for k in
            ("tokens", "pos", "slots", "state", "produced", "max_new", "eos", "status", "ring")}


@pytest.mark.parametrize("stop_free", [False, True])
def test_engine_step_matches_the_host_rule(stop_free):
    rows, pad = 12, 99
    dev = torch.device("cuda")
    dt = DecodeTable(dev, rows, pad, stop_free)
    ht = HostTable(dev, rows, pad, stop_free)
    rng = np.random.default_rng(7 + int(stop_free))
    vocab = [2, USER_ID, ASSISTANT_ID] + list(range(6, 40))
    admitted = 0
    for step in range(40):
        # admit a turn into a free (idle or finished) row now and then
        free = [r for r in range(rows) if ht.status[r] != 1]
        if free and rng.random() < 0.5:
            r = int(rng.choice(free))
            first = int(rng.choice(vocab))
            args = (r, int(rng.integers(1, 500)), int(rng.integers(0, 50)), int(rng.integers(0, 50)),
                    int(rng.integers(1, 12)), 2 if rng.random() < 0.7 else None)
            dt.admit(args[0], torch.tensor([first], dtype=torch.int32, device=dev), *args[1:])
            ht.admit(args[0], torch.tensor([first]), *args[1:])
            admitted += 1
        ids = [int(rng.choice(vocab)) for _ in range(rows)]
        n = int(rng.integers(1, rows + 1))
        dt.advance(torch.tensor(ids, dtype=torch.int32, device=dev), n)
        ht.advance(ids, n)
        got, want = _fields(dt), _fields(ht)
        for k in want:
            assert np.array_equal(got[k], want[k]), (step, k, got[k], want[k])
    assert admitted > 5 and (np.array(ht.status) == 2).any()


def test_snapshot_reads_back_the_rows():
    dev = torch.device("cuda")
    dt = DecodeTable(dev, 4, 9, False)
    dt.admit(2, torch.tensor([17], dtype=torch.int32, device=dev), 30, 1, 1, 5, 2)
    dt.advance(torch.tensor([0, 0, 18, 0], dtype=torch.int32, device=dev), 4)
    dt.snapshot(1)
    produced, status, ring = dt.read(1)
    assert int(produced[2]) == 2 and int(status[2]) == 1 and ring[2, :2].tolist() == [17, 18]
    assert int(dt.pos[2]) == 31 and int(dt.tokens[2]) == 18
