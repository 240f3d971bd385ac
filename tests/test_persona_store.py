"""Persona files in the reference's on-disk format (host logic, CPU).

``tests/golden/persona_ref/`` holds a persona written by the reference's own
``FastWeightState.to_state_dict`` and ``DualTrackCheckpointManager._write_payload_files``
(``tests/golden/make_persona_fixture.py``).
"""

import math
import os

import pytest
import torch

from utttcompanion_b200 import persona_store as ps

from conftest import GOLDEN

REF_DIR = os.path.join(GOLDEN, "persona_ref")
D, H = 8, 16


def _state(seed=0, d=D, h=H):
    g = torch.Generator().manual_seed(seed)
    return {"w_up": torch.randn(1, d, h, generator=g), "w_gate": torch.randn(1, d, h, generator=g),
            "w_down": torch.randn(1, h, d, generator=g), "s_up": torch.randn(1, d, h, generator=g),
            "s_gate": torch.randn(1, d, h, generator=g), "s_down": torch.randn(1, h, d, generator=g),
            "ln_weight": torch.ones(d), "ln_bias": torch.zeros(d), "step": 3, "last_surprise_loss": 0.25,
            "surprise_history": [0.5, 0.25]}


def test_reads_a_persona_file_written_by_the_reference():
    path = ps.find_persona_file(REF_DIR, "alice")
    assert path is not None and path.name == "alice_state.pt"
    state, meta = ps.read_persona_file(path, "alice", D, H, base_fingerprint="fixture-fingerprint")
    raw = torch.load(path, map_location="cpu", weights_only=False)
    for name in ps.STATE_KEYS:
        assert torch.equal(state[name], raw["fast_state"][name]), name
    assert state["step"] == 12 and state["last_surprise_loss"] == 0.5
    assert state["surprise_history"] == [0.9, 0.7, 0.5]
    assert meta["user_id"] == "alice"
    # the alias the reference links beside it reads the same
    alias, _ = ps.read_persona_file(os.path.join(REF_DIR, "alice.pt"), "alice", D, H)
    assert torch.equal(alias["w_down"], state["w_down"])


def test_written_payload_has_the_reference_layout_and_round_trips(tmp_path):
    ref = torch.load(os.path.join(REF_DIR, "alice_state.pt"), map_location="cpu", weights_only=False)
    st = _state(1)
    payload = ps.make_payload("bob", st, base_signature="sig", base_fingerprint="fp", metadata={"note": 1, "_x": 2})
    assert set(payload) == set(ref)
    assert set(payload["fast_state"]) == set(ref["fast_state"])
    for name in ps.STATE_KEYS:
        assert payload["fast_state"][name].dtype == ref["fast_state"][name].dtype == torch.float32
    assert "_x" not in payload["metadata"] and payload["metadata"]["note"] == 1
    primary = ps.write_persona_file(tmp_path, payload)
    assert primary == tmp_path / "bob_state.pt" and (tmp_path / "bob.pt").exists()
    assert not (tmp_path / "bob_state.pt.tmp").exists()
    back, _ = ps.read_persona_file(primary, "bob", D, H, base_fingerprint="fp")
    for name in ps.STATE_KEYS:
        assert torch.equal(back[name], st[name]), name
    assert back["step"] == 3 and back["surprise_history"] == [0.5, 0.25]
    # an id ending in _state writes no alias (it would be another user's canonical file)
    ps.write_persona_file(tmp_path, ps.make_payload("carol_state", st))
    assert (tmp_path / "carol_state_state.pt").exists() and not (tmp_path / "carol_state.pt").exists()


def test_invalid_files_are_rejected_before_use(tmp_path):
    st = _state(2)
    ps.write_persona_file(tmp_path, ps.make_payload("dave", st, base_fingerprint="fp"))
    path = tmp_path / "dave_state.pt"
    with pytest.raises(ValueError):
        ps.read_persona_file(path, "erin", D, H)                       # another user's file
    with pytest.raises(ValueError):
        ps.read_persona_file(path, "dave", D, H, base_fingerprint="other")
    with pytest.raises(ValueError):
        ps.read_persona_file(path, "dave", D + 1, H)                   # wrong shapes
    bad = dict(st)
    bad["w_gate"] = st["w_gate"].clone()
    bad["w_gate"][0, 0, 0] = math.nan
    ps.write_persona_file(tmp_path, ps.make_payload("frank", bad))
    with pytest.raises(ValueError):
        ps.read_persona_file(tmp_path / "frank_state.pt", "frank", D, H)
    neg = dict(st)
    neg["last_surprise_loss"] = -1.0
    ps.write_persona_file(tmp_path, ps.make_payload("gina", neg))
    with pytest.raises(ValueError):
        ps.read_persona_file(tmp_path / "gina_state.pt", "gina", D, H)
    for bad_id in ("", "..", "a/b", "x y"):
        with pytest.raises(ValueError):
            ps.sanitize_id(bad_id)
    assert ps.find_persona_file(tmp_path, "nobody") is None
