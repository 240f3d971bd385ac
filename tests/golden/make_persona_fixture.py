"""Generate ``tests/golden/persona_ref/``: a persona file written by the reference's own code.

Run on a host where the reference checkout is importable::

    python tests/golden/make_persona_fixture.py --reference /path/to/uTTTCompanion

It builds a small seeded ``FastWeightState`` (d=8, h=16) with the reference's
``model.uttt_layer.FastWeightState``, serialises it with ``to_state_dict``, lays out
the payload fields that ``DualTrackCheckpointManager._save_state_to_disk`` writes
(engine/checkpoint_manager.py:546-556), and writes the file with the manager's own
atomic writer ``_write_payload_files`` (:502-528), so the canonical file and its
alias come from the reference.  The fixture is committed; the tests never need the
reference at run time.
"""

from __future__ import annotations

import argparse
import os
import sys
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "persona_ref")
D, H = 8, 16
USER = "alice"


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from engine.checkpoint_manager import DualTrackCheckpointManager
    from model.uttt_layer import FastWeightState

    g = torch.Generator().manual_seed(7)
    st = FastWeightState(
        w_up=torch.randn(1, D, H, generator=g), w_gate=torch.randn(1, D, H, generator=g),
        w_down=torch.randn(1, H, D, generator=g), s_up=torch.randn(1, D, H, generator=g) * 1e-3,
        s_gate=torch.randn(1, D, H, generator=g) * 1e-3, s_down=torch.randn(1, H, D, generator=g) * 1e-3,
        ln_weight=torch.ones(D), ln_bias=torch.zeros(D), step=12, last_surprise_loss=0.5,
        surprise_history=[0.9, 0.7, 0.5])
    payload = {
        "checkpoint_type": "uTTT_User_Persona_State",
        "version": "1.0.0",
        "user_id": USER,
        "base_signature": "fixture-signature",
        "base_fingerprint": "fixture-fingerprint",
        "timestamp": "2026-01-01T00:00:00Z",
        "fast_state": st.to_state_dict(),
        "drift_metrics": {},
        "metadata": {"user_id": USER},
    }
    os.makedirs(OUT, exist_ok=True)

    class _Writer:                       # the manager's writer needs only its disk lock
        _disk_lock = threading.Lock()

    primary = os.path.join(OUT, f"{USER}_state.pt")
    alias = os.path.join(OUT, f"{USER}.pt")
    from pathlib import Path
    DualTrackCheckpointManager._write_payload_files(_Writer(), Path(primary), Path(alias), payload)
    print("wrote", primary, alias)


if __name__ == "__main__":
    main()
