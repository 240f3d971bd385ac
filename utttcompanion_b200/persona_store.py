"""Persona files in the reference's on-disk format (engine/checkpoint_manager.py).

A persona file is one ``torch.save`` payload (checkpoint_manager.py:546-556):
``checkpoint_type``, ``version``, ``user_id``, ``base_signature``,
``base_fingerprint``, ``timestamp``, ``fast_state`` (``FastWeightState.to_state_dict``:
FP32 CPU ``w_up, w_gate, s_up, s_gate (1, d, h)``, ``w_down, s_down (1, h, d)``,
``ln_weight, ln_bias (d,)``, ``step``, ``last_surprise_loss``, the last 100 entries of
``surprise_history``; model/uttt_layer.py:165-179), ``drift_metrics`` and ``metadata``.
It lives at ``personas/{user_id}_state.pt``, and ``personas/{user_id}.pt`` is a hard link
(or copy) alias (:232-240, :502-528).  Files are written atomically: a temporary file,
fsync, then ``os.replace``.  Reading accepts a bare state dict as well, checks the owner,
and validates shapes and finiteness before anything is published (:335-373, :671-687).
So personas move between the reference's store and ``PersonaArena`` unchanged.
"""

from __future__ import annotations

import math
import os
import re
import shutil
import time
from pathlib import Path
from typing import Any, Dict, Optional, Tuple

import torch

STATE_KEYS = ("w_up", "w_gate", "w_down", "s_up", "s_gate", "s_down", "ln_weight", "ln_bias")


def sanitize_id(raw_id: str) -> str:
    """User ids and tags: letters, digits, ``_``, ``-`` and ``.`` only (checkpoint_manager.py:39-44)."""
    cleaned = str(raw_id).strip()
    if not cleaned or cleaned in {".", ".."} or not re.fullmatch(r"[a-zA-Z0-9_.-]+", cleaned):
        raise ValueError("User IDs and snapshot tags must contain only letters, digits, _, -, or .")
    return cleaned


def persona_paths(directory, user_id: str) -> Tuple[Path, Path]:
    """(canonical ``{user_id}_state.pt``, alias ``{user_id}.pt``) under ``directory``."""
    uid = sanitize_id(user_id)
    d = Path(directory)
    return d / f"{uid}_state.pt", d / f"{uid}.pt"


def find_persona_file(directory, user_id: str) -> Optional[Path]:
    """The canonical file, else the alias (never for an id ending in ``_state``)."""
    primary, alias = persona_paths(directory, user_id)
    if primary.exists():
        return primary
    if not user_id.endswith("_state") and alias.exists():
        return alias
    return None


def validate_state(state: Dict[str, Any], d: int, h: int) -> None:
    """Raise ``ValueError`` unless ``state`` has the reference's shapes and finite values."""
    expected = {"w_up": (1, d, h), "w_gate": (1, d, h), "w_down": (1, h, d),
                "s_up": (1, d, h), "s_gate": (1, d, h), "s_down": (1, h, d),
                "ln_weight": (d,), "ln_bias": (d,)}
    for name, shape in expected.items():
        if name not in state:
            raise ValueError(f"persona state lacks {name}")
        t = torch.as_tensor(state[name])
        if tuple(t.shape) != shape:
            raise ValueError(f"persona state {name} has shape {tuple(t.shape)}, expected {shape}")
        if not bool(torch.isfinite(t).all()):
            raise ValueError(f"persona state {name} holds non-finite values")
    step = int(state.get("step", 0))
    last = float(state.get("last_surprise_loss", 0.0))
    hist = list(state.get("surprise_history", []))
    if step < 0 or not math.isfinite(last) or last < 0 or any(not math.isfinite(v) or v < 0 for v in hist):
        raise ValueError("persona state has an invalid step or surprise statistics")


def make_payload(user_id: str, state: Dict[str, Any], base_signature: Optional[str] = None,
                 base_fingerprint: Optional[str] = None, drift_metrics: Optional[dict] = None,
                 metadata: Optional[dict] = None) -> Dict[str, Any]:
    """The persona-file payload for ``state`` (a ``to_state_dict`` layout)."""
    uid = sanitize_id(user_id)
    fast = {name: torch.as_tensor(state[name]).detach().to("cpu", torch.float32).contiguous()
            for name in STATE_KEYS}
    fast["step"] = int(state.get("step", 0))
    fast["last_surprise_loss"] = float(state.get("last_surprise_loss", 0.0))
    fast["surprise_history"] = [float(v) for v in list(state.get("surprise_history", []))[-100:]]
    meta = {"user_id": uid}
    meta.update({k: v for k, v in (metadata or {}).items() if not str(k).startswith("_")})
    return {
        "checkpoint_type": "uTTT_User_Persona_State",
        "version": "1.0.0",
        "user_id": uid,
        "base_signature": base_signature,
        "base_fingerprint": base_fingerprint,
        "timestamp": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()),
        "fast_state": fast,
        "drift_metrics": dict(drift_metrics or {}),
        "metadata": meta,
    }


def write_persona_file(directory, payload: Dict[str, Any]) -> Path:
    """Atomically write ``payload`` to its canonical path and refresh the alias."""
    primary, alias = persona_paths(directory, payload["user_id"])
    primary.parent.mkdir(parents=True, exist_ok=True)
    tmp = Path(str(primary) + ".tmp")
    try:
        with open(tmp, "wb") as f:
            torch.save(payload, f)
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, primary)
    finally:
        tmp.unlink(missing_ok=True)
    if not payload["user_id"].endswith("_state"):   # `x_state.pt` is user x_state's own file
        try:
            if alias.exists() or alias.is_symlink():
                alias.unlink()
            os.link(primary, alias)
        except OSError:
            shutil.copy2(primary, alias)
    return primary


def read_persona_file(path, user_id: str, d: int, h: int,
                      base_fingerprint: Optional[str] = None) -> Tuple[Dict[str, Any], Dict[str, Any]]:
    """(state dict, metadata) of a persona file, validated before use.

    Raises ``ValueError`` for another user's file, a different base fingerprint (when both
    sides give one), wrong shapes or non-finite values."""
    payload = torch.load(Path(path), map_location="cpu", weights_only=False)
    uid = sanitize_id(user_id)
    if not isinstance(payload, dict):
        raise ValueError("persona file does not hold a payload dict")
    if payload.get("user_id", uid) != uid:
        raise ValueError("Persona file belongs to another user")
    saved = payload.get("base_fingerprint")
    if base_fingerprint is not None and saved is not None and saved != base_fingerprint:
        raise ValueError("persona file was written under a different base checkpoint")
    state = dict(payload.get("fast_state", payload))
    validate_state(state, d, h)
    out = {name: torch.as_tensor(state[name]).to(torch.float32) for name in STATE_KEYS}
    out["step"] = int(state.get("step", 0))
    out["last_surprise_loss"] = float(state.get("last_surprise_loss", 0.0))
    out["surprise_history"] = [float(v) for v in state.get("surprise_history", [])]
    return out, dict(payload.get("metadata", {}))
