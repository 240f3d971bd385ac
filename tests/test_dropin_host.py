"""Host side of the drop-in layer (no GPU): the plug-in swap and its undo, the personalizer's
argument checks, and the EvolutionResult fields against the reference's dataclass."""

import dataclasses
import os
import sys
import types

import pytest

from conftest import ROOT
from utttcompanion_b200 import dropin, pool


def _fake_modules():
    ul = types.SimpleNamespace(**{name: (lambda *a, **k: "reference") for name in pool.DROP_INS})
    inf = types.SimpleNamespace(CUDAGraphDecoder=object)
    return ul, inf


def test_install_swaps_every_dropin_and_uninstall_restores_them():
    ul, inf = _fake_modules()
    before = {name: getattr(ul, name) for name in pool.DROP_INS}
    replaced = dropin.install(ul, inf)
    for name, fn in pool.DROP_INS.items():
        assert getattr(ul, name) is fn
        assert replaced["uttt_layer." + name] is before[name]
    assert inf.CUDAGraphDecoder is dropin.CUDAGraphDecoder
    dropin.uninstall(replaced, ul, inf)
    for name in pool.DROP_INS:
        assert getattr(ul, name) is before[name]
    assert inf.CUDAGraphDecoder is object


def test_graph_decoder_exposes_the_reference_protocol():
    for name in ("is_supported", "matches", "reset", "step", "export_kv_caches"):
        assert callable(getattr(dropin.CUDAGraphDecoder, name))


REF = os.path.join(ROOT, "baseline", "_ref")


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "engine")), reason="reference not installed")
def test_evolution_result_carries_every_reference_field():
    if REF not in sys.path:
        sys.path.insert(0, REF)
    from engine.personalizer import EvolutionResult as RefResult
    ours = {f.name for f in dataclasses.fields(dropin.EvolutionResult)}
    theirs = {f.name for f in dataclasses.fields(RefResult)}
    assert theirs <= ours


def test_personalizer_rejects_what_the_reference_rejects():
    serving = types.SimpleNamespace(surprise_threshold=0.25,
                                    engine=types.SimpleNamespace(cfg=types.SimpleNamespace(max_seq_len=4096)))
    p = dropin.uTTTPersonalizerB200(serving)
    with pytest.raises(ValueError):
        p._check(0, None, None, None)                 # max_new_tokens below 1
    with pytest.raises(ValueError):
        p._check(4096, None, None, None)              # no room left for the prompt
    with pytest.raises(ValueError):
        p._check(8, 0.7, None, None)                  # sampling: the path is greedy
    with pytest.raises(ValueError):
        p._check(8, 0.0, 1.5, None)
    with pytest.raises(ValueError):
        p._check(8, 0.0, 0.9, -1)
    assert p._check(None, 0.0, 0.9, 7) == 128
    with pytest.raises(ValueError):
        p._ids("text without a tokenizer", 8, None)
    with pytest.raises(ValueError):
        dropin.uTTTPersonalizerB200(serving, tokenizer=object())   # a tokenizer needs the chat encoder


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "model")), reason="reference not installed")
def test_every_dropin_keeps_the_reference_parameter_names():
    """The reference's callers pass the operator functions' arguments by keyword (e.g. chunk_step
    calls fused_chunk_ttt_step(q_chunk=..., ...)), so names and order must both match."""
    import inspect
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import model.uttt_layer as ul
    for name, fn in pool.DROP_INS.items():
        theirs = list(inspect.signature(getattr(ul, name)).parameters)
        ours = list(inspect.signature(fn).parameters)
        assert ours == theirs, (name, ours, theirs)
