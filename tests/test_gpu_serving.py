"""GPU: the continuous-batching serving engine gives each persona the same
turns as serving it alone (decode -> chunk-first write -> surprise gate ->
elastic pull), with several personas packed in one decode batch, a second
turn of a persona waiting for its first write, and LRU spill to host."""

import numpy as np
import pytest
import torch

from conftest import record
from oracle.numerics import rel_l2
from utttcompanion_b200.model import UtttB200
from utttcompanion_b200.pool import SharedFastWeightPoolB200
from utttcompanion_b200.serving import ServingEngine
from utttcompanion_b200.workloads import ModelConfig, reference_init_state_dict

pytestmark = pytest.mark.gpu


def _cfg():
    return ModelConfig(vocab_size=2048, d_model=256, n_layers=2, n_heads=4, n_kv_heads=2, d_ff_fast=384,
                       sliding_window_size=32, chunk_size=64, max_seq_len=512)


def _masked(logits):
    w = logits.astype(np.float64).copy()
    w[[0, 1, 3]] = -np.inf          # PAD / BOS / UNK, as the greedy pick masks them
    return w


def _sequential(sd, cfg, turns, served, max_new, lam, ratio, threshold):
    """Each persona served alone at batch 1, teacher-forced along the reply the serving engine
    produced for that turn: every reply token is checked against the batch-1 logits (equal
    argmax, or a near-tie within 2e-2), and the turn's write uses the same tokens, so the
    states stay comparable after any flip."""
    eng = UtttB200(sd, cfg, max_personas=1)
    pool = SharedFastWeightPoolB200(*eng.w0, eng.ln_w, eng.ln_b, cfg.momentum_beta, cfg.max_inner_grad_norm,
                                    cfg.normalize_loss_by_dim, cfg.rms_norm_eps)
    states, compared, flips = {}, 0, []
    for (uid, prompt), reply in zip(turns, served):
        st = states.get(uid) or eng.init_fast_state(1)
        tf = eng.teacher_forced_logits(torch.tensor(prompt), reply + [0], st)
        for i, tok in enumerate(reply):
            w = _masked(tf[i].cpu().numpy())
            best = int(np.argmax(w))
            compared += 1
            if best != tok:
                top = np.sort(w)[-2:]
                flips.append((uid, i))
                assert w[best] - w[tok] <= 2e-2 and top[1] - top[0] <= 2e-2, (uid, i, best, tok)
        if len(reply) < max_new and (not reply or reply[-1] != 2):
            # the reply ended on a role id (not yielded): the batch-1 pick there is a role id too
            w = _masked(tf[len(reply)].cpu().numpy())
            assert int(np.argmax(w)) in (4, 5) or np.sort(w)[-1] - max(w[4], w[5]) <= 2e-2, uid
        seq = prompt + reply
        Tp = ((len(seq) + 63) // 64) * 64
        inter = torch.tensor(seq + [0] * (Tp - len(seq)))
        mask = torch.tensor([1.0] * len(seq) + [0.0] * (Tp - len(seq)))
        new, s, _ = eng.test_time_update(inter, st, mask)
        states[uid] = pool.apply_elastic_pull(new, lam, ratio) if s > threshold else st
    return states, compared, flips


@pytest.mark.parametrize("async_writes", [False, True])
def test_serving_matches_sequential_turns_and_spills_lru(async_writes):
    cfg = _cfg()
    sd = reference_init_state_dict(cfg, seed=11)
    gen = torch.Generator().manual_seed(5)
    prompt = lambda n: torch.randint(6, cfg.vocab_size, (n,), generator=gen).tolist()  # noqa: E731
    turns = [("alice", prompt(20)), ("bob", prompt(45)), ("carol", prompt(70)), ("alice", prompt(33)),
             ("dave", prompt(12))]
    lam, ratio, thr, max_new = 0.02, 0.35, 0.0, 10
    eng = UtttB200(sd, cfg, max_personas=4)
    srv = ServingEngine(eng, capacity=3, max_batch=3, surprise_threshold=thr, elastic_anchor_lambda=lam,
                        max_weight_drift_ratio=ratio, async_writes=async_writes)
    handles = [srv.submit(u, p, max_new) for u, p in turns]
    srv.run()
    srv.close()
    torch.cuda.synchronize()
    assert all(h.result is not None for h in handles)
    served = [list(h.result["reply_ids"]) for h in handles]
    states, compared, flips = _sequential(sd, cfg, turns, served, max_new, lam, ratio, thr)
    assert compared == sum(len(r) for r in served) and compared >= len(turns)
    record(f"serving_async{int(async_writes)}", tokens_compared=compared, flips=flips)
    # dave's admission evicted the least recently used persona to host memory
    assert len(srv.arena.host) >= 1
    for uid, st in states.items():
        exported = srv.arena.export_user(uid)
        for n in ("w_up", "w_gate", "w_down"):
            got = torch.as_tensor(exported[n]).reshape(getattr(st, n).shape).numpy()
            assert rel_l2(got, getattr(st, n).cpu().numpy()) < 1e-3, (uid, n)
    alice = [h for h in handles if h.user_id == "alice"]
    assert alice[1].result["step"] > alice[0].result["step"] > 0


def test_arena_persona_files_round_trip_through_a_fresh_engine(tmp_path):
    """A persona written by one serving engine in the reference's file format is
    restored bit-exactly by another engine's arena and resumes there."""
    cfg = _cfg()
    sd = reference_init_state_dict(cfg, seed=11)
    gen = torch.Generator().manual_seed(9)
    eng = UtttB200(sd, cfg, max_personas=3)
    srv = ServingEngine(eng, capacity=2, max_batch=2, surprise_threshold=0.0)
    t = srv.submit("alice", torch.randint(6, cfg.vocab_size, (40,), generator=gen).tolist(), 8)
    srv.run()
    assert t.result["step"] > 0
    path = srv.arena.save_user("alice", tmp_path)
    assert path.name == "alice_state.pt" and (tmp_path / "alice.pt").exists()
    saved = srv.arena.export_user("alice")

    eng2 = UtttB200(sd, cfg, max_personas=3)
    srv2 = ServingEngine(eng2, capacity=2, max_batch=2, surprise_threshold=0.0)
    assert srv2.arena.load_user("alice", tmp_path)
    assert not srv2.arena.load_user("bob", tmp_path)
    srv2.arena.acquire("alice")
    got = srv2.arena.export_user("alice")
    for n in ("w_up", "w_gate", "w_down", "s_up", "s_gate", "s_down"):
        assert torch.equal(got[n], saved[n]), n
    assert got["step"] == saved["step"]
    t2 = srv2.submit("alice", torch.randint(6, cfg.vocab_size, (30,), generator=gen).tolist(), 8)
    srv2.run()
    assert t2.result["step"] > saved["step"]
