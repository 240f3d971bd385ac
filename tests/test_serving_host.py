"""Host logic of the continuous-batching scheduler (``serving.ServingEngine``) on CPU.

The GPU pieces are replaced by fakes: the model engine (prefill, greedy pick,
batched write), the captured decode step and the read-copy refresh.  The fake
decode emits token ``10 + pos % 50`` for every row, or a scripted stop id at a
scripted position; the device rows are restated on the host (``engine_rules.HostTable``, the
rule of ``uttt_engine_step`` that tests/test_gpu_engine.py checks on the GPU), so the test checks
the scheduler itself:
- admission and one turn in flight per user (``engine/personalizer.py``'s
  per-persona serialisation);
- the reference's stop rules (``model/uttt_model.py:1036-1050``): EOS is
  yielded and ends the reply, a role id ends it unyielded, ``max_new_tokens``
  caps it;
- LRU spill of the persona arena and the deferral of a turn that finds every
  slot pinned;
- batched writes (``write_batch``) and the result fields of each turn;
- the streaming event sequence of ``stream_interact_and_evolve``
  (``engine/personalizer.py:369-583``): token events, then ``ttt_status``.
"""

import torch

from engine_rules import HostTable
from utttcompanion_b200 import serving
from utttcompanion_b200.model import ASSISTANT_ID, EOS_ID, FastState
from utttcompanion_b200.workloads import ModelConfig

CFG = ModelConfig(vocab_size=64, d_model=8, n_layers=2, n_heads=2, n_kv_heads=1, d_ff_fast=16,
                  sliding_window_size=16, chunk_size=64, max_seq_len=512)


class FakeEngine:
    def __init__(self, max_personas, stops=None):
        d, h = CFG.d_model, CFG.d_ff_fast
        self.cfg = CFG
        self.device = torch.device("cpu")
        self.max_personas = max_personas
        self.w0 = (torch.full((d, h), 0.1), torch.full((d, h), 0.2), torch.full((h, d), 0.3))
        self.ln_w, self.ln_b = torch.ones(d), torch.zeros(d)
        self.lib = None
        self.stops = stops or {}          # position -> token emitted there
        self.prefills, self.writes = [], []

    def token_at(self, pos):
        return self.stops.get(int(pos), 10 + int(pos) % 50)

    def prefill(self, ids, slot, packed, down, kv_slot):
        self.prefills.append((int(slot), len(ids)))
        return torch.tensor([float(len(ids))])       # carries the prompt length to greedy()

    def prefill_batch(self, prompts, slots, packed, down, state_index):
        for p, s_ in zip(prompts, slots):
            self.prefills.append((int(s_), len(p)))
        return torch.tensor([[float(len(p))] for p in prompts])   # each row carries its prompt length

    def greedy(self, logits, stop_free=True):
        return torch.tensor([self.token_at(int(n)) for n in logits.reshape(-1).tolist()]), None

    def test_time_update_batch(self, ids, state, mask, guard=None):
        self.writes.append((ids.shape[0], [int(m.sum()) for m in mask]))
        new = FastState(state.w_up + 1.0, state.w_gate, state.w_down, state.s_up, state.s_gate, state.s_down,
                        state.ln_weight, state.ln_bias)
        new.step = 2 * CFG.n_layers
        out = (new, [1.0] * ids.shape[0], [[1.0] * CFG.n_layers for _ in range(ids.shape[0])])
        if guard is not None:           # the pulled state's drift sums: 0.25 per matrix
            out += (torch.full((ids.shape[0], 4), 0.25),)
        return out


class FakeGraph:
    """The captured step over the table's first ``batch`` rows: the fake decode's pick for each row,
    then the rows' advance (``engine_rules.HostTable``, the device rule restated)."""

    def __init__(self, engine, batch, read_packed, read_down, stop_free=True, pad_slot=None, table=None):
        self.engine, self.batch, self.table = engine, batch, table

    def step(self):
        ids = torch.tensor([self.engine.token_at(self.table.pos[b] + 1) for b in range(self.batch)],
                           dtype=torch.int32)
        self.table.advance(ids, self.batch)
        return ids, None


def _server(monkeypatch, capacity, max_batch, stops=None, stop_free=False, write_batch=8):
    monkeypatch.setattr(serving, "DecodeGraph", FakeGraph)
    monkeypatch.setattr(serving, "DecodeTable", HostTable)
    monkeypatch.setattr(serving.PersonaArena, "refresh", lambda self, slots: None)
    from utttcompanion_b200 import pool
    monkeypatch.setattr(pool.SharedFastWeightPoolB200, "apply_elastic_pull", lambda self, st, lam, ratio: st)
    monkeypatch.setattr(pool.SharedFastWeightPoolB200, "compute_drift",
                        lambda self, st: {"drift_frobenius": 0.5, "drift_pct": 1.0})
    monkeypatch.setattr(serving.ServingEngine, "_w0_sq", lambda self: [25.0, 25.0, 25.0])
    eng = FakeEngine(capacity + 1, stops)
    srv = serving.ServingEngine(eng, capacity=capacity, max_batch=max_batch, surprise_threshold=0.5,
                                stop_free=stop_free, write_batch=write_batch, write_wait_s=1e9)
    return eng, srv


def test_stop_rules_and_results(monkeypatch):
    # position 23 emits EOS (yielded, ends the reply); position 44 a role id (ends it unyielded)
    eng, srv = _server(monkeypatch, capacity=4, max_batch=4, stops={23: EOS_ID, 44: ASSISTANT_ID})
    a = srv.submit("a", [7] * 20, max_new_tokens=10)      # decodes pos 20.. -> EOS at 23
    b = srv.submit("b", [7] * 40, max_new_tokens=10)      # role id at 44
    c = srv.submit("c", [7] * 100, max_new_tokens=3)      # capped at 3 tokens
    srv.run()
    assert a.result["reply_ids"] == [30, 31, 32, EOS_ID]
    assert b.result["reply_ids"] == [50, 51, 52, 53]
    assert c.result["reply_ids"] == [10 + 100 % 50, 10 + 101 % 50, 10 + 102 % 50]
    for t in (a, b, c):
        r = t.result
        assert r["gate_triggered"] and r["surprise_loss"] == 1.0 and r["step"] == 2 * CFG.n_layers
        # the drift report of a committed turn comes from the write's pulled sums (0.25 per matrix
        # against ||W0_m||^2 = 25): 10 % of the anchor's norm, no drift pass
        assert abs(r["weight_drift_pct"] - 10.0) < 1e-6 and r["user_id"] == t.user_id
    # the write saw prompt + reply of each turn
    assert sorted(n for _, lens in eng.writes for n in lens) == sorted([20 + 4, 40 + 4, 100 + 3])


def test_one_turn_in_flight_per_user_and_ordering(monkeypatch):
    eng, srv = _server(monkeypatch, capacity=4, max_batch=4, stop_free=True)
    first = srv.submit("u", [7] * 10, max_new_tokens=5)
    second = srv.submit("u", [7] * 12, max_new_tokens=5)
    other = srv.submit("v", [7] * 8, max_new_tokens=5)
    srv.run()
    assert all(t.done for t in (first, second, other))
    # u's second turn was prefilled only after its first turn's write finished
    order = [n for _, n in eng.prefills]
    assert order.index(12) > order.index(10)
    assert second.result["step"] == 2 * (2 * CFG.n_layers)             # resumed from the written state
    assert srv.arena.export_user("u")["step"] == 4 * CFG.n_layers


def test_lru_spill_and_full_arena_deferral(monkeypatch):
    # 2 slots, 3 users: the least recently used persona spills to host and comes back
    eng, srv = _server(monkeypatch, capacity=2, max_batch=2, stop_free=True, write_batch=1)
    t1 = srv.submit("p", [7] * 5, max_new_tokens=2)
    t2 = srv.submit("q", [7] * 5, max_new_tokens=2)
    t3 = srv.submit("r", [7] * 5, max_new_tokens=2)       # waits: both slots hold turns in flight
    srv.step()
    assert t3 in srv.waiting and srv.arena.slot_of_user.keys() == {"p", "q"}
    srv.run()
    assert t3.done and "p" in srv.arena.host             # p was least recently used
    p_written = srv.arena.host["p"]["w_up"].clone()
    t4 = srv.submit("p", [7] * 6, max_new_tokens=2)       # p comes back from host with its written state
    srv.run()
    assert t4.result["step"] == 2 * (2 * CFG.n_layers)
    assert torch.equal(srv.arena.export_user("p")["w_up"], p_written + 1.0)


def test_writes_are_batched(monkeypatch):
    # three turns finish first and reach the batch size; the rest are flushed once nothing is decoding
    eng, srv = _server(monkeypatch, capacity=8, max_batch=8, stop_free=True, write_batch=3)
    turns = [srv.submit(f"w{i}", [7] * 10, max_new_tokens=n) for i, n in enumerate((2, 2, 2, 6, 7, 8))]
    srv.run()
    assert all(t.done for t in turns)
    assert [n for n, _ in eng.writes] == [3, 3]


def test_streaming_turn_events(monkeypatch):
    # the event sequence of stream_interact_and_evolve: one token event per reply token as it is
    # decoded (EOS included, as the reference yields it), then ttt_status with the result
    eng, srv = _server(monkeypatch, capacity=4, max_batch=4, stops={23: EOS_ID})
    other = srv.submit("b", [7] * 30, max_new_tokens=6)          # advances with the stream
    gen = srv.stream_interact_and_evolve("a", [7] * 20, max_new_tokens=10)
    events = []
    try:
        while True:
            events.append(next(gen))
    except StopIteration as stop:
        result = stop.value
    assert [e["type"] for e in events] == ["token"] * 4 + ["ttt_status"]
    assert [e["token_id"] for e in events[:4]] == [30, 31, 32, EOS_ID]
    assert events[-1]["result"] is result and result["reply_ids"] == [30, 31, 32, EOS_ID]
    assert result["gate_triggered"] and result["user_id"] == "a"
    srv.run()
    assert other.done and len(other.result["reply_ids"]) == 6
    # callbacks of submitted turns see the same sequence
    seen = []
    t = srv.submit("c", [7] * 5, max_new_tokens=3, on_event=seen.append)
    srv.run()
    assert [e["type"] for e in seen] == ["token"] * 3 + ["ttt_status"] and seen[-1]["result"] is t.result
    for bad in (0, 2.0, "3"):
        try:
            srv.submit("d", [7], max_new_tokens=bad)
        except ValueError:
            continue
        raise AssertionError(bad)
