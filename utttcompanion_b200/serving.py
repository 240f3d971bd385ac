"""Multi-persona serving on one B200: persona arena + continuous batching.

The reference serves one turn at a time on one worker thread
(``server/app.py:163-166,215-217``) and ``stream_generate`` is batch-1
(``model/uttt_model.py:993-994``).  ``ServingEngine`` keeps the same turn
semantics per persona -- generate with the persona's frozen fast weights,
write [prompt + reply] with the chunk-first TTT schedule, gate by surprise,
pull elastically toward W_0, commit (``engine/personalizer.py:369-584``) --
but runs every in-flight turn of every persona in ONE packed decode launch
per token and batches the writes of all turns that finish together.

* ``PersonaArena``: device-resident FP32 masters + momentum and BF16 read
  copies for up to ``capacity`` personas (plus one padding slot), KV rings in
  the model engine indexed by the same slot, host spill of evicted personas
  in the reference's persona-file payload format (``FastWeightState.to_state_dict``).
* ``ServingEngine``: ``submit`` / ``step`` / ``run`` scheduler; a persona is
  never in two in-flight turns (later turns of the same user wait for the
  earlier write to commit, as the reference's serialisation guarantees).
* ``PersonaRouter``: ``gpu = stable_hash(user_id) mod world_size`` -- personas
  partition across the GPUs of a node with no data-path collective.
"""

from __future__ import annotations

import collections
import hashlib
import math
import queue
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Callable, Deque, Dict, Generator, List, Optional

import torch

from . import _lib
from .fastweight import _stream, workspace
from .model import EOS_ID, PAD_ID, DecodeGraph, DecodeTable, FastState, UtttB200, _host_list


class PersonaRouter:
    """Stable user-id -> GPU partition (no collective on the data path)."""

    def __init__(self, world_size: int):
        if world_size < 1:
            raise ValueError("world_size must be >= 1")
        self.world_size = world_size

    def rank_of(self, user_id: str) -> int:
        digest = hashlib.sha256(str(user_id).encode("utf-8")).digest()
        return int.from_bytes(digest[:8], "little") % self.world_size

    def partition(self, user_ids) -> Dict[int, List[str]]:
        out: Dict[int, List[str]] = {r: [] for r in range(self.world_size)}
        for uid in user_ids:
            out[self.rank_of(uid)].append(uid)
        return out


class ArenaFull(RuntimeError):
    """Every slot holds a persona with a turn in flight."""


class PersonaArena:
    """Device-resident persona store with LRU spill to host."""

    def __init__(self, engine: UtttB200, capacity: int):
        if capacity + 1 > engine.max_personas:
            raise ValueError("the model engine needs max_personas >= capacity + 1 (one padding slot)")
        self.engine = engine
        self.capacity = capacity
        self.pad_slot = capacity
        d, h = engine.cfg.d_model, engine.cfg.d_ff_fast
        dev = engine.device
        n = capacity + 1
        w0 = engine.w0
        self.w_up = w0[0].unsqueeze(0).repeat(n, 1, 1).contiguous()
        self.w_gate = w0[1].unsqueeze(0).repeat(n, 1, 1).contiguous()
        self.w_down = w0[2].unsqueeze(0).repeat(n, 1, 1).contiguous()
        self.s_up = torch.zeros_like(self.w_up)
        self.s_gate = torch.zeros_like(self.w_gate)
        self.s_down = torch.zeros_like(self.w_down)
        self.read_packed = torch.empty(n, d, 2 * h, dtype=torch.bfloat16, device=dev)
        self.read_down = torch.empty(n, h, d, dtype=torch.bfloat16, device=dev)
        self.meta: List[Optional[dict]] = [None] * n
        self.slot_of_user: "collections.OrderedDict[str, int]" = collections.OrderedDict()
        self.host: Dict[str, dict] = {}      # evicted personas: reference persona-file payloads
        self.pinned: set = set()             # slots with a turn in flight (never evicted)
        self.refresh(list(range(n)))

    def refresh(self, slots: List[int]) -> None:
        """Rebuild the BF16 read copies of `slots` (after a write commits)."""
        e = self.engine
        d, h = e.cfg.d_model, e.cfg.d_ff_fast
        for s in slots:
            _lib.check(e.lib.uttt_pack_read_copies(1, d, h, self.w_up[s].data_ptr(), self.w_gate[s].data_ptr(),
                                                   self.w_down[s].data_ptr(), self.read_packed[s].data_ptr(),
                                                   self.read_down[s].data_ptr(), _stream(e.device)),
                       "uttt_pack_read_copies")

    def _free_slot(self) -> int:
        used = set(self.slot_of_user.values())
        for s in range(self.capacity):
            if s not in used:
                return s
        for uid, s in self.slot_of_user.items():           # least recently used, not in flight
            if s not in self.pinned:
                self.host[uid] = self.export_slot(s)
                del self.slot_of_user[uid]
                return s
        raise ArenaFull("persona arena full: every slot has a turn in flight")

    def acquire(self, user_id: str) -> int:
        """Slot of `user_id`: resident hit, host promote, or a fresh W_0 persona."""
        if user_id in self.slot_of_user:
            self.slot_of_user.move_to_end(user_id)
            return self.slot_of_user[user_id]
        s = self._free_slot()
        payload = self.host.pop(user_id, None)
        if payload is None:
            for i, w in enumerate(self.engine.w0):
                (self.w_up, self.w_gate, self.w_down)[i][s].copy_(w)
            for t in (self.s_up, self.s_gate, self.s_down):
                t[s].zero_()
            self.meta[s] = {"step": 0, "last_surprise_loss": 0.0, "surprise_history": []}
        else:
            self.import_slot(s, payload)
        self.refresh([s])
        self.slot_of_user[user_id] = s
        return s

    def state(self, slots: List[int]) -> FastState:
        idx = _host_list(list(slots), torch.long, self.w_up.device)
        return FastState(self.w_up[idx], self.w_gate[idx], self.w_down[idx], self.s_up[idx], self.s_gate[idx],
                         self.s_down[idx], self.engine.ln_w, self.engine.ln_b)

    def export_slot(self, s: int) -> dict:
        m = self.meta[s] or {}
        return {"w_up": self.w_up[s:s + 1].cpu(), "w_gate": self.w_gate[s:s + 1].cpu(),
                "w_down": self.w_down[s:s + 1].cpu(), "s_up": self.s_up[s:s + 1].cpu(),
                "s_gate": self.s_gate[s:s + 1].cpu(), "s_down": self.s_down[s:s + 1].cpu(),
                "ln_weight": self.engine.ln_w.cpu(), "ln_bias": self.engine.ln_b.cpu(),
                "step": int(m.get("step", 0)), "last_surprise_loss": float(m.get("last_surprise_loss", 0.0)),
                "surprise_history": list(m.get("surprise_history", []))[-100:]}

    def import_slot(self, s: int, payload: dict) -> None:
        for name in ("w_up", "w_gate", "w_down", "s_up", "s_gate", "s_down"):
            t = torch.as_tensor(payload[name]).to(self.w_up.device, torch.float32)
            getattr(self, name)[s].copy_(t.reshape(getattr(self, name)[s].shape))
        self.meta[s] = {"step": int(payload.get("step", 0)),
                        "last_surprise_loss": float(payload.get("last_surprise_loss", 0.0)),
                        "surprise_history": list(payload.get("surprise_history", []))}

    def export_user(self, user_id: str) -> dict:
        if user_id in self.slot_of_user:
            return self.export_slot(self.slot_of_user[user_id])
        return self.host[user_id]

    def save_user(self, user_id: str, directory, base_signature: Optional[str] = None,
                  base_fingerprint: Optional[str] = None, drift_metrics: Optional[dict] = None):
        """Write ``user_id``'s persona (resident or spilled) as a reference persona file,
        ``{directory}/{user_id}_state.pt`` plus the ``{user_id}.pt`` alias
        (``DualTrackCheckpointManager._save_state_to_disk``, engine/checkpoint_manager.py:530-563)."""
        from . import persona_store
        payload = persona_store.make_payload(user_id, self.export_user(user_id), base_signature, base_fingerprint,
                                             drift_metrics)
        return persona_store.write_persona_file(directory, payload)

    def load_user(self, user_id: str, directory, base_fingerprint: Optional[str] = None) -> bool:
        """Stage ``user_id``'s persona file, if there is one, so the user's next turn resumes
        from it (validated first; engine/checkpoint_manager.py:335-373).  A resident persona
        is overwritten in place unless a turn of it is in flight."""
        from . import persona_store
        path = persona_store.find_persona_file(directory, user_id)
        if path is None:
            return False
        cfg = self.engine.cfg
        state, _ = persona_store.read_persona_file(path, user_id, cfg.d_model, cfg.d_ff_fast, base_fingerprint)
        if user_id in self.slot_of_user:
            s = self.slot_of_user[user_id]
            if s in self.pinned:
                raise ValueError(f"persona {user_id!r} has a turn in flight")
            self.import_slot(s, state)
            self.refresh([s])
        else:
            self.host[user_id] = state
        return True


@dataclass
class Turn:
    user_id: str
    prompt_ids: List[int]
    max_new_tokens: int = 128
    eos_token_id: Optional[int] = EOS_ID
    reply: List[int] = field(default_factory=list)
    slot: int = -1
    row: int = -1            # row of the packed decode batch while decoding
    admit_seq: int = 0       # the first decode step that includes the turn
    seen: int = 0            # reply tokens the host has taken from the device rows
    decoded: bool = False
    done: bool = False
    result: Optional[dict] = None
    # called with {"type": "token", "token_id": id} for every reply token as it is accepted, then
    # once with {"type": "ttt_status", "result": result} when the turn is done (on the thread that
    # finished it: the worker thread with async writes)
    on_event: Optional[Callable[[dict], None]] = None
    # the ids the turn's write runs on, from (prompt ids, reply ids); None: prompt + reply.  A text
    # front end passes the reference's re-tokenised "<|user|> ... <|assistant|> ..." turn
    # (engine/personalizer.py:480-489) here.
    write_ids: Optional[Callable[[List[int], List[int]], List[int]]] = None


class ServingEngine:
    """Continuous batching of persona turns on one GPU (greedy decoding)."""

    def __init__(self, engine: UtttB200, capacity: int, max_batch: int, surprise_threshold: float = 0.25,
                 elastic_anchor_lambda: float = 0.02, max_weight_drift_ratio: Optional[float] = 0.35,
                 online_ttt: bool = True, stop_free: bool = False, write_batch: int = 8,
                 write_wait_s: float = 0.05, async_writes: bool = False, prefill_budget: int = 16384):
        """``prefill_budget``: turns admitted in one step are prefilled together (one batched prefill, the
        prompts packed one after another) up to this many prompt tokens.
        ``stop_free``: replies run to their ``max_new_tokens`` (role ids and EOS are masked
        from the greedy pick, as the reference's graph-vs-eager test does), e.g. for
        forced-length load tests; otherwise stream_generate's stop rules apply.
        Finished turns are written together: once ``write_batch`` are waiting, the oldest has
        waited ``write_wait_s`` seconds, or nothing is left to decode (a one-persona write
        keeps only h/128 CTAs busy; a batch fills the GPU).  ``async_writes``: a worker
        thread runs the writes on their own CUDA stream while decoding goes on; a turn
        is done (and its user's next turn admitted) only after its write has landed.
        Off by default: both paths are HBM-bound, so overlapping them slows each, and
        on the 151M serve sweep at 32 req/s it raised the mean latency from 0.72 s to
        3.1 s (writes between steps form fewer, larger batches)."""
        self.engine = engine
        self._w0_norm2: Optional[List[float]] = None
        self.stop_free = stop_free
        self.prefill_budget = max(1, int(prefill_budget))   # prompt tokens prefilled together per step
        self.write_batch = max(1, write_batch)
        self.write_wait_s = write_wait_s
        self._write_queue: List[Turn] = []
        self._pending_writes: List[Turn] = []
        self._write_since = 0.0
        self._lock = threading.RLock()
        self._writes_in_flight = 0
        self._write_error: Optional[BaseException] = None
        self.async_writes = async_writes
        if async_writes:
            dev = engine.device
            self._dev_index = dev.index if dev.index is not None else torch.cuda.current_device()
            self._write_stream = torch.cuda.Stream(device=self._dev_index)
            self._jobs: "queue.Queue" = queue.Queue()
            self._worker = threading.Thread(target=self._write_worker, name="uttt-writes", daemon=True)
            self._worker.start()
        self.arena = PersonaArena(engine, capacity)
        self.max_batch = max_batch
        self.surprise_threshold = surprise_threshold
        self.elastic_anchor_lambda = elastic_anchor_lambda
        self.max_weight_drift_ratio = max_weight_drift_ratio
        self.online_ttt = online_ttt
        # The rows of the packed decode batch live on the device (DecodeTable): every captured step ends with
        # the stop rules and the rows' advance (uttt_engine_step), so consecutive steps need nothing from the
        # host.  One captured step per batch bucket (1, 2, 4, ... max_batch) over the table's first rows: a
        # step runs the smallest bucket that holds every row in use; idle and finished rows are padding rows
        # (padding slot, no fast-weight state) and read no weights.
        self.table = DecodeTable(engine.device, max_batch, self.arena.pad_slot, stop_free)
        sizes, b = [], 1
        while b < max_batch:
            sizes.append(b)
            b *= 2
        sizes.append(max_batch)
        self.graphs = {n: DecodeGraph(engine, n, self.arena.read_packed, self.arena.read_down, stop_free=stop_free,
                                      pad_slot=self.arena.pad_slot, table=self.table) for n in reversed(sizes)}
        self.graph = self.graphs[max_batch]
        self._seq = 0                  # decode steps launched
        self._snap_next = 0            # host buffer of the next snapshot
        self._snap_pending = None      # (buffer, bucket, step) of the last launched step, not yet read back
        self.stats = collections.Counter()      # seconds and tokens of prefill / decode / write
        self.waiting: Deque[Turn] = collections.deque()
        self.active: List[Optional[Turn]] = [None] * max_batch
        self.finished: List[Turn] = []
        self.in_flight_users: set = set()
        from .pool import SharedFastWeightPoolB200
        self.pool = SharedFastWeightPoolB200(*engine.w0, engine.ln_w, engine.ln_b, engine.cfg.momentum_beta,
                                             engine.cfg.max_inner_grad_norm, engine.cfg.normalize_loss_by_dim,
                                             engine.cfg.rms_norm_eps, engine.device)

    # ------------------------------------------------------------------ API
    def submit(self, user_id: str, prompt_ids: List[int], max_new_tokens: int = 128,
               eos_token_id: Optional[int] = EOS_ID, on_event: Optional[Callable[[dict], None]] = None,
               write_ids: Optional[Callable[[List[int], List[int]], List[int]]] = None) -> Turn:
        if not prompt_ids:
            raise ValueError("empty prompt")
        if type(max_new_tokens) is not int or max_new_tokens < 1:
            raise ValueError("max_new_tokens must be a positive integer")
        t = Turn(str(user_id), list(prompt_ids), max_new_tokens, eos_token_id, on_event=on_event,
                 write_ids=write_ids)
        self.waiting.append(t)
        return t

    def idle(self) -> bool:
        with self._lock:
            busy = self._writes_in_flight
        return (not self.waiting and not self._write_queue and not busy and all(a is None for a in self.active)
                and self._snap_pending is None)

    def close(self) -> None:
        """Stop the write worker (after the writes already queued)."""
        if self.async_writes and self._worker.is_alive():
            self._jobs.put(None)
            self._worker.join()

    def _write_worker(self) -> None:
        torch.cuda.set_device(self._dev_index)
        while True:
            job = self._jobs.get()
            if job is None:
                return
            turns, ready = job
            try:
                t0 = time.perf_counter()
                with torch.cuda.stream(self._write_stream):
                    self._write_stream.wait_event(ready)      # persona imports / resets queued before it
                    self._write(turns)
                self.stats["write_s"] += time.perf_counter() - t0
            except BaseException as exc:                    # surfaced by the next step() / run()
                import traceback
                traceback.print_exc()
                self._write_error = exc
            finally:
                with self._lock:
                    self._writes_in_flight -= 1

    def run(self, max_steps: int = 1_000_000) -> List[Turn]:
        steps = 0
        while not self.idle() and steps < max_steps:
            self.step()
            steps += 1
        self._raise_write_error()
        return self.finished

    def _raise_write_error(self) -> None:
        if self._write_error is not None:
            err, self._write_error = self._write_error, None
            raise err

    def interact_and_evolve(self, user_id: str, prompt_ids: List[int], max_new_tokens: int = 128) -> dict:
        """Synchronous one-turn API with the fields of ``EvolutionResult``
        (``engine/personalizer.py:44-66``) that do not involve text."""
        t = self.submit(user_id, prompt_ids, max_new_tokens)
        while not t.done:
            self.step()
        return t.result

    def stream_interact_and_evolve(self, user_id: str, prompt_ids: List[int],
                                   max_new_tokens: int = 128) -> Generator[Dict[str, Any], None, dict]:
        """Streaming one-turn API, the event sequence of
        ``uTTTPersonalizer.stream_interact_and_evolve`` (``engine/personalizer.py:369-583``):
        ``{"type": "token", ...}`` for each reply token as it is decoded, then, once the
        test-time update and the stability guard have run, ``{"type": "ttt_status",
        "result": ...}``; the generator returns the result.  Token events carry token ids
        (``token_id``); the reference's ``content`` strings come from its tokenizer.  This
        generator drives the engine itself, so other submitted turns advance with it."""
        events: Deque[dict] = collections.deque()
        t = self.submit(user_id, prompt_ids, max_new_tokens, on_event=events.append)
        while True:
            while events:
                ev = events.popleft()
                yield ev
                if ev["type"] == "ttt_status":
                    return t.result
            self.step()

    # ------------------------------------------------------------------ scheduler
    def _admit(self) -> None:
        """Start waiting turns in free rows: one batched prefill of every admitted prompt (up to
        ``prefill_budget`` prompt tokens per step, at least one turn), then each row starts on the device
        from its prompt's greedy pick (no host round trip; the stop rules apply to that first token there
        too)."""
        e = self.engine
        deferred: Deque[Turn] = collections.deque()
        admitted: List[Turn] = []
        tokens = 0
        while self.waiting and None in self.active:
            t = self.waiting.popleft()
            if admitted and tokens + len(t.prompt_ids) > self.prefill_budget:
                deferred.append(t)                          # the rest waits for the next step
                break
            row = self.active.index(None)
            with self._lock:
                if t.user_id in self.in_flight_users:      # its previous turn's write is still landing
                    deferred.append(t)
                    continue
                try:
                    t.slot = self.arena.acquire(t.user_id)
                except ArenaFull:                           # every slot in flight: retry on a later step
                    deferred.append(t)
                    break
                self.arena.pinned.add(t.slot)
                self.in_flight_users.add(t.user_id)
            t.row = row
            self.active[row] = t
            admitted.append(t)
            tokens += len(t.prompt_ids)
        self.waiting.extendleft(reversed(deferred))
        if not admitted:
            return
        t0 = time.perf_counter()
        logits = e.prefill_batch([torch.tensor(t.prompt_ids, dtype=torch.long) for t in admitted],
                                 [t.slot for t in admitted], self.arena.read_packed, self.arena.read_down,
                                 [t.slot for t in admitted])
        picks, _ = e.greedy(logits, stop_free=self.stop_free)
        for i, t in enumerate(admitted):
            self.table.admit(t.row, picks[i:i + 1], len(t.prompt_ids), t.slot, t.slot, t.max_new_tokens,
                             t.eos_token_id)
            t.admit_seq, t.seen = self._seq, 0
        self.stats["prefill_s"] += time.perf_counter() - t0
        self.stats["prefill_tokens"] += tokens
        self.stats["prefill_batches"] += 1

    def _harvest(self, buf: int, bucket: int, seq: int) -> None:
        """Take the results of decode step ``seq`` (snapshot ``buf``): the reply tokens each turn yielded
        since the last look, as token events, and the turns the device finished, which leave the batch
        and queue their writes.  Turns admitted after that step are not in it."""
        produced, status, ring = self.table.read(buf)
        for r in range(min(bucket, len(self.active))):
            t = self.active[r]
            if t is None or t.admit_seq > seq:
                continue
            n = int(produced[r])
            if n - t.seen > ring.shape[1]:
                raise RuntimeError("decode rows advanced past the host's token ring")
            for j in range(t.seen, n):
                tok = int(ring[r, j % ring.shape[1]])
                t.reply.append(tok)
                if t.on_event is not None:
                    t.on_event({"type": "token", "token_id": tok})
            self.stats["decode_tokens"] += n - t.seen
            t.seen = n
            if int(status[r]) == _lib.ROW_FINISHED:
                t.decoded = True
                self.active[r] = None
                self.finished.append(t)
                self._pending_writes.append(t)

    def step(self) -> None:
        """Admit waiting turns, launch one packed decode step, take the previous step's results back
        (the GPU runs this step meanwhile), and write finished turns."""
        self._raise_write_error()
        self._pending_writes = []
        self._admit()
        prev, self._snap_pending = self._snap_pending, None
        t0 = time.perf_counter()
        used = [r for r, t in enumerate(self.active) if t is not None]
        if used:
            bucket = min(n for n in self.graphs if n > max(used))
            self.graphs[bucket].step()
            buf, self._snap_next = self._snap_next, self._snap_next ^ 1
            self.table.snapshot(buf)
            self._snap_pending = (buf, bucket, self._seq)
            self._seq += 1
            self.stats["decode_steps"] += 1
        if prev is not None:
            self._harvest(*prev)
        self.stats["decode_s"] += time.perf_counter() - t0
        if self._pending_writes:
            if not self._write_queue:
                self._write_since = time.perf_counter()
            self._write_queue.extend(self._pending_writes)
        q = self._write_queue
        if q and (len(q) >= self.write_batch or all(a is None for a in self.active)
                  or time.perf_counter() - self._write_since >= self.write_wait_s):
            self._write_queue = []
            self.stats["write_batches"] += 1
            self.stats["write_tokens"] += sum(len(t.prompt_ids) + len(t.reply) for t in q)
            if self.async_writes:
                ready = torch.cuda.Event()
                ready.record(torch.cuda.current_stream(self.engine.device))
                with self._lock:
                    self._writes_in_flight += 1
                self._jobs.put((q, ready))
            else:
                t0 = time.perf_counter()
                self._write(q)
                self.stats["write_s"] += time.perf_counter() - t0
        elif self.async_writes and not used and self._writes_in_flight:
            time.sleep(0.0005)           # nothing to decode (waiting turns wait for their users' writes)

    def _write(self, turns: List[Turn]) -> None:
        """Step 2 + 3 of a turn for every finished turn at once (personalizer.py:480-551)."""
        cfg = self.engine.cfg
        slots = [t.slot for t in turns]
        if not self.online_ttt:
            for t in turns:
                self._finish(t, None, [], False)
            return
        seqs = [t.prompt_ids + t.reply if t.write_ids is None else list(t.write_ids(t.prompt_ids, t.reply))
                for t in turns]
        if any(not s for s in seqs):
            raise ValueError("a turn's write sequence is empty")
        align = min(cfg.chunk_size, 64)
        Tpad = max(((len(s) + align - 1) // align) * align for s in seqs)
        ids = torch.full((len(turns), Tpad), PAD_ID, dtype=torch.long)
        mask = torch.zeros(len(turns), Tpad)
        for r, s in enumerate(seqs):
            ids[r, :len(s)] = torch.tensor(s)
            mask[r, :len(s)] = 1.0
        state = self.arena.state(slots)
        # the elastic pull runs inside each row's last update (model/uttt_layer.py:773-801) and the
        # write returns the pulled state's ||W_m - W0_m||^2; a row whose turn is gated off is simply
        # not committed, so the pull can run for every row
        lam = max(float(self.elastic_anchor_lambda or 0.0), 0.0)
        guard = (self.pool.w_up_init, self.pool.w_gate_init, self.pool.w_down_init, lam)
        new, surprises, per_layer, sums = self.engine.test_time_update_batch(ids, state, mask, guard=guard)
        sums = sums.double().cpu()
        base = self._w0_sq()
        ratio = self.max_weight_drift_ratio
        outcomes = []
        for r, t in enumerate(turns):
            s = surprises[r]
            if not math.isfinite(s) or s < 0:
                raise ValueError("Test-time update returned a non-finite or negative surprise loss; "
                                 "persona was not changed")
            gate = s > self.surprise_threshold
            meta = self.arena.meta[t.slot]
            if gate:
                one = FastState(*(x[r:r + 1] for x in (new.w_up, new.w_gate, new.w_down, new.s_up, new.s_gate,
                                                      new.s_down)), new.ln_weight, new.ln_bias)
                sq = [float(sums[r, m]) for m in range(3)]
                scale = 1.0
                if ratio is not None and ratio > 0.0:    # the drift clamp (:803-818): a pass only when it bites
                    scale = min(ratio * math.sqrt(sum(base) + 1e-8) / math.sqrt(sum(sq) + 1e-8), 1.0)
                    if scale < 1.0:
                        one = self.pool.apply_elastic_pull(one, 0.0, ratio)
                a = self.arena
                for name, src in (("w_up", one.w_up), ("w_gate", one.w_gate), ("w_down", one.w_down),
                                  ("s_up", one.s_up), ("s_gate", one.s_gate), ("s_down", one.s_down)):
                    getattr(a, name)[t.slot].copy_(src[0])
                meta["step"] = int(meta.get("step", 0)) + new.step
                meta["last_surprise_loss"] = s
                meta["surprise_history"] = (meta.get("surprise_history", []) + per_layer[r])[-100:]
                meta["drift"] = self._drift_report([q * scale * scale for q in sq], base)
                a.refresh([t.slot])
            else:
                meta["last_surprise_loss"] = s
                meta["surprise_history"] = (meta.get("surprise_history", []) + [s])[-100:]
            outcomes.append((t, s, per_layer[r], gate))
        # every commit and read-copy refresh has landed before a turn is done: the user's next
        # turn (admitted as soon as this one is done) decodes with the written state
        if self.engine.device.type == "cuda":
            torch.cuda.current_stream(self.engine.device).synchronize()
        for t, s, pl, gate in outcomes:
            self._finish(t, s, pl, gate)

    def _w0_sq(self) -> List[float]:
        """||W0_m||^2 of the shared anchor, m = up, gate, down (computed once)."""
        if self._w0_norm2 is None:
            w0 = [w.unsqueeze(0).contiguous() for w in (self.pool.w_up_init, self.pool.w_gate_init,
                                                          self.pool.w_down_init)]
            d, h = w0[0].shape[1:]
            out = torch.zeros(8, dtype=torch.float32, device=self.engine.device)
            _lib.check(_lib.load().uttt_drift_sums(1, d, h, *(w.data_ptr() for w in w0),
                                                   *(w.data_ptr() for w in w0), out.data_ptr(),
                                                   _stream(self.engine.device)), "uttt_drift_sums")
            self._w0_norm2 = [float(x) for x in out[4:7].double().cpu()]
        return self._w0_norm2

    @staticmethod
    def _drift_report(sq: List[float], base: List[float]) -> Dict[str, float]:
        """compute_drift's report (model/uttt_layer.py:834-874) from the per-matrix sums of squares."""
        d_up, d_gate, d_down = (math.sqrt(max(q, 0.0)) for q in sq)
        b_up, b_gate, b_down = (math.sqrt(q) for q in base)
        total = math.sqrt(d_up ** 2 + d_gate ** 2 + d_down ** 2)
        bn = math.sqrt(b_up ** 2 + b_gate ** 2 + b_down ** 2) + 1e-8
        return {"drift_frobenius": total, "base_frobenius": bn, "drift_pct": total / bn * 100.0,
                "w_up_drift": d_up, "w_gate_drift": d_gate, "w_down_drift": d_down,
                "w_up_drift_pct": d_up / (b_up + 1e-8) * 100.0, "w_gate_drift_pct": d_gate / (b_gate + 1e-8) * 100.0,
                "w_down_drift_pct": d_down / (b_down + 1e-8) * 100.0}

    def _finish(self, t: Turn, surprise, per_layer, gate) -> None:
        meta = self.arena.meta[t.slot]
        drift = meta.get("drift")
        if drift is None:               # a persona this engine has not written: one drift pass
            drift = self.pool.compute_drift(self.arena.state([t.slot]))
            meta["drift"] = drift
        drift = dict(drift, step=int(meta.get("step", 0)), last_surprise_loss=meta.get("last_surprise_loss", 0.0))
        with self._lock:
            self._finish_locked(t, surprise, per_layer, gate, drift)
        if t.on_event is not None:
            t.on_event({"type": "ttt_status", "result": t.result})

    def _finish_locked(self, t: Turn, surprise, per_layer, gate, drift) -> None:
        t.result = {
            "user_id": t.user_id, "prompt_ids": t.prompt_ids, "reply_ids": list(t.reply),
            "surprise_loss": surprise, "surprise_threshold": self.surprise_threshold,
            "gate_triggered": bool(gate), "weight_drift_frobenius": drift["drift_frobenius"],
            "weight_drift_pct": drift["drift_pct"], "step": int(self.arena.meta[t.slot].get("step", 0)),
            "layer_surprise_losses": per_layer, "drift_details": drift,
        }
        t.done = True
        self.arena.pinned.discard(t.slot)
        self.in_flight_users.discard(t.user_id)
