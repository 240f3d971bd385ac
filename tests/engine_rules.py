"""The rows of a packed decode batch as the device holds them (``uttt_engine_step`` /
``uttt_engine_admit``), restated on the host: the CPU scheduler tests run the serving engine
on it, and the GPU test checks the kernels against it.

The rule is stream_generate's (model/uttt_model.py:1036-1050): a USER / ASSISTANT id (4, 5)
ends the reply without being yielded; any other id is yielded, and the reply ends at its
length limit or after the turn's EOS; stop-free rows ignore the stop ids.  A finished row
becomes a padding row (padding KV slot, no fast-weight state).
"""

import torch

RING, IDLE, RUNNING, FINISHED = 8, 0, 1, 2
USER_ID, ASSISTANT_ID = 4, 5


class HostTable:
    """Host restatement of ``model.DecodeTable`` with the same interface."""

    def __init__(self, device, rows, pad_slot, stop_free):
        self.rows, self.pad_slot, self.stop_free = rows, int(pad_slot), bool(stop_free)
        self.tokens, self.pos, self.produced = [0] * rows, [0] * rows, [0] * rows
        self.slots, self.state = [self.pad_slot] * rows, [-1] * rows
        self.max_new, self.eos, self.status = [1] * rows, [-1] * rows, [IDLE] * rows
        self.ring = [[0] * RING for _ in range(rows)]
        self._snap = [None, None]

    def _accept(self, b, tok):
        if not self.stop_free and tok in (USER_ID, ASSISTANT_ID):
            return False
        n = self.produced[b]
        self.ring[b][n % RING] = tok
        self.produced[b] = n + 1
        if n + 1 >= self.max_new[b]:
            return False
        return not (not self.stop_free and self.eos[b] >= 0 and tok == self.eos[b])

    def _retire(self, b):
        self.status[b], self.slots[b], self.state[b] = FINISHED, self.pad_slot, -1

    def admit(self, row, first_id, pos, slot, state, max_new, eos):
        tok = int(torch.as_tensor(first_id).reshape(-1)[0])
        self.produced[row], self.max_new[row] = 0, int(max_new)
        self.eos[row] = -1 if eos is None else int(eos)
        self.status[row] = RUNNING
        if self._accept(row, tok):
            self.tokens[row], self.pos[row], self.slots[row], self.state[row] = tok, int(pos), int(slot), int(state)
        else:
            self.tokens[row], self.pos[row] = 0, 0
            self._retire(row)

    def advance(self, ids, n):
        ids = [int(x) for x in torch.as_tensor(ids).reshape(-1).tolist()]
        for b in range(n):
            if self.status[b] != RUNNING:
                continue
            if self._accept(b, ids[b]):
                self.tokens[b] = ids[b]
                self.pos[b] += 1
            else:
                self._retire(b)

    def snapshot(self, k):
        self._snap[k] = (torch.tensor(self.produced, dtype=torch.int32), torch.tensor(self.status, dtype=torch.int32),
                         torch.tensor(self.ring, dtype=torch.int32))

    def read(self, k):
        return self._snap[k]
