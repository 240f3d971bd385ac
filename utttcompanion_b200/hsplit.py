"""Hidden-dimension split of the fast weights over a process group.

The largest configuration (1.58B: d=2560, h=6912, 34 layers) reads 106 MB of
fast weights per persona, layer and token, so one token of one persona costs
3.6 GB of HBM traffic.  Splitting every persona's hidden units over P GPUs
(rank r owns units [r*h/P, (r+1)*h/P)) divides those bytes, and the decode
latency, by P.  The only exchange is the readout's partial
z = h_slice W_down_slice, a (rows, d) FP32 all-reduce per layer over NCCL;
the LayerNorm and the residual then run on every rank on identical sums.
Every hidden unit's u = x W_up[:, j], g = x W_gate[:, j] and h_j =
silu(g) u are computed whole on one rank, so the result equals the unsplit
readout (swiglu_packed_forward, model/uttt_layer.py:250-257) up to the
order of one FP32 sum.  Everything else of the decode step (slow weights,
attention, KV rings) is replicated.

With ``enable_peer_exchange`` the decode readout's sum needs no NCCL call: one
kernel (``uttt_split_exchange_finish``) stores each rank's partial rows into
its peers' memory over NVLink (CUDA IPC mappings, plain P2P stores), waits for
theirs and applies the LayerNorm, in place of the all-reduce and the finish
launch.  Larger readouts (prefill) and the write's partial sums keep NCCL.
"""

from __future__ import annotations

from typing import Optional, Tuple

import ctypes

import torch

from . import _lib
from .fastweight import _ptr, _stream, workspace


class HiddenSplit:
    """Rank ``rank`` of ``world`` holds hidden units ``bounds(h)`` of every persona."""

    def __init__(self, group=None, rank: Optional[int] = None, world: Optional[int] = None):
        import torch.distributed as dist
        self.group = group
        self.rank = dist.get_rank(group) if rank is None else rank
        self.world = dist.get_world_size(group) if world is None else world
        if not 0 <= self.rank < self.world:
            raise ValueError("rank outside the group")
        # a list: every all-reduce appends its (start, end) CUDA events on the current stream
        self.timing = None
        self._peer = None          # the NVLink exchange (enable_peer_exchange)

    # polls of one exchange flag before the wait gives up (~0.3 s at 64 ns per poll): a peer
    # that never arrives ends the exchange with UTTT_ERR_TIMEOUT instead of a hang
    MAX_POLLS = 1 << 22

    def enable_peer_exchange(self, max_rows: int, d: int, device) -> bool:
        """Set up the NVLink exchange for readouts of up to ``max_rows`` rows of width ``d``:
        every rank allocates its exchange area, the CUDA IPC handles go round the group and
        each rank maps its peers' areas.  A collective: every rank calls it.  Returns False
        (NCCL stays in use) when the group is larger than 8 or a mapping fails on any rank."""
        import torch.distributed as dist
        if self.world < 2 or self.world > 8 or self._peer is not None:
            return self._peer is not None
        import contextlib
        lib = _lib.load()
        dev = torch.device(device)
        with torch.cuda.device(dev) if dev.type == "cuda" else contextlib.nullcontext():
            nbytes = int(lib.uttt_split_exchange_bytes(self.world, max_rows, d))
            own = ctypes.c_void_p()
            handle = (ctypes.c_char * 64)()
            ok = nbytes > 0 and lib.uttt_ipc_alloc(nbytes, ctypes.byref(own), ctypes.byref(handle)) == 0
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle) if ok else None, group=self.group)
            areas, opened = [], []
            for r, h in enumerate(handles):
                if r == self.rank:
                    areas.append(own.value)
                    continue
                p = ctypes.c_void_p()
                hb = ctypes.create_string_buffer(h, 64) if h is not None else None
                if ok and hb is not None and lib.uttt_ipc_open(ctypes.byref(hb), ctypes.byref(p)) == 0:
                    areas.append(p.value)
                    opened.append(p.value)
                else:
                    ok = False
            flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.group)
            if int(flag.item()) != 1:
                for p in opened:
                    lib.uttt_ipc_close(ctypes.c_void_p(p))
                if own.value:
                    lib.uttt_ipc_free(own)
                return False
            arr = (ctypes.c_void_p * self.world)(*areas)
            self._peer = {"areas_arr": arr, "areas": ctypes.cast(arr, ctypes.c_void_p), "own": own.value,
                          "opened": opened,
                          "max_rows": int(max_rows), "d": int(d), "device": dev,
                          "ws": workspace(256, dev, slot=4) if dev.type == "cuda" else None}
        return True

    def check_peer_exchange(self) -> None:
        """Synchronise and raise RuntimeError if a wait of the NVLink exchange expired."""
        if self._peer is not None:
            from .fastweight import check_status
            check_status(self._peer["ws"], "uttt_split_exchange_finish")

    def close_peer_exchange(self) -> None:
        """Unmap the peers' areas and free this rank's.  Every rank calls it after its exchanges have
        completed and after every CUDA graph that captured an exchange has been released (a replay
        would store into the freed areas)."""
        if self._peer is None:
            return
        lib = _lib.load()
        torch.cuda.synchronize(self._peer["device"])
        for p in self._peer["opened"]:
            lib.uttt_ipc_close(ctypes.c_void_p(p))
        lib.uttt_ipc_free(ctypes.c_void_p(self._peer["own"]))
        self._peer = None

    def bounds(self, h: int) -> Tuple[int, int]:
        """[lo, hi) of this rank's hidden units (equal slices, each a multiple of 8)."""
        if h % (8 * self.world) != 0:
            raise ValueError(f"d_ff_fast={h} does not split into {self.world} slices of a multiple of 8")
        n = h // self.world
        return self.rank * n, (self.rank + 1) * n

    def shard(self, w_up: torch.Tensor, w_gate: torch.Tensor, w_down: torch.Tensor):
        """This rank's slices of full (S, d, h) / (S, h, d) masters (contiguous copies)."""
        lo, hi = self.bounds(w_up.shape[-1])
        return (w_up[..., lo:hi].contiguous(), w_gate[..., lo:hi].contiguous(),
                w_down[..., lo:hi, :].contiguous())

    def all_reduce(self, z: torch.Tensor) -> None:
        import torch.distributed as dist
        if self.world > 1:
            if self.timing is None:
                dist.all_reduce(z, op=dist.ReduceOp.SUM, group=self.group)
                return
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            dist.all_reduce(z, op=dist.ReduceOp.SUM, group=self.group)
            e1.record()
            self.timing.append((e0, e1))

    def readout(self, x: torch.Tensor, packed: torch.Tensor, down: torch.Tensor, state_index: torch.Tensor,
                ln_weight: torch.Tensor, ln_bias: torch.Tensor, eps: float) -> torch.Tensor:
        """x + LN(z) for (B, T, d) BF16 ``x`` over this rank's BF16 slices
        ``packed`` (S, d, 2h_local) / ``down`` (S, h_local, d): one partial readout,
        one all-reduce of z (B, T, d) FP32, one LayerNorm finish."""
        lib = _lib.load()
        B, T, d = x.shape
        h = down.shape[-2]
        if packed.shape[-1] != 2 * h or x.dtype != torch.bfloat16:
            raise ValueError("expected BF16 x and packed read-copy slices")
        x = x.contiguous()
        sidx = state_index.to(device=x.device, dtype=torch.int32).contiguous()
        out = torch.empty(B, T, d, dtype=torch.bfloat16, device=x.device)
        ws = workspace(256, x.device, slot=3)
        stream = _stream(x.device)
        z = torch.empty(B, T, d, dtype=torch.float32, device=x.device)
        _lib.check(lib.uttt_fast_readout_partial(B, T, d, h, x.data_ptr(), packed.data_ptr(), down.data_ptr(),
                                                 _ptr(sidx), z.data_ptr(), ws.data_ptr(), ws.numel(), stream),
                   "uttt_fast_readout_partial")
        pe = self._peer
        if pe is not None and B * T <= pe["max_rows"] and d == pe["d"]:
            # sum over the ranks through peer memory and finish, one kernel (z rounded as the decode
            # readout rounds it when T == 1)
            xw = pe["ws"]
            _lib.check(lib.uttt_split_exchange_finish(B * T, d, z.data_ptr(), x.data_ptr(), ln_weight.data_ptr(),
                                                      ln_bias.data_ptr(), float(eps), out.data_ptr(),
                                                      _lib.DTYPE_BF16, 1 if T == 1 else 0, self.rank, self.world,
                                                      pe["max_rows"], pe["areas"], self.MAX_POLLS, xw.data_ptr(),
                                                      xw.numel(), stream), "uttt_split_exchange_finish")
            return out
        self.all_reduce(z)
        # z rounded to BF16 before the LayerNorm exactly where the unsplit readout rounds it (decode)
        _lib.check(lib.uttt_readout_finish(B * T, d, z.data_ptr(), x.data_ptr(), ln_weight.data_ptr(),
                                           ln_bias.data_ptr(), float(eps), out.data_ptr(), _lib.DTYPE_BF16,
                                           1 if T == 1 else 0, stream),
                   "uttt_readout_finish")
        return out
