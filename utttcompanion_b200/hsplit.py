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
"""

from __future__ import annotations

from typing import Optional, Tuple

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
        self.all_reduce(z)
        # z rounded to BF16 before the LayerNorm exactly where the unsplit readout rounds it (decode)
        _lib.check(lib.uttt_readout_finish(B * T, d, z.data_ptr(), x.data_ptr(), ln_weight.data_ptr(),
                                           ln_bias.data_ptr(), float(eps), out.data_ptr(), _lib.DTYPE_BF16,
                                           1 if T == 1 else 0, stream),
                   "uttt_readout_finish")
        return out
