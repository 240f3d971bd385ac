"""CPU: the hidden-dimension split of the readout (2 gloo ranks).

Each rank takes its slice of the hidden units (HiddenSplit.bounds / shard),
computes the slice's partial z with the oracle's BF16 arithmetic, the ranks
sum z through HiddenSplit.all_reduce, and the LayerNorm finish must equal
the oracle's unsplit readout (swiglu_fast_forward, model/uttt_layer.py:
211-247).  Also checks the slice bounds and their error cases."""

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from utttcompanion_b200.hsplit import HiddenSplit


def test_bounds_tile_the_hidden_units():
    spans = [HiddenSplit(rank=r, world=4).bounds(6912) for r in range(4)]
    assert spans == [(0, 1728), (1728, 3456), (3456, 5184), (5184, 6912)]
    with pytest.raises(ValueError):
        HiddenSplit(rank=0, world=4).bounds(6900)       # slices must be multiples of 8
    with pytest.raises(ValueError):
        HiddenSplit(rank=2, world=2)


def _rank_main(rank, world, port, out):
    from oracle.fastweight import _layer_norm, swiglu_fast_forward
    from oracle.numerics import Precision, round_bf16, silu
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(0)                       # the same inputs on every rank
    B, T, d, h = 3, 5, 64, 96
    x = round_bf16(rng.standard_normal((B, T, d)))
    W = [rng.normal(0, 0.1, (B, d, h)).astype(np.float32), rng.normal(0, 0.1, (B, d, h)).astype(np.float32),
         rng.normal(0, 0.1, (B, h, d)).astype(np.float32)]
    lnw = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    lnb = (0.1 * rng.standard_normal(d)).astype(np.float32)
    hs = HiddenSplit()
    wu, wg, wd = (t.numpy() for t in hs.shard(*(torch.from_numpy(w) for w in W)))
    prec = Precision("bf16")
    u = prec.mm(x, round_bf16(wu))
    g = prec.mm(x, round_bf16(wg))
    hh = prec.act(prec.act(silu(g)) * u)
    z = torch.from_numpy(np.einsum("btj,bjd->btd", hh.astype(np.float64), round_bf16(wd).astype(np.float64))
                         .astype(np.float32))
    hs.all_reduce(z)                                     # partial z of every slice -> full z
    ln = _layer_norm(round_bf16(z.numpy()), round_bf16(lnw), round_bf16(lnb), 1e-5, np.float32)
    ours = np.asarray(x, np.float32) + ln
    ref = swiglu_fast_forward(x, *W, lnw, lnb, 1e-5, prec, True)
    out.put((rank, float(np.max(np.abs(ours - ref))), float(np.max(np.abs(ref)))))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_split_readout_equals_unsplit_oracle():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = 29531
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    res = [out.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, diff, scale in res:
        assert diff <= 1e-2 + scale / 128, (rank, diff)


class _FakeIpcLib:
    """The library's IPC entry points on the host: areas are fake addresses, handles carry the
    owner's rank; ``fail_open_on`` makes uttt_ipc_open fail on that rank (a mapping refused)."""

    def __init__(self, rank, fail_open_on):
        import ctypes
        self.ctypes = ctypes
        self.rank, self.fail_open_on = rank, fail_open_on
        self.calls = []

    def uttt_split_exchange_bytes(self, world, rows, d):
        return 4096

    def uttt_ipc_alloc(self, nbytes, ptr, handle):
        self.ctypes.cast(ptr, self.ctypes.POINTER(self.ctypes.c_void_p))[0] = 0x1000 * (self.rank + 1)
        self.ctypes.memmove(handle, bytes([self.rank + 1]) * 64, 64)
        self.calls.append("alloc")
        return 0

    def uttt_ipc_open(self, handle, ptr):
        if self.rank == self.fail_open_on:
            return 3
        owner = self.ctypes.cast(handle, self.ctypes.POINTER(self.ctypes.c_ubyte))[0]
        self.ctypes.cast(ptr, self.ctypes.POINTER(self.ctypes.c_void_p))[0] = 0x100000 * owner
        self.calls.append("open")
        return 0

    def uttt_ipc_close(self, ptr):
        self.calls.append("close")
        return 0

    def uttt_ipc_free(self, ptr):
        self.calls.append("free")
        return 0


def _peer_rank_main(rank, world, port, fail_open_on, out):
    from utttcompanion_b200 import _lib
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    fake = _FakeIpcLib(rank, fail_open_on)
    _lib.load = lambda: fake                          # the host logic only: no GPU, no library calls
    hs = HiddenSplit()
    on = hs.enable_peer_exchange(max_rows=4, d=256, device="cpu")
    areas = list(hs._peer["areas_arr"]) if on else None
    if on:
        hs.close_peer_exchange = lambda: None         # nothing was mapped for real
    out.put((rank, on, areas, fake.calls))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("fail_open_on", [-1, 1], ids=["all_map", "rank1_refused"])
def test_peer_exchange_setup_is_all_or_nothing(fail_open_on):
    """Every rank maps every peer's area (its own at index rank) or, when any rank's mapping is
    refused, every rank keeps NCCL and releases what it had set up."""
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = 29600 + (fail_open_on + 1)
    procs = [ctx.Process(target=_peer_rank_main, args=(r, 2, port, fail_open_on, out)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(out.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    if fail_open_on < 0:
        for rank, on, areas, calls in res:
            assert on
            own = 0x1000 * (rank + 1)
            other = 0x100000 * (2 - rank)              # the other rank's handle byte is its rank + 1
            assert areas[rank] == own and areas[1 - rank] == other
            assert calls == ["alloc", "open"]
    else:
        for rank, on, areas, calls in res:
            assert not on
            assert calls[0] == "alloc" and calls[-1] == "free"
            if rank == 0:
                assert calls == ["alloc", "open", "close", "free"]
