"""GPU (2 ranks, NCCL): the hidden-dimension split of decode and write.

Each rank holds half of every persona's hidden units (FP32 masters and read
copies of its slices).  Prefill and packed decode steps sum the readout's z
across the ranks: the logits must match an unsplit engine on the same inputs
(both teacher-forced on the same tokens) within the logits bound, on both
ranks.  The batched chunk-TTT write (momentum + clipping, ragged masks) sums
every chunk's partial Z and the clip norms across the ranks: each rank's
updated slices must equal the same slices of the unsplit write (state rel-L2
<= 1e-3, update rel-L2 <= 1e-2) with the same per-layer surprise.  The decode
steps are run a second time with the NVLink peer exchange
(uttt_split_exchange_finish) in place of the NCCL all-reduce, within the same
bound.  Skipped with fewer than two visible GPUs."""

import datetime
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-2


def _cfg():
    from utttcompanion_b200.workloads import ModelConfig
    return ModelConfig(vocab_size=2048, d_model=256, n_layers=2, n_heads=2, n_kv_heads=1, d_ff_fast=384,
                       sliding_window_size=32, chunk_size=64, max_seq_len=512)     # head dim 128


def _run(eng, packed, down, prompts, forced):
    """Prefill every persona, then packed decode steps fed with ``forced`` tokens."""
    P = len(prompts)
    logits = [torch.stack([eng.prefill(prompts[p], p, packed, down, p) for p in range(P)])]
    pos = torch.tensor([len(t) for t in prompts], dtype=torch.int32, device=eng.device)
    slots = torch.arange(P, dtype=torch.int32, device=eng.device)
    for step in forced:
        logits.append(eng.decode_step(step.to(eng.device), pos, slots, packed, down, slots))
        pos = pos + 1
    return [lg.float().cpu() for lg in logits]


def _rank_main(rank, world, port, out_dir):
    from utttcompanion_b200.hsplit import HiddenSplit
    from utttcompanion_b200.model import FastState, UtttB200
    from utttcompanion_b200.workloads import perturbed_persona_states, reference_init_state_dict
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    cfg = _cfg()
    sd = reference_init_state_dict(cfg, seed=2)
    P = 2
    full = perturbed_persona_states(sd["fast_weight_pool.w_up_init"], sd["fast_weight_pool.w_gate_init"],
                                    sd["fast_weight_pool.w_down_init"], P, std=1e-2, seed=5, device="cpu")
    gen = torch.Generator().manual_seed(11)
    prompts = [torch.randint(6, cfg.vocab_size, (n,), generator=gen) for n in (40, 70)]
    forced = [torch.randint(6, cfg.vocab_size, (P,), generator=gen, dtype=torch.int32) for _ in range(6)]
    hs = HiddenSplit()
    eng = UtttB200(sd, cfg, device=dev, max_personas=P, hsplit=hs)
    local = [w.to(dev) for w in hs.shard(*full)]
    packed, down = eng.read_copies(*local)
    split = _run(eng, packed, down, prompts, forced)
    # prefill and decode again with the NVLink peer exchange summing the decode readouts in place of
    # the NCCL all-reduce (the prefill's readouts of more rows keep NCCL)
    peer_on = hs.enable_peer_exchange(max_rows=P, d=cfg.d_model, device=dev)
    peer = _run(eng, packed, down, prompts, forced)
    hs.check_peer_exchange()                 # no flag wait expired
    hs.close_peer_exchange()
    # batched write on prompt + forced tokens, ragged (right-padded) with masks
    turns = [prompts[p].tolist() + [int(f[p]) for f in forced] for p in range(P)]
    Tpad = ((max(len(t) for t in turns) + 63) // 64) * 64
    inter = torch.zeros(P, Tpad, dtype=torch.long)
    mask = torch.zeros(P, Tpad)
    for p, t in enumerate(turns):
        inter[p, :len(t)] = torch.tensor(t)
        mask[p, :len(t)] = 1.0
    st = FastState(*local, *(torch.zeros_like(w) for w in local), eng.ln_w.clone(), eng.ln_b.clone())
    new_split, _, pl_split = eng.test_time_update_batch(inter, st, mask)
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()
    ref_eng = UtttB200(sd, cfg, device=dev, max_personas=P)
    rp, rd = ref_eng.read_copies(*(w.to(dev) for w in full))
    ref = _run(ref_eng, rp, rd, prompts, forced)
    worst, worst_peer = 0.0, 0.0
    for a, c, b in zip(split, peer, ref):
        worst = max(worst, (torch.abs(a - b) - (LOGIT_TOL + torch.abs(b) / 128)).max().item())
        worst_peer = max(worst_peer, (torch.abs(c - b) - (LOGIT_TOL + torch.abs(b) / 128)).max().item())
    fullw = [w.to(dev) for w in full]
    st_ref = FastState(*fullw, *(torch.zeros_like(w) for w in fullw), ref_eng.ln_w.clone(), ref_eng.ln_b.clone())
    new_ref, _, pl_ref = ref_eng.test_time_update_batch(inter, st_ref, mask)
    ref_slices = hs.shard(new_ref.w_up, new_ref.w_gate, new_ref.w_down)
    base = hs.shard(*fullw)
    state_err, delta_err = 0.0, 0.0
    for got, want, w0 in zip((new_split.w_up, new_split.w_gate, new_split.w_down), ref_slices, base):
        state_err = max(state_err, float(torch.linalg.norm(got - want) / torch.linalg.norm(want)))
        delta_err = max(delta_err, float(torch.linalg.norm((got - w0) - (want - w0)) / torch.linalg.norm(want - w0)))
    surprise_err = float(np.max(np.abs(np.array(pl_split) - np.array(pl_ref)) / np.abs(np.array(pl_ref))))
    np.save(os.path.join(out_dir, f"rank{rank}.npy"),
            np.array([worst, state_err, delta_err, surprise_err, float(peer_on), worst_peer]))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_hidden_split_decode_and_write_match_unsplit(tmp_path):
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, 2, 29541, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    for r in range(2):
        worst, state_err, delta_err, surprise_err, peer_on, worst_peer = np.load(
            os.path.join(str(tmp_path), f"rank{r}.npy"))
        assert worst <= 0.0, (r, worst)
        assert peer_on == 1.0 and worst_peer <= 0.0, (r, peer_on, worst_peer)
        assert state_err <= 1e-3 and delta_err <= 1e-2, (r, state_err, delta_err)
        assert surprise_err <= 1e-3, (r, surprise_err)
