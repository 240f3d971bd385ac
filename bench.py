#!/usr/bin/env python
"""Benchmark of the uTTT serving hot path on B200 (one JSON line on rank 0).

Headline workload (the isolated chunk-TTT write): 64
independent FP32 fast-weight states per GPU, d=1024, h=2816; per state T=2048
tokens in 32 sequential chunks of C=64; keys/values BF16 ~N(0,1)
L2-normalised per token; MSE (normalize_by_dim) surprise loss; fixed inner lr
1e-2; no decay, momentum or clipping.  A step is one full pass: all 32 chunks
of all states.  Synthetic seeded data stands in for real conversations (the
reference publishes no dataset for this path).

Sub-objects of the same line: packed multi-persona decode + per-turn write of
BASELINE config 3 (N = 1) and config 4 (the 1.58B model; personas partitioned
by user id over the N GPUs), and at N > 1 the 1.58B decode with every
persona's hidden units split over all GPUs (NCCL).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun each rank runs its own 64 states (personas partition by user
id; no data-path collective) -> weak scaling; the timed region is bracketed
by a barrier + synchronize on every rank and the max over ranks is used.
"""

from __future__ import annotations

import argparse
import collections
import json
import math
import os
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "chunk-TTT update tok/s (packed multi-persona decode + chunk-TTT update path, BASELINE config 2)"
UNIT = "tok/s"

CFG = dict(states=64, d=1024, h=2816, tokens=2048, chunk=64, inner_lr=1e-2, momentum=0.0, clip=0.0,
           init_std=0.02, eps=1e-5)


# ----------------------------------------------------------------------------- helpers
def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            p = json.load(fh)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def traffic_record():
    path = os.path.join(ROOT, "profiles", "chunk_write_config2_traffic.json")
    if os.path.exists(path):
        with open(path) as fh:
            return json.load(fh)
    return None


class ClockSampler:
    """SM clock and clock-event (throttle) reasons of this rank's GPU while the timed region runs:
    read through NVML every 20 ms by a background thread (the device found by its PCI bus id), or,
    without NVML, from an nvidia-smi loop every 200 ms.  Read-only: no setting is changed."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits (nvml.h): reported name -> mask
    REASON_BITS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
                   ("sw_power_cap", 0x4))
    PERIOD_S = 0.02

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = None
        self.nv = None
        self.thread = None

    def _nvml_start(self) -> bool:
        try:
            import pynvml
            pynvml.nvmlInit()
            try:
                pr = torch.cuda.get_device_properties(self.idx)
                bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
                handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            except Exception:
                handle = pynvml.nvmlDeviceGetHandleByIndex(self.idx)
            reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            self.nv, self.handle, self.reasons_fn = pynvml, handle, reasons
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM))
            self.samples, self.bits = [], 0
            self.halt = threading.Event()
            self._sample()
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
            return True
        except Exception:
            self.nv = None
            return False

    def _sample(self):
        try:
            self.samples.append(float(self.nv.nvmlDeviceGetClockInfo(self.handle, self.nv.NVML_CLOCK_SM)))
            self.bits |= int(self.reasons_fn(self.handle))
        except Exception:
            pass

    def _run(self):
        while not self.halt.wait(self.PERIOD_S):
            self._sample()

    def start(self):
        if self._nvml_start():
            return
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.nv is not None:
            self.halt.set()
            self.thread.join(timeout=5)
            self._sample()
            try:
                self.nv.nvmlShutdown()
            except Exception:
                pass
            if not self.samples:
                return None
            return {"sm_mhz": float(np.median(self.samples)), "sm_max_mhz": self.max_mhz,
                    "reasons": sorted(nm for nm, bit in self.REASON_BITS if self.bits & bit),
                    "samples": len(self.samples), "source": f"NVML every {int(self.PERIOD_S * 1000)} ms"}
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as fh:
            for line in fh:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = float(parts[2])
                except ValueError:
                    continue
                for nm, val in zip(names, parts[5:9]):
                    if val.lower().startswith("active"):
                        reasons.add(nm)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi every 200 ms"}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ----------------------------------------------------------------------------- workload
def make_states(device, seed):
    from utttcompanion_b200 import fastweight as fw  # noqa: F401  (loads the library)
    g = torch.Generator(device=device).manual_seed(seed)
    B, d, h, T = CFG["states"], CFG["d"], CFG["h"], CFG["tokens"]

    def unit_rows(shape):
        x = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
        return (x / x.norm(dim=-1, keepdim=True)).to(torch.bfloat16)

    st = {
        "k": unit_rows((B, T, d)),
        "v": unit_rows((B, T, d)),
        "eta": torch.full((B, T), CFG["inner_lr"], device=device),
        "alpha": torch.zeros((B, T), device=device),
        "w_up": torch.randn((B, d, h), generator=g, device=device) * CFG["init_std"],
        "w_gate": torch.randn((B, d, h), generator=g, device=device) * CFG["init_std"],
        "w_down": torch.randn((B, h, d), generator=g, device=device) * CFG["init_std"],
        "ln_w": torch.ones(d, device=device),
        "ln_b": torch.zeros(d, device=device),
        "loss": torch.empty((B, T), device=device),
    }
    for n in ("up", "gate", "down"):
        st["s_" + n] = torch.zeros_like(st["w_" + n])
    return st


def run_step(st):
    from utttcompanion_b200 import fastweight as fw
    fw.chunk_write(st["k"], st["v"], st["eta"], st["alpha"], st["w_up"], st["w_gate"], st["w_down"],
                   st["s_up"], st["s_gate"], st["s_down"], st["ln_w"], st["ln_b"], None, CFG["momentum"],
                   CFG["clip"], True, CFG["eps"], chunk_size=CFG["chunk"], token_loss=st["loss"])


def launches_per_step():
    n_chunks = CFG["tokens"] // CFG["chunk"]
    return n_chunks * (3 + (1 if CFG["clip"] > 0 else 0))


def algorithmic_bytes(kind: int) -> float:
    """Minimal HBM bytes one launch of a chunk kernel must move (all states)."""
    B, d, h = CFG["states"], CFG["d"], CFG["h"]
    w = 3.0 * d * h * 4.0                       # FP32 W_up + W_gate + W_down of one state
    if kind == 3:   # bwd+update: read W (+S if momentum), write W (+S when momentum is kept or at the last chunk)
        n_chunks = CFG["tokens"] // CFG["chunk"]
        s_writes = 1.0 if CFG["momentum"] else 1.0 / n_chunks
        return B * w * (2.0 + s_writes + (1.0 if CFG["momentum"] else 0.0))
    if kind == 0:   # fwd: read W once
        return B * w
    return 0.0


# ----------------------------------------------------------------------------- the reference's own code
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def reference_modules():
    """The reference's ``model`` package from ``baseline/_ref`` (an offline install of the unmodified
    reference, which travels with the repository), or None when it is not installed."""
    if not os.path.isdir(os.path.join(REF_DIR, "model")):
        return None
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import model.uttt_layer as ul
    import model.uttt_model as um
    return ul, um


def use_all_host_threads() -> int:
    """Give torch and numpy's BLAS every host core this process may run on, whatever
    OMP_NUM_THREADS says (torchrun sets it to 1); returns the thread count."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(limits=n)
    except Exception:
        pass
    torch.set_num_threads(n)
    return n


def chunk_stepper(seed):
    """One step = one 64-token chunk of one config-2 state on the host cores: the reference's own
    ``fused_chunk_ttt_step`` (PyTorch FP32) from baseline/_ref, else the oracle port (numpy FP32).
    Returns (step, kind, description)."""
    d, h, C = CFG["d"], CFG["h"], CFG["chunk"]
    mods = reference_modules()
    if mods is not None:
        ul, _ = mods
        g = torch.Generator().manual_seed(seed)
        W = [torch.randn(s, generator=g) * CFG["init_std"] for s in ((1, d, h), (1, d, h), (1, h, d))]
        S = [torch.zeros_like(w) for w in W]
        lnw, lnb = torch.ones(d), torch.zeros(d)

        def unit():
            x = torch.randn(1, C, d, generator=g)
            return x / x.norm(dim=-1, keepdim=True)

        def step():
            k, v = unit(), unit()
            eta = torch.full((1, C, 1), CFG["inner_lr"])
            with torch.no_grad():
                r = ul.fused_chunk_ttt_step(k, k, v, eta, torch.zeros_like(eta), *W, *S, lnw, lnb, None,
                                            CFG["momentum"], CFG["clip"], True, CFG["eps"])
            W[:], S[:] = list(r[1:4]), list(r[4:7])
        return step, "reference", "the reference's own fused_chunk_ttt_step (PyTorch FP32, baseline/_ref)"
    from oracle import fastweight as ofw
    from oracle.numerics import Precision
    rng = np.random.default_rng(seed)
    Wn = [rng.normal(0, CFG["init_std"], s).astype(np.float32) for s in ((1, d, h), (1, d, h), (1, h, d))]
    Sn = [np.zeros_like(w) for w in Wn]
    lnwn, lnbn = np.ones(d, np.float32), np.zeros(d, np.float32)
    prec = Precision("f32")

    def step_port():
        k = rng.standard_normal((1, C, d)).astype(np.float32)
        k /= np.linalg.norm(k, axis=-1, keepdims=True)
        v = rng.standard_normal((1, C, d)).astype(np.float32)
        v /= np.linalg.norm(v, axis=-1, keepdims=True)
        eta = np.full((1, C, 1), CFG["inner_lr"], np.float32)
        r = ofw.fused_chunk_ttt_step(k, k, v, eta, np.zeros_like(eta), *Wn, *Sn, lnwn, lnbn, None, CFG["momentum"],
                                     CFG["clip"], True, CFG["eps"], prec=prec)
        Wn[:], Sn[:] = [r.w_up, r.w_gate, r.w_down], [r.s_up, r.s_gate, r.s_down]
    return step_port, "port", "numpy FP32 restatement of fused_chunk_ttt_step (oracle port)"


def cpu_baseline(max_seconds=20.0):
    """The reference's chunk step on the host cores (all threads) on a bounded sample: chunk steps
    of single config-2 states until ~max_seconds.  Returns (tok/s, steps, seconds, kind, desc, cores)."""
    cores = use_all_host_threads()
    step, kind, desc = chunk_stepper(0)
    step()                                   # first call: allocations, thread pools
    n, t0 = 0, time.perf_counter()
    while True:
        step()
        n += 1
        el = time.perf_counter() - t0
        if el > max_seconds or n >= 400:
            break
    return n * CFG["chunk"] / el, n, el, kind, desc, cores


def reference_model(um, cfg, device, dtype, seed=0):
    """The reference's own ``uTTTModel`` of ``cfg``'s architecture holding the same random weights
    as ``workloads.random_state_dict(cfg, seed)`` (built on the meta device and filled, so the 1.58B
    model takes seconds); FP32, or ``dtype`` weights with the FP32 fast-weight pool as served."""
    from utttcompanion_b200 import workloads as wl
    fields = set(um.uTTTConfig.__dataclass_fields__)
    rcfg = um.uTTTConfig(**{k: v for k, v in cfg.to_dict().items() if k in fields})
    with torch.device("meta"):
        m = um.uTTTModel(rcfg)
    m = m.to_empty(device=device)
    sd = wl.random_state_dict(cfg, seed=seed, device=device)
    with torch.no_grad():
        for name, p in m.named_parameters():
            src = sd.get(name)
            if src is None:                   # parameters the serving path never reads
                p.zero_()
            else:
                p.copy_(src.to(p.dtype))
        for mod in m.modules():               # RoPE tables: rebuilt in FP32 as the module builds them
            if hasattr(mod, "_build_cache") and "cos_cached" in mod._buffers:
                mod._buffers.pop("cos_cached")
                mod._buffers.pop("sin_cached")
                mod._build_cache(rcfg.max_seq_len)
    del sd
    m = m.eval().requires_grad_(False)
    if dtype != torch.float32:
        pool = {n: p.detach().clone() for n, p in m.fast_weight_pool.named_parameters()}
        m = m.to(dtype)
        for n, p in m.fast_weight_pool.named_parameters():
            p.data = pool[n]
    return m


def _stop_free_greedy(logits, **kwargs):
    scores = logits.float().clone()
    scores[:, :6] = -torch.inf
    limit = kwargs.get("active_vocab_limit")
    if limit is not None:
        scores[:, limit:] = -torch.inf
    return scores.argmax(dim=-1)


def reference_turns(um, cfg, device, dtype, personas, prompt_len, new_tokens, repeats, graph=False, seed=0):
    """Personas served one after another at batch 1 through the reference's own
    ``stream_generate`` (greedy, forced length) and ``test_time_update`` (prompt + reply, padded to
    64 with a mask), as its server does.  Decode tok/s counts the tokens after the first (the
    prefill is timed apart); with ``graph`` the persona's second turn is timed, so the reference's
    CUDA-graph capture is outside it.  Returns medians over ``repeats`` of per-persona figures."""
    from unittest.mock import patch
    m = reference_model(um, cfg, device, dtype, seed)
    cuda = device.type == "cuda"
    ctx = (lambda: torch.autocast("cuda", dtype=dtype)) if (cuda and dtype != torch.float32) else \
        (lambda: torch.autocast(device.type, enabled=False))
    g = torch.Generator().manual_seed(seed + 1)

    def sync():
        if cuda:
            torch.cuda.synchronize(device)

    dec, pre, wr = [], [], []
    for rep in range(repeats + 1):
        for _ in range(personas):
            st = m.init_fast_state(batch_size=1, dtype=torch.float32, detach=True)
            ids = torch.randint(6, cfg.vocab_size, (1, prompt_len), generator=g).to(device)
            for turn in range(2 if graph else 1):
                toks, stamps = [], []
                sync()
                t0 = time.perf_counter()
                with torch.no_grad(), ctx(), patch.object(m, "_sample_next_token", side_effect=_stop_free_greedy):
                    for t in m.stream_generate(ids, fast_state=st, max_new_tokens=new_tokens, temperature=0.0,
                                               eos_token_id=None, speculative_draft_k=0, use_cuda_graph=graph):
                        toks.append(t)
                        stamps.append(time.perf_counter())
            T = prompt_len + len(toks)
            Tp = ((T + 63) // 64) * 64
            inter = torch.tensor([ids[0].tolist() + toks + [0] * (Tp - T)], device=device)
            mask = torch.tensor([[1.0] * T + [0.0] * (Tp - T)], device=device)
            sync()
            t2 = time.perf_counter()
            with torch.no_grad(), ctx():
                m.test_time_update(inter, st, mask)
            sync()
            t3 = time.perf_counter()
            if rep == 0:
                continue                      # warm-up round
            pre.append(stamps[0] - t0)
            dec.append((len(toks) - 1) / (stamps[-1] - stamps[0]))
            wr.append(T / (t3 - t2))
    m._cuda_graph_decoder = None
    del m
    if cuda:
        torch.cuda.empty_cache()
    return {"decode_tok_s_per_persona": float(np.median(dec)), "prefill_s": float(np.median(pre)),
            "write_tok_s": float(np.median(wr)), "personas": personas, "prompt_tokens": prompt_len,
            "decode_tokens": new_tokens, "repeats": repeats}


def reference_model_baselines(device, spec, cfg):
    """The reference's own serving path beside a decode sub-object: on the host cores (FP32, all
    threads; a bounded sample) and on this B200 (BF16 autocast, batch 1, eager and with its
    CUDAGraphDecoder).  None when baseline/_ref is absent."""
    mods = reference_modules()
    if mods is None:
        return None
    _, um = mods
    out = {"source": "the reference's own uTTTModel.stream_generate + test_time_update from baseline/_ref, "
                     "the same random weights as this sub-object's model"}
    cores = use_all_host_threads()
    cpu = torch.device("cpu")
    if spec["config"] == "151M":
        c = reference_turns(um, cfg, cpu, torch.float32, personas=2, prompt_len=128, new_tokens=16, repeats=3)
        sample = "2 personas x (128-token prompt, 16 greedy tokens, one write of the turn), median of 3"
    else:
        c = reference_turns(um, cfg, cpu, torch.float32, personas=1, prompt_len=48, new_tokens=16, repeats=1)
        sample = "1 persona x (48-token prompt, 16 greedy tokens, one write of the 64-token turn), once"
    out["cpu"] = {**c, "cores": cores, "kind": "reference", "dtype": "f32", "sample": sample}
    g_eager = reference_turns(um, cfg, device, torch.bfloat16, personas=1, prompt_len=512, new_tokens=64, repeats=1)
    g_graph = reference_turns(um, cfg, device, torch.bfloat16, personas=1, prompt_len=512, new_tokens=64, repeats=1,
                              graph=True)
    out["gpu"] = {"eager": g_eager, "cuda_graph": {k: g_graph[k] for k in ("decode_tok_s_per_persona", "prefill_s")},
                  "dtype": "bf16 autocast, FP32 fast-weight masters", "batch": 1,
                  "sample": "1 persona: 512-token prompt, 64 greedy tokens (the reference's own published "
                            "measurement shape), one write of the 576-token turn; eager and CUDA graph"}
    return out


def torch_reference_chunk_gpu(device, st, chunks=4):
    """The reference's own fused_chunk_ttt_step (baseline/_ref) under BF16 autocast on this B200,
    on the headline's 64 states: ``chunks`` sequential chunks after one warm-up chunk.  None when the
    reference is not installed."""
    mods = reference_modules()
    if mods is None:
        return None
    ul, _ = mods
    C = CFG["chunk"]
    W = [st["w_up"].clone(), st["w_gate"].clone(), st["w_down"].clone()]
    S = [torch.zeros_like(w) for w in W]
    B = W[0].shape[0]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def chunk(i):
        k = st["k"][:, i * C:(i + 1) * C]
        v = st["v"][:, i * C:(i + 1) * C]
        eta = st["eta"][:, i * C:(i + 1) * C, None]
        alpha = st["alpha"][:, i * C:(i + 1) * C, None]
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            r = ul.fused_chunk_ttt_step(k, k, v, eta, alpha, *W, *S, st["ln_w"], st["ln_b"], None, CFG["momentum"],
                                        CFG["clip"], True, CFG["eps"])
        W[:], S[:] = list(r[1:4]), list(r[4:7])

    chunk(0)
    torch.cuda.synchronize()
    e0.record()
    for i in range(1, chunks + 1):
        chunk(i)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / chunks
    del W, S
    torch.cuda.empty_cache()
    return {"value": B * C / (ms / 1e3), "unit": UNIT, "ms_per_chunk": ms, "chunks_timed": chunks,
            "sample": f"{chunks} sequential chunks of the headline's {B} states (d={CFG['d']}, h={CFG['h']})",
            "source": "the reference's own fused_chunk_ttt_step from baseline/_ref, BF16 autocast, FP32 masters",
            "dtype": "bf16 autocast"}


def host_threads():
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


# ----------------------------------------------------------------------------- decode + write (configs 3, 4)
def _uniform_prompts(lo, hi):
    def draw(g, n):
        return torch.randint(lo, hi + 1, (n,), generator=g).tolist()
    return draw


def _lognormal_prompts(median, sigma, lo, hi):
    def draw(g, n):
        z = torch.randn(n, generator=g, dtype=torch.float64)
        return [int(min(max(round(median * math.exp(sigma * float(x))), lo), hi)) for x in z]
    return draw


DEC = dict(
    key="decode", label="BASELINE config 3", config="151M", personas=32, prompts=_uniform_prompts(64, 1024),
    prompt_desc="uniform in [64, 1024]", prompt_max=1024, new_tokens=128, warmup_tokens=3, perturb_std=1e-3,
    init="reference")
DEC4 = dict(
    key="decode_1p58b", label="BASELINE config 4", config="1P58B", personas=64, batch1=True,
    prompts=_lognormal_prompts(512, 1.0, 32, 4096), prompt_desc="lognormal, median 512, sigma 1.0 (BASELINE gives "
    "no sigma), clipped to [32, 4096]", prompt_max=4096, new_tokens=256, warmup_tokens=3, perturb_std=1e-3,
    init="random")


def decode_workload(device, rank, lib, spec, baselines=False):
    """Packed multi-persona greedy decode + per-turn chunk-TTT write.  ``spec``'s
    personas start from W_p = W_0 + N(0, perturb_std) with ragged prompts of
    uniform-random ids; they decode ``new_tokens`` greedy tokens as ONE packed
    batch per step (captured CUDA graph), then write prompt + reply with one
    batched chunk-TTT write (right-padded to a multiple of 64, masks; rows leave
    the batch when only padding is left)."""
    from utttcompanion_b200 import _lib
    from utttcompanion_b200 import workloads as wl
    from utttcompanion_b200.model import DecodeGraph, FastState, UtttB200
    cfg = {"151M": wl.CONFIG_151M, "1P58B": wl.CONFIG_1P58B}[spec["config"]]
    P = spec["personas"]
    if spec["init"] == "reference":
        sd = wl.reference_init_state_dict(cfg, seed=0)
        init_desc = "reference seed-0 init"
    else:
        sd = wl.random_state_dict(cfg, seed=0, device=device)
        init_desc = "random init with the reference's distributions (generated on the GPU)"
    eng = UtttB200(sd, cfg, device=device, max_personas=P, max_positions=spec["prompt_max"] + spec["new_tokens"] + 64)
    w0 = (sd["fast_weight_pool.w_up_init"], sd["fast_weight_pool.w_gate_init"], sd["fast_weight_pool.w_down_init"])
    del sd
    w_up, w_gate, w_down = wl.perturbed_persona_states(*w0, P, spec["perturb_std"], seed=100 + rank, device=device)
    del w0
    packed, down = eng.read_copies(w_up, w_gate, w_down)
    graph = DecodeGraph(eng, P, packed, down)          # before prefill: its warm-up touches ring slot 0
    g = torch.Generator().manual_seed(7 + rank)
    lens = spec["prompts"](g, P)
    prompts = [torch.randint(6, cfg.vocab_size, (n,), generator=g) for n in lens]
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    first = torch.stack([eng.prefill(prompts[p], p, packed, down, p) for p in range(P)])
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    ids, _ = eng.greedy(first)
    tokens = ids.clone()
    pos = torch.tensor(lens, dtype=torch.int32, device=device)
    generated = [tokens.clone()]
    for _ in range(spec["warmup_tokens"]):
        ids, _ = graph.step(tokens, pos)
        tokens.copy_(ids)
        pos += 1
        generated.append(tokens.clone())
    steps = spec["new_tokens"] - 1 - spec["warmup_tokens"]
    kv_pos = [[min(n + spec["warmup_tokens"] + i, cfg.sliding_window_size - 1) + 1 for n in lens] for i in range(steps)]
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        ids, _ = graph.step(tokens, pos)
        tokens.copy_(ids)
        pos += 1
        generated.append(tokens.clone())
    e1.record()
    torch.cuda.synchronize()
    dec_ms = e0.elapsed_time(e1) / steps
    # end to end: the serving loop reads every step's ids back to the host (as stream_generate's
    # per-token .item(), model/uttt_model.py:1038) and feeds the next tokens from pinned host memory
    hid = torch.empty(P, dtype=torch.int32).pin_memory()
    htok = torch.empty(P, dtype=torch.int32).pin_memory()
    htok.copy_(tokens)
    e2e_steps = 16
    torch.cuda.synchronize()
    e0.record()
    for _ in range(e2e_steps):
        tokens.copy_(htok, non_blocking=True)
        ids, _ = graph.step(tokens, pos)
        hid.copy_(ids, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        htok.copy_(hid)
        pos += 1
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    # the serving engine's own loop: the rows live on the device (DecodeTable) and advance inside the
    # captured step, and the host reads them back one step behind (no per-step round trip)
    from utttcompanion_b200.model import DecodeTable
    pad = P - 1 if P > 1 else 0
    table = DecodeTable(device, P, pad, stop_free=True)
    tgraph = DecodeGraph(eng, P, packed, down, table=table)
    for p in range(P):
        table.admit(p, tokens[p:p + 1], int(pos[p]), p, p, 1 << 30, None)
    for i in range(3):
        tgraph.step()
    eng_steps = 16
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(eng_steps):
        tgraph.step()
        table.snapshot(i & 1)
        if i:
            table.read((i - 1) & 1)
    table.read((eng_steps - 1) & 1)
    engine_ms = (time.perf_counter() - t0) / eng_steps * 1e3
    del tgraph, table
    # live kernel timing of one eager step (same kernels as the graph)
    lib.uttt_profile_enable(1)
    eng.decode_step(tokens, pos, graph.slots, packed, down, graph.sidx)
    ms = np.zeros(16, np.float32)
    cnt = np.zeros(16, np.int32)
    _lib.check(lib.uttt_profile_read(ms.ctypes.data, cnt.ctypes.data), "profile_read")
    lib.uttt_profile_enable(0)
    readout_s = ms[4] / max(cnt[4], 1) / 1e3
    readout_bytes = P * 3.0 * cfg.d_model * cfg.d_ff_fast * 2.0      # BF16 read copies of every persona
    # bytes one decode step must move: every persona's read copies in every layer, the shared
    # slow weights once, and each persona's valid KV slots (K and V) in every layer
    slow_bytes = sum(t.numel() * t.element_size() for lay in eng.layers for t in (lay.wqkv, lay.wo, lay.w_q, lay.w_o))
    slow_bytes += eng.lm_head.numel() * eng.lm_head.element_size()
    kv_bytes = float(np.mean([sum(kp) for kp in kv_pos])) * cfg.n_kv_heads * cfg.head_dim * 2 * 2 * cfg.n_layers
    step_bytes = readout_bytes * cfg.n_layers + slow_bytes + kv_bytes
    batch1 = decode_batch1(eng, packed, down, int(pos[0]), cfg) if spec.get("batch1") else None
    del graph, packed, down
    # one write per persona on prompt + reply (personalizer.py:483-512), batched over personas
    gen = torch.stack(generated, dim=1).cpu()                          # (P, new_tokens)
    turns = [prompts[p].tolist() + gen[p].tolist() for p in range(P)]
    Tmax = max(len(t) for t in turns)
    Tpad = ((Tmax + 63) // 64) * 64
    inter = torch.zeros(P, Tpad, dtype=torch.long)
    mask = torch.zeros(P, Tpad)
    for p, t in enumerate(turns):
        inter[p, :len(t)] = torch.tensor(t)
        mask[p, :len(t)] = 1.0
    st = FastState(w_up, w_gate, w_down, torch.zeros_like(w_up), torch.zeros_like(w_gate), torch.zeros_like(w_down),
                   eng.ln_w.clone(), eng.ln_b.clone())
    # warm-up on two chunks of every row (workspaces and temporaries at the full row count are
    # allocated before the timed region); st is not modified
    eng.test_time_update_batch(inter[:, :128], st, mask[:, :128])
    torch.cuda.synchronize()
    e0.record()
    new, surprises, _ = eng.test_time_update_batch(inter, st, mask)
    e1.record()
    torch.cuda.synchronize()
    write_ms = e0.elapsed_time(e1)
    del new
    valid = float(mask.sum())
    # bytes the write must move: per row-chunk (a persona's 64-token chunk with a valid token) and
    # layer, FP32 W and S read + written (48 d h) and the chunk-start BF16 read copy read by the
    # readout (6 d h); per row-chunk once, the read-copy rebuild (FP32 read, BF16 written: 18 d h)
    row_chunks = sum((len(t) + 63) // 64 for t in turns)
    dh = float(cfg.d_model) * cfg.d_ff_fast
    write_bytes = row_chunks * (cfg.n_layers * 54.0 * dh + 18.0 * dh)
    return {
        "workload": f"packed multi-persona greedy decode + per-turn chunk-TTT write ({spec['label']})",
        "model": f"uTTT d={cfg.d_model}, {cfg.n_layers} layers, {cfg.n_heads}/{cfg.n_kv_heads} heads, "
                 f"h={cfg.d_ff_fast}, V={cfg.vocab_size}, window {cfg.sliding_window_size}; {init_desc}",
        "personas": P, "prompts": spec["prompt_desc"], "new_tokens": spec["new_tokens"],
        "prompt_tokens": {"min": min(lens), "max": max(lens), "mean": float(np.mean(lens))},
        "decode_tok_s": P / (dec_ms / 1e3), "decode_ms_per_step": dec_ms, "decode_steps_timed": steps,
        "decode_e2e_tok_s": P / (e2e_ms / 1e3),
        "decode_engine_tok_s": P / (engine_ms / 1e3),
        "decode_engine_note": "device-resident rows advanced inside the captured step (uttt_engine_step), read "
                              "back one step behind, wall clock: the serving engine's own decode loop",
        "decode_step_roofline": {"bound": "hbm", "bytes_per_step": step_bytes,
                                 "achieved": step_bytes / (dec_ms / 1e3) / 1e9, "unit": "GB/s"},
        "prefill_s_total": prefill_s,
        "write_tok_s": valid / (write_ms / 1e3), "write_padded_tok_s": P * Tpad / (write_ms / 1e3),
        "write_roofline": {"bound": "hbm", "bytes": write_bytes, "row_chunks": row_chunks,
                           "achieved": write_bytes / (write_ms / 1e3) / 1e9, "unit": "GB/s"},
        "write_ms": write_ms, "mean_surprise": float(np.mean(surprises)),
        "write_config": {"momentum": cfg.momentum_beta, "clip": cfg.max_inner_grad_norm,
                         "inner_lr": cfg.base_inner_lr},
        "readout_roofline": {"bound": "hbm", "kernel": "readout_decode (GEMV + fused LayerNorm)",
                             "achieved": readout_bytes / readout_s / 1e9, "unit": "GB/s",
                             "algorithmic_bytes_per_launch": readout_bytes, "avg_ms": readout_s * 1e3},
        "decode_kernels_ms": {k: float(ms[i]) for i, k in enumerate(
            ["chunk_fwd", "chunk_ln", "chunk_norm", "chunk_bwd", "readout", "readout_ln", "gemm", "finish",
             "attn", "rowwise", "argmax"]) if cnt[i]},
        **({"decode_batch1": batch1} if batch1 else {}),
        **({"reference_baselines": reference_model_baselines(device, spec, cfg)} if baselines else {}),
    }


def decode_batch1(eng, packed, down, pos0, cfg, steps=64):
    """Batch-1 decode of one persona (the reference's only published serving measurement): the
    captured packed step at batch 1, 64 tokens, device time per token; and the same loop reading
    every token back to the host before the next step (``stream_generate``'s per-token ``.item()``)."""
    from utttcompanion_b200.model import DecodeGraph
    dev = eng.device
    g1 = DecodeGraph(eng, 1, packed, down)
    tok = torch.full((1,), 7, dtype=torch.int32, device=dev)
    pos = torch.full((1,), pos0, dtype=torch.int32, device=dev)
    for _ in range(3):
        ids, _ = g1.step(tok, pos)
        tok.copy_(ids)
        pos += 1
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(steps):
        ids, _ = g1.step(tok, pos)
        tok.copy_(ids)
        pos += 1
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    host = torch.empty(1, dtype=torch.int32).pin_memory()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        ids, _ = g1.step(tok, pos)
        host.copy_(ids, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        tok.fill_(int(host[0]))
        pos += 1
    e2e_s = (time.perf_counter() - t0) / steps
    del g1
    fast = cfg.n_layers * 3.0 * cfg.d_model * cfg.d_ff_fast * 2.0
    slow = float(sum(x.numel() * x.element_size() for lay in eng.layers for x in (lay.wqkv, lay.wo, lay.w_q, lay.w_o)))
    slow += eng.lm_head.numel() * eng.lm_head.element_size()
    return {"tok_s": 1e3 / ms, "ms_per_token": ms, "e2e_tok_s": 1.0 / e2e_s, "steps": steps,
            "hbm_gbs": (fast + slow) / (ms / 1e3) / 1e9,
            "reference_published_rtx5090_tok_s": {"eager": 71.4, "cuda_graph": 123.1, "cuda_graph_packed": 127.4,
                                                  "source": "docs/performance_20261029.md:12,19 (RTX 5090)"}}


def hsplit_decode_workload(device, rank, world, lib, spec, steps=48):
    """The 1.58B decode with every persona's hidden units split over all ranks
    (NCCL all-reduce of the readout's z per layer): the same personas, prompts
    and tokens on every rank; the packed step with its 34 all-reduces captured in
    one CUDA graph (eager steps if the capture is refused); max-over-ranks step time."""
    import torch.distributed as dist
    from utttcompanion_b200 import workloads as wl
    from utttcompanion_b200.hsplit import HiddenSplit
    from utttcompanion_b200.model import UtttB200
    cfg = wl.CONFIG_1P58B
    P = spec["personas"]
    hs = HiddenSplit()
    sd = wl.random_state_dict(cfg, seed=0, device=device)          # identical on every rank
    eng = UtttB200(sd, cfg, device=device, max_personas=P, max_positions=spec["prompt_max"] + steps + 64,
                   hsplit=hs)
    # the decode readouts' z sums through NVLink peer memory (one kernel per layer, no NCCL call);
    # NCCL stays for the prefill and the write
    peer = hs.enable_peer_exchange(max_rows=P, d=cfg.d_model, device=device)
    w0 = (sd["fast_weight_pool.w_up_init"], sd["fast_weight_pool.w_gate_init"], sd["fast_weight_pool.w_down_init"])
    del sd
    full = wl.perturbed_persona_states(*w0, P, spec["perturb_std"], seed=100, device=device)
    del w0
    local = hs.shard(*full)
    keep = [w[:PARITY_ROWS].clone() for w in full]        # unsplit copies of the parity rows
    del full
    packed, down = eng.read_copies(*local)
    del local
    g = torch.Generator().manual_seed(7)
    lens = spec["prompts"](g, P)
    prompts = [torch.randint(6, cfg.vocab_size, (n,), generator=g) for n in lens]
    first = torch.stack([eng.prefill(prompts[p], p, packed, down, p) for p in range(P)])
    tokens, _ = eng.greedy(first)
    tokens0 = tokens.clone()
    pos = torch.tensor(lens, dtype=torch.int32, device=device)
    slots = torch.arange(P, dtype=torch.int32, device=device)
    step0 = None
    for i in range(3):
        lg = eng.decode_step(tokens, pos, slots, packed, down, slots)
        if i == 0:
            step0 = lg[:PARITY_ROWS].float().clone()
        tokens, _ = eng.greedy(lg)
        pos += 1
    torch.cuda.synchronize()
    parity = hsplit_parity(device, rank, hs, cfg, keep, prompts[:PARITY_ROWS], first[:PARITY_ROWS].float(),
                           tokens0[:PARITY_ROWS], step0, torch.tensor(lens[:PARITY_ROWS], dtype=torch.int32,
                                                                      device=device))
    del keep
    torch.cuda.empty_cache()
    from utttcompanion_b200.model import DecodeGraph
    graph, mode = None, "graph"
    try:
        graph = DecodeGraph(eng, P, packed, down, stop_free=True)
    except RuntimeError as exc:          # capture of the collectives refused: time eager steps
        graph, mode = None, f"eager ({str(exc).splitlines()[0][:120]})"
        torch.cuda.synchronize()

    def one_step(tokens, pos):
        if graph is not None:
            return graph.step(tokens, pos)[0]
        return eng.greedy(eng.decode_step(tokens, pos, slots, packed, down, slots))[0]

    for _ in range(3):
        tokens = one_step(tokens, pos)
        pos += 1
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        tokens = one_step(tokens, pos)
        pos += 1
    e1.record()
    torch.cuda.synchronize()
    del graph                            # a graph holding NCCL calls goes before the process group
    torch.cuda.synchronize()
    hs.check_peer_exchange()             # raises if a flag wait of the exchange expired
    t = torch.tensor([e0.elapsed_time(e1) / steps], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dec_ms = float(t.item())
    # where an (eager) step's time goes: the all-reduces of z against the kernels every rank runs
    # whole (projections + finish, attention, row-wise, LM head) and the split readout, per step,
    # CUDA events on the step's stream, max over ranks
    bsteps = 3
    hs.timing = []
    lib.uttt_profile_enable(1)
    for _ in range(bsteps):
        tokens = eng.greedy(eng.decode_step(tokens, pos, slots, packed, down, slots))[0]
        pos += 1
    torch.cuda.synchronize()
    pms = np.zeros(16, np.float32)
    pcnt = np.zeros(16, np.int32)
    lib.uttt_profile_read(pms.ctypes.data, pcnt.ctypes.data)
    lib.uttt_profile_enable(0)
    ar_ms = sum(a.elapsed_time(b) for a, b in hs.timing)
    n_ar = len(hs.timing)
    hs.timing = None
    kinds = {"allreduce_z": ar_ms, "readout_partial": float(pms[4]), "readout_finish": float(pms[5]),
             "projections": float(pms[6]), "projection_finish": float(pms[7]), "attention": float(pms[8]),
             "rowwise_argmax": float(pms[9] + pms[10])}
    kt = torch.tensor([v / bsteps for v in kinds.values()], device=device, dtype=torch.float64)
    dist.all_reduce(kt, op=dist.ReduceOp.MAX)
    breakdown = {k: float(v) for k, v in zip(kinds, kt.tolist())}
    breakdown["allreduces_per_step"] = n_ar / bsteps
    breakdown["z_sum"] = ("NVLink peer exchange fused with the finish (uttt_split_exchange_finish; its time is "
                          "readout_finish)" if peer else "NCCL all-reduce + readout finish")
    hs.check_peer_exchange()
    hs.close_peer_exchange()
    slow_bytes = sum(x.numel() * x.element_size() for lay in eng.layers for x in (lay.wqkv, lay.wo, lay.w_q, lay.w_o))
    slow_bytes += eng.lm_head.numel() * eng.lm_head.element_size()
    per_gpu = P * 3.0 * cfg.d_model * (cfg.d_ff_fast // world) * 2.0 * cfg.n_layers + slow_bytes
    del packed, down, eng
    return {
        "workload": f"1.58B packed greedy decode, every persona's fast-weight hidden units split over {world} GPUs "
                    f"(readout z summed per layer {'through NVLink peer memory' if peer else 'by NCCL all-reduce'}), "
                    f"{mode} steps",
        "personas": P, "prompts": spec["prompt_desc"],
        "prompt_tokens": {"min": min(lens), "max": max(lens), "mean": float(np.mean(lens))},
        "decode_tok_s": P / (dec_ms / 1e3), "decode_ms_per_step": dec_ms, "decode_steps_timed": steps,
        "per_gpu_fast_weight_bytes_per_step": per_gpu,
        "per_gpu_hbm_gbs": per_gpu / (dec_ms / 1e3) / 1e9,
        "eager_step_breakdown_ms": breakdown,
        "parity": parity,
    }


PARITY_ROWS = 8


def hsplit_parity(device, rank, hs, cfg, full_rows, prompts, first_split, tokens0, step0_split, pos0):
    """Correctness of the hidden split inside the bench run, against an unsplit engine on rank 0.

    Decode: the split engine's prefill logits and its first packed decode step for the first
    PARITY_ROWS personas, against an unsplit 1.58B engine on rank 0 fed the same prompts, tokens and
    positions: max |logit difference| and whether every greedy id agrees.  Write: one chunk
    (momentum 0.9, clip 1.0) of two personas at the 1.58B layer shape, each rank updating its hidden
    slices with the partial Z and clip norms summed over the ranks; the slices gathered on rank 0
    against the unsplit write of the same inputs (state and update rel-L2).  Every rank takes the
    same collective steps."""
    import torch.distributed as dist
    from utttcompanion_b200 import fastweight as fw
    from utttcompanion_b200.model import UtttB200
    from utttcompanion_b200 import workloads as wl
    out = {"rows": len(prompts)}
    if rank == 0:
        sd = wl.random_state_dict(cfg, seed=0, device=device)
        ref = UtttB200(sd, cfg, device=device, max_personas=len(prompts), max_positions=4096 + 128)
        del sd
        rp, rd = ref.read_copies(*full_rows)
        first = torch.stack([ref.prefill(prompts[p], p, rp, rd, p) for p in range(len(prompts))]).float()
        slots = torch.arange(len(prompts), dtype=torch.int32, device=device)
        step0 = ref.decode_step(tokens0, pos0, slots, rp, rd, slots).float()
        # the unsplit engine against itself: the same prefill and step once more (its atomic FP32
        # accumulation order varies from run to run, and a flipped BF16 rounding of z is amplified
        # by the LayerNorm and 34 layers), the noise floor of any second implementation
        first2 = torch.stack([ref.prefill(prompts[p], p, rp, rd, p) for p in range(len(prompts))]).float()
        step02 = ref.decode_step(tokens0, pos0, slots, rp, rd, slots).float()
        self_diff = max(float((first2 - first).abs().max()), float((step02 - step0).abs().max()))
        d_pre = float((first - first_split).abs().max())
        d_dec = float((step0 - step0_split).abs().max())
        same = bool(torch.equal(first.argmax(-1), first_split.argmax(-1))
                    and torch.equal(step0.argmax(-1), step0_split.argmax(-1)))
        bound = max(2e-2, 2.0 * self_diff)
        # every greedy id that differs must sit at a near-tie of the unsplit logits (top-2 margin within
        # twice the bound), as the parity tests require
        flips = []
        for name, ref_l, got_l in (("prefill", first, first_split), ("decode", step0, step0_split)):
            for r in range(ref_l.shape[0]):
                if int(ref_l[r].argmax()) != int(got_l[r].argmax()):
                    top = torch.topk(ref_l[r], 2).values
                    flips.append({"logits": name, "row": r, "unsplit_top2_margin": float(top[0] - top[1])})
        out.update(max_abs_logit_diff_prefill=d_pre, max_abs_logit_diff_decode=d_dec, greedy_equal=same,
                   within_2e2=max(d_pre, d_dec) <= 2e-2, unsplit_repeat_diff=self_diff, logit_bound=bound,
                   within_bound=max(d_pre, d_dec) <= bound, greedy_flips=flips,
                   flips_at_near_ties=all(f["unsplit_top2_margin"] <= 2 * bound for f in flips))
        del ref, rp, rd
        torch.cuda.empty_cache()
    # one split write of two personas' layer state against the unsplit write
    B, d, h, C = 2, cfg.d_model, cfg.d_ff_fast, 64
    g = torch.Generator(device=device).manual_seed(17)

    def unit():
        x = torch.randn(B, C, d, generator=g, device=device)
        return (x / x.norm(dim=-1, keepdim=True)).to(torch.bfloat16).contiguous()
    k, v = unit(), unit()
    eta = torch.rand(B, C, generator=g, device=device) * 0.04 + 0.005
    alpha = torch.rand(B, C, generator=g, device=device) * 0.01
    lnw, lnb = torch.ones(d, device=device), torch.zeros(d, device=device)
    W = [w[:B].contiguous() for w in full_rows]
    S = [torch.randn(w.shape, generator=g, device=device) * 1e-4 for w in W]
    lo, hi = hs.bounds(h)
    mine = [x.contiguous() for x in hs.shard(*W)] + [x.contiguous() for x in hs.shard(*S)]
    fw.chunk_write(k, v, eta, alpha, *mine, lnw, lnb, None, 0.9, 1.0, True, 1e-5, chunk_size=C,
                   partial_sum=hs.all_reduce)
    parts = []
    for t in mine[:3]:
        bufs = [torch.empty_like(t) for _ in range(hs.world)]
        dist.all_gather(bufs, t)
        parts.append(bufs)
    torch.cuda.synchronize()
    if rank == 0:
        got = [torch.cat(parts[0], dim=2), torch.cat(parts[1], dim=2), torch.cat(parts[2], dim=1)]
        ref_state = [w.clone() for w in W] + [s.clone() for s in S]
        fw.chunk_write(k, v, eta, alpha, *ref_state, lnw, lnb, None, 0.9, 1.0, True, 1e-5, chunk_size=C)
        torch.cuda.synchronize()
        rel = [float(torch.linalg.norm(a - b) / torch.linalg.norm(b)) for a, b in zip(got, ref_state[:3])]
        upd = [float(torch.linalg.norm((a - w) - (b - w)) / torch.linalg.norm(b - w))
               for a, b, w in zip(got, ref_state[:3], W)]
        out.update(write_state_rel_l2=max(rel), write_update_rel_l2=max(upd),
                   write_within_bounds=max(rel) <= 1e-3 and max(upd) <= 2e-2,
                   write_case="one chunk, 2 personas, d=2560, h=6912 split over the ranks, momentum 0.9, clip 1.0")
    del mine, parts, W, S
    return out if rank == 0 else None


# ----------------------------------------------------------------------------- serve sweep (config 5)
def serve_sweep(device, lib, config, rates, duration_s, personas=256, max_batch=64, seed=0, write_batch=32,
                write_wait_s=0.2, async_writes=False, world=1, rank=0):
    """continuous batching of persona turns, personas partitioned by user id.

    Turns arrive as a Poisson process at each rate; each picks a user uniformly among
    ``personas``, a prompt of lognormal length (median 256, sigma 1.0, clipped to [16, 2048])
    with uniform ids and a forced reply length uniform in [32, 256] (greedy); every completed
    turn is written into its user's state (chunk-TTT write, surprise gate, elastic pull).
    Every rank draws the same schedule and serves the turns of the users ``PersonaRouter``
    maps to it (no collective on the data path); the ranks start each rate together and rank 0
    gathers the latencies.  Reports whole-job generated / written tokens per second over the
    slowest rank's wall time and the arrival -> result latency of every turn.  Returns the
    result on rank 0, None elsewhere."""
    from utttcompanion_b200 import workloads as wl
    from utttcompanion_b200.model import UtttB200
    from utttcompanion_b200.serving import PersonaRouter, ServingEngine
    cfg = {"151M": wl.CONFIG_151M, "1P58B": wl.CONFIG_1P58B}[config]
    router = PersonaRouter(world)
    mine = [u for u in (f"user-{i}" for i in range(personas)) if router.rank_of(u) == rank]
    sd = wl.random_state_dict(cfg, seed=seed, device=device)
    eng = UtttB200(sd, cfg, device=device, max_personas=len(mine) + 1, max_positions=2048 + 256 + 64)
    del sd
    srv = ServingEngine(eng, capacity=max(len(mine), 1), max_batch=max_batch, surprise_threshold=cfg.surprise_threshold,
                        stop_free=True, write_batch=write_batch, write_wait_s=write_wait_s,
                        async_writes=async_writes)
    g = torch.Generator().manual_seed(seed)

    def draw_turn(gen=g):
        n = int(min(max(round(256 * math.exp(float(torch.randn(1, generator=gen, dtype=torch.float64)))), 16), 2048))
        reply = int(torch.randint(32, 257, (1,), generator=gen))
        user = f"user-{int(torch.randint(0, personas, (1,), generator=gen))}"
        return user, torch.randint(6, cfg.vocab_size, (n,), generator=gen).tolist(), reply

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    # bytes a decode step must move: every live persona's BF16 read copies in every layer, and the
    # shared slow weights (projections + LM head) once per step
    fast_tok = cfg.n_layers * 3.0 * cfg.d_model * cfg.d_ff_fast * 2.0
    slow_step = float(sum(x.numel() * x.element_size() for lay in eng.layers for x in (lay.wqkv, lay.wo, lay.w_q,
                                                                                           lay.w_o)))
    slow_step += eng.lm_head.numel() * eng.lm_head.element_size()
    hbm_peak = peaks()[0]
    gw = torch.Generator().manual_seed(seed + 1 + rank)   # warm-up turns of this rank's users; the
    for k in range(4):                                     # shared schedule generator stays in step
        _, ids, rl = draw_turn(gw)
        srv.submit(mine[k % len(mine)], ids, rl)
    srv.run()
    out = []
    for lam in rates:
        t, arrivals = 0.0, []
        while True:
            t += float(torch.empty(1).exponential_(lam, generator=g))
            if t > duration_s:
                break
            arrivals.append((t, *draw_turn()))
        arrivals = [a for a in arrivals if router.rank_of(a[1]) == rank]
        srv.stats.clear()
        barrier()
        start = time.perf_counter()
        live, done = [], []
        i = 0
        while i < len(arrivals) or live:
            now = time.perf_counter() - start
            while i < len(arrivals) and arrivals[i][0] <= now:
                at, user, prompt, reply = arrivals[i]
                rec = {}

                def on_event(ev, rec=rec):      # time to first token: the prefill's greedy pick
                    if ev["type"] == "token" and "first" not in rec:
                        rec["first"] = time.perf_counter() - start
                live.append((at, srv.submit(user, prompt, reply, on_event=on_event), rec))
                i += 1
            if srv.idle():
                time.sleep(max(0.0, min(arrivals[i][0] - now, 0.05)) if i < len(arrivals) else 0.0)
                continue
            srv.step()
            now = time.perf_counter() - start
            still = []
            for at, turn, rec in live:
                if turn.done:
                    done.append((now - at, rec.get("first", now) - at))
                else:
                    still.append((at, turn, rec))
            live = still
        wall = time.perf_counter() - start
        st = dict(srv.stats)
        part = {"wall": wall, "lat": [x for x, _ in done], "ttft": [y for _, y in done], "stats": st}
        if world > 1:
            import torch.distributed as dist
            parts = [None] * world
            dist.all_gather_object(parts, part)
        else:
            parts = [part]
        if rank != 0:
            continue
        wall = max(pp["wall"] for pp in parts)
        lat = np.array([x for pp in parts for x in pp["lat"]]) if any(pp["lat"] for pp in parts) else np.zeros(1)
        ttft = np.array([x for pp in parts for x in pp["ttft"]]) if any(pp["ttft"] for pp in parts) else np.zeros(1)
        tot = collections.Counter()
        for pp in parts:
            tot.update(pp["stats"])
        nturns = sum(len(pp["lat"]) for pp in parts)
        out.append({
            "rate_req_s": lam, "turns": nturns, "wall_s": wall,
            "decode_tok_s": tot["decode_tokens"] / wall, "write_tok_s": tot["write_tokens"] / wall,
            "prefill_tok_s": tot["prefill_tokens"] / wall,
            "latency_s": {"p50": float(np.percentile(lat, 50)), "p99": float(np.percentile(lat, 99)),
                          "mean": float(lat.mean())},
            "first_token_s": {"p50": float(np.percentile(ttft, 50)), "p99": float(np.percentile(ttft, 99))},
            "mean_decode_batch": tot["decode_tokens"] / max(tot["decode_steps"], 1),
            "busy_s": {"prefill": tot["prefill_s"], "decode": tot["decode_s"], "write": tot["write_s"]},
            "write_batches": tot["write_batches"],
            "decode_ms_per_step": 1e3 * tot["decode_s"] / max(tot["decode_steps"], 1),
            "write_ms_per_turn": 1e3 * tot["write_s"] / max(nturns, 1),
            "prefill_ms_per_turn": 1e3 * tot["prefill_s"] / max(nturns, 1),
            "turns_per_rank": [len(pp["lat"]) for pp in parts],
        })
        # decode HBM rate per GPU: the bytes its steps had to move over its busy decode time (host
        # scheduling included), averaged over ranks
        rates_gbs = [(pp["stats"].get("decode_tokens", 0) * fast_tok + pp["stats"].get("decode_steps", 0) * slow_step)
                     / max(pp["stats"].get("decode_s", 0.0), 1e-9) / 1e9 for pp in parts]
        out[-1]["decode_hbm_gbs_per_gpu"] = float(np.mean(rates_gbs))
        out[-1]["decode_hbm_frac"] = float(np.mean(rates_gbs)) / hbm_peak
        print(json.dumps(out[-1]), file=sys.stderr, flush=True)
    srv.close()
    if rank != 0:
        return None
    return {"workload": f"continuous-batching serve sweep (BASELINE config 5) on the {config} model, "
                        f"{world} GPU(s), personas partitioned by user id",
            "n_gpus": world, "personas": personas, "max_batch": max_batch, "arrivals": "Poisson",
            "duration_s": duration_s, "write_batch": write_batch, "write_wait_s": write_wait_s,
            "writes_overlap_decode": async_writes,
            "prompts": "lognormal, median 256, sigma 1.0, clipped to [16, 2048]",
            "replies": "uniform in [32, 256] tokens, forced length (greedy, stop ids masked)",
            "writes": "every completed turn: chunk-TTT write + surprise gate + elastic pull", "points": out}


def micro_case(device, kind, batch, tokens, hist, iters=30):
    """Kernel profiling cases at the 1.58B shape (one JSON object; not a bench line).

    ``decode``: one packed decode step of ``batch`` personas through all 34 layers (CUDA graph).

    ``readout``: the decode readout (GEMV + fused LayerNorm, d=2560, h=6912) of ``batch``
    rows, each on its own BF16 read copy; 24 copies (2.5 GB) cycle so every call streams
    its weights from HBM.  ``attn``: the prefill / chunk attention (20 query heads over 5 KV
    heads of dim 128, window 512) of ``batch`` rows x ``tokens`` new tokens after ``hist``
    history positions (RoPE kernel included).  ``write``: the chunk-TTT write of ``batch`` rows
    (one state each) for ``tokens`` tokens at one 1.58B layer (momentum 0.9, clip 1.0, the model
    write's settings), with the time of each kernel kind from live CUDA events; its bytes are
    the update's 48·d·h per row and chunk."""
    from utttcompanion_b200 import _lib
    from utttcompanion_b200.fastweight import _stream
    lib = _lib.load()
    g = torch.Generator(device=device).manual_seed(0)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if kind == "decode":
        # one packed 1.58B decode step of `batch` personas (each its own perturbed read copies),
        # replayed from its CUDA graph; bytes = every persona's read copies in every layer + the
        # slow weights once + each persona's KV window
        from utttcompanion_b200 import workloads as wl
        from utttcompanion_b200.model import DecodeGraph, UtttB200
        cfg = wl.CONFIG_1P58B
        sd = wl.random_state_dict(cfg, seed=0, device=device)
        eng = UtttB200(sd, cfg, device=device, max_personas=batch, max_positions=1024)
        w0 = (sd["fast_weight_pool.w_up_init"], sd["fast_weight_pool.w_gate_init"], sd["fast_weight_pool.w_down_init"])
        del sd
        packed, down = eng.read_copies(*wl.perturbed_persona_states(*w0, batch, 1e-3, seed=1, device=device))
        graph = DecodeGraph(eng, batch, packed, down, stop_free=True)
        tok = torch.full((batch,), 7, dtype=torch.int32, device=device)
        pos = torch.full((batch,), 600, dtype=torch.int32, device=device)

        def call(i):
            graph.step(tok, pos)
        slow = sum(x.numel() * x.element_size() for lay in eng.layers for x in (lay.wqkv, lay.wo, lay.w_q, lay.w_o))
        slow += eng.lm_head.numel() * eng.lm_head.element_size()
        kv = batch * cfg.n_layers * cfg.sliding_window_size * cfg.n_kv_heads * cfg.head_dim * 2 * 2
        nbytes = batch * cfg.n_layers * 3 * cfg.d_model * cfg.d_ff_fast * 2 + slow + kv
    elif kind == "write":
        from utttcompanion_b200 import fastweight as fw
        d, h, B, T = 2560, 6912, batch, tokens
        W = [torch.randn(B, d, h, device=device, generator=g) * d ** -0.5,
             torch.randn(B, d, h, device=device, generator=g) * d ** -0.5,
             torch.randn(B, h, d, device=device, generator=g) * 0.1 * h ** -0.5]
        S = [torch.zeros_like(w) for w in W]
        k = torch.randn(B, T, d, device=device, generator=g)
        k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
        v = torch.randn(B, T, d, device=device, generator=g)
        v = (v / v.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
        eta, alpha = torch.full((B, T), 0.0075, device=device), torch.full((B, T), 0.001, device=device)
        lw, lb = torch.ones(d, device=device), torch.zeros(d, device=device)
        call = lambda i: fw.chunk_write(k, v, eta, alpha, *W, *S, lw, lb, None, 0.9, 1.0, True, 1e-5)  # noqa: E731
        nbytes = B * ((T + 63) // 64) * 48 * d * h
        iters = min(iters, 10)
    elif kind == "readout":
        from utttcompanion_b200.readout import fast_readout
        d, h, S = 2560, 6912, 24
        packed = (torch.randn(S, d, 2 * h, device=device, generator=g) * 0.02).to(torch.bfloat16)
        down = (torch.randn(S, h, d, device=device, generator=g) * 0.02).to(torch.bfloat16)
        lw, lb = torch.ones(d, device=device), torch.zeros(d, device=device)
        x = torch.randn(batch, 1, d, device=device, generator=g).to(torch.bfloat16)
        out = torch.empty_like(x)
        idx = [((torch.arange(batch, device=device) + i * batch) % S).to(torch.int32) for i in range(iters + 3)]
        call = lambda i: fast_readout(x, packed, None, down, lw, lb, state_index=idx[i], packed=True,  # noqa: E731
                                      ln_prepared=True, out=out)
        nbytes = batch * 3 * d * h * 2
    else:
        hd, nh, nkv, W = 128, 20, 5, 512
        L = hist + tokens
        qkv_dim = (nh + 2 * nkv) * hd
        qkv = torch.randn(batch * tokens, qkv_dim, device=device, generator=g).to(torch.bfloat16)
        from utttcompanion_b200.model import rope_tables
        cos, sin = (t.to(device).contiguous() for t in rope_tables(hd, hist + tokens + 8, 10000.0))
        qs = torch.empty(batch * tokens, nh, hd, dtype=torch.bfloat16, device=device)
        kb = torch.randn(batch, nkv, L, hd, device=device, generator=g).to(torch.bfloat16)
        vb = torch.randn_like(kb)
        out = torch.empty(batch * tokens, nh, hd, dtype=torch.bfloat16, device=device)
        st = _stream(device)

        def call(i):
            _lib.check(lib.uttt_attn_prefill(batch, tokens, hist, hist, nh, nkv, hd, W, qkv.data_ptr(), qkv_dim,
                                             cos.data_ptr(), sin.data_ptr(), qs.data_ptr(), kb.data_ptr(),
                                             vb.data_ptr(), out.data_ptr(), st), "uttt_attn_prefill")
        nbytes = batch * nkv * L * hd * 2 * 2
    for i in range(3):
        call(i)
    torch.cuda.synchronize()
    e0.record()
    for i in range(iters):
        call(3 + i)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / iters * 1e3
    out = {"micro": kind, "batch": batch, "tokens": tokens, "hist": hist, "us_per_call": us,
           "bytes_per_call": nbytes, "gb_s": nbytes / us / 1e3, "iters": iters}
    if kind == "write":
        # per kernel kind, live CUDA events on the write's stream (one more pass of `iters` calls)
        lib.uttt_profile_enable(1)
        for i in range(iters):
            call(i)
        ms = np.zeros(16, np.float32)
        cnt = np.zeros(16, np.int32)
        lib.uttt_profile_read(ms.ctypes.data, cnt.ctypes.data)
        lib.uttt_profile_enable(0)
        kinds = {"forward": 0, "layernorm_backward": 1, "clip_norm": 2, "update": 3}
        out["kernels_us_per_call"] = {n: float(ms[i]) * 1e3 / iters for n, i in kinds.items()}
        upd = out["kernels_us_per_call"]["update"]
        out["update_gb_s"] = nbytes / upd / 1e3
        out["update_hbm_frac"] = out["update_gb_s"] / peaks()[0]
    return out


# ----------------------------------------------------------------------------- arms
def reference_arm(args, world, rank):
    """The reference's own CPU implementation of the headline op on the host cores, rank 0 only:
    each step one 64-token chunk of one config-2 state through its fused_chunk_ttt_step (PyTorch
    FP32 from baseline/_ref; the oracle port when the reference is not installed), every host
    thread in use whatever OMP_NUM_THREADS says."""
    if rank != 0:
        return 0
    cores = use_all_host_threads()
    step, kind, desc = chunk_stepper(1)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    C = CFG["chunk"]
    value = args.steps * C / el
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "chunk_ttt_write_isolated (BASELINE config 2)", **CFG,
                   "reference_sample": "one 64-token chunk of one state per step"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": kind,
                         "sample": f"{args.steps} chunk steps of one d=1024,h=2816 state (64 tokens each): {desc}"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def ours_arm(args, world, rank, local):
    from utttcompanion_b200 import _lib
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        import torch.distributed as dist
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x: float) -> float:
        if world == 1:
            return x
        import torch.distributed as dist
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    lib = _lib.load()
    if args.micro:                # kernel profiling cases (1 GPU)
        if rank == 0:
            print(json.dumps(micro_case(device, args.micro, args.micro_batch, args.micro_tokens, args.micro_hist,
                                        iters=args.steps)), flush=True)
        return 0
    if args.only_decode:          # profiling case: the config-3 decode + write workload alone
        if rank == 0:
            print(json.dumps(decode_workload(device, rank, lib, DEC)), flush=True)
        return 0
    if args.serve_sweep:          # BASELINE config 5 (minutes per model): one JSON object from rank 0
        rates = [float(x) for x in args.serve_rates.split(",")]
        res = serve_sweep(device, lib, args.serve_config, rates, args.serve_seconds,
                          personas=args.serve_personas, write_batch=args.serve_write_batch,
                          async_writes=args.serve_async_writes, write_wait_s=args.serve_write_wait,
                          world=world, rank=rank)
        if rank == 0:
            print(json.dumps(res), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        return 0
    st = make_states(device, seed=1234 + rank)
    B, T = CFG["states"], CFG["tokens"]

    for _ in range(args.warmup):
        run_step(st)
    torch.cuda.synchronize()

    # live per-kernel timing on the launch stream (one extra, untimed step)
    lib.uttt_profile_enable(1)
    run_step(st)
    ms = (np.zeros(16, np.float32))
    cnt = np.zeros(16, np.int32)
    _lib.check(lib.uttt_profile_read(ms.ctypes.data, cnt.ctypes.data), "profile_read")
    lib.uttt_profile_enable(0)

    # timed region
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        run_step(st)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    step_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    value = world * B * T / (step_ms / 1e3)

    # end-to-end through the public API: pinned host K/V/eta/alpha in, token losses out, every step.
    # As a serving loop would, the next step's inputs are copied on a second stream while the
    # current step computes (two device input buffers); every copy is inside the timed region.
    names = ("k", "v", "eta", "alpha")
    host = {n: torch.empty_like(st[n], device="cpu").pin_memory() for n in names}
    hl = torch.empty_like(st["loss"], device="cpu").pin_memory()
    for n in names:
        host[n].copy_(st[n])
    bufs = [{n: st[n] for n in names}, {n: torch.empty_like(st[n]) for n in names}]
    comp = torch.cuda.current_stream(device)
    cps = torch.cuda.Stream(device)
    ready = [torch.cuda.Event(), torch.cuda.Event()]
    free = [torch.cuda.Event(), torch.cuda.Event()]

    def h2d_inputs(i):
        with torch.cuda.stream(cps):
            for n in names:
                bufs[i][n].copy_(host[n], non_blocking=True)
            ready[i].record(cps)

    e2e_steps = max(2, args.steps)           # as many steps as the device-timed region
    barrier()
    torch.cuda.synchronize()
    e0.record()
    cps.wait_event(e0)                       # the first copy starts inside the timed region
    h2d_inputs(0)
    for s in range(e2e_steps):
        cur, nxt = s % 2, (s + 1) % 2
        if s + 1 < e2e_steps:
            if s >= 1:
                cps.wait_event(free[nxt])    # step s - 1 has finished reading that buffer
            h2d_inputs(nxt)
        comp.wait_event(ready[cur])
        run_step({**st, **bufs[cur]})
        free[cur].record(comp)
        hl.copy_(st["loss"], non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = hl.numel() * hl.element_size()
    from utttcompanion_b200 import fastweight as fw
    fw.check_status(fw.workspace(0, device), "bench")
    # the reference's own PyTorch op on this GPU, same states (rank 0 of a 1-GPU run)
    torch_ref = None
    if world == 1 and not args.no_cpu_baseline:
        torch_ref = torch_reference_chunk_gpu(device, st)

    # decode + write workloads: at N = 1 configs 3 and 4; at N > 1 every rank serves its own
    # config-4 personas (64 per GPU below 4 GPUs, 256 in total from 4 GPUs up), then all
    # ranks decode 64 personas with the hidden units split across them
    extra = {}
    if not args.no_decode:
        import copy
        specs = [DEC] if world == 1 else []
        if not args.no_1p58b:
            spec4 = copy.copy(DEC4)
            spec4["personas"] = 64 if world < 4 else 256 // world
            specs.append(spec4)
        for spec in specs:
            dec = decode_workload(device, rank, lib, spec, baselines=world == 1 and not args.no_cpu_baseline)
            torch.cuda.empty_cache()
            if world > 1:
                dec_ms = max_over_ranks(dec["decode_ms_per_step"])
                dec_e2e_ms = max_over_ranks(spec["personas"] / dec["decode_e2e_tok_s"] * 1e3)
                write_ms = max_over_ranks(dec["write_ms"])
                valid = sum_over_ranks(dec["write_tok_s"] * dec["write_ms"] / 1e3)
                padded = sum_over_ranks(dec["write_padded_tok_s"] * dec["write_ms"] / 1e3)
                total = spec["personas"] * world
                dec.update({"personas_per_gpu": spec["personas"], "personas": total, "n_gpus": world,
                            "decode_tok_s": total / (dec_ms / 1e3), "decode_ms_per_step": dec_ms,
                            "decode_e2e_tok_s": total / (dec_e2e_ms / 1e3), "write_ms": write_ms,
                            "write_tok_s": valid / (write_ms / 1e3), "write_padded_tok_s": padded / (write_ms / 1e3),
                            "partition": "personas by user id, no collective; step times max over ranks"})
            extra[spec["key"]] = dec
        if world > 1 and not args.no_1p58b:
            extra["decode_1p58b_hsplit"] = hsplit_decode_workload(device, rank, world, lib, DEC4)
            torch.cuda.empty_cache()

    if rank == 0:
        hbm, tflops, src = peaks()
        kinds = {0: "chunk_fwd", 1: "chunk_ln", 2: "chunk_norm", 3: "chunk_bwd_update"}
        per_kind = {kinds[k]: {"ms_total": float(ms[k]), "launches": int(cnt[k])} for k in kinds if cnt[k]}
        dom = max(kinds, key=lambda k: ms[k])
        avg_s = ms[dom] / max(cnt[dom], 1) / 1e3
        alg = algorithmic_bytes(dom)
        achieved = alg / avg_s / 1e9
        traffic = None
        rec = traffic_record()
        if rec and rec.get("kernel") == kinds[dom]:
            traffic = rec.get("bytes_per_launch")
        total_flops = 14.0 * CFG["chunk"] * CFG["d"] * CFG["h"] * (T // CFG["chunk"]) * B
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "chunk_ttt_write_isolated (BASELINE config 2)", **CFG,
                       "parallelism": f"states partitioned over {world} GPU(s), no collective",
                       "l2": "inputs larger than L2 (2.2 GB FP32 state per GPU)"},
            "e2e": {"value": world * B * T / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h), "steps": e2e_steps,
                    "copies": "pinned host inputs of step s+1 copied on a second stream during step s; "
                              "token losses read back every step"},
            "gpu_launches": launches_per_step() * args.steps,
            "roofline": {"bound": "hbm", "kernel": kinds[dom], "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "peak_source": src, "traffic": traffic,
                         "algorithmic_bytes_per_launch": alg},
            "tensor_tflops": total_flops / (step_ms / 1e3) / 1e12,
            "kernels": per_kind,
            "clocks": clk,
        }
        for key, dec in extra.items():
            for rkey in ("readout_roofline", "decode_step_roofline", "write_roofline"):
                if rkey in dec:
                    dec[rkey]["peak"] = hbm
                    dec[rkey]["frac"] = dec[rkey]["achieved"] / hbm
            if "per_gpu_hbm_gbs" in dec:
                dec["per_gpu_hbm_frac"] = dec["per_gpu_hbm_gbs"] / hbm
            line[key] = dec
        if world == 1 and not args.no_cpu_baseline:
            v, n, el, kind, desc, cores = cpu_baseline()
            line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": cores, "kind": kind,
                                    "sample": f"{n} chunk steps of one config-2 state ({n * CFG['chunk']} tokens, "
                                              f"{el:.1f} s): {desc}"}
        if torch_ref is not None:
            line["torch_reference_gpu"] = torch_ref
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode + write workloads (configs 3, 4)")
    ap.add_argument("--no-1p58b", action="store_true", help="skip the 1.58B (config 4) decode + write workload")
    ap.add_argument("--serve-sweep", action="store_true", help="run only the config-5 serve sweep (1 GPU)")
    ap.add_argument("--serve-config", default="151M", choices=("151M", "1P58B"))
    ap.add_argument("--serve-rates", default="1,2,4,8,16,32,64", help="arrival rates, req/s")
    ap.add_argument("--serve-seconds", type=float, default=20.0, help="arrival window per rate")
    ap.add_argument("--serve-personas", type=int, default=256)
    ap.add_argument("--serve-write-batch", type=int, default=32, help="finished turns written together")
    ap.add_argument("--serve-write-wait", type=float, default=0.2, help="longest wait of a finished turn, s")
    ap.add_argument("--serve-async-writes", action="store_true",
                    help="write on a side stream from a worker thread, overlapping decode")
    ap.add_argument("--only-decode", action="store_true",
                    help="profiling: run only the config-3 decode + write workload (one JSON object, 1 GPU)")
    ap.add_argument("--micro", choices=("readout", "attn", "decode", "write"), default=None,
                    help="profiling case: one kernel at the 1.58B layer shape")
    ap.add_argument("--micro-batch", type=int, default=1)
    ap.add_argument("--micro-tokens", type=int, default=64)
    ap.add_argument("--micro-hist", type=int, default=0)
    ap.add_argument("--states", type=int, default=None, help="override states per GPU (profiling cases)")
    ap.add_argument("--tokens", type=int, default=None, help="override tokens per state (profiling cases)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.states:
        CFG["states"] = args.states
    if args.tokens:
        CFG["tokens"] = args.tokens
    world, rank, local = dist_env()
    if args.impl == "reference":
        return reference_arm(args, world, rank)
    return ours_arm(args, world, rank, local)


if __name__ == "__main__":
    sys.exit(main())
