"""Synthetic, seeded workloads with the reference's shapes.

``reference_init_state_dict`` builds a random-init uTTT state dict under the
reference's parameter names and in the order ``uTTTModel.__init__``
(``model/uttt_model.py:279-338``) draws from torch's CPU generator:
embedding, fast-weight pool W_0 (``model/uttt_layer.py:573-580``), each
block's nn.Linear modules (``:996-1001``, ``:1250-1263``), lm_head, then
``_init_slow_weights`` (``model/uttt_model.py:340-352``) re-draws every
non-gate Linear and the embedding from N(0, 0.02) in ``named_modules``
order, and the lm_head is tied to the embedding.  With the same seed it gives
the reference's own initial weights (checked against checksums of the
reference model in ``tests/test_workloads.py``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, asdict
from typing import Dict

import torch
import torch.nn as nn


@dataclass
class ModelConfig:
    """The hot-path fields of ``uTTTConfig`` (``model/uttt_model.py:44-111``), same defaults."""
    vocab_size: int = 32000
    d_model: int = 1024
    n_layers: int = 16
    n_heads: int = 16
    n_kv_heads: int = 4
    d_ff_fast: int = 2816
    sliding_window_size: int = 512
    max_seq_len: int = 4096
    rope_theta: float = 10000.0
    rms_norm_eps: float = 1e-5
    chunk_size: int = 64
    base_inner_lr: float = 0.015
    base_weight_decay: float = 0.005
    momentum_beta: float = 0.90
    max_inner_grad_norm: float = 1.0
    normalize_loss_by_dim: bool = True
    surprise_threshold: float = 0.25
    elastic_anchor_lambda: float = 0.02
    max_weight_drift_ratio: float = 0.35

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads

    @classmethod
    def from_dict(cls, data: Dict) -> "ModelConfig":
        """Flat or nested (model/uttt sections) dict, as ``uTTTConfig.from_dict``."""
        merged = {}
        if "model" in data or "uttt" in data:
            merged.update(data.get("model", {}))
            merged.update(data.get("uttt", {}))
        else:
            merged.update(data)
        fields = cls.__dataclass_fields__
        return cls(**{k: v for k, v in merged.items() if k in fields})

    def to_dict(self) -> Dict:
        return asdict(self)


# Model shapes of the benchmark configurations: the tiny CPU-runnable model, the 151M-class decoder and
# the 1.58B decoder (the dims of the reference's configs/5090_max_config.yaml, with C = 64)
CONFIG_TINY = ModelConfig(vocab_size=8000, d_model=256, n_layers=4, n_heads=4, n_kv_heads=4, d_ff_fast=688,
                          sliding_window_size=128, chunk_size=64)
CONFIG_151M = ModelConfig(vocab_size=32000, d_model=768, n_layers=12, n_heads=12, n_kv_heads=4, d_ff_fast=2048,
                          sliding_window_size=512, chunk_size=64)
CONFIG_1P58B = ModelConfig(vocab_size=32000, d_model=2560, n_layers=34, n_heads=20, n_kv_heads=5, d_ff_fast=6912,
                           sliding_window_size=512, chunk_size=64, base_inner_lr=0.015, base_weight_decay=0.005,
                           surprise_threshold=0.015)


def reference_init_state_dict(cfg: ModelConfig, seed: int = 0) -> Dict[str, torch.Tensor]:
    """FP32 CPU state dict of a freshly initialised reference model (see module docstring)."""
    d, h, V, L = cfg.d_model, cfg.d_ff_fast, cfg.vocab_size, cfg.n_layers
    hd = cfg.head_dim
    gen_state = torch.random.get_rng_state()
    try:
        torch.manual_seed(seed)
        emb = nn.Embedding(V, d)
        w_up = torch.randn(d, h) * (1.0 / math.sqrt(d))
        w_gate = torch.randn(d, h) * (1.0 / math.sqrt(d))
        w_down = torch.randn(h, d) * (0.1 * (1.0 / math.sqrt(h)))
        layers = []
        for _ in range(L):
            mods = {
                "attn.wq": nn.Linear(d, cfg.n_heads * hd, bias=False),
                "attn.wk": nn.Linear(d, cfg.n_kv_heads * hd, bias=False),
                "attn.wv": nn.Linear(d, cfg.n_kv_heads * hd, bias=False),
                "attn.wo": nn.Linear(cfg.n_heads * hd, d, bias=False),
                "uttt.w_q": nn.Linear(d, d, bias=False),
                "uttt.w_k": nn.Linear(d, d, bias=False),
                "uttt.w_v": nn.Linear(d, d, bias=False),
                "uttt.w_o": nn.Linear(d, d, bias=False),
                "uttt.w_eta": nn.Linear(d, 1, bias=True),
                "uttt.w_alpha": nn.Linear(d, 1, bias=True),
            }
            with torch.no_grad():
                mods["uttt.w_eta"].weight.zero_()
                mods["uttt.w_eta"].bias.fill_(0.0)
                mods["uttt.w_alpha"].weight.zero_()
                mods["uttt.w_alpha"].bias.fill_(-1.386)
            layers.append(mods)
        lm_head = nn.Linear(d, V, bias=False)
        with torch.no_grad():
            emb.weight.normal_(0.0, 0.02)
            for mods in layers:
                for name in ("attn.wq", "attn.wk", "attn.wv", "attn.wo", "uttt.w_q", "uttt.w_k", "uttt.w_v",
                             "uttt.w_o"):
                    mods[name].weight.normal_(0.0, 0.02)
            lm_head.weight.normal_(0.0, 0.02)
    finally:
        torch.random.set_rng_state(gen_state)
    sd: Dict[str, torch.Tensor] = {"tok_embeddings.weight": emb.weight.detach().clone()}
    sd["fast_weight_pool.w_up_init"] = w_up
    sd["fast_weight_pool.w_gate_init"] = w_gate
    sd["fast_weight_pool.w_down_init"] = w_down
    sd["fast_weight_pool.ln_weight"] = torch.ones(d)
    sd["fast_weight_pool.ln_bias"] = torch.zeros(d)
    for i, mods in enumerate(layers):
        p = f"layers.{i}."
        sd[p + "attn_norm.weight"] = torch.ones(d)
        sd[p + "uttt_norm.weight"] = torch.ones(d)
        sd[p + "uttt.q_norm.weight"] = torch.ones(d)
        sd[p + "uttt.k_norm.weight"] = torch.ones(d)
        for name, mod in mods.items():
            sd[p + name + ".weight"] = mod.weight.detach().clone()
            if mod.bias is not None:
                sd[p + name + ".bias"] = mod.bias.detach().clone()
    sd["norm.weight"] = torch.ones(d)
    sd["lm_head.weight"] = sd["tok_embeddings.weight"]     # tied (model/uttt_model.py:337-338)
    return sd


def random_state_dict(cfg: ModelConfig, seed: int = 0, device="cuda") -> Dict[str, torch.Tensor]:
    """A randomly initialised model of ``cfg``'s architecture, generated on ``device``:
    the reference's init distributions (embeddings and projections N(0, 0.02), the
    eta / alpha gates at their init values, W_0 as SharedFastWeightPool draws it,
    model/uttt_layer.py:573-580, 1269-1273) but not its RNG stream, so large
    configurations initialise in seconds.  Projections are BF16, the rest FP32."""
    d, h, V, L, hd = cfg.d_model, cfg.d_ff_fast, cfg.vocab_size, cfg.n_layers, cfg.head_dim
    g = torch.Generator(device=device).manual_seed(seed)

    def normal(*shape, std=0.02, dtype=torch.bfloat16):
        return (torch.randn(shape, generator=g, device=device) * std).to(dtype)

    sd: Dict[str, torch.Tensor] = {"tok_embeddings.weight": normal(V, d)}
    sd["fast_weight_pool.w_up_init"] = normal(d, h, std=1.0 / math.sqrt(d), dtype=torch.float32)
    sd["fast_weight_pool.w_gate_init"] = normal(d, h, std=1.0 / math.sqrt(d), dtype=torch.float32)
    sd["fast_weight_pool.w_down_init"] = normal(h, d, std=0.1 / math.sqrt(h), dtype=torch.float32)
    sd["fast_weight_pool.ln_weight"] = torch.ones(d, device=device)
    sd["fast_weight_pool.ln_bias"] = torch.zeros(d, device=device)
    for i in range(L):
        p = f"layers.{i}."
        for n in ("attn_norm", "uttt_norm", "uttt.q_norm", "uttt.k_norm"):
            sd[p + n + ".weight"] = torch.ones(d, device=device)
        sd[p + "attn.wq.weight"] = normal(cfg.n_heads * hd, d)
        sd[p + "attn.wk.weight"] = normal(cfg.n_kv_heads * hd, d)
        sd[p + "attn.wv.weight"] = normal(cfg.n_kv_heads * hd, d)
        sd[p + "attn.wo.weight"] = normal(d, cfg.n_heads * hd)
        for n in ("w_q", "w_k", "w_v", "w_o"):
            sd[p + f"uttt.{n}.weight"] = normal(d, d)
        sd[p + "uttt.w_eta.weight"] = torch.zeros(1, d, dtype=torch.bfloat16, device=device)
        sd[p + "uttt.w_eta.bias"] = torch.zeros(1, device=device)
        sd[p + "uttt.w_alpha.weight"] = torch.zeros(1, d, dtype=torch.bfloat16, device=device)
        sd[p + "uttt.w_alpha.bias"] = torch.full((1,), -1.386, device=device)
    sd["norm.weight"] = torch.ones(d, device=device)
    sd["lm_head.weight"] = sd["tok_embeddings.weight"]     # tied (model/uttt_model.py:337-338)
    return sd


def perturbed_persona_states(w_up0, w_gate0, w_down0, n: int, std: float = 1e-3, seed: int = 0,
                             device="cuda"):
    """Persona states W_0 + N(0, std) (BASELINE configs 3/4), FP32 (n, d, h) / (n, h, d)."""
    g = torch.Generator(device=device).manual_seed(seed)
    out = []
    for w in (w_up0, w_gate0, w_down0):
        w = w.to(device=device, dtype=torch.float32)
        out.append((w.unsqueeze(0) + std * torch.randn((n, *w.shape), generator=g, device=device)).contiguous())
    return out
