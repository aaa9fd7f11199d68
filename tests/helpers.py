"""Shared test helpers: tiny configs in both architectures, weight loading."""

from __future__ import annotations

import torch

import oracle
from moe_engine.model import Model, ModelConfig

# The reference tests' TINY model (tests/test_parity.py:11 of the reference).
TINY = dict(max_seq_length=32, vocab_size=96, num_layers=2, hidden_dim=32, num_experts=4, top_k=2)

ARCHS = {
    # reference architecture: LayerNorm, learned positions, biased GELU experts (8 heads of 4)
    "reference": (
        dict(TINY),
        oracle.Arch(vocab_size=96, hidden_dim=32, num_layers=2, num_heads=8, num_experts=4, top_k=2,
                    expert_hidden_dim=128, max_seq_length=32),
    ),
    # BASELINE architecture at tiny size: RMSNorm, RoPE, SwiGLU (4 heads of 8)
    "baseline": (
        dict(TINY, num_heads=4, norm="rms", pos="rope", expert_act="swiglu", expert_hidden_dim=32, bias=False),
        oracle.Arch(vocab_size=96, hidden_dim=32, num_layers=2, num_heads=4, num_experts=4, top_k=2,
                    expert_hidden_dim=32, max_seq_length=32, norm="rms", pos="rope", expert_act="swiglu",
                    bias=False),
    ),
}


def engine_state_dict(P: dict) -> dict:
    sd = dict(P)
    sd["output_projection.weight"] = P["token_embedding.weight"]
    return sd


def make_pair(kind: str = "reference", seed: int = 0, device="cpu", dtype=torch.float32, **cfg_overrides):
    """(oracle params, oracle arch, engine model) with identical weights."""
    cfg, arch = ARCHS[kind]
    cfg = dict(cfg, **cfg_overrides)
    if cfg_overrides:
        arch = arch.with_(**{k: v for k, v in cfg_overrides.items() if hasattr(arch, k)})
    P = oracle.init_params(arch, seed=seed, bias_std=0.02 if arch.bias else 0.0, norm_std=0.1)
    model = Model(ModelConfig(**cfg)).eval()
    model.load_state_dict(engine_state_dict(P))
    model = model.to(device=device, dtype=dtype)
    return P, arch, model


def load_into(model: Model, P: dict) -> Model:
    model.load_state_dict(engine_state_dict(P))
    return model
