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


def oracle_prefill_with_margins(P: dict, arch, ids: torch.Tensor, kv_dtype=torch.bfloat16):
    """The oracle's prompt forward (as ``oracle.Decoder.forward`` from an empty
    cache) returning (logits [T, vocab], margin [T]): per position the
    smallest gap, over the layers, between the router's second and third
    logits -- below ~1e-3 a bf16 computation of the same layer may select
    another expert pair."""
    from oracle import minimoe as om

    ids = ids.long().reshape(1, -1)
    T = ids.shape[1]
    positions = torch.arange(T)
    cos = sin = None
    if arch.pos == "rope":
        cos, sin = om.rope_tables(arch.max_seq_length, arch.head_dim, arch.rope_base)
    x = om._embed(P, arch, ids, positions)
    margin = torch.full((T,), float("inf"))
    for layer in range(arch.num_layers):
        h = om.norm(x, P, f"MoEBlocks.{layer}.attn_norm", arch)
        q, k, v = om._qkv(h, P, layer, arch, positions, cos, sin)
        k, v = k.to(kv_dtype).float(), v.to(kv_dtype).float()
        x = x + om._out_proj(om.attention(q, k, v, causal=T > 1), P, layer, arch)
        h = om.norm(x, P, f"MoEBlocks.{layer}.moe_norm", arch)
        out, (logits, _, _) = om.moe_forward(h, P, layer, arch)
        top = logits.sort(dim=-1, descending=True).values
        margin = torch.minimum(margin, top[:, 1] - top[:, 2])
        x = x + out
    return om._lm_head(x, P, arch)[0], margin


def baseline_bf16_model(max_seq: int = 1536, num_layers: int = 12, seed: int = 0, device="cuda"):
    """(bf16 engine model on `device`, fp32 oracle params, oracle arch) of the
    BASELINE architecture with `num_layers` layers and context `max_seq`."""
    arch = oracle.BASELINE_ARCH.with_(max_seq_length=max_seq, num_layers=num_layers)
    P = oracle.init_params(arch, seed=seed)
    from moe_engine.model import baseline_config

    m = Model(baseline_config(max_seq_length=max_seq, num_layers=num_layers)).eval()
    m.load_state_dict(engine_state_dict(P))
    return m.to(device, torch.bfloat16), P, arch


def shuffled_paged_cache(m: Model, max_seq: int, shuffle_seed: int = 0):
    """A fresh paged cache (block 16, direct attention) whose free list is
    shuffled, so logical blocks map to scattered physical blocks."""
    import random

    alloc = m.new_block_allocator(num_blocks=-(-max_seq // 16) + 8, block_size=16, attention_mode="direct")
    free = list(alloc.free_blocks)
    random.Random(shuffle_seed).shuffle(free)
    alloc.free_blocks = free
    return alloc.new_cache()
