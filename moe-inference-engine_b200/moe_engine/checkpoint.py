"""Checkpoint loading (reference: src/moe_engine/checkpoint.py:20-43).

The checkpoint format is the reference's: ``{"model": state_dict,
"model_config": dict, "step": int, "tokens_seen": int}``.
"""

from __future__ import annotations

import torch

from .model import Model, ModelConfig


def load_checkpoint(path, device):
    return torch.load(path, map_location=device, weights_only=True)


def load_engine_model(path, device, dtype=None):
    """Build the engine model from a checkpoint; returns (model, config, metadata)."""
    ckpt = load_checkpoint(path, device)
    config = ModelConfig(**ckpt["model_config"])
    model = Model(config)
    model.load_state_dict(ckpt["model"])
    model = model.to(device)
    if dtype is not None:
        model = model.to(dtype)
    model.eval()
    metadata = {"step": ckpt.get("step"), "tokens_seen": ckpt.get("tokens_seen")}
    return model, config, metadata
