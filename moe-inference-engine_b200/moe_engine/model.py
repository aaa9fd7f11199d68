"""Inference-only miniMoE with external KV caches, B200 decode path.

Mirror of the reference engine's ``src/moe_engine/model.py``: the same
classes, method names, arguments, cache layouts (contiguous
``[layer, batch, head, seq, head_dim]``; paged pools
``[layer, num_blocks, head, block_size, head_dim]`` with a Python block table
and its int32 device mirror), mode switches (``--moe reference|direct|auto``,
``attention_mode auto|direct|gather``) and error behaviour.  Parameter names
match the reference checkpoints for the reference architecture.

What is new:

* architecture switches on :class:`ModelConfig` (``norm``, ``pos``,
  ``expert_act``, ``bias``, ``expert_hidden_dim``, ``rope_base``,
  ``norm_eps``); the defaults are the reference architecture and
  :func:`baseline_config` gives the BASELINE one (RMSNorm, RoPE, SwiGLU);
* decode steps run as one fused launch sequence of hand-written sm_100a
  kernels (:mod:`moe_engine.decode`), and greedy ``generate`` replays that
  step as a CUDA graph with device-resident position, token and EOS state;
* contiguous caches get the direct attention kernel too (``KVCache`` has an
  ``attention_mode``; ``"gather"`` keeps the PyTorch SDPA path);
* top-k routing in the PyTorch path breaks ties toward the lower expert id.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import nn
from torch.nn import functional as F

from . import fused_moe, paged_attention

EOS_TOKEN_ID = 50256

_NORMS = ("layer", "rms")
_POSITIONS = ("learned", "rope")
_ACTS = ("gelu", "swiglu")


@dataclass
class ModelConfig:
    """Hyperparameters (model.py:18-27) plus architecture switches."""

    max_seq_length: int = 1024
    vocab_size: int = 50304
    num_layers: int = 6
    hidden_dim: int = 768
    moe_multiplier: float = 0.01  # Retained for checkpoint compatibility.
    num_experts: int = 8
    top_k: int = 2
    num_heads: int = 8
    norm: str = "layer"  # "layer" (reference) | "rms"
    pos: str = "learned"  # "learned" (reference) | "rope"
    expert_act: str = "gelu"  # "gelu" (reference, biased) | "swiglu" (bias-free)
    expert_hidden_dim: int | None = None  # None: 4*hidden for gelu, hidden for swiglu
    bias: bool = True  # QKV / out_proj / LM-head biases (reference: True)
    rope_base: float = 10000.0
    norm_eps: float = 1e-5

    def __post_init__(self):
        if self.norm not in _NORMS:
            raise ValueError(f"unknown norm {self.norm!r}")
        if self.pos not in _POSITIONS:
            raise ValueError(f"unknown pos {self.pos!r}")
        if self.expert_act not in _ACTS:
            raise ValueError(f"unknown expert_act {self.expert_act!r}")

    @property
    def expert_hidden(self) -> int:
        if self.expert_hidden_dim is not None:
            return self.expert_hidden_dim
        return 4 * self.hidden_dim if self.expert_act == "gelu" else self.hidden_dim

    @property
    def head_dim(self) -> int:
        return self.hidden_dim // self.num_heads


def baseline_config(**overrides) -> ModelConfig:
    """The BASELINE miniMoE-shaped architecture (12 x 768, 12 heads x 64,
    RMSNorm, RoPE base 10000, 8 SwiGLU experts of hidden 768, top-2, tied
    bias-free LM head, context 1536)."""
    cfg = dict(
        max_seq_length=1536,
        vocab_size=50304,
        num_layers=12,
        hidden_dim=768,
        num_experts=8,
        top_k=2,
        num_heads=12,
        norm="rms",
        pos="rope",
        expert_act="swiglu",
        expert_hidden_dim=768,
        bias=False,
    )
    cfg.update(overrides)
    return ModelConfig(**cfg)


class RMSNorm(nn.Module):
    """x * rsqrt(mean(x^2) + eps) * weight, computed in float32."""

    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight.float()
        return y.to(x.dtype)


def _make_norm(config: ModelConfig) -> nn.Module:
    if config.norm == "rms":
        return RMSNorm(config.hidden_dim, config.norm_eps)
    return nn.LayerNorm(config.hidden_dim, eps=config.norm_eps)


def rope_tables(max_pos: int, head_dim: int, base: float, device=None):
    """cos/sin [max_pos, head_dim/2]: angles p * base^(-2i/hd) in float64, stored fp32."""
    half = head_dim // 2
    inv = base ** (-(torch.arange(half, dtype=torch.float64) * 2.0 / head_dim))
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cos(ang).float().to(device), torch.sin(ang).float().to(device)


def apply_rope(x, cos, sin):
    """Half-split ("rotate_half") RoPE over the last dim of x [..., T, hd]."""
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h].float(), x[..., h:].float()
    out = torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1)
    return out.to(x.dtype)


def topk_lower_index(logits: torch.Tensor, k: int):
    """Top-k by repeated argmax over the last dim; ties -> lower index.

    ``torch.topk`` gives no tie guarantee on every device; the kernel and the
    reference's Triton router take the lower id (fused_moe.py:146-150).
    """
    work = logits.clone()
    vals, ids = [], []
    for _ in range(k):
        i = work.argmax(-1, keepdim=True)
        vals.append(work.gather(-1, i))
        ids.append(i)
        work = work.scatter(-1, i, float("-inf"))
    return torch.cat(vals, -1), torch.cat(ids, -1)


class KVCache:
    """Contiguous K/V storage shaped [layer, batch, head, sequence, head_dim].

    ``position`` is the number of cached tokens.  ``attention_mode`` selects
    decode attention: "auto" (direct kernel where supported, else SDPA),
    "direct" (kernel or error) or "gather" (PyTorch SDPA, the reference path).
    """

    def __init__(self, config: ModelConfig, batch_size: int, device, dtype=torch.float32, attention_mode="auto"):
        if attention_mode not in ("auto", "direct", "gather"):
            raise ValueError(f"unknown attention_mode {attention_mode!r}")
        head_dim = config.hidden_dim // config.num_heads
        shape = (config.num_layers, batch_size, config.num_heads, config.max_seq_length, head_dim)
        self.k = torch.zeros(shape, device=device, dtype=dtype)
        self.v = torch.zeros(shape, device=device, dtype=dtype)
        self.position = 0
        self.attention_mode = attention_mode

    def write(self, layer_idx, position, k, v):
        seq_len = k.shape[2]
        self.k[layer_idx, :, :, position : position + seq_len] = k
        self.v[layer_idx, :, :, position : position + seq_len] = v

    def read(self, layer_idx, length):
        return self.k[layer_idx, :, :, :length], self.v[layer_idx, :, :, :length]

    def reserve(self, num_tokens: int) -> None:
        """Contiguous storage is preallocated; nothing to reserve."""


class BlockAllocator:
    """Shared K/V block storage for paged sequence caches (model.py:61-105)."""

    def __init__(
        self,
        config: ModelConfig,
        num_blocks: int,
        block_size: int,
        device,
        dtype=torch.float32,
        attention_mode: str = "auto",
    ):
        # "gather": rebuild contiguous K/V then PyTorch attention (oracle path);
        # "direct": require the sm_100a kernel that reads blocks in place;
        # "auto": direct when supported, else gather.
        if attention_mode not in ("auto", "direct", "gather"):
            raise ValueError(f"unknown attention_mode {attention_mode!r}")
        self.attention_mode = attention_mode
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_heads = config.num_heads
        self.head_dim = config.hidden_dim // config.num_heads
        shape = (config.num_layers, num_blocks, config.num_heads, block_size, self.head_dim)
        self.k_pool = torch.zeros(shape, device=device, dtype=dtype)
        self.v_pool = torch.zeros(shape, device=device, dtype=dtype)
        self.free_blocks = list(range(num_blocks))

    def allocate(self) -> int:
        if not self.free_blocks:
            raise RuntimeError("no free KV cache blocks left")
        return self.free_blocks.pop()

    def free(self, block_ids: list[int]) -> None:
        self.free_blocks.extend(block_ids)

    def new_cache(self) -> "PagedKVCache":
        return PagedKVCache(self)


class PagedKVCache:
    """Per-sequence K/V cache backed by blocks from a shared allocator (model.py:108-208)."""

    def __init__(self, allocator: BlockAllocator):
        self.allocator = allocator
        self.attention_mode = allocator.attention_mode
        self.block_table: list[int] = []
        self.position = 0
        # Device mirror of block_table (int32); only the first
        # len(block_table) entries are meaningful.  Appended incrementally.
        self.block_table_device = torch.zeros(
            allocator.num_blocks, dtype=torch.int32, device=allocator.k_pool.device
        )
        self._write_index_key = None

    def _reserve(self, num_tokens: int) -> None:
        """Reserve blocks for ``num_tokens`` without partial allocation (model.py:125-143)."""
        blocks_needed = -(-num_tokens // self.allocator.block_size)
        taken: list[int] = []
        try:
            while len(self.block_table) + len(taken) < blocks_needed:
                taken.append(self.allocator.allocate())
        except RuntimeError:
            self.allocator.free(taken)
            raise
        if taken:
            start = len(self.block_table)
            self.block_table.extend(taken)
            self.block_table_device[start : start + len(taken)] = torch.tensor(
                taken, dtype=torch.int32, device=self.block_table_device.device
            )

    reserve = _reserve

    def _trim(self, num_tokens: int) -> None:
        """Return blocks beyond those ``num_tokens`` need (after run-ahead reservation)."""
        keep = -(-num_tokens // self.allocator.block_size)
        if len(self.block_table) > keep:
            extra = self.block_table[keep:]
            del self.block_table[keep:]
            self.allocator.free(extra)

    def _block_for(self, token_pos: int) -> tuple[int, int]:
        block_size = self.allocator.block_size
        return self.block_table[token_pos // block_size], token_pos % block_size

    def _write_indices(self, position, seq_len):
        """Physical (block, slot) index tensors for a multi-token write."""
        if self._write_index_key != (position, seq_len):
            block_size = self.allocator.block_size
            pos = torch.arange(position, position + seq_len, device=self.block_table_device.device)
            self._write_index = (self.block_table_device[pos // block_size].long(), pos % block_size)
            self._write_index_key = (position, seq_len)
        return self._write_index

    def write(self, layer_idx, position, k, v):
        if k.shape[0] != 1:
            raise ValueError("PagedKVCache holds one sequence; use batch size 1")
        seq_len = k.shape[2]
        self._reserve(position + seq_len)
        if seq_len == 1:
            block_id, slot = self._block_for(position)
            self.allocator.k_pool[layer_idx, block_id, :, slot] = k[0, :, 0]
            self.allocator.v_pool[layer_idx, block_id, :, slot] = v[0, :, 0]
            return
        blocks, slots = self._write_indices(position, seq_len)
        self.allocator.k_pool[layer_idx, blocks, :, slots] = k[0].transpose(0, 1)
        self.allocator.v_pool[layer_idx, blocks, :, slots] = v[0].transpose(0, 1)

    def read(self, layer_idx, length):
        block_size = self.allocator.block_size
        num_blocks = -(-length // block_size)
        block_ids = self.block_table[:num_blocks]

        def read_pool(pool):
            return (
                pool[layer_idx, block_ids]
                .transpose(0, 1)
                .reshape(self.allocator.num_heads, -1, self.allocator.head_dim)[:, :length]
                .unsqueeze(0)
            )

        return read_pool(self.allocator.k_pool), read_pool(self.allocator.v_pool)

    def free(self):
        """Return all blocks and reset the cache."""
        self.allocator.free(self.block_table)
        self.block_table = []
        self.position = 0
        self._write_index_key = None


def attention_kernel_usable(cache, x: torch.Tensor, head_dim: int) -> bool:
    """Whether decode attention for ``cache`` can run on the direct kernel."""
    mode = getattr(cache, "attention_mode", "gather")
    return (
        mode != "gather"
        and paged_attention.is_supported(x)
        and head_dim in paged_attention.SUPPORTED_HEAD_DIMS
        and cache_dtype(cache) == x.dtype
    )


def cache_dtype(cache) -> torch.dtype:
    return cache.allocator.k_pool.dtype if hasattr(cache, "allocator") else cache.k.dtype


class CachedAttention(nn.Module):
    """Causal self-attention with external K/V storage (model.py:211-269)."""

    def __init__(self, dim: int, num_heads: int, bias: bool = True):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.in_proj_weight = nn.Parameter(torch.empty(3 * dim, dim))
        if bias:
            self.in_proj_bias = nn.Parameter(torch.empty(3 * dim))
        else:
            self.register_parameter("in_proj_bias", None)
        self.out_proj = nn.Linear(dim, dim, bias=bias)
        nn.init.xavier_uniform_(self.in_proj_weight)
        if bias:
            nn.init.zeros_(self.in_proj_bias)

    def forward(self, x, cache, layer_idx, position: int, rope=None):
        batch, seq_len, dim = x.shape
        q, k, v = F.linear(x, self.in_proj_weight, self.in_proj_bias).chunk(3, dim=-1)

        def split_heads(t):
            return t.view(batch, seq_len, self.num_heads, self.head_dim).transpose(1, 2)

        q, k, v = split_heads(q), split_heads(k), split_heads(v)
        if rope is not None:
            cos, sin = rope[0][position : position + seq_len], rope[1][position : position + seq_len]
            q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)

        # A forced 'direct' that cannot run must fail before the write below.
        mode = getattr(cache, "attention_mode", "gather")
        use_kernel = attention_kernel_usable(cache, x, self.head_dim)
        if mode == "direct" and not use_kernel:
            raise RuntimeError(
                "attention_mode='direct' needs CUDA, libmie.so, float32/bfloat16 and a supported head_dim; "
                "use 'auto' for automatic fallback or 'gather' for the oracle path"
            )

        cache.write(layer_idx, position, k, v)
        assert position == 0 or seq_len == 1, "prefill must start at position 0"

        if mode != "gather" and position == 0:
            # Prefill fast path: at position 0 the history is exactly k, v.
            out = F.scaled_dot_product_attention(q, k, v, is_causal=seq_len > 1)
        elif use_kernel:
            out = paged_attention.decode(q, cache, layer_idx, context_len=position + 1)
        else:
            keys, values = cache.read(layer_idx, position + seq_len)
            out = F.scaled_dot_product_attention(q, keys, values, is_causal=seq_len > 1)

        out = out.transpose(1, 2).reshape(batch, seq_len, dim)
        return self.out_proj(out)


class Expert(nn.Module):
    """Reference GELU expert (model.py:272-282) or a bias-free SwiGLU expert."""

    def __init__(self, dim, hidden_dim, activation: str = "gelu"):
        super().__init__()
        self.activation = activation
        if activation == "gelu":
            self.net = nn.Sequential(nn.Linear(dim, hidden_dim), nn.GELU(), nn.Linear(hidden_dim, dim))
        else:
            self.gate = nn.Linear(dim, hidden_dim, bias=False)
            self.up = nn.Linear(dim, hidden_dim, bias=False)
            self.down = nn.Linear(hidden_dim, dim, bias=False)

    def forward(self, x):
        if self.activation == "gelu":
            return self.net(x)
        return self.down(F.silu(self.gate(x)) * self.up(x))


def _gelu_groups():
    return {"w1": (lambda e: e.net[0], "weight"), "b1": (lambda e: e.net[0], "bias"),
            "w2": (lambda e: e.net[2], "weight"), "b2": (lambda e: e.net[2], "bias")}


def _swiglu_groups():
    return {"w1": (lambda e: e.gate, "weight"), "w3": (lambda e: e.up, "weight"),
            "w2": (lambda e: e.down, "weight")}


class MoEFeedForward(nn.Module):
    """PyTorch MoE oracle plus fused sm_100a decode dispatch (model.py:285-481)."""

    def __init__(self, dim, hidden_dim, num_experts, top_k, mode="auto", activation="gelu"):
        super().__init__()
        if mode not in ("auto", "direct", "reference"):
            raise ValueError(f"unknown MoE mode {mode!r}")
        self.mode = mode
        self.dim = dim
        self.hidden_dim = hidden_dim
        self.top_k = top_k
        self.num_experts = num_experts
        self.activation = activation
        self.experts = nn.ModuleList(Expert(dim, hidden_dim, activation) for _ in range(num_experts))
        self.router = nn.Linear(dim, num_experts, bias=False)
        self._make_workspaces(self.router.weight.device, self.router.weight.dtype)
        # Re-home the per-expert parameters into canonical contiguous storages
        # (one [E, ...] tensor per group) while keeping every state-dict name as
        # a non-overlapping Parameter view; the kernel selects expert e by a
        # device-side offset.
        self._pack_expert_parameters()
        self.register_load_state_dict_post_hook(self._repack_after_load)

    def _make_workspaces(self, device, dtype):
        # Fixed per-layer workspaces; they never alter checkpoint keys/values.
        def buf(name, t):
            if name in self._buffers:
                self._buffers[name] = t
            else:
                self.register_buffer(name, t, persistent=False)

        buf("_router_logits", torch.empty(self.num_experts, dtype=torch.float32, device=device))
        buf("_expert_ids", torch.empty(self.top_k, dtype=torch.int32, device=device))
        buf("_route_weights", torch.empty(self.top_k, dtype=torch.float32, device=device))
        buf("_expert_hidden", torch.empty(self.top_k, self.hidden_dim, dtype=torch.float32, device=device))
        buf("_direct_out", torch.empty(self.dim, dtype=dtype, device=device))
        buf("_sync", torch.zeros(4, dtype=torch.int32, device=device))

    def _groups(self):
        return _gelu_groups() if self.activation == "gelu" else _swiglu_groups()

    def _pack_parameter_group(self, getter, parameter_name: str) -> torch.Tensor:
        parameters = [getattr(getter(expert), parameter_name) for expert in self.experts]
        shape = parameters[0].shape
        if any(p.shape != shape for p in parameters):
            raise ValueError("all experts must have identical parameter shapes")
        packed = torch.empty((self.num_experts, *shape), device=parameters[0].device, dtype=parameters[0].dtype)
        with torch.no_grad():
            for expert_id, parameter in enumerate(parameters):
                packed[expert_id].copy_(parameter)
                setattr(
                    getter(self.experts[expert_id]),
                    parameter_name,
                    nn.Parameter(packed[expert_id], requires_grad=parameter.requires_grad),
                )
        return packed

    def _pack_expert_parameters(self) -> None:
        self._expert_storage = {name: self._pack_parameter_group(g, p) for name, (g, p) in self._groups().items()}

    def _repack_after_load(self, _module, _incompatible_keys) -> None:
        self._pack_expert_parameters()
        self._quant = None  # loaded weights replace any quantized copy

    def _apply(self, fn, recurse=True):
        result = super()._apply(fn, recurse=recurse)
        self._pack_expert_parameters()
        w = self.router.weight
        self._make_workspaces(w.device, w.dtype)
        if getattr(self, "_quant", None):
            self._quant = {name: q.to(w.device) for name, q in self._quant.items()}
        return result

    def quantize_experts(self, bits: int = 8, group_size: int = 128) -> None:
        """Quantize the expert weights groupwise (int8 or int4, see
        ``fused_moe.quantize_experts``).  The decode kernel then reads the
        quantized values; the expert parameters are overwritten with the
        weights those values stand for, so the prefill, the reference mode and
        the decode all compute with the same effective weights."""
        s = self._expert_storage
        quant = {name: fused_moe.quantize_experts(s[name], bits, group_size) for name in ("w1", "w3", "w2")
                 if name in s}
        with torch.no_grad():
            for name, q in quant.items():
                s[name].copy_(fused_moe.dequantize_experts(q).to(s[name].dtype))
        self._quant = quant

    @property
    def quantized(self) -> bool:
        return bool(getattr(self, "_quant", None))

    def set_mode(self, mode: str) -> None:
        if mode not in ("auto", "direct", "reference"):
            raise ValueError(f"unknown MoE mode {mode!r}")
        self.mode = mode

    def _direct_supported(self, x: torch.Tensor) -> bool:
        return (
            fused_moe.is_supported(
                x, num_experts=self.num_experts, top_k=self.top_k, expert_hidden_dim=self.hidden_dim
            )
            and x.dtype == self.router.weight.dtype
            and self._has_direct_layout()
        )

    def _has_direct_layout(self) -> bool:
        s = self._expert_storage
        return fused_moe.has_canonical_layout(
            self.router.weight, s["w1"], s.get("b1"), s["w2"], s.get("b2"), self._router_logits,
            self._expert_ids, self._route_weights, self._expert_hidden, self._direct_out, s.get("w3"),
        )

    def direct_configuration_supported(self, batch_size: int) -> bool:
        router = self.router.weight
        return (
            fused_moe.is_configuration_supported(
                device=router.device,
                dtype=router.dtype,
                batch_size=batch_size,
                hidden_dim=self.dim,
                num_experts=self.num_experts,
                top_k=self.top_k,
                expert_hidden_dim=self.hidden_dim,
            )
            and self._has_direct_layout()
        )

    def preflight_direct_decode(self, *, batch_size: int) -> None:
        """Reject an unsupported forced decode before any cache mutation."""
        if self.mode != "direct":
            return
        if not self.direct_configuration_supported(batch_size):
            self._raise_direct_unsupported()

    @staticmethod
    def _raise_direct_unsupported() -> None:
        raise RuntimeError(
            "MoE mode 'direct' needs one-token batch-one CUDA float32 or bfloat16 decode "
            "with a kernel-supported shape and libmie.so; use 'auto' for automatic "
            "fallback or 'reference' for the PyTorch oracle"
        )

    def uses_direct(self, x: torch.Tensor, *, decode: bool) -> bool:
        """Resolve reference/direct/auto without reading device results."""
        if not decode or self.mode == "reference":
            return False
        supported = self._direct_supported(x)
        if self.mode == "direct" and not supported:
            self._raise_direct_unsupported()
        return supported

    def _forward_reference(self, x: torch.Tensor) -> torch.Tensor:
        """Vectorised prefill and correctness oracle (model.py:443-461)."""
        batch, seq_len, dim = x.shape
        flat_x = x.reshape(-1, dim)
        with torch.autocast(device_type=x.device.type, enabled=False):
            router_logits = F.linear(flat_x.float(), self.router.weight.float())
            topk_logits, topk_indices = topk_lower_index(router_logits, self.top_k)
            topk_weights = F.softmax(topk_logits, dim=-1)
        out = torch.zeros_like(flat_x)
        for expert_id, expert in enumerate(self.experts):
            token_ids, slot = torch.where(topk_indices == expert_id)
            if token_ids.numel() == 0:
                continue
            weight = topk_weights[token_ids, slot].unsqueeze(-1).to(flat_x.dtype)
            out.index_add_(0, token_ids, weight * expert(flat_x[token_ids]))
        return out.reshape(batch, seq_len, dim)

    def _forward_direct(self, x: torch.Tensor) -> torch.Tensor:
        s = dict(self._expert_storage)
        if self.quantized:
            s.update(self._quant)
        return fused_moe.decode(
            x,
            self.router.weight,
            s["w1"],
            s.get("b1"),
            s["w2"],
            s.get("b2"),
            router_logits=self._router_logits,
            expert_ids=self._expert_ids,
            route_weights=self._route_weights,
            hidden=self._expert_hidden,
            out=self._direct_out,
            w3_base=s.get("w3"),
            sync=self._sync,
        )

    def forward(self, x, *, decode=False):
        if self.uses_direct(x, decode=decode):
            return self._forward_direct(x)
        return self._forward_reference(x)


class TransformerMoEBlock(nn.Module):
    def __init__(self, config: ModelConfig):
        super().__init__()
        self.attention = CachedAttention(config.hidden_dim, config.num_heads, bias=config.bias)
        self.moe = MoEFeedForward(
            config.hidden_dim, config.expert_hidden, config.num_experts, config.top_k,
            activation=config.expert_act,
        )
        self.attn_norm = _make_norm(config)
        self.moe_norm = _make_norm(config)

    def forward(self, x, cache, layer_idx, position, rope=None):
        x = x + self.attention(self.attn_norm(x), cache, layer_idx, position, rope=rope)
        normed = self.moe_norm(x)
        x = x + self.moe(normed, decode=position > 0 and normed.shape[1] == 1)
        return x


@torch.no_grad()
def random_init_(model: "Model", seed: int = 0) -> "Model":
    """Seeded random weights on the model's device: every matrix N(0, 0.02)
    from one generator in ``named_parameters`` order, norm weights 1, ``*bias``
    parameters 0 (the BASELINE configs are random-init from seed 0; no
    checkpoint is involved)."""
    device = model.token_embedding.weight.device
    g = torch.Generator(device=device).manual_seed(seed)
    for name, p in model.named_parameters():
        if name.endswith("norm.weight"):
            p.fill_(1.0)
        elif name.endswith("bias"):
            p.zero_()
        else:
            p.copy_(torch.randn(p.shape, generator=g, device=device, dtype=torch.float32) * 0.02)
    return model


class Model(nn.Module):
    def __init__(self, config: ModelConfig):
        super().__init__()
        self.config = config
        self.max_seq_length = config.max_seq_length
        self.token_embedding = nn.Embedding(config.vocab_size, config.hidden_dim)
        if config.pos == "learned":
            self.positional_embedding = nn.Embedding(config.max_seq_length, config.hidden_dim)
        self.output_projection = nn.Linear(config.hidden_dim, config.vocab_size, bias=config.bias)
        self.MoEBlocks = nn.ModuleList(TransformerMoEBlock(config) for _ in range(config.num_layers))
        self.final_norm = _make_norm(config)
        self.output_projection.weight = self.token_embedding.weight  # Weight tying.
        self._build_rope(None)
        self._decode_runner = None

    # --- RoPE tables stay float32 whatever the model dtype -------------------
    def _build_rope(self, device):
        if self.config.pos != "rope":
            self.rope_cos = self.rope_sin = None
            return
        cos, sin = rope_tables(self.max_seq_length, self.config.head_dim, self.config.rope_base, device)
        for name, t in (("rope_cos", cos), ("rope_sin", sin)):
            if name in self._buffers:
                self._buffers[name] = t
            else:
                self.register_buffer(name, t, persistent=False)

    def _apply(self, fn, recurse=True):
        result = super()._apply(fn, recurse=recurse)
        self._build_rope(self.token_embedding.weight.device)
        self._decode_runner = None
        self._prefill_runner = None
        return result

    @property
    def rope(self):
        return None if self.config.pos != "rope" else (self.rope_cos, self.rope_sin)

    def new_cache(self, batch_size: int = 1, attention_mode: str = "auto") -> KVCache:
        """Create a cache matching the model's device and dtype."""
        weight = self.token_embedding.weight
        return KVCache(self.config, batch_size, weight.device, weight.dtype, attention_mode)

    def set_moe_mode(self, mode: str) -> "Model":
        """Set reference, forced-direct, or automatic MoE dispatch on all layers."""
        for block in self.MoEBlocks:
            block.moe.set_mode(mode)
        return self

    def quantize_experts(self, bits: int = 8, group_size: int = 128) -> "Model":
        """Groupwise int8 / int4 expert weights on every layer (the reference's
        roadmap item, moe-inference-engine.md:36).  Decode steps then run the
        per-layer operators with the quantized MoE kernel (the persistent step
        kernels take bf16 / fp32 experts only); the prefill computes with the
        weights the quantized values stand for."""
        for block in self.MoEBlocks:
            block.moe.quantize_experts(bits, group_size)
        return self

    def new_block_allocator(self, num_blocks: int, block_size: int = 16, attention_mode: str = "auto") -> BlockAllocator:
        """Create a block pool matching the model's device and dtype."""
        weight = self.token_embedding.weight
        return BlockAllocator(self.config, num_blocks, block_size, weight.device, weight.dtype, attention_mode)

    # --- fused decode ---------------------------------------------------------
    def decode_runner(self):
        """The fused-step runner of this model (created on first use)."""
        from .decode import DecodeRunner

        if self._decode_runner is None:
            self._decode_runner = DecodeRunner(self)
        return self._decode_runner

    def prefill_runner(self):
        """The tensor-core prompt prefill of this model (created on first use)."""
        from .prefill import PrefillRunner

        if getattr(self, "_prefill_runner", None) is None:
            self._prefill_runner = PrefillRunner(self)
        return self._prefill_runner

    def prefill_supported(self, cache, token_ids) -> bool:
        """Whether a prompt prefill can run on the sm_100a kernels (bf16 weights
        and cache, SwiGLU experts, no biases, MoE mode not "reference",
        attention mode not "gather")."""
        from .prefill import PrefillRunner

        return PrefillRunner.supports(self, cache, token_ids)

    def fused_decode_supported(self, cache, batch: int) -> bool:
        """Whether a one-token decode step can run as the fused kernel sequence."""
        from .decode import DecodeRunner

        return DecodeRunner.supports(self, cache, batch)

    def forward(self, token_ids, cache):
        """Run a forward pass using a contiguous or paged cache (model.py:543-565)."""
        batch, seq_len = token_ids.shape
        position = cache.position
        assert position + seq_len <= self.max_seq_length, "KV cache is full"

        # Forced direct MoE failures must occur before attention in layer zero
        # can write K/V or reserve a paged-cache block.
        if position > 0 and seq_len == 1:
            for block in self.MoEBlocks:
                block.moe.preflight_direct_decode(batch_size=batch)
            if self.fused_decode_supported(cache, batch):
                return self.decode_runner().forward_step(token_ids, cache)
        if position == 0 and seq_len > 1 and self.prefill_supported(cache, token_ids):
            return self.prefill_runner().run(token_ids, cache)

        pos = torch.arange(position, position + seq_len, device=token_ids.device)
        x = self.token_embedding(token_ids)
        if self.config.pos == "learned":
            x = x + self.positional_embedding(pos)
        rope = self.rope
        for i, block in enumerate(self.MoEBlocks):
            x = block(x, cache, i, position, rope=rope)
        cache.position += seq_len

        x = self.final_norm(x)
        return self.output_projection(x)

    @torch.no_grad()
    def generate(self, token_ids, max_new_tokens, temperature=1.0, top_k=None, cache=None):
        """Generate one sequence. The caller owns any supplied cache (model.py:567-621).

        Greedy decoding (temperature 0) on a fused-capable model and cache
        replays the decode step as a CUDA graph with the EOS check on the
        device; the returned tokens are identical to the step-by-step loop.
        """
        if not math.isfinite(temperature) or temperature < 0:
            raise ValueError("temperature must be a finite non-negative number")
        if top_k is not None and top_k <= 0:
            raise ValueError("top_k must be positive")
        if max_new_tokens < 1:
            raise ValueError("max_new_tokens must be at least 1")

        if token_ids.dim() == 1:
            token_ids = token_ids.unsqueeze(0)
        token_ids = token_ids.to(self.token_embedding.weight.device).long()
        if token_ids.shape[0] != 1:
            raise ValueError("generate() handles one sequence; use batch size 1")
        if token_ids.shape[1] == 0:
            raise ValueError("prompt must contain at least one token")
        if token_ids.shape[1] > self.max_seq_length:
            raise ValueError(
                f"prompt is {token_ids.shape[1]} tokens; max_seq_length is {self.max_seq_length}"
            )
        if cache is None:
            cache = self.new_cache(batch_size=1)
        if cache.position != 0:
            raise ValueError("generate() needs a fresh cache")

        if temperature == 0 and self.fused_decode_supported(cache, 1):
            from .decode import greedy_generate

            return greedy_generate(self, token_ids, max_new_tokens, cache)
        if (temperature > 0 and self.fused_decode_supported(cache, 1)
                and self.decode_runner().supports_sampling(cache, temperature, top_k)):
            from .decode import greedy_generate

            # sampling on the device: the step kernel draws every token after the first
            return greedy_generate(self, token_ids, max_new_tokens, cache, temperature=temperature, top_k=top_k)

        x = token_ids
        step_input = token_ids
        for _ in range(max_new_tokens):
            logits = self(step_input, cache)
            next_token_logits = logits[:, -1, :]
            if temperature == 0:
                next_token = torch.argmax(next_token_logits, dim=-1, keepdim=True)
            else:
                next_token_logits = next_token_logits.float() / temperature
                if top_k is not None:
                    sample_top_k = min(top_k, next_token_logits.size(-1))
                    values, _ = torch.topk(next_token_logits, sample_top_k)
                    next_token_logits[next_token_logits < values[:, [-1]]] = -float("inf")
                probs = F.softmax(next_token_logits, dim=-1)
                next_token = torch.multinomial(probs, num_samples=1)
            if next_token == EOS_TOKEN_ID:
                return x
            x = torch.cat((x, next_token), dim=1)
            step_input = next_token
            if cache.position >= self.max_seq_length:
                break
        return x
