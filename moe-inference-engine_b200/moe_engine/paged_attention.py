"""Direct decode attention on B200 (sm_100a), behind the reference API.

Drop-in for ``src/moe_engine/paged_attention.py`` of the reference engine:
``is_supported(x)`` and ``decode(q, cache, layer_idx, context_len)`` keep
their meaning.  The kernel (``mie_attn_decode``) splits every head's context
over several CTAs and merges the partial softmaxes with a log-sum-exp rescale
in the same launch, reading K/V in place through the block table:

    logical block  = p // block_size
    block offset   = p %  block_size
    physical block = block_table[logical block]

The same kernel serves the contiguous ``KVCache`` (an identity block map over
fixed 16-token tiles): pass a ``KVCache`` instead of a ``PagedKVCache``.
float32 and bfloat16 caches are supported; head_dim in {4, 8, 16, 32, 64, 96,
128}.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import capi

HAS_KERNELS = capi.library_available()
HAS_TRITON = HAS_KERNELS  # name used by callers of the reference module

# Tokens per contiguous-cache tile (the identity "block" of the contiguous twin).
CONTIGUOUS_TILE = 16
MAX_SPLITS = 64
SUPPORTED_HEAD_DIMS = (4, 8, 16, 32, 64, 96, 128)


def is_supported(x: torch.Tensor) -> bool:
    """The kernel path needs CUDA, libmie.so and float32/bfloat16 activations."""
    return HAS_KERNELS and x.is_cuda and x.dtype in (torch.float32, torch.bfloat16)


MIN_BLOCKS_PER_SPLIT = 8  # 128 tokens of bf16 K+V at head_dim 64: one 32 KB stage per CTA


def choose_splits(num_heads: int, num_kv_blocks: int, num_sms: int) -> int:
    """KV splits per head: at most two CTAs per SM (the kernel's shared memory
    holds two at once, so a third would run in a second wave), and at least
    MIN_BLOCKS_PER_SPLIT blocks per split, so a CTA streams a whole stage of
    K/V instead of a few kilobytes between its launch and its merge."""
    want = max(1, 2 * num_sms // num_heads)
    return max(1, min(want, -(-num_kv_blocks // MIN_BLOCKS_PER_SPLIT), MAX_SPLITS))


class _Workspace:
    """Per-device scratch for split partials and per-head merge counters."""

    _by_key: dict = {}

    @classmethod
    def get(cls, device: torch.device, num_heads: int, head_dim: int):
        key = (device.index, num_heads, head_dim)
        ws = cls._by_key.get(key)
        if ws is None:
            ws = (
                torch.empty(num_heads * MAX_SPLITS * (head_dim + 2), dtype=torch.float32, device=device),
                torch.zeros(num_heads, dtype=torch.int32, device=device),
            )
            cls._by_key[key] = ws
        return ws


def cache_geometry(cache, layer_idx: int):
    """(k_base, v_base, block_table | None, num_blocks, block_size, strides, max_ctx)."""
    if hasattr(cache, "allocator"):  # PagedKVCache: pools [L, nb, H, bs, hd]
        alloc = cache.allocator
        k, v = alloc.k_pool[layer_idx], alloc.v_pool[layer_idx]
        nb, H, bs, hd = k.shape
        if k.stride(3) != 1 or k.stride(2) != hd or k.stride(1) != bs * hd or k.stride(0) != H * bs * hd:
            raise ValueError("paged KV pool must be contiguous [num_blocks, heads, block_size, head_dim]")
        max_ctx = len(cache.block_table) * bs
        return k, v, cache.block_table_device, nb, bs, (H * bs * hd, bs * hd, hd), max_ctx
    # KVCache: [L, B, H, S, hd]
    k, v = cache.k[layer_idx], cache.v[layer_idx]
    if k.shape[0] != 1:
        raise ValueError("direct attention decodes one sequence; use batch size 1")
    k, v = k[0], v[0]
    H, S, hd = k.shape
    if not (k.is_contiguous() and v.is_contiguous()):
        raise ValueError("contiguous KV cache must be contiguous [heads, max_seq, head_dim]")
    return k, v, None, 0, CONTIGUOUS_TILE, (CONTIGUOUS_TILE * hd, S * hd, hd), S


def decode(q: torch.Tensor, cache, layer_idx: int, context_len: int, *, out: torch.Tensor | None = None):
    """Single-token attention over cached positions 0..context_len-1.

    q is [1, heads, 1, head_dim]; returns the same shape (paged_attention.py:113-154).
    ``context_len`` is a host int, so no device value is read.
    """
    k, v, table, nb, bs, (s_blk, s_head, s_tok), max_ctx = cache_geometry(cache, layer_idx)
    num_heads, head_dim = q.shape[1], q.shape[3]
    if head_dim not in SUPPORTED_HEAD_DIMS:
        raise RuntimeError(f"direct attention supports head_dim in {SUPPORTED_HEAD_DIMS}, not {head_dim}")
    if q.dtype not in (torch.float32, torch.bfloat16) or k.dtype not in (torch.float32, torch.bfloat16):
        raise RuntimeError("direct attention needs float32 or bfloat16 q and K/V")
    if not 1 <= context_len <= max_ctx:
        raise ValueError(f"context_len {context_len} outside the cache's 1..{max_ctx} tokens")
    q2 = q[0, :, 0]
    if q2.stride(1) != 1:
        q2 = q2.contiguous()
    if q2.stride(0) != head_dim:
        q2 = q2.contiguous()
    if out is None:
        out = torch.empty(num_heads, head_dim, dtype=q.dtype, device=q.device)
    lib = capi.ensure_init(q.device)
    partials, counters = _Workspace.get(q.device, num_heads, head_dim)
    nblk = -(-context_len // bs)
    a = capi.AttnArgs()
    a.kv_dtype = capi.dtype_code(k.dtype)
    a.q_dtype = capi.dtype_code(q2.dtype)
    a.out_dtype = capi.dtype_code(out.dtype)
    a.num_heads, a.head_dim = num_heads, head_dim
    a.q, a.k, a.v = q2.data_ptr(), k.data_ptr(), v.data_ptr()
    a.block_table = capi.ptr(table)
    a.num_blocks = nb
    a.block_size = bs
    a.stride_block, a.stride_head, a.stride_tok = s_blk, s_head, s_tok
    a.ctx_len = context_len
    a.max_ctx = max_ctx
    a.scale = 1.0 / math.sqrt(head_dim)
    a.out = out.data_ptr()
    a.partials, a.counters = partials.data_ptr(), counters.data_ptr()
    a.splits = choose_splits(num_heads, nblk, lib.mie_num_sms(q.device.index or 0))
    a.max_splits = MAX_SPLITS
    capi.check(lib.mie_attn_decode(ctypes.byref(a), capi.stream_handle(q.device)), "mie_attn_decode")
    return out.view(1, num_heads, 1, head_dim)
