"""The attention entry point that allocates nothing (mie_attn_decode_fixed_scratch).

Some callers of this library cannot allocate device memory.  One example is a
host runtime that owns all device memory and gives its plugins no allocator.
Another is a latency-critical caller that must not call cudaMalloc or
cudaFree, because those calls can synchronise the device.  For them,
mie_attn_decode_fixed_scratch keeps the split-K partials and merge counters in
one fixed array inside libmie.so (64 counters + 65,536 floats).

These tests call it through the C ABI and require its output to equal
mie_attn_decode's (the entry point with caller-provided scratch) on the same
inputs, on two calls in a row (the second call reuses the array the first one
left behind).  Both entry points launch the same kernel with the same splits and
the same merge order, so the outputs must be bitwise identical: a tolerance
could hide a wrong partials stride.  A request larger than the array, or one
that asks for a deferred merge, must be refused before anything is launched,
and a malformed request gets the same error as from mie_attn_decode.  This file
is named so that pytest collects it last.
"""

import ctypes
import math

import pytest
import torch

from moe_engine import capi, paged_attention
from moe_engine.model import BlockAllocator, ModelConfig
from tests.golden import make_golden as mg

pytestmark = pytest.mark.gpu
DEV = "cuda"


def paged_inputs(dtype, H=12, hd=64, bs=16, ctx=700, seed=5):
    free, k, v, q, nb = mg.attention_inputs(H, hd, bs, ctx, 1024, seed, True)
    cfg = ModelConfig(max_seq_length=1024, vocab_size=96, num_layers=1, hidden_dim=H * hd, num_heads=H)
    alloc = BlockAllocator(cfg, nb, bs, DEV, dtype)
    alloc.free_blocks = list(free)
    cache = alloc.new_cache()
    cache.write(0, 0, k.to(DEV, dtype), v.to(DEV, dtype))
    cache.position = ctx
    return cache, q.to(DEV, dtype)[0, :, 0].contiguous(), ctx


def attn_args(cache, q, ctx, out, splits, partials=None, counters=None):
    k, v = cache.allocator.k_pool[0], cache.allocator.v_pool[0]
    nb, H, bs, hd = k.shape
    a = capi.AttnArgs()
    a.kv_dtype = a.q_dtype = a.out_dtype = capi.dtype_code(k.dtype)
    a.num_heads, a.head_dim = H, hd
    a.q, a.k, a.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    a.block_table = cache.block_table_device.data_ptr()
    a.num_blocks, a.block_size = nb, bs
    a.stride_block, a.stride_head, a.stride_tok = H * bs * hd, bs * hd, hd
    a.ctx_len, a.max_ctx = ctx, len(cache.block_table) * bs
    a.scale = 1.0 / math.sqrt(hd)
    a.out = out.data_ptr()
    a.partials = capi.ptr(partials)
    a.counters = capi.ptr(counters)
    a.splits = splits
    a.max_splits = paged_attention.MAX_SPLITS
    return a


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fixed_scratch_matches_allocating_entry_point_twice(dtype):
    lib = capi.ensure_init(torch.device(DEV))
    cache, q, ctx = paged_inputs(dtype)
    H, hd = q.shape
    splits = paged_attention.choose_splits(H, -(-ctx // 16), lib.mie_num_sms(0))
    assert splits > 1  # the partials / merge path is exercised
    stream = capi.stream_handle(torch.device(DEV))

    partials = torch.zeros(H * paged_attention.MAX_SPLITS * (hd + 2), dtype=torch.float32, device=DEV)
    counters = torch.zeros(H, dtype=torch.int32, device=DEV)
    want = torch.empty(H, hd, dtype=dtype, device=DEV)
    capi.check(lib.mie_attn_decode(ctypes.byref(attn_args(cache, q, ctx, want, splits, partials, counters)), stream),
               "mie_attn_decode")

    for call in range(2):
        got = torch.full((H, hd), float("nan"), dtype=dtype, device=DEV)
        a = attn_args(cache, q, ctx, got, splits)  # no scratch pointers passed
        capi.check(lib.mie_attn_decode_fixed_scratch(ctypes.byref(a), stream), "mie_attn_decode_fixed_scratch")
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"call {call}: max |diff| {float((got.float() - want.float()).abs().max())}"


def test_fixed_scratch_refuses_requests_beyond_its_size():
    lib = capi.ensure_init(torch.device(DEV))
    cache, q, ctx = paged_inputs(torch.float32, ctx=64)
    H, hd = q.shape
    out = torch.zeros(H, hd, device=DEV)
    a = attn_args(cache, q, ctx, out, splits=2)
    a.num_heads = 65  # more heads than the array has counters
    assert lib.mie_attn_decode_fixed_scratch(ctypes.byref(a), capi.stream_handle(torch.device(DEV))) == \
        capi.MIE_ERR_SCRATCH_LIMIT
    a = attn_args(cache, q, ctx, out, splits=83)  # 12 x 83 x 66 = 65,736 floats > 65,536
    assert lib.mie_attn_decode_fixed_scratch(ctypes.byref(a), capi.stream_handle(torch.device(DEV))) == \
        capi.MIE_ERR_SCRATCH_LIMIT
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0  # nothing was launched
    assert b"fixed scratch" in lib.mie_status_string(capi.MIE_ERR_SCRATCH_LIMIT)


def test_fixed_scratch_refuses_deferred_merge_and_malformed_requests():
    lib = capi.ensure_init(torch.device(DEV))
    cache, q, ctx = paged_inputs(torch.float32, ctx=64)
    H, hd = q.shape
    stream = capi.stream_handle(torch.device(DEV))
    out = torch.zeros(H, hd, device=DEV)
    a = attn_args(cache, q, ctx, out, splits=2)
    a.defer_merge = 1  # partials would stay in the library's array
    assert lib.mie_attn_decode_fixed_scratch(ctypes.byref(a), stream) == capi.MIE_ERR_INVALID
    a = attn_args(cache, q, ctx, out, splits=2)
    a.q = None  # malformed: the same error as the allocating entry point, not a size error
    assert lib.mie_attn_decode_fixed_scratch(ctypes.byref(a), stream) == capi.MIE_ERR_INVALID
    a = attn_args(cache, q, ctx, out, splits=2)
    a.head_dim = 48  # unsupported head size
    assert lib.mie_attn_decode_fixed_scratch(ctypes.byref(a), stream) == capi.MIE_ERR_UNSUPPORTED
    a = attn_args(cache, q, ctx, out, splits=2)
    a.num_heads, a.q = 65, None  # malformed AND beyond the array: the request check comes first
    assert lib.mie_attn_decode_fixed_scratch(ctypes.byref(a), stream) == capi.MIE_ERR_INVALID
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0  # nothing was launched
