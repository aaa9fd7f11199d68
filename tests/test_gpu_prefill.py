"""Prompt prefill on the sm_100a kernels (moe_engine/prefill.py: tcgen05 GEMMs,
per-token norm / RoPE / routing / combine kernels, SDPA for the causal
attention) against the CPU oracle and against the PyTorch module path.

* logits of the prompt positions against the oracle run on the same
  bf16-rounded weights with a bf16 K/V cache (relative error, Frobenius over
  the vocabulary): within 2e-2 (the bf16 decode step's tolerance) at every
  position whose router margins are clear (second minus third logit above
  5e-3 in every layer), median below 1e-2 over all positions.  The GEMM
  operands are bf16, so router logits move by ~1e-3; where the oracle's second
  and third logits lie closer than that (measured at a 40-token prompt:
  margins of 3e-4 to 3e-3 at 4 of 480 routing decisions) the token takes
  another expert and its logits move by ~7 % (BASELINE) -- not a defect of
  the kernels but of comparing discrete choices at a tie;
* the K/V cache the prefill writes equals the module path's: layer 0
  elementwise within 2e-2 (bf16 rounding of differently ordered fp32 sums; the
  module path also rounds q / k to bf16 before RoPE), every layer for at least
  95 % of the elements (later layers inherit the routing differences above);
* paged and contiguous caches give identical logits and cache contents;
* "reference" MoE mode and "gather" attention keep the module path.
"""

import pytest
import torch

import oracle
from moe_engine.model import Model, baseline_config
from tests.helpers import engine_state_dict, oracle_prefill_with_margins

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def params():
    return oracle.init_params(oracle.BASELINE_ARCH, seed=0)


@pytest.fixture(scope="module")
def model(params):
    m = Model(baseline_config()).eval()
    m.load_state_dict(engine_state_dict(params))
    return m.to(DEV, torch.bfloat16)


def prompt(n, seed=3):
    return torch.randint(0, 50304, (n,), generator=torch.Generator().manual_seed(seed))


@pytest.mark.parametrize("n", [40, 300])
def test_prefill_logits_match_oracle(params, model, n):
    p = prompt(n)
    cache = model.new_cache()
    assert model.prefill_supported(cache, p[None].to(DEV))
    with torch.no_grad():
        got = model(p[None].to(DEV), cache)[0].float().cpu()
    assert cache.position == n
    want, margin = oracle_prefill_with_margins(oracle.round_params(params, torch.bfloat16), oracle.BASELINE_ARCH, p)
    rel = (got - want).norm(dim=-1) / want.norm(dim=-1)
    clear = margin > 5e-3  # positions whose routing no bf16 rounding can flip
    assert float(clear.float().mean()) > 0.5  # most positions are checked at 2e-2
    assert float(rel[clear].max()) < 2e-2, rel
    assert float(rel.median()) < 1e-2, rel


def test_prefill_cache_matches_module_path(model):
    p = prompt(64, seed=4)
    fast = model.new_cache()
    with torch.no_grad():
        model(p[None].to(DEV), fast)
    model.set_moe_mode("reference")
    try:
        ref = model.new_cache()
        assert not model.prefill_supported(ref, p[None].to(DEV))
        with torch.no_grad():
            model(p[None].to(DEV), ref)
    finally:
        model.set_moe_mode("auto")
    n = 64
    for a, b in ((fast.k, ref.k), (fast.v, ref.v)):
        a, b = a[:, :, :, :n].float(), b[:, :, :, :n].float()
        torch.testing.assert_close(a[0], b[0], atol=2e-2, rtol=2e-2)
        close = (a - b).abs() <= 2e-2 + 2e-2 * b.abs()
        assert float(close.float().mean()) >= 0.95, float(close.float().mean())


def test_prefill_paged_equals_contiguous(model):
    p = prompt(100, seed=5)
    contiguous = model.new_cache()
    alloc = model.new_block_allocator(num_blocks=40, block_size=16)
    free = list(alloc.free_blocks)
    __import__("random").Random(1).shuffle(free)
    alloc.free_blocks = free
    paged = alloc.new_cache()
    with torch.no_grad():
        a = model(p[None].to(DEV), contiguous)
        b = model(p[None].to(DEV), paged)
    assert torch.equal(a, b)
    for layer in (0, 11):
        for pos in (0, 17, 99):
            blk, slot = paged.block_table[pos // 16], pos % 16
            assert torch.equal(alloc.k_pool[layer, blk, :, slot], contiguous.k[layer, 0, :, pos])
            assert torch.equal(alloc.v_pool[layer, blk, :, slot], contiguous.v[layer, 0, :, pos])


def test_gather_attention_keeps_module_path(model):
    p = prompt(16)
    cache = model.new_cache(attention_mode="gather")
    assert not model.prefill_supported(cache, p[None].to(DEV))
