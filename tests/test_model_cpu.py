"""Engine semantics on CPU, mirroring the reference's tests/test_parity.py,
tests/test_fused_moe.py and tests/test_paged_attention.py (CPU subsets), with
the pinned oracle standing in for the vendored reference model.  Every test
runs in both architectures (reference and BASELINE)."""

import random

import pytest
import torch

import oracle
from moe_engine import paged_attention
from moe_engine.model import Model, ModelConfig, MoEFeedForward, baseline_config
from tests.helpers import ARCHS, TINY, make_pair

KINDS = ["reference", "baseline"]


def ids(n, seed=0, vocab=96):
    return torch.randint(0, vocab, (1, n), generator=torch.Generator().manual_seed(seed))


@pytest.mark.parametrize("kind", KINDS)
def test_full_forward_matches_oracle(kind):
    P, arch, engine = make_pair(kind)
    x = ids(16)
    with torch.no_grad():
        got = engine(x, engine.new_cache())
    torch.testing.assert_close(got, oracle.forward_full(P, arch, x), atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("paged", [False, True])
def test_stepwise_decode_matches_full_forward(kind, paged):
    _, _, engine = make_pair(kind)
    x = ids(16, seed=1)
    with torch.no_grad():
        full = engine(x, engine.new_cache())
        cache = engine.new_block_allocator(num_blocks=8, block_size=4).new_cache() if paged else engine.new_cache()
        steps = [engine(x[:, :4], cache)[:, -1]]
        for t in range(4, 16):
            steps.append(engine(x[:, t : t + 1], cache)[:, -1])
    torch.testing.assert_close(torch.stack(steps, 1), full[:, 3:], atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("kind", KINDS)
def test_paged_cache_shares_pool_without_leaking(kind):
    _, _, engine = make_pair(kind)
    a, b = ids(16, 2), ids(16, 3)
    with torch.no_grad():
        full_a = engine(a, engine.new_cache())
        full_b = engine(b, engine.new_cache())
        alloc = engine.new_block_allocator(num_blocks=8, block_size=4)
        ca, cb = alloc.new_cache(), alloc.new_cache()
        la, lb = engine(a[:, :4], ca), engine(b[:, :4], cb)
        for t in range(4, 16):
            la = engine(a[:, t : t + 1], ca)
            lb = engine(b[:, t : t + 1], cb)
    torch.testing.assert_close(la[:, -1], full_a[:, -1], atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(lb[:, -1], full_b[:, -1], atol=1e-4, rtol=1e-4)


def test_block_allocator_reclaims_freed_blocks():
    _, _, engine = make_pair()
    x = ids(8)
    alloc = engine.new_block_allocator(num_blocks=2, block_size=4)
    ca, cb = alloc.new_cache(), alloc.new_cache()
    with torch.no_grad():
        engine(x, ca)
        with pytest.raises(RuntimeError, match="no free KV cache blocks left"):
            engine(x[:, :1], cb)
        ca.free()
        engine(x[:, :1], cb)


def test_failed_allocation_rolls_back():
    _, _, engine = make_pair()
    alloc = engine.new_block_allocator(num_blocks=1, block_size=4)
    cache = alloc.new_cache()
    x = ids(8)
    with torch.no_grad():
        with pytest.raises(RuntimeError, match="no free KV cache blocks left"):
            engine(x, cache)
        assert cache.block_table == [] and cache.position == 0 and alloc.free_blocks == [0]
        engine(x[:, :4], cache)


def test_paged_cache_rejects_batches():
    _, _, engine = make_pair()
    alloc = engine.new_block_allocator(num_blocks=8, block_size=4)
    x = torch.randint(0, 96, (2, 4))
    with torch.no_grad(), pytest.raises(ValueError, match="batch size 1"):
        engine(x, alloc.new_cache())


@pytest.mark.parametrize("kind", KINDS)
def test_generate_stops_at_context_limit_like_oracle(kind):
    P, arch, engine = make_pair(kind)
    prompt = torch.randint(0, 96, (TINY["max_seq_length"] - 2,), generator=torch.Generator().manual_seed(4))
    out = engine.generate(prompt, max_new_tokens=10, temperature=0)
    assert out.shape[1] == TINY["max_seq_length"] + 1
    assert out[0].tolist() == oracle.generate_greedy(P, arch, prompt, 10)


def test_generate_validates_prompt_and_cache():
    _, _, engine = make_pair()
    with pytest.raises(ValueError, match="max_seq_length"):
        engine.generate(torch.zeros(TINY["max_seq_length"] + 1, dtype=torch.long), max_new_tokens=1)
    alloc = engine.new_block_allocator(num_blocks=8, block_size=4)
    used = alloc.new_cache()
    with torch.no_grad():
        engine(ids(4), used)
    before = list(used.block_table)
    with pytest.raises(ValueError, match="fresh cache"):
        engine.generate(ids(4), max_new_tokens=1, cache=used)
    assert used.block_table == before
    for kw in (dict(temperature=-1), dict(top_k=0), dict(max_new_tokens=0), dict(temperature=float("nan"))):
        args = dict(max_new_tokens=4)
        args.update(kw)
        with pytest.raises(ValueError):
            engine.generate(ids(4), **args)


@pytest.mark.parametrize("kind", KINDS)
def test_greedy_generation_matches_oracle(kind):
    P, arch, engine = make_pair(kind)
    prompt = torch.randint(0, 96, (8,), generator=torch.Generator().manual_seed(5))
    out = engine.generate(prompt, max_new_tokens=12, temperature=0)
    assert out[0].tolist() == oracle.generate_greedy(P, arch, prompt, 12)
    alloc = engine.new_block_allocator(num_blocks=16, block_size=4)
    cache = alloc.new_cache()
    paged = engine.generate(prompt, max_new_tokens=12, temperature=0, cache=cache)
    assert torch.equal(paged, out)


@pytest.mark.parametrize("kind", KINDS)
def test_caches_follow_model_dtype(kind):
    _, _, engine = make_pair(kind)
    engine.double()
    x = ids(8)
    with torch.no_grad():
        full = engine(x, engine.new_cache())
        cache = engine.new_cache()
        engine(x[:, :4], cache)
        step = engine(x[:, 4:5], cache)
        alloc = engine.new_block_allocator(num_blocks=2, block_size=4)
        pc = alloc.new_cache()
        engine(x[:, :4], pc)
        pstep = engine(x[:, 4:5], pc)
    assert full.dtype == torch.float64 and cache.k.dtype == torch.float64 and alloc.k_pool.dtype == torch.float64
    torch.testing.assert_close(step[:, -1], full[:, 4])
    torch.testing.assert_close(pstep[:, -1], full[:, 4], atol=1e-4, rtol=1e-4)


def test_sampling_path_runs_and_is_seeded():
    _, _, engine = make_pair("baseline")
    prompt = ids(6)
    torch.manual_seed(0)
    a = engine.generate(prompt, max_new_tokens=8, temperature=0.8, top_k=5)
    torch.manual_seed(0)
    b = engine.generate(prompt, max_new_tokens=8, temperature=0.8, top_k=5)
    assert torch.equal(a, b) and a.shape[1] <= 14


# --- MoE dispatch (reference tests/test_fused_moe.py CPU subset) ---


@pytest.mark.parametrize("act", ["gelu", "swiglu"])
def test_auto_falls_back_on_cpu_and_forced_direct_fails(act):
    torch.manual_seed(0)
    moe = MoEFeedForward(32, 128, 4, 2, mode="auto", activation=act).eval()
    x = torch.randn(1, 1, 32)
    with torch.no_grad():
        torch.testing.assert_close(moe(x, decode=True), moe._forward_reference(x), atol=0, rtol=0)
    moe.set_mode("direct")
    with pytest.raises(RuntimeError, match="direct"):
        moe(x, decode=True)
    prefill = x.expand(1, 2, 32)
    with torch.no_grad():
        torch.testing.assert_close(moe(prefill, decode=False), moe._forward_reference(prefill), atol=0, rtol=0)
    with pytest.raises(ValueError, match="unknown MoE mode"):
        moe.set_mode("fast")


def test_forward_reference_matches_oracle_moe_and_breaks_ties_low():
    P = oracle.init_params(ARCHS["baseline"][1], seed=7)
    moe = MoEFeedForward(32, 32, 4, 2, activation="swiglu").eval()
    sd = {k[len("MoEBlocks.0.moe."):]: v for k, v in P.items() if k.startswith("MoEBlocks.0.moe.")}
    moe.load_state_dict(sd)
    x = torch.randn(1, 5, 32, generator=torch.Generator().manual_seed(8))
    with torch.no_grad():
        got = moe._forward_reference(x)
    want = oracle.moe_forward(x, P, 0, ARCHS["baseline"][1])[0]
    torch.testing.assert_close(got, want, atol=1e-6, rtol=1e-5)
    with torch.no_grad():
        moe.router.weight.zero_()  # all logits tie: experts 0 and 1 must be picked
        only01 = moe._forward_reference(x[:, :1])
        e0 = moe.experts[0](x[:, :1]) * 0.5 + moe.experts[1](x[:, :1]) * 0.5
    torch.testing.assert_close(only01, e0, atol=1e-6, rtol=1e-5)


def _assert_canonical(moe, device_type, dtype):
    for name, (getter, pname) in moe._groups().items():
        storage = moe._expert_storage[name]
        params = [getattr(getter(e), pname) for e in moe.experts]
        stride = params[0].numel() * params[0].element_size()
        assert storage.device.type == device_type and storage.dtype == dtype and storage.is_contiguous()
        assert storage.data_ptr() == params[0].data_ptr()
        assert [p.data_ptr() for p in params] == [params[0].data_ptr() + i * stride for i in range(moe.num_experts)]


@pytest.mark.parametrize("act", ["gelu", "swiglu"])
def test_canonical_storage_survives_load_and_dtype_apply(act):
    moe = MoEFeedForward(32, 128, 4, 2, activation=act)
    names = set(moe.state_dict())
    if act == "gelu":
        expected = {f"experts.{e}.{l}.{p}" for e in range(4) for l in ("net.0", "net.2") for p in ("weight", "bias")}
    else:
        expected = {f"experts.{e}.{l}.weight" for e in range(4) for l in ("gate", "up", "down")}
    assert names == expected | {"router.weight"}
    ck = {n: torch.randn_like(p) for n, p in moe.state_dict().items()}
    moe.load_state_dict(ck)
    assert all(torch.equal(moe.state_dict()[n], ck[n]) for n in ck)
    _assert_canonical(moe, "cpu", torch.float32)
    ck2 = {n: torch.randn_like(p) for n, p in moe.state_dict().items()}
    moe.load_state_dict(ck2, assign=True)
    assert all(torch.equal(moe.state_dict()[n], ck2[n]) for n in ck2)
    _assert_canonical(moe, "cpu", torch.float32)
    moe.double()
    _assert_canonical(moe, "cpu", torch.float64)
    moe.bfloat16()
    _assert_canonical(moe, "cpu", torch.bfloat16)
    assert moe._router_logits.dtype == torch.float32 and moe._expert_hidden.dtype == torch.float32
    assert moe._direct_out.dtype == torch.bfloat16 and moe._expert_ids.dtype == torch.int32


# --- paged attention fallbacks (reference tests/test_paged_attention.py CPU subset) ---


@pytest.mark.parametrize("kind", KINDS)
def test_auto_mode_matches_gather_mode(kind):
    _, _, model = make_pair(kind)
    x = ids(16, 6)
    logits = {}
    for mode in ["gather", "auto"]:
        cache = model.new_block_allocator(num_blocks=16, block_size=4, attention_mode=mode).new_cache()
        with torch.no_grad():
            steps = [model(x[:, :8], cache)[:, -1]]
            for t in range(8, 16):
                steps.append(model(x[:, t : t + 1], cache)[:, -1])
        logits[mode] = torch.stack(steps, 1)
    torch.testing.assert_close(logits["auto"], logits["gather"], atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("kind", KINDS)
def test_prefill_fast_path_matches_contiguous(kind):
    _, _, model = make_pair(kind)
    x = ids(19, 7)
    with torch.no_grad():
        contiguous = model(x, model.new_cache())
        cache = model.new_block_allocator(num_blocks=16, block_size=4).new_cache()
        paged = model(x, cache)
    torch.testing.assert_close(paged, contiguous, atol=1e-5, rtol=1e-5)


def test_direct_mode_raises_without_cuda_and_leaves_cache_untouched():
    _, _, model = make_pair()
    alloc = model.new_block_allocator(num_blocks=8, block_size=4, attention_mode="direct")
    cache = alloc.new_cache()
    with torch.no_grad(), pytest.raises(RuntimeError, match="direct"):
        model(ids(5), cache)
    assert cache.position == 0 and cache.block_table == []
    assert sorted(alloc.free_blocks) == list(range(8))
    assert (cache.block_table_device == 0).all() and cache._write_index_key is None


def test_invalid_attention_mode_rejected():
    model = Model(ModelConfig(**TINY))
    with pytest.raises(ValueError, match="attention_mode"):
        model.new_block_allocator(num_blocks=4, block_size=4, attention_mode="turbo")
    with pytest.raises(ValueError, match="attention_mode"):
        model.new_cache(attention_mode="turbo")
    with pytest.raises(ValueError):
        ModelConfig(norm="batch")


def test_device_block_table_mirrors_python_table():
    _, _, model = make_pair()
    alloc = model.new_block_allocator(num_blocks=16, block_size=4)
    random.Random(1).shuffle(alloc.free_blocks)
    cache = alloc.new_cache()
    x = ids(10)
    with torch.no_grad():
        model(x, cache)
        for t in range(3):
            model(x[:, t : t + 1], cache)
    assert len(cache.block_table) == 4
    assert cache.block_table_device[:4].tolist() == cache.block_table


def test_paged_trim_returns_tail_blocks():
    _, _, model = make_pair()
    alloc = model.new_block_allocator(num_blocks=8, block_size=4)
    cache = alloc.new_cache()
    cache.reserve(14)
    assert len(cache.block_table) == 4
    cache._trim(5)
    assert len(cache.block_table) == 2 and len(alloc.free_blocks) == 6


def test_split_choice_bounds():
    # at least MIN_BLOCKS_PER_SPLIT (8) blocks per split, at most ~2 CTAs per SM
    assert paged_attention.MIN_BLOCKS_PER_SPLIT == 8
    assert paged_attention.choose_splits(12, 96, 148) == 12   # ctx 1536: 8 blocks (128 tokens) per split
    assert paged_attention.choose_splits(12, 8, 148) == 1     # ctx 128: one split per head
    assert paged_attention.choose_splits(12, 512, 148) == 24  # ctx 8192: two CTAs per SM, one wave
    assert paged_attention.choose_splits(12, 1, 148) == 1
    assert paged_attention.choose_splits(8, 512, 148) == 37
    assert paged_attention.choose_splits(1, 10_000, 148) == paged_attention.MAX_SPLITS


def test_baseline_config_shape():
    cfg = baseline_config()
    assert (cfg.num_layers, cfg.num_heads, cfg.head_dim, cfg.expert_hidden, cfg.max_seq_length) == (12, 12, 64, 768, 1536)
    m = Model(baseline_config(num_layers=1, vocab_size=64))
    active = sum(p.numel() for n, p in m.named_parameters() if "experts" not in n)
    assert m.rope_cos.dtype == torch.float32 and m.rope_cos.shape == (1536, 32)
    m.bfloat16()
    assert m.rope_cos.dtype == torch.float32  # RoPE tables stay fp32
    assert active > 0
