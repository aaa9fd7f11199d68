"""Whole decode step on the GPU vs the CPU oracle.

* full miniMoE-shaped model (12 x 768, 12 heads x 64,
  RMSNorm, RoPE, 8 SwiGLU experts, vocab 50304), random init seed 0, fp32,
  16-token random prompt, 64 greedy tokens -- tokens must be IDENTICAL to the
  oracle's.
* bf16: hidden states (residual stream after the last layer) within 2e-2
  relative error of the oracle run on the same bf16-rounded weights with a
  bf16 KV cache; greedy tokens agree between the paged, contiguous, eager and
  CUDA-graph paths.
* the reference's model-level CUDA tests at TINY size (greedy direct ==
  contiguous, block reuse, forced-direct preflight leaves caches untouched).
"""

import pytest
import torch

import oracle
from moe_engine.model import Model, baseline_config
from tests.helpers import TINY, engine_state_dict, make_pair

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def baseline_params():
    return oracle.init_params(oracle.BASELINE_ARCH, seed=0)


def baseline_model(P, dtype):
    m = Model(baseline_config()).eval()
    m.load_state_dict(engine_state_dict(P))
    return m.to(DEV, dtype)


def prompt16():
    return torch.randint(0, 50304, (16,), generator=torch.Generator().manual_seed(0))


def test_config0_fp32_greedy_tokens_identical(baseline_params):
    P = baseline_params
    prompt = prompt16()
    want = oracle.generate_greedy(P, oracle.BASELINE_ARCH, prompt, 64)
    m = baseline_model(P, torch.float32)
    got = m.generate(prompt, max_new_tokens=64, temperature=0)[0].tolist()
    assert got == want
    alloc = m.new_block_allocator(num_blocks=96, block_size=16, attention_mode="direct")
    cache = alloc.new_cache()
    got_paged = m.generate(prompt, max_new_tokens=64, temperature=0, cache=cache)[0].tolist()
    assert got_paged == want
    assert cache.position == len(want) - 1
    assert len(cache.block_table) == -(-cache.position // 16)
    m.decode_runner().check_status()


def test_bf16_hidden_states_within_2e2(baseline_params):
    P16 = oracle.round_params(baseline_params, torch.bfloat16)
    m = baseline_model(baseline_params, torch.bfloat16)
    prompt = prompt16()
    dec = oracle.Decoder(P16, oracle.BASELINE_ARCH, kv_dtype=torch.bfloat16)
    dec.forward(prompt[None])
    cache = m.new_cache()
    with torch.no_grad():
        m(prompt[None].to(DEV), cache)
        tok = torch.tensor([[123]])
        for step in range(8):
            logits = m(tok.to(DEV), cache)
            ol = dec.forward(tok, record=True)
            hx = m.decode_runner().x.cpu()
            want = dec.hidden[-1]
            rel = (hx - want).norm() / want.norm()
            assert rel < 2e-2, (step, float(rel))
            lrel = (logits[0, 0].float().cpu() - ol[0, 0]).norm() / ol[0, 0].norm()
            assert lrel < 2e-2, (step, float(lrel))
            tok = torch.tensor([[int(ol[0, -1].argmax())]])
    m.decode_runner().check_status()


def test_bf16_graph_paged_contiguous_agree(baseline_params):
    m = baseline_model(baseline_params, torch.bfloat16)
    prompt = torch.randint(0, 50304, (40,), generator=torch.Generator().manual_seed(3))
    contiguous = m.generate(prompt, max_new_tokens=48, temperature=0)
    alloc = m.new_block_allocator(num_blocks=200, block_size=16)
    random_free = list(alloc.free_blocks)
    __import__("random").Random(0).shuffle(random_free)
    alloc.free_blocks = random_free
    cache = alloc.new_cache()
    paged = m.generate(prompt, max_new_tokens=48, temperature=0, cache=cache)
    assert torch.equal(paged, contiguous)
    # eager fused steps produce the same tokens as the graph replays
    cache2 = m.new_cache()
    with torch.no_grad():
        logits = m(prompt[None].to(DEV), cache2)
        seq = prompt.tolist()
        for _ in range(48):
            t = int(logits[0, -1].float().argmax())
            seq.append(t)
            logits = m(torch.tensor([[t]], device=DEV), cache2)
    assert seq[: contiguous.shape[1]] == contiguous[0].tolist()
    m.decode_runner().check_status()


def test_generate_context_limit_and_chunking_on_gpu():
    P, arch, m = make_pair("baseline", device=DEV, max_seq_length=150)
    prompt = torch.randint(0, 96, (20,), generator=torch.Generator().manual_seed(5))
    want = oracle.generate_greedy(P, arch.with_(max_seq_length=150), prompt, 200)
    got = m.generate(prompt, max_new_tokens=200, temperature=0)[0].tolist()
    assert got == want and len(got) == 151
    # A new cache re-captures the step while the device position still holds
    # the full context of the previous request: no false range report.
    again = m.generate(prompt, max_new_tokens=200, temperature=0, cache=m.new_cache())[0].tolist()
    assert again == want
    m.decode_runner().check_status()


@pytest.mark.parametrize("kind", ["reference", "baseline"])
def test_tiny_greedy_direct_paged_matches_contiguous_and_oracle(kind):
    P, arch, m = make_pair(kind, device=DEV)
    prompt = torch.randint(0, 96, (8,), generator=torch.Generator().manual_seed(6))
    want = oracle.generate_greedy(P, arch, prompt, 20)
    contiguous = m.generate(prompt.to(DEV), max_new_tokens=20, temperature=0)
    alloc = m.new_block_allocator(num_blocks=16, block_size=4, attention_mode="direct")
    cache = alloc.new_cache()
    direct = m.generate(prompt.to(DEV), max_new_tokens=20, temperature=0, cache=cache)
    cache.free()
    assert contiguous[0].tolist() == want
    assert torch.equal(direct, contiguous)
    assert sorted(alloc.free_blocks) == list(range(16))
    cache = alloc.new_cache()
    again = m.generate(prompt.to(DEV), max_new_tokens=20, temperature=0, cache=cache)
    cache.free()
    assert torch.equal(again, direct)


@pytest.mark.parametrize("kind", ["reference", "baseline"])
def test_tiny_stepwise_fused_logits_match_full_forward(kind):
    P, arch, m = make_pair(kind, device=DEV)
    x = torch.randint(0, 96, (1, 16), generator=torch.Generator().manual_seed(7))
    full = oracle.forward_full(P, arch, x)
    for paged in (False, True):
        cache = m.new_block_allocator(num_blocks=8, block_size=4).new_cache() if paged else m.new_cache()
        with torch.no_grad():
            steps = [m(x[:, :4].to(DEV), cache)[:, -1]]
            for t in range(4, 16):
                steps.append(m(x[:, t : t + 1].to(DEV), cache)[:, -1])
        torch.testing.assert_close(torch.stack(steps, 1).cpu(), full[:, 3:], atol=1e-4, rtol=1e-4)


def test_forced_direct_preflight_preserves_caches_on_cuda():
    """float64 is not a kernel dtype: forced direct must fail before any write."""
    _, _, m = make_pair("reference", device=DEV)
    m = m.double()
    alloc = m.new_block_allocator(num_blocks=4, block_size=4)
    cache = alloc.new_cache()
    ids = torch.randint(0, 96, (1, 4), device=DEV)
    with torch.no_grad():
        m(ids, cache)
    before = (cache.position, list(cache.block_table), sorted(alloc.free_blocks), alloc.k_pool.clone())
    m.set_moe_mode("direct")
    with torch.no_grad(), pytest.raises(RuntimeError, match="float32"):
        m(ids[:, :1], cache)
    assert (cache.position, list(cache.block_table), sorted(alloc.free_blocks)) == before[:3]
    assert torch.equal(alloc.k_pool, before[3])
    m.set_moe_mode("auto")
    alloc2 = m.new_block_allocator(num_blocks=8, block_size=4, attention_mode="direct")
    c2 = alloc2.new_cache()
    with torch.no_grad(), pytest.raises(RuntimeError, match="direct"):
        m(ids[:, :1], c2)
    assert c2.position == 0 and c2.block_table == [] and (c2.block_table_device == 0).all()


def test_module_level_direct_paths_match_reference_mode():
    """Per-op drop-in path: MoE direct (kernel) vs reference (PyTorch) on CUDA."""
    P, arch, m = make_pair("baseline", device=DEV)
    x = torch.randint(0, 96, (1, 12), generator=torch.Generator().manual_seed(8)).to(DEV)
    out = {}
    for mode in ("reference", "direct"):
        m.set_moe_mode(mode)
        cache = m.new_cache(attention_mode="gather")  # forces the per-op path
        with torch.no_grad():
            steps = [m(x[:, :4], cache)[:, -1]]
            for t in range(4, 12):
                steps.append(m(x[:, t : t + 1], cache)[:, -1])
        out[mode] = torch.stack(steps, 1)
    torch.testing.assert_close(out["direct"], out["reference"], atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_persistent_step_is_used_and_agrees_with_launch_sequence(baseline_params, dtype):
    """The single-launch step and the per-op launch sequence compute the same
    step: hidden states agree to rounding, greedy tokens are identical."""
    m = baseline_model(baseline_params, dtype)
    runner = m.decode_runner()
    assert runner.uses_persistent(m.new_cache())
    prompt = torch.randint(0, 50304, (24,), generator=torch.Generator().manual_seed(9))
    xs = {}
    for persistent in (True, False):
        runner.persistent = persistent
        cache = m.new_block_allocator(num_blocks=64, block_size=16, attention_mode="direct").new_cache()
        hs = []
        with torch.no_grad():
            m(prompt[None].to(DEV), cache)
            tok = torch.tensor([[17]], device=DEV)
            for _ in range(6):
                logits = m(tok, cache)
                hs.append(runner.x.clone())
                tok = logits[0, -1].float().argmax().view(1, 1)
        xs[persistent] = torch.stack(hs)
        runner.check_status()
    runner.persistent = True
    rel = (xs[True] - xs[False]).norm() / xs[False].norm()
    assert rel < (5e-3 if dtype == torch.bfloat16 else 1e-5), float(rel)
    gen = {}
    for persistent in (True, False):
        runner.persistent = persistent
        gen[persistent] = m.generate(prompt, max_new_tokens=40, temperature=0)
    runner.persistent = True
    assert torch.equal(gen[True], gen[False])
    runner.check_status()


def test_multi_step_graph_honours_step_limit(baseline_params):
    """A graph of several programmatic-dependent step launches decodes exactly
    ``step_limit`` tokens (the extra launches change nothing) and the same
    tokens as eager steps; generate's chunks end mid-graph."""
    m = baseline_model(baseline_params, torch.bfloat16)
    runner = m.decode_runner()
    prompt = torch.randint(0, 50304, (24,), generator=torch.Generator().manual_seed(12))
    eager = m.new_cache()
    with torch.no_grad():
        logits = m(prompt[None].to(DEV), eager)
        seq = []
        for _ in range(21):
            t = int(logits[0, -1].float().argmax())
            seq.append(t)
            logits = m(torch.tensor([[t]], device=DEV), eager)
    got = m.generate(prompt, max_new_tokens=21, temperature=0)[0, 24:].tolist()
    assert got == seq

    alloc = m.new_block_allocator(num_blocks=8, block_size=16, attention_mode="direct")
    cache = alloc.new_cache()
    with torch.no_grad():
        m(prompt[None].to(DEV), cache)
    P = cache.position
    cache.reserve(P + 16)
    M = runner.steps_per_graph(cache)
    assert M > 1
    graph = runner.graph_for(cache, P + 16, steps=M)
    runner.token.fill_(seq[0])
    runner.pos.fill_(P)
    runner.done.zero_()
    runner.log_count.zero_()
    runner.step_limit.fill_(5)
    graph.replay()
    torch.cuda.synchronize()
    assert int(runner.log_count) == 5 and int(runner.pos) == P + 5
    runner.step_limit.fill_(16)
    for _ in range(-(-11 // M)):
        graph.replay()
    torch.cuda.synchronize()
    runner.check_status()
    assert int(runner.log_count) == 16 and int(runner.pos) == P + 16
    assert runner.tokens_log[:16].tolist() == seq[1:17]
