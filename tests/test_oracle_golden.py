"""Pin the CPU oracle against outputs of the unmodified reference engine.

The fixtures under tests/golden/ were produced by tests/golden/make_golden.py
running the reference (reference architecture).  Each test regenerates the
same seeded weights and inputs and requires the oracle to reproduce the
reference's outputs.  The three BASELINE substitutions (RMSNorm, RoPE, SwiGLU)
have no reference implementation; they are pinned against independent
formulations below.
"""

import math
import os
import random

import pytest
import torch
import torch.nn.functional as F

import oracle
from tests.golden import make_golden as mg

GOLDEN = os.path.dirname(mg.__file__)


def load(name):
    return torch.load(os.path.join(GOLDEN, name), weights_only=False)


@pytest.fixture(scope="module")
def tiny():
    fx = load("reference_tiny.pt")
    P = oracle.init_params(mg.TINY_ARCH, seed=mg.TINY_SEED, bias_std=0.02, norm_std=0.1)
    return fx, P


def test_full_forward_matches_reference(tiny):
    fx, P = tiny
    logits = oracle.forward_full(P, mg.TINY_ARCH, fx["ids"])
    torch.testing.assert_close(logits, fx["full_logits"], atol=1e-5, rtol=1e-5)


def test_cached_decode_matches_reference(tiny):
    fx, P = tiny
    ids = fx["ids"]
    dec = oracle.Decoder(P, mg.TINY_ARCH)
    steps = [dec.forward(ids[:, :4])[:, -1]]
    for t in range(4, 16):
        steps.append(dec.forward(ids[:, t : t + 1])[:, -1])
    got = torch.stack(steps, 1)
    torch.testing.assert_close(got, fx["cached_step_logits"], atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(got, fx["paged_step_logits"], atol=1e-5, rtol=1e-5)


def test_paged_addressing_matches_reference_pool(tiny):
    """Rebuild the reference's paged K pool with the oracle's block addressing."""
    fx, P = tiny
    arch = mg.TINY_ARCH
    table = fx["paged_block_table"].tolist()
    dec = oracle.Decoder(P, arch)
    ids = fx["ids"]
    dec.forward(ids[:, :4])
    for t in range(4, 16):
        dec.forward(ids[:, t : t + 1])
    pool = torch.zeros_like(fx["paged_k_pool"])
    for layer in range(arch.num_layers):
        for pos in range(16):
            oracle.paged_write(pool[layer], table, pos, dec.k[layer, :, pos])
    torch.testing.assert_close(pool, fx["paged_k_pool"], atol=1e-6, rtol=1e-6)
    for layer in range(arch.num_layers):
        g = oracle.paged_gather(pool[layer], table, 16)
        torch.testing.assert_close(g, dec.k[layer, :, :16], atol=0, rtol=0)


def test_greedy_tokens_match_reference(tiny):
    fx, P = tiny
    got = oracle.generate_greedy(P, mg.TINY_ARCH, fx["greedy_prompt"], 12)
    assert got == fx["greedy_vendored"].tolist()
    assert got == fx["greedy_engine"].tolist()


def test_context_limit_semantics_match_reference(tiny):
    fx, P = tiny
    got = oracle.generate_greedy(P, mg.TINY_ARCH, fx["limit_prompt"], 10)
    assert got == fx["limit_engine"].tolist()
    assert len(got) == mg.TINY["max_seq_length"] + 1


def test_moe_layer_matches_reference_production_shape():
    fx = load("reference_moe.pt")
    router, w1, b1, w2, b2, xs = mg.moe_weights()
    for i, x in enumerate(xs):
        out, logits, ids, weights = oracle.moe_decode_stacked(x, router, w1, b1, w2, b2)
        torch.testing.assert_close(logits, fx["router_logits"][i], atol=1e-6, rtol=1e-6)
        assert torch.equal(ids, fx["expert_ids"][i])
        torch.testing.assert_close(weights, fx["route_weights"][i], atol=1e-7, rtol=1e-6)
        torch.testing.assert_close(out, fx["out"][i], atol=2e-6, rtol=1e-5)


def test_paged_attention_matches_reference_gather_oracle():
    fx = load("reference_attention.pt")
    for i in sorted(fx):
        c = fx[i]
        free, k, v, q, nb = mg.attention_inputs(c["H"], c["hd"], c["bs"], c["ctx"], c["max_seq"], c["seed"], True)
        nblk = -(-c["ctx"] // c["bs"])
        table = [free.pop() for _ in range(nblk)]  # BlockAllocator.allocate pops the tail
        assert table == c["block_table"].tolist()
        pool = torch.zeros(nb, c["H"], c["bs"], c["hd"])
        for pos in range(c["ctx"]):
            oracle.paged_write(pool, table, pos, k[0, :, pos])
        keys = oracle.paged_gather(pool, table, c["ctx"])
        pool_v = torch.zeros_like(pool)
        for pos in range(c["ctx"]):
            oracle.paged_write(pool_v, table, pos, v[0, :, pos])
        vals = oracle.paged_gather(pool_v, table, c["ctx"])
        got = oracle.attention_decode(q[0, :, 0], keys, vals)
        torch.testing.assert_close(got, c["out"], atol=2e-6, rtol=1e-5)


def test_topk_breaks_ties_toward_lower_index():
    vals, ids = oracle.topk_lower_index(torch.zeros(8), 2)
    assert ids.tolist() == [0, 1]
    logits = torch.tensor([0.1, 0.5, 0.5, 0.2, 0.5])
    assert oracle.topk_lower_index(logits, 2)[1].tolist() == [1, 2]


# --- BASELINE substitutions, pinned against independent formulations ---


def test_rms_norm_matches_torch_functional():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(3, 768, generator=g)
    w = 1 + 0.1 * torch.randn(768, generator=g)
    torch.testing.assert_close(oracle.rms_norm(x, w, 1e-5), F.rms_norm(x, (768,), w, 1e-5), atol=1e-6, rtol=1e-6)


def test_rope_matches_complex_rotation():
    hd, base = 64, 10000.0
    cos, sin = oracle.rope_tables(40, hd, base)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(40, hd, dtype=torch.float64, generator=g)
    got = oracle.apply_rope(x.float(), cos, sin).double()
    # Independent formulation: pair (i, i+hd/2) as a complex number rotated by p*theta_i.
    half = hd // 2
    theta = torch.tensor([base ** (-2.0 * i / hd) for i in range(half)], dtype=torch.float64)
    ang = torch.arange(40, dtype=torch.float64)[:, None] * theta[None]
    z = torch.complex(x[:, :half], x[:, half:]) * torch.exp(1j * ang)
    want = torch.cat([z.real, z.imag], dim=1)
    torch.testing.assert_close(got, want, atol=1e-5, rtol=1e-5)
    # Relative-position property: <R_p q, R_s k> depends only on p - s.
    q, k = x[0].float(), x[1].float()
    d1 = oracle.apply_rope(q, cos[7], sin[7]) @ oracle.apply_rope(k, cos[3], sin[3])
    d2 = oracle.apply_rope(q, cos[24], sin[24]) @ oracle.apply_rope(k, cos[20], sin[20])
    assert math.isclose(float(d1), float(d2), rel_tol=1e-4, abs_tol=1e-5)


def test_swiglu_expert_matches_formula():
    arch = oracle.BASELINE_ARCH.with_(num_layers=1, vocab_size=64, max_seq_length=16)
    P = oracle.init_params(arch, seed=3)
    x = torch.randn(2, 768, generator=torch.Generator().manual_seed(4))
    p = "MoEBlocks.0.moe.experts.5."
    g = x @ P[p + "gate.weight"].T
    u = x @ P[p + "up.weight"].T
    want = (g / (1 + torch.exp(-g)) * u) @ P[p + "down.weight"].T
    torch.testing.assert_close(oracle.expert_forward(x, P, p, arch), want, atol=1e-6, rtol=1e-5)


def test_baseline_cached_decode_matches_full_forward():
    arch = oracle.BASELINE_ARCH.with_(num_layers=2, vocab_size=128, max_seq_length=24, hidden_dim=64,
                                      num_heads=4, expert_hidden_dim=64)
    P = oracle.init_params(arch, seed=5, norm_std=0.1)
    ids = torch.randint(0, 128, (1, 12), generator=torch.Generator().manual_seed(6))
    full = oracle.forward_full(P, arch, ids)
    dec = oracle.Decoder(P, arch)
    steps = [dec.forward(ids[:, :5])[:, -1]]
    for t in range(5, 12):
        steps.append(dec.forward(ids[:, t : t + 1])[:, -1])
    torch.testing.assert_close(torch.stack(steps, 1), full[:, 4:], atol=1e-5, rtol=1e-5)
