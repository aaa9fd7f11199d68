"""Device sampler of the persistent step (temperature / top-k, model.py:604-613).

The reference samples with torch.multinomial, whose random stream cannot be
reproduced bit for bit, so the sampler is pinned by its distribution and its
limits:

* top_k = 1 gives the greedy tokens;
* a fixed torch seed gives the same tokens twice, another seed other tokens;
* at one fixed context, 2,000 draws (seeds 0..1999) match softmax(logits / T)
  restricted to the top_k largest logits: every token's frequency within
  4 standard errors + 0.01 of its probability, no token outside the top_k;
  and with top_k = 0 (whole vocabulary) at temperature 0.05.
"""

import pytest
import torch

from moe_engine.model import Model, baseline_config
from moe_engine.paged_attention import cache_geometry
import oracle
from tests.helpers import engine_state_dict

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def model():
    P = oracle.init_params(oracle.BASELINE_ARCH, seed=0)
    m = Model(baseline_config()).eval()
    m.load_state_dict(engine_state_dict(P))
    return m.to(DEV, torch.bfloat16)


def prompt(n=24, seed=21):
    return torch.randint(0, 50304, (n,), generator=torch.Generator().manual_seed(seed))


def test_top1_equals_greedy(model):
    p = prompt()
    greedy = model.generate(p, max_new_tokens=40, temperature=0)
    cache = model.new_cache()
    assert model.decode_runner().supports_sampling(cache, 1.0, 1)
    top1 = model.generate(p, max_new_tokens=40, temperature=1.0, top_k=1, cache=cache)
    assert torch.equal(top1, greedy)


def test_seeded_runs_repeat(model):
    p = prompt(seed=22)
    torch.manual_seed(5)
    a = model.generate(p, max_new_tokens=48, temperature=0.8, top_k=40)
    torch.manual_seed(5)
    b = model.generate(p, max_new_tokens=48, temperature=0.8, top_k=40)
    torch.manual_seed(6)
    c = model.generate(p, max_new_tokens=48, temperature=0.8, top_k=40)
    assert torch.equal(a, b)
    assert not torch.equal(a, c)
    assert a.shape == (1, 24 + 48)


def draws(model, temperature, top_k, n=2000):
    """n device draws at the same context (one eager step launch each)."""
    runner = model.decode_runner()
    cache = model.new_cache()
    p = prompt(seed=23)
    with torch.no_grad():
        model(p[None].to(DEV), cache)
    P = cache.position
    _, _, _, _, bs, _, _ = cache_geometry(cache, 0)
    desc, layers = runner.make_desc(cache, logits=True, graph=False, splits=runner.splits_for(P + 1, bs),
                                    sample=(temperature, top_k))
    assert desc.step_scratch, "persistent step with the device sampler"
    tokens = torch.empty(n, dtype=torch.int64)
    for i in range(n):
        runner.token.fill_(int(p[-1]))
        runner.pos.fill_(P)
        runner.sample_seed.fill_(i)
        runner.launch_step(desc)
        tokens[i] = runner.token.item()
    runner.check_status()
    logits = runner.logits.float().cpu()
    del layers
    return tokens, logits


def check_distribution(tokens, logits, temperature, top_k):
    n = tokens.numel()
    z = logits / temperature
    if top_k:
        thr = torch.topk(logits, top_k).values[-1]
        z[logits < thr] = -float("inf")
    prob = torch.softmax(z, dim=-1)
    support = torch.nonzero(prob > 0).view(-1)
    counts = torch.bincount(tokens, minlength=logits.numel()).float()
    assert counts[prob == 0].sum() == 0, "a token outside the top-k was drawn"
    freq = counts / n
    tol = 4 * torch.sqrt(prob * (1 - prob) / n) + 0.01
    assert torch.all((freq - prob).abs()[support] <= tol[support]), (freq[support], prob[support])


def test_topk_distribution(model):
    tokens, logits = draws(model, 0.5, 8)
    check_distribution(tokens, logits, 0.5, 8)


def test_full_vocab_distribution_low_temperature(model):
    tokens, logits = draws(model, 0.05, 0)
    check_distribution(tokens, logits, 0.05, 0)
