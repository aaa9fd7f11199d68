"""The HTTP server on the GPU (moe_engine/serve.py): the BASELINE model in bf16
with the paged cache and the direct attention kernel, as the reference's
``serve.py --device cuda --cache paged --paged-attention direct`` runs it.
Greedy responses equal ``Model.generate`` on the persistent step; sampled
responses (temperature 0.8, top_k 50) run on the device sampler and repeat
under the same torch seed."""

import pytest
import torch
from fastapi.testclient import TestClient

from moe_engine import serve
from moe_engine.model import Model, baseline_config, random_init_

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def server():
    model = Model(baseline_config()).eval().to(DEV, torch.bfloat16)
    random_init_(model, 0)
    return serve.Server(model, cache_mode="paged", paged_attention="direct", encoder=None)


def test_greedy_matches_generate(server):
    c = TestClient(serve.create_app(server))
    ids = torch.randint(0, 50304, (40,), generator=torch.Generator().manual_seed(8)).tolist()
    body = c.post("/generate", json={"prompt_ids": ids, "max_new_tokens": 48, "temperature": 0}).json()
    cache = server.allocator.new_cache()
    assert server.model.fused_decode_supported(cache, 1)
    want = server.model.generate(torch.tensor(ids, device=DEV), max_new_tokens=48, temperature=0, cache=cache)
    cache.free()
    assert body["token_ids"] == want[0, 40:].tolist()
    assert body["finish_reason"] == "length" and body["tokens_per_sec"] > 0
    assert len(server.allocator.free_blocks) == 96


def test_sampled_requests_repeat(server):
    c = TestClient(serve.create_app(server))
    req = {"prompt_ids": [464, 3139, 286, 4881, 318], "max_new_tokens": 32}
    torch.manual_seed(11)
    a = c.post("/generate", json=req).json()
    torch.manual_seed(11)
    b = c.post("/generate", json=req).json()
    assert a["token_ids"] == b["token_ids"] and a["new_tokens"] == 32
    assert server.model.decode_runner().supports_sampling(server.allocator.new_cache(), 0.8, serve.SAMPLE_TOP_K)
