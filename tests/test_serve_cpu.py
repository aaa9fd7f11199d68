"""The HTTP server (moe_engine/serve.py, reference scripts/serve.py) on CPU with
a tiny model: request validation and HTTP errors, token ids equal to
``Model.generate``, finish reasons, paged blocks returned after a request,
the tokenizer-less host (id prompts only) and the CLI flags."""

import pytest
import torch
from fastapi.testclient import TestClient

from moe_engine import serve
from moe_engine.model import Model, ModelConfig, random_init_
from tests.helpers import TINY


class CharEncoder:
    """Stand-in for the GPT-2 encoding: one token per character, mod 96."""

    def encode(self, text):
        return [ord(c) % 96 for c in text]

    def decode(self, ids):
        return "".join(chr(32 + t % 90) for t in ids)


@pytest.fixture(scope="module")
def model():
    cfg = ModelConfig(**dict(TINY, num_heads=4, norm="rms", pos="rope", expert_act="swiglu", expert_hidden_dim=32,
                             bias=False))
    return random_init_(Model(cfg).eval(), seed=0)


def client(model, **kw):
    kw.setdefault("encoder", CharEncoder())
    return TestClient(serve.create_app(serve.Server(model, **kw)))


def test_id_prompt_greedy_equals_generate(model):
    c = client(model)
    r = c.post("/generate", json={"prompt_ids": [5, 9, 13, 2], "max_new_tokens": 6, "temperature": 0})
    assert r.status_code == 200, r.text
    body = r.json()
    want = model.generate(torch.tensor([5, 9, 13, 2]), max_new_tokens=6, temperature=0)[0, 4:].tolist()
    assert body["token_ids"] == want
    assert body["new_tokens"] == 6 and body["finish_reason"] == "length"
    assert body["text"] == CharEncoder().decode(want)
    assert body["tokens_per_sec"] > 0


def test_text_prompt_and_default_sampling(model):
    c = client(model)
    torch.manual_seed(3)
    a = c.post("/generate", json={"prompt": "hello", "max_new_tokens": 5}).json()
    torch.manual_seed(3)
    b = c.post("/generate", json={"prompt": "hello", "max_new_tokens": 5}).json()
    assert a["token_ids"] == b["token_ids"]  # temperature 0.8, top_k 50 from torch's generator
    assert a["new_tokens"] == 5 and all(0 <= t < 96 for t in a["token_ids"])
    assert a["text"] == CharEncoder().decode(a["token_ids"])


@pytest.mark.parametrize("body", [
    {},                                                   # no prompt
    {"prompt": "a", "prompt_ids": [1]},                   # both
    {"prompt": ""},                                       # empty text
    {"prompt_ids": [1], "max_new_tokens": 0},
    {"prompt_ids": [1], "temperature": -0.5},
    {"prompt_ids": [1], "temperature": "inf"},
])
def test_validation_errors_are_422(model, body):
    assert client(model).post("/generate", json=body).status_code == 422


def test_prompt_errors_are_400(model):
    c = client(model)
    assert c.post("/generate", json={"prompt_ids": []}).status_code == 400
    assert c.post("/generate", json={"prompt_ids": [1, 96]}).status_code == 400  # outside the vocabulary
    r = c.post("/generate", json={"prompt_ids": [1] * 33})
    assert r.status_code == 400 and "context" in r.json()["detail"]


def test_context_limit(model):
    c = client(model)
    body = c.post("/generate", json={"prompt_ids": [3] * 30, "max_new_tokens": 64, "temperature": 0}).json()
    # generate emits max_seq_length - prompt + 1 tokens at the context limit
    assert body["new_tokens"] == 3 and body["finish_reason"] == "context_limit"


def test_finish_reason():
    assert serve.finish_reason(4, 6, 6, 32) == "length"
    assert serve.finish_reason(30, 3, 64, 32) == "context_limit"
    assert serve.finish_reason(4, 2, 6, 32) == "eos"


def test_paged_cache_returns_blocks(model):
    srv = serve.Server(model, cache_mode="paged", paged_attention="gather", encoder=CharEncoder())
    assert len(srv.allocator.free_blocks) == 2  # one maximum-length request of 32 tokens
    c = TestClient(serve.create_app(srv))
    paged = c.post("/generate", json={"prompt_ids": [7, 1, 4], "max_new_tokens": 8, "temperature": 0}).json()
    assert len(srv.allocator.free_blocks) == 2
    contiguous = client(model).post("/generate", json={"prompt_ids": [7, 1, 4], "max_new_tokens": 8,
                                                        "temperature": 0}).json()
    assert paged["token_ids"] == contiguous["token_ids"]


def test_tokenizer_unavailable(model):
    c = client(model, encoder=None)
    r = c.post("/generate", json={"prompt": "hello"})
    assert r.status_code == 503 and "prompt_ids" in r.json()["detail"]
    body = c.post("/generate", json={"prompt_ids": [1, 2], "max_new_tokens": 2}).json()
    assert body["text"] is None and body["new_tokens"] == 2


def test_cli_flags_and_random_init():
    args = serve.build_parser().parse_args(["--random-init", "0", "--cache", "paged", "--paged-attention", "direct",
                                            "--moe", "reference", "--port", "8123"])
    assert (args.cache, args.paged_attention, args.moe, args.port, args.device) == (
        "paged", "direct", "reference", 8123, "cpu")
    with pytest.raises(SystemExit):
        serve.build_parser().parse_args(["--moe", "triton"])
    with pytest.raises(ValueError):
        serve.Server(Model(ModelConfig(**TINY)), cache_mode="ring")


def test_over_http(model):
    """The app under uvicorn on a local port, posted to with a plain HTTP client."""
    import socket
    import threading
    import time

    import requests
    import uvicorn

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    app = serve.create_app(serve.Server(model, encoder=CharEncoder()))
    server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
    t = threading.Thread(target=server.run, daemon=True)
    t.start()
    try:
        for _ in range(200):
            if server.started:
                break
            time.sleep(0.05)
        assert server.started
        r = requests.post(f"http://127.0.0.1:{port}/generate", json={"prompt": "abc", "max_new_tokens": 3,
                                                                      "temperature": 0}, timeout=60)
        assert r.status_code == 200 and r.json()["new_tokens"] == 3
    finally:
        server.should_exit = True
        t.join(timeout=30)
