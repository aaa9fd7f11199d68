"""Synchronous HTTP serving of ``Model.generate`` (reference: scripts/serve.py:1-164).

Usage::

    python -m moe_engine.serve --checkpoint minimoe_sft.pt --device cuda --cache paged --paged-attention direct
    python -m moe_engine.serve --random-init 0 --device cuda --dtype bf16
    curl -s localhost:8000/generate -d '{"prompt": "The capital of France is"}'
    curl -s localhost:8000/generate -d '{"prompt_ids": [464, 3139, 286, 4881, 318]}'

Same as the reference's server: the ``/generate`` endpoint, the request fields
and defaults (``prompt``, ``max_new_tokens`` 64 and at least 1, ``temperature``
0.8, finite and non-negative), sampling with ``top_k = 50``, the response
(``text``, ``new_tokens``, ``finish_reason`` length / context_limit / eos,
``tokens_per_sec``), the HTTP errors (400 for an empty or over-long prompt,
422 for a request that fails validation), one request at a time under a lock,
a fresh KV cache per request (paged: from one pool sized for a
maximum-length request, blocks returned after the request), and the CLI flags
``--checkpoint --port --device --cache --paged-attention --moe``.

On CUDA with a supported model and cache, ``Model.generate`` runs the decode
step as graph replays of the persistent step kernel (greedy, or the device
sampler for ``temperature > 0``).

Additions:

* ``prompt_ids`` -- token ids instead of text (exactly one of ``prompt`` and
  ``prompt_ids``), and ``token_ids`` in the response.  The GPT-2 BPE files are
  downloaded by tiktoken on first use; where they cannot be had, text prompts
  answer 503 and id prompts still work (``text`` is then null);
* ``--random-init SEED`` serves the BASELINE architecture with seeded random
  weights when no checkpoint is at hand; ``--dtype`` casts the weights.
"""

from __future__ import annotations

import argparse
import threading
import time
from typing import Optional

import torch
from fastapi import FastAPI, HTTPException
from pydantic import BaseModel, Field, model_validator

from .model import Model, baseline_config, random_init_

SAMPLE_TOP_K = 50  # the reference server's fixed top-k (scripts/serve.py:115)
BLOCK_SIZE = 16


class GenerateRequest(BaseModel):
    prompt: Optional[str] = Field(None, min_length=1)
    prompt_ids: Optional[list[int]] = None
    max_new_tokens: int = Field(64, ge=1)
    temperature: float = Field(0.8, ge=0.0, allow_inf_nan=False)

    @model_validator(mode="after")
    def _one_prompt(self):
        if (self.prompt is None) == (self.prompt_ids is None):
            raise ValueError("give exactly one of prompt and prompt_ids")
        return self


def gpt2_encoder():
    """tiktoken's GPT-2 encoding, or None where its BPE files cannot be had."""
    try:
        import tiktoken

        return tiktoken.get_encoding("gpt2")
    except Exception:  # missing package or no network for the BPE files
        return None


def finish_reason(prompt_len: int, new_tokens: int, max_new_tokens: int, max_seq_length: int) -> str:
    """Why generation stopped, from the lengths alone (scripts/serve.py:126-132):
    generate() returns tokens only; at the context limit it has emitted
    max_seq_length - prompt_len + 1 tokens."""
    if new_tokens == max_new_tokens:
        return "length"
    if prompt_len + new_tokens > max_seq_length:
        return "context_limit"
    return "eos"


class Server:
    """The model, its cache policy and the request lock behind one app."""

    def __init__(self, model: Model, cache_mode: str = "contiguous", paged_attention: str = "auto",
                 encoder="auto", device=None):
        if cache_mode not in ("contiguous", "paged"):
            raise ValueError(f"unknown cache mode {cache_mode!r}")
        self.model = model
        self.cache_mode = cache_mode
        self.device = device if device is not None else model.token_embedding.weight.device
        self._encoder = encoder
        self.allocator = None
        if cache_mode == "paged":
            # one maximum-length request (scripts/serve.py:147-155)
            num_blocks = -(-model.max_seq_length // BLOCK_SIZE)
            self.allocator = model.new_block_allocator(num_blocks=num_blocks, block_size=BLOCK_SIZE,
                                                       attention_mode=paged_attention)
        # the pool holds one maximum-length sequence: one request at a time
        self.lock = threading.Lock()

    @property
    def encoder(self):
        if self._encoder == "auto":
            self._encoder = gpt2_encoder()
        return self._encoder

    def new_request_cache(self):
        return self.model.new_cache() if self.cache_mode == "contiguous" else self.allocator.new_cache()

    def release_request_cache(self, cache) -> None:
        if self.cache_mode == "paged":
            cache.free()

    def prompt_ids(self, req: GenerateRequest) -> list[int]:
        if req.prompt_ids is not None:
            ids = list(req.prompt_ids)
            vocab = self.model.config.vocab_size
            bad = [t for t in ids if not 0 <= t < vocab]
            if bad:
                raise HTTPException(status_code=400, detail=f"token id {bad[0]} is outside [0, {vocab})")
            return ids
        enc = self.encoder
        if enc is None:
            raise HTTPException(status_code=503,
                                detail="the GPT-2 tokenizer is unavailable on this host; send prompt_ids")
        return enc.encode(req.prompt)

    def generate(self, req: GenerateRequest) -> dict:
        ids = self.prompt_ids(req)
        if len(ids) == 0:
            raise HTTPException(status_code=400, detail="prompt tokenizes to zero tokens")
        limit = self.model.max_seq_length
        if len(ids) > limit:
            raise HTTPException(status_code=400,
                                detail=f"prompt is {len(ids)} tokens; the model's context is {limit}")
        prompt = torch.tensor(ids, dtype=torch.long, device=self.device)
        with self.lock:
            cache = self.new_request_cache()
            start = time.perf_counter()
            try:
                with torch.no_grad():
                    out = self.model.generate(prompt, max_new_tokens=req.max_new_tokens,
                                              temperature=req.temperature, top_k=SAMPLE_TOP_K, cache=cache)
                new_ids = out[0, len(ids):].tolist()  # host copy: the tokens are final
            finally:
                self.release_request_cache(cache)
            elapsed = time.perf_counter() - start
        enc = self._encoder if self._encoder != "auto" else None  # resolved by a text prompt, or given
        return {
            "text": enc.decode(new_ids) if enc is not None else None,
            "token_ids": new_ids,
            "new_tokens": len(new_ids),
            "finish_reason": finish_reason(len(ids), len(new_ids), req.max_new_tokens, limit),
            "tokens_per_sec": round(len(new_ids) / elapsed, 1) if elapsed > 0 else None,
        }


def create_app(server: Server) -> FastAPI:
    app = FastAPI(title="moe-engine")

    @app.post("/generate")
    def generate(req: GenerateRequest):  # sync handler: runs in the server's thread pool
        return server.generate(req)

    app.state.server = server
    return app


def pick_device() -> str:
    return "cuda" if torch.cuda.is_available() else "cpu"


def build_parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser()
    parser.add_argument("--checkpoint", default="checkpoints/minimoe_sft.pt")
    parser.add_argument("--random-init", type=int, default=None, metavar="SEED",
                        help="serve the BASELINE architecture with seeded random weights instead of a checkpoint")
    parser.add_argument("--port", type=int, default=8000)
    parser.add_argument("--device", choices=["auto", "cpu", "cuda"], default="cpu",
                        help="execution device (default: CPU; CUDA requires explicit selection)")
    parser.add_argument("--dtype", choices=["checkpoint", "fp32", "bf16"], default="checkpoint")
    parser.add_argument("--cache", choices=["contiguous", "paged"], default="contiguous",
                        help="KV cache used for serving (default: contiguous for lowest single-request latency)")
    parser.add_argument("--paged-attention", choices=["auto", "direct", "gather"], default="auto",
                        help="paged cache only: direct kernel, gather oracle, or automatic fallback")
    parser.add_argument("--moe", choices=["auto", "direct", "reference"], default="auto",
                        help="MoE decode: fused kernel, PyTorch oracle, or automatic fallback")
    return parser


def load_model(args) -> tuple[Model, dict]:
    device = pick_device() if args.device == "auto" else args.device
    if device == "cuda" and not torch.cuda.is_available():
        raise SystemExit("CUDA was requested but is not available")
    dtype = {"fp32": torch.float32, "bf16": torch.bfloat16}.get(args.dtype)
    if args.random_init is not None:
        model = Model(baseline_config()).eval().to(device=device, dtype=dtype or torch.float32)
        random_init_(model, args.random_init)
        metadata = {"step": f"random-init seed {args.random_init}"}
    else:
        from .checkpoint import load_engine_model

        model, _, metadata = load_engine_model(args.checkpoint, device, dtype)
    model.set_moe_mode(args.moe)
    return model, metadata


def main(argv=None) -> None:
    args = build_parser().parse_args(argv)
    model, metadata = load_model(args)
    server = Server(model, args.cache, args.paged_attention)
    print(f"Serving checkpoint step {metadata['step']} on {server.device} with {args.cache} "
          f"KV cache and {args.moe} MoE")
    import uvicorn

    uvicorn.run(create_app(server), host="127.0.0.1", port=args.port)


if __name__ == "__main__":
    main()
