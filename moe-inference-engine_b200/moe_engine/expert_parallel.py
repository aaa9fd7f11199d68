"""Expert-parallel batch-one decode over several GPUs (BASELINE config[4b]).

The experts of every layer are split evenly over the ranks of a process group:
rank r serves experts [r E/N, (r+1) E/N).  Every rank holds the attention and
router weights and runs the same decode step on the same token, so routing
agrees everywhere.  Per layer each rank computes the contribution of the
selected experts it owns -- or nothing, when both selected experts live
elsewhere -- into a [D] fp32 partial, and an NCCL all-reduce (sum) over the
group completes the MoE output before the next layer consumes it as its
pending residual.  The LM head then runs on every rank, so every rank holds
the same next token.

The reference has no multi-GPU decode; the operator semantics per layer are
those of the single-GPU path (src/moe_engine/model.py:543-565 with the MoE of
src/moe_engine/fused_moe.py:312-380), with the expert sum split across ranks:
sum_k w_k E_k(x) = sum_ranks sum_{k local} w_k E_k(x).

Each step is launched layer by layer (``mie_decode_layer``, the all-reduce,
``mie_decode_head``); the single-GPU persistent step kernel is not used here.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import capi
from .decode import EOS_TOKEN_ID, DecodeRunner
from .paged_attention import cache_geometry


def expert_shard(num_experts: int, rank: int, world: int) -> tuple[int, int]:
    """(first expert, expert count) served by ``rank`` of ``world``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a group of {world}")
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not split evenly over {world} ranks")
    count = num_experts // world
    return rank * count, count


class ExpertParallelDecoder:
    """Greedy decode of one request with the experts split over ``group``.

    ``model`` is the full model on this rank's GPU (all ranks identical); only
    the experts [base, base + count) of every layer are read by this rank.
    """

    def __init__(self, model, group=None):
        self.model = model
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        cfg = model.config
        self.expert_base, self.expert_count = expert_shard(cfg.num_experts, self.rank, self.world)
        self.runner = DecodeRunner(model, expert_base=self.expert_base, expert_count=self.expert_count,
                                   moe_partial=True)

    def _desc(self, cache, max_ctx: int):
        _, _, _, _, bs, _, _ = cache_geometry(cache, 0)
        return self.runner.make_desc(cache, logits=False, graph=True,
                                     splits=self.runner.splits_for(max_ctx, bs))

    def _step(self, desc, stream) -> None:
        lib, r = self.runner.lib, self.runner
        for layer in range(self.model.config.num_layers):
            capi.check(lib.mie_decode_layer(ctypes.byref(desc), layer, stream), "mie_decode_layer")
            dist.all_reduce(r.moe_partial, op=dist.ReduceOp.SUM, group=self.group)
        capi.check(lib.mie_decode_head(ctypes.byref(desc), stream), "mie_decode_head")

    @torch.no_grad()
    def prefill(self, token_ids: torch.Tensor, cache):
        """Prompt prefill by the model's own forward (every rank); returns the
        [1, T] prompt and the first generated token id."""
        if token_ids.dim() == 1:
            token_ids = token_ids.unsqueeze(0)
        logits = self.model(token_ids.to(self.model.token_embedding.weight.device), cache)
        return token_ids, int(torch.argmax(logits[0, -1]).item())

    @torch.no_grad()
    def decode(self, first: int, steps: int, cache) -> torch.Tensor:
        """``steps`` expert-parallel decode steps after the prompt in ``cache``,
        starting from token ``first``; returns the produced tokens (device).
        EOS stops generation on the device (later steps do nothing)."""
        r = self.runner
        P = cache.position
        if hasattr(cache, "allocator"):
            cache.reserve(P + steps)
        desc, layers = self._desc(cache, P + steps)
        r.token.fill_(first)
        r.pos.fill_(P)
        r.done.zero_()
        r.log_count.zero_()
        stream = capi.stream_handle(r.device)
        for _ in range(steps):
            self._step(desc, stream)
        del layers
        r.check_status()
        count = int(r.log_count.item())
        cache.position = P + count
        if hasattr(cache, "_trim"):
            cache._trim(cache.position)
        new = r.tokens_log[:count]
        if count and int(new[-1]) == EOS_TOKEN_ID and int(r.done.item()):
            new = new[:-1]
        return new

    @torch.no_grad()
    def generate(self, token_ids: torch.Tensor, max_new_tokens: int, cache) -> torch.Tensor:
        """Same contract as greedy ``Model.generate`` (temperature 0) on one rank:
        the prompt prefilled by the model on every rank, the decode steps expert
        parallel, tokens read back once at the end."""
        token_ids, first = self.prefill(token_ids, cache)
        if first == EOS_TOKEN_ID:
            return token_ids
        K = min(max_new_tokens - 1, self.model.max_seq_length - cache.position)
        first_t = token_ids.new_tensor([[first]])
        if K <= 0:
            return torch.cat((token_ids, first_t), dim=1)
        new = self.decode(first, K, cache)
        return torch.cat((token_ids, first_t, new.view(1, -1).to(token_ids.dtype).cpu()), dim=1)
