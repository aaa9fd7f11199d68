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

Collectives:

* ``"step"``: each decode step is ONE launch of the persistent cluster step
  kernel on every rank, which completes each layer's all-reduce inside the
  kernel: the CTAs that own a layer's output rows store the rank's partial of
  those rows as tagged fp32 words over NVLink into every rank's receive buffer,
  and every CTA that reads the layer's output polls its own buffer and sums
  the ranks' words in rank order onto x_mid.  Shapes of the cluster step only
  (bf16, head_dim 64, RMSNorm, SwiGLU, no biases).
* ``"fused"``: each step is launched layer by layer (``mie_decode_layer``,
  ``mie_decode_head``) and each layer's MoE kernel completes the all-reduce of
  its partial itself, with the same tagged words.
* ``"peer"``: layer by layer, the same exchange as a kernel of its own after
  the MoE kernel (``mie_peer_reduce``).
* ``"nccl"``: layer by layer, an NCCL all-reduce, whose partial travels as fp32
  or, with ``payload="bf16"``, as bf16 (half the bytes; the residual stream
  then differs from the single-GPU one by the bf16 rounding of each layer's
  MoE output).
* ``"auto"`` (default): ``"step"`` when the cluster step takes the model's
  shapes, else ``"fused"``.

``decode`` captures the steps in CUDA graphs (``GRAPH_STEPS`` steps per graph)
and replays them, so the host issues one graph launch per ``GRAPH_STEPS``
tokens.  Every rank must make the same calls in the same order.  After a
device failure (``KernelError``) the ranks' exchange state may disagree:
``close`` the decoder on every rank and make a new one.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import capi
from .decode import EOS_TOKEN_ID, DecodeRunner
from .paged_attention import cache_geometry


class PeerReducer:
    """All-reduce (sum, rank order) of an fp32 [n] vector over the ranks of
    ``group`` with ``mie_peer_reduce``: every rank stores its words into every
    rank's receive buffer (CUDA IPC mappings; the handles travel through the
    process group once) and polls its own.  Every rank must make the same
    calls in the same order; ``close`` (a collective too) unmaps and frees."""

    def __init__(self, n: int, group=None, device=None, status=None, wait_limit_ns: int = 0):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > capi.MIE_PEER_MAX_RANKS:
            raise ValueError(f"the peer all-reduce takes at most {capi.MIE_PEER_MAX_RANKS} ranks")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        self.lib = capi.ensure_init(self.device)
        self.n = n
        self.local = ctypes.c_void_p()
        nbytes = self.lib.mie_peer_buffer_bytes(n, self.world)
        if nbytes <= 0:
            raise ValueError(f"no peer buffer for n = {n}, world = {self.world}")
        capi.check(self.lib.mie_peer_alloc(nbytes, ctypes.byref(self.local)), "mie_peer_alloc")
        handle = (ctypes.c_char * 64)()
        capi.check(self.lib.mie_peer_handle(self.local, handle), "mie_peer_handle")
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.opened = []
        bufs = []
        for r, hb in enumerate(handles):
            if r == self.rank:
                bufs.append(self.local.value)
                continue
            p = ctypes.c_void_p()
            capi.check(self.lib.mie_peer_open((ctypes.c_char * 64).from_buffer_copy(hb), ctypes.byref(p)),
                       "mie_peer_open")
            self.opened.append(p)
            bufs.append(p.value)
        self.seq = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.status = status if status is not None else torch.zeros(1, dtype=torch.int32, device=self.device)
        self._args = capi.PeerReduceArgs()
        a = self._args
        a.n, a.rank, a.world = n, self.rank, self.world
        for r, b in enumerate(bufs):
            a.bufs[r] = b
        a.seq, a.status, a.wait_limit_ns = self.seq.data_ptr(), self.status.data_ptr(), int(wait_limit_ns)
        dist.barrier(group)  # every rank's buffer zeroed and mapped before the first call

    def __call__(self, inp: torch.Tensor, out: torch.Tensor, stream=None) -> None:
        a = self._args
        a.in_, a.out = inp.data_ptr(), out.data_ptr()
        capi.check(self.lib.mie_peer_reduce(ctypes.byref(a), stream if stream is not None
                                            else capi.stream_handle(self.device)), "mie_peer_reduce")

    def close(self) -> None:
        if self.local is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)  # no rank still writes into a buffer about to go
        for p in self.opened:
            self.lib.mie_peer_close(p)
        self.opened = []
        dist.barrier(self.group)
        self.lib.mie_peer_free(self.local)
        self.local = None


def expert_shard(num_experts: int, rank: int, world: int) -> tuple[int, int]:
    """(first expert, expert count) served by ``rank`` of ``world``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a group of {world}")
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not split evenly over {world} ranks")
    count = num_experts // world
    return rank * count, count


GRAPH_STEPS = 8  # decode steps per captured graph


class ExpertParallelDecoder:
    """Greedy decode of one request with the experts split over ``group``.

    ``model`` is the full model on this rank's GPU (all ranks identical); only
    the experts [base, base + count) of every layer are read by this rank.
    ``payload`` is the all-reduced partial's type: "fp32" or "bf16".
    """

    COLLECTIVES = ("auto", "step", "fused", "peer", "nccl")

    def __init__(self, model, group=None, payload: str = "fp32", use_graph: bool = True,
                 collective: str = "auto"):
        if payload not in ("fp32", "bf16"):
            raise ValueError(f"payload must be fp32 or bf16, not {payload!r}")
        if collective not in self.COLLECTIVES:
            raise ValueError(f"collective must be one of {', '.join(self.COLLECTIVES)}, not {collective!r}")
        if collective != "nccl" and payload != "fp32":
            raise ValueError("the peer all-reduce carries fp32 partials")
        self.model = model
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.payload = payload
        self.collective = collective
        self.use_graph = use_graph
        cfg = model.config
        self.expert_base, self.expert_count = expert_shard(cfg.num_experts, self.rank, self.world)
        self.runner = DecodeRunner(model, expert_base=self.expert_base, expert_count=self.expert_count,
                                   moe_partial=True)
        self._wire = (torch.zeros(cfg.hidden_dim, dtype=torch.bfloat16, device=self.runner.device)
                      if payload == "bf16" else None)
        self._peer = (PeerReducer(cfg.hidden_dim, group, self.runner.device, status=self.runner.status,
                                  wait_limit_ns=getattr(self.runner, "wait_limit_ns", 0))
                      if collective != "nccl" else None)
        self._graphs: dict = {}
        self.active = None  # the collective the last decode ran

    def _step_desc(self, cache, max_ctx: int):
        """Descriptor of the expert-parallel persistent step for ``cache``, or
        (None, None) when the cluster step does not take the shapes."""
        r = self.runner
        if not r.persistent:
            return None, None
        _, _, _, _, bs, _, _ = cache_geometry(cache, 0)
        desc, layers = r.make_desc(cache, logits=False, graph=True, splits=r.splits_for(max_ctx, bs), limit=True,
                                   moe_peer=ctypes.addressof(self._peer._args))
        if not desc.step_scratch:
            return None, None
        return desc, layers

    def collective_for(self, cache, max_ctx: int) -> str:
        """The collective ``decode`` runs for ``cache`` ("auto" resolved)."""
        if self.collective in ("auto", "step"):
            if self._step_desc(cache, max_ctx)[0] is not None:
                return "step"
            if self.collective == "step":
                raise ValueError("the persistent cluster step does not take this model's shapes")
            return "fused"
        return self.collective

    def _desc(self, cache, max_ctx: int):
        _, _, _, _, bs, _, _ = cache_geometry(cache, 0)
        desc, layers = self.runner.make_desc(cache, logits=False, graph=True,
                                             splits=self.runner.splits_for(max_ctx, bs))
        if self.collective == "fused":
            # each layer's MoE kernel completes the all-reduce of its partial itself
            desc.moe_peer = ctypes.addressof(self._peer._args)
        return desc, layers

    def _all_reduce(self) -> None:
        r = self.runner
        if self.collective == "fused":
            return  # done inside the MoE kernel
        if self._peer is not None:
            self._peer(r.moe_partial, r.moe_partial)
        elif self._wire is None:
            dist.all_reduce(r.moe_partial, op=dist.ReduceOp.SUM, group=self.group)
        else:
            self._wire.copy_(r.moe_partial)
            dist.all_reduce(self._wire, op=dist.ReduceOp.SUM, group=self.group)
            r.moe_partial.copy_(self._wire)

    def _step(self, desc, stream) -> None:
        lib = self.runner.lib
        for layer in range(self.model.config.num_layers):
            capi.check(lib.mie_decode_layer(ctypes.byref(desc), layer, stream), "mie_decode_layer")
            self._all_reduce()
        capi.check(lib.mie_decode_head(ctypes.byref(desc), stream), "mie_decode_head")

    def _step_graph(self, cache, max_ctx: int):
        """A CUDA graph of GRAPH_STEPS launches of the expert-parallel
        persistent step (each stops once ``log_count`` reaches ``step_limit``),
        captured on first use for this cache."""
        _, _, _, _, bs, _, _ = cache_geometry(cache, 0)
        k0 = cache_geometry(cache, 0)[0]
        table = getattr(cache, "block_table_device", None)
        key = ("step", k0.data_ptr(), None if table is None else table.data_ptr(), self.runner.splits_for(max_ctx, bs))
        hit = self._graphs.get(key)
        if hit is not None:
            return hit[0]
        desc, layers = self._step_desc(cache, max_ctx)
        r = self.runner
        r.done.fill_(1)  # warm-up: every CTA skips the step, no rank exchanges anything
        r.pos.zero_()
        r.launch_step(desc)
        torch.cuda.synchronize(r.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(GRAPH_STEPS):
                capi.check(r.lib.mie_decode_step(ctypes.byref(desc), capi.stream_handle(r.device)),
                           "mie_decode_step (capture)")
        self._graphs[key] = (g, desc, layers)
        return g

    def _graph(self, cache, max_ctx: int):
        """A CUDA graph of GRAPH_STEPS decode steps (kernels and all-reduces),
        captured on first use for this cache; every rank captures in the same
        order.  Steps after EOS change nothing (the kernels see the device
        flag), so replays past the requested count are harmless."""
        _, _, _, _, bs, _, _ = cache_geometry(cache, 0)
        k0 = cache_geometry(cache, 0)[0]
        table = getattr(cache, "block_table_device", None)
        key = (k0.data_ptr(), None if table is None else table.data_ptr(), self.runner.splits_for(max_ctx, bs))
        hit = self._graphs.get(key)
        if hit is not None:
            return hit[0]
        desc, layers = self._desc(cache, max_ctx)
        r = self.runner
        # warm-up outside the capture (modules, NCCL communicator) with the
        # kernels skipping (done = 1), then capture on a side stream
        r.done.fill_(1)
        stream = torch.cuda.Stream(device=r.device)
        stream.wait_stream(torch.cuda.current_stream(r.device))
        with torch.cuda.stream(stream):
            self._step(desc, capi.stream_handle(r.device))
        torch.cuda.current_stream(r.device).wait_stream(stream)
        torch.cuda.synchronize(r.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for _ in range(GRAPH_STEPS):
                self._step(desc, capi.stream_handle(r.device))
        self._graphs[key] = (g, desc, layers)
        return g

    def release_graphs(self) -> None:
        """Drop the captured graphs (they hold NCCL work: release them before
        the process group is destroyed)."""
        self._graphs.clear()

    def close(self) -> None:
        """Release the graphs and the peer all-reduce's buffers (every rank
        calls it: it synchronises the group)."""
        self.release_graphs()
        if self._peer is not None:
            self._peer.close()
            self._peer = None

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
        self.active = self.collective_for(cache, P + steps)
        if self.active == "step":
            graph = self._step_graph(cache, P + steps) if self.use_graph else None
            desc, layers = self._step_desc(cache, P + steps)
        else:
            graph = self._graph(cache, P + steps) if self.use_graph and steps % GRAPH_STEPS == 0 else None
            desc, layers = self._desc(cache, P + steps)
        r.token.fill_(first)
        r.pos.fill_(P)
        r.done.zero_()
        r.log_count.zero_()
        r.step_limit.fill_(steps)
        # Every rank's steps start together: a rank still capturing or
        # allocating would otherwise keep the others' first bounded waits on
        # its words running, and no rank still reads words of an earlier
        # decode (the collectives share the receive buffers).
        dist.barrier(self.group)
        if self.active == "step":
            if graph is not None:
                for _ in range(-(-steps // GRAPH_STEPS)):
                    graph.replay()
            else:
                for _ in range(steps):
                    r.launch_step(desc)
        elif graph is not None:
            for _ in range(steps // GRAPH_STEPS):
                graph.replay()
        else:
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
