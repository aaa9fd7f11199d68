"""Fused decode step: one launch sequence of sm_100a kernels per token.

A decode step of the reference (``Model.forward`` with one token,
src/moe_engine/model.py:543-565) becomes, per layer,

    qkv   norm -> QKV GEMV -> RoPE -> K/V store at the device position
    attn  split-K attention over the cache with an in-launch LSE merge
    proj  out_proj + residual
    moe   norm -> router -> top-2 -> selected experts -> combine + residual

followed by ``lmhead`` (final norm -> tied LM head -> argmax, position += 1,
EOS flag, token log).  All launches use programmatic dependent launch so a
kernel fetches its weights while its predecessor still runs.

The position, the input token and the EOS flag live on the device, so one
step can be captured once as a CUDA graph and replayed for every token;
greedy generation replays it in chunks and reads the produced tokens back
once per chunk (:func:`greedy_generate`).
"""

from __future__ import annotations

import ctypes
import math
import os

import torch
import torch.nn.functional as F

from . import capi
from .paged_attention import MAX_SPLITS, SUPPORTED_HEAD_DIMS, cache_geometry

EOS_TOKEN_ID = 50256
CHUNK_STEPS = 64  # decode steps between host reads of the token log
# Persistent step: launches captured per graph.  Consecutive launches are
# programmatic-dependent, so each step's CTAs stage their first weights while
# the previous step's last CTA finishes; a device step limit stops the extra
# launches of the last graph of a chunk.
GRAPH_STEPS = 8


def _row_ok(n: int, dtype) -> bool:
    e = 2 if dtype == torch.bfloat16 else 4
    return (n * e) % 16 == 0 and n * e <= 16 * 1024


class DecodeRunner:
    """Device state, scratch and step descriptors for one model on one GPU."""

    @staticmethod
    def supports(model, cache, batch: int) -> bool:
        cfg = model.config
        w = model.token_embedding.weight
        if batch != 1 or w.device.type != "cuda" or not capi.library_available():
            return False
        if w.dtype not in (torch.float32, torch.bfloat16):
            return False
        if getattr(cache, "attention_mode", "gather") == "gather":
            return False
        kv = cache.allocator.k_pool if hasattr(cache, "allocator") else cache.k
        if kv.dtype != w.dtype or kv.device != w.device:
            return False
        if not hasattr(cache, "allocator") and cache.k.shape[1] != 1:
            return False
        hd = cfg.head_dim
        if hd not in SUPPORTED_HEAD_DIMS or cfg.num_heads * hd != cfg.hidden_dim or cfg.top_k != 2:
            return False
        if not (_row_ok(cfg.hidden_dim, w.dtype) and _row_ok(cfg.expert_hidden, w.dtype)):
            return False
        for block in model.MoEBlocks:
            if block.moe.mode == "reference" or not block.moe.direct_configuration_supported(1):
                return False
        if DecodeRunner._quant_format(model) is None:  # quantized layers must share bits and groups
            return False
        return all(p.dtype == w.dtype and p.device == w.device for p in model.parameters())

    @staticmethod
    def _quant_format(model):
        """(bits, group size) of the model's quantized experts, (0, 0) when none
        is quantized, None when the layers disagree (or only some are)."""
        fmts = set()
        for block in model.MoEBlocks:
            q = getattr(block.moe, "_quant", None)
            if not q:
                fmts.add((0, 0))
                continue
            f = {(qe.bits, qe.group_size) for qe in q.values()}
            if len(f) != 1 or set(q) != ({"w1", "w2", "w3"} & set(block.moe._expert_storage)):
                return None
            fmts.add(f.pop())
        return fmts.pop() if len(fmts) == 1 else None

    def __init__(self, model, expert_base: int = 0, expert_count: int = 0, moe_partial: bool = False):
        cfg = model.config
        self.model = model
        self.config = cfg
        dev = model.token_embedding.weight.device
        self.device = dev
        self.lib = capi.ensure_init(dev)
        self.num_sms = self.lib.mie_num_sms(dev.index if dev.index is not None else torch.cuda.current_device())
        D, H, hd, Hx, V = cfg.hidden_dim, cfg.num_heads, cfg.head_dim, cfg.expert_hidden, cfg.vocab_size
        f32 = dict(dtype=torch.float32, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        self.x = torch.zeros(D, **f32)
        self.q = torch.zeros(H * hd, **f32)
        self.attn_out = torch.zeros(H * hd, **f32)
        self.moe_hidden = torch.zeros(2 * Hx, **f32)
        self.moe_partial = torch.zeros(D, **f32) if moe_partial else None
        self.expert_base, self.expert_count = expert_base, expert_count
        self.attn_partials = torch.zeros(H * MAX_SPLITS * (hd + 2), **f32)
        self.attn_counters = torch.zeros(H, **i32)
        self.moe_sync = torch.zeros(4, **i32)
        self.lm_grid = self.num_sms
        self.lm_partial_val = torch.zeros(self.lm_grid, **f32)
        self.lm_partial_idx = torch.zeros(self.lm_grid, **i32)
        self.lm_counter = torch.zeros(1, **i32)
        self.logits = torch.zeros(V, **f32)
        self.status = torch.zeros(1, **i32)
        self.token = torch.zeros(1, dtype=torch.int64, device=dev)
        self.pos = torch.zeros(1, **i32)
        self.done = torch.zeros(1, **i32)
        self.log_capacity = cfg.max_seq_length + 1
        self.tokens_log = torch.zeros(self.log_capacity, dtype=torch.int64, device=dev)
        self.log_count = torch.zeros(1, **i32)
        # (log_count, done) after each queued chunk of steps; two chunks in flight
        self._host_states = [torch.zeros(2, dtype=torch.int32, pin_memory=True) for _ in range(2)]
        self.sample_seed = torch.zeros(1, dtype=torch.int64, device=dev)  # device sampler stream
        self.step_limit = torch.zeros(1, **i32)  # multi-step graphs: tokens to log before steps stop
        self._graphs: dict = {}
        self.use_pdl = True
        # Persistent step (one launch per token) whenever the shapes allow it;
        # MIE_PERSISTENT=0 selects the per-op launch sequence.
        self.persistent = os.environ.get("MIE_PERSISTENT", "1") != "0"
        self.step_scratch = None  # int64 words, zeroed once
        # Persistent step: limit of every device-side wait (0: the library's
        # default, 200 ms) and an optional start gate (an int32 device flag the
        # step waits for before it reads its input).
        self.wait_limit_ns = 0
        self.start_gate = None
        # which persistent kernel: capi.MIE_STEP_AUTO (the cluster step when it
        # takes the shapes), MIE_STEP_FLAT or MIE_STEP_CLUSTER
        self.step_kernel = int(os.environ.get("MIE_STEP_KERNEL", "0"))

    # ---- descriptors --------------------------------------------------------
    def param_signature(self):
        quant = tuple(qe.q.data_ptr() for b in self.model.MoEBlocks for qe in (getattr(b.moe, "_quant", None) or {}).values())
        return tuple(p.data_ptr() for p in self.model.parameters()) + quant

    def splits_for(self, max_ctx: int, block_size: int) -> int:
        nblk = -(-max_ctx // block_size)
        want = -(-self.num_sms // self.config.num_heads)
        return max(1, min(want, max(1, -(-nblk // 2)), MAX_SPLITS))

    def _layers(self, cache):
        m = self.model
        n_layers = self.config.num_layers
        arr = (capi.LayerDesc * n_layers)()
        p = capi.ptr
        for i, blk in enumerate(m.MoEBlocks):
            L = arr[i]
            att, moe = blk.attention, blk.moe
            s = moe._expert_storage
            L.attn_norm_w = p(blk.attn_norm.weight)
            L.attn_norm_b = p(getattr(blk.attn_norm, "bias", None))
            L.qkv_w = p(att.in_proj_weight)
            L.qkv_b = p(att.in_proj_bias)
            L.out_w = p(att.out_proj.weight)
            L.out_b = p(att.out_proj.bias)
            L.moe_norm_w = p(blk.moe_norm.weight)
            L.moe_norm_b = p(getattr(blk.moe_norm, "bias", None))
            L.router_w = p(moe.router.weight)
            eb = self.expert_base
            def view(t):
                if t is None or not self.expert_count:
                    return p(t)
                return t[eb].data_ptr()
            L.w1, L.b1, L.w3, L.w2, L.b2 = (view(s.get(k)) for k in ("w1", "b1", "w3", "w2", "b2"))
            quant = getattr(moe, "_quant", None)
            if quant:  # the quantized values and their group scales replace the expert weights
                L.w1, L.w3, L.w2 = (view(quant[k].q) if k in quant else None for k in ("w1", "w3", "w2"))
                L.w1_scale, L.w3_scale, L.w2_scale = (view(quant[k].scale) if k in quant else None
                                                      for k in ("w1", "w3", "w2"))
            k, v, *_ = cache_geometry(cache, i)
            L.k_cache, L.v_cache = k.data_ptr(), v.data_ptr()
        return arr

    def make_desc(self, cache, *, logits: bool, graph: bool, splits: int, sample=(0.0, 0), limit: bool = False,
                  moe_peer=None):
        """Step descriptor; ``sample`` = (temperature, top_k) selects the device
        sampler (persistent step only) instead of the greedy argmax; ``limit``
        makes steps stop once ``log_count`` reaches ``step_limit``;
        ``moe_peer`` (the address of a ``capi.PeerReduceArgs``) makes the
        persistent step expert parallel, its ranks' MoE partials summed inside
        the step (``moe_partial`` is then not used)."""
        cfg, m = self.config, self.model
        w = m.token_embedding.weight
        d = capi.StepDesc()
        d.dtype = capi.dtype_code(w.dtype)
        _, kv0, table, nb, bs, (s_blk, s_head, s_tok), _ = cache_geometry(cache, 0)
        d.kv_dtype = capi.dtype_code(kv0.dtype)
        d.num_layers = cfg.num_layers
        d.hidden_dim = cfg.hidden_dim
        d.num_heads = cfg.num_heads
        d.head_dim = cfg.head_dim
        d.num_experts = cfg.num_experts
        d.top_k = cfg.top_k
        d.expert_hidden_dim = cfg.expert_hidden
        d.vocab = cfg.vocab_size
        d.norm = capi.MIE_NORM_RMS if cfg.norm == "rms" else capi.MIE_NORM_LAYER
        d.act = capi.MIE_ACT_SWIGLU if cfg.expert_act == "swiglu" else capi.MIE_ACT_GELU
        d.eps = cfg.norm_eps
        d.attn_scale = 1.0 / math.sqrt(cfg.head_dim)
        if table is not None:
            d.max_pos = min(cfg.max_seq_length, nb * bs)
        else:
            d.max_pos = min(cfg.max_seq_length, cache.k.shape[3])
        layers = self._layers(cache)
        d.layers = ctypes.cast(layers, ctypes.c_void_p)
        d.embedding = w.data_ptr()
        pe = getattr(m, "positional_embedding", None)
        d.pos_embedding = capi.ptr(pe.weight) if pe is not None else None
        d.final_norm_w = capi.ptr(m.final_norm.weight)
        d.final_norm_b = capi.ptr(getattr(m.final_norm, "bias", None))
        d.lm_bias = capi.ptr(m.output_projection.bias)
        if cfg.pos == "rope":
            d.rope_cos, d.rope_sin = m.rope_cos.data_ptr(), m.rope_sin.data_ptr()
        d.block_table = capi.ptr(table)
        d.num_blocks = nb
        d.block_size = bs
        d.kv_stride_block, d.kv_stride_head, d.kv_stride_tok = s_blk, s_head, s_tok
        d.token = self.token.data_ptr()
        d.pos = self.pos.data_ptr()
        d.done = self.done.data_ptr() if graph else None
        d.eos_id = EOS_TOKEN_ID
        d.tokens_log = self.tokens_log.data_ptr() if graph else None
        d.log_count = self.log_count.data_ptr() if graph else None
        d.log_capacity = self.log_capacity
        d.x = self.x.data_ptr()
        d.q = self.q.data_ptr()
        d.attn_out = self.attn_out.data_ptr()
        d.moe_hidden = self.moe_hidden.data_ptr()
        d.moe_partial = None if moe_peer else capi.ptr(self.moe_partial)
        d.moe_peer = moe_peer
        d.expert_bits, d.group_size = self._quant_format(m) or (0, 0)
        d.expert_base = self.expert_base
        d.expert_count = self.expert_count
        d.attn_partials = self.attn_partials.data_ptr()
        d.attn_counters = self.attn_counters.data_ptr()
        d.moe_sync = self.moe_sync.data_ptr()
        d.lm_partial_val = self.lm_partial_val.data_ptr()
        d.lm_partial_idx = self.lm_partial_idx.data_ptr()
        d.lm_counter = self.lm_counter.data_ptr()
        d.logits = self.logits.data_ptr() if logits else None
        d.status = self.status.data_ptr()
        d.attn_splits = splits
        d.max_splits = MAX_SPLITS
        d.lm_grid = self.lm_grid
        d.use_pdl = 1 if self.use_pdl else 0
        d.sample_temperature = float(sample[0])
        d.sample_top_k = int(sample[1])
        d.sample_seed = self.sample_seed.data_ptr()
        d.step_limit = self.step_limit.data_ptr() if limit and graph else None
        d.step_scratch = None
        d.step_scratch_bytes = 0
        d.wait_limit_ns = int(self.wait_limit_ns)
        d.start_gate = capi.ptr(self.start_gate)
        d.step_kernel = int(self.step_kernel)
        if self.persistent:
            with torch.cuda.device(self.device):
                need = int(self.lib.mie_step_scratch_bytes(ctypes.byref(d)))
            if need > 0:
                if self.step_scratch is None or self.step_scratch.numel() * 8 < need:
                    self.step_scratch = torch.zeros(-(-need // 8), dtype=torch.int64, device=self.device)
                d.step_scratch = self.step_scratch.data_ptr()
                d.step_scratch_bytes = self.step_scratch.numel() * 8
        return d, layers

    def uses_persistent(self, cache) -> bool:
        """True when decode steps for ``cache`` run as one persistent launch."""
        _, _, _, _, bs, _, _ = cache_geometry(cache, 0)
        desc, _ = self.make_desc(cache, logits=False, graph=True, splits=self.splits_for(bs, bs))
        return bool(desc.step_scratch)

    def step_kernel_for(self, cache) -> int:
        """capi.MIE_STEP_CLUSTER or MIE_STEP_FLAT: the persistent kernel that
        runs decode steps for ``cache`` (0 when steps run as the per-op
        launch sequence)."""
        _, _, _, _, bs, _, _ = cache_geometry(cache, 0)
        desc, _ = self.make_desc(cache, logits=False, graph=True, splits=self.splits_for(bs, bs))
        if not desc.step_scratch:
            return 0
        with torch.cuda.device(self.device):
            k = int(self.lib.mie_step_kernel_of(ctypes.byref(desc)))
        return max(k, 0)

    def steps_per_graph(self, cache) -> int:
        """Decode steps one graph of :meth:`graph_for` may hold for ``cache``:
        GRAPH_STEPS for the persistent step (which honours ``step_limit``),
        else 1."""
        return GRAPH_STEPS if self.uses_persistent(cache) else 1

    # ---- execution ------------------------------------------------------------
    def launch_step(self, desc) -> None:
        capi.check(self.lib.mie_decode_step(ctypes.byref(desc), capi.stream_handle(self.device)), "mie_decode_step")

    def check_status(self) -> None:
        """Synchronise and raise if any kernel recorded a device-side failure."""
        code = int(self.status.item())
        if code:
            self.status.zero_()
            # a step that gave up leaves exchange words and counters mid-step
            if self.step_scratch is not None:
                self.step_scratch.zero_()
            self.lm_counter.zero_()
            raise capi.KernelError(code, "decode step (device status)")

    @torch.no_grad()
    def forward_step(self, token_ids: torch.Tensor, cache) -> torch.Tensor:
        """One eager fused decode step; returns logits [1, 1, V] in the model dtype."""
        position = cache.position
        cache.reserve(position + 1)
        self.token.copy_(token_ids.reshape(1))
        self.pos.fill_(position)
        _, _, _, _, bs, _, _ = cache_geometry(cache, 0)
        desc, layers = self.make_desc(cache, logits=True, graph=False, splits=self.splits_for(position + 1, bs))
        self.launch_step(desc)
        del layers
        cache.position += 1
        dt = self.model.token_embedding.weight.dtype
        return self.logits.to(dt, copy=True).view(1, 1, -1)

    def supports_sampling(self, cache, temperature: float, top_k) -> bool:
        """Whether decode steps for ``cache`` can sample on the device."""
        if temperature <= 0 or (top_k is not None and top_k > 64):
            return False
        _, _, _, _, bs, _, _ = cache_geometry(cache, 0)
        desc, _ = self.make_desc(cache, logits=False, graph=True, splits=self.splits_for(bs, bs),
                                 sample=(temperature, top_k or 0))
        return bool(desc.step_scratch)

    def graph_for(self, cache, max_ctx: int, sample=(0.0, 0), steps: int = 1):
        """The captured decode step for ``cache`` (captured on first use).

        With ``steps`` > 1 the graph holds that many step launches (persistent
        step only, see :meth:`steps_per_graph`) and every replay decodes up to
        ``steps`` tokens: the caller sets ``step_limit`` to the ``log_count``
        at which steps stop."""
        _, _, _, _, bs, _, _ = cache_geometry(cache, 0)
        splits = self.splits_for(max_ctx, bs)
        k0 = cache_geometry(cache, 0)[0]
        table = getattr(cache, "block_table_device", None)
        key = (k0.data_ptr(), None if table is None else table.data_ptr(), splits, self.use_pdl,
               self.persistent, self.step_kernel, self.param_signature(), tuple(sample), steps)
        hit = self._graphs.get(key)
        if hit is not None:
            return hit[0]
        if len(self._graphs) >= 4:
            self._graphs.clear()
        desc, layers = self.make_desc(cache, logits=False, graph=True, splits=splits, sample=sample,
                                      limit=steps > 1)
        if steps > 1 and not desc.step_scratch:
            raise ValueError("several steps per graph need the persistent step")
        # Warm-up with every kernel skipping (done = 1): loads modules, touches
        # nothing; then capture.
        self.done.fill_(1)
        self.pos.zero_()
        self.launch_step(desc)
        torch.cuda.current_stream(self.device).synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(steps):
                rc = self.lib.mie_decode_step(ctypes.byref(desc), capi.stream_handle(self.device))
                if rc:
                    break
        capi.check(rc, "mie_decode_step (capture)")
        self._graphs[key] = (g, desc, layers)
        return g


@torch.no_grad()
def sample_logits(logits: torch.Tensor, temperature: float, top_k) -> torch.Tensor:
    """The reference's sampling of one position's logits (model.py:604-613)."""
    logits = logits.float() / temperature
    if top_k is not None:
        k = min(top_k, logits.size(-1))
        values, _ = torch.topk(logits, k)
        logits[logits < values[..., [-1]]] = -float("inf")
    return torch.multinomial(F.softmax(logits, dim=-1), num_samples=1)


def greedy_generate(model, token_ids: torch.Tensor, max_new_tokens: int, cache, temperature: float = 0.0,
                    top_k=None) -> torch.Tensor:
    """``Model.generate`` with the decode step replayed as a CUDA graph.

    Same results and cache effects as the step-by-step loop (model.py:596-621):
    iteration 0 is the prompt prefill; each further iteration is one graph
    replay; EOS stops generation on the device (later replays are no-ops) and
    the loop ends when the context is full.  With temperature > 0 the first
    token is sampled from the prefill logits as the reference does and every
    later one by the step kernel's device sampler, its random stream seeded
    from torch's default generator (so torch.manual_seed makes a run
    reproducible).
    """
    runner = model.decode_runner()
    max_seq = model.max_seq_length
    logits = model(token_ids, cache)  # prefill (position 0)
    if temperature > 0:
        first = int(sample_logits(logits[0, -1], temperature, top_k).item())
        runner.sample_seed.fill_(int(torch.randint(0, 2**62, (1,)).item()))
    else:
        first = int(torch.argmax(logits[0, -1]).item())
    sample = (float(temperature), int(top_k or 0)) if temperature > 0 else (0.0, 0)
    if first == EOS_TOKEN_ID:
        return token_ids
    P = cache.position
    if P >= max_seq or max_new_tokens == 1:
        return torch.cat((token_ids, token_ids.new_tensor([[first]])), dim=1)
    K = min(max_new_tokens - 1, max_seq - P)
    M = runner.steps_per_graph(cache)
    graph = runner.graph_for(cache, P + K, sample=sample, steps=M)
    runner.token.fill_(first)
    runner.pos.fill_(P)
    runner.done.zero_()
    runner.log_count.zero_()
    produced = 0  # steps issued
    count = 0
    exhausted = False
    paged = hasattr(cache, "allocator")
    if paged:
        try:
            # the whole request at once: the block table (whose update waits
            # for the stream) is not touched while steps are queued
            cache.reserve(P + K)
        except RuntimeError:
            pass  # chunk by chunk below, as far as the pool goes
    stream = torch.cuda.current_stream(runner.device)
    inflight = []  # (host state slot, event) per queued chunk, oldest first
    slot = 0
    while True:
        # keep two chunks queued, so the GPU never waits for this loop
        while produced < K and not exhausted and len(inflight) < 2:
            n = min(CHUNK_STEPS, K - produced)
            if paged and len(cache.block_table) * cache.allocator.block_size < P + produced + n:
                try:
                    cache.reserve(P + produced + n)
                except RuntimeError:
                    # Reserve what the pool still has, run up to it, then fail
                    # like the step that could not get a block.
                    bs = cache.allocator.block_size
                    while cache.allocator.free_blocks and len(cache.block_table) * bs < P + produced + n:
                        cache.reserve(len(cache.block_table) * bs + 1)
                    n = len(cache.block_table) * bs - (P + produced)
                    exhausted = True
            if n <= 0:
                break
            if M > 1:
                runner.step_limit.fill_(produced + n)
            for _ in range(-(-n // M)):
                graph.replay()
            produced += n
            state = runner._host_states[slot]
            slot ^= 1
            state[0:1].copy_(runner.log_count, non_blocking=True)
            state[1:2].copy_(runner.done, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(stream)
            inflight.append((state, ev))
        if not inflight:
            break
        state, ev = inflight.pop(0)
        ev.synchronize()
        count, done = int(state[0]), int(state[1])
        if done:
            break  # a chunk still queued runs as no-op steps
    runner.check_status()
    cache.position = P + count
    if paged:
        cache._trim(cache.position)
    new = runner.tokens_log[:count]
    if count and int(new[-1]) == EOS_TOKEN_ID and int(runner.done.item()):
        new = new[:-1]
    elif exhausted and count < K:
        raise RuntimeError("no free KV cache blocks left")
    first_t = token_ids.new_tensor([[first]])
    return torch.cat((token_ids, first_t, new.view(1, -1).to(token_ids.dtype)), dim=1)
