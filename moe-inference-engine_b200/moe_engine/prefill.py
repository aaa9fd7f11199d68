"""Prompt prefill on the B200: the projections of every layer as tcgen05
tensor-core GEMMs (``mie_gemm``).

The reference prefills the prompt through the same PyTorch module graph as
every other step (src/moe_engine/model.py:543-565): ``F.linear`` for the QKV
and out projections (model.py:226-234,268) and, for the MoE, the reference
loop over experts with a ``nonzero`` host sync per expert
(model.py:443-461).  Here the GEMMs run on the tensor cores of the sm_100a
kernels in csrc/gemm.cu.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import capi


def gemm(a: torch.Tensor, b: torch.Tensor, *, out: torch.Tensor | None = None, epilogue: int = capi.GEMM_F32,
         b2: torch.Tensor | None = None, resid: torch.Tensor | None = None, counts: torch.Tensor | None = None,
         groups: int = 1, rows: int | None = None, a_group_rows: int = 0, b_group_rows: int = 0,
         c_group_rows: int = 0, status: torch.Tensor | None = None, bias: torch.Tensor | None = None,
         bias_group_stride: int = 0) -> torch.Tensor:
    """C = A . B^T on the tensor cores (see ``mie_gemm_args`` in include/mie.h).

    ``a`` [rows, K] and ``b`` [N, K] (``b2`` [N, K] gate/up pair for SwiGLU,
    where the output has N columns per operand) are bf16 row-major.  Grouped
    form: ``groups`` > 1 or ``counts`` (int32, device) set; ``rows`` is then
    the row capacity of one group.
    """
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise ValueError("mie_gemm takes bf16 operands")
    if bias is not None and (bias.dtype != torch.bfloat16 or not bias.is_contiguous()):
        raise ValueError("mie_gemm takes a contiguous bf16 bias")
    if a.dim() != 2 or b.dim() != 2 or a.stride(1) != 1 or b.stride(1) != 1:
        raise ValueError("mie_gemm takes row-major 2-D operands")
    K = a.shape[1]
    if b.shape[1] != K or (b2 is not None and tuple(b2.shape) != tuple(b.shape)):
        raise ValueError("mie_gemm: operand widths differ")
    grouped = groups > 1 or counts is not None
    M = rows if rows is not None else (a_group_rows if grouped else a.shape[0])
    if epilogue == capi.GEMM_SWIGLU:
        if b2 is None:
            raise ValueError("SwiGLU needs the up rows (b2)")
        N = 2 * (b_group_rows if grouped else b.shape[0])
        out_cols = N // 2
    else:
        N = b_group_rows if grouped else b.shape[0]
        out_cols = N
    if out is None:
        out_rows = groups * c_group_rows if grouped else M
        dt = torch.bfloat16 if epilogue in (capi.GEMM_BF16, capi.GEMM_SWIGLU, capi.GEMM_GELU) else torch.float32
        out = torch.empty(out_rows, out_cols, device=a.device, dtype=dt)
    args = capi.GemmArgs(
        a=a.data_ptr(), lda=a.stride(0), b=b.data_ptr(), b2=capi.ptr(b2), ldb=b.stride(0),
        b_rows=b.shape[0], c=out.data_ptr(), ldc=out.stride(0), resid=capi.ptr(resid),
        ldr=resid.stride(0) if resid is not None else 0, counts=capi.ptr(counts), M=M, N=N, K=K,
        epilogue=epilogue, groups=groups, a_group_rows=a_group_rows, b_group_rows=b_group_rows,
        c_group_rows=c_group_rows, status=capi.ptr(status), bias=capi.ptr(bias),
        bias_group_stride=bias_group_stride,
    )
    lib = capi.ensure_init(a.device)
    capi.check(lib.mie_gemm(ctypes.byref(args), capi.stream_handle(a.device)), "mie_gemm")
    return out


def _kv_layout(cache, layer: int):
    """(k, v tensors of this layer, block table or None, block size, strides
    block / head / token) for the K/V slots the prefill writes."""
    if hasattr(cache, "allocator"):
        al = cache.allocator
        k, v = al.k_pool[layer], al.v_pool[layer]  # [blocks, H, bs, hd]
        return k, v, cache.block_table_device, al.block_size, k.stride(0), k.stride(1), k.stride(2)
    k, v = cache.k[layer, 0], cache.v[layer, 0]  # [H, max_seq, hd]
    return k, v, None, k.shape[1], 0, k.stride(0), k.stride(1)


class _Buffers:
    """The prefill's working tensors for one prompt length (reused by every
    prefill of that length, so a captured graph keeps valid pointers)."""

    def __init__(self, cfg, T: int, device, table_len: int):
        D, H, hd, E, Hx, V = cfg.hidden_dim, cfg.num_heads, cfg.head_dim, cfg.num_experts, cfg.expert_hidden, cfg.vocab_size
        bf, f32, i32 = dict(dtype=torch.bfloat16, device=device), dict(dtype=torch.float32, device=device), dict(
            dtype=torch.int32, device=device)
        self.ids = torch.zeros(T, dtype=torch.int64, device=device)
        self.table = torch.zeros(max(1, table_len), **i32)  # copy of the cache's block table
        self.x = torch.empty(T, D, **f32)
        self.xn = torch.empty(T, D, **bf)
        self.qkv = torch.empty(T, 3 * D, **f32)
        self.q, self.k, self.v = (torch.empty(H, T, hd, **bf) for _ in range(3))
        self.o = torch.empty(T, D, **bf)
        self.counts = torch.zeros(E, **i32)
        self.wts = torch.empty(T, 2, **f32)
        self.sel = torch.empty(T, 2, **i32)
        self.rows = torch.empty(T, 2, **i32)
        self.gathered = torch.empty(E * T, D, **bf)
        self.hbuf = torch.empty(E * T, Hx, **bf)
        self.ybuf = torch.empty(E * T, D, **f32)
        self.logits = torch.empty(T, V, **f32)


class PrefillRunner:
    """Prompt prefill of a bf16 model on the sm_100a kernels.

    Per layer: norm -> QKV GEMM (+ bias) -> RoPE + K/V cache write -> causal
    attention (``mie_prefill_attention``, in place of the reference prefill's
    SDPA, model.py:252-256) -> out_proj GEMM (+ bias) + residual -> norm ->
    router, top-2 and per-expert row gather -> grouped up GEMM (SwiGLU, or
    bias + GELU) -> grouped down GEMM (+ bias) -> weighted combine.  Then the
    final norm and the tied LM head GEMM (+ bias) for every position.  The
    residual stream stays fp32.  Both the BASELINE architecture and the
    reference's own (LayerNorm, learned positions, biased GELU experts).

    The ~150 launches of a prefill are captured once per (prompt length,
    cache storage) as a CUDA graph and replayed: the prompt ids and the
    cache's block table are copied into the runner's buffers first, so every
    request of that length replays the same graph.
    """

    MAX_GRAPHS = 4

    @staticmethod
    def supports(model, cache, token_ids) -> bool:
        cfg = model.config
        w = model.token_embedding.weight
        if token_ids.dim() != 2 or token_ids.shape[0] != 1 or token_ids.shape[1] < 2 or cache.position != 0:
            return False
        if w.device.type != "cuda" or w.dtype != torch.bfloat16 or not capi.library_available():
            return False
        if getattr(cache, "attention_mode", "gather") == "gather":
            return False
        kv = cache.allocator.k_pool if hasattr(cache, "allocator") else cache.k
        if kv.dtype != torch.bfloat16 or kv.device != w.device:
            return False
        if not hasattr(cache, "allocator") and cache.k.shape[1] != 1:
            return False
        D, Hx, V = cfg.hidden_dim, cfg.expert_hidden, cfg.vocab_size
        if cfg.top_k != 2 or not 2 <= cfg.num_experts <= 32:
            return False
        # GEMM shapes: K a multiple of 64, N a multiple of 128 (SwiGLU: 2 Hx)
        hx_align = 64 if cfg.expert_act == "swiglu" else 128
        if D % 128 or D > 1024 or Hx % hx_align or V % 128 or cfg.num_heads * cfg.head_dim != D:
            return False
        if any(block.moe.mode == "reference" for block in model.MoEBlocks):
            return False
        return all(p.dtype == torch.bfloat16 and p.device == w.device for p in model.parameters())

    def __init__(self, model):
        self.model = model
        self.cfg = model.config
        self.device = model.token_embedding.weight.device
        self.lib = capi.ensure_init(self.device)
        self.use_graph = True
        self._graphs: dict = {}

    def _call(self, name, args):
        capi.check(getattr(self.lib, name)(ctypes.byref(args), capi.stream_handle(self.device)), name)

    def _norm(self, x, w, b, out, tokens, ids=None):
        cfg = self.cfg
        m = self.model
        args = capi.PrefillNormArgs(
            tokens=tokens, hidden_dim=cfg.hidden_dim, norm=capi.MIE_NORM_RMS if cfg.norm == "rms" else capi.MIE_NORM_LAYER,
            eps=cfg.norm_eps, ids=capi.ptr(ids), embedding=m.token_embedding.weight.data_ptr(),
            pos_embedding=m.positional_embedding.weight.data_ptr() if cfg.pos == "learned" else None, pos0=0,
            x=x.data_ptr(), w=w.data_ptr(), b=capi.ptr(b), out=out.data_ptr(),
        )
        self._call("mie_prefill_norm", args)

    def _storage_key(self, cache):
        if hasattr(cache, "allocator"):
            al = cache.allocator
            return ("paged", al.k_pool.data_ptr(), al.v_pool.data_ptr(), al.block_size)
        return ("contiguous", cache.k.data_ptr(), cache.v.data_ptr())

    @torch.no_grad()
    def run(self, token_ids: torch.Tensor, cache) -> torch.Tensor:
        """Prefill ``token_ids`` [1, T] into the empty ``cache``; returns the
        logits [1, T, vocab] (model dtype) like ``Model.forward``."""
        cfg, dev = self.cfg, self.device
        T = token_ids.shape[1]
        V = cfg.vocab_size
        paged = hasattr(cache, "allocator")
        if paged:
            cache.reserve(T)
        ids = token_ids[0].to(dev, torch.int64).contiguous()
        lo, hi = torch.aminmax(ids)
        if int(lo) < 0 or int(hi) >= V:  # the embedding gather reads row ids[t]
            raise IndexError(f"token id outside [0, {V})")
        key = (T, self._storage_key(cache), self.model.param_signature() if hasattr(self.model, "param_signature")
               else tuple(p.data_ptr() for p in self.model.parameters()))
        hit = self._graphs.get(key)
        if hit is None:
            table_len = len(cache.block_table) if paged else 1
            bufs = _Buffers(cfg, T, dev, table_len)
            graph = None
            if self.use_graph:
                bufs.ids.copy_(ids)
                if paged:
                    bufs.table[:table_len].copy_(cache.block_table_device[:table_len])
                # warm-up outside the capture (module loading, tensor maps), then capture
                self._launch(bufs, cache, T)
                torch.cuda.synchronize(dev)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    self._launch(bufs, cache, T)
            if len(self._graphs) >= self.MAX_GRAPHS:
                self._graphs.pop(next(iter(self._graphs)))
            hit = (bufs, graph)
            self._graphs[key] = hit
        bufs, graph = hit
        bufs.ids.copy_(ids)
        if paged:
            n = len(cache.block_table)
            bufs.table[:n].copy_(cache.block_table_device[:n])
        if graph is not None:
            graph.replay()
        else:
            self._launch(bufs, cache, T)
        cache.position += T
        return bufs.logits.to(torch.bfloat16).view(1, T, V)

    def _launch(self, b: _Buffers, cache, T: int) -> None:
        """Every launch of one prefill of T tokens (eager, or under capture)."""
        cfg, m = self.cfg, self.model
        D, H, hd, E, Hx = cfg.hidden_dim, cfg.num_heads, cfg.head_dim, cfg.num_experts, cfg.expert_hidden
        paged = hasattr(cache, "allocator")
        cap = T
        rope = m.rope
        for i, block in enumerate(m.MoEBlocks):
            att, moe = block.attention, block.moe
            an = block.attn_norm
            self._norm(b.x, an.weight, getattr(an, "bias", None), b.xn, T, ids=b.ids if i == 0 else None)
            gemm(b.xn, att.in_proj_weight, out=b.qkv, bias=att.in_proj_bias)
            kc, vc, _, bs, sb, sh, st = _kv_layout(cache, i)
            self._call("mie_prefill_rope_kv", capi.PrefillRopeArgs(
                tokens=T, num_heads=H, head_dim=hd, pos0=0, qkv=b.qkv.data_ptr(),
                rope_cos=rope[0].data_ptr() if rope else None, rope_sin=rope[1].data_ptr() if rope else None,
                q_out=b.q.data_ptr(), k_out=b.k.data_ptr(), v_out=b.v.data_ptr(), k_cache=kc.data_ptr(),
                v_cache=vc.data_ptr(), block_table=b.table.data_ptr() if paged else None, block_size=bs,
                kv_stride_block=sb, kv_stride_head=sh, kv_stride_tok=st))
            self._call("mie_prefill_attention", capi.PrefillAttnArgs(
                tokens=T, num_heads=H, head_dim=hd, scale=1.0 / math.sqrt(hd), q=b.q.data_ptr(),
                k=b.k.data_ptr(), v=b.v.data_ptr(), out=b.o.data_ptr(), ld_out=b.o.stride(0)))
            gemm(b.o, att.out_proj.weight, out=b.x, epilogue=capi.GEMM_RESID, resid=b.x, bias=att.out_proj.bias)
            mn = block.moe_norm
            self._norm(b.x, mn.weight, getattr(mn, "bias", None), b.xn, T)
            b.counts.zero_()
            self._call("mie_prefill_route", capi.PrefillRouteArgs(
                tokens=T, hidden_dim=D, num_experts=E, group_rows=cap, x=b.xn.data_ptr(), x_res=b.x.data_ptr(),
                norm=capi.MIE_NORM_RMS if cfg.norm == "rms" else capi.MIE_NORM_LAYER, eps=cfg.norm_eps,
                norm_w=mn.weight.data_ptr(), norm_b=capi.ptr(getattr(mn, "bias", None)),
                router_w=moe.router.weight.data_ptr(), logits=None, counts=b.counts.data_ptr(),
                weights=b.wts.data_ptr(), ids_out=b.sel.data_ptr(), rows_out=b.rows.data_ptr(),
                gathered=b.gathered.data_ptr()))
            s = moe._expert_storage
            w1, w2 = s["w1"].view(E * Hx, D), s["w2"].view(E * D, Hx)
            grouped = dict(counts=b.counts, groups=E, rows=cap, a_group_rows=cap, c_group_rows=cap)
            if "w3" in s:
                gemm(b.gathered, w1, b2=s["w3"].view(E * Hx, D), out=b.hbuf, epilogue=capi.GEMM_SWIGLU,
                     b_group_rows=Hx, **grouped)
            else:
                b1 = s.get("b1")
                gemm(b.gathered, w1, out=b.hbuf, epilogue=capi.GEMM_GELU, b_group_rows=Hx,
                     bias=b1.reshape(-1) if b1 is not None else None, bias_group_stride=Hx, **grouped)
            b2 = s.get("b2")
            gemm(b.hbuf, w2, out=b.ybuf, b_group_rows=D, bias=b2.reshape(-1) if b2 is not None else None,
                 bias_group_stride=D, **grouped)
            self._call("mie_prefill_combine", capi.PrefillCombineArgs(
                tokens=T, hidden_dim=D, x=b.x.data_ptr(), y=b.ybuf.data_ptr(), ldy=b.ybuf.stride(0),
                weights=b.wts.data_ptr(), rows=b.rows.data_ptr()))
        fn = m.final_norm
        self._norm(b.x, fn.weight, getattr(fn, "bias", None), b.xn, T)
        gemm(b.xn, m.token_embedding.weight, out=b.logits, bias=m.output_projection.bias)
