"""Functional CPU restatement of the reference miniMoE decode path (TEST ONLY).

Every function names the reference lines it restates.  Paths are relative to
the reference project root (maokner/moe-inference-engine).

Two architectures are covered by one set of switches on :class:`Arch`:

* the reference architecture (``REFERENCE_ARCH``): LayerNorm with bias,
  learned position table, biased ``Linear -> GELU(erf) -> Linear`` experts,
  biased QKV / out / LM-head projections (``src/moe_engine/model.py``);
* the BASELINE architecture (``BASELINE_ARCH``): the same dataflow with three
  substitutions -- RMSNorm (eps 1e-5, weight only), RoPE (base 10000,
  half-split "rotate_half" convention applied to q and k before k is cached)
  and bias-free SwiGLU experts ``down(silu(gate x) * up x)``.

Top-k selection is an explicit repeated argmax, so ties resolve toward the
lower expert index (``torch.topk`` on CPU does not guarantee that); this is the
rule the reference's Triton router uses (``src/moe_engine/fused_moe.py:143-158``).

The oracle is the checker for the CUDA kernels and is never imported by the
product package.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace

import torch
from torch.nn import functional as F

__all__ = [
    "Arch",
    "REFERENCE_ARCH",
    "BASELINE_ARCH",
    "EOS_TOKEN_ID",
    "param_specs",
    "init_params",
    "round_params",
    "reference_state_dict",
    "norm",
    "rms_norm",
    "rope_tables",
    "apply_rope",
    "topk_lower_index",
    "route",
    "expert_forward",
    "moe_forward",
    "moe_decode_stacked",
    "attention",
    "attention_decode",
    "forward_full",
    "Decoder",
    "generate_greedy",
    "paged_slot",
    "paged_gather",
    "paged_write",
]

EOS_TOKEN_ID = 50256  # src/moe_engine/model.py:15


@dataclass(frozen=True)
class Arch:
    """Model hyperparameters (``src/moe_engine/model.py:18-27`` plus switches)."""

    vocab_size: int = 50304
    hidden_dim: int = 768
    num_layers: int = 6
    num_heads: int = 8
    num_experts: int = 8
    top_k: int = 2
    expert_hidden_dim: int = 3072
    max_seq_length: int = 1024
    norm: str = "layer"  # "layer" | "rms"
    pos: str = "learned"  # "learned" | "rope"
    expert_act: str = "gelu"  # "gelu" | "swiglu"
    bias: bool = True  # QKV / out_proj / LM-head biases
    rope_base: float = 10000.0
    norm_eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.hidden_dim // self.num_heads

    def with_(self, **kw) -> "Arch":
        return replace(self, **kw)


REFERENCE_ARCH = Arch()
BASELINE_ARCH = Arch(
    num_layers=12,
    num_heads=12,
    expert_hidden_dim=768,
    max_seq_length=1536,
    norm="rms",
    pos="rope",
    expert_act="swiglu",
    bias=False,
)


# ---------------------------------------------------------------------------
# Parameters
# ---------------------------------------------------------------------------


def param_specs(arch: Arch):
    """Ordered (name, shape, kind) list; names follow the engine's state dict.

    ``kind`` is one of ``weight`` (N(0, std)), ``bias``, ``norm_w``, ``norm_b``.
    The LM head is tied to ``token_embedding.weight`` (model.py:516).
    """
    D, V, E = arch.hidden_dim, arch.vocab_size, arch.num_experts
    Hx = arch.expert_hidden_dim
    specs = [("token_embedding.weight", (V, D), "weight")]
    if arch.pos == "learned":
        specs.append(("positional_embedding.weight", (arch.max_seq_length, D), "weight"))
    for i in range(arch.num_layers):
        p = f"MoEBlocks.{i}."
        specs.append((p + "attention.in_proj_weight", (3 * D, D), "weight"))
        if arch.bias:
            specs.append((p + "attention.in_proj_bias", (3 * D,), "bias"))
        specs.append((p + "attention.out_proj.weight", (D, D), "weight"))
        if arch.bias:
            specs.append((p + "attention.out_proj.bias", (D,), "bias"))
        for e in range(E):
            q = f"{p}moe.experts.{e}."
            if arch.expert_act == "gelu":
                specs += [
                    (q + "net.0.weight", (Hx, D), "weight"),
                    (q + "net.0.bias", (Hx,), "bias"),
                    (q + "net.2.weight", (D, Hx), "weight"),
                    (q + "net.2.bias", (D,), "bias"),
                ]
            else:
                specs += [
                    (q + "gate.weight", (Hx, D), "weight"),
                    (q + "up.weight", (Hx, D), "weight"),
                    (q + "down.weight", (D, Hx), "weight"),
                ]
        specs.append((p + "moe.router.weight", (E, D), "weight"))
        for n in ("attn_norm", "moe_norm"):
            specs.append((p + n + ".weight", (D,), "norm_w"))
            if arch.norm == "layer":
                specs.append((p + n + ".bias", (D,), "norm_b"))
    specs.append(("final_norm.weight", (D,), "norm_w"))
    if arch.norm == "layer":
        specs.append(("final_norm.bias", (D,), "norm_b"))
    if arch.bias:
        specs.append(("output_projection.bias", (V,), "bias"))
    return specs


def init_params(
    arch: Arch,
    seed: int = 0,
    std: float = 0.02,
    bias_std: float = 0.0,
    norm_std: float = 0.0,
) -> dict:
    """Seeded fp32 CPU parameters in ``param_specs`` order.

    Weights are N(0, std) as in the reference's ``_init_weights``
    (``src/moe_engine/vendored/minimoe_model.py:183-189``); biases are zero
    and norm weights one unless ``bias_std`` / ``norm_std`` ask for random
    perturbations (used by the fixtures so every bias path is observable).
    One ``torch.Generator`` seeded with ``seed`` is drawn from in spec order;
    a bias or norm tensor consumes random numbers only when its std is > 0.
    """
    g = torch.Generator().manual_seed(seed)
    out = {}
    for name, shape, kind in param_specs(arch):
        if kind == "weight":
            t = torch.randn(shape, generator=g) * std
        elif kind == "bias":
            t = torch.randn(shape, generator=g) * bias_std if bias_std > 0 else torch.zeros(shape)
        elif kind == "norm_w":
            t = 1.0 + torch.randn(shape, generator=g) * norm_std if norm_std > 0 else torch.ones(shape)
        else:
            t = torch.randn(shape, generator=g) * norm_std if norm_std > 0 else torch.zeros(shape)
        out[name] = t.float().contiguous()
    return out


def round_params(P: dict, dtype: torch.dtype) -> dict:
    """Round every parameter to ``dtype`` and back to fp32 (bf16 oracle input)."""
    return {k: v.to(dtype).float() for k, v in P.items()}


def reference_state_dict(P: dict) -> dict:
    """State dict loadable into the reference engine / vendored model.

    The tied LM head appears under both names in those modules' state dicts.
    """
    sd = dict(P)
    sd["output_projection.weight"] = P["token_embedding.weight"]
    if "output_projection.bias" not in sd:
        raise ValueError("reference modules always carry an LM-head bias")
    return sd


# ---------------------------------------------------------------------------
# Elementary ops
# ---------------------------------------------------------------------------


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """x * rsqrt(mean(x^2) + eps) * w in fp32 (BASELINE substitution for
    ``nn.LayerNorm`` at model.py:491-492,514)."""
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def norm(x: torch.Tensor, P: dict, name: str, arch: Arch) -> torch.Tensor:
    if arch.norm == "rms":
        return rms_norm(x, P[name + ".weight"], arch.norm_eps)
    D = x.shape[-1]
    return F.layer_norm(x.float(), (D,), P[name + ".weight"], P[name + ".bias"], arch.norm_eps)


def rope_tables(max_pos: int, head_dim: int, base: float):
    """cos/sin tables [max_pos, head_dim/2], angles in float64 then fp32.

    theta_i = base^(-2i/head_dim); angle(p, i) = p * theta_i.
    """
    half = head_dim // 2
    inv = base ** (-(torch.arange(half, dtype=torch.float64) * 2.0 / head_dim))
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cos(ang).float(), torch.sin(ang).float()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """rotate_half RoPE: out = [x1 c - x2 s, x2 c + x1 s] over the last dim."""
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1)


def topk_lower_index(logits: torch.Tensor, k: int):
    """Repeated argmax top-k over the last dim; ties -> lower index.

    Restates the two-argmax router of fused_moe.py:146-150 for any k.
    """
    work = logits.clone()
    ids, vals = [], []
    for _ in range(k):
        i = work.argmax(-1)
        ids.append(i)
        vals.append(work.gather(-1, i[..., None])[..., 0])
        work = work.scatter(-1, i[..., None], float("-inf"))
    return torch.stack(vals, -1), torch.stack(ids, -1)


def route(flat_x: torch.Tensor, router_w: torch.Tensor, top_k: int):
    """fp32 router + top-k + softmax over the selected logits (model.py:448-452)."""
    logits = F.linear(flat_x.float(), router_w.float())
    vals, ids = topk_lower_index(logits, top_k)
    weights = F.softmax(vals, dim=-1)
    return logits, ids, weights


def expert_forward(x: torch.Tensor, P: dict, prefix: str, arch: Arch) -> torch.Tensor:
    """One expert: GELU(erf) MLP with biases (model.py:272-282) or SwiGLU."""
    if arch.expert_act == "gelu":
        h = F.gelu(F.linear(x, P[prefix + "net.0.weight"], P[prefix + "net.0.bias"]))
        return F.linear(h, P[prefix + "net.2.weight"], P[prefix + "net.2.bias"])
    g = F.linear(x, P[prefix + "gate.weight"])
    u = F.linear(x, P[prefix + "up.weight"])
    return F.linear(F.silu(g) * u, P[prefix + "down.weight"])


def moe_forward(x: torch.Tensor, P: dict, layer: int, arch: Arch):
    """``MoEFeedForward._forward_reference`` (model.py:443-461).

    Experts are visited in ascending id order and accumulated with
    ``index_add_``, as the reference does.  Returns (out, (logits, ids, weights)).
    """
    B, T, D = x.shape
    flat = x.reshape(-1, D).float()
    p = f"MoEBlocks.{layer}.moe."
    logits, ids, weights = route(flat, P[p + "router.weight"], arch.top_k)
    out = torch.zeros_like(flat)
    for e in range(arch.num_experts):
        tok, slot = torch.where(ids == e)
        if tok.numel() == 0:
            continue
        w = weights[tok, slot].unsqueeze(-1)
        out.index_add_(0, tok, w * expert_forward(flat[tok], P, f"{p}experts.{e}.", arch))
    return out.reshape(B, T, D), (logits, ids, weights)


def moe_decode_stacked(x, router_w, w1, b1, w2, b2, w3=None, top_k=2):
    """Single-token MoE over stacked canonical storages (fused_moe.py:312-380).

    ``w1`` [E, Hx, D] (GELU fc1, or SwiGLU gate), ``w3`` [E, Hx, D] (SwiGLU
    up, None for GELU), ``w2`` [E, D, Hx]; ``b1``/``b2`` may be None.
    Returns (out [D], logits [E], ids [k], weights [k]) in fp32.
    """
    xf = x.reshape(1, -1).float()
    logits, ids, weights = route(xf, router_w, top_k)
    out = torch.zeros(xf.shape[-1])
    for e in range(router_w.shape[0]):
        hit = (ids[0] == e).nonzero()
        if hit.numel() == 0:
            continue
        wgt = weights[0, hit[0, 0]]
        pre = F.linear(xf, w1[e].float(), None if b1 is None else b1[e].float())
        if w3 is None:
            h = F.gelu(pre)
        else:
            h = F.silu(pre) * F.linear(xf, w3[e].float())
        y = F.linear(h, w2[e].float(), None if b2 is None else b2[e].float())
        out += wgt * y[0]
    return out, logits[0], ids[0], weights[0]


def attention(q, k, v, causal: bool, q_offset: int = 0):
    """Explicit softmax attention in fp32: q [.., Tq, hd], k/v [.., Tk, hd].

    Restates the SDPA calls at model.py:256,266 (scale 1/sqrt(hd)); with
    ``causal`` the query at row i (absolute position q_offset+i) sees keys
    0..q_offset+i.
    """
    scale = 1.0 / math.sqrt(q.shape[-1])
    s = torch.matmul(q.float(), k.float().transpose(-1, -2)) * scale
    if causal:
        Tq, Tk = s.shape[-2], s.shape[-1]
        qi = torch.arange(Tq)[:, None] + q_offset
        kj = torch.arange(Tk)[None, :]
        s = s.masked_fill(kj > qi, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.matmul(p, v.float())


def attention_decode(q, k, v):
    """One query per head: q [H, hd], k/v [H, T, hd] -> [H, hd] (fp32)."""
    return attention(q[:, None, :], k, v, causal=False)[:, 0, :]


# ---------------------------------------------------------------------------
# Whole-model forward passes
# ---------------------------------------------------------------------------


def _embed(P, arch, ids, positions):
    x = P["token_embedding.weight"][ids].float()
    if arch.pos == "learned":
        x = x + P["positional_embedding.weight"][positions].float()
    return x


def _qkv(h, P, layer, arch, positions, cos, sin):
    B, T, D = h.shape
    H, hd = arch.num_heads, arch.head_dim
    p = f"MoEBlocks.{layer}.attention."
    y = F.linear(h, P[p + "in_proj_weight"], P.get(p + "in_proj_bias"))
    q, k, v = y.chunk(3, dim=-1)

    def split(t):
        return t.view(B, T, H, hd).transpose(1, 2)

    q, k, v = split(q), split(k), split(v)
    if arch.pos == "rope":
        c, s = cos[positions], sin[positions]
        q, k = apply_rope(q, c, s), apply_rope(k, c, s)
    return q, k, v


def _out_proj(a, P, layer, arch):
    B, H, T, hd = a.shape
    p = f"MoEBlocks.{layer}.attention.out_proj."
    a = a.transpose(1, 2).reshape(B, T, H * hd)
    return F.linear(a, P[p + "weight"], P.get(p + "bias"))


def _lm_head(x, P, arch):
    x = norm(x, P, "final_norm", arch)
    return F.linear(x, P["token_embedding.weight"], P.get("output_projection.bias"))


def forward_full(P: dict, arch: Arch, ids: torch.Tensor) -> torch.Tensor:
    """Full causal forward without a cache (vendored/minimoe_model.py:191-217)."""
    ids = ids.long().reshape(1, -1)
    T = ids.shape[1]
    positions = torch.arange(T)
    cos = sin = None
    if arch.pos == "rope":
        cos, sin = rope_tables(T, arch.head_dim, arch.rope_base)
    x = _embed(P, arch, ids, positions)
    for layer in range(arch.num_layers):
        h = norm(x, P, f"MoEBlocks.{layer}.attn_norm", arch)
        q, k, v = _qkv(h, P, layer, arch, positions, cos, sin)
        x = x + _out_proj(attention(q, k, v, causal=T > 1), P, layer, arch)
        h = norm(x, P, f"MoEBlocks.{layer}.moe_norm", arch)
        x = x + moe_forward(h, P, layer, arch)[0]
    return _lm_head(x, P, arch)


class Decoder:
    """KV-cached forward with a contiguous cache (model.py:30-58, 543-565).

    ``kv_dtype`` rounds cached K/V the way a cache of that dtype stores them
    (bf16 for the bf16 kernels).  ``record`` keeps per-layer residual streams
    of the last forward for hidden-state comparisons, and per layer the router
    gap of the last position (second minus third largest logit): below ~1e-3 a
    bf16 computation of the same layer may select another expert pair.
    """

    def __init__(self, P: dict, arch: Arch, kv_dtype=torch.float32, max_seq=None):
        self.P, self.arch = P, arch
        S = max_seq or arch.max_seq_length
        shape = (arch.num_layers, arch.num_heads, S, arch.head_dim)
        self.k = torch.zeros(shape, dtype=kv_dtype)
        self.v = torch.zeros(shape, dtype=kv_dtype)
        self.position = 0
        self.max_seq = S
        self.cos = self.sin = None
        if arch.pos == "rope":
            self.cos, self.sin = rope_tables(S, arch.head_dim, arch.rope_base)
        self.hidden = []

    @torch.no_grad()
    def forward(self, ids: torch.Tensor, record: bool = False) -> torch.Tensor:
        arch, P = self.arch, self.P
        ids = ids.long().reshape(1, -1)
        T = ids.shape[1]
        pos0 = self.position
        if pos0 + T > self.max_seq:
            raise ValueError("KV cache is full")
        positions = torch.arange(pos0, pos0 + T)
        x = _embed(P, arch, ids, positions)
        self.hidden = []
        self.router_gap = []
        for layer in range(arch.num_layers):
            h = norm(x, P, f"MoEBlocks.{layer}.attn_norm", arch)
            q, k, v = _qkv(h, P, layer, arch, positions, self.cos, self.sin)
            self.k[layer, :, pos0 : pos0 + T] = k[0].to(self.k.dtype)
            self.v[layer, :, pos0 : pos0 + T] = v[0].to(self.v.dtype)
            keys = self.k[layer, :, : pos0 + T].float()[None]
            vals = self.v[layer, :, : pos0 + T].float()[None]
            a = attention(q, keys, vals, causal=T > 1, q_offset=pos0)
            x = x + _out_proj(a, P, layer, arch)
            h = norm(x, P, f"MoEBlocks.{layer}.moe_norm", arch)
            out, (logits, _, _) = moe_forward(h, P, layer, arch)
            x = x + out
            if record:
                self.hidden.append(x[0, -1].clone())
                top = logits[-1].sort(descending=True).values
                self.router_gap.append(float(top[arch.top_k - 1] - top[arch.top_k]))
        self.position += T
        return _lm_head(x, P, arch)


@torch.no_grad()
def generate_greedy(
    P: dict,
    arch: Arch,
    prompt,
    max_new_tokens: int,
    stop_at_eos: bool = True,
    kv_dtype=torch.float32,
    max_seq=None,
):
    """Greedy generation with ``Model.generate`` semantics (model.py:567-621).

    Returns the full sequence (prompt + new tokens) as a Python list.  With
    ``stop_at_eos`` False the EOS check is skipped.
    """
    prompt = torch.as_tensor(prompt).long().reshape(-1)
    dec = Decoder(P, arch, kv_dtype=kv_dtype, max_seq=max_seq)
    out = prompt.tolist()
    step = prompt[None]
    for _ in range(max_new_tokens):
        logits = dec.forward(step)
        nxt = int(logits[0, -1].argmax())
        if stop_at_eos and nxt == EOS_TOKEN_ID:
            return out
        out.append(nxt)
        step = torch.tensor([[nxt]])
        if dec.position >= dec.max_seq:
            break
    return out


# ---------------------------------------------------------------------------
# Paged block-table addressing (model.py:145-201)
# ---------------------------------------------------------------------------


def paged_slot(block_table, pos: int, block_size: int):
    """Logical position -> (physical block, slot) (model.py:145-147)."""
    return block_table[pos // block_size], pos % block_size


def paged_write(pool_l: torch.Tensor, block_table, pos: int, kv: torch.Tensor):
    """Store one token's [H, hd] K or V into a layer pool [nb, H, bs, hd]."""
    blk, slot = paged_slot(block_table, pos, pool_l.shape[2])
    pool_l[blk, :, slot] = kv.to(pool_l.dtype)


def paged_gather(pool_l: torch.Tensor, block_table, length: int) -> torch.Tensor:
    """Contiguous [H, length, hd] view rebuilt from a layer pool (model.py:186-201)."""
    bs = pool_l.shape[2]
    nblk = -(-length // bs)
    ids = list(block_table[:nblk])
    g = pool_l[ids]  # [nblk, H, bs, hd]
    H, hd = g.shape[1], g.shape[3]
    return g.transpose(0, 1).reshape(H, nblk * bs, hd)[:, :length]
