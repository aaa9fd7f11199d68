"""Fused batch-one MoE decode on B200 (sm_100a), behind the reference API.

Drop-in for ``src/moe_engine/fused_moe.py`` of the reference engine: the same
``is_configuration_supported`` / ``is_supported`` / ``has_canonical_layout`` /
``route`` / ``decode`` entry points, argument meanings and error types.  The
three Triton launches of the reference become one persistent CUDA kernel
(``mie_moe_decode`` in ``libmie.so``) that reads only the two selected
experts' weights.

Differences from the reference, all widening what is supported:

* float32 **and** bfloat16 weights (workspaces stay float32, ``out`` follows
  the weight dtype);
* any hidden / expert-hidden size whose rows are a multiple of 16 bytes and
  at most 16 KB, 2..32 experts (top-k is 2, as in the reference);
* SwiGLU experts: pass ``w3_base`` (the "up" projection) and the kernel
  computes ``down(silu(w1 x) * (w3 x))``; without it the expert is the
  reference's ``Linear -> GELU(erf) -> Linear`` with optional biases;
* top-2 ties resolve to the lower expert id;
* quantized experts (the reference's roadmap item, moe-inference-engine.md:36,
  which has no code there): ``quantize_experts`` turns a stacked [E, rows,
  cols] weight into int8 or int4 values with one fp32 scale per group of
  ``group_size`` consecutive elements of a row, and ``decode`` takes such
  ``QuantizedExperts`` for ``w1_base`` / ``w2_base`` / ``w3_base``
  (``mie_moe_decode`` with ``expert_bits`` 8 or 4: half or a quarter of the
  bf16 expert bytes are read).
"""

from __future__ import annotations

import ctypes

import torch

from . import capi

HAS_KERNELS = capi.library_available()
# The reference exposes HAS_TRITON; callers that test it keep working.
HAS_TRITON = HAS_KERNELS

# Production shape of the reference checkpoint (fused_moe.py:27-30).
HIDDEN_DIM = 768
NUM_EXPERTS = 8
TOP_K = 2
EXPERT_HIDDEN_DIM = 3072

_SUPPORTED_DTYPES = (torch.float32, torch.bfloat16)
_MAX_ROW_BYTES = 16 * 1024


def _row_ok(n: int, dtype: torch.dtype) -> bool:
    e = 2 if dtype == torch.bfloat16 else 4
    return n > 0 and (n * e) % 16 == 0 and n * e <= _MAX_ROW_BYTES


def is_configuration_supported(
    *,
    device: torch.device,
    dtype: torch.dtype,
    batch_size: int,
    hidden_dim: int,
    num_experts: int,
    top_k: int,
    expert_hidden_dim: int,
) -> bool:
    """Whether model metadata can use the fused decode kernel (fused_moe.py:33-53)."""
    return (
        HAS_KERNELS
        and torch.device(device).type == "cuda"
        and dtype in _SUPPORTED_DTYPES
        and batch_size == 1
        and top_k == TOP_K
        and 2 <= num_experts <= 32
        and _row_ok(hidden_dim, dtype)
        and _row_ok(expert_hidden_dim, dtype)
    )


def is_supported(x: torch.Tensor, *, num_experts: int, top_k: int, expert_hidden_dim: int) -> bool:
    """Whether ``x`` ([1, 1, D]) and the model shape can use the kernel (fused_moe.py:56-74)."""
    if x.dim() != 3 or x.shape[0] != 1 or x.shape[1] != 1 or not x.is_contiguous():
        return False
    return is_configuration_supported(
        device=x.device,
        dtype=x.dtype,
        batch_size=x.shape[0],
        hidden_dim=x.shape[-1],
        num_experts=num_experts,
        top_k=top_k,
        expert_hidden_dim=expert_hidden_dim,
    )


def has_canonical_layout(
    router_weight: torch.Tensor,
    w1: torch.Tensor,
    b1: torch.Tensor | None,
    w2: torch.Tensor,
    b2: torch.Tensor | None,
    router_logits: torch.Tensor,
    expert_ids: torch.Tensor,
    route_weights: torch.Tensor,
    hidden: torch.Tensor,
    out: torch.Tensor,
    w3: torch.Tensor | None = None,
) -> bool:
    """Validate shapes, contiguity, dtypes and devices (fused_moe.py:77-114).

    Weights share one dtype (float32 or bfloat16) and device; ``router_logits``,
    ``route_weights`` and ``hidden`` are float32, ``expert_ids`` int32, ``out``
    the weight dtype.
    """
    if router_weight.dim() != 2 or w1.dim() != 3:
        return False
    E, D = router_weight.shape
    Hx = w1.shape[1]
    wdt, device = router_weight.dtype, router_weight.device
    if wdt not in _SUPPORTED_DTYPES:
        return False
    weights = [(router_weight, (E, D)), (w1, (E, Hx, D)), (w2, (E, D, Hx))]
    if b1 is not None:
        weights.append((b1, (E, Hx)))
    if b2 is not None:
        weights.append((b2, (E, D)))
    if w3 is not None:
        weights.append((w3, (E, Hx, D)))
    work = [
        (router_logits, (E,), torch.float32),
        (route_weights, (TOP_K,), torch.float32),
        (hidden, (TOP_K, Hx), torch.float32),
        (expert_ids, (TOP_K,), torch.int32),
        (out, (D,), wdt),
    ]
    return all(
        t.shape == shape and t.is_contiguous() and t.device == device and t.dtype == wdt for t, shape in weights
    ) and all(t.shape == shape and t.is_contiguous() and t.device == device and t.dtype == dt for t, shape, dt in work)


def _require_cuda(*tensors: torch.Tensor) -> None:
    """fused_moe.py:265-271, widened to bfloat16."""
    if not HAS_KERNELS or any(not t.is_cuda for t in tensors):
        raise RuntimeError("direct MoE needs CUDA and the sm_100a kernels (libmie.so)")
    if any(t.dtype not in _SUPPORTED_DTYPES for t in tensors):
        raise RuntimeError("direct MoE needs float32 or bfloat16 activations and parameters")
    if any(t.device != tensors[0].device for t in tensors[1:]):
        raise ValueError("direct MoE tensors must be on the same CUDA device")


_SYNC_WORDS: dict = {}


def _sync_words(device: torch.device) -> torch.Tensor:
    """Grid-barrier words shared by calls on one device (zeroed once)."""
    key = (device.type, device.index)
    t = _SYNC_WORDS.get(key)
    if t is None:
        t = torch.zeros(4, dtype=torch.int32, device=device)
        _SYNC_WORDS[key] = t
    return t


class QuantizedExperts:
    """Stacked expert weights [E, rows, cols] quantized in groups of
    ``group_size`` consecutive elements of each row, symmetric:
    ``w[e, r, i] ~ scale[e, r, i // group_size] * q[e, r, i]`` with
    ``|q| <= 127`` (``bits`` 8, ``q`` int8 [E, rows, cols]) or ``|q| <= 7``
    (``bits`` 4, ``q`` uint8 [E, rows, cols / 2] holding two values per byte,
    the even element in the low nibble)."""

    def __init__(self, q: torch.Tensor, scale: torch.Tensor, bits: int, group_size: int, shape):
        self.q, self.scale, self.bits, self.group_size = q, scale, bits, group_size
        self.shape = torch.Size(shape)

    @property
    def device(self):
        return self.q.device

    @property
    def is_cuda(self):
        return self.q.is_cuda

    def to(self, device) -> "QuantizedExperts":
        return QuantizedExperts(self.q.to(device), self.scale.to(device), self.bits, self.group_size, self.shape)

    def nbytes(self) -> int:
        return self.q.numel() * self.q.element_size() + self.scale.numel() * 4


def quantize_experts(w: torch.Tensor, bits: int = 8, group_size: int = 128) -> QuantizedExperts:
    """Groupwise symmetric absmax quantization of a stacked [E, rows, cols]
    weight: per group, ``scale = max|w| / qmax`` (fp32, qmax 127 or 7) and
    ``q = clamp(round_half_even(w / scale), -qmax, qmax)`` (0 where the group
    is all zero)."""
    if bits not in (8, 4):
        raise ValueError(f"expert weights quantize to 8 or 4 bits, not {bits}")
    if w.dim() != 3:
        raise ValueError("quantize_experts needs a stacked [E, rows, cols] weight")
    E, R, C = w.shape
    if group_size < 32 or group_size & (group_size - 1) or C % group_size:
        raise ValueError(f"group_size must be a power of two >= 32 dividing the row length {C}")
    qmax = 127 if bits == 8 else 7
    g = w.detach().float().reshape(E, R, C // group_size, group_size)
    amax = g.abs().amax(-1)
    # tensor / tensor: a correctly rounded division on every device (a CUDA
    # division by a Python scalar multiplies by its reciprocal instead)
    scale = amax / torch.full_like(amax, float(qmax))
    safe = torch.where(scale > 0, scale, torch.ones_like(scale))
    q = torch.clamp(torch.round(g / safe.unsqueeze(-1)), -qmax, qmax).to(torch.int8).reshape(E, R, C)
    if bits == 4:
        u = (q.to(torch.int16) & 0xF).to(torch.uint8)
        q = u[..., 0::2] | (u[..., 1::2] << 4)
    return QuantizedExperts(q.contiguous(), scale.contiguous(), bits, group_size, (E, R, C))


def dequantize_experts(qe: QuantizedExperts) -> torch.Tensor:
    """The fp32 weights a QuantizedExperts stands for: scale * q."""
    E, R, C = qe.shape
    if qe.bits == 4:
        lo = (qe.q & 0xF).to(torch.int16)
        hi = ((qe.q >> 4) & 0xF).to(torch.int16)
        lo = torch.where(lo >= 8, lo - 16, lo)
        hi = torch.where(hi >= 8, hi - 16, hi)
        q = torch.stack((lo, hi), dim=-1).reshape(E, R, C)
    else:
        q = qe.q
    g = q.float().reshape(E, R, C // qe.group_size, qe.group_size)
    return (g * qe.scale.unsqueeze(-1)).reshape(E, R, C)


def _args(x, router_weight, w1, b1, w2, b2, w3, router_logits, expert_ids, route_weights, hidden, out, sync):
    E, D = router_weight.shape
    a = capi.MoeArgs()
    a.dtype = capi.dtype_code(router_weight.dtype)
    a.x_dtype = capi.dtype_code(x.dtype)
    a.out_dtype = capi.dtype_code(out.dtype) if out is not None else a.dtype
    a.hidden_dim = D
    a.expert_hidden_dim = w1.shape[1] if w1 is not None else 16
    a.num_experts = E
    a.top_k = TOP_K
    a.act = capi.MIE_ACT_SWIGLU if w3 is not None else capi.MIE_ACT_GELU
    a.norm = capi.MIE_NORM_NONE
    a.x = capi.ptr(x)
    a.router_w = capi.ptr(router_weight)
    a.w1, a.b1, a.w3, a.w2, a.b2 = (capi.ptr(t) for t in (w1, b1, w3, w2, b2))
    a.router_logits = capi.ptr(router_logits)
    a.expert_ids = capi.ptr(expert_ids)
    a.route_weights = capi.ptr(route_weights)
    a.hidden = capi.ptr(hidden)
    a.out = capi.ptr(out)
    a.residual = 0
    a.sync = capi.ptr(sync)
    return a


def route(
    x: torch.Tensor,
    router_weight: torch.Tensor,
    router_logits: torch.Tensor,
    expert_ids: torch.Tensor,
    route_weights: torch.Tensor,
) -> None:
    """Router GEMV + top-2 + 2-way softmax into the workspaces (fused_moe.py:274-309)."""
    _require_cuda(x, router_weight)
    E = router_weight.shape[0] if router_weight.dim() == 2 else -1
    D = router_weight.shape[1] if router_weight.dim() == 2 else -1
    if (
        x.numel() != D
        or not x.is_contiguous()
        or router_weight.dim() != 2
        or not router_weight.is_contiguous()
        or not 2 <= E <= 32
    ):
        raise ValueError("direct MoE router needs x [D] and router weight [E, D]")
    if (
        not expert_ids.is_cuda
        or expert_ids.device != x.device
        or expert_ids.dtype != torch.int32
        or expert_ids.shape != (TOP_K,)
    ):
        raise ValueError("direct MoE expert id workspace must be CUDA int32")
    if (
        router_logits.shape != (E,)
        or route_weights.shape != (TOP_K,)
        or router_logits.dtype != torch.float32
        or route_weights.dtype != torch.float32
    ):
        raise ValueError("direct MoE router workspaces have invalid shapes")
    lib = capi.ensure_init(x.device)
    a = _args(x, router_weight, None, None, None, None, None, router_logits, expert_ids, route_weights, None, None, None)
    capi.check(lib.mie_moe_route(ctypes.byref(a), capi.stream_handle(x.device)), "mie_moe_route")


def decode(
    x: torch.Tensor,
    router_weight: torch.Tensor,
    w1_base: torch.Tensor,
    b1_base: torch.Tensor | None,
    w2_base: torch.Tensor,
    b2_base: torch.Tensor | None,
    *,
    router_logits: torch.Tensor,
    expert_ids: torch.Tensor,
    route_weights: torch.Tensor,
    hidden: torch.Tensor,
    out: torch.Tensor,
    w3_base: torch.Tensor | None = None,
    sync: torch.Tensor | None = None,
) -> torch.Tensor:
    """Router, the two selected experts and the weighted combine in one launch.

    Same signature and workspaces as fused_moe.py:312-380; ``w3_base`` selects
    SwiGLU experts, ``sync`` (int32 [4], zeroed once) holds the kernel's grid
    barrier words (a per-device default is used when omitted).  Returns
    ``out.view(1, 1, D)``.
    """
    if isinstance(w1_base, QuantizedExperts):
        return _decode_quantized(x, router_weight, w1_base, b1_base, w2_base, b2_base, router_logits, expert_ids,
                                 route_weights, hidden, out, w3_base, sync)
    tensors = [x, router_weight, w1_base, w2_base, router_logits, route_weights, hidden, out]
    tensors += [t for t in (b1_base, b2_base, w3_base) if t is not None]
    _require_cuda(*tensors)
    if not has_canonical_layout(
        router_weight, w1_base, b1_base, w2_base, b2_base, router_logits, expert_ids, route_weights, hidden, out,
        w3_base,
    ):
        raise ValueError("direct MoE weights and workspaces must use canonical layouts")
    D = router_weight.shape[1]
    if x.numel() != D or not x.is_contiguous():
        raise ValueError("direct MoE needs one contiguous token x of the router's width")
    if sync is None:
        sync = _sync_words(x.device)
    lib = capi.ensure_init(x.device)
    a = _args(x, router_weight, w1_base, b1_base, w2_base, b2_base, w3_base, router_logits, expert_ids,
              route_weights, hidden, out, sync)
    capi.check(lib.mie_moe_decode(ctypes.byref(a), capi.stream_handle(x.device)), "mie_moe_decode")
    return out.view(1, 1, D)


def _decode_quantized(x, router_weight, w1, b1, w2, b2, router_logits, expert_ids, route_weights, hidden, out, w3,
                      sync):
    """``decode`` with QuantizedExperts for w1 / w2 (/ w3): the same launch
    with ``expert_bits`` and the group scales set."""
    quant = [w1, w2] + ([w3] if w3 is not None else [])
    if not all(isinstance(q, QuantizedExperts) for q in quant):
        raise ValueError("quantized MoE needs QuantizedExperts for w1, w2 (and w3)")
    if len({(q.bits, q.group_size) for q in quant}) != 1:
        raise ValueError("quantized MoE weights must share bits and group size")
    tensors = [x, router_weight, router_logits, route_weights, hidden, out]
    tensors += [t for t in (b1, b2) if t is not None]
    _require_cuda(*tensors)
    if any(q.device != x.device for q in quant):
        raise ValueError("direct MoE tensors must be on the same CUDA device")
    if router_weight.dim() != 2:
        raise ValueError("direct MoE router weight must be [E, D]")
    E, D = router_weight.shape
    Hx = w1.shape[1]
    rows = [(w1, (E, Hx, D)), (w2, (E, D, Hx))] + ([(w3, (E, Hx, D))] if w3 is not None else [])
    wdt = router_weight.dtype
    ok = all(q.shape == shape and q.q.is_contiguous() and q.scale.is_contiguous() and q.scale.dtype == torch.float32
             for q, shape in rows)
    ok = ok and router_weight.is_contiguous() and all(
        t is None or (t.is_contiguous() and t.dtype == wdt and t.shape == shape)
        for t, shape in ((b1, (E, Hx)), (b2, (E, D))))
    ok = ok and (router_logits.shape == (E,) and router_logits.dtype == torch.float32
                 and route_weights.shape == (TOP_K,) and route_weights.dtype == torch.float32
                 and hidden.shape == (TOP_K, Hx) and hidden.dtype == torch.float32 and hidden.is_contiguous()
                 and expert_ids.shape == (TOP_K,) and expert_ids.dtype == torch.int32
                 and out.numel() == D and out.dtype == wdt and out.is_contiguous())
    if not ok:
        raise ValueError("direct MoE weights and workspaces must use canonical layouts")
    if x.numel() != D or not x.is_contiguous():
        raise ValueError("direct MoE needs one contiguous token x of the router's width")
    if sync is None:
        sync = _sync_words(x.device)
    lib = capi.ensure_init(x.device)
    a = _args(x, router_weight, w1.q, b1, w2.q, b2, w3.q if w3 is not None else None, router_logits, expert_ids,
              route_weights, hidden, out, sync)
    a.expert_hidden_dim = Hx
    a.expert_bits, a.group_size = w1.bits, w1.group_size
    a.w1_scale, a.w2_scale = w1.scale.data_ptr(), w2.scale.data_ptr()
    a.w3_scale = w3.scale.data_ptr() if w3 is not None else None
    capi.check(lib.mie_moe_decode(ctypes.byref(a), capi.stream_handle(x.device)), "mie_moe_decode")
    return out.view(1, 1, D)
