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

import torch

from . import capi


def gemm(a: torch.Tensor, b: torch.Tensor, *, out: torch.Tensor | None = None, epilogue: int = capi.GEMM_F32,
         b2: torch.Tensor | None = None, resid: torch.Tensor | None = None, counts: torch.Tensor | None = None,
         groups: int = 1, rows: int | None = None, a_group_rows: int = 0, b_group_rows: int = 0,
         c_group_rows: int = 0, status: torch.Tensor | None = None) -> torch.Tensor:
    """C = A . B^T on the tensor cores (see ``mie_gemm_args`` in include/mie.h).

    ``a`` [rows, K] and ``b`` [N, K] (``b2`` [N, K] gate/up pair for SwiGLU,
    where the output has N columns per operand) are bf16 row-major.  Grouped
    form: ``groups`` > 1 or ``counts`` (int32, device) set; ``rows`` is then
    the row capacity of one group.
    """
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise ValueError("mie_gemm takes bf16 operands")
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
        dt = torch.bfloat16 if epilogue in (capi.GEMM_BF16, capi.GEMM_SWIGLU) else torch.float32
        out = torch.empty(out_rows, out_cols, device=a.device, dtype=dt)
    args = capi.GemmArgs(
        a=a.data_ptr(), lda=a.stride(0), b=b.data_ptr(), b2=capi.ptr(b2), ldb=b.stride(0),
        b_rows=b.shape[0], c=out.data_ptr(), ldc=out.stride(0), resid=capi.ptr(resid),
        ldr=resid.stride(0) if resid is not None else 0, counts=capi.ptr(counts), M=M, N=N, K=K,
        epilogue=epilogue, groups=groups, a_group_rows=a_group_rows, b_group_rows=b_group_rows,
        c_group_rows=c_group_rows, status=capi.ptr(status),
    )
    lib = capi.ensure_init(a.device)
    capi.check(lib.mie_gemm(ctypes.byref(args), capi.stream_handle(a.device)), "mie_gemm")
    return out
