"""Prefill GEMM on the tcgen05 tensor cores (csrc/gemm.cu, mie_gemm) against
an fp32 PyTorch matmul of the same bf16 operands.

Tolerance: both sides accumulate the exact bf16 x bf16 products in fp32, in
different orders; |error| <= 1e-3 + 1e-3 |ref| for K = 768 with N(0, 1)
activations and N(0, 0.02) weights (bf16 outputs: one bf16 rounding more).
"""

import pytest
import torch

from moe_engine import capi
from moe_engine.prefill import gemm

pytestmark = pytest.mark.gpu
DEV = "cuda"


def operands(M, N, K, seed=0):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g).to(DEV, torch.bfloat16)
    b = (0.02 * torch.randn(N, K, generator=g)).to(DEV, torch.bfloat16)
    return a, b


def ref(a, b):
    return a.float() @ b.float().t()


@pytest.mark.parametrize("M", [512, 128, 300, 1])
@pytest.mark.parametrize("N", [2304, 768, 128])
def test_dense_fp32_out(M, N):
    a, b = operands(M, N, 768)
    out = gemm(a, b)
    torch.cuda.synchronize()
    torch.testing.assert_close(out, ref(a, b), atol=1e-3, rtol=1e-3)


def test_dense_bf16_out_and_k_multiple():
    a, b = operands(256, 384, 1536, seed=1)
    out = gemm(a, b, epilogue=capi.GEMM_BF16)
    torch.cuda.synchronize()
    assert out.dtype == torch.bfloat16
    torch.testing.assert_close(out.float(), ref(a, b), atol=2e-2, rtol=1e-2)


def test_residual_in_place():
    a, b = operands(384, 768, 768, seed=2)
    x = torch.randn(384, 768, device=DEV)
    want = x + ref(a, b)
    gemm(a, b, out=x, epilogue=capi.GEMM_RESID, resid=x)
    torch.cuda.synchronize()
    torch.testing.assert_close(x, want, atol=1e-3, rtol=1e-3)


def test_swiglu():
    a, w1 = operands(300, 768, 768, seed=3)
    _, w3 = operands(1, 768, 768, seed=4)
    h = gemm(a, w1, b2=w3, epilogue=capi.GEMM_SWIGLU)
    torch.cuda.synchronize()
    g, u = ref(a, w1), ref(a, w3)
    want = torch.nn.functional.silu(g) * u
    assert h.shape == (300, 768) and h.dtype == torch.bfloat16
    torch.testing.assert_close(h.float(), want, atol=2e-2, rtol=1e-2)


def test_grouped_counts():
    """Eight groups (experts) of capacity 256 rows with ragged counts, one
    weight matrix per group; rows past a group's count are left untouched."""
    E, cap, N, K = 8, 256, 768, 768
    g = torch.Generator().manual_seed(5)
    a = torch.randn(E * cap, K, generator=g).to(DEV, torch.bfloat16)
    w = (0.02 * torch.randn(E * N, K, generator=g)).to(DEV, torch.bfloat16)
    counts = torch.tensor([0, 1, 127, 128, 129, 256, 200, 64], dtype=torch.int32, device=DEV)
    out = torch.full((E * cap, N), 7.0, device=DEV)
    gemm(a, w, out=out, counts=counts, groups=E, rows=cap, a_group_rows=cap, b_group_rows=N, c_group_rows=cap)
    torch.cuda.synchronize()
    for e in range(E):
        n = int(counts[e])
        want = ref(a[e * cap:e * cap + n], w[e * N:(e + 1) * N])
        torch.testing.assert_close(out[e * cap:e * cap + n], want, atol=1e-3, rtol=1e-3)
        assert torch.all(out[e * cap + n:(e + 1) * cap] == 7.0)


def test_grouped_swiglu():
    E, cap, H, K = 4, 128, 768, 768
    g = torch.Generator().manual_seed(6)
    a = torch.randn(E * cap, K, generator=g).to(DEV, torch.bfloat16)
    w1 = (0.02 * torch.randn(E * H, K, generator=g)).to(DEV, torch.bfloat16)
    w3 = (0.02 * torch.randn(E * H, K, generator=g)).to(DEV, torch.bfloat16)
    counts = torch.tensor([128, 5, 0, 77], dtype=torch.int32, device=DEV)
    h = torch.zeros(E * cap, H, device=DEV, dtype=torch.bfloat16)
    gemm(a, w1, b2=w3, out=h, epilogue=capi.GEMM_SWIGLU, counts=counts, groups=E, rows=cap, a_group_rows=cap,
         b_group_rows=H, c_group_rows=cap)
    torch.cuda.synchronize()
    for e in range(E):
        n = int(counts[e])
        ae = a[e * cap:e * cap + n]
        want = torch.nn.functional.silu(ref(ae, w1[e * H:(e + 1) * H])) * ref(ae, w3[e * H:(e + 1) * H])
        torch.testing.assert_close(h[e * cap:e * cap + n].float(), want, atol=2e-2, rtol=1e-2)


def test_rejects_bad_shapes():
    a, b = operands(128, 128, 768)
    with pytest.raises(ValueError):
        gemm(a, b[:, :700].contiguous())
    with pytest.raises(Exception):
        gemm(a[:, :96].contiguous(), b[:, :96].contiguous())  # K not a multiple of 64


def test_bias_and_gelu_epilogues():
    a, b = operands(200, 3072, 768, seed=7)
    bias = (0.1 * torch.randn(3072, generator=torch.Generator().manual_seed(8))).to(DEV, torch.bfloat16)
    out = gemm(a, b, bias=bias)
    h = gemm(a, b, bias=bias, epilogue=capi.GEMM_GELU)
    torch.cuda.synchronize()
    want = ref(a, b) + bias.float()
    torch.testing.assert_close(out, want, atol=1e-3, rtol=1e-3)
    torch.testing.assert_close(h.float(), torch.nn.functional.gelu(want), atol=2e-2, rtol=1e-2)


def test_grouped_gelu_with_per_group_bias():
    """The GELU expert up projection of the reference architecture: hidden 3072,
    one bias row per expert."""
    E, cap, H, K = 3, 128, 3072, 768
    g = torch.Generator().manual_seed(9)
    a = torch.randn(E * cap, K, generator=g).to(DEV, torch.bfloat16)
    w1 = (0.02 * torch.randn(E * H, K, generator=g)).to(DEV, torch.bfloat16)
    b1 = (0.1 * torch.randn(E, H, generator=g)).to(DEV, torch.bfloat16)
    counts = torch.tensor([100, 0, 128], dtype=torch.int32, device=DEV)
    h = torch.zeros(E * cap, H, device=DEV, dtype=torch.bfloat16)
    gemm(a, w1, out=h, epilogue=capi.GEMM_GELU, counts=counts, groups=E, rows=cap, a_group_rows=cap,
         b_group_rows=H, c_group_rows=cap, bias=b1.reshape(-1), bias_group_stride=H)
    torch.cuda.synchronize()
    for e in range(E):
        n = int(counts[e])
        want = torch.nn.functional.gelu(ref(a[e * cap:e * cap + n], w1[e * H:(e + 1) * H]) + b1[e].float())
        torch.testing.assert_close(h[e * cap:e * cap + n].float(), want, atol=2e-2, rtol=1e-2)
