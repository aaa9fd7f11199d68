"""Groupwise expert-weight quantization on the CPU: the product's quantizer
(``fused_moe.quantize_experts``, torch) against the numpy restatement in
``oracle/quant.py`` -- integer values, scales and the int4 packing bit for
bit -- plus the round-to-nearest error bound and the model-level switch."""

import numpy as np
import pytest
import torch

from moe_engine import fused_moe
from moe_engine.model import Model, baseline_config
from oracle import quant as oq


def weights(E=3, R=40, C=256, seed=0):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(E, R, C, generator=g) * 0.02
    w[0, 0, :32] = 0.0  # an all-zero group (scale 0)
    w[0, 1, 0] = 5.0    # one outlier dominating its group
    # a group of exact half-steps: scale 1/64 (max 127/64), values (k + 0.5)/64
    w[1, 2, :128] = (torch.arange(128) - 64 + 0.5) / 64.0
    w[1, 2, 127] = 127.0 / 64.0
    return w


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_quantizer_matches_numpy_restatement_bit_for_bit(bits, group):
    w = weights()
    qe = fused_moe.quantize_experts(w, bits, group)
    q_ref, s_ref = oq.quantize(w.numpy(), bits, group)
    assert np.array_equal(qe.scale.numpy(), s_ref)
    if bits == 8:
        assert qe.q.dtype == torch.int8
        assert np.array_equal(qe.q.numpy(), q_ref)
    else:
        assert qe.q.dtype == torch.uint8 and qe.q.shape[-1] == w.shape[-1] // 2
        assert np.array_equal(qe.q.numpy(), oq.pack4(q_ref))
        assert np.array_equal(oq.unpack4(qe.q.numpy()), q_ref)
    deq = fused_moe.dequantize_experts(qe)
    assert np.array_equal(deq.numpy(), oq.dequantize(q_ref, s_ref, group))


@pytest.mark.parametrize("bits", [8, 4])
def test_round_to_nearest_error_bound_and_ties(bits):
    w = weights()
    group = 128
    qe = fused_moe.quantize_experts(w, bits, group)
    deq = fused_moe.dequantize_experts(qe)
    half = (qe.scale / 2).repeat_interleave(group, dim=-1)
    assert bool(((deq - w).abs() <= half * (1 + 1e-6)).all())
    assert bool((deq[0, 0, :32] == 0).all())
    if bits == 8:
        # the half-step group rounds to even integers
        q = qe.q[1, 2, :127].to(torch.int32)
        exact = (torch.arange(127) - 64 + 0.5)
        assert bool(((q - exact).abs() == 0.5).all()) and bool((q % 2 == 0).all())


def test_int4_packing_layout():
    # element 2i in the low nibble, 2i + 1 in the high nibble, two's complement
    w = torch.zeros(1, 1, 32)
    w[0, 0, :8] = torch.tensor([7.0, -7.0, 1.0, -1.0, 0.0, 3.0, -4.0, 2.0])
    qe = fused_moe.quantize_experts(w, 4, 32)
    assert float(qe.scale[0, 0, 0]) == 1.0
    b = qe.q[0, 0, :4].tolist()
    assert b == [0x97, 0xF1, 0x30, 0x2C]


def test_quantizer_rejects_bad_shapes():
    w = torch.zeros(2, 4, 96)
    with pytest.raises(ValueError):
        fused_moe.quantize_experts(w, 3, 32)
    with pytest.raises(ValueError):
        fused_moe.quantize_experts(w, 8, 48)  # not a multiple of 32
    with pytest.raises(ValueError):
        fused_moe.quantize_experts(w, 8, 64)  # does not divide 96
    with pytest.raises(ValueError):
        fused_moe.quantize_experts(torch.zeros(2, 4, 192), 8, 96)  # not a power of two
    with pytest.raises(ValueError):
        fused_moe.quantize_experts(w[0], 8, 32)  # not stacked


@pytest.mark.parametrize("bits", [8, 4])
def test_model_quantize_experts_rewrites_expert_parameters(bits):
    """After Model.quantize_experts every expert parameter holds the weights the
    quantized values stand for (the prefill and the reference mode compute
    with them); the quantized copy sits beside them for the decode kernel."""
    cfg = baseline_config()
    cfg.num_layers = 2
    m = Model(cfg).eval()
    before = {k: v.clone() for k, v in m.MoEBlocks[0].moe._expert_storage.items()}
    m.quantize_experts(bits, 128)
    moe = m.MoEBlocks[0].moe
    assert moe.quantized and set(moe._quant) == {"w1", "w3", "w2"}
    for name, qe in moe._quant.items():
        q_ref, s_ref = oq.quantize(before[name].numpy(), bits, 128)
        deq = oq.dequantize(q_ref, s_ref, 128)
        assert np.array_equal(moe._expert_storage[name].numpy(), deq)
        # the per-expert parameters are views of the storage
        e0 = moe.experts[0]
        assert e0.gate.weight.data_ptr() == moe._expert_storage["w1"][0].data_ptr()


def test_decode_descriptor_quant_format():
    """The step descriptors carry one (bits, group) for the whole model: (0, 0)
    without quantized experts, the shared format when every layer is quantized
    alike, and no fused decode (None) when layers differ."""
    from moe_engine.decode import DecodeRunner

    cfg = baseline_config()
    cfg.num_layers = 2
    m = Model(cfg).eval()
    assert DecodeRunner._quant_format(m) == (0, 0)
    m.quantize_experts(8, 64)
    assert DecodeRunner._quant_format(m) == (8, 64)
    m.MoEBlocks[1].moe.quantize_experts(4, 64)
    assert DecodeRunner._quant_format(m) is None
    m.MoEBlocks[1].moe._quant = None
    assert DecodeRunner._quant_format(m) is None
