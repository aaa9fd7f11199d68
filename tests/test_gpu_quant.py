"""Quantized experts on the GPU (int8 / int4 groupwise, ``mie_moe_decode`` with
expert_bits set).  The reference has no quantized path (a roadmap item,
moe-inference-engine.md:36), so the checker is the MoE oracle
(``oracle.moe_decode_stacked``) run on the weights the quantized values stand
for (``oracle/quant.py``).

Tolerances:
* against the oracle on the dequantized weights: expert ids exact; fp32
  activations within the fp32 MoE bar (atol 3e-4, rtol 2e-4); bf16 within 1e-2
  (the bf16 output rounding);
* against the unquantized bf16 layer (what quantization costs, not a kernel
  error): relative Frobenius error below 2e-2 for int8 and 3e-1 for int4 at
  group 128 on N(0, 0.02) weights (measured: ~0.2 for int4, the cost of 15
  levels per group through two projections);
* model level: fp32 greedy tokens of the int8 and int4 models (the per-layer
  launch sequence with the quantized MoE kernel) identical to the oracle's on
  the dequantized weights; the bf16 model with int8 experts through the
  persistent cluster step agrees with the per-layer launch sequence on the
  same quantized weights (hidden states within 5e-3, the bar between the two
  paths in bf16; greedy tokens identical).
"""

import numpy as np
import pytest
import torch

import oracle
from moe_engine import fused_moe
from moe_engine.model import Model, baseline_config
from oracle import quant as oq
from tests.helpers import engine_state_dict

pytestmark = pytest.mark.gpu
DEV = "cuda"


def stacked(E, Hx, D, act, seed, bias=False):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g) * 0.02  # noqa: E731
    w = {"router": r(E, D), "w1": r(E, Hx, D), "w2": r(E, D, Hx)}
    if act == "swiglu":
        w["w3"] = r(E, Hx, D)
    if bias:
        w["b1"], w["b2"] = r(E, Hx), r(E, D)
    return w


def workspaces(E, Hx, D, dtype):
    f = dict(device=DEV, dtype=torch.float32)
    return dict(router_logits=torch.empty(E, **f), expert_ids=torch.empty(2, dtype=torch.int32, device=DEV),
                route_weights=torch.empty(2, **f), hidden=torch.empty(2, Hx, **f),
                out=torch.empty(D, dtype=dtype, device=DEV))


def run_quantized(w, x, bits, group, dtype):
    E, Hx, D = w["w1"].shape
    qs = {k: fused_moe.quantize_experts(w[k].to(DEV), bits, group) for k in ("w1", "w2", "w3") if k in w}
    for k, qe in qs.items():  # the quantizer on the GPU gives the CPU restatement's values
        q_ref, s_ref = oq.quantize(w[k].numpy(), bits, group)
        assert np.array_equal(qe.scale.cpu().numpy(), s_ref), k
        assert np.array_equal(qe.q.cpu().numpy(), q_ref if bits == 8 else oq.pack4(q_ref)), k
    ws = workspaces(E, Hx, D, dtype)
    out = fused_moe.decode(x.to(DEV, dtype).view(1, 1, D), w["router"].to(DEV, dtype), qs["w1"],
                           w["b1"].to(DEV, dtype) if "b1" in w else None, qs["w2"],
                           w["b2"].to(DEV, dtype) if "b2" in w else None, w3_base=qs.get("w3"), **ws)
    torch.cuda.synchronize()
    return out.view(D).float().cpu(), ws, qs


def oracle_on_dequantized(w, x, bits, group, dtype):
    deq = {}
    for k in ("w1", "w2", "w3"):
        if k in w:
            q, s = oq.quantize(w[k].numpy(), bits, group)
            deq[k] = torch.from_numpy(oq.dequantize(q, s, group))
    rd = lambda t: None if t is None else t.to(dtype).float()  # noqa: E731
    return oracle.moe_decode_stacked(x.to(dtype).float(), rd(w["router"]), deq["w1"], rd(w.get("b1")), deq["w2"],
                                     rd(w.get("b2")), w3=deq.get("w3"))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("group", [32, 128])
def test_quantized_swiglu_config1_shape_matches_oracle(dtype, bits, group):
    """config[1] shapes: 8 SwiGLU experts of 768 x 768, x ~ N(0, 1); several
    tokens so different experts are selected."""
    E, Hx, D = 8, 768, 768
    w = stacked(E, Hx, D, "swiglu", seed=bits + group)
    seen = set()
    for t in range(6):
        x = torch.randn(D, generator=torch.Generator().manual_seed(100 + t))
        got, ws, _ = run_quantized(w, x, bits, group, dtype)
        want, logits, ids, wts = oracle_on_dequantized(w, x, bits, group, dtype)
        assert ws["expert_ids"].cpu().tolist() == ids.tolist()
        seen.update(ids.tolist())
        if dtype == torch.float32:
            torch.testing.assert_close(got, want, atol=3e-4, rtol=2e-4)
            torch.testing.assert_close(ws["router_logits"].cpu(), logits, atol=2e-5, rtol=1e-5)
        else:
            torch.testing.assert_close(got, want, atol=1e-2, rtol=1e-2)
    assert len(seen) >= 4


@pytest.mark.parametrize("bits", [8, 4])
def test_quantized_gelu_biased_reference_shape(bits):
    """The reference checkpoint's expert shape: GELU(erf) experts of 3072
    hidden units with biases (rows of 3072 / 768 elements: several register
    segments per row for int8), fp32."""
    E, Hx, D = 8, 3072, 768
    w = stacked(E, Hx, D, "gelu", seed=7 + bits, bias=True)
    for t in range(3):
        x = torch.randn(D, generator=torch.Generator().manual_seed(200 + t))
        got, ws, _ = run_quantized(w, x, bits, 128, torch.float32)
        want, _, ids, _ = oracle_on_dequantized(w, x, bits, 128, torch.float32)
        assert ws["expert_ids"].cpu().tolist() == ids.tolist()
        torch.testing.assert_close(got, want, atol=3e-4, rtol=2e-4)


@pytest.mark.parametrize("bits,bound", [(8, 2e-2), (4, 3e-1)])
def test_quantization_error_against_bf16_layer(bits, bound):
    E, Hx, D = 8, 768, 768
    w = stacked(E, Hx, D, "swiglu", seed=11)
    errs = []
    for t in range(8):
        x = torch.randn(D, generator=torch.Generator().manual_seed(300 + t))
        got, ws, _ = run_quantized(w, x, bits, 128, torch.bfloat16)
        full = workspaces(E, Hx, D, torch.bfloat16)
        ref = fused_moe.decode(x.to(DEV, torch.bfloat16).view(1, 1, D), w["router"].to(DEV, torch.bfloat16),
                               w["w1"].to(DEV, torch.bfloat16), None, w["w2"].to(DEV, torch.bfloat16), None,
                               w3_base=w["w3"].to(DEV, torch.bfloat16), **full).view(D).float().cpu()
        if full["expert_ids"].cpu().tolist() != ws["expert_ids"].cpu().tolist():
            continue  # quantization moved a near-tie in the router: not comparable
        errs.append(float((got - ref).norm() / ref.norm()))
    assert len(errs) >= 6
    assert max(errs) < bound, errs


def test_quantized_decode_rejects_mixed_or_bad_weights():
    E, Hx, D = 8, 768, 768
    w = stacked(E, Hx, D, "swiglu", seed=3)
    q8 = {k: fused_moe.quantize_experts(w[k].to(DEV), 8, 128) for k in ("w1", "w2", "w3")}
    q4 = fused_moe.quantize_experts(w["w2"].to(DEV), 4, 128)
    ws = workspaces(E, Hx, D, torch.float32)
    x = torch.randn(1, 1, D, device=DEV)
    r = w["router"].to(DEV)
    with pytest.raises(ValueError, match="share bits"):
        fused_moe.decode(x, r, q8["w1"], None, q4, None, w3_base=q8["w3"], **ws)
    with pytest.raises(ValueError, match="QuantizedExperts"):
        fused_moe.decode(x, r, q8["w1"], None, w["w2"].to(DEV), None, w3_base=q8["w3"], **ws)
    four = fused_moe.quantize_experts(w["w2"][:4].to(DEV), 8, 128)  # 4 experts where the router has 8
    with pytest.raises(ValueError, match="canonical"):
        fused_moe.decode(x, r, q8["w1"], None, four, None, w3_base=q8["w3"], **ws)


@pytest.mark.parametrize("bits", [8, 4])
def test_model_quantized_experts_fp32_tokens_identical_to_oracle(bits):
    """A 2-layer BASELINE-architecture model (vocab 512) in fp32 with int8 or
    int4 experts: 24 greedy tokens through Model.generate (the per-layer launch
    sequence with the quantized MoE kernel) equal the oracle's on the
    dequantized weights."""
    arch = oracle.BASELINE_ARCH.with_(num_layers=2, vocab_size=512)
    P = oracle.init_params(arch, seed=5)
    m = Model(baseline_config(num_layers=2, vocab_size=512)).eval()
    m.load_state_dict(engine_state_dict(P))
    m = m.to(DEV, torch.float32).quantize_experts(bits, 128)
    cache = m.new_cache()
    assert m.fused_decode_supported(cache, 1)
    assert not m.decode_runner().uses_persistent(cache)  # fp32: the per-layer launch sequence
    Pq = dict(P)
    for i in range(arch.num_layers):
        for name in ("gate", "up", "down"):
            keys = [f"MoEBlocks.{i}.moe.experts.{e}.{name}.weight" for e in range(arch.num_experts)]
            st = torch.stack([P[k] for k in keys]).numpy()
            q, s = oq.quantize(st, bits, 128)
            deq = torch.from_numpy(oq.dequantize(q, s, 128))
            for e, k in enumerate(keys):
                Pq[k] = deq[e]
    prompt = torch.randint(0, 512, (12,), generator=torch.Generator().manual_seed(1))
    want = oracle.generate_greedy(Pq, arch, prompt, 24)
    got = m.generate(prompt, max_new_tokens=24, temperature=0)[0].tolist()
    assert got == want
    assert np.array_equal(m.MoEBlocks[0].moe._quant["w1"].scale.cpu().numpy(),
                          oq.quantize(torch.stack([P[f"MoEBlocks.0.moe.experts.{e}.gate.weight"]
                                                   for e in range(arch.num_experts)]).numpy(), bits, 128)[1])


@pytest.mark.parametrize("group", [128, 32])
def test_bf16_int8_persistent_step_agrees_with_launch_sequence(group):
    """The BASELINE model in bf16 with int8 experts: decode steps run the
    persistent cluster step (int8 rows and their group scales staged by the
    producer warp) and agree with the per-layer launch sequence (the quantized
    MoE kernel) on the same weights: hidden states within 5e-3 over 6 steps,
    40 greedy tokens identical.  int4 experts run the launch sequence."""
    from moe_engine import capi
    from tests.helpers import baseline_bf16_model

    m, _, _ = baseline_bf16_model(max_seq=512)
    m.quantize_experts(8, group)
    runner = m.decode_runner()
    assert runner.step_kernel_for(m.new_cache()) == capi.MIE_STEP_CLUSTER
    prompt = torch.randint(0, 50304, (24,), generator=torch.Generator().manual_seed(9))
    xs = {}
    for persistent in (True, False):
        runner.persistent = persistent
        cache = m.new_block_allocator(num_blocks=40, block_size=16, attention_mode="direct").new_cache()
        hs = []
        with torch.no_grad():
            m(prompt[None].to(DEV), cache)
            tok = torch.tensor([[17]], device=DEV)
            for _ in range(6):
                logits = m(tok, cache)
                hs.append(runner.x.clone())
                tok = logits[0, -1].float().argmax().view(1, 1)
        xs[persistent] = torch.stack(hs)
        runner.check_status()
    runner.persistent = True
    rel = (xs[True] - xs[False]).norm() / xs[False].norm()
    assert rel < 5e-3, float(rel)
    gen = {}
    for persistent in (True, False):
        runner.persistent = persistent
        gen[persistent] = m.generate(prompt, max_new_tokens=40, temperature=0)
    runner.persistent = True
    assert torch.equal(gen[True], gen[False])
    runner.check_status()

    m4, _, _ = baseline_bf16_model(max_seq=512, num_layers=2)
    m4.quantize_experts(4, group)
    assert m4.fused_decode_supported(m4.new_cache(), 1)
    assert m4.decode_runner().step_kernel_for(m4.new_cache()) == 0
