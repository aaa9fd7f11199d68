"""Batch-one decode benchmark on B200 -- driver contract.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload (config[3]): the miniMoE-shaped model (12 x 768, 12 heads x 64,
RMSNorm, RoPE, 8 SwiGLU experts of hidden 768, top-2, vocab 50304, tied LM
head), random init, bf16, paged KV cache (block 16, direct attention), MoE
direct.  A 512-token random prompt is prefilled once; one bench STEP is the
greedy decode of 1024 tokens from that prompt (context 513..1536), replaying
the captured decode-step CUDA graph once per token.  `value` is decode tokens
per second over K steps (device time, CUDA events, max over ranks).  The
per-token weight bytes (219 MB) exceed the 126 MB L2, so every step streams
from HBM.

`e2e` is the same metric through the public API: ``Model.generate`` from a
host (pinned) prompt tensor to host output tokens, prefill included.

`--impl reference` times the reference algorithm's CPU path (the oracle
restatement of ``--moe reference`` with a contiguous fp32 KV cache) on the
host cores on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "moe-inference-engine_b200"))
sys.path.insert(0, REPO)

METRIC = "batch-1 decode tok/s (bf16, config[3]: 512-token prompt + 1024 greedy tokens)"
# ncu capture of one persistent step launch of the cluster step kernel
# (--profile 12, 7th step, context 518; 224.8 us under ncu):
# dram__bytes_read.sum + dram__bytes_write.sum
STEP_CAPTURE_DRAM_BYTES = 238.445312e6 + 3.497216e6
STEP_CAPTURE_CTX = 518
PROMPT_LEN = 512
NEW_TOKENS = 1024
# active weight bytes per token in bf16: 2 B x 109,506,048 active params
ACTIVE_PARAMS = 109_506_048
KV_BYTES_PER_CTX = 36_864  # 12 layers x 12 heads x 64 x 2 (K+V) x 2 B
MOE_LAYER_BYTES = 7_090_176  # router 12,288 + 2 experts x 3 x 1,179,648


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (measured)"
    return 6650.0, "fallback 6.65 TB/s"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during timing."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        mhz, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not mhz:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
                "samples": len(mhz)}


def build_model(device, dtype, seed=0):
    from moe_engine.model import Model, baseline_config, random_init_

    torch.manual_seed(seed)
    model = Model(baseline_config()).eval().to(device=device, dtype=dtype)
    return random_init_(model, seed)


def time_graph_calls(fn, calls: int, reps: int = 5):
    """Average device time of fn() when `calls` launches run back to back in a graph."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(calls):
            fn()
    for _ in range(2):
        g.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / 1e3 / (reps * calls)


def moe_microbench(model, hbm_peak):
    """config[1]: the isolated fused top-2 MoE layer (``fused_moe.decode``,
    bf16), the 12 layers' weights cycled (340 MB > L2): graphs of 240
    back-to-back calls, x ~ N(0, 1) per layer (seed 1)."""
    from moe_engine import fused_moe

    dev = model.token_embedding.weight.device
    layers = [(blk.moe, blk.moe._expert_storage) for blk in model.MoEBlocks]
    L = len(layers)
    xs = torch.randn(L, 768, generator=torch.Generator().manual_seed(1)).to(dev, torch.bfloat16)
    state = {"i": 0}

    def timed_call():
        i = state["i"] % L
        state["i"] += 1
        moe, s = layers[i]
        fused_moe.decode(xs[i].view(1, 1, 768), moe.router.weight, s["w1"], None, s["w2"], None,
                         router_logits=moe._router_logits, expert_ids=moe._expert_ids,
                         route_weights=moe._route_weights, hidden=moe._expert_hidden, out=moe._direct_out,
                         w3_base=s["w3"], sync=moe._sync)

    t = time_graph_calls(timed_call, 240)
    return {"us": t * 1e6, "bytes": MOE_LAYER_BYTES, "gbs": MOE_LAYER_BYTES / t / 1e9,
            "frac": MOE_LAYER_BYTES / t / 1e9 / hbm_peak, "calls_per_graph": 240}


def moe_q_microbench(model, hbm_peak, bits: int, group: int = 128):
    """config[1] with quantized experts (``fused_moe.quantize_experts``, int8
    or int4 in groups of 128): the 12 layers' experts quantized, copies added
    until the working set is >= 256 MB (twice L2), cycled in graphs of 240
    back-to-back calls.  Algorithmic bytes per call: the bf16 router plus two
    experts' quantized rows and fp32 group scales."""
    from moe_engine import fused_moe

    dev = model.token_embedding.weight.device
    base = []
    for blk in model.MoEBlocks:
        s = blk.moe._expert_storage
        base.append((blk.moe, {k: fused_moe.quantize_experts(s[k], bits, group) for k in ("w1", "w3", "w2")}))
    per_layer = sum(q.nbytes() for q in base[0][1].values())
    copies = max(1, -(-256 * 2**20 // (per_layer * len(base))))
    layers = [(moe, {k: fused_moe.QuantizedExperts(q.q.clone(), q.scale.clone(), q.bits, q.group_size, q.shape)
                     for k, q in qs.items()}) for _ in range(copies) for moe, qs in base]
    L = len(layers)
    xs = torch.randn(len(base), 768, generator=torch.Generator().manual_seed(1)).to(dev, torch.bfloat16)
    state = {"i": 0}

    def timed_call():
        i = state["i"] % L
        state["i"] += 1
        moe, q = layers[i]
        fused_moe.decode(xs[i % len(base)].view(1, 1, 768), moe.router.weight, q["w1"], None, q["w2"], None,
                         router_logits=moe._router_logits, expert_ids=moe._expert_ids,
                         route_weights=moe._route_weights, hidden=moe._expert_hidden, out=moe._direct_out,
                         w3_base=q["w3"], sync=moe._sync)

    t = time_graph_calls(timed_call, 240)
    E = model.config.num_experts
    nbytes = 12288 + 2 * per_layer // E
    return {"us": t * 1e6, "bytes": nbytes, "gbs": nbytes / t / 1e9, "frac": nbytes / t / 1e9 / hbm_peak,
            "calls_per_graph": 240, "bits": bits, "group": group, "working_set_mb": round(per_layer * L / 2**20)}


def attn_microbench(device, hbm_peak, contexts=(128, 512, 2048, 8192)):
    """config[2]: one query [12 heads, 64] bf16 over a paged cache (block 16,
    K/V ~ N(0, 1) bf16, shuffled block tables), through the C ABI entry point
    ``mie_attn_decode`` with the operator's split choice.  Per context, graphs
    of back-to-back calls: "cold" rotates among R disjoint block tables of one
    pool of >= 256 MB (twice L2), so no call finds its K/V in L2; "hot" reuses
    one table (the K/V of every call in L2)."""
    import ctypes
    import math

    from moe_engine import capi, paged_attention

    lib = capi.ensure_init(device)
    stream = capi.stream_handle(device)
    H, hd, bs = 12, 64, 16
    out = {}
    for ctx in contexts:
        nb = -(-ctx // bs)
        per_table = nb * H * bs * hd * 2 * 2
        R = max(8, -(-256 * 2**20 // per_table))
        nblocks = R * nb
        gen = torch.Generator().manual_seed(2)
        k = torch.randn(nblocks, H, bs, hd, generator=gen).to(device, torch.bfloat16)
        v = torch.randn(nblocks, H, bs, hd, generator=gen).to(device, torch.bfloat16)
        tables = torch.randperm(nblocks, generator=gen).view(R, nb).to(torch.int32).to(device)
        q = torch.randn(H, hd, generator=gen).to(device, torch.bfloat16)
        o = torch.empty(H, hd, dtype=torch.bfloat16, device=device)
        splits = paged_attention.choose_splits(H, nb, lib.mie_num_sms(device.index or 0))
        partials = torch.zeros(H * paged_attention.MAX_SPLITS * (hd + 2), dtype=torch.float32, device=device)
        counters = torch.zeros(H, dtype=torch.int32, device=device)

        def args_for(r):
            a = capi.AttnArgs()
            a.kv_dtype = a.q_dtype = a.out_dtype = capi.dtype_code(torch.bfloat16)
            a.num_heads, a.head_dim = H, hd
            a.q, a.k, a.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
            a.block_table = tables[r].data_ptr()
            a.num_blocks, a.block_size = nblocks, bs
            a.stride_block, a.stride_head, a.stride_tok = H * bs * hd, bs * hd, hd
            a.ctx_len, a.max_ctx = ctx, nb * bs
            a.scale = 1.0 / math.sqrt(hd)
            a.out = o.data_ptr()
            a.partials, a.counters = partials.data_ptr(), counters.data_ptr()
            a.splits, a.max_splits = splits, paged_attention.MAX_SPLITS
            return a

        cold_args = [args_for(r) for r in range(R)]
        hot_args = [args_for(0)] * R
        res = {"splits": splits, "ctx": ctx, "bytes": ctx * H * hd * 2 * 2}
        for name, arglist in (("cold", cold_args), ("hot", hot_args)):
            for a in arglist[:3]:
                capi.check(lib.mie_attn_decode(ctypes.byref(a), stream), "mie_attn_decode")
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                st = capi.stream_handle(device)
                for a in arglist:
                    capi.check(lib.mie_attn_decode(ctypes.byref(a), st), "mie_attn_decode")
            gr.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(3):
                gr.replay()
            e1.record()
            torch.cuda.synchronize()
            t = e0.elapsed_time(e1) / 1e3 / (3 * R)
            res[name] = {"us": t * 1e6, "gbs": res["bytes"] / t / 1e9, "frac": res["bytes"] / t / 1e9 / hbm_peak,
                         "calls_per_graph": R}
            del gr
        out[f"attn_decode_ctx{ctx}"] = res
        del k, v
    return out


def kernel_rooflines(model, hbm_peak):
    """Isolated per-op kernels: config[1] (MoE) and config[2] (attention)."""
    out = {"moe_decode": moe_microbench(model, hbm_peak)}
    for bits in (8, 4):
        out[f"moe_decode_int{bits}"] = moe_q_microbench(model, hbm_peak, bits)
    out.update(attn_microbench(model.token_embedding.weight.device, hbm_peak))
    return out


def run_b200(args, rank, world, device):
    from moe_engine import capi
    from moe_engine.decode import greedy_generate  # noqa: F401  (public path is Model.generate)

    dtype = torch.bfloat16
    hbm_peak, peak_src = peaks()
    model = build_model(device, dtype)
    gen = torch.Generator().manual_seed(3 + rank)
    prompt = torch.randint(0, 50304, (PROMPT_LEN,), generator=gen)
    max_blocks = -(-(PROMPT_LEN + NEW_TOKENS) // 16)
    # room for the device-loop request and one public-API (e2e) request at a time
    alloc = model.new_block_allocator(num_blocks=2 * max_blocks + 8, block_size=16, attention_mode="direct")
    runner = model.decode_runner()

    # prefill once, then the device-resident decode loop
    cache = alloc.new_cache()
    with torch.no_grad():
        logits = model(prompt[None].to(device), cache)
    first = int(logits[0, -1].float().argmax())
    P = cache.position
    cache.reserve(P + NEW_TOKENS)
    # persistent step: graphs of M step launches (programmatic-dependent)
    M = runner.steps_per_graph(cache)
    assert NEW_TOKENS % M == 0
    graph = runner.graph_for(cache, P + NEW_TOKENS, steps=M)
    # one persistent launch per token, else 4 launches per layer + the LM head
    launches_per_token = 1 if runner.uses_persistent(cache) else 4 * 12 + 1

    def reset():
        runner.token.fill_(first)
        runner.pos.fill_(P)
        runner.done.zero_()
        runner.log_count.zero_()
        runner.step_limit.fill_(NEW_TOKENS)

    def one_step():
        reset()
        for _ in range(NEW_TOKENS // M):
            graph.replay()

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    runner.check_status()

    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index or 0) as clocks:
        e0.record()
        for _ in range(args.steps):
            one_step()
        e1.record()
        torch.cuda.synchronize()
    elapsed = e0.elapsed_time(e1) / 1e3
    if world > 1:
        t = torch.tensor([elapsed], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        elapsed = float(t)
        torch.distributed.barrier()
    runner.check_status()
    single_tokens = runner.tokens_log[:NEW_TOKENS].tolist()  # this replica's greedy tokens
    tokens = args.steps * NEW_TOKENS * world
    value = tokens / elapsed

    # per-token latency distribution (events between replays of M steps, per
    # step; separate pass)
    reset()
    R = NEW_TOKENS // M
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(R + 1)]
    evs[0].record()
    for i in range(R):
        graph.replay()
        evs[i + 1].record()
    torch.cuda.synchronize()
    per_tok = sorted(evs[i].elapsed_time(evs[i + 1]) / M for i in range(R))
    p50 = per_tok[len(per_tok) // 2]
    p99 = per_tok[min(len(per_tok) - 1, int(len(per_tok) * 0.99))]

    # end to end through the public API (host prompt -> host tokens)
    host_prompt = prompt.clone().pin_memory()
    e2e_times = []
    out_len = 0
    for it in range(max(1, min(args.steps, 5)) + 1):
        c = alloc.new_cache()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        out = model.generate(host_prompt, max_new_tokens=NEW_TOKENS, temperature=0, cache=c)
        out_host = out.cpu()
        t1 = time.perf_counter()
        c.free()
        out_len = out_host.shape[1]
        if it > 0:  # first call warms the graph for this cache
            e2e_times.append(t1 - t0)
    new_tokens = out_len - PROMPT_LEN
    e2e_value = new_tokens / statistics.median(e2e_times)
    if world > 1:
        t = torch.tensor([e2e_value], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN)
        e2e_value = float(t) * world

    # the prompt prefill alone (graph-replayed after its first run): GPU time
    # (CUDA events) and wall time of model(prompt) into a fresh cache
    pf_gpu, pf_wall = [], []
    dprompt = prompt[None].to(device)
    for it in range(4):
        c = alloc.new_cache()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        e0p, e1p = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0p.record()
        with torch.no_grad():
            model(dprompt, c)
        e1p.record()
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        c.free()
        if it > 0:
            pf_gpu.append(e0p.elapsed_time(e1p))
            pf_wall.append((t1 - t0) * 1e3)
    prefill = {"tokens": PROMPT_LEN, "gpu_ms": statistics.median(pf_gpu), "wall_ms": statistics.median(pf_wall),
               "note": "model(prompt) into a fresh paged cache: tcgen05 GEMMs, the causal attention kernel and "
                       "the per-token kernels, replayed from the captured prefill graph"}

    # rooflines
    step_s = elapsed / (args.steps * NEW_TOKENS)  # seconds per token on each replica
    weights_bytes = 2 * ACTIVE_PARAMS
    mean_ctx = PROMPT_LEN + NEW_TOKENS / 2
    kv_bytes = KV_BYTES_PER_CTX * mean_ctx
    k_roof = kernel_rooflines(model, hbm_peak) if rank == 0 else {}
    persistent = launches_per_token == 1
    # dominant kernel: the persistent step kernel (one launch per token) or,
    # on the per-op path, the fused MoE kernel timed in isolation
    traffic = None
    if persistent:
        from moe_engine import capi as _capi

        dominant = ("cstep_kernel (persistent decode step on thread-block clusters, one launch per token)"
                    if runner.step_kernel_for(cache) == _capi.MIE_STEP_CLUSTER
                    else "step_kernel (persistent decode step, one CTA per SM, one launch per token)")
        step_bytes = weights_bytes + kv_bytes
        kr = {"us": step_s * 1e6, "gbs": step_bytes / step_s / 1e9, "bytes": step_bytes}
        kr["frac"] = kr["gbs"] / hbm_peak
        # DRAM bytes of one step launch measured by ncu at context
        # STEP_CAPTURE_CTX (dram__bytes_read.sum + dram__bytes_write.sum),
        # scaled to the mean context: the same ratio to the algorithmic bytes
        cap_traffic, cap_alg = STEP_CAPTURE_DRAM_BYTES, weights_bytes + KV_BYTES_PER_CTX * STEP_CAPTURE_CTX
        traffic = step_bytes * cap_traffic / cap_alg
        roof_note = ("per-launch average of the graph-replayed step over the timed region (CUDA events); "
                     "algorithmic bytes = active bf16 weights + the K/V bytes at the mean context; traffic = "
                     f"ncu dram read+write of one launch at context {STEP_CAPTURE_CTX} "
                     f"({cap_traffic / 1e6:.1f} MB), scaled to the mean context by the algorithmic bytes")
    else:
        dominant = "moe_decode"
        kr = k_roof.get(dominant, {"us": None, "gbs": None, "frac": None, "bytes": MOE_LAYER_BYTES})
        roof_note = "fused MoE kernel timed in isolation (graph of 240 launches over 12 layers' experts)"

    result = {
        "metric": METRIC,
        "value": value,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (random-init weights N(0,0.02), seeded random prompt ids)",
        "config": {
            "workload": "config[3] full-model decode, 512-token prompt + 1024 greedy tokens, paged KV bs16, "
                        f"MoE direct, the decode step captured in a CUDA graph ({M} programmatic-dependent step "
                        "launches per replay); step = one 1024-token decode",
            "model": "miniMoE-shaped 12x768, 12 heads x 64, 8 SwiGLU experts top-2, vocab 50304",
            "global_batch": world,
            "seq_len": PROMPT_LEN + NEW_TOKENS,
            "parallelism": f"replicas x{world}",
            "l2": "inputs larger than L2 (219 MB of weights per token > 126 MB L2)",
        },
        "latency_ms_per_token": {"p50": p50, "p99": p99, "mean": sum(per_tok) / len(per_tok),
                                 "note": f"CUDA events around each graph replay of {M} steps, divided by {M}"},
        "step_roofline": {
            "bound": "hbm",
            "weights_bytes_per_token": weights_bytes,
            "kv_bytes_per_token_mean": kv_bytes,
            "us_per_token": step_s * 1e6,
            "achieved_gbs_weights": weights_bytes / step_s / 1e9,
            "frac_weights_only": weights_bytes / step_s / 1e9 / hbm_peak,
            "frac_total": (weights_bytes + kv_bytes) / step_s / 1e9 / hbm_peak,
            "peak_gbs": hbm_peak,
            "peak_source": peak_src,
        },
        "roofline": {
            "kernel": dominant,
            "bound": "hbm",
            "achieved": kr["gbs"],
            "peak": hbm_peak,
            "unit": "GB/s",
            "frac": kr["frac"],
            "traffic": traffic,
            "algorithmic_bytes_per_launch": kr["bytes"],
            "us_per_launch": kr["us"],
            "peak_source": peak_src,
            "note": roof_note,
        },
        "kernels": k_roof,
        "prefill": prefill,
        "clocks": clocks.summary(),
        "e2e": {
            "value": e2e_value,
            "unit": "tok/s",
            "h2d_bytes_per_step": PROMPT_LEN * 8,
            "d2h_bytes_per_step": (PROMPT_LEN + NEW_TOKENS) * 8,
            "note": "Model.generate from a pinned host prompt to host tokens, prefill included",
        },
        "gpu_launches": args.steps * NEW_TOKENS * launches_per_token,
    }
    if world > 1:
        # independent replicas: each stream decodes at value / world
        result["per_stream_tok_s"] = value / world
        result["per_stream_e2e_tok_s"] = e2e_value / world
        # config[4b] on the same group: one request, experts split over the ranks
        eps = {}
        if model.config.num_experts % world == 0:
            want = [int(t) for t in single_tokens] if rank == 0 else None
            for key, payload, coll in (("step", "fp32", "step"), ("fused", "fp32", "fused"), ("peer", "fp32", "peer"),
                                       ("fp32", "fp32", "nccl"), ("bf16", "bf16", "nccl")):
                try:
                    eps[key] = measure_expert_parallel(model, alloc, device, world, max(1, min(args.steps, 2)), 1,
                                                       payload, want, collective=coll)
                except Exception as e:  # one variant's failure is recorded, the replica line stands
                    eps[key] = {"payload": payload, "collective": coll, "tok_s": None,
                                "error": f"{type(e).__name__}: {e}"[:300]}
        allreduce = {f"allreduce_us_nccl_{pl}": measure_allreduce(device, pl, model.config.hidden_dim)
                     for pl in ("fp32", "bf16")}
        allreduce["allreduce_us_peer_fp32"] = measure_peer_allreduce(device, model.config.hidden_dim)
        result["expert_parallel"] = {
            "n_gpus": world,
            "experts_per_rank": model.config.num_experts // world,
            **allreduce,
            "note": "one request; aggregate = per-stream tok/s; the all-reduce of the [768] MoE partial per layer: "
                    "step: inside the single-launch persistent cluster step (tagged words over NVLink into every "
                    "rank's memory, summed in rank order by every reader); fused: completed inside each layer's "
                    "MoE kernel (layer-by-layer kernels); peer: the same exchange as a kernel of its own; "
                    "fp32 / bf16: NCCL with that payload; every variant's steps captured in CUDA graphs; tokens "
                    "compared with rank 0's single-GPU greedy tokens of the same prompt; allreduce_us_*: the "
                    "collective alone",
            **{f"{k}_tok_s": v["tok_s"] for k, v in eps.items()},
            **{f"{k}_tokens": {kk: vv for kk, vv in v.items() if kk not in ("tok_s",)} for k, v in eps.items()},
        }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(seconds=args.cpu_seconds)
    return result


class CpuWindows:
    """The reference algorithm's CPU decode path (``--moe reference`` with a
    contiguous fp32 KV cache, restated by the oracle -- the reference engine
    cannot run BASELINE's architecture unmodified) at three points of the
    bench's context range: prefixes of 512, 1024 and 1480 tokens are prefilled
    once (untimed), then timed greedy decode steps continue from each, so the
    sample covers contexts 513-1536 like the GPU run."""

    STARTS = (PROMPT_LEN, 1024, 1480)

    def __init__(self):
        import oracle

        self.cores = len(os.sched_getaffinity(0))
        torch.set_num_threads(self.cores)
        P = oracle.init_params(oracle.BASELINE_ARCH, seed=0)
        ids = torch.randint(0, 50304, (1, max(self.STARTS)), generator=torch.Generator().manual_seed(3))
        self.windows = []
        with torch.no_grad():
            for start in self.STARTS:
                dec = oracle.Decoder(P, oracle.BASELINE_ARCH)
                logits = dec.forward(ids[:, :start])
                self.windows.append([dec, logits[0, -1].argmax().view(1, 1)])
        self.ctx_seen = [[None, None] for _ in self.STARTS]

    def sample(self, seconds: float):
        """Decode steps for about `seconds`, a third in each window; returns
        the per-step times."""
        times = []
        with torch.no_grad():
            for wi, w in enumerate(self.windows):
                dec, tok = w
                t_end = time.perf_counter() + seconds / len(self.windows)
                while time.perf_counter() < t_end and dec.position < dec.max_seq:
                    ctx = dec.position + 1
                    t0 = time.perf_counter()
                    logits = dec.forward(tok)
                    tok = logits[0, -1].argmax().view(1, 1)
                    times.append(time.perf_counter() - t0)
                    lo, hi = self.ctx_seen[wi]
                    self.ctx_seen[wi] = [ctx if lo is None else lo, ctx]
                w[1] = tok
        return times

    def describe(self, times) -> str:
        ranges = ", ".join(f"{lo}-{hi}" for lo, hi in self.ctx_seen if lo is not None)
        times = sorted(times)
        return (f"BASELINE arch fp32, {len(times)} greedy decode steps at contexts {ranges} after prefills of "
                f"{', '.join(map(str, self.STARTS))} tokens (p50 {times[len(times) // 2] * 1e3:.1f} ms/token)")


def cpu_baseline(seconds: float = 15.0):
    """The reference path on the host cores (see CpuWindows); bounded sample."""
    w = CpuWindows()
    times = w.sample(seconds)
    return {"value": len(times) / sum(times), "unit": "tok/s", "cores": w.cores, "kind": "port",
            "sample": w.describe(times)}


def run_reference(args):
    """--impl reference: the reference algorithm's CPU path (oracle port), each
    step a bounded sample spread over the bench's context range."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    w = CpuWindows()
    for _ in range(args.warmup):
        w.sample(1.0)
    steps_t, all_times = [], []
    for _ in range(args.steps):
        t = w.sample(args.cpu_seconds / max(1, args.steps))
        all_times += t
        steps_t.append(len(t) / sum(t))
    value = statistics.median(steps_t)
    cb = {"value": value, "unit": "tok/s", "cores": w.cores, "kind": "port", "sample": w.describe(all_times)}
    return {
        "metric": METRIC,
        "value": value,
        "unit": "tok/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "impl": "reference",
        "config": {"workload": "config[3]-shaped decode on the host cores: greedy decode steps at contexts spread "
                               "over 513-1536 (see cpu_baseline.sample)"},
        "cpu_baseline": cb,
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def measure_allreduce(device, payload: str, n: int, calls: int = 96, reps: int = 5) -> float:
    """The expert-parallel step's collective alone: device time of one NCCL
    all-reduce (sum) of the [n] MoE partial, fp32 or bf16, from a CUDA graph of
    ``calls`` back-to-back all-reduces (max over ranks), in us."""
    import torch.distributed as dist

    buf = torch.ones(n, device=device, dtype=torch.float32 if payload == "fp32" else torch.bfloat16)
    s = torch.cuda.Stream(device=device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        for _ in range(3):
            dist.all_reduce(buf)
    torch.cuda.current_stream(device).wait_stream(s)
    torch.cuda.synchronize(device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(calls):
            dist.all_reduce(buf)
    g.replay()
    torch.cuda.synchronize(device)
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize(device)
    t = torch.tensor([e0.elapsed_time(e1) * 1e3 / (reps * calls)], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del g  # NCCL work in the graph: released before the group goes
    return float(t)


def measure_peer_allreduce(device, n: int, calls: int = 96, reps: int = 5) -> float:
    """``mie_peer_reduce`` alone (this repository's all-reduce over peer
    memory): device time of one call of the [n] fp32 partial from a CUDA graph
    of ``calls`` back-to-back calls, max over ranks, in us."""
    import torch.distributed as dist

    from moe_engine.expert_parallel import PeerReducer

    red = PeerReducer(n, None, device)
    try:
        buf = torch.ones(n, device=device)
        for _ in range(3):
            red(buf, buf)
        torch.cuda.synchronize(device)
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device=device)
        with torch.cuda.graph(g, stream=s):
            for _ in range(calls):
                red(buf, buf)
        g.replay()
        torch.cuda.synchronize(device)
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize(device)
        t = torch.tensor([e0.elapsed_time(e1) * 1e3 / (reps * calls)], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        del g
        if int(red.status.item()):
            raise RuntimeError("mie_peer_reduce reported a timeout")
        return float(t)
    finally:
        red.close()


def measure_expert_parallel(model, alloc, device, world, steps: int, warmup: int, payload: str, want=None,
                            collective: str = "nccl"):
    """config[4b] on the job's process group: one request (the seed-3 prompt
    of rank 0's replica) decoded with the experts of every layer split 8/N
    over the ranks and an NCCL all-reduce of the [768] MoE partial per layer,
    the steps graph-captured with their all-reduces.  Returns tok/s (device
    time, CUDA events, max over ranks) and, when ``want`` holds the
    single-GPU tokens of the same prompt, how many leading tokens agree."""
    from moe_engine.expert_parallel import ExpertParallelDecoder

    prompt = torch.randint(0, 50304, (PROMPT_LEN,), generator=torch.Generator().manual_seed(3))
    ep = ExpertParallelDecoder(model, payload=payload, collective=collective)
    times, new = [], None
    try:
        for it in range(warmup + steps):
            cache = alloc.new_cache()
            _, first = ep.prefill(prompt, cache)
            torch.distributed.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            new = ep.decode(first, NEW_TOKENS, cache)
            e1.record()
            torch.cuda.synchronize()
            cache.free()
            if it >= warmup:
                times.append(e0.elapsed_time(e1) / 1e3)
    finally:
        ep.close()  # graphs (NCCL work) and peer buffers released before the group goes
    t = torch.tensor([sum(times)], device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    out = {"payload": payload, "collective": ep.active, "tok_s": steps * NEW_TOKENS / float(t),
           "tokens": int(new.numel())}
    if want is not None:
        got = new.tolist()
        agree = 0
        for a, b in zip(got, want):
            if a != b:
                break
            agree += 1
        out["tokens_equal_single_gpu"] = agree == len(want) == len(got)
        out["leading_tokens_equal"] = agree
    return out


def run_expert_parallel(args, rank, world, device):
    """--mode ep: the expert-parallel measurement alone, as its own JSON line."""
    model = build_model(device, torch.bfloat16)
    max_blocks = -(-(PROMPT_LEN + NEW_TOKENS) // 16)
    alloc = model.new_block_allocator(num_blocks=max_blocks + 8, block_size=16, attention_mode="direct")
    res = measure_expert_parallel(model, alloc, device, world, args.steps, args.warmup, "fp32", collective="auto")
    value = res["tok_s"]
    return {
        "metric": METRIC + " -- expert parallel",
        "value": value,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": NEW_TOKENS / value * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (random-init weights N(0,0.02), seeded random prompt ids)",
        "config": {"workload": "config[4b] expert parallel: config[3] request, experts split %d/%d per rank, "
                               "NCCL all-reduce of the fp32 [768] MoE partial per layer, steps graph-captured"
                               % (model.config.num_experts // world, model.config.num_experts),
                   "parallelism": f"ep{world}"},
        "per_stream_tok_s": value,
        "aggregate_tok_s": value,
    }


def run_profile(steps: int):
    """Profiling workload (``--profile N``): the bench's model, prompt and paged
    cache, then N decode steps replayed from the captured graph; no timing.
    Kept small so an ncu capture of one step launch ends quickly."""
    device = torch.device("cuda", 0)
    model = build_model(device, torch.bfloat16)
    prompt = torch.randint(0, 50304, (PROMPT_LEN,), generator=torch.Generator().manual_seed(3))
    alloc = model.new_block_allocator(num_blocks=-(-(PROMPT_LEN + steps) // 16) + 8, block_size=16,
                                      attention_mode="direct")
    cache = alloc.new_cache()
    runner = model.decode_runner()
    with torch.no_grad():
        logits = model(prompt[None].to(device), cache)
    P = cache.position
    cache.reserve(P + steps)
    graph = runner.graph_for(cache, P + steps)
    runner.token.fill_(int(logits[0, -1].float().argmax()))
    runner.pos.fill_(P)
    runner.done.zero_()
    runner.log_count.zero_()
    for _ in range(steps):
        graph.replay()
    torch.cuda.synchronize()
    runner.check_status()
    print(json.dumps({"profile_steps": steps, "tokens": int(runner.log_count.item())}), flush=True)


def run_profile_ops(reps: int):
    """Profiling workload (``--profile-ops N``): N calls of the per-op fused MoE
    kernel (config[1] shapes, the 12 layers cycled; then N with int8 and N with
    int4 experts, groups of 128) and N calls of the per-op
    attention kernel (config[2], context 8192, rotating block tables of a
    256 MB pool); no timing."""
    import ctypes
    import math

    from moe_engine import capi, fused_moe, paged_attention

    device = torch.device("cuda", 0)
    model = build_model(device, torch.bfloat16)
    layers = [(blk.moe, blk.moe._expert_storage) for blk in model.MoEBlocks]
    xs = torch.randn(len(layers), 768, generator=torch.Generator().manual_seed(1)).to(device, torch.bfloat16)
    for i in range(reps):
        moe, s = layers[i % len(layers)]
        fused_moe.decode(xs[i % len(layers)].view(1, 1, 768), moe.router.weight, s["w1"], None, s["w2"], None,
                         router_logits=moe._router_logits, expert_ids=moe._expert_ids,
                         route_weights=moe._route_weights, hidden=moe._expert_hidden, out=moe._direct_out,
                         w3_base=s["w3"], sync=moe._sync)
    # the same calls with int8, then int4 experts (groups of 128)
    for bits in (8, 4):
        qs = [{k: fused_moe.quantize_experts(s[k], bits, 128) for k in ("w1", "w3", "w2")} for _, s in layers]
        for i in range(reps):
            moe, _ = layers[i % len(layers)]
            q = qs[i % len(layers)]
            fused_moe.decode(xs[i % len(layers)].view(1, 1, 768), moe.router.weight, q["w1"], None, q["w2"], None,
                             router_logits=moe._router_logits, expert_ids=moe._expert_ids,
                             route_weights=moe._route_weights, hidden=moe._expert_hidden, out=moe._direct_out,
                             w3_base=q["w3"], sync=moe._sync)
        del qs
    lib = capi.ensure_init(device)
    H, hd, bs, ctx = 12, 64, 16, 8192
    nb = ctx // bs
    R = 11
    gen = torch.Generator().manual_seed(2)
    k = torch.randn(R * nb, H, bs, hd, generator=gen).to(device, torch.bfloat16)
    v = torch.randn(R * nb, H, bs, hd, generator=gen).to(device, torch.bfloat16)
    tables = torch.randperm(R * nb, generator=gen).view(R, nb).to(torch.int32).to(device)
    q = torch.randn(H, hd, generator=gen).to(device, torch.bfloat16)
    o = torch.empty(H, hd, dtype=torch.bfloat16, device=device)
    partials = torch.zeros(H * paged_attention.MAX_SPLITS * (hd + 2), dtype=torch.float32, device=device)
    counters = torch.zeros(H, dtype=torch.int32, device=device)
    for i in range(reps):
        a = capi.AttnArgs()
        a.kv_dtype = a.q_dtype = a.out_dtype = capi.dtype_code(torch.bfloat16)
        a.num_heads, a.head_dim = H, hd
        a.q, a.k, a.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
        a.block_table = tables[i % R].data_ptr()
        a.num_blocks, a.block_size = R * nb, bs
        a.stride_block, a.stride_head, a.stride_tok = H * bs * hd, bs * hd, hd
        a.ctx_len, a.max_ctx = ctx, nb * bs
        a.scale = 1.0 / math.sqrt(hd)
        a.out, a.partials, a.counters = o.data_ptr(), partials.data_ptr(), counters.data_ptr()
        a.splits = paged_attention.choose_splits(H, nb, lib.mie_num_sms(0))
        a.max_splits = paged_attention.MAX_SPLITS
        capi.check(lib.mie_attn_decode(ctypes.byref(a), capi.stream_handle(device)), "mie_attn_decode")
    torch.cuda.synchronize()
    print(json.dumps({"profile_ops": reps}), flush=True)


def run_profile_prefill(reps: int):
    """Profiling workload (``--profile-prefill N``): the bench's model and
    512-token prompt prefilled N times into fresh paged caches (tensor-core
    GEMMs of the prefill); no timing."""
    device = torch.device("cuda", 0)
    model = build_model(device, torch.bfloat16)
    prompt = torch.randint(0, 50304, (PROMPT_LEN,), generator=torch.Generator().manual_seed(3))
    alloc = model.new_block_allocator(num_blocks=-(-PROMPT_LEN // 16) + 8, block_size=16, attention_mode="direct")
    for _ in range(reps):
        cache = alloc.new_cache()
        with torch.no_grad():
            model(prompt[None].to(device), cache)
        cache.free()
    torch.cuda.synchronize()
    print(json.dumps({"profile_prefill": reps, "prompt": PROMPT_LEN}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--mode", choices=["replicas", "ep"], default="replicas",
                    help="N>1: independent replicas (default) or one request expert parallel")
    ap.add_argument("--profile", type=int, default=0, metavar="N",
                    help="profiling workload: N decode steps after the prompt, no timing")
    ap.add_argument("--profile-prefill", type=int, default=0, metavar="N",
                    help="profiling workload: N prefills of the 512-token prompt, no timing")
    ap.add_argument("--profile-ops", type=int, default=0, metavar="N",
                    help="profiling workload: N calls each of the per-op MoE and attention kernels, no timing")
    args = ap.parse_args()
    if args.profile:
        run_profile(args.profile)
        return
    if args.profile_prefill:
        run_profile_prefill(args.profile_prefill)
        return
    if args.profile_ops:
        run_profile_ops(args.profile_ops)
        return
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")

    if args.impl == "reference":
        res = run_reference(args)
        if res is not None:
            print(json.dumps(res), flush=True)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=device)
    try:
        if args.mode == "ep":
            if world < 2:
                ap.error("--mode ep needs torchrun with 2 or more ranks")
            res = run_expert_parallel(args, rank, world, device)
        else:
            res = run_b200(args, rank, world, device)
        if rank == 0:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
