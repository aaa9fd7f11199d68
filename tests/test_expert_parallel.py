"""Expert-parallel decode (config[4b]): experts split over ranks, the MoE
output completed by an all-reduce of per-rank partials.

* CPU (gloo, 2 and 4 ranks): the decomposition the product relies on -- each
  rank's weighted sum over the selected experts it owns, summed over ranks,
  equals the full MoE output of the oracle; and the expert shard arithmetic.
* GPU (2 ranks, needs 2 GPUs): expert-parallel greedy decode of the
  BASELINE model in fp32 gives the same tokens as the oracle and as the
  single-GPU path with each collective -- the all-reduce fused into the MoE
  kernel, the peer all-reduce kernel, NCCL; the peer all-reduce alone is
  bitwise the rank-order sum, eager and in a CUDA graph.
* GPU (2 ranks): the expert-parallel persistent step (collective "step", the
  all-reduce inside the single-launch cluster step) on the BASELINE model in
  bf16 gives the single-GPU persistent step's greedy tokens for two requests
  on one decoder (graphs of several steps, a step limit that ends mid-graph),
  and hidden states equal to rounding.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from moe_engine.expert_parallel import expert_shard


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_expert_shard():
    assert [expert_shard(8, r, 2) for r in range(2)] == [(0, 4), (4, 4)]
    assert [expert_shard(8, r, 8) for r in range(8)] == [(r, 1) for r in range(8)]
    assert expert_shard(8, 0, 1) == (0, 8)
    with pytest.raises(ValueError):
        expert_shard(8, 0, 3)
    with pytest.raises(ValueError):
        expert_shard(8, 2, 2)


def _decomposition_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        arch = oracle.BASELINE_ARCH.with_(num_layers=1, vocab_size=64, max_seq_length=8, hidden_dim=64,
                                          num_heads=4, expert_hidden_dim=48)
        P = oracle.init_params(arch, seed=7)
        x = torch.randn(1, 1, arch.hidden_dim, generator=torch.Generator().manual_seed(8))
        full, (logits, ids, weights) = oracle.moe_forward(x, P, 0, arch)
        base, count = expert_shard(arch.num_experts, rank, world)
        part = torch.zeros(arch.hidden_dim)
        for slot in range(ids.shape[-1]):
            e = int(ids.view(-1)[slot])
            if base <= e < base + count:
                part += weights.view(-1)[slot] * oracle.expert_forward(x.view(1, -1), P, f"MoEBlocks.0.moe.experts.{e}.",
                                                                       arch).view(-1)
        dist.all_reduce(part)
        if rank == 0:
            out.put((part, full.view(-1)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_partials_all_reduced_equal_full_moe(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_decomposition_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    part, full = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    torch.testing.assert_close(part, full, atol=1e-6, rtol=1e-5)


def _ep_gpu_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from moe_engine.expert_parallel import ExpertParallelDecoder
        from moe_engine.model import Model, baseline_config
        from tests.helpers import engine_state_dict

        P = oracle.init_params(oracle.BASELINE_ARCH, seed=0)
        m = Model(baseline_config()).eval()
        m.load_state_dict(engine_state_dict(P))
        m = m.to(dev, torch.float32)
        prompt = torch.randint(0, 50304, (16,), generator=torch.Generator().manual_seed(0))
        alloc = m.new_block_allocator(num_blocks=16, block_size=16, attention_mode="direct")
        got = {}
        for collective in ("fused", "peer", "nccl"):
            ep = ExpertParallelDecoder(m, collective=collective)
            try:
                got[collective] = ep.generate(prompt, 24, alloc.new_cache())[0].tolist()
                ep.runner.check_status()
            finally:
                ep.close()
        single = m.generate(prompt, max_new_tokens=24, temperature=0)[0].tolist() if rank == 0 else None
        if rank == 0:
            out.put((got, single, oracle.generate_greedy(P, oracle.BASELINE_ARCH, prompt, 24)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="expert parallel needs 2 GPUs")
def test_expert_parallel_greedy_matches_oracle_and_single_gpu():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_ep_gpu_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got, single, want = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for collective in ("fused", "peer", "nccl"):
        assert got[collective] == want, collective
        assert got[collective] == single, collective


def _peer_reduce_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from moe_engine.expert_parallel import PeerReducer

        n = 768
        red = PeerReducer(n, None, dev)
        try:
            errs = 0
            # eager calls, then a graph of 10 calls replayed 3 times: the call counter and the two
            # buffer halves advance on the device
            for call in range(6):
                ins = [torch.randn(n, generator=torch.Generator().manual_seed(100 * call + r)) for r in range(world)]
                x = ins[rank].to(dev)
                red(x, x)  # in place
                want = ins[0].clone()
                for r in range(1, world):
                    want += ins[r]
                errs += int(not torch.equal(x.cpu(), want))
            buf = torch.full((n,), float(rank + 1), device=dev)
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream(device=dev)
            with torch.cuda.graph(g, stream=s):
                for _ in range(10):
                    red(buf, buf)
            for _ in range(3):
                buf.fill_(float(rank + 1))
                g.replay()
                torch.cuda.synchronize(dev)
                total = float(sum(r + 1 for r in range(world)))
                # each call sums the previous sums of every rank: total * world^(calls - 1)
                errs += int(not torch.equal(buf.cpu(), torch.full((n,), total * world ** 9)))
            del g
            status = int(red.status.item())
        finally:
            red.close()
        if rank == 0:
            out.put((errs, status))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="the peer all-reduce needs 2 GPUs")
def test_peer_all_reduce_sums_in_rank_order_eager_and_in_a_graph():
    """mie_peer_reduce on 2 GPUs: bitwise the rank-order fp32 sum, in place,
    over eager calls and CUDA-graph replays; no timeout recorded."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_peer_reduce_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    errs, status = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert errs == 0 and status == 0


def _ep_step_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from moe_engine.expert_parallel import ExpertParallelDecoder
        from tests.helpers import baseline_bf16_model

        m, _, _ = baseline_bf16_model(max_seq=1024, device=dev)
        alloc = m.new_block_allocator(num_blocks=80, block_size=16, attention_mode="direct")
        prompts = [torch.randint(0, 50304, (n,), generator=torch.Generator().manual_seed(40 + n)) for n in (24, 300)]
        lengths = (40, 33)  # 33: the last graph of 8 steps ends after one step
        got, xs = [], []
        ep = ExpertParallelDecoder(m)  # "auto": the persistent step takes these shapes
        try:
            for prompt, n in zip(prompts, lengths):
                cache = alloc.new_cache()
                got.append(ep.generate(prompt, n, cache)[0].tolist())
                ep.runner.check_status()
                xs.append(ep.runner.x.cpu())
                cache.free()
            active = ep.active
            seq = int(ep._peer.seq.item())
        finally:
            ep.close()
        if rank == 0:
            single, xs1 = [], []
            for prompt, n in zip(prompts, lengths):
                single.append(m.generate(prompt, max_new_tokens=n, temperature=0)[0].tolist())
                xs1.append(m.decode_runner().x.cpu())
            out.put((active, seq, got, single, xs, xs1, m.decode_runner().step_kernel_for(alloc.new_cache())))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="expert parallel needs 2 GPUs")
def test_expert_parallel_persistent_step_matches_single_gpu_step():
    from moe_engine import capi

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_ep_step_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    active, seq, got, single, xs, xs1, kernel = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert kernel == capi.MIE_STEP_CLUSTER
    assert active == "step"
    # one advance of the group's step counter per decoded token after the first
    assert seq == (40 - 1) + (33 - 1)
    for g, s, a, b in zip(got, single, xs, xs1):
        assert g == s
        rel = float((a - b).norm() / b.norm())
        assert rel < 1e-3, rel
