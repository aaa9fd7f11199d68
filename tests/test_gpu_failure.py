"""Bounded device waits end the step with an error status, never a hang.

Every wait of the persistent decode step -- on another CTA's exchange words,
on a bulk copy, on the optional start gate -- gives up after
``mie_step_desc.wait_limit_ns`` (default 200 ms).  These tests make a wait run
out without any GPU fault: the step is queued behind a start gate that nothing
opens, with a 1 ms limit.  The step must end on its own, report
MIE_ERR_TIMEOUT through the device status word (``check_status()`` raises
``KernelError``), leave the position, token and cache untouched, and the next
step after the scratch reset must be bit-identical to an undisturbed one.  A
gate opened by a copy on another stream while the step waits lets it run.
The reference has only the host-side counterpart of this atomicity: a forced
direct step that cannot run raises before it touches the cache
(src/moe_engine/model.py:408-432).
"""

import time

import pytest
import torch

from moe_engine import capi
from tests.helpers import baseline_bf16_model, shuffled_paged_cache

pytestmark = pytest.mark.gpu
DEV = "cuda"


KERNELS = [capi.MIE_STEP_FLAT, capi.MIE_STEP_CLUSTER]


def prefilled(kernel):
    m, _, _ = baseline_bf16_model(max_seq=256, num_layers=2)
    m.decode_runner().step_kernel = kernel
    cache = shuffled_paged_cache(m, 256)
    prompt = torch.randint(0, 50304, (20,), generator=torch.Generator().manual_seed(12))
    with torch.no_grad():
        logits = m(prompt[None].to(DEV), cache)
    runner = m.decode_runner()
    assert runner.step_kernel_for(cache) == kernel
    return m, runner, cache, int(logits[0, -1].float().argmax())


@pytest.mark.parametrize("kernel", KERNELS)
def test_closed_start_gate_times_out_and_changes_nothing(kernel):
    m, runner, cache, tok = prefilled(kernel)
    p = cache.position
    t = torch.tensor([[tok]], device=DEV)
    ref_logits = runner.forward_step(t, cache).clone()
    ref_x = runner.x.clone()
    ref_token = int(runner.token.item())
    runner.check_status()

    pools = (cache.allocator.k_pool.clone(), cache.allocator.v_pool.clone())
    cache.position = p
    gate = torch.zeros(1, dtype=torch.int32, device=DEV)
    runner.start_gate, runner.wait_limit_ns = gate, 1_000_000  # 1 ms, nothing opens the gate
    runner.x.zero_()
    t0 = time.perf_counter()
    runner.forward_step(t, cache)
    with pytest.raises(capi.KernelError) as err:
        runner.check_status()  # synchronises
    assert time.perf_counter() - t0 < 5.0
    assert err.value.code == capi.MIE_ERR_TIMEOUT
    assert int(runner.pos.item()) == p and int(runner.token.item()) == tok
    assert torch.equal(cache.allocator.k_pool, pools[0]) and torch.equal(cache.allocator.v_pool, pools[1])
    assert torch.count_nonzero(runner.x) == 0

    # the next step, gate removed, after check_status() reset the scratch
    runner.start_gate, runner.wait_limit_ns = None, 0
    cache.position = p
    logits = runner.forward_step(t, cache)
    runner.check_status()
    assert torch.equal(runner.x, ref_x) and torch.equal(logits, ref_logits)
    assert int(runner.token.item()) == ref_token


@pytest.mark.parametrize("kernel", KERNELS)
def test_gate_opened_from_another_stream_lets_the_step_run(kernel):
    m, runner, cache, tok = prefilled(kernel)
    p = cache.position
    t = torch.tensor([[tok]], device=DEV)
    ref_logits = runner.forward_step(t, cache).clone()
    runner.check_status()
    cache.position = p
    gate = torch.zeros(1, dtype=torch.int32, device=DEV)
    zeroed = torch.cuda.Event()
    zeroed.record()
    one = torch.ones(1, dtype=torch.int32).pin_memory()
    runner.start_gate, runner.wait_limit_ns = gate, 2_000_000_000  # 2 s
    logits = runner.forward_step(t, cache)  # queued; every CTA waits for the gate
    time.sleep(0.05)
    side = torch.cuda.Stream()
    side.wait_event(zeroed)
    with torch.cuda.stream(side):
        gate.copy_(one, non_blocking=True)  # a copy-engine write: needs no SM
    side.synchronize()
    runner.check_status()
    runner.start_gate, runner.wait_limit_ns = None, 0
    assert torch.equal(logits, ref_logits)


def test_peer_exchange_wait_runs_out_then_completes():
    """The expert-parallel exchange (mie_peer_reduce) on one GPU with two
    rank slots in local buffers, as sequential launches (no launch waits on a
    concurrently running one).  Rank 0 alone: its wait for rank 1's words runs
    out after 1 ms and it records MIE_ERR_TIMEOUT.  Rank 1 then: rank 0's words
    of the same call are already there, so it completes with the rank-order
    sum and no error."""
    import ctypes

    lib = capi.ensure_init(torch.device(DEV))
    n, world = 768, 2
    nbytes = lib.mie_peer_buffer_bytes(n, world)
    assert nbytes == 2 * world * n * 8
    bufs = [torch.zeros(nbytes // 8, dtype=torch.int64, device=DEV) for _ in range(world)]
    seqs = [torch.zeros(1, dtype=torch.int32, device=DEV) for _ in range(world)]
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    g = torch.Generator().manual_seed(5)
    ins = [torch.randn(n, generator=g).to(DEV) for _ in range(world)]
    outs = [torch.full((n,), float("nan"), device=DEV) for _ in range(world)]

    def call(rank, limit_ns):
        a = capi.PeerReduceArgs()
        a.n, a.rank, a.world = n, rank, world
        a.in_, a.out = ins[rank].data_ptr(), outs[rank].data_ptr()
        for r in range(world):
            a.bufs[r] = bufs[r].data_ptr()
        a.seq, a.status, a.wait_limit_ns = seqs[rank].data_ptr(), status.data_ptr(), limit_ns
        capi.check(lib.mie_peer_reduce(ctypes.byref(a), capi.stream_handle(torch.device(DEV))), "mie_peer_reduce")

    t0 = time.perf_counter()
    call(0, 1_000_000)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 5.0
    assert int(status.item()) == capi.MIE_ERR_TIMEOUT
    assert int(seqs[0].item()) == 1  # the call is counted all the same
    status.zero_()
    call(1, 1_000_000)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(outs[1], ins[0] + ins[1])
    # invalid requests are refused on the host
    a = capi.PeerReduceArgs()
    a.n, a.rank, a.world = n, 2, world
    assert lib.mie_peer_reduce(ctypes.byref(a), None) == capi.MIE_ERR_INVALID
