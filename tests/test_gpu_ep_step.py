"""The expert-parallel persistent step on one GPU, the other ranks emulated.

With ``moe_peer`` (world > 1) the cluster step computes only the selected
experts of its rank's shard and completes each layer's all-reduce inside the
kernel: its down-row owners store the rank's partial as tagged words into
every rank's buffer, and every reader sums the ranks' words in rank order
onto x_mid.  The layer outputs of all steps alternate between two slots of
the buffer (index seq * L + l).  Here one GPU runs rank ``rank`` of ``world``
for a 2-layer model, whose two layer outputs of a step take the two slots, so
one step's words of every layer fit at once.  Before each step the host writes the other
ranks' words -- value 0 with the step's tags -- into this rank's buffer, so no
kernel waits on another launch.

With the other ranks contributing nothing, the step computes the model whose
experts outside the shard output 0.  The checker is the single-GPU persistent
step on that model: the same weights with those experts' down projections
zeroed (the routing is unchanged).  The two differ only in the order of the
combine (x_mid + the rank-order sum of partials, against fused multiply-adds
onto x_mid): hidden states agree to rounding, greedy tokens are identical.  A
rank whose peers never write gives up after the wait limit with
MIE_ERR_TIMEOUT and no fault.
"""

import ctypes
import time

import pytest
import torch

from moe_engine import capi
from moe_engine.decode import DecodeRunner
from tests.helpers import baseline_bf16_model

pytestmark = pytest.mark.gpu
DEV = "cuda"
LAYERS = 2


def peer_slot(seq: int, layer: int) -> int:
    """Buffer slot of ``layer``'s output in the step that starts with the
    group's step counter at ``seq``."""
    return (seq * LAYERS + layer) & 1


def peer_tag(pstep: int, layer: int) -> int:
    """Tag of the cross-GPU exchange words of ``layer``'s output in step
    ``pstep`` (the group's step counter + 1)."""
    return 0x80000000 | ((pstep & 0x7FFFFF) << 8) | layer


class EmulatedGroup:
    """Rank ``rank``'s view of a group of ``world``: every rank's buffer (only
    this rank's is read by the kernel), the device step counter, and the args
    the step descriptor points to."""

    def __init__(self, runner, world: int, rank: int):
        D = runner.config.hidden_dim
        self.D, self.world, self.rank = D, world, rank
        nbytes = runner.lib.mie_peer_buffer_bytes(D, world)
        assert nbytes == 2 * world * D * 8
        self.bufs = [torch.zeros(nbytes // 8, dtype=torch.int64, device=DEV) for _ in range(world)]
        self.seq = torch.zeros(1, dtype=torch.int32, device=DEV)
        a = capi.PeerReduceArgs()
        a.n, a.rank, a.world = D, rank, world
        for r, b in enumerate(self.bufs):
            a.bufs[r] = b.data_ptr()
        a.seq, a.status = self.seq.data_ptr(), runner.status.data_ptr()
        self.args = a

    def others_contribute_zero(self, layers: int = LAYERS) -> None:
        """The other ranks' words of this step's layer outputs, value 0."""
        seq = int(self.seq.item())
        mine = self.bufs[self.rank].view(2, self.world, self.D)
        for layer in range(1, layers + 1):
            word = peer_tag(seq + 1, layer) << 32  # payload bits 0 = +0.0
            word -= 1 << 64  # the top bit is set: as a signed 64-bit word
            for k in range(self.world):
                if k != self.rank:
                    mine[peer_slot(seq, layer), k].fill_(word)


def ep_step(runner, group, cache, token: int):
    """One eager expert-parallel step of ``runner`` (rank ``group.rank``)."""
    P = cache.position
    cache.reserve(P + 1)
    runner.token.fill_(token)
    runner.pos.fill_(P)
    desc, layers = runner.make_desc(cache, logits=True, graph=False, splits=runner.splits_for(P + 1, 16),
                                    moe_peer=ctypes.addressof(group.args))
    assert desc.step_scratch, "the cluster step must take the expert-parallel descriptor"
    runner.launch_step(desc)
    del layers
    cache.position = P + 1
    return runner.logits.clone()


def zero_outside(m, base: int, count: int):
    """The model's experts outside [base, base + count) output 0: their down
    projections zeroed in place."""
    E = m.config.num_experts
    with torch.no_grad():
        for blk in m.MoEBlocks:
            w2 = blk.moe._expert_storage["w2"]
            for e in range(E):
                if not base <= e < base + count:
                    w2[e].zero_()
    return m


def prefilled_pair(m_ref, prompt):
    caches = []
    for _ in range(2):
        alloc = m_ref.new_block_allocator(num_blocks=24, block_size=16, attention_mode="direct")
        c = alloc.new_cache()
        with torch.no_grad():
            logits = m_ref(prompt[None].to(DEV), c)
        caches.append(c)
    return caches, int(logits[0, -1].float().argmax())


@pytest.mark.parametrize("world,rank", [(2, 0), (2, 1), (4, 2)])
def test_ep_step_with_silent_peers_equals_model_without_their_experts(world, rank):
    m, _, _ = baseline_bf16_model(max_seq=320, num_layers=LAYERS)
    E = m.config.num_experts
    count = E // world
    base = rank * count
    m_ref, _, _ = baseline_bf16_model(max_seq=320, num_layers=LAYERS)
    zero_outside(m_ref, base, count)
    prompt = torch.randint(0, 50304, (40,), generator=torch.Generator().manual_seed(21 + rank))
    (c_ref, c_ep), tok = prefilled_pair(m_ref, prompt)

    ref = m_ref.decode_runner()
    assert ref.step_kernel_for(c_ref) == capi.MIE_STEP_CLUSTER
    ep = DecodeRunner(m, expert_base=base, expert_count=count)
    group = EmulatedGroup(ep, world, rank)

    xs_ref, xs_ep, toks_ref, toks_ep = [], [], [], []
    t = tok
    for _ in range(10):
        lr = ref.forward_step(torch.tensor([[t]], device=DEV), c_ref).view(-1).float()
        group.others_contribute_zero()
        le = ep_step(ep, group, c_ep, t).float()
        xs_ref.append(ref.x.clone())
        xs_ep.append(ep.x.clone())
        toks_ref.append(int(lr.argmax()))
        toks_ep.append(int(ep.token.item()))
        assert toks_ep[-1] == int(le.argmax())
        t = toks_ref[-1]  # both sides decode the reference's token
    ref.check_status()
    ep.check_status()
    # one step per launch: the device step counter advanced once per step
    assert int(group.seq.item()) == 10
    assert toks_ep == toks_ref
    a, b = torch.stack(xs_ep), torch.stack(xs_ref)
    rel = float((a - b).norm() / b.norm())
    assert rel < 1e-3, rel
    # every rank's buffer received this rank's partial of the last step's
    # layer outputs, with the last step's tags
    for k in range(world):
        words = group.bufs[k].view(2, world, group.D)[:, rank]
        tags = ((words >> 32) & 0xFFFFFFFF).tolist()
        assert tags[peer_slot(9, 1)] == [peer_tag(10, 1)] * group.D
        assert tags[peer_slot(9, 2)] == [peer_tag(10, 2)] * group.D


def test_ep_step_without_peer_words_times_out_cleanly():
    m, _, _ = baseline_bf16_model(max_seq=320, num_layers=LAYERS)
    prompt = torch.randint(0, 50304, (24,), generator=torch.Generator().manual_seed(5))
    (c_ep, c_ok), tok = prefilled_pair(m, prompt)
    ep = DecodeRunner(m, expert_base=0, expert_count=m.config.num_experts // 2)
    group = EmulatedGroup(ep, 2, 0)
    ep.wait_limit_ns = 2_000_000  # 2 ms; rank 1 never writes
    P = c_ep.position
    t0 = time.perf_counter()
    ep_step(ep, group, c_ep, tok)
    with pytest.raises(capi.KernelError) as err:
        ep.check_status()  # synchronises
    assert time.perf_counter() - t0 < 5.0
    assert err.value.code == capi.MIE_ERR_TIMEOUT
    assert int(ep.pos.item()) == P and int(group.seq.item()) == 0  # the step changed nothing it reports
    # the context is intact: a single-GPU step of the same model runs
    runner = m.decode_runner()
    runner.forward_step(torch.tensor([[tok]], device=DEV), c_ok)
    runner.check_status()
