"""The head-shard exchange kernel (csrc/peer_gather.cu) on ONE GPU: the two ranks' slabs are two local buffers, and the
words a peer would send are written by the host before the launch, so no launch ever waits for another launch. The two-GPU
run of the same kernel over real peer memory is tests/test_gpu_multi.py."""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


class _Rank:
    """What one rank holds: its receive area ll[slot][parity][source][word] of {data, flag} pairs, its gathered rows, call
    counters, status."""

    def __init__(self, B, dl, world, n_slots, dev):
        from freesolo_b200 import lib as L
        n = B * dl // 2
        assert L.load().fsattn_peer_ll_bytes(B, dl, world, n_slots) == n_slots * 2 * world * n * 8
        self.ll = torch.zeros(n_slots, 2, world, n, 2, dtype=torch.int32, device=dev)
        self.y = torch.zeros(B, world * dl, dtype=torch.bfloat16, device=dev)
        self.epoch = torch.zeros(n_slots, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)


def _call(ranks, r, y_local, slot, timeout_ns=10_000_000):
    from freesolo_b200 import lib as L
    B, dl = y_local.shape
    a = L.PeerGather()
    a.y_local, a.y_out = y_local.data_ptr(), ranks[r].y.data_ptr()
    for p, rk in enumerate(ranks):
        a.ll_dst[p] = rk.ll.data_ptr()
    a.epoch, a.status = ranks[r].epoch.data_ptr(), ranks[r].status.data_ptr()
    a.B, a.dl, a.rank, a.world, a.slot, a.pdl = B, dl, r, len(ranks), slot, 0
    a.timeout_ns = timeout_ns
    return L.load().fsattn_peer_gather(C.byref(a), torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("B,dl,world", [(1, 512, 2), (3, 192, 4), (8, 1024, 2)])
def test_exchange_assembles_every_ranks_columns(B, dl, world):
    from freesolo_b200 import lib as L
    dev = _dev()
    n_slots = 3
    ranks = [_Rank(B, dl, world, n_slots, dev) for _ in range(world)]
    g = torch.Generator().manual_seed(B + dl)
    for step in (1, 2, 3):
        for slot in range(n_slots):
            ys = [torch.randn(B, dl, generator=g).to(torch.bfloat16).to(dev) for _ in range(world)]
            want = torch.cat(ys, dim=1)
            for r in range(world):
                # what the peers that have not run yet WOULD have sent by now: the host writes it (no launch waits for a launch)
                for p in range(r + 1, world):
                    ranks[r].ll[slot, step & 1, p, :, 0] = ys[p].view(torch.int32).view(-1)
                    ranks[r].ll[slot, step & 1, p, :, 1] = step
                assert _call(ranks, r, ys[r], slot) == L.OK
                torch.cuda.synchronize()
                assert torch.equal(ranks[r].y, want), (step, slot, r)
            for r in range(world):
                assert int(ranks[r].status.item()) == 0
                assert int(ranks[r].epoch[slot].item()) == step
                # every peer's rows arrived in this rank's receive area with the call count as flag
                for p in range(world):
                    if p != r:
                        assert torch.equal(ranks[r].ll[slot, step & 1, p, :, 0], ys[p].view(torch.int32).view(-1))
                        assert bool((ranks[r].ll[slot, step & 1, p, :, 1] == step).all())


def test_a_peer_that_never_sends_raises_the_status_and_the_call_returns():
    """Words that nothing writes: the poll runs out after its bound (2 ms here), bit 1 of the status word is set, the launch
    returns and the context stays usable; this rank's own columns are written and its rows were sent all the same."""
    from freesolo_b200 import lib as L
    dev = _dev()
    ranks = [_Rank(1, 256, 2, 1, dev) for _ in range(2)]
    y0 = torch.randn(1, 256).to(torch.bfloat16).to(dev)
    assert _call(ranks, 0, y0, 0, timeout_ns=2_000_000) == L.OK
    torch.cuda.synchronize()
    assert int(ranks[0].status.item()) == 0b10
    assert torch.equal(ranks[0].y[:, :256], y0)
    assert torch.equal(ranks[1].ll[0, 1, 0, :, 0], y0.view(torch.int32).view(-1)) and bool((ranks[1].ll[0, 1, 0, :, 1] == 1).all())
    assert int(ranks[0].epoch[0].item()) == 1
    assert float(torch.ones(4, device=dev).sum().item()) == 4.0


def test_bad_arguments_are_refused_on_the_host():
    from freesolo_b200 import lib as L
    _dev()
    a = L.PeerGather()
    assert L.load().fsattn_peer_gather(C.byref(a), None) == L.EINVAL
