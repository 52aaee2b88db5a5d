"""The protocol of the head-shard exchange kernel (csrc/peer_gather.cu) among CPU processes: a Python restatement of what
one launch does - call count from a local counter, {data, flag} words stored into every peer's receive area
ll[slot][call parity][source rank][word], a bounded poll of the rank's own area, a status bit when the poll runs out - run by
two processes over shared memory with random delays between their calls. It pins the part no single-GPU test can: that a
word is never overwritten before its reader has taken it, although the ranks run unsynchronised, and that a rank whose peer
never sends returns with its status bit set instead of waiting for ever. (The kernel itself runs in tests/test_gpu_peer.py
on one GPU and in tests/test_gpu_multi.py over real peer memory.)"""
import random
import time

import torch
import torch.multiprocessing as mp


def _word(data: int, flag: int) -> int:
    return (flag << 32) | (data & 0xFFFFFFFF)           # one 8-byte store carries both, as in the kernel


def gather_call(ll, epoch, status, y_out, rows, rank, world, slot, timeout_s):
    """One call of rank `rank` for `slot`. ll[r]: rank r's receive area (n_slots, 2, world, n) int64; epoch / status / y_out:
    this rank's own. rows: this rank's n data words. Mirrors peer_gather_kernel step by step."""
    n = rows.numel()
    e = int(epoch[slot]) + 1
    par = e & 1
    for p in range(world):                              # 1. my rows: to every peer with the flag, and into my own columns
        if p != rank:
            for i in range(n):
                ll[p][slot, par, rank, i] = _word(int(rows[i]), e)
    y_out[rank] = rows
    t0 = time.monotonic()
    for p in range(world):                              # 2. the peers' rows out of my own receive area
        if p == rank:
            continue
        for i in range(n):
            while True:
                w = int(ll[rank][slot, par, p, i])
                if (w >> 32) == e:
                    y_out[p, i] = w & 0xFFFFFFFF
                    break
                if time.monotonic() - t0 > timeout_s:
                    status[0] |= 1 << p
                    break
            if int(status[0]) & (1 << p):
                break
    epoch[slot] = e


def _rows(rank, slot, step, n):
    return torch.tensor([(rank * 1000003 + slot * 7919 + step * 104729 + i * 31) & 0x7FFFFFFF for i in range(n)], dtype=torch.int64)


def _rank_main(rank, world, ll, out, n_slots, n, steps, silent_rank):
    rng = random.Random(17 + rank)
    epoch = torch.zeros(n_slots, dtype=torch.int64)
    status = torch.zeros(1, dtype=torch.int64)
    y = torch.zeros(world, n, dtype=torch.int64)
    ok = True
    if rank != silent_rank:
        for step in range(1, steps + 1):
            for slot in range(n_slots):
                if rng.random() < 0.3:
                    time.sleep(rng.random() * 0.003)    # the ranks drift apart: up to a slot, never more (the protocol's own bound)
                gather_call(ll, epoch, status, y, _rows(rank, slot, step, n), rank, world, slot,
                            timeout_s=0.3 if silent_rank >= 0 else 20.0)
                if silent_rank < 0:
                    want = torch.stack([_rows(r, slot, step, n) for r in range(world)])
                    ok = ok and bool(torch.equal(y, want))
                if int(status[0]):
                    break
            if int(status[0]):
                break
    out[rank, 0] = int(ok)
    out[rank, 1] = int(status[0])
    out[rank, 2] = int(epoch.sum())


def _run(world, n_slots, n, steps, silent_rank=-1):
    ll = [torch.zeros(n_slots, 2, world, n, dtype=torch.int64).share_memory_() for _ in range(world)]
    out = torch.full((world, 3), -1, dtype=torch.int64).share_memory_()
    mp.spawn(_rank_main, args=(world, ll, out, n_slots, n, steps, silent_rank), nprocs=world, join=True)
    return out


def test_unsynchronised_ranks_always_read_the_call_they_wait_for():
    out = _run(world=2, n_slots=3, n=16, steps=40)
    assert out[:, 0].tolist() == [1, 1], "a rank read rows of another call"
    assert out[:, 1].tolist() == [0, 0]
    assert out[:, 2].tolist() == [120, 120]


def test_two_slots_are_enough_for_the_parity_buffers():
    out = _run(world=2, n_slots=1, n=8, steps=60)       # one layer only: the call parity alone keeps the calls apart
    assert out[:, 0].tolist() == [1, 1] and out[:, 1].tolist() == [0, 0]


def test_a_rank_whose_peer_never_sends_returns_with_its_status_bit():
    out = _run(world=2, n_slots=2, n=8, steps=3, silent_rank=1)
    assert int(out[0, 1]) == 0b10                       # rank 0 gave up on rank 1 after its bound
    assert int(out[0, 2]) == 1                          # and returned from that first call (its counter advanced once)
