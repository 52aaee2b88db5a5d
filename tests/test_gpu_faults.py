"""The failure paths of the device-side waits and counters, made on the host (nothing here faults, traps or hangs a GPU):
a grid barrier whose counter can never reach its target gives up after its bound, sets the status word and lets the kernel
run to its end; a slot store with no free slot counts the overflow instead of writing out of bounds."""
import numpy as np
import pytest
import torch

from conftest import bf16_from_bits, load_golden
from oracle import fsl

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def test_grid_barrier_that_cannot_complete_sets_the_status_word(dev):
    """fsattn_trunk_layer's three grid barriers count arrivals in bar[0..2], which the host owns. With bar[1] preset far
    below zero the second barrier can never see all CTAs arrive: its bounded poll must run out, raise *status and return,
    the launch must complete, and the context must stay usable."""
    from freesolo_b200 import ops
    torch.manual_seed(1)
    M, d, f = 2, 1024, 2816
    bf = dict(device=dev, dtype=torch.bfloat16)
    x, y = torch.randn(M, d, **bf), torch.randn(M, d, **bf)
    w_o = (torch.randn(d, d, device=dev) * 0.03).to(torch.bfloat16)
    w_gu = (torch.randn(2 * f, d, device=dev) * 0.03).to(torch.bfloat16)
    w_dn = (torch.randn(d, f, device=dev) * 0.03).to(torch.bfloat16)
    n2 = torch.ones(d, **bf)
    act = torch.zeros(M, f, **bf)
    bar = torch.zeros(4, dtype=torch.int32, device=dev)
    bar[1] = -(1 << 30)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.trunk_layer(x, y, w_o, n2, 1e-6, w_gu, act, w_dn, bar, status)
    torch.cuda.synchronize()                     # the kernel came back by itself
    assert int(status.item()) == 1, "the barrier's bounded wait did not report that it ran out"
    assert int(bar[0].item()) > 0 and int(bar[1].item()) < 0
    # the context is intact: the same call with honest counters works and reports nothing
    bar.zero_(); status.zero_()
    x2 = torch.randn(M, d, **bf)
    xr = x2.clone()
    ops.trunk_gemv(y, w_o, res=xr, out=xr)
    act_r = ops.trunk_gemv(xr, w_gu, norm_w=n2, eps=1e-6, swiglu=True)
    ops.trunk_gemv(act_r, w_dn, res=xr, out=xr)
    ops.trunk_layer(x2, y, w_o, n2, 1e-6, w_gu, act, w_dn, bar, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0 and torch.equal(x2, xr)


def test_slot_store_without_a_free_slot_counts_the_overflow(dev):
    """A bounded store whose free slots the host has marked as taken (an undersized store): when the next cell closes the
    kernel finds no slot, must count it in the status words and skip the store - no out-of-bounds write, finite outputs -
    and a later block refresh, which wants that cell in its pool, must count the missing slot as well."""
    from freesolo_b200 import lib as L, ops
    g = load_golden("fsl_randn")
    Q, K, V = (bf16_from_bits(g[k]) for k in ("Q", "K", "V"))
    N, T = 1000, 72
    B, H, _, D = Q.shape
    Qd, Kd, Vd = Q.to(dev), K.to(dev), V.to(dev)
    cos, sin = (t.to(dev) for t in fsl.rope_tables(D, 4096, torch.bfloat16, orig_len=4096))
    pd = {k: torch.from_numpy(g[k]).to(dev).float().contiguous() for k in ("lam", "sigma", "lrs", "norm_w")}
    st = ops.FslDecodeState(B, H, D, N + T, dev, mode="bounded")
    st.prefill(Kd[:, :, :N], Vd[:, :, :N], N)
    assert st.faults() == (0, 0, 0)
    guard_k, guard_v = st.kq.clone(), st.vq.clone()
    free = st.cell_in < 0
    assert free.any()
    st.cell_in[free] = 0                          # every free slot now claims to hold cell 0 (which keeps its real slot too)
    pos_t = torch.zeros((), dtype=torch.int64, device=dev)
    ys = []
    for t in range(T):
        pos_t.fill_(N + t)
        ys.append(ops.fsl_decode_step(st, Qd[:, :, N + t], Kd[:, :, N + t], Vd[:, :, N + t], pos_t, cos, sin, pd["lam"], pd["sigma"],
                                      pd["lrs"], pd["norm_w"], scale=0.125, eps=float(g["eps"]), splits=4).clone())
    torch.cuda.synchronize()
    overflow, no_slot, bad_index = st.faults()
    n_closed = (N + T) // 32 - N // 32
    assert overflow == n_closed * B * H, f"{overflow} overflows counted for {n_closed} closed cells x {B * H} heads"
    assert no_slot > 0, "cells without a slot were read without being counted"
    assert bad_index == 0
    assert all(torch.isfinite(y.float()).all() for y in ys)
    # nothing was written into the store: the rows are exactly what the prefill left
    assert torch.equal(st.kq, guard_k) and torch.equal(st.vq, guard_v)
