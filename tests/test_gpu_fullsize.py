"""Size-independent properties at BASELINE's full sizes (131 072 tokens, 16 heads x 64): the oracle cannot run there in
seconds, so the kernels are checked through invariants of the domain instead - codec round trip, visibility and
distinctness of selections, determinism, and the structure of the FS-B forests."""
import pytest
import torch

pytestmark = pytest.mark.gpu

S, H, D, N = 32, 16, 64, 131072


@pytest.fixture(scope="module")
def data():
    from freesolo_b200 import ops
    dev = torch.device("cuda:0")
    g = torch.Generator(device="cuda").manual_seed(1)
    K = torch.randn(1, H, N, D, device=dev, generator=g).to(torch.bfloat16)
    V = torch.randn(1, H, N, D, device=dev, generator=g).to(torch.bfloat16)
    Q = torch.randn(1, H, N, D, device=dev, generator=g).to(torch.bfloat16)
    ncell = N // S
    kbar = torch.zeros(1, H, ncell, D, device=dev)
    ceil = torch.zeros(1, H, ncell, device=dev)
    kq = torch.zeros(1, H, N, D, dtype=torch.int8, device=dev)
    ks = torch.ones(1, H, ncell, dtype=torch.bfloat16, device=dev)
    ops.cell_ingest(K, V, ncell=ncell, kbar=kbar, ceil=ceil, kq=kq, ks=ks,
                    vq=torch.zeros_like(kq), vs=torch.ones_like(ks))
    return dict(dev=dev, Q=Q, K=K, V=V, kbar=kbar, ceil=ceil, kq=kq, ks=ks, ncell=ncell)


def test_codec_round_trip_and_statistics(data):
    """int8 cell codec at full size: |dequant - x| <= scale / 2 everywhere (the reference's own property,
    tests/test_kv_int8.py:16-39), scale = bf16(amax / 127); ceilings equal the largest token norm of their cell."""
    from freesolo_b200 import ops
    K, kq, ks, ncell = data["K"], data["kq"], data["ks"], data["ncell"]
    deq = ops.dequant_cells(kq, ks)
    err = (deq.float() - K.float()).abs().view(1, H, ncell, S * D).amax(-1)
    bound = ks.float() * 0.5 + K.float().abs().view(1, H, ncell, S * D).amax(-1) * 2 ** -8      # + bf16 rounding of the product
    assert (err <= bound * (1 + 1e-6)).all()
    amax = K.float().abs().view(1, H, ncell, S * D).amax(-1)
    assert torch.equal(ks, (amax / 127.0).to(torch.bfloat16))
    norms = K.float().view(1, H, ncell, S, D).norm(dim=-1).amax(-1)
    assert torch.allclose(data["ceil"], norms, rtol=2e-6, atol=0)


def test_fsl_selection_properties(data):
    from freesolo_b200 import ops
    Q, kbar, ceil, ncell, dev = data["Q"], data["kbar"], data["ceil"], data["ncell"], data["dev"]
    nb = N // 128
    lam = torch.ones(H, device=dev)
    sig = torch.full((H,), 16.0, device=dev)
    topp = ops.fsl_prefix_topp(ceil, ncell, 128, nb, 64)
    # top-P lists: ascending block prefixes only ever admit cells of the prefix, and hold the prefix's largest ceilings
    tp = topp.view(H, nb, 64)
    vis = (torch.arange(nb, device=dev) * 4).view(1, nb, 1)
    assert ((tp < vis) | (tp == -1)).all()
    b = nb - 1
    want = torch.topk(ceil[0, :, :b * 4], 64, dim=-1).values.sort(-1).values
    got = torch.gather(ceil[0], 1, tp[:, b].clamp(min=0).long()).sort(-1).values
    assert torch.equal(got, want)
    sel = ops.fsl_select(Q, kbar, ceil, topp, lam, sig, N=N, ncell=ncell, Bq=128, nb=nb, P=64, Wc=8, kk=4, scale=0.125)
    sel2 = ops.fsl_select(Q, kbar, ceil, topp, lam, sig, N=N, ncell=ncell, Bq=128, nb=nb, P=64, Wc=8, kk=4, scale=0.125)
    assert torch.equal(sel, sel2), "selection is not deterministic"
    blk_cells = (torch.arange(N, device=dev) // 128 * 4).view(1, 1, N, 1)
    assert ((sel < blk_cells) | (sel == -1)).all(), "a selected cell is not complete before its query block"
    srt = sel.sort(-1).values
    dup = (srt[..., 1:] == srt[..., :-1]) & (srt[..., 1:] >= 0)
    assert not dup.any(), "a query selected the same cell twice"
    assert (sel[:, :, 128 * 8:] >= 0).all(), "later blocks always have four visible candidates"


def test_fsb_forest_structure_and_selection_properties(data):
    from freesolo_b200 import ops
    Q, K, kbar, ceil, ncell, dev = data["Q"], data["K"], data["kbar"], data["ceil"], data["ncell"], data["dev"]
    tau = torch.quantile(ceil[0, :, :512], 0.5, dim=-1)
    tau_u = torch.quantile(ceil[0, :, :512], 0.9, dim=-1)
    fo = ops.FsbForests(kbar, ceil, tau, tau_u, cap_cells=ncell)
    fo.ingest(ncell)
    m_cap, k_cap = fo.m_cap, fo.k_cap
    for i, th in enumerate((tau, tau_u)):
        mt = fo.m_tot[i]
        admit = ceil[0] >= th.view(H, 1)
        assert torch.equal(mt.long(), admit.sum(-1)), "admission count"
        for t in (0, H - 1):
            m = int(mt[t])
            adm = fo.adm[i][t, :m].long()
            assert torch.equal(adm, torch.nonzero(admit[t]).flatten()), "admitted ids ascending"
            aux = fo.node_aux[i][t]
            for k in range(k_cap + 1):
                nodes = (2 << k) - 1
                nbase = k * m_cap - m_cap + (m_cap >> k)
                for j in range(0, m >> k, 2):
                    if j > 6 and j < (m >> k) - 3:
                        continue                                   # first and last chunks of every height
                    n0 = nbase + (j >> 1) * nodes
                    meta = aux[n0:n0 + nodes, 3].view(torch.int32)
                    leaves = meta[(1 << k) - 1:].long()
                    want = adm[j << k:(j + 1) << k]
                    assert torch.equal(leaves.sort().values, want), (i, t, k, j, "leaves are not the chunk's cells")
                    assert int(aux[n0, 2].view(torch.int32)) == int(want.min()), "root pmin"
                    assert aux[n0, 1] == ceil[0, t][want].max().clamp(min=0), "root amax"
                    if k > 0:      # a parent covers its children: amax is the max, pmin the min of the two
                        assert aux[n0, 1] == torch.maximum(aux[n0 + 1, 1], aux[n0 + 2, 1])
                        assert int(aux[n0, 2].view(torch.int32)) == min(int(aux[n0 + 1, 2].view(torch.int32)),
                                                                          int(aux[n0 + 2, 2].view(torch.int32)))
                        assert (aux[n0:n0 + (1 << k) - 1, 0] >= 0).all()
    lam = torch.ones(H, device=dev)
    sig = torch.full((H,), 16.0, device=dev)
    sel = ops.fsb_select(fo, Q, K, lam, sig, scale=0.125, N=N)
    sel2 = ops.fsb_select(fo, Q, K, lam, sig, scale=0.125, N=N)
    assert torch.equal(sel, sel2), "FS-B selection is not deterministic"
    blk_cells = (torch.arange(N, device=dev) // 128 * 4).view(1, 1, N, 1)
    assert ((sel < blk_cells) | (sel == -1)).all()
    ok = (ceil[0] >= torch.minimum(tau, tau_u).view(H, 1))             # every selected cell was admitted to a forest
    picked = torch.gather(ok, 1, sel[0].clamp(min=0).long().view(H, -1)).view(H, N, 4)
    assert (picked | (sel[0] < 0)).all()
    srt = sel.sort(-1).values
    assert not ((srt[..., 1:] == srt[..., :-1]) & (srt[..., 1:] >= 0)).any()
    assert (sel[:, :, -128:] >= 0).all()


def test_fsl_selection_of_the_last_blocks_equals_the_oracle(data):
    """The oracle itself at full size, on the part it can do in seconds: the last four 128-query blocks of the 131 072-token
    sequence (each sees ~4090 cells; its pool is the stable top-64 of their ceilings plus the eight newest). Selections must
    be identical wherever the oracle's fp32 margin exceeds 1e-4."""
    from freesolo_b200 import ops
    from oracle import fsl
    Q, kbar, ceil, ncell, dev = data["Q"], data["kbar"], data["ceil"], data["ncell"], data["dev"]
    nb = N // 128
    lam = 0.5 + torch.rand(H, generator=torch.Generator().manual_seed(5)) * 2
    sig = 2.0 + torch.rand(H, generator=torch.Generator().manual_seed(6)) * 60
    topp = ops.fsl_prefix_topp(ceil, ncell, 128, nb, 64)
    sel = ops.fsl_select(Q, kbar, ceil, topp, lam.to(dev), sig.to(dev), N=N, ncell=ncell, Bq=128, nb=nb, P=64, Wc=8, kk=4,
                         scale=0.125).cpu()
    kb, ce = kbar.cpu(), ceil.cpu()
    n_diff = n_q = 0
    for n in range(nb - 4, nb):
        blk_start = n * 128
        vis = blk_start // S
        tp = fsl.stable_topk(ce[:, :, :vis], 64)
        assert torch.equal(topp.view(1, H, nb, 64)[:, :, n].cpu().long(), tp), f"block {n}: top-P list differs from the oracle"
        cand_c, ok = fsl.fsl_candidates(tp, blk_start, S, 8)
        C = cand_c.shape[-1]
        kbc = torch.gather(kb, 2, cand_c[..., None].expand(1, H, C, D))
        clc = torch.gather(ce, 2, cand_c)
        q = Q[:, :, blk_start:blk_start + 128].float().cpu()
        qpos = blk_start + torch.arange(128, dtype=torch.float32)
        score = fsl.fsl_scores(q, kbc, clc, cand_c, ok, qpos, lam, sig, 0.125, S)
        want, margin = fsl._pick(score, cand_c, ok, 4)
        got = sel[:, :, blk_start:blk_start + 128].long()
        diff = (got != want.long()).any(-1)
        assert not (diff & (margin > 1e-4)).any(), f"block {n}: selections differ from the oracle outside the margin"
        n_diff += int(diff.sum()); n_q += diff.numel()
    assert n_diff <= 0.02 * n_q


def test_fsb_selection_at_16k_equals_the_oracle(data):
    """FS-B against the oracle at 16 384 tokens (512 cells per row, forests of height 9): two heads, the first blocks that
    see anything, two in the middle and the last four, exact outside the margin (beam cut-offs and re-rank)."""
    from freesolo_b200 import ops
    from oracle import fsb
    Q, K, kbar, ceil, dev = data["Q"], data["K"], data["kbar"], data["ceil"], data["dev"]
    n, hs = 16384, [3, 12]
    nc = n // S
    Qs, Ks = Q[:, hs, :n].contiguous(), K[:, hs, :n].contiguous()
    kb, ce = kbar[:, hs, :nc].contiguous(), ceil[:, hs, :nc].contiguous()
    tau = torch.quantile(ce[0], 0.5, dim=-1)
    tau_u = torch.quantile(ce[0], 0.9, dim=-1)
    g = torch.Generator().manual_seed(8)
    lam = 0.5 + torch.rand(2, generator=g) * 2
    sig = 2.0 + torch.rand(2, generator=g) * 60
    fo = ops.FsbForests(kb, ce, tau, tau_u, cap_cells=nc)
    fo.ingest(nc)
    sel = ops.fsb_select(fo, Qs, Ks, lam, sig, scale=0.125, N=n).cpu().long()
    blocks = [1, 2, 37, 64, 124, 125, 126, 127]
    so, mo = fsb.fsb_select_prefill(Qs.float().cpu(), Ks.float().cpu(), kb.cpu(), ce.cpu(), tau.cpu(), tau_u.cpu(), lam, sig, 0.125,
                                    blocks=blocks)
    n_diff = n_q = 0
    for b in blocks:
        sl = slice(b * 128, (b + 1) * 128)
        diff = (sel[:, :, sl] != so[:, :, sl]).any(-1)
        bad = diff & (mo[:, :, sl] > 1e-4)
        assert int(bad.sum()) == 0, f"block {b}: {int(bad.sum())} selections differ from the oracle outside the margin"
        n_diff += int(diff.sum()); n_q += diff.numel()
    assert n_diff <= 0.05 * n_q
