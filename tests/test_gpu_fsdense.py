"""The dense FS variant (no candidate pool: every completed visible cell is scored) on the GPU, through the C ABI, against
the CPU oracle on the same bf16 inputs and against fixtures recorded from the reference (tests/golden/fsdense_*.npz).
Bars as for FS-L: selections identical wherever the oracle's fp32 margin exceeds 1e-4, outputs within max-abs 2e-2 and
mean-rel 1e-3."""
import numpy as np
import pytest
import torch

from conftest import bf16_from_bits, load_golden
from oracle import fsl

pytestmark = pytest.mark.gpu
S, BQ, KK, W = 32, 128, 4, 512


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def _g(kind):
    g = load_golden(f"fsdense_{kind}")
    Q, K, V = (bf16_from_bits(g[k]) for k in ("Q", "K", "V"))
    return g, Q, K, V


def _outside_margin(got, want, margin):
    diff = (got.long() != want.long()).any(-1)
    return int((diff & (margin > 1e-4)).sum()), diff.float().mean().item()


@pytest.mark.parametrize("kind", ["randn", "vocab"])
def test_dense_prefill_selection(dev, kind):
    from freesolo_b200 import ops
    g, Q, K, V = _g(kind)
    N = int(g["N"])
    lam, sigma = torch.from_numpy(g["lam"]), torch.from_numpy(g["sigma"])
    Kd = K[:, :, :N].to(dev)
    kbar, ceil = ops.cell_stats(Kd, N // S)
    nb = (N + BQ - 1) // BQ
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    sel = ops.fs_dense_select(Q[:, :, :N].to(dev), kbar, ceil, lam, sigma, N=N, ncell=N // S, Bq=BQ, nb=nb, kk=KK, scale=0.125,
                              status=status).cpu()
    assert int(status.item()) == 0, "a bounded wait inside the tensor-core kernel ran out"
    # the oracle on the statistics the GPU produced: the comparison isolates the selection arithmetic
    want, margin = fsl.fs_dense_select_prefill(Q[:, :, :N].float(), kbar.cpu(), ceil.cpu(), lam, sigma, 0.125, S, BQ, KK, N)
    bad, frac = _outside_margin(sel[:, :, :N], want[:, :, :N], margin[:, :, :N])
    assert bad == 0, f"{bad} dense selections differ from the oracle outside the margin"
    assert frac < 0.02
    assert (sel[:, :, :BQ] == -1).all()
    # and against the reference's own selections (fp32 chunk means there): as sets, on almost every query
    ref = torch.from_numpy(g["sel_prefill"]).long()
    same = (sel[:, :, :N].long().sort(-1).values == ref.sort(-1).values).all(-1)
    assert same.float().mean() > 0.9


def test_dense_prefill_selection_many_cells_and_ragged(dev):
    """More cells than one 64-cell tile per block, several tiles in flight, a ragged last block, sigma large enough that
    the erf path covers whole tiles, batch 2."""
    from freesolo_b200 import ops
    B, H, N, D = 2, 3, 5000, 64
    gen = torch.Generator().manual_seed(4)
    Q = torch.randn(B, H, N, D, generator=gen).to(torch.bfloat16)
    K = (torch.randn(B, H, N, D, generator=gen) * (0.5 + torch.rand(B, H, N, 1, generator=gen))).to(torch.bfloat16)
    lam = torch.tensor([0.7, 1.5, 2.2])
    sigma = torch.tensor([3.0, 40.0, 300.0])
    kbar, ceil = ops.cell_stats(K.to(dev), N // S)
    nb = (N + BQ - 1) // BQ
    sel = ops.fs_dense_select(Q.to(dev), kbar, ceil, lam, sigma, N=N, ncell=N // S, Bq=BQ, nb=nb, kk=KK, scale=0.125).cpu()
    want, margin = fsl.fs_dense_select_prefill(Q.float(), kbar.cpu(), ceil.cpu(), lam, sigma, 0.125, S, BQ, KK, N)
    bad, frac = _outside_margin(sel[:, :, :N], want[:, :, :N], margin[:, :, :N])
    assert bad == 0 and frac < 0.02, (bad, frac)


@pytest.mark.parametrize("splits", [1, 2, 8])
def test_dense_decode_selection(dev, splits):
    from freesolo_b200 import ops
    g, Q, K, V = _g("randn")
    N, T = int(g["N"]), int(g["T"])
    lam, sigma = torch.from_numpy(g["lam"]), torch.from_numpy(g["sigma"])
    lam_d, sig_d = lam.to(dev), sigma.to(dev)
    Kd, Qd = K.to(dev), Q.to(dev)
    pos_t = torch.zeros((), dtype=torch.int64, device=dev)
    for t in range(T):
        pos = N + t
        nc = (pos + 1) // S
        kbar, ceil = ops.cell_stats(Kd[:, :, :nc * S], nc)
        pos_t.fill_(pos)
        sel = ops.fs_dense_decode_select(Qd[:, :, pos], kbar, ceil, lam_d, sig_d, pos_t, Bq=BQ, kk=KK, scale=0.125, ncell_cap=nc,
                                         splits=splits).cpu()
        want, margin = fsl.fs_dense_decode_select(Q[:, :, pos:pos + 1].float(), kbar.cpu(), ceil.cpu(), pos, lam, sigma, 0.125, S, BQ, KK)
        bad, _ = _outside_margin(sel.unsqueeze(2), want, margin)
        assert bad == 0, f"step {t}: dense decode selection differs from the oracle outside the margin"


def _dense_layer(g, dev):
    from freesolo_b200.fsattn import FSAttn, FSKVCache
    from freesolo_b200.serving import serve_kwargs
    H, D = int(g["H"]), int(g["D"])
    a = FSAttn(d_model=H * D, n_heads=H, causal=True, bias=False, max_seq_len=4096, **serve_kwargs("dense")).to(dev).eval()
    with torch.no_grad():
        a.sel_scale.copy_(torch.from_numpy(g["lam"]))
        a.log_sigma.copy_(torch.from_numpy(g["sigma"]).log())
        a.long_range_scale.copy_(torch.from_numpy(g["lrs"]).view(H, 1, 1))
        a.lr_norm.scale.copy_(torch.from_numpy(g["norm_w"]))
    c = FSKVCache(a)
    c.reserve = int(g["T"]) + 8
    return a, c


@pytest.mark.parametrize("kind", ["randn", "vocab"])
@pytest.mark.parametrize("int8", [False, True])
def test_dense_layer_prefill_then_decode(dev, kind, int8, monkeypatch):
    """FSAttn in the dense configuration behind FSKVCache: prefill and the decode run of the fixture, against the oracle on
    the same bf16 inputs and against the reference's fp32 outputs on the rows whose selections agree."""
    monkeypatch.setenv("FSATTN_KEEP_SEL", "1")
    g, Q, K, V = _g(kind)
    N, T = int(g["N"]), int(g["T"])
    H, D = int(g["H"]), int(g["D"])
    a, c = _dense_layer(g, dev)
    if int8:
        c.enable_int8()
    Qd, Kd, Vd = Q.to(dev), K.to(dev), V.to(dev)
    p = dict(lam=torch.from_numpy(g["lam"]), sigma=torch.from_numpy(g["sigma"]), lrs=torch.from_numpy(g["lrs"]),
             norm_w=torch.from_numpy(g["norm_w"]))
    with torch.no_grad():
        y0 = a._prefill(Qd[:, :, :N], Kd[:, :, :N], Vd[:, :, :N], c).clone()
    sel0 = a._last_sel[:, :, :N].cpu()
    Qf, Kf, Vf = Q.float(), K.float(), V.float()
    kbar, ceil = fsl.cell_stats(K[:, :, :N], S)
    so, mo = fsl.fs_dense_select_prefill(Qf[:, :, :N], kbar, ceil, p["lam"], p["sigma"], 0.125, S, BQ, KK, N)
    bad, _ = _outside_margin(sel0, so[:, :, :N], mo[:, :, :N])
    assert bad == 0
    cos, sin = fsl.rope_tables(D, 4096, torch.bfloat16, orig_len=4096)
    sr = fsl.window_attention(Qf[:, :, :N], Kf[:, :, :N], Vf[:, :, :N], cos, sin, W, 0.125, act_dtype=torch.bfloat16).to(torch.bfloat16)
    pad = torch.full((1, H, (-N) % BQ, KK), -1, dtype=torch.int32)
    o = fsl.cell_readout(Qf[:, :, :N], Kf[:, :, :N], Vf[:, :, :N], torch.cat([sel0, pad], dim=2), S, BQ, 0.125, 0, N)
    want = fsl.lr_norm_combine(sr, o, p["norm_w"], p["lrs"], float(g["eps"]))
    d = (y0.float().cpu() - want.float()).abs()
    assert d.max() <= 2e-2 and d.mean() / want.float().abs().mean() <= 1e-3, (d.max().item(), (d.mean() / want.float().abs().mean()).item())
    # decode: the oracle's FS-L layer model with the dense selection swapped in
    orc = fsl.FSLLayerOracle(H, D, eps=float(g["eps"]), rope_len=4096, rope_orig_len=4096, int8=int8, **p)
    orc.K, orc.V, orc.pos = K[:, :, :N].clone(), V[:, :, :N].clone(), N
    num = den = 0.0
    for t in range(T):
        pos = N + t
        with torch.no_grad():
            y = a._decode_one(Qd[:, :, pos], Kd[:, :, pos], Vd[:, :, pos], c)
        sel = a._last_sel.cpu()
        orc.K = torch.cat([orc.K, K[:, :, pos:pos + 1]], dim=2)
        orc.V = torch.cat([orc.V, V[:, :, pos:pos + 1]], dim=2)
        kb, ce = fsl.cell_stats(orc.K, S)
        sw, mw = fsl.fs_dense_decode_select(Qf[:, :, pos:pos + 1], kb, ce, pos, p["lam"], p["sigma"], 0.125, S, BQ, KK)
        bad, frac = _outside_margin(sel.unsqueeze(2), sw, mw)
        assert bad == 0, f"step {t}: decode selection differs outside the margin"
        Kr, Vr = orc._kv_read()
        j0 = max(0, pos - W)
        sr = fsl.window_attention(Qf[:, :, pos:pos + 1], Kr[:, :, j0:pos + 1].float(), Vr[:, :, j0:pos + 1].float(), orc.cos, orc.sin, W,
                                  0.125, q_pos0=pos, k_pos0=j0, act_dtype=torch.bfloat16).to(torch.bfloat16)
        o = fsl.cell_readout(Qf[:, :, pos:pos + 1], Kr.float(), Vr.float(), sel.unsqueeze(2), S, BQ, 0.125, pos, pos + 1)
        yo = fsl.lr_norm_combine(sr, o, p["norm_w"], p["lrs"], float(g["eps"]))
        dd = (y.float().cpu().view(-1) - yo.float().view(-1)).abs()
        assert dd.max() <= 2e-2, f"step {t}: max-abs {dd.max().item():.3e}"
        num += dd.sum().item(); den += yo.float().abs().sum().item()
        if not int8:
            ref_sel = torch.from_numpy(g["sel_decode"][t]).long()
            if (sel.long().sort(-1).values == ref_sel.sort(-1).values).all():
                dr = (y.float().cpu().view(-1) - torch.from_numpy(g["y_decode"][:, t]).view(-1)).abs()
                assert dr.max() <= 2e-2
    assert num / den <= 1e-3, f"decode outputs: mean-rel over the run {num / den:.3e}"
    assert c.state.faults() == (0, 0, 0)


def test_dense_model_graph_decoder_matches_eager_steps(dev):
    """A dense-FS model through the whole-step graph decoder: tokens equal the un-captured steps across a block change."""
    from freesolo_b200.serving import FreeSoloLM, GraphedDecoder, serve_kwargs
    torch.manual_seed(0)
    m = FreeSoloLM.from_config("debug", max_seq_len=2048, **serve_kwargs("dense")).to(dev).to(torch.bfloat16).eval()
    P0, T = 700, 150
    ids = torch.randint(0, 32000, (2, P0), generator=torch.Generator().manual_seed(3))
    runs = []
    for eager in (10 ** 9, 2):
        gd = GraphedDecoder(m, ids, Lmax=P0 + T + 8, device=dev, kv="int8", eager_steps=eager)
        toks = [gd.prefill().clone()]
        for _ in range(T - 1):
            toks.append(gd.step().clone())
        runs.append((torch.cat(toks, dim=1).cpu(), gd))
    assert runs[0][1].graph is None and runs[1][1].graph is not None
    assert torch.equal(runs[0][0], runs[1][0]), "graph replay diverges from the un-captured steps"
    assert runs[1][1].kv_faults() == (0, 0, 0)
