"""The FS-B CPU oracle against fixtures produced by the reference itself (tests/golden/make_golden.py, fsb_*.npz):
forest tables, spines, beam cells and visit counts bit for bit; selections and layer outputs."""
import numpy as np
import pytest
import torch

from conftest import bf16_from_bits, load_golden
from oracle import fsb

KINDS = ["randn", "vocab"]
S = 32


def _inputs(g):
    return tuple(bf16_from_bits(g[k]).float() for k in ("Q", "K", "V"))


def _ulp_close(a, b, ulps=1):
    """Equal to within `ulps` fp32 units in the last place: the reference's CPU radii come from torch's vectorised
    sqrt, which is not correctly rounded; the oracle's are IEEE (oracle/fsb.py: ieee_sqrt)."""
    a, b = torch.as_tensor(a, dtype=torch.float32), torch.as_tensor(b, dtype=torch.float32)
    return bool(((a - b).abs() <= ulps * 1.1920929e-07 * torch.maximum(a.abs(), b.abs())).all())


def _padded_stats(K, N):
    """Cell statistics the way the reference's prefill takes them: the last partial cell zero-padded
    (src/fsattn/fsb_tree.py:2372-2383, 2400-2401)."""
    B, H, _, D = K.shape
    M = (N + S - 1) // S
    Kp = torch.cat([K[:, :, :N], torch.zeros(B, H, M * S - N, D)], 2).view(B, H, M, S, D)
    return Kp.mean(3), Kp.norm(dim=-1).amax(-1)


@pytest.mark.parametrize("kind", KINDS)
def test_forest_tables_bit_exact(kind):
    g = load_golden(f"fsb_{kind}")
    _, K, _ = _inputs(g)
    H, D, N = int(g["H"]), int(g["D"]), int(g["N"])
    kbar, ceil = _padded_stats(K, N)
    for tag, tau in (("f", g["tau"]), ("fu", g["tau_u"])):
        ks, bases, lb = list(g[tag + "_ks"]), g[tag + "_bases"], g[tag + "_leafbases"]
        for t in range(H):
            adm = fsb.admitted(ceil[0, t], float(tau[t]))
            mt = int(g[tag + "_mtot"][t])
            assert adm.numel() == mt and np.array_equal(adm.numpy(), g[tag + "_adm"][t, :mt])
            F = fsb.build_forest_row(kbar[0, t], ceil[0, t], adm)
            assert sorted(F["chunks"]) == [k for k in ks if (mt >> k) > 0]
            for k, tb in F["chunks"].items():
                i = ks.index(k)
                nodes = (2 << k) - 1
                C = tb["mu"].shape[0]
                ref = torch.from_numpy(g[tag + "_node"][t, bases[i]:bases[i] + C * nodes]).view(C, nodes, D + 9)
                assert torch.equal(ref[..., :D], tb["mu"]), (tag, t, k, "mu")
                assert _ulp_close(ref[..., D], tb["rad"]), (tag, t, k, "rad")
                assert torch.equal(ref[..., D + 1], tb["amax"]), (tag, t, k, "amax")
                assert torch.equal(ref[..., D + 2].long(), tb["pmin"]), (tag, t, k, "pmin")
                rl = torch.from_numpy(g[tag + "_leaf"][t, lb[i]:lb[i] + (C << k)]).view(C, 1 << k).long()
                assert torch.equal(rl, tb["leaf"]), (tag, t, k, "leaf")


@pytest.mark.parametrize("kind", KINDS)
def test_spines_beams_selections_bit_exact(kind):
    g = load_golden(f"fsb_{kind}")
    Q, K, _ = _inputs(g)
    H, D, N = int(g["H"]), int(g["D"]), int(g["N"])
    ncell = N // S
    kbar, ceil = _padded_stats(K, N)
    kb, ce = kbar[:, :, :ncell], ceil[:, :, :ncell]         # the product's forest: complete cells only
    lam, sigma = g["lam"], g["sigma"]
    scale = D ** -0.5
    Bq = 128
    nb = (N + Bq - 1) // Bq
    sel_ref = torch.from_numpy(g["sel_prefill"]).long()
    n_same = n_all = 0
    for t in range(H):
        rf = fsb.RowForests(kb[0, t], ce[0, t], float(g["tau"][t]), float(g["tau_u"][t]))
        for blk in range(nb):
            row = t * nb + blk
            q0 = blk * Bq
            n = min(Bq, N - q0)
            q = torch.zeros(Bq, D)
            q[:n] = Q[0, t, q0:q0 + n]
            qpos = torch.arange(q0, q0 + Bq, dtype=torch.float32)
            want = {}
            sel, mar = fsb.select_block(rf, min(q0 // S, ncell), q, qpos, float(lam[t]), float(sigma[t]), scale, S,
                                        ce[0, t], K[0, t], want=want)
            assert want["m_b"] == (int(g["sp_mb"][row]), int(g["spu_mb"][row]))
            assert want["height"] == (int(g["sp_height"][row]), int(g["spu_height"][row]))
            for tag, F, flat, mb in (("sp", rf.F, rf.flat, want["m_b"][0]), ("spu", rf.Fu, rf.flatu, want["m_b"][1])):
                sp = fsb.spine(F, flat, mb, D)
                ref = torch.from_numpy(g[tag + "_node"][row])
                for k in range(ref.shape[0]):
                    if ref[k, D + 3] > 0:
                        nd = sp["nodes"][k]
                        assert torch.equal(ref[k, :D], nd["mu"]) and _ulp_close(ref[k, D], nd["rad"], 4)
                        assert ref[k, D + 1] == nd["amax"] and int(ref[k, D + 2]) == nd["pmin"]
                        assert int(ref[k, D + 3]) == nd["cnt"]
                    else:
                        assert k not in sp["nodes"]
            # beams: identical wherever no frontier cut-off was closer than 1e-4 (the radii differ by an ulp)
            clear = want["beam_margin"][:n] > 1e-4
            for mine, ref_c in ((want["main"], g["beam_cells"][row]), (want["union"], g["beamu_cells"][row])):
                same = (mine[:n] == torch.from_numpy(ref_c).long()[:n]).all(-1)
                assert (same | ~clear).all(), (t, blk, "beam differs outside the margin")
                n_same += int(same.sum()); n_all += n
            nv = torch.from_numpy(g["beam_nvis"][row] + g["beamu_nvis"][row])
            assert torch.equal(want["nvis"][:n].int()[clear], nv[:n].int()[clear])
            bad = (sel[:n] != sel_ref[0, t, q0:q0 + n]).any(-1) & (mar[:n] > 1e-4) & clear
            assert not bad.any(), (t, blk, "selection differs outside the margin")
    assert n_same >= 0.999 * n_all, (n_same, n_all)


@pytest.mark.parametrize("kind", KINDS)
def test_layer_prefill_and_decode(kind):
    g = load_golden(f"fsb_{kind}")
    Q, K, V = _inputs(g)
    H, D, N, T = int(g["H"]), int(g["D"]), int(g["N"]), int(g["T"])
    L = fsb.FSBLayerOracle(H, D, tau=g["tau"], tau_u=g["tau_u"], lam=torch.from_numpy(g["lam"]),
                           sigma=torch.from_numpy(g["sigma"]), lrs=torch.from_numpy(g["lrs"]),
                           norm_w=torch.from_numpy(g["norm_w"]), eps=float(g["eps"]), act_dtype=torch.float32,
                           rope_len=4096, rope_orig_len=4096)
    y, sel, margin = L.prefill(Q[:, :, :N], K[:, :, :N], V[:, :, :N])
    diff = (sel != torch.from_numpy(g["sel_prefill"]).long()).any(-1)
    assert not (diff & (margin > 1e-4)).any()
    assert (y - torch.from_numpy(g["y_prefill"])).abs().max() < 2e-5
    for t in range(T):
        sl = slice(N + t, N + t + 1)
        y, sel, margin = L.decode(Q[:, :, sl], K[:, :, sl], V[:, :, sl])
        bad = (sel[:, :, 0] != torch.from_numpy(g["sel_decode"][t]).long()).any(-1) & (margin[:, :, 0] > 1e-4)
        assert not bad.any(), f"decode step {t}"
        assert (y - torch.from_numpy(g["y_decode"][:, t:t + 1])).abs().max() < 2e-5


def test_det_sum_order():
    """The halving order is the contract a device build has to keep: check it on a case where order matters."""
    x = torch.tensor([1e8, 1.0, -1e8, 1.0, 3.0, 0.5])
    # pad to 8: [1e8,1,-1e8,1,3,.5,0,0] -> [1e8+3, 1.5, -1e8, 1] -> [(1e8+3)-1e8, 2.5] -> sum
    a = torch.tensor(1e8) + 3.0
    want = (a + torch.tensor(-1e8)) + (torch.tensor(1.5) + 1.0)
    assert fsb.det_sum(x, 0) == want
    assert fsb.det_sum(torch.ones(3, 5), 1).tolist() == [5.0, 5.0, 5.0]


def test_decode_forest_equals_prefix_forest():
    """A forest over the visible prefix is the same whether the prefix is cut by m_vis or the inputs are sliced."""
    g = torch.Generator().manual_seed(3)
    kb = torch.randn(50, 16, generator=g)
    ce = torch.rand(50, generator=g)
    a = fsb.RowForests(kb, ce, 0.3, 0.6, m_vis=37)
    b = fsb.RowForests(kb[:37], ce[:37], 0.3, 0.6)
    assert torch.equal(a.F["adm"], b.F["adm"]) and torch.equal(a.flat["mu"], b.flat["mu"])
    assert torch.equal(a.flatu["cell"], b.flatu["cell"])
