"""The CPU oracle against the fixtures produced by the reference itself (tests/golden/make_golden.py)."""
import numpy as np
import pytest
import torch

from conftest import bf16_from_bits, load_golden
from oracle import fsl

KINDS = ["randn", "vocab", "periodic", "lowprec"]
TIE_FREE = {"randn", "lowprec"}      # kinds whose ceilings have no exact ties (the reference's CPU topk is not tie-stable)


def _inputs(g):
    return tuple(bf16_from_bits(g[k]).float() for k in ("Q", "K", "V"))


def _layer(g, act=torch.float32, **kw):
    n = int(g["N"]) + int(g["T"])
    return fsl.FSLLayerOracle(int(g["H"]), int(g["D"]), lam=torch.from_numpy(g["lam"]), sigma=torch.from_numpy(g["sigma"]),
                              lrs=torch.from_numpy(g["lrs"]), norm_w=torch.from_numpy(g["norm_w"]), eps=float(g["eps"]),
                              act_dtype=act, rope_len=4096, rope_orig_len=4096, **kw)


@pytest.mark.parametrize("kind", KINDS)
def test_cell_stats_and_codec(kind):
    g = load_golden(f"fsl_{kind}")
    Q, K, V = _inputs(g)
    N = int(g["N"])
    kbar, ceil = fsl.cell_stats(K[:, :, :N], 32)
    assert torch.equal(kbar, torch.from_numpy(g["kbar"]))
    assert torch.equal(ceil, torch.from_numpy(g["ceil"]))
    qk, sk = fsl.quantize_cells(K[:, :, :N].to(torch.bfloat16), 32)
    qv, sv = fsl.quantize_cells(V[:, :, :N].to(torch.bfloat16), 32)
    assert np.array_equal(qk.numpy(), g["qk"]) and np.array_equal(qv.numpy(), g["qv"])
    assert np.array_equal(sk.view(torch.int16).numpy(), g["sk"]) and np.array_equal(sv.view(torch.int16).numpy(), g["sv"])
    deq = fsl.dequant_cells(qk, sk, 32)
    assert np.array_equal(deq.view(torch.int16).numpy(), g["deq_k"])
    # the reference's own codec properties (tests/test_kv_int8.py:16-39)
    x = K[:, :, :(N // 32) * 32]
    deq32 = fsl.dequant_cells(qk, sk, 32, dtype=torch.float32)
    err = (deq32 - x).abs().reshape(x.shape[0], x.shape[1], -1, 32 * x.shape[-1]).amax(-1)
    assert (err <= sk.float() * 0.5 * (1 + 1e-6)).all()


@pytest.mark.parametrize("kind", KINDS)
def test_rope_tables(kind):
    g = load_golden(f"fsl_{kind}")
    n = int(g["N"]) + int(g["T"])
    cos, sin = fsl.rope_tables(int(g["D"]), n, orig_len=4096)
    assert torch.equal(cos, torch.from_numpy(g["rope_cos"])) and torch.equal(sin, torch.from_numpy(g["rope_sin"]))


@pytest.mark.parametrize("kind", KINDS)
def test_prefill_selection_window_output(kind):
    g = load_golden(f"fsl_{kind}")
    Q, K, V = _inputs(g)
    N = int(g["N"])
    L = _layer(g)
    y, sel, margin = L.prefill(Q[:, :, :N], K[:, :, :N], V[:, :, :N])
    ref = torch.from_numpy(g["sel_prefill"])
    diff = (sel != ref).any(-1)
    assert not (diff & (margin > 1e-4)).any(), "selection differs from the reference outside the score margin"
    assert diff.float().mean() < 0.01
    assert (y - torch.from_numpy(g["y_prefill"])).abs().max() < 2e-5
    sr = fsl.window_attention(Q[:, :, :N], K[:, :, :N], V[:, :, :N], L.cos, L.sin, 512, L.scale)
    assert (sr - torch.from_numpy(g["window_prefill"])).abs().max() < 5e-6


@pytest.mark.parametrize("kind", KINDS)
def test_decode_steps(kind):
    g = load_golden(f"fsl_{kind}")
    Q, K, V = _inputs(g)
    N, T = int(g["N"]), int(g["T"])
    L = _layer(g)
    L.prefill(Q[:, :, :N], K[:, :, :N], V[:, :, :N])
    for t in range(T):
        sl = slice(N + t, N + t + 1)
        y, sel, margin = L.decode(Q[:, :, sl], K[:, :, sl], V[:, :, sl])
        ref = torch.from_numpy(g["sel_decode"][t])
        got = torch.full_like(ref, -1)
        got[..., :sel.shape[-1]] = sel[:, :, 0]
        bad = (got != ref).any(-1) & (margin[:, :, 0] > 1e-4)
        assert not bad.any(), f"decode step {t}: selection differs outside the margin"
        # outputs agree even where tied cells were swapped only if the cells hold equal tokens (periodic): check loosely
        assert (y - torch.from_numpy(g["y_decode"][:, t:t + 1])).abs().max() < 2e-5


@pytest.mark.parametrize("kind", sorted(TIE_FREE))
def test_decode_pool(kind):
    g = load_golden(f"fsl_{kind}")
    Q, K, V = _inputs(g)
    N = int(g["N"])
    kbar, ceil = fsl.cell_stats(K[:, :, :N], 32)
    pool = fsl.fsl_decode_pool(kbar, ceil, (N // 128) * 128, 32, 64, 8)
    if kind == "randn":
        assert np.array_equal(pool["cand_c"].numpy(), g["pool_cand_c"])
    assert np.array_equal(pool["ok_cell"].numpy(), g["pool_ok"])
    # as sets the pool always agrees with the reference's (ties only permute equal ceilings)
    a = np.where(g["pool_ok"], g["pool_cand_c"], -1)
    b = np.where(pool["ok_cell"].numpy(), pool["cand_c"].numpy(), -1)
    assert np.array_equal(np.sort(ceil.numpy()[0, 0][np.maximum(a[0, 0], 0)]), np.sort(ceil.numpy()[0, 0][np.maximum(b[0, 0], 0)]))


def test_int8_mode_matches_full_precision_selection():
    """Statistics come from the un-quantised keys, so selections do not depend on the int8 store (kv_int8.py:7-8)."""
    g = load_golden("fsl_randn")
    Q, K, V = _inputs(g)
    N, T = int(g["N"]), 6
    La, Lb = _layer(g), _layer(g, int8=True)
    La.prefill(Q[:, :, :N], K[:, :, :N], V[:, :, :N])
    Lb.prefill(Q[:, :, :N], K[:, :, :N], V[:, :, :N])
    for t in range(T):
        sl = slice(N + t, N + t + 1)
        ya, sa, _ = La.decode(Q[:, :, sl], K[:, :, sl], V[:, :, sl])
        yb, sb, _ = Lb.decode(Q[:, :, sl], K[:, :, sl], V[:, :, sl])
        assert torch.equal(sa, sb)
        assert (ya - yb).abs().max() < 0.05


def test_bounded_keep_set_is_readable_set():
    """kv_bounded.py:4-19: a cell outside a block's top-P stays outside every later top-P."""
    torch.manual_seed(3)
    ceil = torch.rand(1, 2, 200)
    s, Bq, P, Wc, W = 32, 128, 16, 4, 512
    for N in (640, 1000, 3000, 6400):
        nc = N // s
        keep = fsl.bounded_keep_set(ceil[:, :, :nc], N, s, Bq, P, Wc, W)
        blk = (N // Bq) * Bq
        m_vis = min(blk // s, nc)
        # every cell a step of the first decode block can read is kept
        pool = fsl.stable_topk(ceil[:, :, :m_vis], min(P, m_vis))
        assert keep.gather(2, pool).all()
        lo = fsl.bounded_readable_from(blk, m_vis, s, W, Wc)
        assert keep[:, :, lo:].all()
        assert keep.sum(-1).max() <= P + max(-(-W // s), Wc) + Bq // s + 1


def test_config1_fixture_consistency():
    g = load_golden("fsl_config1")
    assert g["sel_prefill"].shape == (1, 16, 4096, 4) and g["sel_decode"].shape == (1, 16, 4)
    sel = g["sel_prefill"].astype(np.int64)
    q = np.arange(4096)[None, None, :, None]
    vis = (sel + 1) * 32 <= (q // 128) * 128
    assert ((sel < 0) | vis).all(), "a selected cell is not visible to its query block"
    assert (sel[:, :, :128] == -1).all(), "block 0 has no long-range read (strict causal)"
    x = torch.randn(1, 4097, 1024, generator=torch.Generator().manual_seed(1234))
    assert abs(float(x.double().sum()) - float(g["x_checksum"])) < 1e-6 * 4097 * 1024


@pytest.mark.parametrize("kind", ["randn", "vocab"])
def test_streaming_cache_fixture_equals_the_fsl_oracle_over_the_whole_sequence(kind):
    """The reference's LinearFSCache (src/fsattn/linear_cache.py), fed 3000 tokens in uneven pieces, selects the cells and
    produces the outputs of the standard FS-L prefill over the same tokens: the FS-L oracle run once over the whole
    sequence is therefore the oracle of the streaming cache too (selections equal in order, outputs to fp32 rounding)."""
    g = load_golden(f"linear_{kind}")
    Q, K, V = _inputs(g)
    H, D, N = int(g["H"]), int(g["D"]), int(g["N"])
    L = fsl.FSLLayerOracle(H, D, W=int(g["W"]), P=int(g["P"]), Wc=int(g["Wc"]), lam=torch.from_numpy(g["lam"]),
                           sigma=torch.from_numpy(g["sigma"]), lrs=torch.from_numpy(g["lrs"]), norm_w=torch.from_numpy(g["norm_w"]),
                           eps=float(g["eps"]), act_dtype=torch.float32, rope_len=4096, rope_orig_len=4096)
    y, sel, margin = L.prefill(Q, K, V)
    ref_sel = torch.from_numpy(g["sel"]).long()
    differ = (sel != ref_sel).any(-1)
    assert int((differ & (margin > 1e-4)).sum()) == 0
    assert differ.float().mean() < 0.01
    ref_y = torch.from_numpy(g["y"]).transpose(1, 2).reshape(1, N, H * D)
    assert (y - ref_y).abs().max() < 1e-4
    # the reference's counters: 92 eligible cells after 3000 tokens, 23 block changes, at most P + 4 candidates per merge
    assert g["counters"].tolist() == [N, (N // 128) * 128 // 32, int(g["P"]) + 4, g["counters"][3], N // 128]
