"""Parity of the FS-L CUDA path (through the C ABI) with the CPU oracle and the reference's golden outputs.

Bars: int8 codes, scales, pool lists and selected cells bit-exact (selections wherever the oracle's fp32 score margin
exceeds 1e-4; exact ties are margin 0); attention outputs within max-abs 2e-2 and mean-rel 1e-3 of the oracle run on the
same bf16 inputs (mean-rel = mean|a-b| / mean|b|), and within max-abs 2e-2 of the reference's fp32 output.
"""
import numpy as np
import pytest
import torch

from conftest import bf16_from_bits, load_golden
from oracle import fsl

pytestmark = pytest.mark.gpu

KINDS = ["randn", "vocab", "periodic", "lowprec"]
MAX_ABS, MEAN_REL, MARGIN = 2e-2, 1e-3, 1e-4
# Against the reference's own fp32 run the bf16 pipeline differs by the bf16 rounding of Q/K/V and of the stored output
# (2^-9 relative per value, about 2e-3 in the mean) before any kernel arithmetic: that comparison alone has a wider bar.
REF_FP32_REL = 4e-3


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def _g(kind):
    g = load_golden(f"fsl_{kind}")
    Q, K, V = (bf16_from_bits(g[k]) for k in ("Q", "K", "V"))
    return g, Q, K, V


def _params(g, dev=None):
    p = dict(lam=torch.from_numpy(g["lam"]), sigma=torch.from_numpy(g["sigma"]), lrs=torch.from_numpy(g["lrs"]),
             norm_w=torch.from_numpy(g["norm_w"]))
    if dev is not None:
        p = {k: v.to(dev).float().contiguous() for k, v in p.items()}
    return p


def _oracle(g, **kw):
    p = _params(g)
    return fsl.FSLLayerOracle(int(g["H"]), int(g["D"]), eps=float(g["eps"]), rope_len=4096, rope_orig_len=4096, **p, **kw)


def _close(got, ref, what, max_abs=MAX_ABS, mean_rel=MEAN_REL):
    got, ref = got.float().cpu(), ref.float().cpu()
    assert got.shape == ref.shape, f"{what}: shape {tuple(got.shape)} vs {tuple(ref.shape)}"
    d = (got - ref).abs()
    ma, mr = d.max().item(), (d.mean() / ref.abs().mean().clamp_min(1e-12)).item()
    assert ma <= max_abs and mr <= mean_rel, f"{what}: max-abs {ma:.3e} (<= {max_abs}), mean-rel {mr:.3e} (<= {mean_rel})"
    return ma, mr


class _RunError:
    """Mean-rel error aggregated over a whole decode run: sum |got - want| / sum |want| over every step's row. One row
    holds only H*D values, so its own mean-rel is a noisy statistic (it keeps a looser bar); the run's must meet MEAN_REL."""

    def __init__(self):
        self.num = self.den = 0.0

    def add(self, got, ref):
        got, ref = got.float().cpu().reshape(-1), ref.float().cpu().reshape(-1)
        self.num += (got - ref).abs().sum().item()
        self.den += ref.abs().sum().item()

    def check(self, what, bar=MEAN_REL):
        mr = self.num / max(self.den, 1e-12)
        assert mr <= bar, f"{what}: mean-rel over the whole run {mr:.3e} (<= {bar})"
        return mr


def _sel_check(got, ref, margin, what):
    """Selections must agree wherever the oracle's margin exceeds MARGIN; returns the fraction excused."""
    got, ref, margin = got.cpu(), ref.cpu(), margin.cpu()
    k = min(got.shape[-1], ref.shape[-1])
    g2 = torch.full_like(got, -1); g2[..., :k] = got[..., :k]
    r2 = torch.full_like(got, -1); r2[..., :ref.shape[-1]] = ref
    diff = (g2 != r2).any(-1)
    hard = diff & (margin > MARGIN)
    assert not hard.any(), (f"{what}: {int(hard.sum())} of {diff.numel()} selections differ outside the margin; first at "
                            f"{hard.nonzero()[0].tolist()} got {g2[hard][0].tolist()} want {r2[hard][0].tolist()}")
    return diff.float().mean().item()


# ---------------------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("kind", KINDS)
def test_cell_ingest_matches_reference_codes(dev, kind):
    from freesolo_b200 import ops
    g, Q, K, V = _g(kind)
    N = int(g["N"])
    nc = N // 32
    Kd, Vd = K[:, :, :N].to(dev), V[:, :, :N].to(dev)
    B, H, _, D = Kd.shape
    kbar = torch.empty(B, H, nc, D, device=dev)
    ceil = torch.empty(B, H, nc, device=dev)
    kq = torch.empty(B, H, nc * 32, D, dtype=torch.int8, device=dev); vq = torch.empty_like(kq)
    ks = torch.empty(B, H, nc, dtype=torch.bfloat16, device=dev); vs = torch.empty_like(ks)
    ops.cell_ingest(Kd, Vd, ncell=nc, kbar=kbar, ceil=ceil, kq=kq, ks=ks, vq=vq, vs=vs)
    assert np.array_equal(kq.cpu().numpy(), g["qk"]), "int8 K codes differ from the reference"
    assert np.array_equal(vq.cpu().numpy(), g["qv"]), "int8 V codes differ from the reference"
    assert np.array_equal(ks.cpu().view(torch.int16).numpy(), g["sk"]) and np.array_equal(vs.cpu().view(torch.int16).numpy(), g["sv"])
    # statistics: the oracle on the same bf16 tensor (mean taken in bf16); ceilings also against the fp32 reference
    kb_o, ce_o = fsl.cell_stats(K[:, :, :N], 32)
    kb = kbar.cpu()
    mism = (kb != kb_o)
    assert not mism.any(), f"chunk-mean keys: {int(mism.sum())} values differ from torch bf16 mean"
    assert ((kb - kb_o).abs() <= kb_o.abs() * 2 ** -7 + 1e-30).all(), "chunk-mean key off by more than one bf16 ulp"
    ce = ceil.cpu()
    assert ((ce - ce_o).abs() <= ce_o * 4e-7).all(), "ceilings differ from the oracle by more than 3 ulp"
    assert ((ce - torch.from_numpy(g["ceil"])).abs() <= ce_o * 4e-7).all(), "ceilings differ from the reference"
    deq = ops.dequant_cells(kq, ks)
    assert np.array_equal(deq.cpu().view(torch.int16).numpy(), g["deq_k"]), "dequantised keys differ from the reference"
    # the separate entry points give the same bits
    q2, s2 = ops.quantize_cells(Kd)
    assert torch.equal(q2, kq) and torch.equal(s2, ks)
    kb2, ce2 = ops.cell_stats(Kd, nc)
    assert torch.equal(kb2, kbar) and torch.equal(ce2, ceil)


def test_cell_ingest_strided_token_major_and_zero_cell(dev):
    """K as a (B,H,N,D) view of a token-major (B,N,3*H*D) projection; an all-zero cell keeps scale 1 and codes 0."""
    from freesolo_b200 import ops
    B, H, D, N = 2, 3, 64, 160
    g = torch.Generator().manual_seed(1)
    qkv = torch.randn(B, N, 3 * H * D, generator=g).to(torch.bfloat16)
    qkv[:, 32:64] = 0
    K = qkv[..., H * D:2 * H * D].view(B, N, H, D).transpose(1, 2)
    Kd = qkv.to(dev)[..., H * D:2 * H * D].view(B, N, H, D).transpose(1, 2)
    q, sc = ops.quantize_cells(Kd)
    qo, so = fsl.quantize_cells(K, 32)
    assert torch.equal(q.cpu(), qo) and torch.equal(sc.cpu(), so)
    assert (sc.cpu()[:, :, 1].float() == 1.0).all() and (q.cpu()[:, :, 32:64] == 0).all()
    kb, ce = ops.cell_stats(Kd, N // 32)
    kbo, ceo = fsl.cell_stats(K, 32)
    assert ((kb.cpu() - kbo).abs() <= kbo.abs() * 2 ** -7).all() and ((ce.cpu() - ceo).abs() <= ceo * 4e-7).all()


@pytest.mark.parametrize("D", [96, 128])
def test_cell_ingest_other_head_dims(dev, D):
    from freesolo_b200 import ops
    B, H, N = 1, 2, 128
    K = torch.randn(B, H, N, D, generator=torch.Generator().manual_seed(D)).to(torch.bfloat16)
    q, sc = ops.quantize_cells(K.to(dev))
    qo, so = fsl.quantize_cells(K, 32)
    assert torch.equal(q.cpu(), qo) and torch.equal(sc.cpu(), so)
    kb, ce = ops.cell_stats(K.to(dev), N // 32)
    kbo, ceo = fsl.cell_stats(K, 32)
    assert ((kb.cpu() - kbo).abs() <= kbo.abs() * 2 ** -7).all() and ((ce.cpu() - ceo).abs() <= ceo * 4e-7).all()


@pytest.mark.parametrize("kind", KINDS)
def test_prefix_topp_is_the_stable_topk(dev, kind):
    from freesolo_b200 import ops
    g, Q, K, V = _g(kind)
    N = int(g["N"])
    ceil = torch.from_numpy(g["ceil"])
    nb = (N + 127) // 128 + 1
    for P in (64, 5):
        got = ops.fsl_prefix_topp(ceil.to(dev), N // 32, 128, nb, P).cpu()
        w = fsl.fsl_prefix_topp(ceil, 32, 128, nb, P)                       # (B,H,nb,min(P,M))
        want = torch.full((w.shape[0] * w.shape[1], nb, P), -1, dtype=torch.int32)
        want[:, :, :w.shape[-1]] = w.reshape(-1, nb, w.shape[-1]).to(torch.int32)
        assert torch.equal(got, want), f"top-{P} lists differ"


@pytest.mark.parametrize("impl", [0, 1])
@pytest.mark.parametrize("kind", KINDS)
def test_prefill_selection_bit_exact_outside_margin(dev, kind, impl):
    """impl 0: dot products on tensor-core tiles; impl 1: the CUDA-core kernel. Same bar for both."""
    from freesolo_b200 import ops
    g, Q, K, V = _g(kind)
    N = int(g["N"])
    p, pd = _params(g), _params(g, dev)
    Kd = K[:, :, :N].to(dev)
    kbar, ceil = ops.cell_stats(Kd, N // 32)
    nb = (N + 127) // 128
    topp = ops.fsl_prefix_topp(ceil, N // 32, 128, nb, 64 if N // 32 >= 64 else (N + 31) // 32)
    P = topp.shape[-1]
    sel, mg = ops.fsl_select(Q[:, :, :N].to(dev), kbar, ceil, topp, pd["lam"], pd["sigma"], N=N, ncell=N // 32, Bq=128, nb=nb,
                             P=P, Wc=8, kk=4, scale=0.125, want_margin=True, impl=impl)
    # the oracle on the statistics the GPU produced: the comparison isolates the selection arithmetic
    want, margin = fsl.fsl_select_prefill(Q[:, :, :N].float(), kbar.cpu(), ceil.cpu(), p["lam"], p["sigma"], 0.125, 32, 128, 64, 8, 4, N)
    frac = _sel_check(sel[:, :, :N], want[:, :, :N], margin[:, :, :N], f"{kind} prefill selection")
    assert frac < 0.02
    # the kernel's own margins agree with the oracle's where both are finite
    m1, m2 = mg[:, :, :N].cpu(), margin[:, :, :N]
    fin = torch.isfinite(m1) & torch.isfinite(m2)
    assert (torch.isfinite(m1) == torch.isfinite(m2)).float().mean() > 0.99
    assert ((m1 - m2).abs()[fin] < 1e-3).all()


@pytest.mark.parametrize("kind", ["randn", "lowprec"])
@pytest.mark.parametrize("impl", [0, 1])
def test_window_prefill(dev, kind, impl):
    from freesolo_b200 import ops
    g, Q, K, V = _g(kind)
    N = int(g["N"])
    cos, sin = fsl.rope_tables(64, 4096, torch.bfloat16, orig_len=4096)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    out = ops.window_prefill(Q[:, :, :N].to(dev), K[:, :, :N].to(dev), V[:, :, :N].to(dev), cos.to(dev), sin.to(dev), 512,
                             0.125, impl=impl, status=status)
    assert int(status.item()) == 0, "a bounded wait inside the tensor-core kernel ran out"
    B, H = Q.shape[:2]
    got = out.view(B, N, H, 64).transpose(1, 2)
    want = fsl.window_attention(Q[:, :, :N].float(), K[:, :, :N].float(), V[:, :, :N].float(), cos, sin, 512, 0.125,
                                act_dtype=torch.bfloat16)
    # the tensor-core kernel multiplies V with probabilities split into bf16 high + low parts (about 16 bits), so it
    # meets the same bar against the exact oracle as the CUDA-core kernel
    _close(got, want.to(torch.bfloat16), f"{kind} window (impl {impl}) vs oracle")
    _close(got, torch.from_numpy(g["window_prefill"]), f"{kind} window (impl {impl}) vs reference fp32", mean_rel=REF_FP32_REL)


@pytest.mark.parametrize("N,W,pos0", [(1, 512, 0), (31, 512, 0), (513, 512, 0), (700, 64, 5), (300, 0, 0), (1100, 512, 37)])
def test_window_prefill_shapes(dev, N, W, pos0):
    from freesolo_b200 import ops
    B, H, D = 2, 2, 64
    g = torch.Generator().manual_seed(N)
    Q, K, V = (torch.randn(B, H, N, D, generator=g).to(torch.bfloat16) for _ in range(3))
    cos, sin = fsl.rope_tables(D, 2048, torch.bfloat16)
    for impl in (0, 1):
        want = fsl.window_attention(Q.float(), K.float(), V.float(), cos, sin, W, 0.125, q_pos0=pos0, k_pos0=pos0,
                                    act_dtype=torch.bfloat16)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        out = ops.window_prefill(Q.to(dev), K.to(dev), V.to(dev), cos.to(dev), sin.to(dev), W, 0.125, pos0=pos0, impl=impl,
                                 status=status)
        assert int(status.item()) == 0, "a bounded wait inside the tensor-core kernel ran out"
        _close(out.view(B, N, H, D).transpose(1, 2), want.to(torch.bfloat16), f"window N={N} W={W} pos0={pos0} impl={impl}")


def test_window_prefill_in_chunks_is_bit_identical(dev, monkeypatch):
    """A long single sequence goes through the tensor-core window kernel in query chunks (last chunk first, each starting a
    window early, the wrong halo rows overwritten by the chunk before): the result equals the one-call result bit for bit."""
    from freesolo_b200 import ops
    H, D, N, W = 2, 64, 5000, 512
    g = torch.Generator().manual_seed(5)
    Q, K, V = (torch.randn(1, H, N, D, generator=g).to(torch.bfloat16).to(dev) for _ in range(3))
    cos, sin = (t.to(dev) for t in fsl.rope_tables(D, 8192, torch.bfloat16))
    whole = ops.window_prefill(Q, K, V, cos, sin, W, 0.125, pos0=3)
    monkeypatch.setattr(ops, "WINDOW_CHUNK", 1024)
    parts = ops.window_prefill(Q, K, V, cos, sin, W, 0.125, pos0=3)
    assert torch.equal(whole, parts)
    monkeypatch.setattr(ops, "WINDOW_CHUNK", 640)          # chunks that are not whole multiples of the window
    assert torch.equal(whole, ops.window_prefill(Q, K, V, cos, sin, W, 0.125, pos0=3))


@pytest.mark.parametrize("kind", KINDS)
def test_readout_combine(dev, kind):
    from freesolo_b200 import ops
    g, Q, K, V = _g(kind)
    N = int(g["N"])
    p, pd = _params(g), _params(g, dev)
    sel = torch.from_numpy(g["sel_prefill"])
    B, H = Q.shape[:2]
    sr = torch.randn(B, N, H * 64, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    y = ops.readout_combine(Q[:, :, :N].to(dev), K[:, :, :N].to(dev), V[:, :, :N].to(dev), sel.to(dev).contiguous(), sr.to(dev),
                            pd["norm_w"], pd["lrs"], float(g["eps"]), scale=0.125, Bq=128, n_kv=N)
    o = fsl.cell_readout(Q[:, :, :N].float(), K[:, :, :N].float(), V[:, :, :N].float(), sel, 32, 128, 0.125, 0, N)
    want = fsl.lr_norm_combine(sr.view(B, N, H, 64).transpose(1, 2), o, p["norm_w"], p["lrs"], float(g["eps"]))
    _close(y, want, f"{kind} readout+combine")
    # sr = None means a zero window output; in place gives the same bits
    y0 = ops.readout_combine(Q[:, :, :N].to(dev), K[:, :, :N].to(dev), V[:, :, :N].to(dev), sel.to(dev).contiguous(), None,
                             pd["norm_w"], pd["lrs"], float(g["eps"]), scale=0.125, Bq=128, n_kv=N)
    want0 = fsl.lr_norm_combine(torch.zeros(B, H, N, 64), o, p["norm_w"], p["lrs"], float(g["eps"]))
    _close(y0, want0, f"{kind} readout alone")
    srd = sr.to(dev).clone()
    y2 = ops.readout_combine(Q[:, :, :N].to(dev), K[:, :, :N].to(dev), V[:, :, :N].to(dev), sel.to(dev).contiguous(), srd,
                             pd["norm_w"], pd["lrs"], float(g["eps"]), scale=0.125, Bq=128, n_kv=N, out=srd)
    assert torch.equal(y2, y)


def _run_layer(dev, g, Q, K, V, mode, splits, T=None, window_path=0):
    """Prefill + T decode steps of one layer through ops; returns (y_prefill, sel_prefill, [y_t], [sel_t], state)."""
    from freesolo_b200 import ops
    N = int(g["N"]); T = int(g["T"]) if T is None else T
    pd = _params(g, dev)
    B, H, _, D = Q.shape
    cos, sin = (t.to(dev) for t in fsl.rope_tables(D, 4096, torch.bfloat16, orig_len=4096))
    Qd, Kd, Vd = Q.to(dev), K.to(dev), V.to(dev)
    sr = ops.window_prefill(Qd[:, :, :N], Kd[:, :, :N], Vd[:, :, :N], cos, sin, 512, 0.125)
    kbar, ceil = ops.cell_stats(Kd[:, :, :N], N // 32)
    st = ops.FslDecodeState(B, H, D, N + T, dev, mode=mode)
    st.prefill(Kd[:, :, :N], Vd[:, :, :N], N, kbar, ceil)
    nb = (N + 127) // 128
    P = min(64, (N + 31) // 32)
    topp = ops.fsl_prefix_topp(ceil, N // 32, 128, nb, P)
    sel = ops.fsl_select(Qd[:, :, :N], kbar, ceil, topp, pd["lam"], pd["sigma"], N=N, ncell=N // 32, Bq=128, nb=nb, P=P, Wc=8,
                         kk=4, scale=0.125)
    y = ops.readout_combine(Qd[:, :, :N], Kd[:, :, :N], Vd[:, :, :N], sel, sr, pd["norm_w"], pd["lrs"], float(g["eps"]),
                            scale=0.125, Bq=128, n_kv=N)
    pos_t = torch.zeros((), dtype=torch.int64, device=dev)
    ys, sels = [], []
    for t in range(T):
        pos_t.fill_(N + t)
        so = torch.empty(B, H, 4, dtype=torch.int32, device=dev)
        yd = ops.fsl_decode_step(st, Qd[:, :, N + t], Kd[:, :, N + t], Vd[:, :, N + t], pos_t, cos, sin, pd["lam"], pd["sigma"],
                                 pd["lrs"], pd["norm_w"], scale=D ** -0.5, eps=float(g["eps"]), sel_out=so, splits=splits,
                                 window_path=window_path)
        ys.append(yd.clone()); sels.append(so)
    return y, sel[:, :, :N], ys, sels, st


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("mode", ["bf16", "int8", "bounded"])
def test_layer_prefill_then_decode(dev, kind, mode):
    g, Q, K, V = _g(kind)
    N, T = int(g["N"]), int(g["T"])
    y, sel, ys, sels, st = _run_layer(dev, g, Q, K, V, mode, splits=4)
    orc = _oracle(g, int8=(mode != "bf16"))
    y0, sel0, mg0 = orc.prefill(Q[:, :, :N], K[:, :, :N], V[:, :, :N])
    _sel_check(sel, sel0, mg0, f"{kind}/{mode} prefill selection")
    _close(y, y0, f"{kind}/{mode} prefill output vs oracle")
    # against the reference's fp32 run: it took its chunk means in fp32, so a few of its selections differ from the bf16
    # semantics; the output bound applies to the rows where every head reads the reference's cells
    agree = (sel.cpu() == torch.from_numpy(g["sel_prefill"])).all(-1).all(1)           # (B, N)
    assert agree.float().mean() > 0.9
    _close(y[agree], torch.from_numpy(g["y_prefill"])[agree], f"{kind}/{mode} prefill output vs reference fp32", mean_rel=REF_FP32_REL)
    run = _RunError()
    for t in range(T):
        sl = slice(N + t, N + t + 1)
        yo, so, mo = orc.decode(Q[:, :, sl], K[:, :, sl], V[:, :, sl])
        excused = _sel_check(sels[t].unsqueeze(2), so, mo, f"{kind}/{mode} decode step {t} (pos {N + t}) selection")
        if excused == 0:
            _close(ys[t].view(-1), yo.reshape(-1), f"{kind}/{mode} decode step {t} (pos {N + t}) output")
            run.add(ys[t], yo)
    run.check(f"{kind}/{mode} decode outputs")
    assert st.faults() == (0, 0, 0), f"device status words {st.faults()}"
    # against the reference's fp32 decode outputs (bf16 path: no quantisation error on top)
    if mode == "bf16":
        ref = torch.from_numpy(g["y_decode"])
        got = torch.stack([y_.view(Q.shape[0], -1) for y_ in ys], dim=1)
        _close(got, ref, f"{kind} decode outputs vs reference fp32", mean_rel=REF_FP32_REL)


@pytest.mark.parametrize("mode", ["int8", "bounded"])
@pytest.mark.parametrize("N", [1000, 40, 300])
def test_decode_staged_window_is_bit_identical(dev, mode, N):
    """The window rows staged through shared memory by bulk copies (the many-sequences path) against per-lane loads: same
    per-row arithmetic, same row-to-warp assignment, same merge order, so the outputs and selections are identical bit for
    bit - over a run that closes cells, refreshes the block's pool, frees slots, and (N = 40, 300) starts with a window that
    is still growing."""
    g, Q, K, V = _g("randn")
    T = 300
    rep = 2
    Q2, K2, V2 = (torch.cat([t] * rep, dim=2) for t in (Q, K, V))
    g2 = dict(g); g2["N"] = np.int64(N); g2["T"] = np.int64(T)
    _, _, ys_a, sels_a, st_a = _run_layer(dev, g2, Q2, K2, V2, mode, 1, T=T, window_path=1)
    _, _, ys_b, sels_b, st_b = _run_layer(dev, g2, Q2, K2, V2, mode, 1, T=T, window_path=2)
    for t in range(T):
        assert torch.equal(sels_a[t], sels_b[t]), f"step {t}: selections differ"
        assert torch.equal(ys_a[t], ys_b[t]), f"step {t}: outputs differ between the staged and the direct window"
    assert st_a.faults() == (0, 0, 0) and st_b.faults() == (0, 0, 0)


@pytest.mark.parametrize("D", [96, 128])
def test_decode_staged_window_other_head_dims(dev, D):
    from freesolo_b200 import ops
    B, H, N, T = 3, 2, 700, 70
    gen = torch.Generator().manual_seed(D + 1)
    Q, K, V = (torch.randn(B, H, N + T, D, generator=gen).to(torch.bfloat16).to(dev) for _ in range(3))
    lam, sig, lrs, nw = (torch.ones(H, device=dev) * 1.5, torch.ones(H, device=dev) * 6, torch.ones(H, device=dev) * 0.3,
                         torch.ones(D, device=dev))
    cos, sin = (t.to(dev) for t in fsl.rope_tables(D, 1024, torch.bfloat16))
    outs = []
    for path in (1, 2):
        st = ops.FslDecodeState(B, H, D, N + T, dev, mode="int8")
        st.prefill(K[:, :, :N], V[:, :, :N], N)
        pos_t = torch.zeros((), dtype=torch.int64, device=dev)
        ys = []
        for t in range(T):
            pos_t.fill_(N + t)
            ys.append(ops.fsl_decode_step(st, Q[:, :, N + t], K[:, :, N + t], V[:, :, N + t], pos_t, cos, sin, lam, sig, lrs, nw,
                                          scale=D ** -0.5, eps=1e-8, splits=1, window_path=path).clone())
        outs.append(torch.stack(ys))
        assert st.faults() == (0, 0, 0)
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("splits", [1, 2, 8])
def test_decode_splits_agree(dev, splits):
    g, Q, K, V = _g("randn")
    _, _, ys_a, sels_a, _ = _run_layer(dev, g, Q, K, V, "int8", 4, T=40)
    _, _, ys_b, sels_b, _ = _run_layer(dev, g, Q, K, V, "int8", splits, T=40)
    for t in range(40):
        assert torch.equal(sels_a[t], sels_b[t]), f"step {t}: selections depend on the split count"
        _close(ys_b[t], ys_a[t], f"step {t}: outputs with {splits} vs 4 splits")


def test_bounded_store_reads_equal_full_int8_store(dev):
    """The reference's invariant (tests/test_kv_bounded.py): same cells, same values, so identical outputs; and the
    store holds exactly the readable set without faults."""
    g, Q, K, V = _g("randn")
    # a longer run that crosses several block refreshes: tile the fixture's tokens
    rep = 3
    Q2, K2, V2 = (torch.cat([t] * rep, dim=2) for t in (Q, K, V))
    g2 = dict(g); g2["N"] = np.int64(1000); g2["T"] = np.int64(Q2.shape[2] - 1000)
    T = 600
    _, sel_a, ys_a, sels_a, st_a = _run_layer(dev, g2, Q2, K2, V2, "int8", 4, T=T)
    _, sel_b, ys_b, sels_b, st_b = _run_layer(dev, g2, Q2, K2, V2, "bounded", 4, T=T)
    assert torch.equal(sel_a, sel_b)
    for t in range(T):
        assert torch.equal(sels_a[t], sels_b[t]), f"step {t}: selections differ between the stores"
        assert torch.equal(ys_a[t], ys_b[t]), f"step {t}: outputs differ between the stores"
    assert st_b.faults() == (0, 0, 0)
    # held set == readable set of the current block (kv_bounded.py:4-19)
    pos = 1000 + T
    blk = (pos // 128) * 128
    m_vis = blk // 32
    ceil = st_b.ceil.cpu()[:, :, :pos // 32]
    top = fsl.stable_topk(ceil[:, :, :m_vis], 64)
    lo = fsl.bounded_readable_from(blk, m_vis, 32, 512, 8)
    want = torch.zeros_like(ceil, dtype=torch.bool)
    want[:, :, lo:] = True
    want.scatter_(2, top, True)
    held = st_b.slot_of.cpu()[:, :, :pos // 32] >= 0
    assert torch.equal(held, want), "bounded store does not hold exactly the readable cells"
    ti = st_b.top_idx.cpu().long()
    assert torch.equal(ti[:, :, :top.shape[-1]], top) and (ti[:, :, top.shape[-1]:] == -1).all(), \
        "top-P list differs from the stable top-k of the ceilings"
    cin = st_b.cell_in.cpu()
    so = st_b.slot_of.cpu()
    for b in range(cin.shape[0]):
        for h in range(cin.shape[1]):
            occ = cin[b, h][cin[b, h] >= 0]
            assert len(set(occ.tolist())) == len(occ) and (so[b, h][occ.long()] >= 0).all()


@pytest.mark.parametrize("N", [1, 20, 32, 127, 128, 160, 511])
def test_short_prompts_then_decode(dev, N):
    """Prompts of any length (shorter than a cell, a block, the window) followed by decode steps across the first cell,
    block and window boundaries, as tests/test_cached_decode_short_prompt.py does for the reference."""
    g, Q, K, V = _g("randn")
    T = 150
    g2 = dict(g); g2["N"] = np.int64(N); g2["T"] = np.int64(T)
    for mode in ("bf16", "int8"):
        y, sel, ys, sels, st = _run_layer(dev, g2, Q[:, :, :N + T], K[:, :, :N + T], V[:, :, :N + T], mode, 2, T=T)
        orc = _oracle(g, int8=(mode != "bf16"))
        y0, sel0, mg0 = orc.prefill(Q[:, :, :N], K[:, :, :N], V[:, :, :N])
        _sel_check(sel, sel0, mg0, f"N={N} prefill selection")
        _close(y, y0, f"N={N}/{mode} prefill output")
        run = _RunError()
        for t in range(T):
            sl = slice(N + t, N + t + 1)
            yo, so, mo = orc.decode(Q[:, :, sl], K[:, :, sl], V[:, :, sl])
            excused = _sel_check(sels[t].unsqueeze(2), so, mo, f"N={N}/{mode} decode step {t} selection")
            _close(ys[t].view(-1), yo.reshape(-1), f"N={N}/{mode} decode step {t} output")
            if excused == 0:
                run.add(ys[t], yo)
        run.check(f"N={N}/{mode} decode outputs")
        assert st.faults() == (0, 0, 0)


@pytest.mark.parametrize("D", [96, 128])
def test_other_head_dims_layer(dev, D):
    B, H, N, T = 2, 2, 300, 40
    gen = torch.Generator().manual_seed(D)
    Q, K, V = (torch.randn(B, H, N + T, D, generator=gen).to(torch.bfloat16) for _ in range(3))
    g = dict(N=np.int64(N), T=np.int64(T), H=H, D=D, eps=np.float32(1e-8), lam=np.ones(H, np.float32) * 1.5,
             sigma=np.ones(H, np.float32) * 6, lrs=np.ones(H, np.float32) * 0.3, norm_w=np.ones(D, np.float32))
    from freesolo_b200 import ops
    pd = _params(g, dev)
    sc = 1.0 / D ** 0.5
    cos, sin = (t.to(dev) for t in fsl.rope_tables(D, 1024, torch.bfloat16))
    Qd, Kd, Vd = Q.to(dev), K.to(dev), V.to(dev)
    orc = fsl.FSLLayerOracle(H, D, eps=1e-8, rope_len=1024, int8=True, **_params(g))
    sr = ops.window_prefill(Qd[:, :, :N], Kd[:, :, :N], Vd[:, :, :N], cos, sin, 512, sc)
    kbar, ceil = ops.cell_stats(Kd[:, :, :N], N // 32)
    st = ops.FslDecodeState(B, H, D, N + T, dev, mode="int8")
    st.prefill(Kd[:, :, :N], Vd[:, :, :N], N, kbar, ceil)
    nb, P = (N + 127) // 128, min(64, (N + 31) // 32)
    topp = ops.fsl_prefix_topp(ceil, N // 32, 128, nb, P)
    sel = ops.fsl_select(Qd[:, :, :N], kbar, ceil, topp, pd["lam"], pd["sigma"], N=N, ncell=N // 32, Bq=128, nb=nb, P=P, Wc=8,
                         kk=4, scale=sc)
    y = ops.readout_combine(Qd[:, :, :N], Kd[:, :, :N], Vd[:, :, :N], sel, sr, pd["norm_w"], pd["lrs"], 1e-8, scale=sc, Bq=128,
                            n_kv=N)
    y0, sel0, mg0 = orc.prefill(Q[:, :, :N], K[:, :, :N], V[:, :, :N])
    _sel_check(sel[:, :, :N], sel0, mg0, f"D={D} prefill selection")
    _close(y, y0, f"D={D} prefill output")
    pos_t = torch.zeros((), dtype=torch.int64, device=dev)
    run = _RunError()
    for t in range(T):
        pos_t.fill_(N + t)
        so = torch.empty(B, H, 4, dtype=torch.int32, device=dev)
        yd = ops.fsl_decode_step(st, Qd[:, :, N + t], Kd[:, :, N + t], Vd[:, :, N + t], pos_t, cos, sin, pd["lam"], pd["sigma"],
                                 pd["lrs"], pd["norm_w"], scale=sc, eps=1e-8, sel_out=so, splits=2)
        sl = slice(N + t, N + t + 1)
        yo, s_o, mo = orc.decode(Q[:, :, sl], K[:, :, sl], V[:, :, sl])
        excused = _sel_check(so.unsqueeze(2), s_o, mo, f"D={D} decode step {t} selection")
        _close(yd.view(-1), yo.reshape(-1), f"D={D} decode step {t} output")
        if excused == 0:
            run.add(yd, yo)
    run.check(f"D={D} decode outputs")


@pytest.mark.parametrize("kind", KINDS)
def test_readout_combine_tensor_core_tiles(dev, kind):
    """The mma.sync readout (whole 128-query blocks, head_dim 64) against the oracle and against the CUDA-core kernel."""
    from freesolo_b200 import ops
    g, Q, K, V = _g(kind)
    N = int(g["N"])
    p, pd = _params(g), _params(g, dev)
    sel = torch.from_numpy(g["sel_prefill"])
    B, H = Q.shape[:2]
    sr = torch.randn(B, N, H * 64, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    args = (Q[:, :, :N].to(dev), K[:, :, :N].to(dev), V[:, :, :N].to(dev), sel.to(dev).contiguous(), sr.to(dev),
            pd["norm_w"], pd["lrs"], float(g["eps"]))
    y2 = ops.readout_combine(*args, scale=0.125, Bq=128, n_kv=N, impl=2)
    y1 = ops.readout_combine(*args, scale=0.125, Bq=128, n_kv=N, impl=1)
    o = fsl.cell_readout(Q[:, :, :N].float(), K[:, :, :N].float(), V[:, :, :N].float(), sel, 32, 128, 0.125, 0, N)
    want = fsl.lr_norm_combine(sr.view(B, N, H, 64).transpose(1, 2), o, p["norm_w"], p["lrs"], float(g["eps"]))
    _close(y2, want, f"{kind} tensor-core readout+combine vs oracle")
    _close(y2, y1, f"{kind} tensor-core vs CUDA-core readout", mean_rel=5e-4)
    # without a window output, and in place
    y0 = ops.readout_combine(*args[:4], None, *args[5:], scale=0.125, Bq=128, n_kv=N, impl=2)
    want0 = fsl.lr_norm_combine(torch.zeros(B, H, N, 64), o, p["norm_w"], p["lrs"], float(g["eps"]))
    _close(y0, want0, f"{kind} tensor-core readout alone")
    srd = sr.to(dev).clone()
    y3 = ops.readout_combine(*args[:4], srd, *args[5:], scale=0.125, Bq=128, n_kv=N, out=srd, impl=2)
    assert torch.equal(y3, y2)
