"""The streaming FS-L cache (freesolo_b200/fsattn/linear_cache.py, ref: src/fsattn/linear_cache.py) on the GPU: against the
reference's own LinearFSCache run (tests/golden/linear_*.npz), against the FS-L oracle, and against this package's standard
prefill."""
import numpy as np
import pytest
import torch

from conftest import bf16_from_bits, load_golden
from oracle import fsl

pytestmark = pytest.mark.gpu


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def _layer(g, dev, **over):
    from freesolo_b200 import FSAttn
    from freesolo_b200.serving import serve_kwargs
    H, D = int(g["H"]), int(g["D"])
    kw = serve_kwargs("sparse")
    kw.update(over)
    a = FSAttn(d_model=H * D, n_heads=H, causal=True, bias=False, max_seq_len=4096, **kw).to(torch.bfloat16).to(dev).eval()
    # the per-head parameters keep the fixture's fp32 values (a cast of the module to bf16 would round them)
    a.sel_scale.data = torch.from_numpy(g["lam"]).to(dev)
    a.log_sigma.data = torch.from_numpy(g["sigma"]).log().to(dev)
    a.long_range_scale.data = torch.from_numpy(g["lrs"]).view(H, 1, 1).to(dev)
    a.lr_norm.scale.data = torch.from_numpy(g["norm_w"]).to(dev)
    return a


def _oracle(g):
    H, D = int(g["H"]), int(g["D"])
    return fsl.FSLLayerOracle(H, D, W=int(g["W"]), P=int(g["P"]), Wc=int(g["Wc"]), lam=torch.from_numpy(g["lam"]),
                              sigma=torch.from_numpy(g["sigma"]), lrs=torch.from_numpy(g["lrs"]), norm_w=torch.from_numpy(g["norm_w"]),
                              eps=float(g["eps"]), act_dtype=torch.bfloat16, rope_len=4096, rope_orig_len=4096)


def _run(cache, Q, K, V, pieces):
    """attend over consecutive pieces; records the cell ids every query selected."""
    picked, inner = [], cache.select

    def select(q):
        slots, ids = inner(q)
        pad = cache.attn.cell_topk - ids.shape[-1]
        picked.append(torch.nn.functional.pad(ids, (0, pad), value=-1) if pad else ids.clone())
        return slots, ids
    cache.select = select
    ys, o = [], 0
    with torch.no_grad():
        for n in pieces:
            ys.append(cache.attend(Q[:, :, o:o + n], K[:, :, o:o + n], V[:, :, o:o + n]))
            o += n
    sel = torch.cat(picked, dim=2)
    sel = torch.nn.functional.pad(sel, (0, 0, o - sel.shape[2], 0), value=-1)
    y = torch.cat(ys, dim=2)
    B, H, N, D = y.shape
    return y.transpose(1, 2).reshape(B, N, H * D), sel


def _rel(a, b):
    return float((a.float() - b.float()).abs().mean() / b.float().abs().mean())


@pytest.mark.parametrize("kind", ["randn", "vocab"])
def test_streaming_cache_against_the_reference_run_and_the_oracle(kind):
    from freesolo_b200.fsattn.linear_cache import LinearFSCache
    dev = _dev()
    g = load_golden(f"linear_{kind}")
    Q, K, V = (bf16_from_bits(g[k]) for k in ("Q", "K", "V"))
    H, D, N = int(g["H"]), int(g["D"]), int(g["N"])
    a = _layer(g, dev)
    c = LinearFSCache(a)
    y, sel = _run(c, Q.to(dev), K.to(dev), V.to(dev), [int(n) for n in g["pieces"]])
    torch.cuda.synchronize()
    y, sel = y.cpu(), sel.cpu()
    # the oracle on the bf16 tensors themselves: the chunk mean is then taken in bf16, as the reference takes it in bf16 inference
    want_y, want_sel, margin = _oracle(g).prefill(Q, K, V)
    # selections: the oracle's wherever its fp32 margin exceeds 1e-4
    differ = (sel.sort(-1).values != want_sel.sort(-1).values).any(-1)
    assert int((differ & (margin > 1e-4)).sum()) == 0, "selections differ from the oracle outside the margin"
    assert differ.float().mean() < 0.01
    # the reference's own fp32 run (fp32 chunk means): the same selection for all but the near-ties the bf16 mean moves
    ref_sel = torch.from_numpy(g["sel"]).long()
    assert (sel.sort(-1).values == ref_sel.sort(-1).values).all(-1).float().mean() > 0.99
    # outputs: 1e-3 mean relative against the oracle (bf16 roundings restated) on the queries with the same selection;
    # against the reference's fp32 run the bf16 activations themselves cost a few 1e-3
    same = ~differ[0].any(0)
    assert _rel(y[0][same], want_y[0][same]) < 1e-3
    ref_y = torch.from_numpy(g["y"]).transpose(1, 2).reshape(1, N, H * D)
    assert _rel(y[0][same], ref_y[0][same]) < 6e-3
    assert float((y.float() - want_y.float()).abs().max()) < 5e-2
    # state: the reference's counters, the same cells left in the top list, a fixed number of bytes
    assert [c.pos, c.eligible, c.max_merge_cells, c.merged_cells, c.updates] == g["counters"].tolist()
    top = c.ids[:, :, :c.P].sort(-1).values.cpu().numpy().astype(np.int32)
    assert np.array_equal(top, g["top_ids"])
    nbytes = c.state_bytes()
    with torch.no_grad():
        c.attend(Q[:, :, :200].to(dev), K[:, :, :200].to(dev), V[:, :, :200].to(dev))
    assert c.state_bytes() <= nbytes + 2 * 2 * H * 160 * D * 2          # only the open cells' rows vary


def test_streaming_cache_does_not_depend_on_the_piece_sizes():
    from freesolo_b200.fsattn.linear_cache import LinearFSCache
    dev = _dev()
    g = load_golden("linear_randn")
    Q, K, V = (bf16_from_bits(g[k]).to(dev) for k in ("Q", "K", "V"))
    N = 1500
    a = _layer(g, dev)
    y1, s1 = _run(LinearFSCache(a), Q, K, V, [N])
    y2, s2 = _run(LinearFSCache(a), Q, K, V, [1] * 40 + [333, 95, 128, 129, N - 40 - 685])
    assert torch.equal(s1.sort(-1).values, s2.sort(-1).values)
    assert _rel(y2, y1) < 1e-3 and float((y1.float() - y2.float()).abs().max()) < 3e-2
    # a fork continues independently of its parent
    c = LinearFSCache(a)
    with torch.no_grad():
        c.attend(Q[:, :, :700], K[:, :, :700], V[:, :, :700])
    f = c.fork()
    with torch.no_grad():
        ya = c.attend(Q[:, :, 700:900], K[:, :, 700:900], V[:, :, 700:900])
        yb = f.attend(Q[:, :, 700:900], K[:, :, 700:900], V[:, :, 700:900])
    assert torch.equal(ya, yb) and f.pos == c.pos == 900


def test_streaming_cache_equals_the_standard_prefill_of_this_package():
    """The same layer through FSKVCache (one prefill call) and through LinearFSCache (2048-token chunks): same selections
    up to near-ties, outputs within the activation rounding."""
    import os
    from freesolo_b200 import FSKVCache
    from freesolo_b200.fsattn.linear_cache import LinearFSCache
    dev = _dev()
    g = load_golden("linear_randn")
    H, D, N = int(g["H"]), int(g["D"]), 2900
    a = _layer(g, dev)
    x = torch.randn(1, N, H * D, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).to(dev)
    os.environ["FSATTN_KEEP_SEL"] = "1"
    try:
        with torch.no_grad():
            y_std = a(x, cache=FSKVCache(a))
        sel_std = a._last_sel[:, :, :N].long().cpu()
    finally:
        del os.environ["FSATTN_KEEP_SEL"]
    c = LinearFSCache(a)
    picked, inner = [], c.select

    def select(q):
        slots, ids = inner(q)
        pad = a.cell_topk - ids.shape[-1]
        picked.append(torch.nn.functional.pad(ids, (0, pad), value=-1) if pad else ids.clone())
        return slots, ids
    c.select = select
    with torch.no_grad():
        y_lin = torch.cat([a(x[:, o:o + 2048], cache=c) for o in range(0, N, 2048)], dim=1)
    sel_lin = torch.cat(picked, dim=2).cpu()
    sel_lin = torch.nn.functional.pad(sel_lin, (0, 0, N - sel_lin.shape[2], 0), value=-1)
    same = (sel_std.sort(-1).values == sel_lin.sort(-1).values).all(-1)
    assert same.float().mean() > 0.995
    rows = same[0].all(0).to(dev)
    assert _rel(y_lin[0][rows], y_std[0][rows]) < 2e-3


def test_linear_prefill_of_a_model_matches_its_standard_prefill():
    """experiments/scaling/kv_cache.py:529-538: the prompt in 2048-token chunks through streaming caches, then greedy tokens
    one at a time through the same caches; the last-token logits stay within the model-level bar of the standard path."""
    from freesolo_b200.fsattn.kv_cache import linear_prefill, make_caches
    from freesolo_b200.serving import FreeSoloLM, lm_head, serve_kwargs, trunk_cached
    dev = _dev()
    torch.manual_seed(0)
    m = FreeSoloLM(vocab_size=512, d_model=256, n_layers=3, n_heads=4, d_ff=512, max_seq_len=8192,
                   **serve_kwargs("sparse")).to(torch.bfloat16).to(dev).eval()
    ids = torch.randint(0, 512, (1, 4500), generator=torch.Generator().manual_seed(9)).to(dev)
    with torch.no_grad():
        std = make_caches(m, reserve=8)
        h_std = trunk_cached(m, ids, std, last_n=1)
        lin = make_caches(m, linear=True)
        h_lin = linear_prefill(m, ids, lin, chunk_size=2048)
        l_std, l_lin = lm_head(m, h_std[:, -1]).float(), lm_head(m, h_lin[:, -1]).float()
        assert float((l_std - l_lin).abs().max() / l_std.abs().max()) < 0.05
        tok = l_lin.argmax(-1).view(1, 1)
        for _ in range(3):                               # decode continues through the streaming caches, one token per call
            h = trunk_cached(m, tok, lin)
            tok = lm_head(m, h[:, -1]).argmax(-1).view(1, 1)
    assert lin[0].pos == 4503 and lin[0].state_bytes() == lin[1].state_bytes()


def test_the_direct_block_calls_equal_the_per_operation_path():
    """A long attend call of one sequence drives its blocks through argument structs built once per call; a cache whose
    `select` is wrapped takes the per-operation path. Same outputs, same state, bit for bit."""
    from freesolo_b200.fsattn.linear_cache import LinearFSCache
    dev = _dev()
    g = load_golden("linear_vocab")
    Q, K, V = (bf16_from_bits(g[k]).to(dev) for k in ("Q", "K", "V"))
    a = _layer(g, dev)
    pieces = [700, 1, 333, 129, 600]
    slow = LinearFSCache(a)
    y_slow, _ = _run(slow, Q, K, V, pieces)
    fast = LinearFSCache(a)
    ys, o = [], 0
    with torch.no_grad():
        for n in pieces:
            ys.append(fast.attend(Q[:, :, o:o + n], K[:, :, o:o + n], V[:, :, o:o + n]))
            o += n
    y_fast = torch.cat(ys, dim=2)
    B, H, N, D = y_fast.shape
    assert torch.equal(y_fast.transpose(1, 2).reshape(B, N, H * D), y_slow)
    for name in LinearFSCache._TENSORS:
        assert torch.equal(getattr(fast, name), getattr(slow, name)), name
    assert [fast.pos, fast.eligible, fast.max_merge_cells, fast.merged_cells, fast.updates] == \
           [slow.pos, slow.eligible, slow.max_merge_cells, slow.merged_cells, slow.updates]
