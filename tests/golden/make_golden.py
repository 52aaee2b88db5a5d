"""Generate the golden fixtures in this directory by running the REFERENCE implementation (zekun-shi/freesolo) on CPU.

Usage (only where a checkout of the reference exists; the fixtures it writes are committed and travel on their own):

    python tests/golden/make_golden.py --reference /path/to/freesolo [--only fsl_small,...]

The script imports the reference as a library, drives its own FSAttn / FSKVCache / kv_int8 / local_attention code
in fp32 on CPU with seeded inputs, and stores inputs (as bf16 bit patterns, so every consumer sees identical
values) together with the reference's outputs. Nothing here is imported by the product.

Fixtures:
  fsl_<kind>.npz   one FS-L layer driven at the Q/K/V level (projections replaced by fixed tensors, W_o = identity):
                   cell statistics, int8 codes, prefill selections (deterministic tie rule), prefill W_o input,
                   window branch alone, and a run of decode steps that crosses cell and block boundaries.
  fsb_<kind>.npz   one FS-B layer (serve configuration, two forests) driven the same way: the reference's forest
                   tables, spines and beam cells of the prefill stage, prefill and decode selections, outputs.
  model_<variant>.npz  the reference's whole FreeSoloLM at a debug size (4 layers x 256, 4 heads x 64, vocabulary cut to
                   1024), seed-0 init rounded to bf16-representable values, FS-L ("fsl") or FS-B ("fsb", thresholds from
                   the reference's fsb_calibrate_tau): prefill of 330 tokens + 72 greedy tokens through its KV caches in
                   fp32, then the same token sequence fed through the module cast to bf16 (teacher forcing, so every
                   step's logits stay comparable); token ids and the last-token logits of every step of both runs.
  linear_<kind>.npz  the reference's streaming cache (src/fsattn/linear_cache.py LinearFSCache) of one FS-L layer at the
                   Q/K/V level: 3000 tokens pushed through `attend` in pieces of uneven sizes (single tokens included),
                   fp32: the outputs, the cell ids every query selected, the ids left in the top-P list at the end and
                   the cache's counters.
  fsl_config1.npz  BASELINE config 1: FSAttn(d_model=1024, 16 heads) with its own seeded projections, 4096-token
                   prefill + 1 decode step, fp32; selections, margins and a strided sample of the outputs.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _bf16_bits(x: torch.Tensor) -> np.ndarray:
    return x.to(torch.bfloat16).contiguous().view(torch.int16).numpy()


def make_inputs(kind: str, B: int, H: int, N: int, D: int, seed: int):
    """Q, K, V (B,H,N,D) with bf16-representable values, as fp32. Kinds follow the reference's own adversarial
    inputs (tests/test_fsl_fast_select.py:41-61): randn, vocab (tied ceilings), periodic (equal cells), lowprec."""
    g = torch.Generator().manual_seed(seed)
    if kind == "randn":
        x = torch.randn(B, N, 3, H, D, generator=g)
    elif kind == "vocab":
        voc = torch.randn(40, 3, H, D, generator=g)
        x = voc[torch.randint(0, 40, (B, N), generator=g)]
    elif kind == "periodic":
        voc = torch.randn(32, 3, H, D, generator=g)
        x = voc[(torch.arange(N) % 32).expand(B, N)]
    elif kind == "lowprec":
        x = torch.randint(-2, 3, (B, N, 3, H, D), generator=g).float() * 0.25
    else:
        raise ValueError(kind)
    x = x.to(torch.bfloat16).float()
    return tuple(x[:, :, i].transpose(1, 2).contiguous() for i in range(3))


class _Fixed(torch.nn.Module):
    """Stands in for a projection: returns rows [cursor, cursor + n) of a fixed (B, Ntot, H*D) tensor."""

    def __init__(self, full):
        super().__init__()
        self.full = full
        self.cursor = 0
        self.bias = None
        self.weight = torch.nn.Parameter(torch.zeros(1, 1), requires_grad=False)

    def forward(self, x):
        n = x.shape[1]
        out = self.full[:, self.cursor:self.cursor + n]
        self.cursor += n
        return out


def _layer(ref, H, D, seed, fused):
    from src.fsattn import FSAttn
    from bench_efficiency import serve_kwargs
    kw = serve_kwargs("sparse")
    kw.update(fs_fused_attn=1 if fused else 0, cell_prune_stable_ties=1)
    a = FSAttn(d_model=H * D, n_heads=H, causal=True, bias=False, max_seq_len=4096, **kw).eval()
    a.cell_prune_stable_ties = 1
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        a.sel_scale.copy_(0.5 + torch.rand(H, generator=g) * 2)
        a.log_sigma.copy_(torch.log(1.0 + torch.rand(H, generator=g) * 40))
        a.long_range_scale.copy_((0.05 + torch.rand(H, generator=g)).view(H, 1, 1))
        a.lr_norm.scale.copy_(0.5 + torch.rand(D, generator=g))
        a.W_o.weight.copy_(torch.eye(H * D))
    return a


def gen_fsl(kind: str, B=1, H=2, D=64, N=1000, T=72, seed=7):
    """One FS-L layer at the Q/K/V level: prefill of N tokens, then T decode steps."""
    from kv_cache import FSKVCache
    from src.fsattn import kv_int8
    from src.fsattn.attention import _apply_rotary_emb
    from src.utils.local_attention import local_attention
    Q, K, V = make_inputs(kind, B, H, N + T, D, seed)
    flat = [t.transpose(1, 2).reshape(B, N + T, H * D).contiguous() for t in (Q, K, V)]
    out = {"kind": kind, "B": B, "H": H, "D": D, "N": N, "T": T,
           "Q": _bf16_bits(Q), "K": _bf16_bits(K), "V": _bf16_bits(V)}
    x = torch.zeros(B, N + T, H * D)

    def run(fused):
        a = _layer(None, H, D, seed + 1, fused)
        a.W_q, a.W_k, a.W_v = _Fixed(flat[0]), _Fixed(flat[1]), _Fixed(flat[2])
        sels = []
        if fused:
            from src.fsattn import fsb_tree

            def grab(Qx, Kx, Vx, sel, s, Bq, bias=None, q_pos=0):
                sels.append(sel.clone())
                return torch.zeros_like(Qx)
            a._cell_fused_lr = grab
        c = FSKVCache(a)
        ys = []
        with torch.no_grad():
            ys.append(a(x[:, :N], cache=c))
            stats = (c._kbar.clone(), c._ceil.clone())
            for t in range(T):
                ys.append(a(x[:, N + t:N + t + 1], cache=c))
        return a, ys, sels, stats, c

    a, ys, _, stats, c = run(False)
    out["lam"] = a.sel_scale.detach().numpy()
    out["sigma"] = a.sigma.detach().numpy()
    out["lrs"] = a.long_range_scale.detach().reshape(H).numpy()
    out["norm_w"] = a.lr_norm.scale.detach().numpy()
    out["eps"] = np.float32(a.lr_norm.eps)
    out["y_prefill"] = ys[0].numpy()
    out["y_decode"] = torch.cat(ys[1:], dim=1).numpy()
    out["kbar"] = stats[0].numpy()
    out["ceil"] = stats[1].numpy()
    out["kbar_end"] = c._kbar.numpy()
    out["ceil_end"] = c._ceil.numpy()
    _, _, sels, _, _ = run(True)
    out["sel_prefill"] = sels[0][:, :, :N].numpy().astype(np.int32)
    kk = a.cell_topk
    sd = np.full((T, B, H, kk), -1, np.int32)
    for t, s_ in enumerate(sels[1:]):
        sd[t, :, :, :s_.shape[-1]] = s_[:, :, 0].numpy()
    out["sel_decode"] = sd
    # window branch alone, the reference's own rope + band attention
    with torch.no_grad():
        cos, sin = a.rope(N)
        sr = local_attention(_apply_rotary_emb(Q[:, :, :N], cos, sin), _apply_rotary_emb(K[:, :, :N], cos, sin),
                             V[:, :, :N], a.window_size, scale=a.scale, causal=True, sigma=None)
    out["window_prefill"] = sr.numpy()
    out["rope_cos"] = a.rope.cos_cached[:N + T].numpy()
    out["rope_sin"] = a.rope.sin_cached[:N + T].numpy()
    # int8 codec on the bf16 tensors themselves
    qk, sk = kv_int8.quantize_cells(K[:, :, :N].to(torch.bfloat16), a.cell_stride)
    qv, sv = kv_int8.quantize_cells(V[:, :, :N].to(torch.bfloat16), a.cell_stride)
    out["qk"], out["qv"] = qk.numpy(), qv.numpy()
    out["sk"], out["sv"] = _bf16_bits(sk), _bf16_bits(sv)
    out["deq_k"] = _bf16_bits(kv_int8.dequant_cells(qk, sk, a.cell_stride))
    # the decode pool of the first decode block, as the reference builds it
    with torch.no_grad():
        blk = (N // a._cell_block) * a._cell_block
        ncell0 = N // a.cell_stride

        class _C:
            bounded_kv = False

            def completed_cells(self_):
                return stats[0], stats[1], ncell0
        pc = a._build_decode_pool(_C(), blk, a.cell_stride, torch.device("cpu"), need_tokens=False)
    out["pool_cand_c"] = pc["cand_c"].numpy()
    out["pool_ok"] = pc["ok_cell"].numpy()
    np.savez_compressed(os.path.join(HERE, f"fsl_{kind}.npz"), **out)
    print("wrote", f"fsl_{kind}.npz")


def gen_fs_dense(kind: str, B=1, H=2, D=64, N=1000, T=40, seed=31):
    """The dense FS variant (serve preset "dense": cell_prune_kernel = 0, every completed visible cell is a candidate) at the
    Q/K/V level: selections and layer outputs of an N-token prefill and of T decode steps after it."""
    from kv_cache import FSKVCache
    from src.fsattn import FSAttn
    from bench_efficiency import serve_kwargs
    Q, K, V = make_inputs(kind, B, H, N + T, D, seed)
    flat = [t.transpose(1, 2).reshape(B, N + T, H * D).contiguous() for t in (Q, K, V)]
    out = {"kind": kind, "B": B, "H": H, "D": D, "N": N, "T": T, "Q": _bf16_bits(Q), "K": _bf16_bits(K), "V": _bf16_bits(V)}
    x = torch.zeros(B, N + T, H * D)
    os.environ["FS_PRUNE_KERNEL"] = "0"
    try:
        def run(fused):
            kw = serve_kwargs("dense")
            kw.update(fs_fused_attn=1 if fused else 0)
            a = FSAttn(d_model=H * D, n_heads=H, causal=True, bias=False, max_seq_len=4096, **kw).eval()
            g = torch.Generator().manual_seed(seed + 1)
            with torch.no_grad():
                a.sel_scale.copy_(0.5 + torch.rand(H, generator=g) * 2)
                a.log_sigma.copy_(torch.log(1.0 + torch.rand(H, generator=g) * 40))
                a.long_range_scale.copy_((0.05 + torch.rand(H, generator=g)).view(H, 1, 1))
                a.lr_norm.scale.copy_(0.5 + torch.rand(D, generator=g))
                a.W_o.weight.copy_(torch.eye(H * D))
            a.W_q, a.W_k, a.W_v = _Fixed(flat[0]), _Fixed(flat[1]), _Fixed(flat[2])
            sels = []
            if fused:
                def grab(Qx, Kx, Vx, sel, s, Bq, bias=None, q_pos=0):
                    sels.append(sel.clone())
                    return torch.zeros_like(Qx)
                a._cell_fused_lr = grab
            c = FSKVCache(a)
            ys = []
            with torch.no_grad():
                ys.append(a(x[:, :N], cache=c))
                for t in range(T):
                    ys.append(a(x[:, N + t:N + t + 1], cache=c))
            return a, ys, sels
        a, ys, _ = run(False)
        y = ys[0]
        out["y_decode"] = torch.cat(ys[1:], dim=1).numpy()
        out["lam"] = a.sel_scale.detach().numpy()
        out["sigma"] = a.sigma.detach().numpy()
        out["lrs"] = a.long_range_scale.detach().reshape(H).numpy()
        out["norm_w"] = a.lr_norm.scale.detach().numpy()
        out["eps"] = np.float32(a.lr_norm.eps)
        out["y_prefill"] = y.numpy()
        _, _, sels = run(True)
        out["sel_prefill"] = sels[0][:, :, :N].numpy().astype(np.int32)
        kk = a.cell_topk
        sd = np.full((T, B, H, kk), -1, np.int32)
        for t, s_ in enumerate(sels[1:]):
            sd[t, :, :, :s_.shape[-1]] = s_[:, :, 0].numpy()
        out["sel_decode"] = sd
    finally:
        os.environ["FS_PRUNE_KERNEL"] = "1"
    np.savez_compressed(os.path.join(HERE, f"fsdense_{kind}.npz"), **out)
    print("wrote", f"fsdense_{kind}.npz", {k_: v_.shape for k_, v_ in out.items() if hasattr(v_, "shape") and v_.ndim})


def gen_linear(kind: str, B=1, H=2, D=64, N=3000, seed=41):
    """The reference's LinearFSCache driven directly with Q/K/V pieces (its attend splits them at query-block boundaries)."""
    from src.fsattn.linear_cache import LinearFSCache
    Q, K, V = make_inputs(kind, B, H, N, D, seed)
    a = _layer(None, H, D, seed + 1, False)
    c = LinearFSCache(a)
    picked = []
    inner = c.select

    def select(q):
        slots, ids = inner(q)
        if ids is None:
            picked.append(torch.full((B, H, q.shape[2], a.cell_topk), -1, dtype=torch.int64))
        else:
            pad = a.cell_topk - ids.shape[-1]
            picked.append(torch.nn.functional.pad(ids, (0, pad), value=-1) if pad else ids.clone())
        return slots, ids
    c.select = select
    pieces = [700, 129, 1, 1, 1, 37, 900, 3, 128, 512]
    pieces.append(N - sum(pieces))
    ys, o = [], 0
    with torch.no_grad():
        for n in pieces:
            ys.append(c.attend(Q[:, :, o:o + n], K[:, :, o:o + n], V[:, :, o:o + n]))
            o += n
    sel = torch.cat(picked, dim=2)
    # the queries of the first block see no completed cell: the cache does not call select for them
    sel = torch.nn.functional.pad(sel, (0, 0, N - sel.shape[2], 0), value=-1)
    out = {"kind": kind, "B": B, "H": H, "D": D, "N": N, "pieces": np.array(pieces, np.int64),
           "Q": _bf16_bits(Q), "K": _bf16_bits(K), "V": _bf16_bits(V),
           "lam": a.sel_scale.detach().numpy(), "sigma": a.sigma.detach().numpy(),
           "lrs": a.long_range_scale.detach().reshape(H).numpy(), "norm_w": a.lr_norm.scale.detach().numpy(),
           "eps": np.float32(a.lr_norm.eps), "W": a.window_size, "P": c.P, "Wc": c.Wc,
           "y": torch.cat(ys, dim=2).numpy(), "sel": sel.numpy().astype(np.int32),
           "top_ids": c._top["ids"].sort(-1).values.numpy().astype(np.int32),
           "counters": np.array([c.pos, c.eligible, c.max_merge_cells, c.merged_cells, c.updates], np.int64),
           "state_bytes": np.int64(c.state_bytes())}
    np.savez_compressed(os.path.join(HERE, f"linear_{kind}.npz"), **out)
    print("wrote", f"linear_{kind}.npz")


def gen_config1():
    """single random-init FS-L layer, d_model 1024, 16 heads x 64, fp32 on CPU, 4096-token
    prefix then one decode step."""
    from src.fsattn import FSAttn
    from bench_efficiency import serve_kwargs
    from kv_cache import FSKVCache
    out = {}

    def run(fused):
        torch.manual_seed(0)
        kw = serve_kwargs("sparse")
        kw.update(fs_fused_attn=1 if fused else 0, cell_prune_stable_ties=1)
        a = FSAttn(d_model=1024, n_heads=16, causal=True, bias=False, max_seq_len=4352, **kw).eval()
        a.cell_prune_stable_ties = 1
        x = torch.randn(1, 4097, 1024, generator=torch.Generator().manual_seed(1234))
        sels = []
        if fused:
            def grab(Qx, Kx, Vx, sel, s, Bq, bias=None, q_pos=0):
                sels.append(sel.clone())
                return torch.zeros_like(Qx)
            a._cell_fused_lr = grab
        c = FSKVCache(a)
        with torch.no_grad():
            y0 = a(x[:, :4096], cache=c)
            y1 = a(x[:, 4096:4097], cache=c)
        return a, x, y0, y1, sels, c

    a, x, y0, y1, _, c = run(False)
    _, _, _, _, sels, _ = run(True)
    out["x_checksum"] = np.float64(x.double().sum().item())
    out["w_checksum"] = np.float64(sum(p.double().sum().item() for p in a.parameters()))
    out["sel_prefill"] = sels[0][:, :, :4096].numpy().astype(np.int16)
    out["sel_decode"] = sels[1][:, :, 0].numpy().astype(np.int16)
    out["y_prefill_rows"] = np.arange(0, 4096, 16)
    out["y_prefill"] = y0[:, ::16].numpy()
    out["y_decode"] = y1.numpy()
    out["ceil"] = c._ceil.numpy()
    np.savez_compressed(os.path.join(HERE, "fsl_config1.npz"), **out)
    print("wrote fsl_config1.npz")


def gen_fsb(kind: str, B=1, H=2, D=64, N=2000, T=140, seed=23, q_main=0.3, q_union=0.7):
    """One FS-B layer (the serve configuration: fixed policy, width 16, bound score with radius coefficient 8, token
    LSE re-rank to 4, second beam over a second forest) at the Q/K/V level: prefill of N tokens, then T decode steps
    that cross a 128-token block boundary. The two admission thresholds are per-head quantiles of the ceilings.
    Stores the reference's forest tables (main forest), the spines and beam cells of every (row, block), the
    selections and the layer outputs."""
    from kv_cache import FSKVCache
    from bench_efficiency import serve_kwargs
    from src.fsattn import FSAttn, fsb_tree
    Q, K, V = make_inputs(kind, B, H, N + T, D, seed)
    flat = [t.transpose(1, 2).reshape(B, N + T, H * D).contiguous() for t in (Q, K, V)]
    out = {"kind": kind, "B": B, "H": H, "D": D, "N": N, "T": T,
           "Q": _bf16_bits(Q), "K": _bf16_bits(K), "V": _bf16_bits(V)}
    x = torch.zeros(B, N + T, H * D)
    s = 32
    ncell = N // s
    ceil0 = K[:, :, :ncell * s].reshape(B, H, ncell, s, D).norm(dim=-1).amax(-1)
    tau = torch.quantile(ceil0[0], q_main, dim=-1)
    tau_u = torch.quantile(ceil0[0], q_union, dim=-1)
    rec = {"beam": [], "spines": [], "forest": []}

    def run(fused, record):
        kw = serve_kwargs("fsb", 0.5)
        kw.update(fs_fused_attn=1 if fused else 0)
        a = FSAttn(d_model=H * D, n_heads=H, causal=True, bias=False, max_seq_len=4096, **kw).eval()
        g = torch.Generator().manual_seed(seed + 1)
        with torch.no_grad():
            a.sel_scale.copy_(0.5 + torch.rand(H, generator=g) * 2)
            a.log_sigma.copy_(torch.log(1.0 + torch.rand(H, generator=g) * 40))
            a.long_range_scale.copy_((0.05 + torch.rand(H, generator=g)).view(H, 1, 1))
            a.lr_norm.scale.copy_(0.5 + torch.rand(D, generator=g))
            a.W_o.weight.copy_(torch.eye(H * D))
            a.fsb_tau.copy_(tau)
            a.fsb_tau_union.copy_(tau_u)
        a.W_q, a.W_k, a.W_v = _Fixed(flat[0]), _Fixed(flat[1]), _Fixed(flat[2])
        sels = []
        if fused:
            def grab(Qx, Kx, Vx, sel, s_, Bq, bias=None, q_pos=0):
                sels.append(sel.clone())
                return torch.zeros_like(Qx)
            a._cell_fused_lr = grab
        c = FSKVCache(a)
        ys, dsel = [], []
        orig = (fsb_tree._forest_beam, fsb_tree.build_spines, fsb_tree.build_forest)
        if record:
            def beam(*args, **kws):
                r = orig[0](*args, **kws)
                rec["beam"].append((r[0].clone(), r[1].clone()))
                return r

            def spines(F, m_b, t_idx, out=None):
                r = orig[1](F, m_b, t_idx, out=out)
                rec["spines"].append({k_: v_.clone() for k_, v_ in r.items()})
                return r

            def forest(*args, **kws):
                r = orig[2](*args, **kws)
                rec["forest"].append(r)
                return r
            fsb_tree._forest_beam, fsb_tree.build_spines, fsb_tree.build_forest = beam, spines, forest
        try:
            with torch.no_grad():
                ys.append(a(x[:, :N], cache=c))
        finally:
            fsb_tree._forest_beam, fsb_tree.build_spines, fsb_tree.build_forest = orig
        with torch.no_grad():
            for t in range(T):
                ys.append(a(x[:, N + t:N + t + 1], cache=c))
                fc = getattr(c, "_fsb_forest", None)
                ls = getattr(fc, "_last_sel", None) if fc is not None else None
                dsel.append(None if ls is None else ls.clone().reshape(B, H, -1))
        return a, ys, sels, dsel, c

    a, ys, _, dsel, c = run(False, record=True)
    out["lam"] = a.sel_scale.detach().numpy()
    out["sigma"] = a.sigma.detach().numpy()
    out["lrs"] = a.long_range_scale.detach().reshape(H).numpy()
    out["norm_w"] = a.lr_norm.scale.detach().numpy()
    out["eps"] = np.float32(a.lr_norm.eps)
    out["tau"] = tau.numpy()
    out["tau_u"] = tau_u.numpy()
    out["y_prefill"] = ys[0].numpy()
    out["y_decode"] = torch.cat(ys[1:], dim=1).numpy()
    sd = np.full((T, B, H, 4), -1, np.int32)
    for t, s_ in enumerate(dsel):
        if s_ is not None:
            sd[t] = s_.numpy()
    out["sel_decode"] = sd
    _, _, sels, _, _ = run(True, record=False)
    out["sel_prefill"] = sels[0][:, :, :N].numpy().astype(np.int32)
    # the recorded stage: forests [main, second], spines [main, second], beams [main, second]
    assert len(rec["forest"]) == 2 and len(rec["spines"]) == 2 and len(rec["beam"]) == 2, \
        [len(v) for v in rec.values()]
    for tag, F in zip(("f", "fu"), rec["forest"]):
        out[tag + "_node"] = F["node"].numpy()
        out[tag + "_leaf"] = F["leaf"].numpy().astype(np.int32)
        out[tag + "_adm"] = F["adm"].numpy().astype(np.int32)
        out[tag + "_mtot"] = F["m_tot"].numpy().astype(np.int32)
        ks = sorted(F["bases"])
        out[tag + "_ks"] = np.array(ks, np.int32)
        out[tag + "_bases"] = np.array([F["bases"][k] for k in ks], np.int32)
        out[tag + "_leafbases"] = np.array([F["leafbases"][k] for k in ks], np.int32)
        out[tag + "_Kmax"] = np.int32(F["Kmax"])
    for tag, SP in zip(("sp", "spu"), rec["spines"]):
        out[tag + "_node"] = SP["node"].numpy()
        out[tag + "_root"] = SP["root"].numpy().astype(np.int32)
        out[tag + "_height"] = SP["height"].numpy().astype(np.int32)
        out[tag + "_mb"] = SP["m_b"].numpy().astype(np.int32)
        out[tag + "_tidx"] = SP["t_idx"].numpy().astype(np.int32)
    for tag, (cells, nv) in zip(("beam", "beamu"), rec["beam"]):
        out[tag + "_cells"] = cells.numpy().astype(np.int32)
        out[tag + "_nvis"] = nv.numpy().astype(np.int32)
    out["kbar"] = c._kbar.numpy() if hasattr(c, "_kbar") else np.zeros(0)
    out["ceil"] = c._ceil.numpy() if hasattr(c, "_ceil") else np.zeros(0)
    np.savez_compressed(os.path.join(HERE, f"fsb_{kind}.npz"), **out)
    print("wrote", f"fsb_{kind}.npz", {k_: v_.shape for k_, v_ in out.items() if hasattr(v_, "shape") and v_.ndim})


MODEL_DEBUG = dict(vocab_size=1024, d_model=256, n_layers=4, n_heads=4, d_ff=688, max_seq_len=1024)


def gen_model(variant: str, P0=330, T=72, seed=0):
    """The reference's FreeSoloLM + FSKVCache + its greedy loop (experiments/scaling/kv_cache.py:484-526) on CPU."""
    from bench_efficiency import serve_kwargs
    from kv_cache import make_caches, _trunk_cached
    from longctx_infer import _lm_head_fp32, extend_rope_cache
    from model import FreeSoloLM
    from src.fsattn import fsb_tree
    os.environ["FS_PRUNE_KERNEL"] = "1" if variant == "fsl" else "0"
    kw = serve_kwargs("sparse") if variant == "fsl" else serve_kwargs("fsb", 0.9)
    gi = torch.Generator().manual_seed(100 + seed)
    ids = torch.randint(0, MODEL_DEBUG["vocab_size"], (2, P0), generator=gi)
    warm = torch.randint(0, MODEL_DEBUG["vocab_size"], (1, 512), generator=gi)
    out = {"variant": variant, "P0": P0, "T": T, "ids": ids.numpy().astype(np.int32), "warm": warm.numpy().astype(np.int32)}
    for prec in ("fp32", "bf16"):
        torch.manual_seed(seed)
        m = FreeSoloLM(**MODEL_DEBUG, **kw).eval()
        with torch.no_grad():
            for p_ in m.parameters():                     # both sides hold exactly these weights
                p_.copy_(p_.to(torch.bfloat16).float())
        out["w_checksum"] = np.float64(sum(p_.double().sum().item() for p_ in m.parameters()))
        out["w_abs_checksum"] = np.float64(sum(p_.double().abs().sum().item() for p_ in m.parameters()))
        extend_rope_cache(m, P0 + T + 64)
        if prec == "bf16":
            m = m.to(torch.bfloat16)
        if variant == "fsb":
            with torch.no_grad():
                r1 = fsb_tree.fsb_calibrate_tau(m, [warm], 0.5, target="fsb_tau")
                r2 = fsb_tree.fsb_calibrate_tau(m, [warm], 0.9, target="fsb_tau_union")
            out[f"tau_{prec}"] = r1["tau"].numpy()
            out[f"tau_u_{prec}"] = r2["tau"].numpy()
        caches = make_caches(m, reserve=T + 8)
        logits, toks = [], []
        step_in = ids
        with torch.no_grad():
            for t in range(T):
                hidden = _trunk_cached(m, step_in, caches)
                lg = _lm_head_fp32(m, hidden[:, -1:, :], 4096)[:, 0, :]
                nxt = lg.argmax(dim=-1)
                logits.append(lg.float())
                toks.append(nxt)
                # the bf16 run is fed the fp32 run's tokens
                step_in = (nxt if prec == "fp32" else torch.from_numpy(out["tokens_fp32"][:, t]).long()).unsqueeze(1)
        out[f"logits_{prec}"] = torch.stack(logits, 1).numpy()          # (B, T, V)
        out[f"tokens_{prec}"] = torch.stack(toks, 1).numpy().astype(np.int32)
    os.environ["FS_PRUNE_KERNEL"] = "1"
    np.savez_compressed(os.path.join(HERE, f"model_{variant}.npz"), **out)
    print(f"wrote model_{variant}.npz")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("FREESOLO_REFERENCE", "/root/reference"),
                    help="checkout of the reference project (zekun-shi/freesolo)")
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    sys.path[:0] = [os.path.join(args.reference, "experiments", "scaling"), args.reference]
    os.environ.update(FS_STRICT_CAUSAL="1", FS_PRUNE_KERNEL="1", FSB_TRAIN_GRAPH="0")
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    only = set(filter(None, args.only.split(",")))
    jobs = {
        "fsl_randn": lambda: gen_fsl("randn"),
        "fsl_vocab": lambda: gen_fsl("vocab", N=1000, T=40, seed=11),
        "fsl_periodic": lambda: gen_fsl("periodic", N=640, T=8, seed=13),
        "fsl_lowprec": lambda: gen_fsl("lowprec", N=640, T=8, seed=17),
        "fsl_config1": gen_config1,
        "linear_randn": lambda: gen_linear("randn"),
        "linear_vocab": lambda: gen_linear("vocab", seed=43),
        "fsb_randn": lambda: gen_fsb("randn"),
        "fsb_vocab": lambda: gen_fsb("vocab", N=1500, T=40, seed=29),
        "fsdense_randn": lambda: gen_fs_dense("randn"),
        "fsdense_vocab": lambda: gen_fs_dense("vocab", N=900, T=24, seed=37),
        "model_fsl": lambda: gen_model("fsl"),
        "model_fsb": lambda: gen_model("fsb"),
    }
    for name, fn in jobs.items():
        if not only or name in only:
            fn()


if __name__ == "__main__":
    main()
