"""CPU restatement of the FS-B long-range path (two forests, beam search, candidate re-rank). TEST INFRASTRUCTURE ONLY.

Nothing in the product may import this file; the tests, the smoke check and the benchmark's CPU baseline use it as
the checker. Each function cites the file:line of zekun-shi/freesolo it restates (paths inside that project). The
restatement is pinned by executing the reference on CPU: tests/golden/make_golden.py stores the reference's own
forest tables, spines, beam cells, selections and outputs in tests/golden/fsb_*.npz, and tests/test_oracle_golden.py
requires this file to reproduce them (tables and candidates bit for bit).

Everything here is fp32 with IEEE add/mul/div/sqrt in one fixed association order (`det_sum`: repeated halving),
so a device build that keeps that order and never contracts a multiply-add reproduces the trees exactly.

Own data layout (not the reference's packed arena): a forest is a dict holding, per chunk height k, tensors over the
chunks j of that height: mu (C, 2^{k+1}-1, D), rad/amax/pmin (C, 2^{k+1}-1), leaf (C, 2^k); nodes of a chunk are in
level order (node n has children 2n+1, 2n+2; the nodes of level l are n = 2^l-1 .. 2^{l+1}-2 and hold 2^{k-l} cells).
"""
from __future__ import annotations

import math

import torch

NEG = -1e9


# ---------------------------------------------------------------------------------------------------------------
# deterministic reductions (src/fsattn/det_reduce.py: det_sum; src/fsattn/fsb_tree.py:602-613)
# ---------------------------------------------------------------------------------------------------------------
def det_sum(x: torch.Tensor, dim: int) -> torch.Tensor:
    """Sum over `dim` by repeated halving: pad with zeros to a power of two, then y[i] = x[i] + x[i + n/2]."""
    x = x.movedim(dim, -1)
    n = x.shape[-1]
    p = 1
    while p < n:
        p *= 2
    if p != n:
        x = torch.cat([x, x.new_zeros(*x.shape[:-1], p - n)], dim=-1)
    while p > 1:
        p //= 2
        x = x[..., :p] + x[..., p:2 * p]
    return x[..., 0]


def ieee_sqrt(x: torch.Tensor) -> torch.Tensor:
    """Correctly rounded fp32 square root. torch's vectorised CPU sqrt is not (it is off by one ulp for about 5% of
    inputs on AVX2 hosts, measured against numpy and float64), while CUDA's sqrtf and numpy's are; the restatement
    uses the IEEE result so that it does not depend on the host CPU. The reference's CPU fixtures therefore match radii
    to one ulp only."""
    import numpy as np
    return torch.from_numpy(np.asarray(np.sqrt(x.detach().contiguous().numpy()), dtype=np.float32)).reshape(x.shape)


def det_dot(a, b):
    return det_sum(a * b, -1)


def det_norm(a):
    return ieee_sqrt(det_sum(a * a, -1))


# ---------------------------------------------------------------------------------------------------------------
# forest build (src/fsattn/fsb_tree.py:616-678 build_trees, 881-951 build_forest)
# ---------------------------------------------------------------------------------------------------------------
def admitted(ceil_row: torch.Tensor, tau: float, m_vis: int | None = None) -> torch.Tensor:
    """Ids of the cells of one row whose ceiling is >= tau, ascending (fsb_tree.py:936-941). m_vis: only cells
    [0, m_vis) are candidates (the decode-time prefix, fsb_tree.py:3636-3641)."""
    c = ceil_row if m_vis is None else ceil_row[:m_vis]
    return torch.nonzero(c >= tau).flatten()


def chunk_trees(X: torch.Tensor, ce: torch.Tensor, ids: torch.Tensor) -> dict:
    """Trees of C chunks of n = 2^k cells each. X (C, n, D) fp32 chunk-mean keys in admission order, ce (C, n)
    ceilings, ids (C, n) cell ids. Restates build_trees (fsb_tree.py:638-675) for a full chunk: every node of level l
    holds exactly n >> l cells, so the reference's slot padding only ever adds zeros and drops out.

    Per node: mu = det_sum(x)/m; rad = sqrt(max |x-mu|^2); amax = max(ceiling, 0); pmin = min id; split: start from
    the member farthest from mu, two power iterations of the centred scatter, project, STABLE ascending sort, lower
    half left."""
    C, n, D = X.shape
    k = int(math.log2(n))
    assert 1 << k == n
    mu_l, rad_l, am_l, pm_l = [], [], [], []
    order = torch.arange(n).expand(C, n).clone()           # slot -> position inside the chunk
    for l in range(k + 1):
        m = n >> l
        nodes = 1 << l
        idx = order.view(C, nodes, m)
        Xn = torch.gather(X, 1, order[..., None].expand(-1, -1, D)).view(C, nodes, m, D)
        mu = det_sum(Xn, 2) / float(m)
        Xc = Xn - mu[:, :, None, :]
        d2 = det_sum(Xc * Xc, -1)
        mu_l.append(mu)
        rad_l.append(ieee_sqrt(d2.amax(-1)))
        am_l.append(torch.gather(ce, 1, order).view(C, nodes, m).amax(-1).clamp(min=0.0))
        pm_l.append(torch.gather(ids, 1, order).view(C, nodes, m).amin(-1))
        if l == k:
            break
        far = d2.argmax(-1)                                  # first maximum
        v = torch.gather(Xc, 2, far[..., None, None].expand(-1, -1, 1, D)).squeeze(2)
        v = v / det_norm(v)[..., None].clamp_min(1e-6)
        for _ in range(2):
            pv = det_sum(Xc * v[:, :, None, :], -1)
            v = det_sum(Xc * pv[..., None], 2)
            v = v / det_norm(v)[..., None].clamp_min(1e-6)
        proj = det_sum(Xc * v[:, :, None, :], -1)
        srt = proj.argsort(dim=-1, stable=True)
        order = torch.gather(idx, 2, srt).reshape(C, n)
    return {"k": k, "mu": torch.cat(mu_l, 1), "rad": torch.cat(rad_l, 1), "amax": torch.cat(am_l, 1),
            "pmin": torch.cat(pm_l, 1), "leaf": torch.gather(ids, 1, order)}


def build_forest_row(kbar: torch.Tensor, ceil_row: torch.Tensor, adm: torch.Tensor) -> dict:
    """Forest of one row: for every height k, the chunks (k, j) = admitted positions [j 2^k, (j+1) 2^k) that lie
    wholly inside the admitted sequence (fsb_tree.py:897-911). kbar (M, D) fp32, adm = admitted ids ascending."""
    m_tot = int(adm.numel())
    F = {"adm": adm, "m_tot": m_tot, "chunks": {}}
    k = 0
    while (m_tot >> k) > 0:
        C = m_tot >> k
        ids = adm[:C << k].view(C, 1 << k)
        F["chunks"][k] = chunk_trees(kbar[ids], ceil_row[ids], ids)
        k += 1
    return F


def beam_tables(F: dict) -> None:
    """The beams' view of the chunk nodes (fsb_tree.py:1049-1066): mu rounded to bf16 and each radius inflated by the
    rounding error's norm, so (q.mu + |q| rad) stays an upper bound. Adds mu16 / rad_b to every chunk table."""
    for t in F["chunks"].values():
        mu16 = t["mu"].to(torch.bfloat16)
        t["mu16"] = mu16
        t["rad_b"] = t["rad"] + det_norm(t["mu"] - mu16.float())


def flatten_row(F: dict, D: int) -> dict:
    """One flat node table per row for the beam: node id = base[k] + j (2^{k+1}-1) + n. Columns follow the beam's
    needs: mu (bf16 values as fp32), rad (inflated), amax, pmin, cnt, child ids (-1 at leaves), cell (leaf's cell id,
    -1 for inner nodes). The exact fp32 means and radii of the chunk ROOTS are kept too, for the spines."""
    if "mu16" not in next(iter(F["chunks"].values()), {"mu16": None}):
        beam_tables(F)
    mu, rad, amax, pmin, cnt, chl, chr_, cell = [], [], [], [], [], [], [], []
    base = {}
    nb = 0
    for k, t in sorted(F["chunks"].items()):
        C = t["mu"].shape[0]
        nodes = (2 << k) - 1
        base[k] = nb
        n = torch.arange(nodes)
        lvl = torch.floor(torch.log2((n + 1).double())).long()
        inner = n < (1 << k) - 1
        g = nb + torch.arange(C)[:, None] * nodes
        mu.append(t["mu16"].float().reshape(-1, D)); rad.append(t["rad_b"].reshape(-1))
        amax.append(t["amax"].reshape(-1)); pmin.append(t["pmin"].reshape(-1))
        cnt.append((1 << (k - lvl)).expand(C, nodes).reshape(-1))
        chl.append(torch.where(inner[None], g + 2 * n[None] + 1, torch.full((C, nodes), -1)).reshape(-1))
        chr_.append(torch.where(inner[None], g + 2 * n[None] + 2, torch.full((C, nodes), -1)).reshape(-1))
        cl = torch.full((C, nodes), -1, dtype=torch.long)
        cl[:, (1 << k) - 1:] = t["leaf"]
        cell.append(cl.reshape(-1))
        nb += C * nodes
    cat = lambda xs, e: torch.cat(xs) if xs else e
    return {"mu": cat(mu, torch.zeros(0, D)), "rad": cat(rad, torch.zeros(0)), "amax": cat(amax, torch.zeros(0)),
            "pmin": cat(pmin, torch.zeros(0, dtype=torch.long)), "cnt": cat(cnt, torch.zeros(0, dtype=torch.long)),
            "chl": cat(chl, torch.zeros(0, dtype=torch.long)), "chr": cat(chr_, torch.zeros(0, dtype=torch.long)),
            "cell": cat(cell, torch.zeros(0, dtype=torch.long)), "base": base, "n": nb}


# ---------------------------------------------------------------------------------------------------------------
# spines (src/fsattn/fsb_tree.py:1070-1132 build_spines)
# ---------------------------------------------------------------------------------------------------------------
def spine(F: dict, flat: dict, m_b: int, D: int) -> dict:
    """The nodes that join the chunk roots named by the bits of m_b into one tree over the first m_b admitted cells.
    Walks k upward with a running node r: the first present root becomes r, each further present root c gives a new
    node {children: (c, r)}. Uses the roots' exact fp32 means and un-inflated radii (the reference reads its packed
    fp32 rows there, fsb_tree.py:1088-1090). Spine node for height k gets the id flat['n'] + k."""
    S = max(F["chunks"].keys(), default=-1) + 1
    nodes = {}
    r = None            # (mu, rad, amax, pmin, cnt, id)
    npres = 0
    for k in range(S):
        if not (m_b >> k) & 1:
            continue
        npres += 1
        j = (m_b >> (k + 1)) << 1
        t = F["chunks"][k]
        c = (t["mu"][j, 0], t["rad"][j, 0], t["amax"][j, 0], int(t["pmin"][j, 0]), 1 << k,
             flat["base"][k] + j * ((2 << k) - 1))
        if r is None:
            r = c
            continue
        tot = torch.tensor(float(c[4] + r[4]))
        mu = (float(c[4]) * c[0] + float(r[4]) * r[0]) / tot
        rad = torch.maximum(c[1] + det_norm(c[0] - mu), r[1] + det_norm(r[0] - mu))
        nid = flat["n"] + k
        nodes[k] = {"mu": mu, "rad": rad, "amax": torch.maximum(c[2], r[2]), "pmin": min(c[3], r[3]),
                    "cnt": c[4] + r[4], "chl": c[5], "chr": r[5]}
        r = (mu, rad, nodes[k]["amax"], nodes[k]["pmin"], nodes[k]["cnt"], nid)
    height = 0
    if m_b > 1:
        height = int(math.floor(math.log2(m_b))) + (1 if npres >= 2 else 0)
    return {"nodes": nodes, "root": (r[5] if r is not None else -1), "height": height, "S": S}


def row_tables(flat: dict, sp: dict, D: int) -> dict:
    """Chunk table + this spine's nodes as one table (spine node of height k at index flat['n'] + k)."""
    S = sp["S"]
    ext = {"mu": torch.zeros(S, D), "rad": torch.zeros(S), "amax": torch.zeros(S),
           "pmin": torch.zeros(S, dtype=torch.long), "cnt": torch.zeros(S, dtype=torch.long),
           "chl": torch.full((S,), -1), "chr": torch.full((S,), -1), "cell": torch.full((S,), -1)}
    for k, nd in sp["nodes"].items():
        for f in ("mu", "rad", "amax", "pmin", "cnt", "chl", "chr"):
            ext[f][k] = nd[f]
    return {f: torch.cat([flat[f], ext[f]]) for f in ext}


# ---------------------------------------------------------------------------------------------------------------
# beam (src/fsattn/fsb_tree.py:1321-1400 _forest_beam; policy 2263-2270)
# ---------------------------------------------------------------------------------------------------------------
def beam_policy(height: int, width: int, delta: int):
    """Fixed policy (fsb_tree.py:2267-2270): stop depth D0 = max(height - delta, 0); frontier W = min(width, 2^D0);
    a node is expanded while it holds more than budget = 2^(height - D0) cells."""
    d0 = max(height - delta, 0)
    return min(width, 1 << d0), 1 << (height - d0)


def beam_row(tab: dict, root: int, q: torch.Tensor, qpos: torch.Tensor, lam: float, sig: float, scale: float,
             s: int, W: int, budget: int, W_max: int, rc: float, iters: int):
    """Beam over one (row, block): q (Bq, D) fp32, qpos (Bq,). Returns the final frontier's cells (Bq, W_max) (-1
    pad; one cell per frontier slot, the budget-1 case of the serve configuration) and the visit counts (Bq,).

    Each iteration: a frontier node with cnt > budget is replaced by its two children, which are scored
    (q.mu)*scale + (|q| rc rad)*scale + (lam amax) erf(|p - (pmin+.5) s| / (2 sig)); the others are carried. The
    new frontier is the carried nodes in slot order, then children by (score desc, position asc), cut to W."""
    Bq, D = q.shape
    ref = torch.full((Bq, W_max), -1, dtype=torch.long)
    ref[:, 0] = root
    qn = det_norm(q) * rc
    nvis = torch.zeros(Bq)
    slot = torch.arange(W_max)
    margin = torch.full((Bq,), float("inf"))      # smallest score gap at a frontier cut-off (test bookkeeping)
    for _ in range(iters):
        act = ref >= 0
        rc_ = ref.clamp(min=0)
        expand = act & (tab["cnt"][rc_] > budget)
        carried = act & ~expand
        ch = torch.stack([tab["chl"][rc_], tab["chr"][rc_]], -1)
        ch = torch.where(expand[..., None], ch, torch.full_like(ch, -1)).view(Bq, 2 * W_max)
        cc = ch.clamp(min=0)
        content = det_dot(q[:, None, :], tab["mu"][cc]) * scale
        content = content + qn[:, None] * tab["rad"][cc] * scale
        ppos = (tab["pmin"][cc].float() + 0.5) * s
        erf = torch.erf((qpos[:, None] - ppos).abs() / (2.0 * sig))
        score = (content + lam * tab["amax"][cc] * erf).masked_fill(ch < 0, NEG)
        cand = torch.cat([ref.masked_fill(~carried, -1), ch], -1)
        csc = torch.cat([torch.where(carried, 1e30, NEG), score], -1)
        tv, ti = torch.sort(csc, dim=-1, descending=True, stable=True)
        tv, ti = tv[:, :W_max], ti[:, :W_max]
        ok = (tv > NEG / 2) & (slot[None] < W)
        ref = torch.gather(cand, 1, ti).masked_fill(~ok, -1)
        nvis = nvis + (ch >= 0).sum(-1).float()
        sv = torch.sort(score, dim=-1, descending=True).values
        nk = (W - carried.sum(-1)).clamp(min=0)
        cut = (nk > 0) & (nk < (ch >= 0).sum(-1))
        i1 = nk.clamp(min=1, max=2 * W_max - 1)
        gap = sv.gather(1, (i1 - 1)[:, None])[:, 0] - sv.gather(1, i1[:, None])[:, 0]
        margin = torch.where(cut, torch.minimum(margin, gap), margin)
    cells = torch.where(ref >= 0, tab["cell"][ref.clamp(min=0)], torch.full_like(ref, -1))
    return cells, nvis, margin


def union_candidates(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Main candidates then the second beam's, with the second beam's repeats of a main cell blanked
    (fsb_tree.py:711-713)."""
    dup = (b[..., :, None] == a[..., None, :]).any(-1)
    return torch.cat([a, b.masked_fill(dup, -1)], -1)


# ---------------------------------------------------------------------------------------------------------------
# re-rank (src/fsattn/fsb_tree.py:820-869 rerank_top, score 'lse_pos'; src/fsattn/fsb_rerank.py:83-125)
# ---------------------------------------------------------------------------------------------------------------
def rerank_scores(cand: torch.Tensor, q: torch.Tensor, qpos: torch.Tensor, lam: float, sig: float,
                  ceil_row: torch.Tensor, Ktok: torch.Tensor, scale: float, s: int) -> torch.Tensor:
    """u = LSE over the cell's s tokens of (q.k_t)*scale + lam ceil erf(|p - (c+.5) s| / (2 sig)); -inf for empty
    slots. cand (Bq, C) cell ids, q (Bq, D) fp32, Ktok (>= ncell*s, D) raw keys of the row (any float dtype)."""
    Bq, C = cand.shape
    ok = cand >= 0
    cc = cand.clamp(min=0)
    tok = cc[..., None] * s + torch.arange(s)
    kt = Ktok[tok].float()                                            # (Bq, C, s, D)
    sc = det_sum(kt * q[:, None, None, :], -1) * scale
    m = sc.amax(-1)
    lse = m + torch.log(det_sum(torch.exp(sc - m[..., None]), -1))
    erf = torch.erf((qpos[:, None] - (cc.float() + 0.5) * s).abs() / (2.0 * sig))
    u = lse + lam * ceil_row[cc] * erf
    return u.masked_fill(~ok, float("-inf"))


def rerank_top(cand, u, K: int):
    """Stable descending sort of u; the first K candidates; -inf picks become -1. Also returns the margin: the
    smallest gap between consecutive scores among the best K+1 finite ones (inf when fewer than two)."""
    tv, ti = torch.sort(u, dim=-1, descending=True, stable=True)
    out = torch.gather(cand, -1, ti[..., :K]).masked_fill(tv[..., :K] == float("-inf"), -1)
    top = tv[..., :K + 1]
    gap = (top[..., :-1] - top[..., 1:])
    gap = torch.where(torch.isfinite(gap), gap, torch.full_like(gap, float("inf")))
    return out, gap.amin(-1)


# ---------------------------------------------------------------------------------------------------------------
# drivers: prefill (src/fsattn/fsb_tree.py:2368-2520 fsb_long_range, 2622-2644 prefill_forests, 1183-1317
# traverse_forest in the serve configuration) and decode (3598-3674 fsb_decode_prepare, 3002-3064)
# ---------------------------------------------------------------------------------------------------------------
SERVE = {"width": 16, "delta": 0, "W_max": 16, "union_width": 16, "union_W_max": 16, "rc": 8.0, "read_top": 4}
"""The released serve configuration (experiments/scaling/bench_efficiency.py:79-82; fsb_tree.py:41-133)."""


class RowForests:
    """Both forests of one (batch, head) row over the cells [0, m_vis): admission tau (main) and tau_u (second
    beam). The streaming forest of the reference equals the forest built from scratch over the same prefix
    (tests/test_fsb_cache.py), so decode uses this class as well."""

    def __init__(self, kbar: torch.Tensor, ceil_row: torch.Tensor, tau: float, tau_u: float | None, m_vis=None):
        D = kbar.shape[-1]
        self.D = D
        self.F = build_forest_row(kbar, ceil_row, admitted(ceil_row, tau, m_vis))
        self.flat = flatten_row(self.F, D)
        if tau_u is None:
            self.Fu, self.flatu = self.F, self.flat
        else:
            self.Fu = build_forest_row(kbar, ceil_row, admitted(ceil_row, tau_u, m_vis))
            self.flatu = flatten_row(self.Fu, D)

    def prefix_counts(self, E: int):
        """Admitted cells with id < E in each forest (fsb_tree.py:2640-2641)."""
        return int((self.F["adm"] < E).sum()), int((self.Fu["adm"] < E).sum())


def select_block(rf: RowForests, E: int, q, qpos, lam, sig, scale, s, ceil_row, Ktok, cfg=SERVE, want=None):
    """Selections of the queries of one block whose visible cells are [0, E): both beams, union, re-rank, top-K.
    q (Bq, D) fp32, qpos (Bq,) fp32. Returns sel (Bq, K) int64 (-1 pad) and the margin (Bq,): the smaller of the
    re-rank margin (smallest gap among the best K+1 re-rank scores) and the beam margin (smallest score gap at any
    frontier cut-off of either beam), i.e. how far the fp32 scores are from changing the selection anywhere on the way.
    `want`, when a dict, also receives the two beams' cells, the visit counts, the spine heights and the two margins
    separately (`rerank_margin`, `beam_margin`)."""
    Bq = q.shape[0]
    m_b, m_bu = rf.prefix_counts(E)
    outs = []
    for F, flat, mb, width, wmax in ((rf.F, rf.flat, m_b, cfg["width"], cfg["W_max"]),
                                     (rf.Fu, rf.flatu, m_bu, cfg["union_width"], cfg["union_W_max"])):
        sp = spine(F, flat, mb, rf.D)
        if sp["root"] < 0:
            outs.append((torch.full((Bq, wmax), -1, dtype=torch.long), torch.zeros(Bq), sp,
                         torch.full((Bq,), float("inf"))))
            continue
        W, budget = beam_policy(sp["height"], width, cfg["delta"])
        tab = row_tables(flat, sp, rf.D)
        cells, nv, bm = beam_row(tab, sp["root"], q, qpos, lam, sig, scale, s, W, budget, wmax, cfg["rc"],
                                 sp["height"] + 1)
        outs.append((cells, nv, sp, bm))
    cand = union_candidates(outs[0][0], outs[1][0])
    u = rerank_scores(cand, q, qpos, lam, sig, ceil_row, Ktok, scale, s)
    sel, margin = rerank_top(cand, u, cfg["read_top"])
    beam_margin = torch.minimum(outs[0][3], outs[1][3])
    if want is not None:
        want.update(main=outs[0][0], union=outs[1][0], nvis=outs[0][1] + outs[1][1], cand=cand, u=u,
                    height=(outs[0][2]["height"], outs[1][2]["height"]), m_b=(m_b, m_bu),
                    beam_margin=beam_margin, rerank_margin=margin)
    return sel, torch.minimum(margin, beam_margin)


def fsb_select_prefill(Q, K, kbar, ceil_c, tau, tau_u, lam, sigma, scale, s=32, Bq=128, cfg=SERVE, blocks=None):
    """Prefill selections of every query. Q, K (B, H, N, D); kbar (B, H, M, D) fp32 and ceil_c (B, H, M) for the
    M = N // s complete cells; tau, tau_u (H,) (tau_u None: the second beam searches the main forest). Block b sees
    the cells that end at or before its first query: E = (b Bq) // s. Returns sel (B, H, nb Bq, K) and margins."""
    B, H, N, D = Q.shape
    Bq = min(Bq, N)
    nb = (N + Bq - 1) // Bq
    K_ = cfg["read_top"]
    sel = torch.full((B, H, nb * Bq, K_), -1, dtype=torch.long)
    mar = torch.full((B, H, nb * Bq), float("inf"))
    M = kbar.shape[2]
    for b in range(B):
        for h in range(H):
            rf = RowForests(kbar[b, h].float(), ceil_c[b, h].float(), float(tau[h]),
                            None if tau_u is None else float(tau_u[h]))
            Ktok = K[b, h]
            for blk in (range(nb) if blocks is None else blocks):
                q0 = blk * Bq
                n = min(Bq, N - q0)
                q = torch.zeros(Bq, D)
                q[:n] = Q[b, h, q0:q0 + n].float()
                qpos = torch.arange(q0, q0 + Bq, dtype=torch.float32)
                E = min(q0 // s, M)
                sb, mb_ = select_block(rf, E, q, qpos, float(lam[h]), float(sigma[h]), scale, s,
                                       ceil_c[b, h].float(), Ktok, cfg)
                sel[b, h, q0:q0 + Bq] = sb
                mar[b, h, q0:q0 + Bq] = mb_
    return sel, mar


def fsb_select_decode(q_t, pos, Ktok, kbar, ceil_c, ncell, tau, tau_u, lam, sigma, scale, s=32, Bq=128, cfg=SERVE,
                      cache=None):
    """Selections of one decode query per row at position pos. q_t (B, H, D); Ktok (B, H, >= ncell s, D) the raw keys
    as the cache reads them; kbar/ceil_c the completed cells' statistics. Visible cells: [0, min(blk_start // s,
    ncell)) with blk_start = (pos // Bq) Bq (fsb_tree.py:3604,3636). `cache`: a dict reused across the steps of one
    block so that the forests are built once per block, as the reference does."""
    B, H, D = q_t.shape
    blk = (pos // Bq) * Bq
    E = min(blk // s, ncell)
    sel = torch.full((B, H, cfg["read_top"]), -1, dtype=torch.long)
    mar = torch.full((B, H), float("inf"))
    for b in range(B):
        for h in range(H):
            key = (b, h, blk)
            rf = cache.get(key) if cache is not None else None
            if rf is None:
                rf = RowForests(kbar[b, h, :ncell].float(), ceil_c[b, h, :ncell].float(), float(tau[h]),
                                None if tau_u is None else float(tau_u[h]), m_vis=E)
                if cache is not None:
                    cache[key] = rf
            sb, mb_ = select_block(rf, E, q_t[b, h].float()[None], torch.tensor([float(pos)]), float(lam[h]),
                                   float(sigma[h]), scale, s, ceil_c[b, h].float(), Ktok[b, h], cfg)
            sel[b, h] = sb[0]
            mar[b, h] = mb_[0]
    return sel, mar


class FSBLayerOracle:
    """Functional model of one FS-B attention layer behind the FSAttn / FSKVCache boundary: the FS-L layer model with
    the selection replaced by the two-forest beam + re-rank (src/fsattn/attention.py:936-1131 with fsb_enabled;
    src/fsattn/fsb_tree.py:2368-2520 prefill, 3598-3674 + 2909-2999 decode). Window, readout and combine are the
    FS-L oracle's."""

    def __init__(self, H, D, *, tau, tau_u=None, cfg=SERVE, **kw):
        from .fsl import FSLLayerOracle
        self.base = FSLLayerOracle(H, D, **kw)
        self.tau, self.tau_u, self.cfg = tau, tau_u, cfg
        self._dec_cache = {}

    def prefill(self, Q, K, V):
        from .fsl import cell_readout, cell_stats, lr_norm_combine, window_attention
        b = self.base
        B, H, N, D = Q.shape
        sr = window_attention(Q, K, V, b.cos, b.sin, b.W, b.scale, act_dtype=b.act).to(b.act)
        kbar, ceil = cell_stats(K, b.s)
        sel, margin = fsb_select_prefill(Q, K, kbar, ceil, self.tau, self.tau_u, b.lam, b.sigma, b.scale, b.s, b.Bq,
                                         self.cfg)
        o = cell_readout(Q, K, V, sel, b.s, min(b.Bq, N), b.scale, 0, N)
        y = lr_norm_combine(sr, o, b.norm_w, b.lrs, b.eps, b.act)
        b.K, b.V, b.pos = K.clone(), V.clone(), N
        return y, sel[:, :, :N], margin[:, :, :N]

    def decode(self, q, k, v):
        from .fsl import cell_readout, cell_stats, lr_norm_combine, window_attention
        b = self.base
        pos = b.pos
        b.K = torch.cat([b.K, k], dim=2) if b.K is not None else k.clone()
        b.V = torch.cat([b.V, v], dim=2) if b.V is not None else v.clone()
        kbar, ceil = cell_stats(b.K, b.s)
        Kr, Vr = b._kv_read()
        j0 = max(0, pos - b.W)
        sr = window_attention(q, Kr[:, :, j0:pos + 1], Vr[:, :, j0:pos + 1], b.cos, b.sin, b.W, b.scale,
                              q_pos0=pos, k_pos0=j0, act_dtype=b.act).to(b.act)
        sel, margin = fsb_select_decode(q[:, :, 0], pos, Kr, kbar, ceil, kbar.shape[2], self.tau, self.tau_u, b.lam,
                                        b.sigma, b.scale, b.s, b.Bq, self.cfg, cache=self._dec_cache)
        sel = sel[:, :, None, :]
        o = cell_readout(q, Kr, Vr, sel, b.s, b.Bq, b.scale, pos, pos + 1)
        y = lr_norm_combine(sr, o, b.norm_w, b.lrs, b.eps, b.act)
        b.pos = pos + 1
        return y, sel, margin[:, :, None]
