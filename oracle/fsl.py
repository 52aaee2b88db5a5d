"""CPU oracle (test infrastructure, never on the product path): FS-L selection, bounded retention pool, int8 KV codec,
cell readout + combine and the RoPE window branch, restated in torch-on-CPU fp32.

Conventions: B batch, H heads, D head dim, N tokens, s cell (chunk) size, Bq query block, kk cells read per query,
P pool size, Wc newest-cell slots, W window. "cell" is the reference's word for a 32-token chunk.

Parity status: pinned by execution against the reference (tests/golden/make_golden.py -> tests/golden/*.npz).
"""
from __future__ import annotations

import math

import torch

NEG = -1e9


# ---------------------------------------------------------------------------------------------------------------
# cell statistics and int8 codec
# ---------------------------------------------------------------------------------------------------------------
def cell_stats(K: torch.Tensor, s: int):
    """Chunk-mean key and ceiling of every completed cell.

    Follows src/fsattn/attention.py:727-737 and experiments/scaling/kv_cache.py:274-285: the mean is taken in the key
    dtype and then widened, the ceiling is the largest fp32 L2 norm of the cell's token keys.
    K (B,H,N,D) -> kbar (B,H,M,D) fp32, ceil (B,H,M) fp32 with M = N // s."""
    B, H, N, D = K.shape
    M = N // s
    Kc = K[:, :, :M * s].reshape(B, H, M, s, D)
    return Kc.mean(dim=3).float(), Kc.float().norm(dim=-1).amax(dim=-1)


def quantize_cells(x: torch.Tensor, s: int):
    """Per-(batch, head, cell) symmetric int8 with a bf16 scale; src/fsattn/kv_int8.py:51-59.
    scale = bf16(max|x| / 127) (1.0 for an all-zero cell), q = rint(x / f32(scale))."""
    B, H, N, D = x.shape
    nc = N // s
    xc = x[:, :, :nc * s].reshape(B, H, nc, s, D).float()
    sc = xc.abs().amax(dim=(3, 4)) / 127.0
    sc = torch.where(sc > 0, sc, torch.ones_like(sc)).to(torch.bfloat16)
    q = torch.round(xc / sc[:, :, :, None, None].float()).to(torch.int8)
    return q.reshape(B, H, nc * s, D).contiguous(), sc.contiguous()


def dequant_cells(q: torch.Tensor, sc: torch.Tensor, s: int, dtype=torch.bfloat16):
    """Inverse read of quantize_cells: dtype(f32(q) * f32(scale)); src/fsattn/kv_int8.py:63-71."""
    B, H, N, D = q.shape
    nc = N // s
    x = q.view(B, H, nc, s, D).float() * sc[:, :, :nc, None, None].float()
    return x.to(dtype).reshape(B, H, nc * s, D)


# ---------------------------------------------------------------------------------------------------------------
# FS-L candidate pool
# ---------------------------------------------------------------------------------------------------------------
def stable_topk(values: torch.Tensor, k: int) -> torch.Tensor:
    """Indices of the k largest along the last dim under the total order (value descending, index ascending): the
    order the reference defines for pool membership (src/fsattn/kv_bounded.py:7-10, src/fsattn/prefix_topp.py:6-12)."""
    return values.argsort(dim=-1, descending=True, stable=True)[..., :k]


def fsl_prefix_topp(ceil: torch.Tensor, s: int, Bq: int, nb: int, P: int) -> torch.Tensor:
    """For every query block n the top-P visible cells by ceiling; src/fsattn/attention.py:766-778 with the
    deterministic tie rule of prefix_topp.stable_topk_slots. A cell c is visible to block n iff (c+1)*s <= n*Bq.
    ceil (B,H,M) -> (B,H,nb,Pk) int64, Pk = min(P, M); unused slots hold -1."""
    B, H, M = ceil.shape
    Pk = min(P, M)
    out = torch.full((B, H, nb, Pk), -1, dtype=torch.int64)
    for n in range(nb):
        vis = min(M, (n * Bq) // s)
        if vis <= 0:
            continue
        k = min(Pk, vis)
        out[:, :, n, :k] = stable_topk(ceil[:, :, :vis], k)
    return out


def fsl_candidates(topp: torch.Tensor, blk_start: int, s: int, Wc: int):
    """Candidate slots of one block: the top-P list followed by the Wc newest visible cells hi, hi-1, ...;
    src/fsattn/attention.py:779-792 (prefill) and 1339-1357 (decode). Returns (cand_c, ok): the clamped cell id of
    every slot and whether the slot is valid, visible and the first occurrence of its cell.
    topp (..., Pk) int64 -> cand_c (..., Pk+Wc) int64, ok (..., Pk+Wc) bool."""
    hi = blk_start // s - 1
    near = hi - torch.arange(Wc, dtype=torch.int64)
    near = near.expand(*topp.shape[:-1], Wc)
    cand = torch.cat([topp, near], dim=-1)
    valid = cand >= 0
    cand_c = cand.clamp(min=0)
    vis = ((cand_c + 1) * s <= blk_start) & valid
    C = cand.shape[-1]
    tri = torch.tril(torch.ones(C, C, dtype=torch.bool), diagonal=-1)
    dup = ((cand_c[..., None, :] == cand_c[..., :, None]) & tri).any(dim=-1)
    return cand_c, vis & ~dup


def fsl_scores(q, kbar_cand, ceil_cand, cand_c, ok, qpos, lam, sigma, scale: float, s: int):
    """Selection score of queries against candidate slots; src/fsattn/attention.py:801-807:
    score = (q . kbar) * scale + lam * ceil * erf(|p - (c + 0.5) s| / (2 sigma)), NEG where the slot is not ok.
    q (B,H,Nq,D), kbar_cand (B,H,C,D) fp32, ceil_cand/cand_c/ok (B,H,C), qpos (Nq,) fp32, lam/sigma (H,)."""
    H = q.shape[1]
    content = torch.einsum("bhqd,bhcd->bhqc", q.float(), kbar_cand.float()) * scale
    cen = (cand_c.to(torch.float32) + 0.5) * s
    dist = (qpos.view(1, 1, -1, 1) - cen[:, :, None, :]).abs()
    erf = torch.erf(dist / (2.0 * sigma.float().view(1, H, 1, 1)))
    score = content + lam.float().view(1, H, 1, 1) * ceil_cand[:, :, None, :] * erf
    return score.masked_fill(~ok[:, :, None, :], NEG)


def _pick(score, cand_c, ok, kk):
    """top-kk by (score desc, slot asc); returns (cells (-1 for not-ok picks), margin): margin is the smallest gap
    between consecutive entries of the best kk+1 scores, i.e. how far the fp32 scores are from changing either the
    selected set or its order. Not-ok slots (score NEG) never count as close."""
    C = score.shape[-1]
    k = min(kk, C)
    order = score.argsort(dim=-1, descending=True, stable=True)
    top = order[..., :k]
    shape = score.shape
    cells = torch.gather(cand_c[:, :, None, :].expand(shape), -1, top)
    okp = torch.gather(ok[:, :, None, :].expand(shape), -1, top)
    sel = cells.to(torch.int32).masked_fill(~okp, -1)
    srt = torch.gather(score, -1, order[..., :min(k + 1, C)])
    gaps = srt[..., :-1] - srt[..., 1:]
    # a gap below a NEG entry (both not ok) says nothing about the selection: ignore it
    both_neg = srt[..., :-1] <= NEG / 2
    gaps = gaps.masked_fill(both_neg, float("inf"))
    margin = gaps.amin(dim=-1) if gaps.shape[-1] > 0 else torch.full(shape[:-1], float("inf"))
    return sel, margin


def fsl_select_prefill(Q, kbar, ceil, lam, sigma, scale: float, s: int, Bq: int, P: int, Wc: int, kk: int, N: int):
    """Selected cells of every prefill query (strict causal, pruned pool); src/fsattn/attention.py:675-822
    (_cell_score_On_chunked_strict with fs_fused_attn building sel_full).
    Returns sel_full (B,H,nb*Bq,kk_eff) int32 (-1 = nothing) and the per-query fp32 margin (B,H,nb*Bq)."""
    B, H, _, D = Q.shape
    M = (N + s - 1) // s
    kk = min(kk, M)
    Bq = min(Bq, N)
    nb = (N + Bq - 1) // Bq
    if kbar.shape[2] < M:       # a ragged last cell exists but is never visible: pad the statistics
        pad = M - kbar.shape[2]
        kbar = torch.cat([kbar, kbar.new_zeros(B, H, pad, D)], dim=2)
        ceil = torch.cat([ceil, ceil.new_zeros(B, H, pad)], dim=2)
    topp = fsl_prefix_topp(ceil, s, Bq, nb, P)
    sel_full = torch.full((B, H, nb * Bq, kk), -1, dtype=torch.int32)
    margin = torch.full((B, H, nb * Bq), float("inf"))
    for n in range(nb):
        blk_start = n * Bq
        cand_c, ok = fsl_candidates(topp[:, :, n], blk_start, s, Wc)
        C = cand_c.shape[-1]
        q = Q.new_zeros(B, H, Bq, D)
        n_real = max(0, min(blk_start + Bq, N) - blk_start)
        q[:, :, :n_real] = Q[:, :, blk_start:blk_start + n_real]
        kb = torch.gather(kbar, 2, cand_c[..., None].expand(B, H, C, D))
        cl = torch.gather(ceil, 2, cand_c)
        qpos = blk_start + torch.arange(Bq, dtype=torch.float32)
        score = fsl_scores(q, kb, cl, cand_c, ok, qpos, lam, sigma, scale, s)
        sel, mg = _pick(score, cand_c, ok, kk)
        sel_full[:, :, blk_start:blk_start + Bq] = sel
        margin[:, :, blk_start:blk_start + Bq] = mg
    return sel_full, margin


def fs_dense_select_prefill(Q, kbar, ceil, lam, sigma, scale: float, s: int, Bq: int, kk: int, N: int):
    """Selected cells of every prefill query of the dense FS variant (cell_prune_kernel = 0, strict causal): every
    completed cell that ends at or before the query's block start is a candidate, no pool; src/fsattn/attention.py:
    362-423 with _cell_select_blk_logits(per_query=True, topk_k=kk) (472-517) and _cell_sel_cells (339-342). The
    reference takes torch.topk over the logits, whose order among equal scores is unspecified: here (score desc, cell asc).
    Returns sel_full (B,H,nb*Bq,kk_eff) int32 (-1 = nothing) and the per-query fp32 margin (B,H,nb*Bq)."""
    B, H, _, D = Q.shape
    M = (N + s - 1) // s
    kk = min(kk, M)
    Bq = min(Bq, N)
    nb = (N + Bq - 1) // Bq
    if kbar.shape[2] < M:
        pad = M - kbar.shape[2]
        kbar = torch.cat([kbar, kbar.new_zeros(B, H, pad, D)], dim=2)
        ceil = torch.cat([ceil, ceil.new_zeros(B, H, pad)], dim=2)
    kbar, ceil = kbar[:, :, :M], ceil[:, :, :M]
    cells = torch.arange(M, dtype=torch.int64).expand(B, H, M)
    sel_full = torch.full((B, H, nb * Bq, kk), -1, dtype=torch.int32)
    margin = torch.full((B, H, nb * Bq), float("inf"))
    for n in range(nb):
        blk_start = n * Bq
        ok = ((cells + 1) * s <= blk_start)
        q = Q.new_zeros(B, H, Bq, D)
        n_real = max(0, min(blk_start + Bq, N) - blk_start)
        q[:, :, :n_real] = Q[:, :, blk_start:blk_start + n_real]
        qpos = blk_start + torch.arange(Bq, dtype=torch.float32)
        score = fsl_scores(q, kbar, ceil, cells, ok, qpos, lam, sigma, scale, s)
        sel, mg = _pick(score, cells, ok, kk)
        sel_full[:, :, blk_start:blk_start + Bq] = sel
        margin[:, :, blk_start:blk_start + Bq] = mg
    return sel_full, margin


def fs_dense_decode_select(q, kbar, ceil, pos: int, lam, sigma, scale: float, s: int, Bq: int, kk: int):
    """Selected cells of one decode query of the dense FS variant at position pos: all cells completed before the
    query's block start are scored; src/fsattn/attention.py:1159-1185 (_lr_decode_step_dense; torch.topk there, (score
    desc, cell asc) here). q (B,H,1,D), kbar (B,H,ncell,D), ceil (B,H,ncell). Returns (sel (B,H,1,kk) int32, -1 padded when
    fewer than kk cells are visible; margin (B,H,1))."""
    B, H, _, D = q.shape
    blk_start = (pos // Bq) * Bq
    M_vis = min(blk_start // s, ceil.shape[2])
    if M_vis <= 0:
        return torch.full((B, H, 1, kk), -1, dtype=torch.int32), torch.full((B, H, 1), float("inf"))
    cells = torch.arange(M_vis, dtype=torch.int64).expand(B, H, M_vis)
    ok = torch.ones(B, H, M_vis, dtype=torch.bool)
    score = fsl_scores(q, kbar[:, :, :M_vis], ceil[:, :, :M_vis], cells, ok, torch.tensor([float(pos)]), lam, sigma, scale, s)
    sel, mg = _pick(score, cells, ok, kk)
    if sel.shape[-1] < kk:
        sel = torch.cat([sel, sel.new_full((B, H, 1, kk - sel.shape[-1]), -1)], dim=-1)
    return sel, mg


def fsl_decode_pool(kbar, ceil, blk_start: int, s: int, P: int, Wc: int):
    """Candidate pool of the decode block starting at blk_start; src/fsattn/attention.py:1313-1360 with the
    (ceiling desc, index asc) tie rule. kbar (B,H,ncell,D), ceil (B,H,ncell). Returns None when nothing is visible."""
    ncell = ceil.shape[2]
    M_vis = min(blk_start // s, ncell)
    if M_vis <= 0:
        return None
    B, H, _, D = kbar.shape
    Pk = min(P, M_vis)
    topP = stable_topk(ceil[:, :, :M_vis], Pk)
    cand_c, ok = fsl_candidates(topP, blk_start, s, Wc)
    C = cand_c.shape[-1]
    return {
        "M_vis": M_vis, "C": C, "cand_c": cand_c, "ok_cell": ok,
        "Kbar_cand": torch.gather(kbar, 2, cand_c[..., None].expand(B, H, C, D)),
        "ceil_cand": torch.gather(ceil, 2, cand_c),
        "cen_cand": (cand_c.float() + 0.5) * s,
    }


def fsl_decode_select(q, pool, pos: int, lam, sigma, scale: float, s: int, kk: int):
    """The cells one decode query reads; src/fsattn/attention.py:1242-1272. q (B,H,1,D).
    Returns sel (B,H,1,kk_eff) int32 and margin (B,H,1); all -1 when the pool is empty."""
    B, H = q.shape[:2]
    if pool is None:
        return torch.full((B, H, 1, kk), -1, dtype=torch.int32), torch.full((B, H, 1), float("inf"))
    kk = min(kk, pool["M_vis"])
    qpos = torch.tensor([float(pos)])
    score = fsl_scores(q, pool["Kbar_cand"], pool["ceil_cand"], pool["cand_c"], pool["ok_cell"], qpos, lam, sigma,
                       scale, s)
    return _pick(score, pool["cand_c"], pool["ok_cell"], kk)


def bounded_keep_set(ceil, N: int, s: int, Bq: int, P: int, Wc: int, W: int):
    """Cells of a prompt of N tokens that the bounded store keeps after the prefill; src/fsattn/kv_bounded.py:110-135:
    the top-P of the cells visible to the first decode block and every cell from c_lo on.
    ceil (B,H,ncell) -> keep (B,H,ncell) bool."""
    B, H, ncell = ceil.shape
    blk = (N // Bq) * Bq
    m_vis = min(blk // s, ncell)
    keep = torch.zeros(B, H, ncell, dtype=torch.bool)
    c_lo = max(0, min((blk - W) // s, m_vis - Wc)) if m_vis > 0 else 0
    keep[:, :, c_lo:] = True
    if m_vis > 0:
        keep.scatter_(2, stable_topk(ceil[:, :, :m_vis], min(P, m_vis)), True)
    return keep


def bounded_readable_from(blk_start: int, m_vis: int, s: int, W: int, Wc: int) -> int:
    """Oldest cell a block reads outside its top-P; src/fsattn/kv_bounded.py:105-108."""
    return max(0, min((blk_start - W) // s, m_vis - Wc))


# ---------------------------------------------------------------------------------------------------------------
# readout + combine
# ---------------------------------------------------------------------------------------------------------------
def cell_readout(Q, K, V, sel, s: int, Bq: int, scale: float, q_pos0: int = 0, n_kv: int | None = None):
    """Softmax attention of every query over the tokens of its valid, distinct selected cells;
    src/fsattn/cell_select_triton.py:97-282 and src/fsattn/fsb_tree.py:2313-2339 (masked_readout).
    A selected cell counts when 0 <= c < ceil(n_kv/s), (c+1)*s <= block start of the query, and no earlier slot of the
    same query holds it; a token counts when tok < n_kv and tok < query position. Queries with no token give 0.
    Q (B,H,Nq,D); K,V (B,H,>=n_kv,D); sel (B,H,>=Nq,kk). Returns fp32 (B,H,Nq,D)."""
    B, H, Nq, D = Q.shape
    n_kv = K.shape[2] if n_kv is None else n_kv
    n_cells = (n_kv + s - 1) // s
    kk = sel.shape[-1]
    out = torch.zeros(B, H, Nq, D)
    Kf, Vf, Qf = K.float(), V.float(), Q.float()
    off = torch.arange(s)
    for i in range(Nq):
        qp = q_pos0 + i
        bs = (qp // Bq) * Bq
        cells = sel[:, :, i, :].long()                                       # (B,H,kk)
        ok = (cells >= 0) & (cells < n_cells) & ((cells + 1) * s <= bs)
        for a in range(kk):
            for b_ in range(a):
                ok[..., a] &= ~(ok[..., b_] & (cells[..., b_] == cells[..., a]))
        tok = cells.clamp(min=0)[..., None] * s + off                        # (B,H,kk,s)
        tok_ok = ok[..., None] & (tok < n_kv) & (tok < qp)
        tok = tok.clamp(max=K.shape[2] - 1).reshape(B, H, kk * s)
        tok_ok = tok_ok.reshape(B, H, kk * s)
        kc = torch.gather(Kf, 2, tok[..., None].expand(B, H, kk * s, D))
        vc = torch.gather(Vf, 2, tok[..., None].expand(B, H, kk * s, D))
        sc = torch.einsum("bhd,bhkd->bhk", Qf[:, :, i], kc) * scale
        sc = sc.masked_fill(~tok_ok, float("-inf"))
        any_ok = tok_ok.any(-1, keepdim=True)
        w = torch.softmax(sc.masked_fill(~any_ok, 0.0), dim=-1) * any_ok
        out[:, :, i] = torch.einsum("bhk,bhkd->bhd", w, vc)
    return out


def lr_norm_combine(sr, o, norm_w, lrs, eps: float, act_dtype=torch.bfloat16):
    """W_o's input from the window output and the long-range readout; src/fsattn/attention.py:57-65, 321-327 and
    src/fsattn/readout_triton.py:94-105: o is rounded to the activation dtype, lr = (o * rsqrt(mean(o^2) + eps)) * w,
    y = act_dtype(sr + lrs_h * lr) laid out (B, N, H*D).
    sr, o (B,H,N,D); norm_w (D,); lrs (H,) or (H,1,1)."""
    B, H, N, D = o.shape
    ob = o.to(act_dtype).float()
    r = torch.rsqrt(ob.pow(2).mean(-1, keepdim=True) + eps)
    lr = (ob * r) * norm_w.float()
    y = sr.float() + lrs.float().view(1, H, 1, 1) * lr
    return y.to(act_dtype).transpose(1, 2).reshape(B, N, H * D)


# ---------------------------------------------------------------------------------------------------------------
# window branch
# ---------------------------------------------------------------------------------------------------------------
def rope_inv_freq(D: int, orig_len: int, base: float = 10000.0, beta_fast: float = 32.0, beta_slow: float = 1.0):
    """RoPE frequencies as the reference builds them with YaRN scale 1; experiments/scaling/yarn_rope.py:8-58: the
    interpolated and extrapolated frequencies coincide, but they are still blended through the ramp mask, which
    moves some entries by an ulp, so the blend is restated here."""
    a = 1.0 / (base ** (torch.arange(0, D, 2, dtype=torch.float32) / D))

    def corr(rot):
        return (D * math.log(orig_len / (rot * 2 * math.pi))) / (2 * math.log(base))
    low = max(math.floor(corr(beta_fast)), 0)
    high = min(math.ceil(corr(beta_slow)), D - 1)
    hi = high + 0.001 if low == high else high
    ramp = ((torch.arange(D // 2, dtype=torch.float32) - low) / (hi - low)).clamp(0.0, 1.0)
    m = 1.0 - ramp
    return a * (1.0 - m) + a * m


def rope_tables(D: int, L: int, dtype=torch.float32, base: float = 10000.0, orig_len: int | None = None):
    """cos/sin tables (L, D), both halves equal; experiments/scaling/yarn_rope.py:97-121 (YaRN scale 1): built in
    fp32, then cast with the module. orig_len is the max_seq_len the module was constructed with."""
    inv_freq = rope_inv_freq(D, L if orig_len is None else orig_len, base)
    t = torch.arange(L, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def apply_rope(x, cos, sin):
    """Rotate-half RoPE; src/fsattn/attention.py:14-19. x (B,H,n,D), cos/sin (n,D) rows of the absolute positions."""
    d = x.shape[-1] // 2
    x1, x2 = x[..., :d], x[..., d:]
    c = cos[:, :d][None, None]
    sn = sin[:, :d][None, None]
    return torch.cat([x1 * c - x2 * sn, x2 * c + x1 * sn], dim=-1)


def window_attention(Q, K, V, cos, sin, W: int, scale: float, q_pos0: int = 0, k_pos0: int = 0,
                     act_dtype=None, p_dtype=None):
    """Causal sliding-window softmax attention with RoPE on Q and K only; src/utils/local_attention.py:317-353
    (generic loop, uniform window) and src/fsattn/attention.py:225-231. Query at absolute position p attends keys
    max(0, p - W) <= j <= p. The rotated Q and K are rounded to act_dtype (the dtype they are stored in before the
    score product) when it is given. Q (B,H,Nq,D) at positions q_pos0.., K/V (B,H,Nk,D) at positions k_pos0...
    p_dtype: when given, the softmax weights are rounded to it before they multiply V, as the reference's low-precision
    path does (`w = torch.softmax(scores, dim=-1).to(Vw.dtype)`, src/fsattn/attention.py:1155; SDPA's bf16 kernels do the
    same with their probabilities). Returns fp32 (B,H,Nq,D)."""
    B, H, Nq, D = Q.shape
    Nk = K.shape[2]
    cf, sf = cos.float(), sin.float()
    qr = apply_rope(Q.float(), cf[q_pos0:q_pos0 + Nq], sf[q_pos0:q_pos0 + Nq])
    kr = apply_rope(K.float(), cf[k_pos0:k_pos0 + Nk], sf[k_pos0:k_pos0 + Nk])
    if act_dtype is not None:
        qr, kr = qr.to(act_dtype).float(), kr.to(act_dtype).float()
    out = torch.empty(B, H, Nq, D)
    Vf = V.float()
    CH = 256
    for c0 in range(0, Nq, CH):
        c1 = min(c0 + CH, Nq)
        p0, p1 = q_pos0 + c0, q_pos0 + c1
        j0 = max(k_pos0, p0 - W)
        j1 = p1
        ks = kr[:, :, j0 - k_pos0:j1 - k_pos0]
        sc = torch.einsum("bhqd,bhkd->bhqk", qr[:, :, c0:c1], ks) * scale
        qi = torch.arange(p0, p1)[:, None]
        kj = torch.arange(j0, j1)[None, :]
        band = (qi - kj >= 0) & (qi - kj <= W)
        sc = sc.masked_fill(~band, float("-inf"))
        wts = torch.softmax(sc, -1)
        if p_dtype is not None:
            wts = wts.to(p_dtype).float()
        out[:, :, c0:c1] = torch.einsum("bhqk,bhkd->bhqd", wts, Vf[:, :, j0 - k_pos0:j1 - k_pos0])
    return out


# ---------------------------------------------------------------------------------------------------------------
# one FS-L attention layer, prefill + decode, composed from the pieces above (the semantic model of FSAttn)
# ---------------------------------------------------------------------------------------------------------------
class FSLLayerOracle:
    """Functional model of one FS-L attention layer behind the FSAttn / FSKVCache boundary
    (src/fsattn/attention.py:936-1131, experiments/scaling/kv_cache.py:179-272,384-392) for checking the CUDA path:
    prefill over N tokens, then token-by-token decode. Keeps the full K/V history (optionally through the int8
    codec, whose reads equal the bounded store's by construction, src/fsattn/kv_bounded.py:26-28)."""

    def __init__(self, H: int, D: int, *, s=32, Bq=128, kk=4, W=512, P=64, Wc=8, lam=None, sigma=None, lrs=None,
                 norm_w=None, eps=1e-8, act_dtype=torch.bfloat16, int8=False, rope_len=1 << 16, rope_orig_len=None):
        self.H, self.D, self.s, self.Bq, self.kk, self.W, self.P, self.Wc = H, D, s, Bq, kk, W, P, Wc
        self.scale = 1.0 / math.sqrt(D)
        self.lam = torch.ones(H) if lam is None else lam.float()
        self.sigma = torch.full((H,), 4.0) if sigma is None else sigma.float()
        self.lrs = torch.full((H,), 0.1) if lrs is None else lrs.float().reshape(H)
        self.norm_w = torch.ones(D) if norm_w is None else norm_w.float()
        self.eps, self.act, self.int8 = eps, act_dtype, int8
        self.cos, self.sin = rope_tables(D, rope_len, act_dtype, orig_len=rope_orig_len)
        self.K = self.V = None
        self.pos = 0

    def _kv_read(self):
        """K/V as a decode step reads them with the int8 store: cells completed BEFORE the current token through the
        codec, the open cell (which includes the current token, even when it is the cell's last) raw. This is the
        graph decoder's order: the step reads, then the bookkeeping closes the cell
        (experiments/scaling/decode_graph.py:223-241, 261-289)."""
        if not self.int8:
            return self.K, self.V
        n_q = ((self.K.shape[2] - 1) // self.s) * self.s
        out = []
        for x in (self.K, self.V):
            q, sc = quantize_cells(x[:, :, :n_q], self.s)
            out.append(torch.cat([dequant_cells(q, sc, self.s, x.dtype), x[:, :, n_q:]], dim=2))
        return out

    def prefill(self, Q, K, V):
        """Q,K,V (B,H,N,D) un-rotated. Returns (y (B,N,H*D), sel_full, margin)."""
        B, H, N, D = Q.shape
        sr = window_attention(Q, K, V, self.cos, self.sin, self.W, self.scale, act_dtype=self.act).to(self.act)
        kbar, ceil = cell_stats(K, self.s)
        sel, margin = fsl_select_prefill(Q, kbar, ceil, self.lam, self.sigma, self.scale, self.s, self.Bq, self.P,
                                         self.Wc, self.kk, N)
        o = cell_readout(Q, K, V, sel, self.s, min(self.Bq, N), self.scale, 0, N)
        y = lr_norm_combine(sr, o, self.norm_w, self.lrs, self.eps, self.act)
        self.K, self.V, self.pos = K.clone(), V.clone(), N
        return y, sel[:, :, :N], margin[:, :, :N]

    def decode(self, q, k, v):
        """One token: q,k,v (B,H,1,D). Returns (y (B,1,H*D), sel (B,H,1,kk), margin)."""
        pos = self.pos
        self.K = torch.cat([self.K, k], dim=2) if self.K is not None else k.clone()
        self.V = torch.cat([self.V, v], dim=2) if self.V is not None else v.clone()
        # statistics always come from the un-quantised keys (src/fsattn/kv_int8.py:7-8)
        kbar, ceil = cell_stats(self.K, self.s)
        Kr, Vr = self._kv_read()
        j0 = max(0, pos - self.W)
        sr = window_attention(q, Kr[:, :, j0:pos + 1], Vr[:, :, j0:pos + 1], self.cos, self.sin, self.W, self.scale,
                              q_pos0=pos, k_pos0=j0, act_dtype=self.act).to(self.act)
        blk_start = (pos // self.Bq) * self.Bq
        pool = fsl_decode_pool(kbar, ceil, blk_start, self.s, self.P, self.Wc) if kbar.shape[2] > 0 else None
        sel, margin = fsl_decode_select(q, pool, pos, self.lam, self.sigma, self.scale, self.s, self.kk)
        o = cell_readout(q, Kr, Vr, sel, self.s, self.Bq, self.scale, pos, pos + 1)
        y = lr_norm_combine(sr, o, self.norm_w, self.lrs, self.eps, self.act)
        self.pos = pos + 1
        return y, sel, margin
