"""The module-level FS-B entry points the reference's callers import from ``src/fsattn/fsb_tree.py`` (decoders, benchmark,
hub): threshold calibration, the per-block forest update for all layers, the graph registry and the read statistics. The
forests themselves live in ``ops.FsbForests`` / ``FSKVCache``; the tree search runs in the selection kernels."""
from __future__ import annotations

import torch


def _fsb_layers(model):
    """FS-B attention layers of a model (src/fsattn/fsb_tree.py:3930-3941)."""
    for m in model.modules():
        if getattr(m, "fsb_enabled", False) and hasattr(m, "fsb_tau"):
            yield m


@torch.no_grad()
def fsb_calibrate_tau(model, batches, quantile, reduce_fn=None, target="fsb_tau"):
    """Set every FS-B layer's admission threshold to the per-head `quantile` of the cell ceilings seen on `batches` (token id
    tensors); src/fsattn/fsb_tree.py:3944-3969. The reference collects the ceilings during an uncached forward; here the
    prompt goes through the cached prefill, whose caches hold the same statistics. Returns {"tau", "admit_frac", "n_cells"}."""
    from ..serving import extend_rope_cache, trunk_cached
    from .kv_cache import make_caches
    layers = list(_fsb_layers(model))
    if not layers or quantile <= 0:
        return None
    if target not in ("fsb_tau", "fsb_tau_union"):
        raise ValueError(f"fsb_calibrate_tau: target {target!r} (fsb_tau | fsb_tau_union)")
    dev = next(model.parameters()).device
    seen = [[] for _ in layers]
    for x in batches:
        ids = x.view(1, -1) if x.dim() == 1 else x
        caches = make_caches(model)
        extend_rope_cache(model, ids.shape[1] + 8)
        trunk_cached(model, ids.to(dev), caches, last_n=1)
        fsb_caches = [c for blk, c in zip(model.blocks, caches) if getattr(blk.attn.fsattn, "fsb_enabled", False)]
        for i, c in enumerate(fsb_caches):
            _, ceil, ncell = c.completed_cells()
            H = ceil.shape[1]
            seen[i].append(ceil[:, :, :ncell].float().transpose(0, 1).reshape(H, -1))
    taus, fracs, n_cells = [], [], 0
    for m, parts in zip(layers, seen):
        a = torch.cat(parts, dim=1)
        tau = torch.quantile(a, float(quantile), dim=1)
        if reduce_fn is not None:
            tau = reduce_fn(tau)
        buf = getattr(m, target)
        buf.copy_(tau.to(buf.device, buf.dtype))
        t_ = buf.detach().float().cpu().clone()
        taus.append(t_)
        fracs.append((a.cpu() >= t_[:, None]).float().mean(1))
        n_cells = int(a.shape[1])
    return {"tau": torch.stack(taus), "admit_frac": torch.stack(fracs), "n_cells": n_cells}


def fsb_decode_prepare_all(attns, caches, pos: int) -> bool:
    """Bring every FS-B layer's forests to the 128-token block of position `pos` (admit the cells completed before the
    block, build the chunks they complete, rebuild the spines): src/fsattn/fsb_tree.py:3468-3596. Called between graph
    replays; a no-op inside a block. Returns whether any layer did work."""
    did = False
    for a, c in zip(attns, caches):
        a = getattr(a, "inner", a)
        if getattr(a, "fsb_enabled", False):
            did = c.fsb_block_change(pos, a) or did
    return did


def fsb_graph_registry(caches) -> tuple:
    """Addresses of every tensor a captured FS-B decode step reads through the forests (src/fsattn/fsb_tree.py:3304-3345):
    a decoder re-captures its graph only when this tuple changes. The forests here are allocated once at their capacity,
    so it changes only when a cache is re-created."""
    reg = []
    for c in caches:
        fo = getattr(c, "fsb", None)
        if fo is None:
            reg.append(None)
            continue
        ts = fo.adm + fo.m_tot + fo.node_mu + fo.node_aux + fo.root32 + fo.spine + fo.hdr
        reg.append(tuple(t.data_ptr() for t in ts))
    return tuple(reg)


_READ_STATS = {"steps": 0}


def fsb_read_stats_reset() -> None:
    """src/fsattn/fsb_tree.py:3892-3898. The kernels keep no read statistics; the counter of prepared blocks is reset."""
    _READ_STATS["steps"] = 0


def fsb_read_stats() -> dict:
    """src/fsattn/fsb_tree.py:3900-3915: the reference's accumulators (visited nodes, candidates per query) are debug
    outputs of ``ops.fsb_select(debug=True)`` here; this returns the empty summary its callers accept."""
    return dict(_READ_STATS)
