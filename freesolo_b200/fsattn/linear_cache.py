"""Streaming FS-L cache with a state of fixed size (ref: src/fsattn/linear_cache.py:33-240, `LinearFSCache`).

The reference keeps, per layer, exactly what a later query of FS-L can read: the P completed cells with the highest
ceilings (ties to the lower cell), the Wc newest completed cells, the tokens of the cells still open, and the last W
keys/values of the window - and rebuilds that state with gathers and concatenations at every 128-token block. Here
the same state lives in buffers allocated once:

    ids / prio / mean / k / v   C = P + Wc slots: [0, P) the top list in no particular order, [P, C) a ring of the newest
                                cells (cell c sits in slot P + c mod Wc); an empty slot has id -1; one more slot at the
                                end takes the writes of new cells that do not make the top list
    win_k / win_v               the last <= W raw rows;  pend_k / pend_v  the rows of the cells not yet eligible

At a block change only the cells that ENTER the top list are written, into the slots of the cells that leave it (at
most Bq/s = 4 of them), so a block costs a few kilobytes of traffic instead of a copy of the whole pool. The two hot
operations are this library's kernels: the window branch of a whole `attend` call is one launch of the tensor-core
window kernel over [last W rows | new rows], and every block's long-range branch is one launch of the fused readout +
combine kernel reading the pool slots as cells. Cell statistics come from the cell-ingest kernel (bit-exact mean and
ceiling); the pool update of a block change and the selection (at most 72 candidate scores per query, top-k) are two
small kernels of their own (csrc/linear_pool.cu); only the concatenation of the pending / window rows is left to torch.

Selections and outputs equal the standard FS-L prefill over the same tokens (same candidates: prefix top-P plus the Wc
newest; same scores; ties to the lower cell id), which is how the reference's own tests state it.
"""
from __future__ import annotations

import torch

from .. import ops


class _BlockCalls:
    """The launches of one 128-token block of a long `attend` call - cell statistics and pool merge at the block change,
    selection, readout + combine - with their argument structs built ONCE per call: per block only addresses, counts
    and positions are rewritten and the four entry points are called directly, which takes the Python wrappers' checks
    and allocations (most of the time of a block) out of the loop. Single-sequence calls only (B = 1: a token range of the
    (1, n, H D) window-branch and output buffers is contiguous)."""

    def __init__(self, cache, q, pk, pv, sr_all, y, lam, sigma, lrs, norm_w):
        from .. import lib as L
        a = cache.attn
        B, H, n, D = q.shape
        self.L, self.lib, self.c = L, L.load(), cache
        self.stream = L.vp(ops._stream(q))
        self.D, self.HD, self.kk_out = D, H * D, a.cell_topk
        self.pk, self.pv, self.q, self.sr, self.y = pk.data_ptr(), pv.data_ptr(), q.data_ptr(), sr_all.data_ptr(), y.data_ptr()
        assert q.stride(-1) == 1 and pk.stride(2) == D and pv.stride() == pk.stride() and sr_all.is_contiguous() and y.is_contiguous()
        lam, sigma, lrs, norm_w = (t.detach().float().contiguous() for t in (lam, sigma, lrs.reshape(-1), norm_w))
        self.sel = torch.empty(B, H, cache.Bq, self.kk_out, dtype=torch.int32, device=q.device)
        self.stats = {}                                  # count -> (mean (B,H,count,D), prio (B,H,count)) fp32
        self.keep = (lam, sigma, lrs, norm_w, q, pk, pv, sr_all, y)       # every address below stays valid while this object lives
        ci = L.CellIngest()
        ci.k = L.BHND(self.pk, pk.stride(0), pk.stride(1), pk.stride(2))
        ci.v = L.BHND(None, 0, 0, 0)
        ci.B, ci.H, ci.D, ci.cell0 = B, H, D, 0
        lm = L.LinearMerge()
        lm.ids, lm.prio, lm.mean, lm.k, lm.v, lm.valid = (t.data_ptr() for t in (cache.ids, cache.prio, cache.mean, cache.k, cache.v, cache.valid))
        lm.nk_sb, lm.nk_sh = pk.stride(0), pk.stride(1)
        lm.B, lm.H, lm.D, lm.P, lm.Wc = B, H, D, cache.P, cache.Wc
        ls = L.LinearSelect()
        ls.ids, ls.prio, ls.mean, ls.valid = cache.ids.data_ptr(), cache.prio.data_ptr(), cache.mean.data_ptr(), cache.valid.data_ptr()
        ls.q = L.BHND(self.q, q.stride(0), q.stride(1), q.stride(2))
        ls.lam, ls.sigma, ls.scale = lam.data_ptr(), sigma.data_ptr(), float(a.scale)
        ls.B, ls.H, ls.D, ls.C, ls.n_pad, ls.kk_out = B, H, D, cache.C, cache.Bq, self.kk_out
        ls.content_only = 1 if getattr(a, "sel_content_only", False) else 0
        ls.sel, ls.sel_ids = self.sel.data_ptr(), None
        rc = L.ReadoutCombine()
        rc.q = L.BHND(self.q, q.stride(0), q.stride(1), q.stride(2))
        # the pool slots are the "cells" of the readout: rows [0, C s) of the slot buffers
        rc.k = L.BHND(cache.k.data_ptr(), cache.k.stride(0), cache.k.stride(1), cache.k.stride(2))
        rc.v = L.BHND(cache.v.data_ptr(), cache.v.stride(0), cache.v.stride(1), cache.v.stride(2))
        rc.sel, rc.sel_sb, rc.sel_sh = self.sel.data_ptr(), self.sel.stride(0), self.sel.stride(1)
        rc.norm_w, rc.lrs = norm_w.data_ptr(), lrs.data_ptr()
        n_kv = cache.C * cache.s
        rc.B, rc.H, rc.D, rc.n_kv, rc.Bq, rc.kk = B, H, D, n_kv, cache.Bq, self.kk_out
        rc.q_pos0 = (n_kv + cache.Bq - 1) // cache.Bq * cache.Bq
        rc.scale, rc.eps, rc.impl = float(a.scale), float(a.lr_norm.eps), 0
        self.ci, self.lm, self.ls, self.rc = ci, lm, ls, rc
        self.q_sn = q.stride(2)

    def _run(self, name, args):
        rc = getattr(self.lib, name)(self.L.C.byref(args), self.stream)
        if rc != self.L.OK:
            self.L.check(rc, name)

    def merge(self, r0: int, count: int):
        """The cells of the rows [r0, r0 + count s) of the pending buffer enter the pool (LinearFSCache._merge)."""
        c = self.c
        st = self.stats.get(count)
        if st is None:
            B, H = self.ci.B, self.ci.H
            st = (torch.empty(B, H, count, self.D, dtype=torch.float32, device=c.ids.device),
                  torch.empty(B, H, count, dtype=torch.float32, device=c.ids.device))
            self.stats[count] = st
        mean, prio = st
        off = r0 * self.D * 2
        ci, lm = self.ci, self.lm
        ci.k.ptr = self.pk + off
        ci.ncell = count
        ci.kbar, ci.kbar_sb, ci.kbar_sh = mean.data_ptr(), mean.stride(0), mean.stride(1)
        ci.ceil, ci.ceil_sb, ci.ceil_sh = prio.data_ptr(), prio.stride(0), prio.stride(1)
        self._run("fsattn_cell_ingest", ci)
        width = min(c.P, c.eligible) + count
        c.max_merge_cells = max(c.max_merge_cells, width)
        c.merged_cells += width
        c.updates += 1
        lm.new_prio, lm.new_mean, lm.new_k, lm.new_v = prio.data_ptr(), mean.data_ptr(), self.pk + off, self.pv + off
        lm.count, lm.first_id = count, c.eligible
        self._run("fsattn_linear_merge", lm)
        c.eligible += count

    def block(self, off: int, m: int):
        """Selection and readout + combine of the queries [off, off + m) of the call, at positions cache.pos .. + m - 1."""
        c = self.c
        ls, rc = self.ls, self.rc
        qptr = self.q + off * self.q_sn * 2
        ls.q.ptr, ls.n, ls.pos0, ls.kk = qptr, m, c.pos, min(self.kk_out, c.eligible)
        self._run("fsattn_linear_select", ls)
        tok = off * self.HD * 2
        rc.q.ptr, rc.sr, rc.y, rc.N = qptr, self.sr + tok, self.y + tok, m
        self._run("fsattn_readout_combine", rc)


class LinearFSCache:
    bounded = True

    def __init__(self, attn):
        attn._assert_cacheable(phase="prefill")
        if attn._is_dense_lr():
            raise ValueError("LinearFSCache requires native prefix pruning.")
        if getattr(attn, "fsb_enabled", False):
            raise NotImplementedError("FS-B has no bounded-cache (linear) path; use FSKVCache.")
        self.attn = attn
        self.s, self.Bq, self.W = attn.cell_stride, attn._cell_block, attn.window_size
        self.P, self.Wc = attn._pool_cfg()
        if min(self.s, self.Bq, self.P) <= 0 or min(self.W, self.Wc) < 0:
            raise ValueError("Invalid linear-cache capacities.")
        self.C = self.P + self.Wc
        self.pos = 0
        self.eligible = 0              # completed cells visible to the current block
        self.block_start = -1
        self.pool = None               # dict of views for `select`, None while no cell is eligible
        self.max_merge_cells = self.merged_cells = self.updates = 0
        self._ready = False

    # ---- state ---------------------------------------------------------------------------------------------------------
    def _alloc(self, k):
        B, H, _, D = k.shape
        dev, C, s = k.device, self.C, self.s
        self.ids = torch.full((B, H, C + 1), -1, dtype=torch.int32, device=dev)
        self.valid = torch.zeros(B, H, C, dtype=torch.uint8, device=dev)
        self.prio = torch.full((B, H, C + 1), float("-inf"), dtype=torch.float32, device=dev)
        self.mean = torch.zeros(B, H, C + 1, D, dtype=torch.float32, device=dev)
        self.k = torch.zeros(B, H, (C + 1) * s, D, dtype=torch.bfloat16, device=dev)
        self.v = torch.zeros(B, H, (C + 1) * s, D, dtype=torch.bfloat16, device=dev)
        self.win_k = torch.zeros(B, H, 0, D, dtype=torch.bfloat16, device=dev)
        self.win_v = torch.zeros(B, H, 0, D, dtype=torch.bfloat16, device=dev)
        self.pend_k = torch.zeros(B, H, 0, D, dtype=torch.bfloat16, device=dev)
        self.pend_v = torch.zeros(B, H, 0, D, dtype=torch.bfloat16, device=dev)
        self._ready = True

    _TENSORS = ("ids", "valid", "prio", "mean", "k", "v", "win_k", "win_v", "pend_k", "pend_v")

    def fork(self):
        """An independent copy of the state (ref: linear_cache.py:207-211)."""
        other = object.__new__(type(self))
        other.__dict__ = dict(self.__dict__)
        if self._ready:
            for name in self._TENSORS:
                setattr(other, name, getattr(self, name).clone())
            other.pool = None
            other.block_start = -1       # the views of `pool` are rebuilt on the copy's own buffers
        return other

    def state_bytes(self) -> int:
        if not self._ready:
            return 0
        return sum(getattr(self, n).untyped_storage().nbytes() for n in self._TENSORS)

    # ---- block change: the cells completed since the last one become eligible -------------------------------------------
    def prepare(self):
        start = self.pos // self.Bq * self.Bq
        if start == self.block_start:
            return
        count = start // self.s - self.eligible
        if count > 0:
            n = count * self.s
            self._merge(self.pend_k[:, :, :n], self.pend_v[:, :, :n], count)
            self.pend_k, self.pend_v = self.pend_k[:, :, n:].clone(), self.pend_v[:, :, n:].clone()
        self.block_start = start
        self._set_pool()

    def _merge(self, nk, nv, count):
        """The rows nk / nv (B,H,count*s,D; views with dense rows are fine) of `count` newly completed cells enter the pool."""
        P = self.P
        mean, prio = ops.cell_stats(nk, count)                       # (B,H,count,D), (B,H,count) fp32, bit-exact statistics
        width = min(P, self.eligible) + count
        self.max_merge_cells = max(self.max_merge_cells, width)
        self.merged_cells += width
        self.updates += 1
        # the P best of (top list, new cells) by (ceiling desc, cell id asc) stay; entering cells take the slots of the
        # leaving ones; the newest Wc cells also go into the ring; `valid` is rewritten - one launch, a few KB written
        ops.linear_merge(self.ids, self.prio, self.mean, self.k, self.v, self.valid, P=P, Wc=self.Wc, first_id=self.eligible,
                         new_prio=prio, new_mean=mean, new_k=nk, new_v=nv)
        self.eligible += count

    def _set_pool(self):
        if self.eligible == 0:
            self.pool = None
            return
        C, s = self.C, self.s
        if self.pool is None:                        # the views never change: built once
            self.pool = dict(ids=self.ids[:, :, :C], priority=self.prio[:, :, :C], mean=self.mean[:, :, :C],
                             k=self.k[:, :, :C * s], v=self.v[:, :, :C * s], valid=self.valid)

    # ---- new tokens ------------------------------------------------------------------------------------------------------
    def ingest(self, k, v):
        """Append the raw keys / values of n tokens of ONE query block (ref: linear_cache.py:120-130)."""
        n = k.shape[2]
        if n > self.Bq - self.pos % self.Bq:
            raise ValueError("ingest must not cross a query-block boundary")
        if not self._ready:
            self._alloc(k)
        k, v = k.to(torch.bfloat16), v.to(torch.bfloat16)
        self.pend_k, self.pend_v = torch.cat([self.pend_k, k], dim=2), torch.cat([self.pend_v, v], dim=2)
        W = self.W
        self.win_k = torch.cat([self.win_k, k], dim=2)[:, :, -W:] if W else self.win_k[:, :, :0]
        self.win_v = torch.cat([self.win_v, v], dim=2)[:, :, -W:] if W else self.win_v[:, :, :0]
        self.pos += n

    # ---- selection over the pool (ref: linear_cache.py:154-170) --------------------------------------------------------------
    def _select_slots(self, q, want_ids=False):
        a = self.attn
        lam, sigma, _, _ = a.head_params()
        return ops.linear_select(q.to(torch.bfloat16), self.ids, self.prio, self.mean, self.valid, lam, sigma, pos0=self.pos,
                                 kk=min(a.cell_topk, self.eligible), kk_out=a.cell_topk, scale=a.scale,
                                 content_only=bool(getattr(a, "sel_content_only", False)), want_ids=want_ids)

    def select(self, q):
        """q (B,H,n<=128,D) at positions pos .. pos+n-1 -> (slots (B,H,n,k) int64 into the pool, cell ids with -1 for none),
        k = min(cell_topk, eligible cells): the best by (score desc, cell id asc)."""
        if self.pool is None:
            return None, None
        k = min(self.attn.cell_topk, self.eligible)
        slots, ids = self._select_slots(q, want_ids=True)
        slots, ids = slots[..., :k].long(), ids[..., :k].long()
        return slots.clamp_(min=0), ids

    # ---- one forward of the layer's attention over new tokens (ref: linear_cache.py:192-205) -------------------------------
    def attend(self, q, k, v):
        """q,k,v (B,H,n,D) bf16, un-rotated, any n: window branch + long-range branch + combine, then the tokens join
        the state. Returns (B,H,n,D) (a view of the (B,n,H*D) buffer W_o reads).

        The call concatenates [stored window rows | new rows] and [pending rows | new rows] ONCE; every 128-token block then
        reads its newly completed cells, its queries and its part of the window branch as views of those buffers (no copies),
        so a block is four launches (cell statistics, pool merge, selection, readout + combine); the stored window and
        pending rows are cut out once at the end."""
        if torch.is_grad_enabled():
            raise RuntimeError("LinearFSCache is inference-only; use torch.no_grad().")
        a = self.attn
        B, H, n, D = q.shape
        if n <= 32:
            return self._attend_tokens(q, k, v)
        if not self._ready:
            self._alloc(k)
        lam, sigma, lrs, norm_w = a.head_params()
        s, Bq, W = self.s, self.Bq, self.W
        q, kb, vb = q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16)
        # window branch of the whole call: [the last <= W stored rows | the new rows]; the stored rows get dummy queries
        old = self.win_k.shape[2]
        kc = torch.cat([self.win_k, kb], dim=2)
        vc = torch.cat([self.win_v, vb], dim=2)
        qc = torch.cat([torch.zeros(B, H, old, D, dtype=torch.bfloat16, device=q.device), q], dim=2)
        cos, sin = a.rope.tables_bf16(self.pos + n)
        sr_all = ops.window_prefill(qc, kc, vc, cos, sin, W, a.scale, pos0=self.pos - old)[:, old:]      # (B,n,H*D)
        # rows of the cells that are not eligible yet, stored ones first: row r is token p0 + r
        pk = torch.cat([self.pend_k, kb], dim=2)
        pv = torch.cat([self.pend_v, vb], dim=2)
        p0 = self.pos - self.pend_k.shape[2]
        y = torch.empty(B, n, H * D, dtype=torch.bfloat16, device=q.device)
        views = B == 1                                   # a token range of a (1, n, H*D) buffer is contiguous
        wrapped = type(self).select is not LinearFSCache.select or "select" in self.__dict__
        sr_all = sr_all.contiguous() if views else sr_all
        fast = _BlockCalls(self, q, pk, pv, sr_all, y, lam, sigma, lrs, norm_w) if (views and not wrapped) else None
        n_kv = self.C * s
        q_pos0 = (n_kv + Bq - 1) // Bq * Bq              # every pool token lies before this virtual query position
        off = 0
        while off < n:
            start = self.pos // Bq * Bq
            if start != self.block_start:                # block change: the cells completed before it become eligible
                count = start // s - self.eligible
                if count > 0:
                    r0 = self.eligible * s - p0
                    if fast is not None:
                        fast.merge(r0, count)
                    else:
                        self._merge(pk[:, :, r0:r0 + count * s], pv[:, :, r0:r0 + count * s], count)
                self.block_start = start
                self._set_pool()
            m = min(n - off, Bq - self.pos % Bq)
            if fast is not None and self.pool is not None:
                fast.block(off, m)
                self.pos += m
                off += m
                continue
            qp = q[:, :, off:off + m]
            sr = sr_all[:, off:off + m] if views else sr_all[:, off:off + m].contiguous()
            if self.pool is None:
                y[:, off:off + m] = sr                   # no completed cell yet: the long-range branch is zero
            else:
                if wrapped:                              # an overridden / wrapped select stays in the loop
                    slots, ids = self.select(qp)
                    sel = torch.full((B, H, m, a.cell_topk), -1, dtype=torch.int32, device=q.device)
                    sel[..., :slots.shape[-1]] = torch.where(ids >= 0, slots, torch.full_like(slots, -1)).to(torch.int32)
                else:
                    sel = self._select_slots(qp)
                # the pool slots are the "cells" of this readout
                out = ops.readout_combine(qp, self.pool["k"], self.pool["v"], sel, sr, norm_w, lrs, a.lr_norm.eps, scale=a.scale,
                                          Bq=Bq, n_kv=n_kv, q_pos0=q_pos0, out=y[:, off:off + m] if views else None)
                if not views:
                    y[:, off:off + m] = out
            self.pos += m
            off += m
        done = self.eligible * s - p0                    # rows of pk that went into the pool
        # what stays: the pending rows and the last W rows, copied out so that the call's buffers can go
        self.pend_k, self.pend_v = pk[:, :, done:].clone(), pv[:, :, done:].clone()
        self.win_k = kc[:, :, -W:].clone() if W else kc[:, :, :0]
        self.win_v = vc[:, :, -W:].clone() if W else vc[:, :, :0]
        return y.view(B, n, H, D).transpose(1, 2)

    def _attend_tokens(self, q, k, v):
        """`attend` for a few tokens (a decode step): block by block through prepare / ingest, whose small concatenations are
        cheaper than the buffers of the long-call path below."""
        if torch.is_grad_enabled():
            raise RuntimeError("LinearFSCache is inference-only; use torch.no_grad().")
        a = self.attn
        B, H, n, D = q.shape
        if not self._ready:
            self._alloc(k)
        lam, sigma, lrs, norm_w = a.head_params()
        # window branch of the whole call: [the last <= W stored rows | the new rows]; the stored rows get dummy queries
        old = self.win_k.shape[2]
        kc = torch.cat([self.win_k, k.to(torch.bfloat16)], dim=2)
        vc = torch.cat([self.win_v, v.to(torch.bfloat16)], dim=2)
        qc = torch.cat([torch.zeros(B, H, old, D, dtype=torch.bfloat16, device=q.device), q.to(torch.bfloat16)], dim=2)
        cos, sin = a.rope.tables_bf16(self.pos + n)
        sr_all = ops.window_prefill(qc, kc, vc, cos, sin, self.W, a.scale, pos0=self.pos - old)[:, old:]      # (B,n,H*D)
        y = torch.empty(B, n, H * D, dtype=torch.bfloat16, device=q.device)
        off = 0
        while off < n:
            self.prepare()
            m = min(n - off, self.Bq - self.pos % self.Bq)
            qp = q[:, :, off:off + m]
            sr = sr_all[:, off:off + m].contiguous()
            if self.pool is None:
                y[:, off:off + m] = sr                  # no completed cell yet: the long-range branch is zero
            else:
                if type(self).select is not LinearFSCache.select or "select" in self.__dict__:
                    slots, ids = self.select(qp)                 # an overridden / wrapped select stays in the loop
                    sel = torch.full((B, H, m, a.cell_topk), -1, dtype=torch.int32, device=q.device)
                    sel[..., :slots.shape[-1]] = torch.where(ids >= 0, slots, torch.full_like(slots, -1)).to(torch.int32)
                else:
                    sel = self._select_slots(qp)
                # the pool slots are the "cells" of this readout; every pool token lies before the virtual query position
                n_kv = self.C * self.s
                out = ops.readout_combine(qp.to(torch.bfloat16), self.pool["k"], self.pool["v"], sel, sr, norm_w, lrs,
                                          a.lr_norm.eps, scale=a.scale, Bq=self.Bq, n_kv=n_kv,
                                          q_pos0=(n_kv + self.Bq - 1) // self.Bq * self.Bq)
                y[:, off:off + m] = out
            self.ingest(k[:, :, off:off + m], v[:, :, off:off + m])
            off += m
        return y.view(B, n, H, D).transpose(1, 2)
