"""FSKVCache: the reference's per-layer KV-cache protocol (experiments/scaling/kv_cache.py:20-464) over the device-side
decode state of the sm_100a kernels.

Three stores, as in the reference: bf16 (default), int8 (``enable_int8``: per-cell symmetric int8 + bf16 scale, the open
cell's rows bf16 in a hot buffer) and bounded int8 (``enable_bounded``: only the cells a later decode step can read).
Differences from the reference that callers can observe:
  * capacity is fixed at prefill time to N + reserve rows (set ``reserve`` first; the reference doubles on demand);
  * cell statistics, quantisation, slot allocation and pool refresh at decode time run inside the decode-step kernel,
    driven by the device position, so ``advance_in_place`` only advances the host-side position.
"""
from __future__ import annotations

import os

import torch

from .. import ops
from . import kv_int8 as _kvi

CELL = ops.CELL


class FSKVCache:
    def __init__(self, attn, lean_prefill=False, retain_kv: bool = True):
        attn._assert_cacheable(phase="prefill")
        self.attn = attn
        self.s = attn.cell_stride
        self.W = attn.window_size
        self.pos = 0
        self.lean_prefill = lean_prefill
        self.retain_kv = bool(retain_kv)
        self.reserve = 0
        self.bounded = False            # (the reference's LinearFSCache marker; this cache is never that)
        self._int8_ok = False
        self.use_int8 = False
        self.bounded_kv = False
        self.state: ops.FslDecodeState | None = None
        self.pos_t = None               # device int64 scalar mirroring pos for eager decode steps
        self._ncell = 0
        self._prefill_cell_stats = None  # (kbar, ceil) handed over by the layer's own prefill, consumed by prefill()
        self._kbar = None               # statistics of the last prefill when retain_kv=False
        self._ceil = None
        self._lr_decode_pool = None

    # ---- switches (experiments/scaling/kv_cache.py:54-61) ----------------------------------------------------------------
    def enable_int8(self):
        self._int8_ok = True

    def enable_bounded(self):
        self._int8_ok = True
        self.bounded_kv = True

    def _mode(self, dtype, device) -> str:
        if self.bounded_kv:
            return "bounded"
        if self._int8_ok and _kvi.int8_supported(dtype, device):
            return "int8"
        return "bf16"

    def _new_state(self, B, cap_rows, device, dtype) -> ops.FslDecodeState:
        a = self.attn
        P, Wc = a._pool_cfg()
        mode = self._mode(dtype, device)
        self.use_int8 = mode != "bf16"
        return ops.FslDecodeState(B, a.n_heads, a.head_dim, cap_rows, device, mode=mode, P=P, Wc=Wc, W=a.window_size,
                                  Bq=a._cell_block, kk=a.cell_topk)

    def preallocate(self, B, N, dtype, device, keep=False):
        """Buffers for a prompt of N tokens plus `reserve` decode tokens (experiments/scaling/kv_cache.py:148-177)."""
        cap = N + max(0, int(self.reserve))
        self.state = self._new_state(B, max(cap, 1), device, dtype)

    def decode_state(self, like: torch.Tensor) -> ops.FslDecodeState:
        """The device state a decode step runs on; created empty (a decode without a prefill) when missing."""
        if self.state is None:
            cap = max(int(self.reserve), 1) + self.pos
            self.state = self._new_state(like.shape[0], cap, like.device, like.dtype)
        if self.pos_t is None or self.pos_t.device != like.device:
            self.pos_t = torch.zeros((), dtype=torch.int64, device=like.device)
        return self.state

    # ---- prefill -----------------------------------------------------------------------------------------------------------
    @torch.no_grad()
    def prefill(self, K, V, cell_stats=None):
        """Take the prompt's un-rotated K, V (B,H,N,D): cell statistics, int8 codes / bf16 copy / bounded slots, the first
        decode block's top-P list, the open cell. Returns (kbar (B,H,ncell,D), ceil (B,H,ncell)) for the layer's own
        selection. With retain_kv=False only the statistics are computed (the reference's prefill benchmark protocol,
        experiments/scaling/kv_cache.py:184-189)."""
        B, H, N, D = K.shape
        ncell = N // self.s
        handed, self._prefill_cell_stats = self._prefill_cell_stats, None
        cell_stats = handed if cell_stats is None else cell_stats
        if cell_stats is not None:
            kbar, ceil = cell_stats[-2:]            # the reference hands (K, Kbar, ceil); (Kbar, ceil) is accepted too
        else:
            kbar, ceil = ops.cell_stats(K, ncell)
        self._ncell = ncell
        self.pos = N
        # forests of an earlier prompt describe that prompt's cells: a new prefill starts them over
        fo = getattr(self, "fsb", None)
        if fo is not None:
            fo.reset()
        self._fsb_blk = -1
        if not self.retain_kv:
            self._kbar, self._ceil = kbar, ceil
            return kbar, ceil
        cap = N + max(0, int(self.reserve))
        if self.state is None or self.state.cap_rows < cap or self.state.B != B or self.state.kbar.device != K.device \
                or self.state.mode != self._mode(K.dtype, K.device):
            self.state = self._new_state(B, cap, K.device, K.dtype)
        self.state.prefill(K, V, N, kbar, ceil)
        self.pos_t = torch.full((), N, dtype=torch.int64, device=K.device)
        return kbar, ceil

    # ---- FS-B forests (src/fsattn/fsb_tree.py:1403-2260 ForestCache, 3598-3674 fsb_decode_prepare) --------------------------
    def fsb_forests(self, kbar, ceil, attn):
        """The layer's forests, created on first use over the cache's own statistics buffers (so the decode-time ingest
        sees the cells the decode kernel closes) or, when the prompt's K/V are not retained, over the given tensors."""
        if self.bounded_kv:
            raise NotImplementedError("FS-B reads any admitted cell: it needs a full KV store, not the bounded slot store")
        if self.state is not None:
            kb, ce, cap = self.state.kbar, self.state.ceil, self.state.cap_cells
        else:
            kb, ce, cap = kbar.contiguous(), ceil.contiguous(), kbar.shape[2]
        fo = getattr(self, "fsb", None)
        if fo is None or fo.kbar.data_ptr() != kb.data_ptr() or fo.m_cap < cap:
            tau_u = attn.fsb_tau_union if attn._fsb_union_tau_on() else None
            fo = ops.FsbForests(kb, ce, attn.fsb_tau, tau_u, cap_cells=cap)
            self.fsb = fo
            self._fsb_blk = -1
        elif fo.n_seen == 0:
            # reused for a new prompt: the thresholds may have been re-calibrated since the forests were created
            fo.taus[0].copy_(attn.fsb_tau.detach().float())
            if fo.nf > 1:
                fo.taus[1].copy_(attn.fsb_tau_union.detach().float())
        return fo

    def fsb_block_change(self, pos: int, attn) -> bool:
        """Bring the forests to the 128-token block of position pos: admit the cells completed before the block starts,
        build the chunks they complete, rebuild the spines. Happens once per block, on the host's side of the step
        (the reference does the same between graph replays, fsb_tree.py:3634-3660). Returns whether anything ran."""
        blk = (pos // attn._cell_block) * attn._cell_block
        if getattr(self, "_fsb_blk", -1) == blk and getattr(self, "fsb", None) is not None:
            return False
        if self.state is None:
            raise RuntimeError("FS-B decode needs the device KV state (prefill with retain_kv=True, or decode from empty)")
        fo = self.fsb_forests(None, None, attn)
        n_vis = min(blk // self.s, pos // self.s)
        fo.ingest(n_vis)
        fo.build_spines(n_vis, widths=(attn.fsb_width, attn._fsb_w2(fo)))
        self._fsb_blk = blk
        return True

    # ---- decode bookkeeping --------------------------------------------------------------------------------------------------
    def advance_in_place(self):
        """The token the decode step wrote becomes part of the cache (experiments/scaling/kv_cache.py:394-404). The cell
        close itself already happened on the device."""
        self.pos += 1
        if self.pos % self.s == 0:
            self._ncell = self.pos // self.s

    def append(self, k_t, v_t):
        raise NotImplementedError("rows are appended by the decode-step kernel; call the layer with the cache instead")

    # ---- read access used by callers and tests ----------------------------------------------------------------------------------
    def completed_cells(self):
        """(kbar, ceil, ncell) over the completed cells (experiments/scaling/kv_cache.py:442-447)."""
        if self.bounded_kv:
            self._no_history("completed_cells")
        ncell = self.pos // self.s
        if self.state is None:
            if self._kbar is None:
                return None, None, 0
            return self._kbar, self._ceil, self._kbar.shape[2]
        if ncell == 0:
            return None, None, 0
        return self.state.kbar[:, :, :ncell], self.state.ceil[:, :, :ncell], ncell

    def _no_history(self, what):
        raise RuntimeError(f"FSKVCache.{what} reads the full K / V history, which the bounded store does not keep")

    def int8_state(self):
        """(qk, qv, sk, sv, k_hot, v_hot, nq_t, s) (experiments/scaling/kv_cache.py:67-73); nq_t is derived from pos."""
        st = self.state
        nq = torch.full((), (self.pos // self.s) * self.s, dtype=torch.int64, device=st.kq.device)
        return (st.kq, st.vq, st.ks, st.vs, st.khot, st.vhot, nq, self.s)

    def slot_table(self):
        return self.state.slot_of if self.bounded_kv else None

    def bounded_pool(self, blk_start, out=None):
        """The bounded store's candidate pool of the block starting at blk_start (experiments/scaling/kv_cache.py:79-81,
        src/fsattn/kv_bounded.py:175-221), from its cell-indexed ceilings and slot-indexed mean keys. Read-only here:
        slots are freed by the decode-step kernel at its own block refresh."""
        from .attention import _pool_from_stats
        st = self.state
        M_vis = min(blk_start // self.s, self.pos // self.s)
        if M_vis <= 0:
            return {"empty": True}
        return _pool_from_stats(st.kbar, st.ceil[:, :, :M_vis], st.slot_of, blk_start, self.s, st.P, st.Wc)

    def graph_kv(self):
        """(mode, args) a captured decode step reads KV through (experiments/scaling/kv_cache.py:90-99)."""
        if self.bounded_kv:
            self._no_history("graph_kv")
        st = self.state
        if st is None:
            return (None, None)
        if st.mode == "bf16":
            return ("bf16", (st.kbuf, st.vbuf))
        return ("int8", self.int8_state())

    def rerank_keys(self):
        """What the FS-B re-rank reads token keys from (experiments/scaling/kv_cache.py:101-107): the int8 read state, or
        the bf16 history."""
        if self.bounded_kv:
            self._no_history("rerank_keys")
        st = self.state
        if st.mode == "bf16":
            return st.kbuf
        nq = torch.full((), (self.pos // self.s) * self.s, dtype=torch.int64, device=st.kq.device)
        return _kvi.Int8Keys(st.kq, st.ks, st.khot, nq, self.s)

    def row_capacity(self) -> int:
        if self.bounded_kv:
            self._no_history("row_capacity")
        return 0 if self.state is None else self.state.cap_rows

    def lr_tokens(self):
        """bf16 (K, V) over the stored history [0, pos) (experiments/scaling/kv_cache.py:458-464); int8 mode materialises."""
        if self.bounded_kv:
            self._no_history("lr_tokens")
        st, n = self.state, self.pos
        if st.mode == "bf16":
            return st.kbuf[:, :, :n], st.vbuf[:, :, :n]
        nq = (n // self.s) * self.s
        outs = []
        for q, sc, hot in ((st.kq, st.ks, st.khot), (st.vq, st.vs, st.vhot)):
            full = torch.empty(st.B, st.H, n, st.D, dtype=torch.bfloat16, device=q.device)
            if nq > 0:
                deq = ops.dequant_cells(q[:, :, :nq], sc, self.s)
                full[:, :, :nq].copy_(deq)
            if n > nq:
                full[:, :, nq:n].copy_(hot[:, :, :n - nq])
            outs.append(full)
        return outs[0], outs[1]

    read_full_kv = lr_tokens

    def sr_window(self, at=None):
        """(K, V, positions) of the window of the token at `at` (experiments/scaling/kv_cache.py:427-440)."""
        kh, vh = self.lr_tokens()
        end = self.pos if at is None else at + 1
        Lw = min(self.W + 1, end)
        return kh[:, :, end - Lw:end], vh[:, :, end - Lw:end], torch.arange(end - Lw, end, device=kh.device)

    def kv_faults(self):
        return (0, 0, 0) if self.state is None else self.state.faults()


def make_caches(model, *, lean_prefill=False, reserve=0, linear=None, retain_kv: bool = True) -> list:
    """One FSKVCache per layer, or one LinearFSCache (fixed-size streaming state) with linear=True or FSL_LINEAR_CACHE=1
    (experiments/scaling/kv_cache.py:467-481)."""
    linear = os.environ.get("FSL_LINEAR_CACHE", "0") == "1" if linear is None else linear
    caches = []
    for blk in model.blocks:
        a = blk.attn.fsattn
        a = getattr(a, "inner", a)                               # a head shard wraps its layer
        if linear:
            from .linear_cache import LinearFSCache
            caches.append(LinearFSCache(a))
            continue
        c = FSKVCache(a, lean_prefill=lean_prefill, retain_kv=retain_kv)
        c.reserve = reserve
        caches.append(c)
    return caches


@torch.no_grad()
def linear_prefill(model, idx, cache, *, chunk_size=2048, trunk=None):
    """Prompt through the model in chunks of chunk_size tokens with streaming caches in every layer: activations and
    state stay bounded whatever the prompt length (experiments/scaling/kv_cache.py:529-538). Returns the last position's
    hidden state (B,1,d). `trunk(model, ids, caches)` runs the blocks (the serving module's trunk_cached by default)."""
    if chunk_size <= 0 or idx.shape[1] == 0:
        raise ValueError("linear_prefill needs a positive chunk size and nonempty input")
    if not all(getattr(c, "bounded", False) for c in cache):
        raise ValueError("linear_prefill requires bounded caches in every layer")
    if trunk is None:
        from ..serving import trunk_cached as trunk
    device = model.tok_emb.weight.device
    hidden = None
    for start in range(0, idx.shape[1], chunk_size):
        hidden = trunk(model, idx[:, start:start + chunk_size].to(device), cache)
    return hidden[:, -1:].clone()
