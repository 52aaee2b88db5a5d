"""FS-L bounded retention pool: the reference's ``src/fsattn/kv_bounded.py`` names.

The store keeps exactly the cells a later decode step can still read: the top-P cells by (ceiling desc, index asc) and
every cell from c_lo = max(0, min((blk - W) // s, m_vis - Wc)) on; S = P + max(ceil(W/s), Wc) + Bq/s + 1 slots of s rows
of int8 K and V with a bf16 scale per slot and tensor. In this implementation the slot bookkeeping at decode time (lowest
free slot for a completed cell, freeing at a block refresh, fault counters) runs inside the fused decode-step kernel; the
prefill fill is ``fsattn_slot_prefill``. ``SlotStore`` is a view of ``ops.FslDecodeState`` in "bounded" mode."""
from __future__ import annotations

import os

import torch

from .. import ops


def bounded_on() -> bool:
    """FSL_KV_BOUNDED switch (src/fsattn/kv_bounded.py:48-49)."""
    return os.environ.get("FSL_KV_BOUNDED", "1") == "1"


def _cfg(attn):
    """(P, Wc, W, Bq, s) of an FS-L layer (src/fsattn/kv_bounded.py:52-56)."""
    return (attn._prune_cfg("cell_prune_pool", "FS_PRUNE_POOL", 64),
            attn._prune_cfg("cell_prune_window", "FS_PRUNE_WINDOW", 8),
            int(attn.window_size), int(attn._cell_block), int(attn.cell_stride))


def slot_count(attn) -> int:
    """src/fsattn/kv_bounded.py:59-61."""
    P, Wc, W, Bq, s = _cfg(attn)
    return P + max(-(-W // s), Wc) + -(-Bq // s) + 1


def supported(attns, dtype, device) -> bool:
    """Whether every layer can decode on the bounded store (src/fsattn/kv_bounded.py:64-82)."""
    if torch.device(device).type != "cuda" or dtype != torch.bfloat16:
        return False
    for a in attns:
        P, Wc, W, Bq, s = _cfg(a)
        if (getattr(a, "fsb_enabled", False) or a._is_dense_lr() or a.head_dim not in (64, 96, 128) or s != ops.CELL
                or Bq % s or P < 1 or P > 128 or not 0 <= Wc <= 8 or not 1 <= a.cell_topk <= 8):
            return False
    return True


class SlotStore:
    """One layer's bounded K / V (src/fsattn/kv_bounded.py:85-234) over an ``ops.FslDecodeState`` in bounded mode."""

    def __init__(self, attn, B: int, n_cells: int, device):
        self.P, self.Wc, self.W, self.Bq, self.s = _cfg(attn)
        self.state = ops.FslDecodeState(B, attn.n_heads, attn.head_dim, max(1, n_cells) * self.s, device, mode="bounded",
                                        P=self.P, Wc=self.Wc, W=self.W, Bq=self.Bq, kk=attn.cell_topk)
        st = self.state
        self.B, self.H, self.D = B, attn.n_heads, attn.head_dim
        self.n_slots, self.n_cells = st.n_slots, st.cap_cells
        self.qk, self.qv, self.sk, self.sv, self.kbar = st.kq, st.vq, st.ks, st.vs, st.kbar
        self.cell_in, self.slot_of, self.ceil, self.flags = st.cell_in, st.slot_of, st.ceil, st.status

    def fits(self, B, H, D, n_cells, device) -> bool:
        return (self.B, self.H, self.D) == (B, H, D) and self.n_cells >= n_cells and self.qk.device == torch.device(device)

    def _readable_from(self, blk_start: int, m_vis: int) -> int:
        return max(0, min((blk_start - self.W) // self.s, m_vis - self.Wc))

    @torch.no_grad()
    def prefill(self, K, V, kbar, ceil, N: int):
        self.state.prefill(K, V, N, kbar, ceil)

    def held(self) -> torch.Tensor:
        return (self.cell_in >= 0).sum(-1)

    def faults(self) -> tuple:
        f = self.state.faults()
        return f[0], f[1]

    def nbytes(self) -> int:
        return self.state.nbytes()
