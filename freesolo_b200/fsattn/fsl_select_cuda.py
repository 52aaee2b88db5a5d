"""The names the reference's callers import from ``src/fsattn/fsl_select_cuda.py``: the cell-statistics helper of the KV
cache and the status dictionary its benchmark prints. The selection itself is ``ops.fsl_prefix_topp`` + ``ops.fsl_select``."""
from __future__ import annotations

from .. import lib as _lib
from .. import ops


def cache_cell_stats(K, ncell: int, s: int = ops.CELL):
    """(Kbar (B,H,ncell,D) fp32, ceil (B,H,ncell) fp32) of the first ncell cells of K (src/fsattn/fsl_select_cuda.py:212-249)."""
    if s != ops.CELL:
        raise RuntimeError(f"cell size {s} unsupported (kernels are specialised for {ops.CELL})")
    return ops.cell_stats(K, ncell)


def status() -> dict:
    """src/fsattn/fsl_select_cuda.py:85-94: which selection path runs. There is one path and no fallback latch here."""
    return {"available": True, "backend": "libfsattn_b200 (sm_100a, ahead-of-time)", "version": int(_lib.load().fsattn_version()),
            "fallback": False, "error": None}
