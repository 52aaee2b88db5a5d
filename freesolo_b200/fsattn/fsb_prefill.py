"""``fast_status`` of the reference's ``src/fsattn/fsb_prefill.py:84-103``: its benchmark prints which FS-B prefill path ran
and whether a fallback latched. One path exists here (``ops.fsb_select``: beams per query block + block-cooperative re-rank)."""
from __future__ import annotations


def fast_status() -> dict:
    return {"fast": True, "fallback": False, "overflow_redo": 0, "error": None}
