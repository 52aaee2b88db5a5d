"""int8 long-range KV codec: the reference's ``src/fsattn/kv_int8.py`` names on the CUDA kernels.

Per (batch, head, cell, K-or-V): scale = bf16(max|x| / 127) (1.0 for an all-zero cell), q = rint(x / f32(scale));
reads return bf16(f32(q) * f32(scale)). The codes are bit-identical to the reference's quantize_cells."""
from __future__ import annotations

import os

import torch

from .. import ops


def int8_on() -> bool:
    """FS_KV_INT8 switch of the reference (src/fsattn/kv_int8.py:32-33)."""
    return os.environ.get("FS_KV_INT8", "1") == "1"


def int8_supported(dtype, device) -> bool:
    """src/fsattn/kv_int8.py:36-37: bf16 keys/values on a CUDA device."""
    return int8_on() and torch.device(device).type == "cuda" and dtype == torch.bfloat16


class Int8Keys:
    """Token keys of an int8-mode cache (src/fsattn/kv_int8.py:40-47): int8 cell rows + bf16 cell scales, the open cell's
    bf16 rows, and the device scalar n_q."""
    __slots__ = ("q", "sc", "hot", "nq_t", "s")

    def __init__(self, q, sc, hot, nq_t, s):
        self.q, self.sc, self.hot, self.nq_t, self.s = q, sc, hot, nq_t, s


@torch.no_grad()
def quantize_cells(x: torch.Tensor, s: int):
    """x (B,H,N,D) bf16 -> (q int8 (B,H,nc*s,D), scale bf16 (B,H,nc)); src/fsattn/kv_int8.py:51-59."""
    return ops.quantize_cells(x, s)


@torch.no_grad()
def quantize_cells_fast(x: torch.Tensor, s: int, q: torch.Tensor = None, sc: torch.Tensor = None):
    """src/fsattn/kv_int8.py:102-118: same, into preallocated slices of the cache buffers."""
    return ops.quantize_cells(x, s, q, sc)


@torch.no_grad()
def dequant_cells(q: torch.Tensor, sc: torch.Tensor, s: int, dtype=torch.bfloat16, out: torch.Tensor = None):
    """Inverse read over the quantised region; src/fsattn/kv_int8.py:63-71."""
    return ops.dequant_cells(q, sc, s, dtype, out)
