"""The helper names the reference's model and decoders import from ``src/utils/trunk_triton.py`` (experiments/scaling/
model.py:127-145,212-233, decode_graph.py:11-24): one-pass RMSNorm and SiLU * up gates. The reference implements them as
Triton kernels; here they run this library's CUDA kernels where those apply and report "not ok" otherwise, in which case
the callers use their eager torch ops (the protocol the reference itself follows)."""
from __future__ import annotations

import torch

from .. import ops

MIN_ROWS = 16
_GRAPH_WARMUP = False


def available() -> bool:
    return torch.cuda.is_available()


def autocast_dtype():
    """src/utils/trunk_triton.py:975-978."""
    if not torch.is_autocast_enabled():
        return None
    return torch.get_autocast_dtype("cuda") if hasattr(torch, "get_autocast_dtype") else torch.get_autocast_gpu_dtype()


def _rows(x: torch.Tensor) -> int:
    return x.numel() // x.shape[-1] if x.dim() > 0 and x.shape[-1] > 0 else 0


def rms_norm_ok(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """Whether rms_norm_cast may be used (src/utils/trunk_triton.py:994-1003): no-grad CUDA inference on bf16 rows with a
    bf16 weight, under bf16 autocast."""
    return (not torch.is_grad_enabled() and x.is_cuda and x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16
            and autocast_dtype() == torch.bfloat16 and x.is_contiguous() and x.shape[-1] % 8 == 0 and x.numel() > 0
            and x.shape[-1] == weight.shape[0])


def rms_norm_cast(x: torch.Tensor, weight: torch.Tensor, eps: float, dtype: torch.dtype, res: torch.Tensor | None = None):
    """RMSNorm(x [+ res]) * weight written once in `dtype` (src/utils/trunk_triton.py:1011-1044); fp32 arithmetic."""
    if res is not None:
        x.add_(res)
    if x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16 and dtype == torch.bfloat16 and x.is_cuda:
        return ops.rms_norm(x, weight, eps)
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * weight.float()).to(dtype)


def silu_mul_ok(g: torch.Tensor, u: torch.Tensor) -> bool:
    """src/utils/trunk_triton.py:1047-1051. The one-pass gate of this library takes the fused (gate | up) projection
    (``ops.swiglu``); for two separate tensors the callers keep their eager ops."""
    return False


def silu_mul(g: torch.Tensor, u: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    r = torch.nn.functional.silu(g) * u
    if out is not None:
        out.copy_(r)
        return out
    return r
