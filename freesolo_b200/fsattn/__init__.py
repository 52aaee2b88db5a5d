"""Host-side mirror of the reference's ``src.fsattn`` package for the inference hot path (same class, argument and
attribute names; the computation runs in the sm_100a kernels of libfsattn_b200)."""
from .attention import FSAttn, RMSNorm  # noqa: F401
from .kv_cache import FSKVCache, make_caches  # noqa: F401
from . import kv_int8, kv_bounded, fsb_tree, fsb_prefill, fsl_select_cuda  # noqa: F401
