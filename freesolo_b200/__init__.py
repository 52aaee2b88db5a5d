"""freesolo_b200: B200-native (sm_100a) kernels and host code for the FreeSolo sparse-attention inference hot path.

Layout:
  csrc/            CUDA kernels + the C ABI (built into libfsattn_b200.so by csrc/build.sh)
  lib.py           ctypes binding of the C ABI (no fallback: raises when the library is missing)
  ops.py           torch-tensor front end of the entry points
  fsattn/          host-side mirror of the reference's src/fsattn module API (FSAttn, FSKVCache, kv_int8, kv_bounded)
  serving.py       minimal FreeSoloLM trunk, graphed decoder and prefill driver used by bench.py
"""
from . import lib, ops  # noqa: F401
from .fsattn import FSAttn, FSKVCache  # noqa: F401
