"""Import-path alias: makes this package answer to the reference's module paths (``src.fsattn``, ``src.fsattn.attention``,
``src.fsattn.kv_int8`` ..., ``src.utils.trunk_triton``), so that code written against the reference - its FreeSoloLM, KV
cache and decoders do ``from src.fsattn import FSAttn`` - picks up this implementation without an edit.

    import freesolo_b200.compat as compat
    compat.install()          # before the caller's first ``import src...``

Refuses when a different ``src`` package is already imported (the reference itself, or an unrelated package of that name)."""
from __future__ import annotations

import sys
import types

ALIASES = {
    "src.fsattn": "freesolo_b200.fsattn",
    "src.fsattn.attention": "freesolo_b200.fsattn.attention",
    "src.fsattn.kv_int8": "freesolo_b200.fsattn.kv_int8",
    "src.fsattn.kv_bounded": "freesolo_b200.fsattn.kv_bounded",
    "src.fsattn.kv_cache": "freesolo_b200.fsattn.kv_cache",
    "src.fsattn.fsb_tree": "freesolo_b200.fsattn.fsb_tree",
    "src.fsattn.fsb_prefill": "freesolo_b200.fsattn.fsb_prefill",
    "src.fsattn.fsl_select_cuda": "freesolo_b200.fsattn.fsl_select_cuda",
    "src.utils": "freesolo_b200.utils",
    "src.utils.trunk_triton": "freesolo_b200.utils.trunk_triton",
}


def install() -> None:
    import importlib
    existing = sys.modules.get("src")
    if existing is not None and not getattr(existing, "__freesolo_b200_alias__", False):
        raise RuntimeError("a package named 'src' is already imported; install the alias before it, or in a fresh process")
    root = types.ModuleType("src")
    root.__path__ = []                       # a package, with no files of its own
    root.__freesolo_b200_alias__ = True
    sys.modules["src"] = root
    for alias, target in ALIASES.items():
        mod = importlib.import_module(target)
        sys.modules[alias] = mod
        parent, _, leaf = alias.rpartition(".")
        setattr(sys.modules[parent], leaf, mod)


def uninstall() -> None:
    for name in ["src"] + list(ALIASES):
        m = sys.modules.get(name)
        if m is not None and (name != "src" or getattr(m, "__freesolo_b200_alias__", False)):
            del sys.modules[name]
