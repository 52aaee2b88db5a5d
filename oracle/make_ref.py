"""Recipe for oracle/_ref/: a runnable copy of the reference implementation's inference sources (test infrastructure).

    python oracle/make_ref.py [--reference /path/to/freesolo]

Copies the reference's `src/` package and `experiments/scaling/*.py` (what its own `bench_efficiency.py` imports) from a
checkout of zekun-shi/freesolo into oracle/_ref/, unmodified. oracle/_ref/ is listed in .gitignore, so no reference
source ever enters this repository's history; it exists so that the benchmark's reference arm and its `cpu_baseline` leg can
time the reference's OWN eager CPU path on a machine that has no checkout of it. Nothing under freesolo_b200/ imports it.
Without a checkout the script does nothing and returns False; the benchmark then falls back to the CPU port
(oracle/model.py) and says so.
"""
from __future__ import annotations

import argparse
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
DEST = os.path.join(HERE, "_ref")


def make_ref(reference: str = "/root/reference") -> bool:
    src_pkg = os.path.join(reference, "src")
    scaling = os.path.join(reference, "experiments", "scaling")
    if not (os.path.isdir(src_pkg) and os.path.isdir(scaling)):
        return False
    if os.path.isdir(DEST):
        shutil.rmtree(DEST)
    os.makedirs(os.path.join(DEST, "experiments", "scaling"))
    shutil.copytree(src_pkg, os.path.join(DEST, "src"), ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
    for name in sorted(os.listdir(scaling)):
        if name.endswith(".py"):
            shutil.copy2(os.path.join(scaling, name), os.path.join(DEST, "experiments", "scaling", name))
    for pkg in ("experiments", os.path.join("experiments", "scaling")):
        init = os.path.join(reference, pkg, "__init__.py")
        if os.path.isfile(init):
            shutil.copy2(init, os.path.join(DEST, pkg, "__init__.py"))
    return True


def ref_available() -> bool:
    return os.path.isfile(os.path.join(DEST, "src", "fsattn", "attention.py"))


def import_reference():
    """Put oracle/_ref on sys.path the way the reference's own scripts expect and set its semantic switches
    (strict-causal selection, FS-L pool pruning). Returns False when oracle/_ref is absent."""
    if not ref_available():
        return False
    for p in (DEST, os.path.join(DEST, "experiments", "scaling")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(FS_STRICT_CAUSAL="1", FS_PRUNE_KERNEL="1", FSB_TRAIN_GRAPH="0")
    return True


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("FREESOLO_REFERENCE", "/root/reference"))
    ok = make_ref(ap.parse_args().reference)
    print("oracle/_ref written" if ok else "no reference checkout found: nothing written")
