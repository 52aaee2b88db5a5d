"""The C-ABI shared library: it loads, exports every symbol include/fsattn_b200.h declares, and the ctypes mirrors of the
argument structs have the sizes the C compiler gives them. No compute calls (no GPU needed)."""
import ctypes
import os
import re
import subprocess
import sys

import pytest
import torch

from conftest import ROOT
from freesolo_b200 import lib as L

HEADER = os.path.join(ROOT, "include", "fsattn_b200.h")


def _declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*FSATTN_API\s+(?:int|int64_t|const char\*)\s+(fsattn_\w+)\s*\(", src, flags=re.M)))


def test_every_declared_symbol_is_exported_and_bound(built_lib):
    names = _declared()
    assert len(names) >= 10
    for n in names:
        assert hasattr(built_lib, n), f"{n} declared in the header but not exported"
    assert sorted(L.ENTRY_POINTS) == names, "lib.ENTRY_POINTS and the header disagree"
    assert built_lib.fsattn_version() >= 1


def test_struct_sizes_match_the_c_compiler(tmp_path):
    structs = {"fsattn_bhnd_t": L.BHND, "fsattn_cell_ingest_t": L.CellIngest, "fsattn_dequant_t": L.Dequant,
               "fsattn_fsl_topp_t": L.FslTopp, "fsattn_fsl_select_t": L.FslSelect,
               "fsattn_window_prefill_t": L.WindowPrefill, "fsattn_readout_combine_t": L.ReadoutCombine,
               "fsattn_fsl_state_t": L.FslState, "fsattn_fsl_decode_t": L.FslDecode, "fsattn_slot_prefill_t": L.SlotPrefill}
    extra = getattr(L, "EXTRA_STRUCTS", {})
    structs.update(extra)
    prog = '#include <stdio.h>\n#include <stddef.h>\n#include "fsattn_b200.h"\nint main(void){\n'
    for n in structs:
        prog += f'  printf("{n} %zu\\n", sizeof({n}));\n'
    prog += '  printf("off_splits %zu\\n", offsetof(fsattn_fsl_decode_t, splits));\n  return 0;}\n'
    c = tmp_path / "sz.c"
    c.write_text(prog)
    exe = tmp_path / "sz"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(c), "-o", str(exe)], check=True)
    out = dict(l.split() for l in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines())
    for n, st in structs.items():
        assert int(out[n]) == ctypes.sizeof(st), f"{n}: C says {out[n]}, ctypes says {ctypes.sizeof(st)}"
    assert int(out["off_splits"]) == L.FslDecode.splits.offset


def test_bad_arguments_are_rejected_on_the_host(built_lib):
    a = L.FslTopp()
    rc = built_lib.fsattn_fsl_prefix_topp(ctypes.byref(a), None)
    assert rc == L.EINVAL and b"null" in built_lib.fsattn_last_error()
    d = L.FslDecode()
    assert built_lib.fsattn_fsl_decode_step(ctypes.byref(d), None) == L.EINVAL
    w = L.WindowPrefill()
    assert built_lib.fsattn_window_prefill(ctypes.byref(w), None) == L.EINVAL


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(L, "_lib", None)
    monkeypatch.setattr(L, "LIB_PATH", str(tmp_path / "nope.so"))
    with pytest.raises(RuntimeError, match="no fallback"):
        L.load()


def test_cpu_tensors_are_refused():
    from freesolo_b200 import ops
    K = torch.zeros(1, 1, 64, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ops.cell_stats(K, 2)
