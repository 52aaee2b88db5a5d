"""The drop-in boundary on the host: this package's FSAttn against the reference's own class (same constructor keywords,
same parameter / buffer names and shapes, state dicts load both ways), and the import-path alias. The comparisons with the
reference need a copy of its sources (oracle/_ref, written by oracle/make_ref.py where a checkout exists) and are skipped
without one."""
import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _reference_fsattn():
    from oracle.make_ref import import_reference
    if not import_reference():
        pytest.skip("no copy of the reference sources (oracle/_ref)")
    from src.fsattn import FSAttn as RefFSAttn        # the reference's own package
    return RefFSAttn


@pytest.mark.parametrize("preset", ["sparse", "fsb"])
def test_state_dict_is_interchangeable_with_the_reference(preset):
    RefFSAttn = _reference_fsattn()
    from freesolo_b200.fsattn import FSAttn
    from freesolo_b200.serving import serve_kwargs
    kw = serve_kwargs("sparse") if preset == "sparse" else serve_kwargs("fsb", 0.9)
    os.environ["FS_PRUNE_KERNEL"] = "1" if preset == "sparse" else "0"
    try:
        torch.manual_seed(0)
        ref = RefFSAttn(d_model=256, n_heads=4, causal=True, bias=False, max_seq_len=512, **kw)
        torch.manual_seed(0)
        ours = FSAttn(d_model=256, n_heads=4, causal=True, bias=False, max_seq_len=512, **kw)
    finally:
        os.environ["FS_PRUNE_KERNEL"] = "1"
    sd_r, sd_o = ref.state_dict(), ours.state_dict()
    assert sorted(sd_r) == sorted(sd_o), f"state-dict keys differ: {sorted(set(sd_r) ^ set(sd_o))}"
    for k in sd_r:
        assert tuple(sd_r[k].shape) == tuple(sd_o[k].shape) and sd_r[k].dtype == sd_o[k].dtype, k
    # the same seeded construction gives the same initial values, and each loads the other's dict strictly
    for k in sd_r:
        assert torch.equal(sd_r[k], sd_o[k]), f"{k}: initial values differ"
    with torch.no_grad():
        for p in ref.parameters():
            p.add_(0.125)
    ours.load_state_dict(ref.state_dict(), strict=True)
    assert all(torch.equal(a, b) for a, b in zip(ref.state_dict().values(), ours.state_dict().values()))
    ref.load_state_dict(ours.state_dict(), strict=True)
    # non-persistent buffers exist under the reference's names too
    for name in ("rope.inv_freq", "rope.cos_cached", "rope.sin_cached") + (("fsb_tau_union",) if preset == "fsb" else ()):
        assert name in dict(ours.named_buffers()) and name in dict(ref.named_buffers()), name
    for attr in ("n_heads", "head_dim", "window_size", "cell_stride", "_cell_block", "cell_topk", "d_model", "scale"):
        assert getattr(ref, attr) == getattr(ours, attr), attr
    assert torch.allclose(ref.sigma, ours.sigma)


def test_import_path_alias_in_a_fresh_interpreter():
    code = (
        "import freesolo_b200.compat as c; c.install();"
        "from src.fsattn import FSAttn; from src.fsattn.attention import FSAttn as A2;"
        "from src.fsattn import kv_int8, kv_bounded;"
        "from src.fsattn.fsb_tree import fsb_decode_prepare_all, fsb_graph_registry, fsb_calibrate_tau, fsb_read_stats_reset, fsb_read_stats;"
        "from src.fsattn.fsl_select_cuda import cache_cell_stats, status; from src.fsattn.fsb_prefill import fast_status;"
        "from src.utils import trunk_triton as tt;"
        "assert FSAttn is A2 and FSAttn.__module__.startswith('freesolo_b200');"
        "assert all(hasattr(tt, n) for n in ('rms_norm_ok','rms_norm_cast','silu_mul_ok','silu_mul','autocast_dtype','_rows','_GRAPH_WARMUP'));"
        "assert all(hasattr(FSAttn, n) for n in ('graph_decode_layer','graph_decode_layer_fsb','_build_decode_pool',"
        "'_build_dense_decode_pool','_ensure_qkv_cache','_is_dense_lr','_prune_cfg','_assert_cacheable'));"
        "print('alias ok')")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "alias ok" in r.stdout, r.stderr[-2000:]


def test_alias_refuses_when_another_src_package_is_loaded():
    code = ("import sys, types; sys.modules['src'] = types.ModuleType('src');"
            "import freesolo_b200.compat as c\n"
            "try:\n    c.install()\nexcept RuntimeError as e:\n    print('refused')")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert "refused" in r.stdout, r.stderr[-2000:]
