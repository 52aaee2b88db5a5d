"""Host-side mirror of the reference API: construction, names, configuration errors (CPU only)."""
import os

import pytest
import torch

from freesolo_b200 import FSAttn, FSKVCache
from freesolo_b200.fsattn import kv_bounded
from freesolo_b200.fsattn.attention import Rotary
from freesolo_b200.serving import FreeSoloLM, MODEL_CONFIGS, serve_kwargs
from oracle import fsl


def _attn(**over):
    kw = serve_kwargs("sparse")
    kw.update(over)
    return FSAttn(d_model=256, n_heads=4, causal=True, bias=False, max_seq_len=1024, **kw)


def test_state_dict_names_match_the_reference():
    a = _attn()
    keys = set(a.state_dict().keys())
    # src/fsattn/attention.py:129-158: parameters and persistent buffers of an FS-L layer (rope tables are non-persistent)
    assert keys == {"sel_scale", "log_sigma", "long_range_scale", "lr_norm.scale", "W_q.weight", "W_k.weight", "W_v.weight",
                    "W_o.weight"}
    assert tuple(a.long_range_scale.shape) == (4, 1, 1) and a.head_dim == 64 and a._cell_block == 128
    assert torch.allclose(a.sigma, torch.full((4,), 4.0))


def test_lm_parameter_count_and_names():
    m = FreeSoloLM.from_config("debug", max_seq_len=512, **serve_kwargs("sparse"))
    names = dict(m.named_parameters())
    assert "blocks.0.attn.fsattn.W_q.weight" in names and "blocks.3.ffn.w_down.weight" in names and "ln_final.weight" in names
    assert m.lm_head.weight is m.tok_emb.weight
    c = MODEL_CONFIGS["340m"]
    d, f, L_, V = c["d_model"], c["d_ff"], c["n_layers"], c["vocab_size"]
    per_layer = 4 * d * d + 3 * d * f + 2 * d + 2 * 16 + 64   # log_sigma is a buffer when the window is uniform
    assert L_ * per_layer + V * d + d == 341_101_824      # the reference's 341M


def test_rotary_tables_match_oracle_and_grow_in_fp32():
    r = Rotary(64, 4096)
    cos, sin = fsl.rope_tables(64, 4096, orig_len=4096)
    assert torch.equal(r.cos_cached, cos) and torch.equal(r.sin_cached, sin)
    r = r.to(torch.bfloat16)
    r._build_cache(6000)
    cos2, _ = fsl.rope_tables(64, 6000, orig_len=4096)
    assert r.cos_cached.dtype == torch.bfloat16 and torch.equal(r.cos_cached, cos2.to(torch.bfloat16))


def test_uncacheable_configurations_raise():
    for over in (dict(rope_long_range=True), dict(sel_strict_causal=0), dict(cell_stride=64), dict(fs_uniform_sr=False),
                 dict(cell_prune_kernel=0, cell_topk=8)):
        with pytest.raises(NotImplementedError):
            FSKVCache(_attn(**over))
    FSKVCache(_attn(cell_prune_kernel=0))                                         # the dense FS variant is cacheable
    FSKVCache(_attn(fsb_enabled=True, fsb_read_top=4, cell_prune_kernel=0))     # an FS-B layer is cacheable
    c = FSKVCache(_attn(fsb_enabled=True, fsb_read_top=4, cell_prune_kernel=0))
    c.enable_bounded()
    with pytest.raises(NotImplementedError):                                      # ... but not on the bounded slot store
        c.fsb_forests(None, None, c.attn)
    a = _attn()
    with pytest.raises(NotImplementedError):
        a(torch.zeros(1, 4, 256))            # no cache: the training forward is not part of this build
    with pytest.raises(RuntimeError):
        a(torch.zeros(1, 4, 256), cache=FSKVCache(a))    # CPU / fp32 activations: no fallback


def test_bounded_slot_count_and_config():
    a = _attn()
    assert kv_bounded.slot_count(a) == 64 + 16 + 4 + 1 == 85          # src/fsattn/kv_bounded.py:59-61
    assert kv_bounded._cfg(a) == (64, 8, 512, 128, 32)
    assert not kv_bounded.supported([a], torch.bfloat16, "cpu")


def test_fused_projection_weights_are_views():
    a = _attn()
    w, dm = a._ensure_qkv_cache()
    assert w.shape == (768, 256) and a.W_k.weight.data_ptr() == w[dm:].data_ptr()
    w2, _ = a._ensure_qkv_cache()
    assert w2 is w


def test_fsb_layer_construction_and_refusals():
    """FS-B keywords of the reference layer (src/fsattn/fsb_tree.py:41-155): the serve preset builds, its persistent
    buffer is named like the reference's, and configurations outside the built one are refused at construction."""
    import pytest
    a = FSAttn(256, 4, causal=True, bias=False, **serve_kwargs("fsb", 0.9))
    assert a.fsb_enabled and "fsb_tau" in a.state_dict() and "fsb_tau_union" not in a.state_dict()
    assert (a.fsb_width, a.fsb_union_width, a.fsb_read_top, a.fsb_W_max, a.fsb_delta) == (16, 16, 4, 16, 0)
    assert a._fsb_union_tau_on()
    assert not FSAttn(256, 4, causal=True, bias=False, **serve_kwargs("fsb"))._fsb_union_tau_on()
    for bad in (dict(fsb_delta=1), dict(fsb_policy="learned"), dict(fsb_node_score="mean"), dict(fsb_tree="rebuild"),
                dict(fsb_rerank_score="leaf"), dict(fsb_width=32), dict(fsb_hybrid="pool"), dict(fsb_read_top=2)):
        kw = serve_kwargs("fsb", 0.9)
        kw.update(bad)
        with pytest.raises(NotImplementedError):
            FSAttn(256, 4, causal=True, bias=False, **kw)


def test_streaming_cache_construction_and_refusals():
    """make_caches(linear=True) gives one LinearFSCache per layer (ref: experiments/scaling/kv_cache.py:467-481); the dense
    and FS-B variants are refused as the reference refuses them; linear_prefill checks its arguments."""
    from freesolo_b200.fsattn.kv_cache import linear_prefill, make_caches
    from freesolo_b200.fsattn.linear_cache import LinearFSCache
    from freesolo_b200.serving import FreeSoloLM, serve_kwargs
    m = FreeSoloLM(vocab_size=64, d_model=128, n_layers=2, n_heads=2, d_ff=256, max_seq_len=256, **serve_kwargs("sparse"))
    caches = make_caches(m, linear=True)
    assert len(caches) == 2 and all(isinstance(c, LinearFSCache) and c.bounded for c in caches)
    c = caches[0]
    assert (c.s, c.Bq, c.W, c.P, c.Wc, c.C) == (32, 128, 512, 64, 8, 72) and c.state_bytes() == 0 and c.pool is None
    os.environ["FSL_LINEAR_CACHE"] = "1"
    try:
        assert isinstance(make_caches(m)[0], LinearFSCache)
    finally:
        del os.environ["FSL_LINEAR_CACHE"]
    assert not isinstance(make_caches(m)[0], LinearFSCache)
    dense = FreeSoloLM(vocab_size=64, d_model=128, n_layers=1, n_heads=2, d_ff=256, max_seq_len=256, **serve_kwargs("dense"))
    with pytest.raises(ValueError):
        make_caches(dense, linear=True)
    fsb = FreeSoloLM(vocab_size=64, d_model=128, n_layers=1, n_heads=2, d_ff=256, max_seq_len=256, **serve_kwargs("fsb"))
    with pytest.raises((ValueError, NotImplementedError)):        # no pool pruning in the FS-B configuration either
        make_caches(fsb, linear=True)
    ids = torch.zeros(1, 8, dtype=torch.long)
    with pytest.raises(ValueError):
        linear_prefill(m, ids, caches, chunk_size=0)
    with pytest.raises(ValueError):
        linear_prefill(m, ids, make_caches(m))          # FSKVCache is not a bounded streaming cache
    with pytest.raises(ValueError):
        c.ingest(torch.zeros(1, 2, 129, 64), torch.zeros(1, 2, 129, 64))      # more than one query block at once
