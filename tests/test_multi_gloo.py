"""Head sharding on CPU ranks (gloo, world size 2): the partition arithmetic, the parameter slices and the all-gather
order of freesolo_b200.parallel, with the CPU oracle standing in for the per-head attention kernels (which are CUDA-only).
The sharded layer must reproduce the unsharded computation."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _core(attn, Q, K, V):
    """Stand-in for FSAttn._prefill: the oracle's FS-L layer on this module's heads (returns W_o's input (B,N,H*D))."""
    from oracle import fsl
    H, D = attn.n_heads, attn.head_dim
    L = fsl.FSLLayerOracle(H, D, lam=attn.sel_scale.detach(), sigma=attn.sigma.detach(),
                           lrs=attn.long_range_scale.detach().reshape(H), norm_w=attn.lr_norm.scale.detach(),
                           eps=attn.lr_norm.eps, act_dtype=torch.float32, rope_len=1024, rope_orig_len=1024)
    y, _, _ = L.prefill(Q.float(), K.float(), V.float())
    return y


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        torch.set_num_threads(2)
        from freesolo_b200.fsattn import FSAttn
        from freesolo_b200.parallel import HeadShard, ShardedFSAttn
        from freesolo_b200.serving import serve_kwargs
        torch.manual_seed(0)                                     # every rank builds the same full layer
        H, D, N = 4, 64, 320
        full = FSAttn(H * D, H, causal=True, bias=False, max_seq_len=1024, **serve_kwargs("sparse")).eval()
        with torch.no_grad():
            full.sel_scale.copy_(0.5 + torch.rand(H))
            full.long_range_scale.copy_((0.1 + torch.rand(H)).view(H, 1, 1))
            full.lr_norm.scale.copy_(0.5 + torch.rand(D))
        x = torch.randn(1, N, H * D)
        # unsharded reference: project, per-head core, W_o
        Qf, Kf, Vf = full._project_qkv(x)
        want = full.W_o(_core(full, Qf, Kf, Vf))
        # ---- partition arithmetic ----
        sh = HeadShard(H, D, rank, world)
        assert (sh.Hl, sh.h0, sh.h1, sh.dl) == (H // world, rank * H // world, (rank + 1) * H // world, H * D // world)
        w_qkv, _ = full._ensure_qkv_cache()
        wl = sh.qkv_rows(w_qkv)
        assert wl.shape == (3 * sh.dl, H * D)
        assert torch.equal(wl[:sh.dl], full.W_q.weight[sh.h0 * D:sh.h1 * D])
        assert torch.equal(wl[2 * sh.dl:], full.W_v.weight[sh.h0 * D:sh.h1 * D])
        # gather order: rank-major == head-major, for many rows and for the single decode row
        y_l = torch.full((1, 3, sh.dl), float(rank)) + torch.arange(sh.dl) / 1000.0
        y_g = sh.gather(y_l)
        assert y_g.shape == (1, 3, H * D)
        for r in range(world):
            assert torch.equal(y_g[..., r * sh.dl:(r + 1) * sh.dl], torch.full((1, 3, sh.dl), float(r)) + torch.arange(sh.dl) / 1000.0)
        out = torch.empty(1, H * D)
        sh.gather(y_l[:, 0], out=out)
        assert torch.equal(out, y_g[:, 0])
        # ---- the sharded layer with the oracle as its kernel ----
        s_attn = ShardedFSAttn(full, rank, world)
        assert s_attn.inner.n_heads == sh.Hl and torch.equal(s_attn.inner.sel_scale, full.sel_scale[sh.h0:sh.h1])
        assert torch.equal(s_attn.inner.long_range_scale, full.long_range_scale[sh.h0:sh.h1])
        assert torch.equal(s_attn.inner.lr_norm.scale, full.lr_norm.scale) and s_attn.W_o is full.W_o
        s_attn.inner._assert_cacheable = lambda phase="decode": None
        s_attn.inner._prefill = lambda Q, K, V, cache: _core(s_attn.inner, Q, K, V)

        class _Cache:
            pos = 0
        got = s_attn(x, cache=_Cache())
        err = (got - want).abs().max().item()
        assert err < 1e-4, f"rank {rank}: sharded layer differs from the unsharded one by {err}"
        # every rank holds the same result (the residual stream stays replicated)
        both = [torch.empty_like(got) for _ in range(world)]
        dist.all_gather(both, got)
        assert torch.equal(both[0], both[1])
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put((rank, traceback.format_exc()))


def test_head_sharding_world2_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    for rank, msg in res:
        assert msg == "ok", f"rank {rank}:\n{msg}"


def test_heads_must_divide():
    from freesolo_b200.parallel import HeadShard
    with pytest.raises(ValueError):
        HeadShard(16, 64, 0, 3)
    sh = HeadShard(16, 64, 3, 8)
    assert (sh.h0, sh.h1, sh.dl, sh.d) == (6, 8, 128, 1024)
