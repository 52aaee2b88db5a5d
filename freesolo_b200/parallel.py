"""Head sharding of one long sequence across the GPUs of a box: one process per GPU, NCCL over NVLink.

Everything on the long-range path is strictly per (batch, head): chunk statistics, forests, beams, pools, windows, int8
stores, readout. Rank r owns heads [r H/g, (r+1) H/g): the rows of W_q / W_k / W_v that produce them, their KV state, their
slices of the per-head parameters. The single exchange step of a layer is an all-gather of the head outputs (B, N, H/g D)
-> (B, N, d) in front of a replicated W_o; norms, FFN, embeddings and the LM head are replicated, so every rank computes the
same residual stream and no second collective is needed. (The reference has no multi-GPU path; this follows the partition
its per-head data layout allows.)

In the captured decode step that exchange is one small kernel of this library per rank and layer over peer memory
(`PeerExchange`: stores + a flag into slabs the ranks opened from one another through CUDA IPC, a bounded wait on the rank's
own flags); the prefill, and a decoder built with FSATTN_PEER_GATHER=0, use the NCCL all-gather.

Batch sharding needs no code here: sequences are independent, each rank runs its own sequences with a full replica and the
host gathers the sampled tokens.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

PER_HEAD = ("sel_scale", "log_sigma", "long_range_scale", "fsb_tau", "fsb_tau_union")


class HeadShard:
    """Index arithmetic of the partition (no device code): which heads a rank owns and how tensors are cut and joined."""

    def __init__(self, n_heads: int, head_dim: int, rank: int, world: int):
        if n_heads % world:
            raise ValueError(f"{n_heads} heads do not split over {world} ranks")
        self.H, self.D, self.rank, self.world = n_heads, head_dim, rank, world
        self.Hl = n_heads // world
        self.h0, self.h1 = rank * self.Hl, (rank + 1) * self.Hl
        self.d, self.dl = n_heads * head_dim, self.Hl * head_dim

    def qkv_rows(self, w_qkv: torch.Tensor) -> torch.Tensor:
        """Rows of the fused (3d, d_in) projection weight that produce this rank's heads: (3 dl, d_in), q then k then v."""
        d, lo, hi = self.d, self.h0 * self.D, self.h1 * self.D
        return torch.cat([w_qkv[i * d + lo:i * d + hi] for i in range(3)], dim=0).contiguous()

    def per_head(self, t: torch.Tensor) -> torch.Tensor:
        return t[self.h0:self.h1]

    def gather(self, y_local: torch.Tensor, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
        """All-gather of head outputs: y_local (B, N, dl) (or (B, dl)) -> (B, N, d) with heads in global order."""
        lead = y_local.shape[:-1]
        rows = math.prod(lead) if len(lead) else 1
        flat = torch.empty(self.world * rows, self.dl, dtype=y_local.dtype, device=y_local.device)
        dist.all_gather_into_tensor(flat, y_local.reshape(rows, self.dl).contiguous(), group=group)
        buf = flat.view(self.world, rows, self.dl)
        if rows == 1 and out is not None:
            out.view(-1).copy_(buf.view(-1))                     # rank-major == head-major for a single row
            return out
        y = buf.permute(1, 0, 2).reshape(*lead, self.d)
        if out is not None:
            out.copy_(y)
            return out
        return y


class _RawBytes:
    """A device address as something torch.as_tensor can wrap (the CUDA array interface)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 2}


class PeerExchange:
    """The per-layer exchange of head outputs of a decode step over peer memory (csrc/peer_gather.cu).

    One slab per rank, allocated by the library with cudaMalloc and zeroed: the receive area (8-byte words of data + flag,
    per slot, call parity and source rank), n_slots call counters, one status word. The ranks swap the slabs' IPC handles
    once (a collective over `group`) and open them; after that a layer's exchange is one launch per rank and no library
    call. `status()` is non-zero if a wait ever ran out (bit p: rank p's rows did not arrive within `timeout_ms`)."""

    def __init__(self, shard: HeadShard, B: int, n_slots: int, device, group=None, timeout_ms: float = 1000.0, exchange=None):
        import ctypes as C
        from . import lib as L
        self.shard, self.B, self.n_slots, self.group = shard, int(B), int(n_slots), group
        self.dev = torch.device(device)
        self.timeout_ns = int(timeout_ms * 1e6)
        lib = L.load()
        up = lambda n: (n + 255) // 256 * 256
        self.off_epoch = up(int(lib.fsattn_peer_ll_bytes(self.B, shard.dl, shard.world, self.n_slots)))
        self.off_status = self.off_epoch + up(self.n_slots * 4)
        self.nbytes = self.off_status + 256
        with torch.cuda.device(self.dev):
            ptr = C.c_void_p()
            L.check(lib.fsattn_peer_alloc(self.nbytes, C.byref(ptr)), "fsattn_peer_alloc")
            self.ptr = int(ptr.value)
            h = C.create_string_buffer(L.PEER_HANDLE_BYTES)
            L.check(lib.fsattn_peer_export(self.ptr, h), "fsattn_peer_export")
            mine = bytes(h.raw)
            if exchange is not None:                  # a caller's own channel: the handles of all ranks in rank order
                handles = exchange(mine)
            elif shard.world == 1:
                handles = [mine]
            else:
                handles = [None] * shard.world
                dist.all_gather_object(handles, mine, group=group)
            self.base, self._opened = [], []
            for r, hr in enumerate(handles):
                if r == shard.rank:
                    self.base.append(self.ptr)
                    continue
                q = C.c_void_p()
                L.check(lib.fsattn_peer_open(hr, C.byref(q)), "fsattn_peer_open")
                self.base.append(int(q.value))
                self._opened.append(int(q.value))
            raw = torch.as_tensor(_RawBytes(self.ptr, self.nbytes), device=self.dev)
        self._raw = raw
        self.epoch = raw[self.off_epoch:self.off_epoch + self.n_slots * 4].view(torch.int32)
        self._status = raw[self.off_status:self.off_status + 4].view(torch.int32)
        self.y = torch.zeros(self.B, shard.d, dtype=torch.bfloat16, device=self.dev)      # the gathered rows W_o reads
        a = L.PeerGather()
        for r, b in enumerate(self.base):
            a.ll_dst[r] = b
        a.y_out = self.y.data_ptr()
        a.epoch, a.status = self.ptr + self.off_epoch, self.ptr + self.off_status
        a.B, a.dl, a.rank, a.world = self.B, shard.dl, shard.rank, shard.world
        a.timeout_ns = self.timeout_ns
        self._args = a

    def gather(self, y_local: torch.Tensor, slot: int, pdl: bool = True) -> torch.Tensor:
        """y_local (B, dl) bf16 -> the gathered rows (B, d): valid when the launch has completed with status 0."""
        import ctypes as C
        from . import lib as L
        from .ops import _stream
        if not (y_local.is_cuda and y_local.dtype == torch.bfloat16 and y_local.is_contiguous()
                and y_local.numel() == self.B * self.shard.dl and 0 <= slot < self.n_slots):
            raise ValueError("PeerExchange.gather: y_local must be a contiguous (B, dl) bf16 CUDA tensor and slot < n_slots")
        a = self._args
        a.y_local = y_local.data_ptr()
        a.slot, a.pdl = slot, int(pdl)
        L.check(L.load().fsattn_peer_gather(C.byref(a), _stream(y_local)), "fsattn_peer_gather")
        return self.y

    def status(self) -> int:
        return int(self._status.item())

    def close(self):
        """Unmap the peers' slabs, then (after every rank has done so) free this rank's. A collective over `group`."""
        from . import lib as L
        if self.ptr is None:
            return
        torch.cuda.synchronize(self.dev)
        lib = L.load()
        with torch.cuda.device(self.dev):
            for q in self._opened:
                lib.fsattn_peer_close(q)
            self._opened = []
            if self.shard.world > 1 and dist.is_initialized():
                dist.barrier(group=self.group)
            self.epoch = self._status = self._raw = None
            lib.fsattn_peer_free(self.ptr)
        self.ptr = None


class ShardedFSAttn(nn.Module):
    """An FSAttn layer cut to this rank's heads. The kernels run through an inner FSAttn of H/g heads (whose own projection
    weights are unused); this module owns the local rows of the fused QKV weight and the replicated W_o."""

    def __init__(self, full, rank: int, world: int, group=None):
        super().__init__()
        from .fsattn import FSAttn
        self.shard = HeadShard(full.n_heads, full.head_dim, rank, world)
        self.group = group
        sh = self.shard
        kw = dict(full._ctor_kwargs)
        self.inner = FSAttn(sh.dl, sh.Hl, **kw)
        dev, dt = full.W_o.weight.device, full.W_o.weight.dtype
        self.inner.to(dev)
        with torch.no_grad():
            for name in PER_HEAD:
                src = getattr(full, name, None)
                dst = getattr(self.inner, name, None)
                if src is not None and dst is not None:
                    dst.data = sh.per_head(src.data).clone().to(dst.dtype)
            self.inner.lr_norm.scale.data = full.lr_norm.scale.data.clone()
            if full.use_rope:
                self.inner.rope = full.rope                    # tables are shared
            w_qkv, _ = full._ensure_qkv_cache()
            self.w_qkv = nn.Parameter(sh.qkv_rows(w_qkv.data).to(dt), requires_grad=False)
        for p in ("W_q", "W_k", "W_v", "W_o"):                 # the inner layer's own projections are never used
            getattr(self.inner, p).weight.data = torch.empty(0, device=dev, dtype=dt)
        self.W_o = full.W_o
        self.d_model, self.n_heads, self.head_dim = full.d_model, full.n_heads, full.head_dim
        self.fsb_enabled, self._cell_block, self.window_size = full.fsb_enabled, full._cell_block, full.window_size
        self.rope = getattr(full, "rope", None)

    # ---- what GraphedDecoder and make_caches ask of a layer ----------------------------------------------------------
    def _ensure_qkv_cache(self):
        return self.w_qkv, self.d_model

    def graph_decode_attn(self, qkv, buf, y=None, pdl=True):
        """qkv (B, 3 dl) of this rank's heads -> W_o's input (B, d) after the all-gather (captured with the step)."""
        y_local = self.inner.graph_decode_attn(qkv, buf, pdl=pdl)
        px = buf.get("peer")
        if px is not None:                          # one launch over peer memory; returns the slot's own gathered buffer
            return px.gather(y_local.view(y_local.shape[0], -1), buf["peer_slot"], pdl=pdl)
        return self.shard.gather(y_local, self.group, out=y)

    @torch.no_grad()
    def forward(self, x, mask=None, cache=None, pre_norm=None):
        if cache is None:
            raise NotImplementedError("cached inference only")
        sh = self.shard
        B, N, _ = x.shape
        if pre_norm is None:
            qkv = F.linear(x, self.w_qkv)
        else:                                 # long prefill: the block's input norm applied here in token chunks (see FSAttn.forward)
            chunk = self.inner.PROJ_CHUNK
            qkv = torch.empty(B, N, self.w_qkv.shape[0], dtype=x.dtype, device=x.device)
            for s0 in range(0, N, chunk):
                qkv[:, s0:s0 + chunk] = F.linear(pre_norm(x[:, s0:s0 + chunk]), self.w_qkv)
        q, k, v = (qkv[..., i * sh.dl:(i + 1) * sh.dl].view(B, N, sh.Hl, sh.D).transpose(1, 2) for i in range(3))
        a = self.inner
        a._assert_cacheable(phase="prefill" if (cache.pos == 0 and N > 1) else "decode")
        if cache.pos == 0 and N > 1:
            y_local = a._prefill(q, k, v, cache)
        else:
            ys = [a._decode_one(q[:, :, t], k[:, :, t], v[:, :, t], cache) for t in range(N)]
            y_local = torch.stack(ys, dim=1) if N > 1 else ys[0].unsqueeze(1)
        return self.W_o(sh.gather(y_local, self.group))


def shard_model_heads(model, rank: int, world: int, group=None):
    """Replace every block's attention layer by its head shard (in place); the rest of the model stays replicated."""
    for blk in model.blocks:
        blk.attn.fsattn = ShardedFSAttn(blk.attn.fsattn, rank, world, group)
    return model
