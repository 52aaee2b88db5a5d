"""Serving plumbing around the attention hot path: the FreeSoloLM trunk (embedding, RMSNorm, SwiGLU, tied LM head; module
and parameter names of experiments/scaling/model.py so a reference state dict loads), the serve presets of
experiments/scaling/bench_efficiency.py:72-87, a cached prefill driver and the whole-step CUDA-graph decoder
(experiments/scaling/decode_graph.py:27-289).

The trunk's dense layers are library GEMMs (cuBLAS through torch); the attention layer is ``fsattn.FSAttn``.
"""
from __future__ import annotations

import os

import torch
import torch.nn as nn
import torch.nn.functional as F

from .fsattn import FSAttn, FSKVCache, make_caches
from .fsattn import kv_bounded as _kvb
from .fsattn.attention import CACHE_GEN as _CACHE_GEN

MODEL_CONFIGS = {   # experiments/scaling/model.py:38-80 (vocab 32000 as the benchmark loads them)
    "debug": dict(d_model=256, n_layers=4, n_heads=4, d_ff=688, max_seq_len=1024, vocab_size=32000),
    "340m": dict(d_model=1024, n_layers=24, n_heads=16, d_ff=2816, max_seq_len=2048, vocab_size=32000),
    "800m": dict(d_model=1536, n_layers=24, n_heads=16, d_ff=4224, max_seq_len=2048, vocab_size=32000),
}


def serve_kwargs(serve: str, fsb_union_tau_quantile: float = 0.0) -> dict:
    """experiments/scaling/bench_efficiency.py:72-87."""
    kw = dict(window_size=512, long_range_variant="cell_topk", cell_stride=32, cell_topk=4, cell_select="score",
              sel_strict_causal=1, use_rope=True, fs_uniform_sr=True, rope_long_range=False)
    if serve == "sparse":
        kw.update(cell_prune_kernel=1, cell_prune_pool=64, cell_prune_window=8, cell_prune_blkchunk=16)
    elif serve == "fsb":
        kw.update(cell_prune_kernel=0, fsb_enabled=True, fsb_policy="fixed", fsb_width=16, fsb_delta=0,
                  fsb_node_score="bound", fsb_bound_radius_coef=8.0, fsb_tree="forest", fsb_read_top=4,
                  fsb_rerank_score="lse_pos", fsb_rerank_query="raw", fsb_union_width=16)
        if fsb_union_tau_quantile > 0:
            kw["fsb_union_tau_quantile"] = fsb_union_tau_quantile
    else:
        kw.update(cell_prune_kernel=0)
    return kw


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        if x.is_cuda and x.dtype == torch.bfloat16 and self.weight.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0 and x.numel() > 0:
            from . import ops
            return ops.rms_norm(x, self.weight, self.eps)              # one read, one write
        return F.rms_norm(x, (x.shape[-1],), self.weight, self.eps)


class SwiGLU(nn.Module):
    def __init__(self, d_model: int, d_ff: int):
        super().__init__()
        self.w_gate = nn.Linear(d_model, d_ff, bias=False)
        self.w_up = nn.Linear(d_model, d_ff, bias=False)
        self.w_down = nn.Linear(d_ff, d_model, bias=False)

    def _ensure_gu_cache(self):
        """One fused (2*d_ff, d) weight the gate and up weights are views of (experiments/scaling/model.py:111-125)."""
        wg, wu = self.w_gate.weight, self.w_up.weight
        key = (wg.data_ptr(), wg._version, wu.data_ptr(), wu._version, wg.dtype)
        c = getattr(self, "_w_gu_cache", None)
        if c is None or c[0] != key:
            d_ff = wg.shape[0]
            gu = torch.cat([wg.data, wu.data], dim=0)
            self.w_gate.weight.data = gu[:d_ff]
            self.w_up.weight.data = gu[d_ff:]
            wg, wu = self.w_gate.weight, self.w_up.weight
            c = ((wg.data_ptr(), wg._version, wu.data_ptr(), wu._version, wg.dtype), gu)
            self._w_gu_cache = c
            _CACHE_GEN[0] += 1
        return c[1], self.w_gate.weight.shape[0]

    def forward(self, x):
        gu_w, d_ff = self._ensure_gu_cache()
        gu = F.linear(x, gu_w)
        if gu.is_cuda and gu.dtype == torch.bfloat16 and d_ff % 8 == 0:
            from . import ops
            return self.w_down(ops.swiglu(gu))                      # one elementwise pass, same roundings
        return self.w_down(F.silu(gu[..., :d_ff]) * gu[..., d_ff:])


class AttentionWithRoPE(nn.Module):
    def __init__(self, d_model, n_heads, max_seq_len, attn_type="fsattn", causal=True, layer_idx=0, **attn_kwargs):
        super().__init__()
        if attn_type != "fsattn":
            raise ValueError(f"attn_type {attn_type!r} is not part of this build")
        self.attn_type = attn_type
        use_rope = attn_kwargs.pop("use_rope", True)
        self.fsattn = FSAttn(d_model, n_heads, causal=causal, bias=False, use_rope=use_rope, max_seq_len=max_seq_len,
                             **attn_kwargs)

    def forward(self, x, cache=None, pre_norm=None):
        return self.fsattn(x, cache=cache, pre_norm=pre_norm)


class TransformerBlock(nn.Module):
    def __init__(self, d_model, n_heads, d_ff, max_seq_len, attn_type="fsattn", layer_idx=0, **attn_kwargs):
        super().__init__()
        self.ln1 = RMSNorm(d_model)
        self.attn = AttentionWithRoPE(d_model, n_heads, max_seq_len, attn_type=attn_type, causal=True, layer_idx=layer_idx,
                                      **attn_kwargs)
        self.ln2 = RMSNorm(d_model)
        self.ffn = SwiGLU(d_model, d_ff)

    def forward(self, x, cache=None):
        """RMSNorm -> attention -> residual -> RMSNorm -> SwiGLU -> residual (experiments/scaling/model.py:211-237); the
        FFN of a long prefill runs in token chunks to bound its intermediate."""
        N = x.shape[1]
        chunk = 16384
        if N > chunk and not torch.is_grad_enabled():
            # long prefill: the input norm runs inside the attention in token chunks, the residuals are added in place
            # (x is this forward's own activation: the embedding output or the previous block's result), the FFN in chunks
            x.add_(self.attn(x, cache=cache, pre_norm=self.ln1))
            for s0 in range(0, N, chunk):
                xc = x[:, s0:s0 + chunk]
                xc.add_(self.ffn(self.ln2(xc)))
            return x
        x = x + self.attn(self.ln1(x), cache=cache)
        return x + self.ffn(self.ln2(x))


class FreeSoloLM(nn.Module):
    """experiments/scaling/model.py:248-359, inference part."""

    def __init__(self, vocab_size=32000, d_model=1024, n_layers=24, n_heads=16, d_ff=2816, max_seq_len=2048,
                 attn_type="fsattn", **attn_kwargs):
        super().__init__()
        self.d_model, self.vocab_size = d_model, vocab_size
        self.tok_emb = nn.Embedding(vocab_size, d_model)
        self.blocks = nn.ModuleList([TransformerBlock(d_model, n_heads, d_ff, max_seq_len, attn_type, layer_idx=i,
                                                      **attn_kwargs) for i in range(n_layers)])
        self.ln_final = RMSNorm(d_model)
        self.lm_head = nn.Linear(d_model, vocab_size, bias=False)
        self.lm_head.weight = self.tok_emb.weight
        self._init_weights()

    def _init_weights(self):
        """N(0, 0.02) for every matrix (experiments/scaling/model.py:318-323)."""
        for name, p in self.named_parameters():
            if p.dim() > 1 and "tok_emb" not in name and "long_range_scale" not in name:
                nn.init.normal_(p, mean=0.0, std=0.02)
        nn.init.normal_(self.tok_emb.weight, mean=0.0, std=0.02)

    @classmethod
    def from_config(cls, name: str, **kwargs):
        cfg = dict(MODEL_CONFIGS[name])
        cfg.update(kwargs)
        return cls(**cfg)

    def count_params(self) -> int:
        return sum(p.numel() for p in self.parameters())


def extend_rope_cache(model, n: int):
    for blk in model.blocks:
        blk.attn.fsattn.rope.tables_bf16(n)


@torch.no_grad()
def trunk_cached(model, idx, caches, last_n: int | None = None):
    """experiments/scaling/kv_cache.py:541-547: embedding, blocks with their caches, final norm."""
    x = model.tok_emb(idx)
    for i, blk in enumerate(model.blocks):
        x = blk(x, cache=caches[i])
    if last_n is not None and x.shape[1] > last_n:
        x = x[:, -last_n:].contiguous()
    return model.ln_final(x)


def lm_head(model, hidden):
    """Last-token logits with the tied head (experiments/scaling/longctx_infer.py:281-290 under bf16 autocast)."""
    return F.linear(hidden, model.lm_head.weight)


class GraphedDecoder:
    """Whole-step CUDA-graph greedy decoder for FS-L models (experiments/scaling/decode_graph.py:27-289), any batch size.

    One graph replay per token and nothing else: the token id, the position and every layer's KV bookkeeping (row append,
    cell close, top-P refresh, slot frees) live on the device, so consecutive steps need no host work between replays.
    kv: "bounded" (default, as the reference's FSL_KV_BOUNDED=1), "int8" or "bf16"."""

    def __init__(self, model, prompt_ids, Lmax, device="cuda", dtype=torch.bfloat16, kv="bounded", eager_steps=2):
        self.m = model
        self.dev = torch.device(device)
        self.dt = dtype
        self.Lmax = int(Lmax)
        self.blocks = list(model.blocks)
        self.attn = [b.attn.fsattn for b in self.blocks]
        self.attn_core = [getattr(a, "inner", a) for a in self.attn]      # the layer the kernels run through (head shards wrap it)
        self.prompt = prompt_ids
        self.kv = kv
        self.cache = None
        self.graph = None
        self.eager_steps = eager_steps
        self._steps = 0
        self.bounded_kv = False

    @torch.no_grad()
    def prefill(self):
        m = self.m
        seq = self.prompt.to(self.dev)
        if seq.dim() == 1:
            seq = seq.view(1, -1)
        B, P0 = seq.shape
        extend_rope_cache(m, self.Lmax + 8)
        self.cache = make_caches(m, reserve=max(0, self.Lmax - P0))
        kv = self.kv
        self.fsb = any(a.fsb_enabled for a in self.attn)
        self.dense = any(a._is_dense_lr() and not a.fsb_enabled for a in self.attn_core)
        if kv == "bounded" and (self.fsb or self.dense):
            kv = "int8"      # FS-B and the dense variant read any completed cell: they keep the full (int8) store
        if kv == "bounded" and not (P0 >= self.attn[0].window_size and _kvb.supported(self.attn_core, self.dt, self.dev)):
            kv = "int8"      # prompts shorter than the window keep the full store (decode_graph.py:89-93)
        for c in self.cache:
            if kv == "bounded":
                c.enable_bounded()
            elif kv == "int8":
                c.enable_int8()
        self.bounded_kv = kv == "bounded"
        hidden = trunk_cached(m, seq, self.cache, last_n=1)
        logits = lm_head(m, hidden[:, -1])
        self.prefill_logits = logits                # (B, V): the last prompt token's logits
        self.tok = logits.argmax(dim=-1).view(B, 1)
        self.pos = P0
        self.pos_t = torch.full((), P0, dtype=torch.int64, device=self.dev)
        self.bufs = [{"pos_t": self.pos_t, "cache": c} for c in self.cache]
        # head shards: the per-layer exchange of head outputs as one launch over peer memory (parallel.PeerExchange; a
        # collective set-up over the shard's group); FSATTN_PEER_GATHER=0 keeps the NCCL all-gather in the step
        self.peer = None
        shard = getattr(self.attn[0], "shard", None)
        if shard is not None and shard.world > 1 and os.environ.get("FSATTN_PEER_GATHER", "1") == "1":
            import torch.distributed as dist
            from .parallel import PeerExchange
            try:
                self.peer = PeerExchange(shard, B, len(self.blocks), self.dev, group=self.attn[0].group)
            except RuntimeError as e:                 # e.g. the box does not let the ranks open one another's memory
                self.peer_error = str(e)
            # the ranks agree: one that could not map its peers sends every rank back to the library all-gather
            ok = torch.tensor([int(self.peer is not None)], device=self.dev)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.attn[0].group)
            if int(ok.item()) == 0:
                self.peer = None
            else:
                for i, b in enumerate(self.bufs):
                    b["peer"], b["peer_slot"] = self.peer, i
        for blk in self.blocks:
            blk.ffn._ensure_gu_cache()
        d, f = m.d_model, self.blocks[0].ffn.w_gate.weight.shape[0]
        z = dict(dtype=torch.bfloat16, device=self.dev)
        self.x = torch.zeros(B, d, **z)             # residual stream of the current token
        self.qkv = torch.zeros(B, self.attn[0]._ensure_qkv_cache()[0].shape[0], **z)      # 3 d, or 3 d / g for a head shard
        self.y = torch.zeros(B, d, **z)
        self.act = torch.zeros(B, f, **z)
        self.logits = torch.zeros(B, m.vocab_size, **z)
        # Fused per-layer trunk kernel (opt-in): three barrier counters per layer (zeroed once per step), one status word.
        # Off by default: on a B200 a grid-wide barrier plus the restaging of the activations costs about as much as a
        # programmatic dependent launch, and the 341M step measured 0.79 ms fused against 0.63 ms with separate launches.
        self.fused_trunk = os.environ.get("FSATTN_TRUNK_FUSED", "0") == "1"
        self.tl_bar = torch.zeros(len(self.blocks), 4, dtype=torch.int32, device=self.dev)
        self.tl_status = torch.zeros(1, dtype=torch.int32, device=self.dev)
        return self.tok

    def _trunk_step(self):
        """One token through the model: reads self.tok and pos_t, overwrites self.tok with the greedy next token and
        advances pos_t, all on the device. Per layer five launches of this library: RMSNorm+QKV projection, the fused
        attention step, W_o + residual, RMSNorm + gate/up + SwiGLU, down projection + residual (each projection kernel
        starts streaming its weights before its producer has finished: programmatic dependent launch)."""
        from . import ops
        m = self.m
        x = self.x
        pdl = os.environ.get("FSATTN_PDL", "1") == "1"
        if x.shape[0] > 8:
            x.copy_(m.tok_emb(self.tok).view(x.shape))
            return self._trunk_step_batched()
        if self.fused_trunk:
            x.copy_(m.tok_emb(self.tok).view(x.shape))
            return self._trunk_step_fused(pdl)
        ops.embed_rows(self.tok, m.tok_emb.weight, x)
        for i, blk in enumerate(self.blocks):
            a = self.attn[i]
            wqkv, _ = a._ensure_qkv_cache()
            ops.trunk_gemv(x, wqkv, norm_w=blk.ln1.weight, eps=blk.ln1.eps, out=self.qkv, pdl=pdl)
            y = a.graph_decode_attn(self.qkv, self.bufs[i], y=self.y, pdl=pdl)      # self.y, or a head shard's gathered buffer
            ops.trunk_gemv(y, a.W_o.weight, res=x, out=x, pdl=pdl)
            wgu, _ = blk.ffn._ensure_gu_cache()
            ops.trunk_gemv(x, wgu, norm_w=blk.ln2.weight, eps=blk.ln2.eps, swiglu=True, out=self.act, pdl=pdl)
            ops.trunk_gemv(self.act, blk.ffn.w_down.weight, res=x, out=x, pdl=pdl)
        ops.trunk_gemv(x, m.lm_head.weight, norm_w=m.ln_final.weight, eps=m.ln_final.eps, out=self.logits, pdl=pdl)
        ops.argmax_advance(self.logits, self.tok, self.pos_t)

    def _trunk_step_fused(self, pdl: bool):
        """The same step with two launches per layer: the attention step, then ONE cooperative kernel for everything up to
        the next layer's QKV projection (W_o + residual, RMSNorm + gate/up + SwiGLU, down + residual, RMSNorm + QKV; after
        the last layer the final norm + LM head), its phases separated by grid-wide barriers instead of launches."""
        from . import ops
        m, x = self.m, self.x
        nL = len(self.blocks)
        self.tl_bar.zero_()
        a0 = self.attn[0]
        ops.trunk_gemv(x, a0._ensure_qkv_cache()[0], norm_w=self.blocks[0].ln1.weight, eps=self.blocks[0].ln1.eps, out=self.qkv, pdl=pdl)
        for i, blk in enumerate(self.blocks):
            a = self.attn[i]
            y = a.graph_decode_attn(self.qkv, self.bufs[i], y=self.y, pdl=pdl)
            if i + 1 < nL:
                nb = self.blocks[i + 1]
                nxt = dict(norm_next_w=nb.ln1.weight, eps_next=nb.ln1.eps, w_next=self.attn[i + 1]._ensure_qkv_cache()[0], out_next=self.qkv)
            else:
                nxt = dict(norm_next_w=m.ln_final.weight, eps_next=m.ln_final.eps, w_next=m.lm_head.weight, out_next=self.logits)
            ops.trunk_layer(x, y, a.W_o.weight, blk.ln2.weight, blk.ln2.eps, blk.ffn._ensure_gu_cache()[0], self.act,
                            blk.ffn.w_down.weight, self.tl_bar[i], self.tl_status, pdl=pdl, **nxt)
        self.tok.copy_(self.logits.argmax(dim=-1, keepdim=True))
        self.pos_t.add_(1)

    def peer_status(self) -> int:
        """Head shards: non-zero if a wait for a peer's head outputs ever ran out (bit p = rank p; one host sync)."""
        return 0 if self.peer is None else self.peer.status()

    def trunk_status(self) -> int:
        """Non-zero if a grid barrier of the fused layer kernel ever ran out of its bound (one host sync)."""
        return int(self.tl_status.item())

    def launches_per_step(self) -> int:
        """Kernels of this library per decode step (batch <= 8): the attention step and the fused rest of the layer (plus
        the FS-B selection), the first QKV projection; without the fused kernel 5 per layer (6 with FS-B) + the head, the
        embedding lookup and the argmax."""
        nL = len(self.blocks)
        if self.fused_trunk and self.x.shape[0] <= 8:
            return 2 * nL + 1 + (nL if (self.fsb or self.dense) else 0)
        return 5 * nL + 3 + (nL if (self.fsb or self.dense) else 0)       # + the embedding lookup and the argmax / advance

    def _trunk_step_batched(self):
        """More than 8 sequences per step: the projections are real GEMMs (weights read once for all rows), so they go to
        the library (cuBLAS through torch) instead of the row-streaming GEMV kernels; the attention step is the same
        single launch per layer, now bandwidth-bound on the sequences' KV state."""
        m, x = self.m, self.x
        for i, blk in enumerate(self.blocks):
            a = self.attn[i]
            wqkv, _ = a._ensure_qkv_cache()
            torch.matmul(blk.ln1(x), wqkv.t(), out=self.qkv)
            y = a.graph_decode_attn(self.qkv, self.bufs[i], y=self.y, pdl=False)
            x.add_(F.linear(y, a.W_o.weight))
            wgu, f = blk.ffn._ensure_gu_cache()
            gu = F.linear(blk.ln2(x), wgu)
            x.add_(F.linear(F.silu(gu[:, :f]) * gu[:, f:], blk.ffn.w_down.weight))
        torch.matmul(m.ln_final(x), m.lm_head.weight.t(), out=self.logits)
        self.tok.copy_(self.logits.argmax(dim=-1, keepdim=True))
        self.pos_t.add_(1)

    def _graph_inputs(self) -> list:
        """The cached tensors whose device addresses a captured step bakes in and that only module-level caches own: the
        bf16 RoPE tables, the per-head parameter tuple and the fused projection weights of every layer."""
        keep = []
        for a, blk in zip(self.attn_core, self.blocks):
            keep.append(a.rope._bf16)
            keep.append(getattr(a, "_head_params", None))
            keep.append(getattr(a, "_w_qkv_cache", None))
            keep.append(getattr(blk.ffn, "_w_gu_cache", None))
        return keep

    @torch.no_grad()
    def _capture(self):
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._trunk_step()
        # the graph holds raw pointers into these: keep them alive for its lifetime, and notice when a cache replaces one
        # (a longer RoPE table, a changed parameter) so that the step is captured again instead of reading the old buffer
        self._graph_keep = self._graph_inputs()
        self._graph_gen = _CACHE_GEN[0]

    def _graph_stale(self) -> bool:
        if _CACHE_GEN[0] == self._graph_gen:           # nothing was rebuilt anywhere since the last look
            return False
        stale = any(x is not y for x, y in zip(self._graph_keep, self._graph_inputs()))
        if not stale:
            self._graph_gen = _CACHE_GEN[0]
        return stale

    @torch.no_grad()
    def step(self):
        """Advance one token; returns the device tensor holding the new token ids (B,1)."""
        if self.pos + 1 >= self.Lmax:
            raise RuntimeError(f"decoder sized for {self.Lmax} positions")
        if self.fsb and self.pos % self.attn[0]._cell_block == 0 or self.fsb and self._steps == 0:
            # FS-B (experiments/scaling/decode_graph.py:499-541, src/fsattn/fsb_tree.py:3598-3674): at a query-block
            # change every layer's forests take in the cells completed before the block and rebuild their spines, as
            # plain launches ahead of the replay; buffers keep their addresses, so the graph is never re-captured
            for a, c in zip(self.attn_core, self.cache):
                if a.fsb_enabled:
                    c.fsb_block_change(self.pos, a)
        if self.graph is not None and self._graph_stale():
            self.graph = None
        if self.graph is None and self._steps >= self.eager_steps:
            self._capture()
        if self.graph is None:
            self._trunk_step()
        else:
            self.graph.replay()
        self._steps += 1
        self.pos += 1
        return self.tok

    @torch.no_grad()
    def step_host(self, tok_host: torch.Tensor, out_host: torch.Tensor):
        """One token end to end for a caller whose token ids live on the host: the id in `tok_host` (pinned (B,1) int64) goes
        to the device, the step runs, and the sampled id lands in `out_host` (pinned (B,1) int64) - one graph launch whose
        first and last nodes are the two copies. The caller synchronises the stream before reading `out_host`. The same
        tensors must be passed on every call (their addresses are part of the captured graph)."""
        if self.graph is None or self.fsb and self.pos % self.attn[0]._cell_block == 0:
            # not captured yet, or a step with host-side work (an FS-B block change): the plain sequence
            self.tok.copy_(tok_host, non_blocking=True)
            self.step()
            out_host.copy_(self.tok, non_blocking=True)
            return
        key = (tok_host.data_ptr(), out_host.data_ptr())
        if getattr(self, "_host_graph_key", None) != key or self._host_graph_src is not self.graph:
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.tok.copy_(tok_host, non_blocking=True)
                self._trunk_step()
                out_host.copy_(self.tok, non_blocking=True)
            self._host_graph, self._host_graph_key, self._host_graph_src = g, key, self.graph
        if self._graph_stale():
            self.graph = None
            self._host_graph_key = None
            return self.step_host(tok_host, out_host)
        if self.pos + 1 >= self.Lmax:
            raise RuntimeError(f"decoder sized for {self.Lmax} positions")
        self._host_graph.replay()
        self._steps += 1
        self.pos += 1

    def sync_caches(self):
        for c in self.cache:
            c.pos = self.pos
            c._ncell = self.pos // c.s

    def fsb_bytes(self) -> int:
        return sum(c.fsb.nbytes() for c in self.cache if getattr(c, "fsb", None) is not None)

    def kv_faults(self) -> tuple:
        """(slot overflows, readable cells without a slot, rejected indices) over all layers; one host sync."""
        tot = torch.stack([c.state.status for c in self.cache]).sum(0).tolist()
        return int(tot[0]), int(tot[1]), int(tot[2])

    def kv_bytes(self) -> int:
        return sum(c.state.nbytes() for c in self.cache)


class GraphedPrefiller:
    """Whole-forward CUDA-graph prefill at a fixed (B, L) shape (experiments/scaling/decode_graph.py:623-709): the token
    input, every layer's cache buffers and the outputs are static, one eager pass allocates the cache state and opts the
    kernels into their shared-memory sizes, then the whole prefill - embedding, every block with its cache, final norm,
    last-token logits - is captured once and replayed for every prompt of that shape. At short contexts the prefill is a
    chain of short launches, and the replay removes the host's share of it; the kernels and their results are the eager
    path's. `retain_kv=False` is the reference's prefill-benchmark protocol (chunk statistics only, no KV store fill).
    kv: None keeps the caches' default store, "int8" / "bounded" select one before the first pass."""

    def __init__(self, model, L: int, B: int = 1, device="cuda", dtype=torch.bfloat16, reserve: int = 0,
                 tail_tokens: int = 64, retain_kv: bool = True, kv: str | None = None):
        self.m = model
        self.dev = torch.device(device)
        self.dt = dtype
        self.B, self.L, self.reserve = int(B), int(L), int(reserve)
        self.tail_tokens = min(int(tail_tokens), self.L) if tail_tokens > 0 else 1
        self.retain_kv = bool(retain_kv)
        self.kv = kv
        self.graph = None
        self.x_static = self.static_logits = self.static_tail = self.cache = None

    def _body(self):
        for c in self.cache:
            c.pos = 0
        h = trunk_cached(self.m, self.x_static, self.cache, last_n=self.tail_tokens)
        tail = h[:, -self.tail_tokens:, :].clone()
        return lm_head(self.m, h[:, -1]), tail

    @torch.no_grad()
    def capture(self, sample_ids: torch.Tensor | None = None):
        m = self.m
        extend_rope_cache(m, self.L + max(self.reserve, 256))
        self.x_static = torch.zeros((self.B, self.L), dtype=torch.int64, device=self.dev)
        if sample_ids is not None:
            self.x_static.copy_(sample_ids.to(self.dev).view(self.B, self.L))
        self.cache = make_caches(m, reserve=self.reserve, linear=False, retain_kv=self.retain_kv)
        if self.retain_kv and self.kv in ("int8", "bounded"):
            for c in self.cache:
                c.enable_bounded() if self.kv == "bounded" else c.enable_int8()
        side = torch.cuda.Stream(device=self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(side):
            self._body()                       # allocates the caches' state; every later pass reuses it
        torch.cuda.current_stream(self.dev).wait_stream(side)
        torch.cuda.synchronize(self.dev)
        torch.cuda.empty_cache()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.static_logits, self.static_tail = self._body()
        return self

    @torch.no_grad()
    def run(self, prompt_ids: torch.Tensor):
        """Prefill one prompt of the captured shape; returns the last token's logits (B, V) (a static buffer)."""
        if prompt_ids.numel() != self.B * self.L:
            raise ValueError(f"GraphedPrefiller was built for prompts of shape ({self.B}, {self.L})")
        if self.graph is None:
            self.capture(prompt_ids)
        else:
            self.x_static.copy_(prompt_ids.to(self.dev).view(self.B, self.L))
        self.graph.replay()
        for c in self.cache:
            c.pos = self.L
        return self.static_logits

    @torch.no_grad()
    def tail_logits(self):
        """Logits of the last `tail_tokens` positions of the prompt run last (B, tail, V)."""
        return lm_head(self.m, self.static_tail)


@torch.no_grad()
def calibrate_fsb_tau(model, ids, quantile: float, target: str = "fsb_tau"):
    """Set every FS-B layer's admission threshold to the per-head `quantile` of the cell ceilings seen on the token ids
    `ids` (B, L): the reference's fsb_calibrate_tau (src/fsattn/fsb_tree.py:3944-3969) for one batch. target:
    'fsb_tau' (main forest) or 'fsb_tau_union' (second forest; the layer must have been built with
    fsb_union_tau_quantile > 0 for it to take effect). Returns the thresholds (layers, H)."""
    if target not in ("fsb_tau", "fsb_tau_union"):
        raise ValueError(f"calibrate_fsb_tau: target {target!r} (fsb_tau | fsb_tau_union)")
    ids = ids.view(1, -1) if ids.dim() == 1 else ids
    caches = make_caches(model)
    extend_rope_cache(model, ids.shape[1] + 8)
    trunk_cached(model, ids.to(next(model.parameters()).device), caches, last_n=1)
    taus = []
    for blk, c in zip(model.blocks, caches):
        a = blk.attn.fsattn
        if not a.fsb_enabled:
            continue
        _, ceil, ncell = c.completed_cells()
        H = ceil.shape[1]
        t = torch.quantile(ceil[:, :, :ncell].float().transpose(0, 1).reshape(H, -1), float(quantile), dim=1)
        getattr(a, target).copy_(t)
        taus.append(t)
    return torch.stack(taus) if taus else None


@torch.no_grad()
def cached_generate(model, prompt_ids, max_new_tokens, device="cuda", kv="bf16"):
    """Greedy generation through the eager per-token path (experiments/scaling/kv_cache.py:484-526)."""
    seq = prompt_ids.to(device)
    if seq.dim() == 1:
        seq = seq.view(1, -1)
    caches = make_caches(model, reserve=max_new_tokens)
    for c in caches:
        if kv == "int8":
            c.enable_int8()
        elif kv == "bounded":
            c.enable_bounded()
    extend_rope_cache(model, seq.shape[1] + max_new_tokens + 8)
    step_in = seq
    out = []
    for _ in range(max_new_tokens):
        hidden = trunk_cached(model, step_in, caches, last_n=1)
        nxt = lm_head(model, hidden[:, -1]).argmax(dim=-1)
        out.append(nxt)
        step_in = nxt.view(-1, 1)
    gen = torch.stack(out, dim=1) if out else seq[:, :0]
    return torch.cat([seq, gen], dim=1)
