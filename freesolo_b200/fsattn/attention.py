"""FSAttn: the reference's attention-layer API (src/fsattn/attention.py) on the sm_100a kernels, inference only.

    out = W_o( window_branch + long_range_scale * RMSNorm(long_range_branch) )

* window branch: causal sliding-window softmax attention over the last W+1 tokens, RoPE on Q/K only here;
* long-range branch (FS-L): per query the kk best completed 32-token cells among the block's candidate pool (top-P
  cells by ceiling + the Wc newest), scored on the un-rotated chunk-mean key, then softmax over those kk*32 tokens.

Same constructor keywords, parameter / buffer names (a reference state dict loads with ``load_state_dict``), forward
signature and cache protocol as the reference. Only the cacheable serving configuration exists here (causal, window RoPE,
un-rotated long range, strict-causal selection, uniform window): anything else raises, there is no eager fallback, and
``forward`` without a cache (training) is not provided.
"""
from __future__ import annotations

import math
import os

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops


class RMSNorm(nn.Module):
    """src/fsattn/attention.py:57-65 (parameter holder; the arithmetic is fused into the readout kernels)."""

    def __init__(self, dim: int, eps: float = 1e-8):
        super().__init__()
        self.eps = eps
        self.scale = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        rms = torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps)
        return x * rms * self.scale


class Rotary(nn.Module):
    """RoPE tables as the reference builds them with YaRN scale 1 (experiments/scaling/yarn_rope.py:36-121): fp32
    frequencies blended through the YaRN ramp (which moves some by an ulp), tables built in fp32 and cast with the
    module; grown in fp32 even after a cast to bf16."""

    def __init__(self, dim: int, max_seq_len: int, base: float = 10000.0, beta_fast: float = 32.0, beta_slow: float = 1.0):
        super().__init__()
        self.dim, self.base, self.original_max_seq_len = dim, base, max_seq_len
        self.beta_fast, self.beta_slow = beta_fast, beta_slow
        self.register_buffer("inv_freq", self._inv_freq(), persistent=False)
        self._build_cache(max_seq_len)

    def _inv_freq(self) -> torch.Tensor:
        D, base, L0 = self.dim, self.base, self.original_max_seq_len
        a = 1.0 / (base ** (torch.arange(0, D, 2, dtype=torch.float32) / D))

        def corr(rot):
            return (D * math.log(L0 / (rot * 2 * math.pi))) / (2 * math.log(base))
        low = max(math.floor(corr(self.beta_fast)), 0)
        high = min(math.ceil(corr(self.beta_slow)), D - 1)
        hi = high + 0.001 if low == high else high
        ramp = ((torch.arange(D // 2, dtype=torch.float32) - low) / (hi - low)).clamp(0.0, 1.0)
        m = 1.0 - ramp
        return a * (1.0 - m) + a * m

    def _build_cache(self, seq_len: int):
        old = getattr(self, "cos_cached", None)
        dev = self.inv_freq.device
        start = 0
        if self.inv_freq.dtype != torch.float32 and old is not None and seq_len > old.shape[0]:
            start = old.shape[0]
        inv = self._inv_freq().to(dev)
        t = torch.arange(start, seq_len, dtype=torch.float32, device=dev)
        freqs = torch.outer(t, inv)
        emb = torch.cat([freqs, freqs], dim=-1)
        cos, sin = emb.cos(), emb.sin()
        if start > 0:
            cos = torch.cat([old, cos.to(old.dtype)])
            sin = torch.cat([self.sin_cached, sin.to(old.dtype)])
        elif old is not None:
            cos, sin = cos.to(old.dtype), sin.to(old.dtype)
        self.register_buffer("cos_cached", cos, persistent=False)
        self.register_buffer("sin_cached", sin, persistent=False)
        self._bf16 = None
        CACHE_GEN[0] += 1

    def forward(self, seq_len: int):
        if seq_len > self.cos_cached.shape[0]:
            self._build_cache(seq_len)
        return self.cos_cached[:seq_len], self.sin_cached[:seq_len]

    def tables_bf16(self, need: int):
        """Contiguous bf16 (L, D) tables covering at least `need` positions (what the kernels read)."""
        if need > self.cos_cached.shape[0]:
            self._build_cache(need)
        c = self._bf16
        if c is None or c[0].shape[0] != self.cos_cached.shape[0] or c[0].device != self.cos_cached.device:
            cos, sin = self.cos_cached.to(torch.bfloat16).contiguous(), self.sin_cached.to(torch.bfloat16).contiguous()
            # every layer of a model builds the same tables (33 MB per layer at 131 072 positions): the layers share one copy
            key = (cos.device, self.dim, self.base, self.original_max_seq_len, self.beta_fast, self.beta_slow)
            sh = _SHARED_ROPE.get(key)
            if sh is not None and sh[0].shape == cos.shape and torch.equal(sh[0], cos) and torch.equal(sh[1], sin):
                cos, sin = sh
                if self.cos_cached.dtype == torch.bfloat16:      # the module's own buffers were duplicates of it
                    self.register_buffer("cos_cached", cos, persistent=False)
                    self.register_buffer("sin_cached", sin, persistent=False)
            else:
                _SHARED_ROPE[key] = (cos, sin)
            c = (cos, sin)
            self._bf16 = c
            CACHE_GEN[0] += 1
        return c


_SHARED_ROPE = {}
# Bumped whenever a module replaces one of the cached tensors a captured decode graph holds addresses of (rope tables,
# per-head parameters, fused projection weights): a decoder compares it before a replay instead of walking every layer.
CACHE_GEN = [0]


_SIDE_STREAMS = {}


def _side_stream(device):
    """One extra stream per device for work that overlaps the main stream inside a layer."""
    key = (device.type, device.index)
    if key not in _SIDE_STREAMS:
        _SIDE_STREAMS[key] = torch.cuda.Stream(device=device)
    return _SIDE_STREAMS[key]


def _pool_from_stats(kbar, ceil, slot_of, blk_start: int, s: int, P: int, Wc: int) -> dict:
    """Pool dictionary (keys of the reference's _build_decode_pool) from the visible cells' statistics. kbar is indexed by
    cell, or by slot when slot_of (B,H,cells) is given (bounded store)."""
    B, H, M_vis = ceil.shape
    Pk = min(P, M_vis)
    topP = ceil.argsort(dim=-1, descending=True, stable=True)[..., :Pk]
    hi = blk_start // s - 1
    near = (hi - torch.arange(Wc, device=ceil.device)).expand(B, H, Wc)
    cand = torch.cat([topP, near], dim=-1)
    valid = cand >= 0
    cand_c = cand.clamp(min=0)
    vis = ((cand_c + 1) * s <= blk_start) & valid
    C = cand.shape[-1]
    tri = torch.tril(torch.ones(C, C, dtype=torch.bool, device=ceil.device), diagonal=-1)
    dup = ((cand_c[..., None, :] == cand_c[..., :, None]) & tri).any(dim=-1)
    ok = vis & ~dup
    rows = cand_c if slot_of is None else torch.gather(slot_of.long(), 2, cand_c).clamp(min=0)
    D = kbar.shape[-1]
    kb = torch.gather(kbar, 2, rows[..., None].expand(B, H, C, D))
    return {"M_vis": M_vis, "C": C, "cand_c": cand_c, "ok_cell": ok, "Kbar_cand": kb, "Kbar_cand_t": kb.transpose(2, 3).contiguous(),
            "ceil_cand": torch.gather(ceil, 2, cand_c), "cen_cand": (cand_c.float() + 0.5) * s}


class FSAttn(nn.Module):
    VARIANTS = ("cell_topk",)

    def __init__(self, d_model: int, n_heads: int, window_size: int = 128, sigma_init: float = 4.0,
                 learnable_sigma: bool = True, dropout: float = 0.0, bias: bool = True, causal: bool = False,
                 long_range_variant: str = "cell_topk", use_rope: bool = False, rope_long_range: bool = True,
                 max_seq_len: int = 8192, lr_scale_mode: str = "learn", cell_stride: int = 64, cell_topk: int = 1,
                 cell_select: str = "score", **kwargs):
        super().__init__()
        # everything but the width, so that a head shard of this layer can be constructed the same way
        self._ctor_kwargs = dict(window_size=window_size, sigma_init=sigma_init, learnable_sigma=learnable_sigma,
                                 dropout=dropout, bias=bias, causal=causal, long_range_variant=long_range_variant,
                                 use_rope=use_rope, rope_long_range=rope_long_range, max_seq_len=max_seq_len,
                                 lr_scale_mode=lr_scale_mode, cell_stride=cell_stride, cell_topk=cell_topk,
                                 cell_select=cell_select, **kwargs)
        assert d_model % n_heads == 0, "d_model must be divisible by n_heads"
        assert long_range_variant in self.VARIANTS, f"Unknown variant '{long_range_variant}'"
        assert cell_select in ("score",), f"bad cell_select '{cell_select}'"
        self.d_model, self.n_heads = d_model, n_heads
        self.head_dim = d_model // n_heads
        self.scale = 1.0 / math.sqrt(self.head_dim)
        self.window_size = window_size
        self.causal = causal
        self.long_range_variant = long_range_variant
        self.disable_short_range = kwargs.get("disable_short_range", False)
        self.disable_long_range = kwargs.get("disable_long_range", False)
        self.fs_uniform_sr = bool(kwargs.get("fs_uniform_sr", False))
        self.sel_content_only = bool(kwargs.get("sel_content_only", False))
        self.use_rope = use_rope
        self.rope_long_range = rope_long_range
        self.cell_stride = cell_stride if cell_stride > 0 else window_size
        self.cell_topk = max(1, cell_topk)
        self._cell_block = 128
        self.cell_select = cell_select
        self.cell_prune_kernel = kwargs.get("cell_prune_kernel", None)
        self.cell_prune_pool = kwargs.get("cell_prune_pool", None)
        self.cell_prune_window = kwargs.get("cell_prune_window", None)
        self.cell_prune_blkchunk = kwargs.get("cell_prune_blkchunk", None)
        self.sel_strict_causal = kwargs.get("sel_strict_causal", None)
        self.fs_fused_attn = kwargs.get("fs_fused_attn", None)
        self.cell_fused_select = kwargs.get("cell_fused_select", None)
        self.fsb_enabled = bool(kwargs.get("fsb_enabled", False))
        self._fsb_init(n_heads, kwargs)
        self.decode_splits = int(kwargs.get("decode_splits", os.environ.get("FSATTN_DECODE_SPLITS", "0")))   # 0 = by batch size
        if dropout != 0.0:
            raise NotImplementedError("inference only: dropout must be 0")
        self.sel_scale = nn.Parameter(torch.ones(n_heads))
        log_sigma = torch.full((n_heads,), math.log(sigma_init))
        if learnable_sigma and not self.fs_uniform_sr:
            self.log_sigma = nn.Parameter(log_sigma)
        else:
            self.register_buffer("log_sigma", log_sigma)
        if lr_scale_mode == "learn":
            self.long_range_scale = nn.Parameter(torch.full((n_heads, 1, 1), 0.1))
        else:
            self.register_buffer("long_range_scale", torch.ones(n_heads, 1, 1))
        self.lr_norm = RMSNorm(self.head_dim)
        if use_rope:
            self.rope = Rotary(self.head_dim, max_seq_len)
        self.W_q = nn.Linear(d_model, d_model, bias=bias)
        self.W_k = nn.Linear(d_model, d_model, bias=bias)
        self.W_v = nn.Linear(d_model, d_model, bias=bias)
        self.W_o = nn.Linear(d_model, d_model, bias=bias)
        self.dropout = nn.Dropout(dropout)
        self._last_sel = None          # selections of the last call when FSATTN_KEEP_SEL=1 (tests, diagnostics)
        self._last_margin = None

    def _splits(self, B: int) -> int:
        """CTAs per (sequence, head) of the decode kernel. Four (one long-range CTA + three window CTAs) is fastest while
        the grid fits the machine (batch 1: 64 CTAs on 148 SMs, latency is everything); with many sequences the grid is
        several waves deep and fewer, fatter CTAs win (measured at batch 32: 13.4k tok/s with 1 against 10.9k with 4)."""
        if self.decode_splits > 0:
            return self.decode_splits
        s = 4
        while s > 1 and B * self.n_heads * s > 296:
            s //= 2
        return s

    def _fsb_init(self, n_heads: int, kw: dict):
        """The FS-B keywords of the reference layer (src/fsattn/fsb_tree.py:41-135, 136-155). Only the released serve
        configuration is built: fixed policy, delta 0, 'bound' node score, forest, token-LSE re-rank with the raw query,
        optional second beam and second forest. Anything else is refused at construction, as the reference refuses its
        own inconsistent combinations."""
        self.fsb_width = int(kw.get("fsb_width", 16))
        self.fsb_delta = int(kw.get("fsb_delta", 0))
        self.fsb_node_score = kw.get("fsb_node_score", "bound")
        self.fsb_bound_radius_coef = float(kw.get("fsb_bound_radius_coef", 8.0))
        self.fsb_tree = kw.get("fsb_tree", "forest")
        self.fsb_read_top = int(kw.get("fsb_read_top", 4))
        self.fsb_rerank_score = kw.get("fsb_rerank_score", "lse_pos")
        self.fsb_rerank_query = kw.get("fsb_rerank_query", "raw")
        self.fsb_union_width = int(kw.get("fsb_union_width", 0) or 0)
        self.fsb_union_tau_quantile = float(kw.get("fsb_union_tau_quantile", 0.0) or 0.0)
        self.fsb_policy_mode = kw.get("fsb_policy", "fixed") or "fixed"
        self.fsb_W_max = 16
        self.fsb_union_W_max = 16
        self.fsb_kk = self.fsb_read_top
        if not self.fsb_enabled:        # the reference registers the FS-B buffers only on FS-B layers (attention.py:122-128)
            return
        self.register_buffer("fsb_tau", torch.zeros(n_heads), persistent=True)
        self.register_buffer("fsb_tau_union", torch.zeros(n_heads), persistent=False)
        bad = []
        if self.fsb_policy_mode != "fixed": bad.append(f"fsb_policy={self.fsb_policy_mode!r} (fixed)")
        if self.fsb_delta != 0: bad.append(f"fsb_delta={self.fsb_delta} (0)")
        if self.fsb_node_score != "bound": bad.append(f"fsb_node_score={self.fsb_node_score!r} ('bound')")
        if self.fsb_tree != "forest": bad.append(f"fsb_tree={self.fsb_tree!r} ('forest')")
        if self.fsb_rerank_score != "lse_pos" or self.fsb_rerank_query != "raw":
            bad.append("re-rank other than fsb_rerank_score='lse_pos' with fsb_rerank_query='raw'")
        if not 1 <= self.fsb_width <= 16 or not 0 <= self.fsb_union_width <= 16:
            bad.append(f"beam widths {self.fsb_width}/{self.fsb_union_width} (1..16 / 0..16)")
        if not 1 <= self.fsb_read_top <= 8 or self.fsb_read_top != self.cell_topk:
            bad.append(f"fsb_read_top={self.fsb_read_top} (must equal cell_topk={self.cell_topk}, at most 8)")
        if not 0 <= self.fsb_union_tau_quantile < 1:
            bad.append(f"fsb_union_tau_quantile={self.fsb_union_tau_quantile} (0 = off, else in (0, 1))")
        if self.fsb_union_tau_quantile > 0 and self.fsb_union_width <= 0:
            bad.append("fsb_union_tau_quantile needs fsb_union_width > 0")
        for k in ("fsb_hybrid", "fsb_beam_quota", "fsb_union_quota", "fsb_read_margin", "fsb_route_adapter", "fsb_rerank_rr",
                  "fsb_leaf_radius"):
            if kw.get(k) not in (None, 0, 0.0, "off", "none", False):
                bad.append(f"{k}={kw[k]!r}")
        if bad:
            raise NotImplementedError("FS-B: only the released serve configuration is implemented; got " + "; ".join(bad))

    def _fsb_union_tau_on(self) -> bool:
        return self.fsb_union_tau_quantile > 0

    def _fsb_w2(self, fo) -> int:
        """Width of the second beam. Without a second forest the reference runs it over the main forest, where it finds
        the main beam's cells again and union_candidates blanks every one of them (src/fsattn/fsb_tree.py:1226-1231,
        711-713): the selection is the same without it, so it is not launched."""
        return self.fsb_union_width if fo.nf > 1 else 0

    # ---- configuration helpers (same names as the reference) ---------------------------------------------------------
    @property
    def sigma(self) -> torch.Tensor:
        return self.log_sigma.exp()

    def _prune_cfg(self, attr, env, dflt):
        """src/fsattn/attention.py:335-337: keyword over environment over default."""
        v = getattr(self, attr, None)
        return int(v) if v is not None else int(os.environ.get(env, str(dflt)))

    def _is_dense_lr(self):
        return not bool(self._prune_cfg("cell_prune_kernel", "FS_PRUNE_KERNEL", 0))

    def _assert_cacheable(self, phase="decode"):
        """src/fsattn/attention.py:872-891, plus the configurations this implementation does not cover."""
        if not self.causal:
            raise NotImplementedError("FSKVCache requires causal=True.")
        if not self.use_rope or self.rope_long_range:
            raise NotImplementedError("only the deployed window-RoPE + un-rotated long-range configuration "
                                      "(use_rope=True, rope_long_range=False) is implemented")
        if self.disable_short_range or self.disable_long_range:
            raise NotImplementedError("FSKVCache requires both SR and LR branches enabled.")
        if not bool(self._prune_cfg("sel_strict_causal", "FS_STRICT_CAUSAL", 0)):
            raise NotImplementedError("FSKVCache requires sel_strict_causal=1 (block-causal path is non-cacheable).")
        if not self.fs_uniform_sr:
            raise NotImplementedError("only the uniform window (fs_uniform_sr=True) is implemented")
        if self.sel_content_only:
            raise NotImplementedError("sel_content_only is not implemented")
        if self.cell_stride != ops.CELL:
            raise NotImplementedError(f"cell_stride {self.cell_stride}: the kernels are specialised for {ops.CELL}")
        if self._is_dense_lr() and not self.fsb_enabled and (self.head_dim != 64 or self.cell_topk > 4):
            raise NotImplementedError("the dense FS variant (cell_prune_kernel=0) is built for head_dim 64 and cell_topk <= 4")

    def _pool_cfg(self):
        return (self._prune_cfg("cell_prune_pool", "FS_PRUNE_POOL", 64), self._prune_cfg("cell_prune_window", "FS_PRUNE_WINDOW", 8))

    def _ensure_qkv_cache(self):
        """src/fsattn/attention.py:1396-1410: one fused (3d, d) projection weight the three Linear weights are views of."""
        wq, wk, wv = self.W_q.weight, self.W_k.weight, self.W_v.weight
        dm = self.d_model
        key = (wq.data_ptr(), wq._version, wk.data_ptr(), wk._version, wv.data_ptr(), wv._version, wq.dtype)
        c = getattr(self, "_w_qkv_cache", None)
        if c is None or c[0] != key:
            qkv_w = torch.cat([wq.data, wk.data, wv.data], dim=0)
            self.W_q.weight.data = qkv_w[:dm]
            self.W_k.weight.data = qkv_w[dm:2 * dm]
            self.W_v.weight.data = qkv_w[2 * dm:]
            wq, wk, wv = self.W_q.weight, self.W_k.weight, self.W_v.weight
            key = (wq.data_ptr(), wq._version, wk.data_ptr(), wk._version, wv.data_ptr(), wv._version, wq.dtype)
            c = (key, qkv_w)
            self._w_qkv_cache = c
            CACHE_GEN[0] += 1
        return c[1], dm

    def head_params(self):
        """fp32 device tensors the kernels read: (lam (H), sigma (H), lrs (H), norm_w (D)). Cached per parameter version."""
        ps = (self.sel_scale, self.log_sigma, self.long_range_scale, self.lr_norm.scale)
        key = tuple((p.data_ptr(), p._version, p.device) for p in ps)
        c = getattr(self, "_head_params", None)
        if c is None or c[0] != key:
            vals = (self.sel_scale.detach().float().contiguous(), self.log_sigma.detach().float().exp().contiguous(),
                    self.long_range_scale.detach().float().reshape(-1).contiguous(), self.lr_norm.scale.detach().float().contiguous())
            c = (key, vals)
            self._head_params = c
            CACHE_GEN[0] += 1
        return c[1]

    # ---- forward ---------------------------------------------------------------------------------------------------------
    def forward(self, x: torch.Tensor, mask: torch.Tensor | None = None, cache=None, pre_norm=None) -> torch.Tensor:
        """pre_norm (optional, not in the reference's signature): the block's input norm, applied here to x in token chunks
        on the way into the projection, so that a long prefill never holds a normalised copy of the whole sequence."""
        if cache is None:
            raise NotImplementedError("this build covers cached inference only: pass an FSKVCache (the training forward "
                                      "stays with the reference implementation)")
        return self._forward_cached(x, cache, pre_norm)

    PROJ_CHUNK = 16384          # tokens per projection call when the input norm is applied here

    def _project_qkv(self, x, pre_norm=None):
        B, N, _ = x.shape
        H, D = self.n_heads, self.head_dim
        if self.W_q.bias is not None:
            raise NotImplementedError("projection biases are not supported (the LM uses bias=False)")
        w, dm = self._ensure_qkv_cache()
        if pre_norm is None:
            qkv = F.linear(x, w)                               # (B, N, 3d), one GEMM
        else:
            qkv = torch.empty(B, N, 3 * dm, dtype=x.dtype, device=x.device)
            wt = w.t()
            for b in range(B):
                for s0 in range(0, N, self.PROJ_CHUNK):
                    torch.mm(pre_norm(x[b, s0:s0 + self.PROJ_CHUNK]), wt, out=qkv[b, s0:s0 + self.PROJ_CHUNK])
        q, k, v = (qkv[..., i * dm:(i + 1) * dm].view(B, N, H, D).transpose(1, 2) for i in range(3))
        return q, k, v

    @torch.no_grad()
    def _forward_cached(self, x, cache, pre_norm=None):
        B, N, _ = x.shape
        self._assert_cacheable(phase="prefill" if (cache.pos == 0 and N > 1) else "decode")
        if x.dtype != torch.bfloat16 or not x.is_cuda:
            raise RuntimeError("FSAttn runs on bf16 CUDA activations only (there is no CPU or fp32 path)")
        Q, K, V = self._project_qkv(x, pre_norm)
        if getattr(cache, "attend", None) is not None:
            # the streaming cache runs the layer's attention itself (src/fsattn/attention.py:995-999)
            out = cache.attend(Q, K, V)
            del Q, K, V
            return self.W_o(out.transpose(1, 2).reshape(B, N, self.d_model))
        if cache.pos == 0 and N > 1:
            y = self._prefill(Q, K, V, cache)
        else:
            ys = [self._decode_one(Q[:, :, t], K[:, :, t], V[:, :, t], cache) for t in range(N)]
            y = torch.stack(ys, dim=1) if N > 1 else ys[0].unsqueeze(1)
        del Q, K, V                                            # the projections are dead: W_o's output reuses their memory
        return self.W_o(y)

    def _prefill(self, Q, K, V, cache):
        """src/fsattn/attention.py:1003-1078 (standard prefill): window branch, cell statistics + KV store, per-block
        candidate pools, selection, fused readout + combine. Returns W_o's input (B,N,H*D)."""
        B, H, N, D = Q.shape
        s = self.cell_stride
        P, Wc = self._pool_cfg()
        cos, sin = self.rope.tables_bf16(N)
        ncell = N // s
        fo = build_done = None
        if self.fsb_enabled and ncell > 0:
            # FS-B: statistics first, then the forest build on a side stream while the window branch runs on this one.
            # The build is a chain of dependent levels on a few SMs (its largest chunk sets the time), so it hides behind
            # the window kernel (the reference overlaps its window branch the same way, attention.py:254 FSB_WINDOW_OVERLAP)
            kbar, ceil = cache.prefill(K, V)
            fo = cache.fsb_forests(kbar, ceil, self)
            cur = torch.cuda.current_stream(Q.device)
            side = _side_stream(Q.device)
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                fo.ingest(ncell)
                build_done = torch.cuda.Event()
                build_done.record(side)
        sr = ops.window_prefill(Q, K, V, cos, sin, self.window_size, self.scale)
        if fo is None:
            kbar, ceil = cache.prefill(K, V)
        M = (N + s - 1) // s
        kk = min(self.cell_topk, M)
        Bq = min(self._cell_block, N)
        nb = (N + Bq - 1) // Bq
        lam, sigma, lrs, norm_w = self.head_params()
        if ncell == 0:
            # nothing completed: every selection is empty; the readout still applies the combine (lr = 0)
            sel = torch.full((B, H, nb * Bq, kk), -1, dtype=torch.int32, device=Q.device)
            margin = None
        elif self.fsb_enabled:
            # src/fsattn/fsb_tree.py:2368-2520: both forests over the prompt's cells, then per 128-query block the two
            # beams, the union of their candidates and the token-level re-rank
            torch.cuda.current_stream(Q.device).wait_event(build_done)
            sel = ops.fsb_select(fo, Q, K, lam, sigma, scale=self.scale, N=N, Bq=Bq, width=self.fsb_width,
                                 width2=self._fsb_w2(fo), read_top=self.fsb_read_top,
                                 radius_coef=self.fsb_bound_radius_coef)
            # the prompt's queries were the only ones that name earlier prefixes: keep one chunk per height for the decode
            # (the reference's decode arena, src/fsattn/fsb_tree.py:1496-1522) and release the rest
            if os.environ.get("FSATTN_FSB_KEEP_ARENA", "0") != "1":
                fo.compact_arena((N // self._cell_block) * self._cell_block // s)
            margin = None
        elif self._is_dense_lr():
            # dense FS (src/fsattn/attention.py:362-423): every cell completed before the query's block is a candidate
            if Bq == self._cell_block:
                sel = ops.fs_dense_select(Q, kbar, ceil, lam, sigma, N=N, ncell=ncell, Bq=Bq, nb=nb, kk=kk, scale=self.scale)
            else:       # a prompt shorter than one query block: block 0 sees no completed cell
                sel = torch.full((B, H, nb * Bq, kk), -1, dtype=torch.int32, device=Q.device)
            margin = None
        else:
            st = cache.state
            topp = getattr(st, "prefill_topp", None) if st is not None else None
            if topp is None or topp.shape[2] != min(P, M) or topp.shape[1] < nb or Bq != self._cell_block:
                topp = ops.fsl_prefix_topp(ceil, ncell, Bq, nb, min(P, M))
            if st is not None:
                st.prefill_topp = None
            keep = os.environ.get("FSATTN_KEEP_SEL", "0") == "1"
            res = ops.fsl_select(Q, kbar, ceil, topp, lam, sigma, N=N, ncell=ncell, Bq=Bq, nb=nb, P=min(P, M), Wc=Wc,
                                 kk=kk, scale=self.scale, want_margin=keep)
            sel, margin = res if keep else (res, None)
        if os.environ.get("FSATTN_KEEP_SEL", "0") == "1":
            self._last_sel, self._last_margin = sel, margin
        return ops.readout_combine(Q, K, V, sel, sr, norm_w, lrs, self.lr_norm.eps, scale=self.scale, Bq=Bq, n_kv=N,
                                   out=sr)

    def _decode_one(self, q, k, v, cache, pos_t=None, y=None):
        """One token through the fused decode-step kernel (src/fsattn/attention.py:1116-1131 and 1493-1559).
        q,k,v (B,H,D) views; returns W_o's input (B, H*D)."""
        st = cache.decode_state(q)
        if pos_t is None:
            if cache.pos >= st.cap_rows:
                raise RuntimeError(f"KV store holds {st.cap_rows} positions; set cache.reserve before the prefill")
            pos_t = cache.pos_t
            pos_t.fill_(cache.pos)
        cos, sin = self.rope.tables_bf16(st.cap_rows)
        lam, sigma, lrs, norm_w = self.head_params()
        sel_out = None
        if os.environ.get("FSATTN_KEEP_SEL", "0") == "1":
            sel_out = torch.empty(st.B, st.H, st.kk, dtype=torch.int32, device=q.device)
            self._last_sel = sel_out
        ext = None
        if self.fsb_enabled:
            cache.fsb_block_change(cache.pos, self)
            ext = self._fsb_decode_select(q, st, cache, pos_t, lam, sigma)
        elif self._is_dense_lr():
            ext = self._dense_decode_select(q, st, pos_t, lam, sigma)
        y = ops.fsl_decode_step(st, q, k, v, pos_t, cos, sin, lam, sigma, lrs, norm_w, scale=self.scale,
                                eps=self.lr_norm.eps, y=y, sel_out=sel_out, splits=self._splits(st.B), ext_sel=ext)
        cache.advance_in_place()
        return y

    def _fsb_decode_select(self, q, st, cache, pos_t, lam, sigma, pdl=False):
        """src/fsattn/fsb_tree.py:2909-3064: the decode query's two beams over the block's forests, union, re-rank with
        the token keys as the cache reads them (raw bf16, or the int8 codes). q (B,H,D) view -> (B,H,1,kk) int32."""
        fo = cache.fsb
        q4 = q.unsqueeze(2)
        if st.mode == "bf16":
            return ops.fsb_select(fo, q4, st.kbuf, lam, sigma, scale=self.scale, width=self.fsb_width,
                                  width2=self._fsb_w2(fo), read_top=self.fsb_read_top,
                                  radius_coef=self.fsb_bound_radius_coef, pos=pos_t, pdl=pdl)
        return ops.fsb_select(fo, q4, None, lam, sigma, scale=self.scale, width=self.fsb_width,
                              width2=self._fsb_w2(fo), read_top=self.fsb_read_top,
                              radius_coef=self.fsb_bound_radius_coef, pos=pos_t, kq=st.kq, ks=st.ks, pdl=pdl)

    def _dense_decode_select(self, q, st, pos_t, lam, sigma, pdl=False):
        """src/fsattn/attention.py:1159-1185: the dense variant's decode query scores every cell completed before its query
        block (statistics of the layer's own KV state). q (B,H,D) view -> (B,H,kk) int32 for the decode step's ext_sel."""
        if st.mode == "bounded":
            raise NotImplementedError("the dense FS variant reads any completed cell: it needs a full KV store")
        splits = 8
        while splits > 1 and st.B * st.H * splits > 296:
            splits //= 2
        return ops.fs_dense_decode_select(q, st.kbar, st.ceil, lam, sigma, pos_t, Bq=self._cell_block, kk=st.kk, scale=self.scale,
                                          ncell_cap=st.cap_cells, splits=splits, pdl=pdl)

    def graph_decode_layer(self, x, buf):
        """One decode token inside a captured whole-step graph (src/fsattn/attention.py:1493-1559): x (B,1,d); buf holds
        the shared device position `pos_t` and the layer's `cache`. Everything the reference does around its graph replay
        for this layer (pool refresh, cell close) happens inside the one kernel launch."""
        B, N, _ = x.shape
        H, D = self.n_heads, self.head_dim
        w, dm = self._ensure_qkv_cache()
        qkv = F.linear(x.view(B, dm), w).view(B, 3, H, D)
        cache = buf["cache"]
        st = cache.decode_state(qkv)
        cos, sin = self.rope.tables_bf16(st.cap_rows)
        lam, sigma, lrs, norm_w = self.head_params()
        ext = None
        if self.fsb_enabled:
            ext = self._fsb_decode_select(qkv[:, 0], st, cache, buf["pos_t"], lam, sigma)
        elif self._is_dense_lr():
            ext = self._dense_decode_select(qkv[:, 0], st, buf["pos_t"], lam, sigma)
        y = ops.fsl_decode_step(st, qkv[:, 0], qkv[:, 1], qkv[:, 2], buf["pos_t"], cos, sin, lam, sigma, lrs, norm_w,
                                scale=self.scale, eps=self.lr_norm.eps, y=buf.get("y"), splits=self._splits(st.B),
                                ext_sel=ext)
        return self.W_o(y.view(B, 1, dm))

    def graph_decode_layer_fsb(self, x, cache, buf):
        """src/fsattn/attention.py:1450-1491: the FS-B layer's decode token inside a captured whole-step graph, the cache
        passed explicitly. The forests must have been brought to the token's block (fsb_tree.fsb_decode_prepare_all /
        cache.fsb_block_change) outside the graph."""
        return self.graph_decode_layer(x, dict(buf, cache=cache))

    @torch.no_grad()
    def _build_decode_pool(self, cache, blk_start, s, dev, need_tokens: bool = True, out: dict | None = None):
        """The candidate pool of the decode block starting at blk_start as the reference hands it to its decode kernels
        (src/fsattn/attention.py:1313-1369): top-P cells by (ceiling desc, index asc) among the visible ones, then the Wc
        newest. The decode-step kernel of this library refreshes its own pool on the device; this method serves callers
        that want the pool itself (inspection, tests). Returns {"empty": True} when nothing is visible."""
        if getattr(cache, "bounded_kv", False):
            if need_tokens:
                cache._no_history("_build_decode_pool(need_tokens=True)")
            return cache.bounded_pool(blk_start, out=out)
        P, Wc = self._pool_cfg()
        kbar, ceil, ncell = cache.completed_cells()
        M_vis = min(blk_start // s, ncell)
        if M_vis <= 0 or ncell <= 0:
            return {"empty": True}
        return _pool_from_stats(kbar[:, :, :M_vis], ceil[:, :, :M_vis], None, blk_start, s, P, Wc)

    @torch.no_grad()
    def _build_dense_decode_pool(self, cache, blk_start, s, dev, out: dict | None = None):
        """src/fsattn/attention.py:1278-1311: the dense FS variant's "pool" is every visible cell."""
        kbar, ceil, ncell = cache.completed_cells()
        M_vis = min(blk_start // s, ncell)
        if M_vis <= 0 or ncell <= 0:
            return {"empty": True}
        cells = torch.arange(M_vis, device=ceil.device)
        return {"dense": True, "M_vis": M_vis, "C": M_vis, "Kbar_cand": kbar[:, :, :M_vis], "ceil_cand": ceil[:, :, :M_vis],
                "cen_cand": (cells.float() + 0.5) * s, "cand_c": cells.expand(ceil.shape[0], ceil.shape[1], M_vis)}

    def graph_decode_attn(self, qkv, buf, y=None, pdl=True):
        """The attention part of one decode token given the fused projection qkv (B, 3*d) bf16: returns W_o's input
        (B, d). Used by the decoder whose trunk projections run in this library's own GEMV kernels."""
        B = qkv.shape[0]
        H, D = self.n_heads, self.head_dim
        q4 = qkv.view(B, 3, H, D)
        st = buf["cache"].decode_state(q4)
        cos, sin = self.rope.tables_bf16(st.cap_rows)
        lam, sigma, lrs, norm_w = self.head_params()
        ext = None
        if self.fsb_enabled:
            # the selection kernel reads q, so it waits for the projection like any dependent launch; the decode kernel
            # then depends on it through ext_sel
            ext = self._fsb_decode_select(q4[:, 0], st, buf["cache"], buf["pos_t"], lam, sigma, pdl=pdl)
        elif self._is_dense_lr():
            ext = self._dense_decode_select(q4[:, 0], st, buf["pos_t"], lam, sigma, pdl=pdl)
        return ops.fsl_decode_step(st, q4[:, 0], q4[:, 1], q4[:, 2], buf["pos_t"], cos, sin, lam, sigma, lrs, norm_w,
                                   scale=self.scale, eps=self.lr_norm.eps, y=y, splits=self._splits(st.B),
                                   pdl=pdl, ext_sel=ext)
