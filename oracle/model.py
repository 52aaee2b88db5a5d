"""CPU port of FS-L model decode (test infrastructure / timed CPU baseline only, never on the product path).

A torch-on-CPU fp32 restatement of what the reference's eager path does per decode token for the FS-L serve preset
(experiments/scaling/kv_cache.py:484-547 driving model.py:211-237 and src/fsattn/attention.py:1116-1276): RMSNorm, QKV
projection, KV append with incremental cell statistics (kv_cache.py:326-392), RoPE window attention over the last W+1
tokens, the block's candidate pool (refreshed every Bq tokens), chunk-mean-key scoring, top-kk, readout, lr_norm, combine,
W_o, SwiGLU. The attention pieces are the functions of oracle/fsl.py, so what is timed is what the parity tests check.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import fsl


class CpuFSLModel:
    def __init__(self, d_model=1024, n_layers=24, n_heads=16, d_ff=2816, vocab=32000, *, s=32, Bq=128, kk=4, W=512, P=64, Wc=8,
                 seed=0, max_len=8192):
        g = torch.Generator().manual_seed(seed)
        self.d, self.L, self.H, self.D, self.V = d_model, n_layers, n_heads, d_model // n_heads, vocab
        self.s, self.Bq, self.kk, self.W, self.P, self.Wc = s, Bq, kk, W, P, Wc
        self.scale = 1.0 / math.sqrt(self.D)

        def w(*shape):
            return torch.randn(*shape, generator=g) * 0.02
        self.emb = w(vocab, d_model)
        self.layers = [dict(wqkv=w(3 * d_model, d_model), wo=w(d_model, d_model), wgu=w(2 * d_ff, d_model), wdown=w(d_model, d_ff),
                            ln1=torch.ones(d_model), ln2=torch.ones(d_model), lam=torch.ones(n_heads), sigma=torch.full((n_heads,), 4.0),
                            lrs=torch.full((n_heads,), 0.1), norm_w=torch.ones(self.D)) for _ in range(n_layers)]
        self.ln_f = torch.ones(d_model)
        self.cos, self.sin = fsl.rope_tables(self.D, max_len)
        self.max_len = max_len
        self.state = None
        self.pos = 0

    def synthetic_context(self, B: int, ctx: int, seed=1):
        """A cache as a ctx-token prefill would leave it, filled with seeded random keys/values (the decode step's cost does
        not depend on their values)."""
        g = torch.Generator().manual_seed(seed)
        self.state = []
        for _ in range(self.L):
            K = torch.zeros(B, self.H, self.max_len, self.D)
            V = torch.zeros(B, self.H, self.max_len, self.D)
            K[:, :, :ctx] = torch.randn(B, self.H, ctx, self.D, generator=g) * 0.6
            V[:, :, :ctx] = torch.randn(B, self.H, ctx, self.D, generator=g) * 0.6
            kbar, ceil = fsl.cell_stats(K[:, :, :ctx], self.s)
            nc = ctx // self.s
            kb = torch.zeros(B, self.H, self.max_len // self.s, self.D); kb[:, :, :nc] = kbar
            ce = torch.zeros(B, self.H, self.max_len // self.s); ce[:, :, :nc] = ceil
            self.state.append(dict(K=K, V=V, kbar=kb, ceil=ce, pool=None, pool_blk=-1))
        self.pos = ctx

    @staticmethod
    def _rms(x, w, eps=1e-6):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w

    def _attn(self, li, x):
        lp, st = self.layers[li], self.state[li]
        B = x.shape[0]
        H, D, s, pos = self.H, self.D, self.s, self.pos
        qkv = F.linear(x, lp["wqkv"]).view(B, 3, H, 1, D)
        q, k, v = qkv[:, 0], qkv[:, 1], qkv[:, 2]
        st["K"][:, :, pos:pos + 1] = k
        st["V"][:, :, pos:pos + 1] = v
        if (pos + 1) % s == 0:          # the cell closes: its statistics join the tables
            c = pos // s
            kb, ce = fsl.cell_stats(st["K"][:, :, c * s:(c + 1) * s], s)
            st["kbar"][:, :, c:c + 1] = kb
            st["ceil"][:, :, c:c + 1] = ce
        j0 = max(0, pos - self.W)
        sr = fsl.window_attention(q, st["K"][:, :, j0:pos + 1], st["V"][:, :, j0:pos + 1], self.cos, self.sin, self.W, self.scale,
                                  q_pos0=pos, k_pos0=j0)
        blk = (pos // self.Bq) * self.Bq
        ncell = pos // s
        if st["pool_blk"] != blk:
            st["pool"] = fsl.fsl_decode_pool(st["kbar"][:, :, :ncell], st["ceil"][:, :, :ncell], blk, s, self.P, self.Wc) if ncell > 0 else None
            st["pool_blk"] = blk
        sel, _ = fsl.fsl_decode_select(q, st["pool"], pos, lp["lam"], lp["sigma"], self.scale, s, self.kk)
        o = fsl.cell_readout(q, st["K"], st["V"], sel, s, self.Bq, self.scale, pos, pos + 1)
        y = fsl.lr_norm_combine(sr, o, lp["norm_w"], lp["lrs"], 1e-8, act_dtype=torch.float32)
        return F.linear(y, lp["wo"])

    @torch.no_grad()
    def step(self, tok):
        """tok (B,1) int64 -> next greedy token (B,1)."""
        x = self.emb[tok]
        for li, lp in enumerate(self.layers):
            x = x + self._attn(li, self._rms(x, lp["ln1"]))
            gu = F.linear(self._rms(x, lp["ln2"]), lp["wgu"])
            f = gu.shape[-1] // 2
            x = x + F.linear(F.silu(gu[..., :f]) * gu[..., f:], lp["wdown"])
        logits = F.linear(self._rms(x, self.ln_f)[:, -1], self.emb)
        self.pos += 1
        return logits.argmax(-1, keepdim=True)
