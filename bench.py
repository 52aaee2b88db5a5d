"""Benchmark of the FS-L / FS-B decode hot path: `python bench.py --gpus N --steps K --warmup W [--impl reference]`.

Headline workload (BASELINE config 2 at its largest published context): FS-L 341M model (24 layers, d_model 1024, 16 heads x
64, vocab 32000), random-init bf16 weights, batch 1, uniform random token ids; an untimed prefill of `--ctx` tokens (default
131072) through this repo's kernels, then greedy decode. A step = one decoded token through the whole model (one CUDA-graph
replay).
  value  : tok/s over exactly K replays timed with CUDA events (inputs resident in HBM), max over ranks
  e2e    : tok/s through the public decoder API (GraphedDecoder.step_host) with the token id copied from pinned host
           memory every step and the sampled token read back to the host every step
The same JSON line carries, outside the headline's timed region: the roofline of the step's dominant kernel (the trunk
projection GEMV) and of the attention decode kernel, the prefill figures, the window-attention kernel against the tensor peak,
short legs at 4k / 16k / 64k for FS-L and FS-B, BASELINE config 3 (FS-B at the headline context), the dense FS variant,
config 4 (743M-class, batch 32, 32k, int8 KV) and a CPU baseline.
With N > 1 ranks (torchrun) every rank decodes its own sequence (batch sharding, no collective): weak scaling; the line then
also carries a head-sharded leg (one sequence, heads split over the ranks: strong scaling) and config 4's 32 sequences
split 32/N.
`--impl reference` times the reference's own eager CPU decode (oracle/ref_cpu.py) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# the reference's published A100-40GB figures (README.md:61-63 of the reference), by context length
PUBLISHED = {
    "fsl_decode_tps": {4096: 515.6, 16384: 522.0, 65536: 514.5, 131072: 515.1},
    "fsl_prefill_ktoks": {4096: 146.4, 16384: 187.5, 65536: 190.2, 131072: 189.8},
    "fsb_decode_tps": {4096: 504.7, 16384: 497.9, 65536: 473.8, 131072: 462.7},
    "fsb_prefill_ktoks": {4096: 127.7, 16384: 149.3, 65536: 143.1, 131072: 137.8},
    "dense_decode_tps": {4096: 500.2, 16384: 488.1, 65536: 431.1, 131072: 385.8},
    "dense_prefill_ktoks": {4096: 147.2, 16384: 179.5, 65536: 159.5, 131072: 134.8},
}
# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) from ncu --set full captures of the current kernels
# (a 32k-context run; neither kernel's traffic depends on the context). trunk_gemv: the weighted mean over one step's 97
# launches (24 x (6.32 + 2.13 + 11.56 + 5.81) + 66.0 MB). None where no capture of that shape exists.
NCU_DRAM_BYTES = {"fsl_decode_kernel/340m/b1": 1.85e6, "trunk_gemv_kernel/340m/b1": 7.07e6}


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.isfile(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""
    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            self.t.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[0])); mx.append(float(r[1]))
            except Exception:
                continue
            for n, v in zip(names, r[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---- algorithmic bytes ------------------------------------------------------------------------------------------------------
def attn_bytes_per_layer(B, H, D, W, P, Wc, kk, s, int8=True):
    """Algorithmic bytes one FS-L decode-step launch of one layer moves (window rows of K and V, the pool's mean keys +
    per-slot scalars, the kk cells read, the new row)."""
    e = 1 if int8 else 2
    win = (W + 1) * D * 2 * e
    pool = (P + Wc) * (D * 4 + 17)
    read = kk * s * D * 2 * e
    new = 2 * D * 2
    return B * H * (win + pool + read + new)


def fsb_attn_bytes_per_layer(B, H, D, W, kk, s, m_main, m_union, width=16, width2=16, int8=True):
    """Algorithmic bytes of one FS-B decode step of one layer: the window, both beams' visited nodes (bf16 mean + 36 bytes of
    node data each; a beam of width w visits min(2^l, 2w) children at level l of a forest of height ceil(log2 m)), the
    token keys of the <= width + width2 candidate cells for the re-rank, the kk cells' values, the new row."""
    e = 1 if int8 else 2

    def beam(m, w):
        h = max(0, math.ceil(math.log2(max(m, 1))))
        return sum(min(2 ** l, 2 * w) for l in range(1, h + 1)) * (2 * D + 36)
    win = (W + 1) * D * 2 * e
    rerank = (width + width2) * s * D * e
    read = kk * s * D * e
    new = 2 * D * 2
    return B * H * (win + beam(m_main, width) + beam(m_union, width2) + rerank + read + new)


def weight_bytes(model) -> int:
    """All linear weights + the tied embedding / LM head, bf16, read once per decode step."""
    return 2 * sum(p.numel() for _, p in model.named_parameters() if p.dim() > 1)


# ---- the reference arm -------------------------------------------------------------------------------------------------------
def run_reference(args):
    """The reference's own eager decode on the host cores (oracle/_ref), a bounded sample of the headline workload."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle.ref_cpu import time_fsl_decode
    steps, warm = min(args.steps, 24), min(args.warmup, 3)
    r = time_fsl_decode(min(args.ctx, args.cpu_ctx), steps, warm)
    cb = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
    line = {"impl": "reference", "metric": "fsl_decode_tok_s", "value": r["value"], "unit": "tok/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": warm, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"FS-L 340m decode after a {args.ctx}-token prefill, batch 1 (CPU sample: {r['sample']})"},
            "cpu_baseline": cb,
            "e2e": {"value": r["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---- kernel timers (outside the headline's timed region) ---------------------------------------------------------------
def time_decode_kernel(gd, n=48):
    """Average duration of the fused attention decode-step kernel launched alone, L2 flushed before every launch (in the real
    step hundreds of MB of weights pass through L2 between two launches of the same layer, so its KV rows are cold)."""
    from freesolo_b200 import ops
    dev = gd.dev
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    pos_t = gd.pos_t.clone()
    times = []
    L = len(gd.cache)
    a0 = gd.attn_core[0]
    B = gd.tok.shape[0]
    qkv = torch.randn(B, 3, a0.n_heads, a0.head_dim, device=dev).to(torch.bfloat16)
    y = torch.empty(B, a0.n_heads * a0.head_dim, dtype=torch.bfloat16, device=dev)
    for i in range(n + 4):
        a = gd.attn_core[i % L]
        st = gd.cache[i % L].state
        cos, sin = a.rope.tables_bf16(st.cap_rows)
        lam, sigma, lrs, nw = a.head_params()
        flush.fill_(i & 255)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ops.fsl_decode_step(st, qkv[:, 0], qkv[:, 1], qkv[:, 2], pos_t, cos, sin, lam, sigma, lrs, nw, scale=a.scale,
                            eps=a.lr_norm.eps, y=y, splits=a._splits(B))
        e1.record()
        times.append((e0, e1))
    torch.cuda.synchronize()
    ms = sorted(e0.elapsed_time(e1) for e0, e1 in times[4:])
    return sum(ms) / len(ms), ms[len(ms) // 2]


def time_gemv_chain(gd, reps=20):
    """The trunk projection kernel (trunk_gemv_kernel) in the launch chain it has inside a decode step: the 4 projections
    of every layer + the LM head, chained by programmatic dependent launch exactly as in the step, captured once and
    replayed `reps` times with the attention launches left out. Every replay streams all weights (> L2), so the launches
    run on cold weights as they do in the step. Returns (launches per replay, ms per replay)."""
    from freesolo_b200 import ops
    m, x = gd.m, gd.x

    def chain():
        for i, blk in enumerate(gd.blocks):
            a = gd.attn[i]
            ops.trunk_gemv(x, a._ensure_qkv_cache()[0], norm_w=blk.ln1.weight, eps=blk.ln1.eps, out=gd.qkv)
            ops.trunk_gemv(gd.y, a.W_o.weight, res=x, out=x)
            ops.trunk_gemv(x, blk.ffn._ensure_gu_cache()[0], norm_w=blk.ln2.weight, eps=blk.ln2.eps, swiglu=True, out=gd.act)
            ops.trunk_gemv(gd.act, blk.ffn.w_down.weight, res=x, out=x)
        ops.trunk_gemv(x, m.lm_head.weight, norm_w=m.ln_final.weight, eps=m.ln_final.eps, out=gd.logits)
    x.zero_(); gd.y.zero_()
    chain()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        chain()
    for _ in range(3):
        g.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return 4 * len(gd.blocks) + 1, e0.elapsed_time(e1) / reps


def time_window_kernel(attn, dev, ctx: int, reps: int = 5):
    """Prefill window attention alone (RoPE pre-pass + tcgen05 kernel) on random Q/K/V of the model's shape: useful
    FLOPs 4*H*D*(sum_i min(i+1, W+1)) over its CUDA-event time, against the measured bf16 tensor peak. The operands
    (3 x ctx*H*D*2 B = 805 MB at 131k) exceed L2, so no flush is needed between repetitions."""
    from freesolo_b200 import ops
    H, D, W = attn.n_heads, attn.head_dim, attn.window_size
    n = min(ctx, 131072)
    g = torch.Generator(device=dev).manual_seed(7)
    Q, K, V = (torch.randn(1, n, 3 * H * D, device=dev, generator=g).to(torch.bfloat16).view(1, n, 3, H, D)[:, :, j].transpose(1, 2)
               for j in range(3))
    cos, sin = attn.rope.tables_bf16(n)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.empty(1, n, H * D, dtype=torch.bfloat16, device=dev)
    times = []
    for i in range(reps + 2):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ops.window_prefill(Q, K, V, cos, sin, W, attn.scale, out=out, status=status)
        e1.record()
        times.append((e0, e1))
    torch.cuda.synchronize()
    if int(status.item()) != 0:
        raise RuntimeError("a bounded wait inside the window kernel ran out")
    ms = sorted(a.elapsed_time(b) for a, b in times[2:])[reps // 2]
    flops = 4.0 * H * D * ((W + 1) * n - W * (W + 1) / 2.0) if n > W else 4.0 * H * D * n * (n + 1) / 2.0
    _, peak, kind = _peaks()
    return {"kernel": "rope_qk_kernel + window_tc_kernel", "bound": "tensor", "achieved": flops / (ms * 1e-3) / 1e12, "peak": peak,
            "unit": "TFLOP/s", "frac": flops / (ms * 1e-3) / 1e12 / peak, "peak_kind": kind, "ms": ms, "tokens": n, "heads": H,
            "how": "launched alone on random operands larger than L2, median of 5, CUDA events on the launching stream; "
                   "useful FLOPs only (masked parts of the key tiles not counted)"}


def timed_prefill(make_decoder, reps: int = 3):
    """The reference's prefill protocol (experiments/scaling/bench_efficiency.py:166-198, `--warm 1 --nmed 3`): one untimed
    prefill at the full context (the allocator's pools and every kernel attribute are warm afterwards), then the median of
    `reps` timed ones, each on a fresh decoder (fresh KV stores / forests). Returns (last decoder, median ms, all ms).
    PREFILL_PEAK_GIB[0] = the peak allocated bytes over the timed prefills (statistics reset after the warm-up one, the
    reference's `_reset_mem`; unlike its `retain_kv=False` prefill this one fills the KV store the decode then reads)."""
    gd = make_decoder()
    gd.prefill()
    torch.cuda.synchronize()
    times = []
    for i in range(reps):
        del gd
        if i == 0:
            torch.cuda.synchronize()
            if reps > 1:                      # (a single timed run keeps the allocator's pools: it must not pay for cudaMalloc)
                torch.cuda.empty_cache()
            torch.cuda.reset_peak_memory_stats()
        gd = make_decoder()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        gd.prefill()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    PREFILL_PEAK_GIB[0] = torch.cuda.max_memory_allocated() / 2 ** 30
    return gd, sorted(times)[len(times) // 2], times


PREFILL_PEAK_GIB = [None]


def timed_graph_prefill(model, ids, dev, reps: int = 3):
    """The reference's graphed prefill protocol (experiments/scaling/bench_efficiency.py:201-229): the whole prefill of this
    shape captured once (`GraphedPrefiller`, `retain_kv=False`: chunk statistics, selection, readout, last-token logits; no
    KV store fill), one untimed replay, then the median of `reps` replays between CUDA events."""
    from freesolo_b200.serving import GraphedPrefiller
    import gc
    B, L = ids.shape
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    torch.cuda.reset_peak_memory_stats()
    gp = GraphedPrefiller(model, L, B=B, device=dev, tail_tokens=min(64, L), retain_kv=False)
    ids = ids.to(dev)
    gp.capture(ids)
    gp.run(ids)
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        gp.run(ids)
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    peak = torch.cuda.max_memory_allocated() / 2 ** 30
    ms = sorted(times)[len(times) // 2]
    gp.graph = None
    del gp
    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return {"ktok_s": B * L / ms, "ms": ms, "runs_ms": times, "peak_gib": peak,
            "note": "whole prefill as one CUDA-graph replay, retain_kv=False (the reference's prefill benchmark protocol)"}


def timed_decode(gd, K, Wm):
    """Wm untimed steps (the graph is captured there), then K graph replays between two CUDA events. Returns ms."""
    for _ in range(Wm):
        gd.step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K):
        gd.step()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def fsl_step_bytes(model, gd, B, int8=True):
    a0 = gd.attn_core[0]
    P, Wc = a0._pool_cfg()
    kb = attn_bytes_per_layer(B, a0.n_heads, a0.head_dim, a0.window_size, P, Wc, a0.cell_topk, 32, int8)
    return weight_bytes(model) + len(gd.cache) * kb + B * a0.d_model * 2, kb


def fsb_step_bytes(model, gd, B, int8=True):
    a0 = gd.attn_core[0]
    nL = len(gd.cache)
    tot = 0
    for c in gd.cache:                      # admitted cells differ per layer: every layer's own forest heights
        fo = c.fsb
        mm = float(fo.m_tot[0].float().mean())
        mu = float(fo.m_tot[1].float().mean()) if fo.nf > 1 else 0.0
        tot += fsb_attn_bytes_per_layer(B, a0.n_heads, a0.head_dim, a0.window_size, a0.fsb_read_top, 32, mm, mu,
                                        a0.fsb_width, a0.fsb_union_width if fo.nf > 1 else 0, int8)
    return weight_bytes(model) + tot + B * a0.d_model * 2, tot // nL


# ---- legs outside the headline ------------------------------------------------------------------------------------------------
def _pub(table, ctx, value):
    ref = PUBLISHED[table].get(ctx)
    return (value / ref) if ref else None


def context_leg(model, variant, ctx, dev, K, Wm, peak):
    """One shorter context of BASELINE's 4k-131k range: prefill Ktok/s (one untimed run, one timed, fresh stores) and K
    graph-replayed decode steps, with the step's fraction of the HBM roofline."""
    from freesolo_b200.serving import GraphedDecoder
    ids = torch.randint(0, model.vocab_size, (1, ctx), generator=torch.Generator().manual_seed(4321 + ctx))
    kv = "bounded" if variant == "fsl" else "int8"
    gd, pms, _ = timed_prefill(lambda: GraphedDecoder(model, ids, Lmax=ctx + Wm + K + 40, device=dev, kv=kv), reps=1)
    ms = timed_decode(gd, K, Wm)
    sb, _ = (fsl_step_bytes if variant == "fsl" else fsb_step_bytes)(model, gd, 1)
    tps, ktoks = K / (ms * 1e-3), ctx / pms
    out = {"ctx": ctx, "prefill_ktok_s": ktoks, "decode_tok_s": tps, "decode_ms_per_step": ms / K, "decode_steps": K,
           "step_bytes": sb, "step_frac": sb / (ms / K * 1e-3) / 1e9 / peak,
           "vs_published_prefill": _pub(f"{variant}_prefill_ktoks", ctx, ktoks),
           "vs_published_decode": _pub(f"{variant}_decode_tps", ctx, tps), "kv_faults": list(gd.kv_faults())}
    del gd
    torch.cuda.empty_cache()
    g = timed_graph_prefill(model, ids, dev, reps=3)
    out["prefill_graph_ktok_s"] = g["ktok_s"]
    out["vs_published_prefill_graph"] = _pub(f"{variant}_prefill_ktoks", ctx, g["ktok_s"])
    return out


def make_fsb_model(args, dev, ctx):
    """the serve configuration with the second forest; thresholds = the 50th / 90th percentile of the
    cell ceilings of a 4096-token warm-up (the reference's fsb_calibrate_tau)."""
    from freesolo_b200.serving import FreeSoloLM, calibrate_fsb_tau, serve_kwargs
    torch.manual_seed(0)
    model = FreeSoloLM.from_config(args.model, max_seq_len=ctx + 512, **serve_kwargs("fsb", 0.9)).to(torch.bfloat16).to(dev).eval()
    warm_ids = torch.randint(0, model.vocab_size, (1, 4096), generator=torch.Generator().manual_seed(99))
    calibrate_fsb_tau(model, warm_ids, 0.5, "fsb_tau")
    calibrate_fsb_tau(model, warm_ids, 0.9, "fsb_tau_union")
    return model


def time_fsb_select(gd, ctx, dev, reps=3):
    """The FS-B prefill selection (both beams + re-rank) of one layer alone: forests rebuilt over layer 0's cell statistics
    and thresholds (the decoder's own were reduced to the decode arena after its prefill), random bf16 queries and token keys
    of the model's shape - random queries make a block's beams diverge, the slow case of the block-shared beam kernel; inside
    a real prefill they coincide - median of `reps` CUDA-event timings."""
    from freesolo_b200 import ops
    a, live = gd.attn_core[0], gd.cache[0].fsb
    fo = ops.FsbForests(live.kbar, live.ceil, live.taus[0], live.taus[1] if live.nf > 1 else None, cap_cells=ctx // 32)
    fo.ingest(ctx // 32)
    g = torch.Generator(device=dev).manual_seed(11)
    Q, K = (torch.randn(1, a.n_heads, ctx, a.head_dim, device=dev, generator=g).to(torch.bfloat16) for _ in range(2))
    lam, sigma, _, _ = a.head_params()
    ts = []
    for _ in range(reps + 1):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ops.fsb_select(fo, Q, K, lam, sigma, scale=a.scale, N=ctx, Bq=a._cell_block, width=a.fsb_width, width2=a._fsb_w2(fo),
                       read_top=a.fsb_read_top, radius_coef=a.fsb_bound_radius_coef)
        e1.record()
        ts.append((e0, e1))
    torch.cuda.synchronize()
    return sorted(x.elapsed_time(y) for x, y in ts[1:])[reps // 2]


def run_fsb_section(args, dev, K, Wm, peak, peak_kind):
    """FS-B 341M on the same box: prefill + forest build at args.ctx, K graph-replayed decode steps (int8 KV store; the
    forests take in new cells at every 128-token block), the step's roofline, and the shorter contexts."""
    from freesolo_b200.serving import GraphedDecoder
    ctx = args.ctx
    model = make_fsb_model(args, dev, ctx)
    ids = torch.randint(0, model.vocab_size, (args.batch, ctx), generator=torch.Generator().manual_seed(4321 + ctx))
    gd, prefill_ms, _ = timed_prefill(lambda: GraphedDecoder(model, ids, Lmax=ctx + Wm + K + 40, device=dev, kv="int8"))
    prefill_peak = PREFILL_PEAK_GIB[0]
    ms = timed_decode(gd, K, Wm)
    decode_peak = torch.cuda.max_memory_allocated() / 2 ** 30
    fo = gd.cache[0].fsb
    nL = len(gd.cache)
    sb, kb = fsb_step_bytes(model, gd, args.batch)
    tps, ktoks = args.batch * K / (ms * 1e-3), args.batch * ctx / prefill_ms
    out = {"workload": f"FS-B {args.model} (two forests, beam 16+16, token-LSE re-rank to 4), prefill + forest build at {ctx}, "
                       f"then {K} decode steps, batch {args.batch}, int8 KV",
           "decode_tok_s": tps, "decode_ms_per_step": ms / K, "prefill_ktok_s": ktoks, "prefill_ms": prefill_ms,
           "vs_published_decode": _pub("fsb_decode_tps", ctx, tps), "vs_published_prefill": _pub("fsb_prefill_ktoks", ctx, ktoks),
           "prefill_peak_gib": prefill_peak, "decode_peak_gib": decode_peak,
           "roofline": {"what": "whole decode step: weights + per layer window, both beams' visited nodes, the candidates' token "
                                "keys, the cells read", "bound": "hbm", "step_bytes": sb, "attn_bytes_per_layer": kb,
                        "achieved": sb / (ms / K * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                        "frac": sb / (ms / K * 1e-3) / 1e9 / peak, "peak_kind": peak_kind},
           "prefill_select_ms_per_layer": time_fsb_select(gd, ctx, dev),
           "gpu_launches": K * gd.launches_per_step(), "forest_bytes_per_layer": gd.fsb_bytes() // nL,
           "admitted_cells_layer0": {"main": fo.m_tot[0].tolist(), "second": fo.m_tot[1].tolist()},
           "kv_faults": list(gd.kv_faults())}
    del gd
    torch.cuda.empty_cache()
    if args.batch == 1:
        g = timed_graph_prefill(model, ids, dev)
        g["vs_published"] = _pub("fsb_prefill_ktoks", ctx, g["ktok_s"])
        out["prefill_graphed"] = g
    if not args.no_contexts:
        out["contexts"] = [context_leg(model, "fsb", c, dev, 32, Wm, peak) for c in (4096, 16384, 65536) if c < ctx]
    del model
    torch.cuda.empty_cache()
    return out


def run_linear_section(args, dev, ctx):
    """The streaming cache (LinearFSCache, a state of fixed size per layer): the 341M FS-L model takes a ctx-token prompt
    in 2048-token chunks, then a few greedy tokens through the same caches (eager, one attend per layer per token)."""
    from freesolo_b200.fsattn.kv_cache import linear_prefill, make_caches
    from freesolo_b200.serving import FreeSoloLM, extend_rope_cache, lm_head, serve_kwargs, trunk_cached
    torch.manual_seed(0)
    model = FreeSoloLM.from_config(args.model, max_seq_len=ctx + 512, **serve_kwargs("sparse")).to(torch.bfloat16).to(dev).eval()
    extend_rope_cache(model, ctx + 64)
    ids = torch.randint(0, model.vocab_size, (1, ctx), generator=torch.Generator().manual_seed(4321 + ctx)).to(dev)
    with torch.no_grad():
        linear_prefill(model, ids[:, :4096], make_caches(model, linear=True))        # untimed: handles, allocator pools
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats()
        caches = make_caches(model, linear=True)
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        h = linear_prefill(model, ids, caches)
        e1.record()
        tok = lm_head(model, h[:, -1]).argmax(-1).view(1, 1)
        steps = 8
        for _ in range(steps):
            tok = lm_head(model, trunk_cached(model, tok, caches)[:, -1]).argmax(-1).view(1, 1)
        e2.record()
        torch.cuda.synchronize()
    pms, dms = e0.elapsed_time(e1), e1.elapsed_time(e2)
    out = {"workload": f"FS-L {args.model} through LinearFSCache: {ctx}-token prompt in 2048-token chunks, then {steps} eager tokens",
           "prefill_ktok_s": ctx / pms, "prefill_ms": pms, "decode_tok_s": steps / (dms * 1e-3),
           "state_bytes_per_layer": caches[0].state_bytes(), "peak_gib": torch.cuda.max_memory_allocated() / 2 ** 30,
           "note": "state and activations do not grow with the prompt; every 128-token block of every layer is four launches "
                   "(cell statistics, pool merge, selection, readout + combine) issued from Python, so the rate is bound by "
                   "the host (the reference's is pure torch)"}
    del caches, model
    torch.cuda.empty_cache()
    return out


def dense_step_bytes(model, gd, B, ctx, int8=True):
    """Dense FS decode step: weights + per layer the window, the fp32 mean key and ceiling of EVERY visible cell, the kk
    cells read, the new row."""
    a0 = gd.attn_core[0]
    e = 1 if int8 else 2
    m_vis = (ctx // a0._cell_block) * a0._cell_block // 32
    per = (a0.window_size + 1) * a0.head_dim * 2 * e + m_vis * (a0.head_dim * 4 + 4) + a0.cell_topk * 32 * a0.head_dim * 2 * e + 4 * a0.head_dim
    return weight_bytes(model) + len(gd.cache) * B * a0.n_heads * per + B * a0.d_model * 2


def run_dense_section(args, dev, K, Wm, peak, peak_kind):
    """The reference's third serving variant, FS (dense): no candidate pool, every completed visible cell is scored (tensor-core
    selection in prefill, a cluster split top-k per decode token), int8 KV store."""
    from freesolo_b200.serving import FreeSoloLM, GraphedDecoder, serve_kwargs
    ctx = args.ctx
    torch.manual_seed(0)
    model = FreeSoloLM.from_config(args.model, max_seq_len=ctx + 512, **serve_kwargs("dense")).to(torch.bfloat16).to(dev).eval()
    ids = torch.randint(0, model.vocab_size, (1, ctx), generator=torch.Generator().manual_seed(4321 + ctx))
    gd, pms, _ = timed_prefill(lambda: GraphedDecoder(model, ids, Lmax=ctx + Wm + K + 40, device=dev, kv="int8"))
    prefill_peak = PREFILL_PEAK_GIB[0]
    ms = timed_decode(gd, K, Wm)
    decode_peak = torch.cuda.max_memory_allocated() / 2 ** 30
    sb = dense_step_bytes(model, gd, 1, ctx)
    tps, ktoks = K / (ms * 1e-3), ctx / pms
    out = {"workload": f"FS (dense) {args.model}: every visible cell scored, prefill at {ctx}, then {K} decode steps, batch 1, int8 KV",
           "decode_tok_s": tps, "decode_ms_per_step": ms / K, "prefill_ktok_s": ktoks, "prefill_ms": pms,
           "vs_published_decode": _pub("dense_decode_tps", ctx, tps), "vs_published_prefill": _pub("dense_prefill_ktoks", ctx, ktoks),
           "prefill_peak_gib": prefill_peak, "decode_peak_gib": decode_peak,
           "roofline": {"what": "whole decode step", "bound": "hbm", "step_bytes": sb, "achieved": sb / (ms / K * 1e-3) / 1e9, "peak": peak,
                        "unit": "GB/s", "frac": sb / (ms / K * 1e-3) / 1e9 / peak, "peak_kind": peak_kind},
           "gpu_launches": K * gd.launches_per_step(), "kv_faults": list(gd.kv_faults())}
    del gd
    torch.cuda.empty_cache()
    g = timed_graph_prefill(model, ids, dev)
    g["vs_published"] = _pub("dense_prefill_ktoks", ctx, g["ktok_s"])
    out["prefill_graphed"] = g
    del model
    torch.cuda.empty_cache()
    return out


def run_config4(dev, K, Wm, peak, peak_kind, batch=32, ctx=32768, dist=None, seed_off=0):
    """FS-L, the 743M-class model ("800m": 24 x 1536, 16 heads x 96), `batch` sequences of `ctx` tokens on
    this GPU, full int8 KV store. With `dist` (N > 1) the 32 sequences are split 32/N over the ranks, no collective in the
    step; the time is the max over ranks. Above 8 sequences per GPU the trunk projections are library GEMMs."""
    from freesolo_b200.serving import FreeSoloLM, GraphedDecoder, serve_kwargs
    torch.manual_seed(0)
    model = FreeSoloLM.from_config("800m", max_seq_len=ctx + 512, **serve_kwargs("sparse")).to(torch.bfloat16).to(dev).eval()
    ids = torch.randint(0, model.vocab_size, (batch, ctx), generator=torch.Generator().manual_seed(777 + seed_off))
    gd = GraphedDecoder(model, ids, Lmax=ctx + Wm + K + 40, device=dev, kv="int8")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    gd.prefill()
    e1.record()
    torch.cuda.synchronize()
    pms = e0.elapsed_time(e1)
    if dist is not None:
        dist.barrier()
    ms = timed_decode(gd, K, Wm)
    world = 1
    if dist is not None:
        t = torch.tensor([ms, pms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, pms = t.tolist()
        world = dist.get_world_size()
    sb, kb = fsl_step_bytes(model, gd, batch)
    k_avg, _ = time_decode_kernel(gd, n=24)
    nL = len(gd.cache)
    out = {"workload": f"FS-L 800m (24 x 1536, 16 heads x 96), {batch * world} sequences of {ctx} tokens ({batch} per GPU x {world}), "
                       f"full int8 KV store, {K} graph-replayed decode steps",
           "decode_tok_s": batch * world * K / (ms * 1e-3), "decode_ms_per_step": ms / K, "decode_steps": K,
           "prefill_ktok_s": batch * world * ctx / pms, "prefill_ms": pms, "prefill_note": "one cold run",
           "step_bytes_per_gpu": sb, "step_frac": sb / (ms / K * 1e-3) / 1e9 / peak,
           "decode_kernel": {"kernel": "fsl_decode_kernel", "bytes_per_launch": kb, "avg_launch_us": k_avg * 1e3,
                             "achieved": kb / (k_avg * 1e-3) / 1e9, "unit": "GB/s", "frac": kb / (k_avg * 1e-3) / 1e9 / peak,
                             "peak_kind": peak_kind, "how": "launched alone, L2 flushed before every launch, CUDA events"},
           "kv_bytes_per_layer": gd.kv_bytes() // nL, "kv_faults": list(gd.kv_faults())}
    del gd, model
    torch.cuda.empty_cache()
    return out


def run_head_sharded(args, dev, K, Wm, rank, world, dist):
    """One sequence, heads split over the ranks (BASELINE config 5's partition on the headline model): rank r owns heads
    [r H/g, (r+1) H/g), its KV stores and pools; the head outputs meet once per layer in front of W_o. Strong scaling."""
    from freesolo_b200.parallel import shard_model_heads
    from freesolo_b200.serving import FreeSoloLM, GraphedDecoder, serve_kwargs
    ctx = args.ctx
    torch.manual_seed(0)
    model = FreeSoloLM.from_config(args.model, max_seq_len=ctx + 512, **serve_kwargs("sparse")).to(torch.bfloat16).to(dev).eval()
    n_heads = model.blocks[0].attn.fsattn.n_heads
    shard_model_heads(model, rank, world)
    ids = torch.randint(0, model.vocab_size, (1, ctx), generator=torch.Generator().manual_seed(4321 + ctx))
    import gc

    def one(peer: bool):
        """prefill + K timed steps with the exchange over peer memory (this library's kernel) or as NCCL all-gathers"""
        os.environ["FSATTN_PEER_GATHER"] = "1" if peer else "0"
        try:
            gd = GraphedDecoder(model, ids, Lmax=ctx + Wm + K + 40, device=dev, kv=args.kv)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            gd.prefill()
            e1.record()
            torch.cuda.synchronize()
            pms = e0.elapsed_time(e1)
            dist.barrier()
            ms = timed_decode(gd, K, Wm)
            t = torch.tensor([ms, pms, float(gd.peer_status())], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            faults = list(gd.kv_faults())
            used_peer = gd.peer is not None
            # a graph that captured collectives keeps the communicator busy: it goes before the process group does
            gd.graph = None
            if gd.peer is not None:
                gd.peer.close()
            del gd
            gc.collect()
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
            return t.tolist() + [faults, used_peer]
        finally:
            del os.environ["FSATTN_PEER_GATHER"]

    ms, pms, status, faults, used_peer = one(True)
    ms_nccl, _, _, _, _ = one(False)
    out = {"workload": f"FS-L {args.model}, ONE sequence of {ctx} tokens, {n_heads} heads split over "
                       f"{world} GPUs, exchange of the head outputs once per layer, {K} graph-replayed decode steps",
           "scaling": "strong", "decode_tok_s": K / (ms * 1e-3), "decode_ms_per_step": ms / K,
           "exchange": ("one launch of this library per rank and layer: stores + flag into the peers' memory, bounded wait"
                        if used_peer else "NCCL all-gather"),
           "peer_wait_status": int(status),
           "decode_tok_s_nccl_allgather": K / (ms_nccl * 1e-3), "decode_ms_per_step_nccl_allgather": ms_nccl / K,
           "prefill_ktok_s": ctx / pms, "prefill_ms": pms, "prefill_note": "one cold run", "kv_faults": faults}
    del model
    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def run_config5(args, dev, rank, world, dist):
    """BASELINE config 5's shape: FS-B, the 743M-class model (16 heads x 96), ONE sequence of `--config5-ctx` tokens (default
    262144), heads split over the ranks (each rank builds and searches the forests of its own heads; the head outputs meet once
    per layer), thresholds from a 4096-token warm-up, int8 KV store, up to 128 graph-replayed decode steps."""
    from freesolo_b200.parallel import shard_model_heads
    from freesolo_b200.serving import FreeSoloLM, GraphedDecoder, calibrate_fsb_tau, serve_kwargs
    ctx, nL = args.config5_ctx, args.config5_layers
    torch.manual_seed(0)
    model = FreeSoloLM.from_config("800m", n_layers=nL, max_seq_len=ctx + 512, **serve_kwargs("fsb", 0.9)).to(torch.bfloat16).to(dev).eval()
    warm_ids = torch.randint(0, model.vocab_size, (1, 4096), generator=torch.Generator().manual_seed(99))
    calibrate_fsb_tau(model, warm_ids, 0.5, "fsb_tau")
    calibrate_fsb_tau(model, warm_ids, 0.9, "fsb_tau_union")
    n_heads = model.blocks[0].attn.fsattn.n_heads
    if world > 1:
        shard_model_heads(model, rank, world)
    K, Wm = min(args.steps, 128), 3
    ids = torch.randint(0, model.vocab_size, (1, ctx), generator=torch.Generator().manual_seed(4321 + ctx))
    torch.cuda.reset_peak_memory_stats()
    gd = GraphedDecoder(model, ids, Lmax=ctx + Wm + K + 40, device=dev, kv="int8")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    gd.prefill()
    e1.record()
    torch.cuda.synchronize()
    pms = e0.elapsed_time(e1)
    if world > 1:
        dist.barrier()
    ms = timed_decode(gd, K, Wm)
    if world > 1:
        t = torch.tensor([ms, pms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, pms = t.tolist()
    fo = gd.cache[0].fsb
    out = {"workload": f"FS-B 800m-class ({nL} layers x 1536, {n_heads} heads x 96), ONE sequence of {ctx} tokens, heads split over "
                       f"{world} GPU(s), int8 KV, {K} graph-replayed decode steps",
           "layers": nL, "ctx": ctx, "decode_tok_s": K / (ms * 1e-3), "decode_ms_per_step": ms / K,
           "prefill_ktok_s": ctx / pms, "prefill_ms": pms, "prefill_note": "one cold run, forest build included",
           "forest_bytes_per_layer_per_gpu": gd.fsb_bytes() // nL, "forest_cells_cap": fo.m_cap,
           "admitted_cells_layer0_rank0": {"main": fo.m_tot[0].tolist(), "second": fo.m_tot[1].tolist()},
           "kv_bytes_per_layer_per_gpu": gd.kv_bytes() // nL, "peak_mem_gib_per_gpu": torch.cuda.max_memory_allocated() / 2 ** 30,
           "exchange": "peer memory" if gd.peer is not None else ("NCCL all-gather" if world > 1 else "none"),
           "peer_wait_status": gd.peer_status(), "kv_faults": list(gd.kv_faults())}
    gd.graph = None
    if gd.peer is not None:
        gd.peer.close()
    del gd, model
    import gc
    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


# ---- the measured arm ---------------------------------------------------------------------------------------------------------
def run_ours(args):
    import torch.distributed as dist
    from freesolo_b200.serving import FreeSoloLM, GraphedDecoder, serve_kwargs
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        # a stuck collective aborts the run after two minutes instead of holding the GPUs
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    ctx, K, Wm = args.ctx, args.steps, max(args.warmup, 3)
    hbm_peak, _, peak_kind = _peaks()
    torch.manual_seed(0)
    model = FreeSoloLM.from_config(args.model, max_seq_len=ctx + 512, **serve_kwargs("sparse")).to(torch.bfloat16).to(dev).eval()
    B = args.batch
    heads = world > 1 and args.shard == "heads"
    if heads:
        # one sequence, 16/g heads per rank, the head outputs exchanged once per layer inside the step graph
        from freesolo_b200.parallel import shard_model_heads
        shard_model_heads(model, rank, world)
    ids = torch.randint(0, model.vocab_size, (B, ctx), generator=torch.Generator().manual_seed(4321 + ctx + (0 if heads else rank)))
    total = Wm + 2 * K + 40
    # one short untimed prefill first: library handles, kernel attributes and allocator pools are initialised there
    warm = GraphedDecoder(model, ids[:, :min(ctx, 2048)], Lmax=min(ctx, 2048) + 64, device=dev, kv=args.kv)
    warm.prefill()
    del warm
    gd, prefill_ms, prefill_all = timed_prefill(lambda: GraphedDecoder(model, ids, Lmax=ctx + total, device=dev, kv=args.kv))
    prefill_peak = PREFILL_PEAK_GIB[0]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(Wm):
        gd.step()
    torch.cuda.synchronize()
    assert gd.graph is not None

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- device-timed: K graph replays, inputs resident in HBM -----------------------------------------------------
    barrier()
    with ClockSampler(local) as cs:
        e0.record()
        for _ in range(K):
            gd.step()
        e1.record()
        barrier()
    ms = e0.elapsed_time(e1)
    decode_peak = torch.cuda.max_memory_allocated() / 2 ** 30       # the timed prefills + the graph capture + the decode steps
    # ---- end to end: token id from pinned host memory in, sampled token back to the host, every step --------------
    tok_host = torch.zeros(B, 1, dtype=torch.int64).pin_memory()
    tok_host.copy_(gd.tok.cpu())
    out_host = torch.zeros(B, 1, dtype=torch.int64).pin_memory()
    gd.step_host(tok_host, out_host)                  # untimed: captures the graph that carries the two copies
    torch.cuda.current_stream().synchronize()
    tok_host.copy_(out_host)
    barrier()
    t0 = time.perf_counter()
    for _ in range(K):
        gd.step_host(tok_host, out_host)              # pinned host id in, step, sampled id back to pinned host memory
        torch.cuda.current_stream().synchronize()
        tok_host.copy_(out_host)
    barrier()
    e2e_s = time.perf_counter() - t0
    t = torch.tensor([ms, e2e_s * 1e3], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = t.tolist()
    faults = gd.kv_faults()
    a0 = gd.attn_core[0]
    int8 = args.kv != "bf16"
    nL = len(gd.cache)
    step_bytes, kbytes = fsl_step_bytes(model, gd, B, int8)
    seqs = B if heads else world * B
    value = seqs * K / (ms * 1e-3)
    w_mb = weight_bytes(model) / 1e6
    line = {
        "metric": "fsl_decode_tok_s", "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": Wm,
        "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong" if heads else "weak",
        "vs_baseline": _pub("fsl_decode_tps", ctx, value) if (args.model == "340m" and B == 1 and world == 1) else None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"FS-L {args.model} decode after a {ctx}-token prefill, batch {B} per GPU, kv store {args.kv}, greedy, "
                               "one CUDA-graph replay per token", "ctx": ctx, "batch_per_gpu": B, "kv": args.kv,
                   "l2": f"every step streams all weights ({w_mb:.0f} MB for {args.model}) > 126 MB L2, no flush needed",
                   "parallelism": (f"head-sharded x{world}, head outputs exchanged once per layer" if heads
                                   else f"batch-sharded x{world}, no collective")},
        "clocks": cs.summary(),
        "e2e": {"value": seqs * K / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": 8 * B, "d2h_bytes_per_step": 8 * B},
        "gpu_launches": K * (gd.launches_per_step() if B <= 8 else nL),      # above 8 rows the projections are library GEMMs
        "step_roofline": {"step_bytes": step_bytes, "achieved_gbs": step_bytes / (ms / K * 1e-3) / 1e9,
                          "frac": step_bytes / (ms / K * 1e-3) / 1e9 / hbm_peak, "peak_kind": peak_kind},
        "prefill": {"ktok_s": B * ctx / prefill_ms, "ms": prefill_ms, "runs_ms": prefill_all,
                    "vs_published": _pub("fsl_prefill_ktoks", ctx, B * ctx / prefill_ms) if (args.model == "340m" and B == 1) else None,
                    "peak_gib": prefill_peak,
                    "note": "median of 3 after one untimed full-context prefill (the reference's --warm 1 --nmed 3), incl. KV store "
                            "fill and last-token logits; outside the headline's timed region"},
        "kv_bytes_per_layer": gd.kv_bytes() // nL, "kv_faults": list(faults),
    }
    # ---- rooflines of the step's kernels, measured live (rank 0 reports; every rank runs them so the ranks stay in step) ----
    k_avg_ms, k_med_ms = time_decode_kernel(gd)
    dk = {"kernel": "fsl_decode_kernel", "bound": "hbm (latency-bound at batch 1: 1.6 MB per launch)", "bytes_per_launch": kbytes,
          "avg_launch_us": k_avg_ms * 1e3, "median_launch_us": k_med_ms * 1e3, "achieved": kbytes / (k_avg_ms * 1e-3) / 1e9,
          "peak": hbm_peak, "unit": "GB/s", "frac": kbytes / (k_avg_ms * 1e-3) / 1e9 / hbm_peak, "peak_kind": peak_kind,
          "traffic": NCU_DRAM_BYTES.get(f"fsl_decode_kernel/{args.model}/b{B}"),
          "traffic_source": "ncu dram__bytes_read + dram__bytes_write per launch, 32k-context capture (the FS-L decode read does "
                            "not depend on the context); null = no capture of this shape, not measured in this run",
          "how": "launched alone with an L2 flush before every launch, CUDA events on the launching stream"}
    if B <= 8 and not heads:
        n_launch, chain_ms = time_gemv_chain(gd)
        wb = weight_bytes(model)
        line["roofline"] = {
            "kernel": "trunk_gemv_kernel", "bound": "hbm", "achieved": wb / (chain_ms * 1e-3) / 1e9, "peak": hbm_peak, "unit": "GB/s",
            "frac": wb / (chain_ms * 1e-3) / 1e9 / hbm_peak, "peak_kind": peak_kind,
            "traffic": NCU_DRAM_BYTES.get(f"trunk_gemv_kernel/{args.model}/b{B}"),
            "traffic_source": "ncu dram__bytes_read + dram__bytes_write, weighted mean over one step's 97 launches; null = no "
                              "capture of this shape, not measured in this run",
            "bytes_per_launch": wb / n_launch, "avg_launch_us": chain_ms * 1e3 / n_launch, "launches_per_step": n_launch,
            "share_of_step": chain_ms / (ms / K),
            "why": "the step's dominant kernel: the 4 projections of every layer + the LM head stream all weights once per token",
            "how": "the step's own chain of projection launches (programmatic dependent launch, attention launches left out) "
                   "captured once and replayed 20 times between two CUDA events; algorithmic bytes = all weights / launches"}
        line["decode_kernel_roofline"] = dk
    else:
        line["roofline"] = dk
    line["peak_mem_gib"] = decode_peak
    if world == 1 and args.model == "340m":
        line["window_roofline"] = time_window_kernel(gd.attn_core[0], dev, ctx)
    del gd
    torch.cuda.empty_cache()
    if world == 1 and B == 1:
        g = timed_graph_prefill(model, ids, dev)
        g["vs_published"] = _pub("fsl_prefill_ktoks", ctx, g["ktok_s"])
        line["prefill"]["graphed"] = g
    if world == 1 and args.model == "340m" and B == 1 and not args.no_contexts:
        line["contexts"] = [context_leg(model, "fsl", c, dev, 32, Wm, hbm_peak) for c in (4096, 16384, 65536) if c < ctx]
    del model
    torch.cuda.empty_cache()
    if world == 1 and not args.no_fsb:
        line["fsb"] = run_fsb_section(args, dev, K, Wm, hbm_peak, peak_kind)
    if world == 1 and not args.no_dense and args.model == "340m":
        line["fs_dense"] = run_dense_section(args, dev, K, Wm, hbm_peak, peak_kind)
    if world == 1 and args.linear_ctx > 0 and args.model == "340m" and B == 1:
        line["linear_cache"] = run_linear_section(args, dev, args.linear_ctx)
    if not args.no_config4 and args.model == "340m" and B == 1 and not heads:
        per = max(1, 32 // world)
        key = "config4" if world == 1 else "config4_split"
        line[key] = run_config4(dev, min(K, 24), Wm, hbm_peak, peak_kind, batch=per, ctx=args.config4_ctx,
                                dist=dist if world > 1 else None, seed_off=rank)
    if world > 1 and not heads and not args.no_head_leg and args.model == "340m" and B == 1:
        line["head_sharded"] = run_head_sharded(args, dev, K, Wm, rank, world, dist)
        line["head_sharded"]["speedup_vs_one_rank_of_this_run"] = line["head_sharded"]["decode_tok_s"] / (value / world)
    if args.config5:
        line["config5"] = run_config5(args, dev, rank, world, dist)
    if world > 1:
        # every rank leaves the group together; what follows on rank 0 needs no communication
        barrier()
        import gc
        gc.collect()
        torch.cuda.synchronize()
        dist.destroy_process_group()
    if rank != 0:
        return
    if world == 1 and not args.no_cpu:
        from oracle.ref_cpu import time_fsl_decode
        r = time_fsl_decode(args.cpu_sample_ctx, 12, 2)
        line["cpu_baseline"] = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ctx", type=int, default=131072)
    ap.add_argument("--cpu-ctx", type=int, default=2304, help="context of the reference arm's CPU sample (72 cells fill the FS-L pool)")
    ap.add_argument("--cpu-sample-ctx", type=int, default=1152, help="context of the cpu_baseline leg inside the measured arm")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--model", default="340m")
    ap.add_argument("--kv", default="bounded", choices=["bounded", "int8", "bf16"])
    ap.add_argument("--shard", default="batch", choices=["batch", "heads"],
                    help="N > 1: 'batch' = one sequence per rank, no collective (weak scaling); 'heads' = one sequence, heads "
                         "split over the ranks, head outputs exchanged once per layer (strong scaling)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-fsb", action="store_true", help="skip the FS-B section (BASELINE config 3) of the N=1 line")
    ap.add_argument("--no-dense", action="store_true", help="skip the dense FS section of the N=1 line")
    ap.add_argument("--linear-ctx", type=int, default=16384,
                    help="prompt length of the streaming-cache (LinearFSCache) leg of the N=1 line; 0 skips it")
    ap.add_argument("--no-contexts", action="store_true", help="skip the 4k / 16k / 64k legs")
    ap.add_argument("--no-config4", action="store_true", help="skip BASELINE config 4 (743M-class, 32 sequences)")
    ap.add_argument("--no-head-leg", action="store_true", help="N > 1: skip the head-sharded leg")
    ap.add_argument("--config5", action="store_true",
                    help="also run BASELINE config 5's shape (FS-B 743M-class, one long sequence, heads split over the ranks)")
    ap.add_argument("--config5-ctx", type=int, default=262144)
    ap.add_argument("--config5-layers", type=int, default=24)
    ap.add_argument("--config4-ctx", type=int, default=32768, help="context of config 4's sequences (smaller for profiler captures)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
