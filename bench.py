"""Benchmark of the FS-L decode hot path: `python bench.py --gpus N --steps K --warmup W [--impl reference]`.

Workload (the largest single-GPU point): FS-L 341M model (24 layers, d_model 1024, 16 heads x 64, vocab
32000), random-init bf16 weights, batch 1, uniform random token ids; an untimed prefill of `--ctx` tokens (default 131072)
through this repo's kernels, then greedy decode. A step = one decoded token through the whole model (one CUDA-graph replay).
  value  : tok/s over exactly K replays timed with CUDA events (inputs resident in HBM), max over ranks
  e2e    : tok/s through the public decoder API with the token id copied from pinned host memory every step and the
           sampled token read back to the host every step
With N > 1 ranks (torchrun) every rank decodes its own sequence (batch sharding, no collective): weak scaling.
`--impl reference` times the CPU port of the reference's eager decode (oracle/model.py) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PUBLISHED_FSL_DECODE_TPS_131K = 515.1      # A100-40GB, README.md:62 of the reference
NCU_DECODE_KERNEL_DRAM_BYTES = 1.87e6       # profiles/fsl_decode_kernel_340m_ncu_full.md
PUBLISHED_FSB_DECODE_TPS_131K = 462.7      # A100-40GB, README.md:63 of the reference
PUBLISHED_FSB_PREFILL_KTOKS_131K = 137.8   # A100-40GB, README.md:63 of the reference
W_BYTES_341M = 2 * (24 * (4 * 1024 ** 2 + 3 * 1024 * 2816) + 32000 * 1024)


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.isfile(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


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


def attn_bytes_per_layer(B, H, D, W, P, Wc, kk, s, int8=True):
    """Algorithmic bytes one decode-step launch of one layer moves (window rows of K and V, the pool's
    mean keys + per-slot scalars, the kk cells read, the new row)."""
    e = 1 if int8 else 2
    win = (W + 1) * D * 2 * e
    pool = (P + Wc) * (D * 4 + 17)
    read = kk * s * D * 2 * e
    new = 2 * D * 2
    return B * H * (win + pool + read + new)


def run_reference(args):
    """The reference's eager decode restated on CPU (oracle/model.py), all host threads, a bounded sample of the workload."""
    from oracle.model import CpuFSLModel
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    ctx = min(args.ctx, args.cpu_ctx)
    steps, warm = min(args.steps, 24), min(args.warmup, 3)
    torch.set_num_threads(os.cpu_count() or 1)
    m = CpuFSLModel(max_len=ctx + steps + warm + 64)
    m.synthetic_context(1, ctx)
    tok = torch.zeros(1, 1, dtype=torch.long)
    for _ in range(warm):
        tok = m.step(tok)
    t0 = time.perf_counter()
    for _ in range(steps):
        tok = m.step(tok)
    dt = time.perf_counter() - t0
    tps = steps / dt
    sample = f"{steps} greedy decode steps of the 341M FS-L model, fp32, batch 1, synthetic {ctx}-token context (the decode step's cost is context-independent for FS-L)"
    line = {"impl": "reference", "metric": "fsl_decode_tok_s", "value": tps, "unit": "tok/s", "n_gpus": args.gpus, "steps": steps,
            "warmup": warm, "ms_per_step": dt / steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"FS-L 341M decode, batch 1, ctx {args.ctx} (CPU sample at ctx {ctx})"},
            "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port", "sample": sample},
            "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cpu_baseline_sample(ctx=4096, steps=12, warm=2):
    from oracle.model import CpuFSLModel
    nt = torch.get_num_threads()
    torch.set_num_threads(os.cpu_count() or 1)
    m = CpuFSLModel(max_len=ctx + steps + warm + 64)
    m.synthetic_context(1, ctx)
    tok = torch.zeros(1, 1, dtype=torch.long)
    for _ in range(warm):
        tok = m.step(tok)
    t0 = time.perf_counter()
    for _ in range(steps):
        tok = m.step(tok)
    dt = time.perf_counter() - t0
    cores = torch.get_num_threads()
    torch.set_num_threads(nt)
    return {"value": steps / dt, "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{steps} decode steps of the 341M FS-L model (oracle/model.py, fp32, batch 1) at a synthetic {ctx}-token context"}


def time_decode_kernel(gd, n=48):
    """Average duration of the fused decode-step kernel launched alone, L2 flushed before every launch (in the real step
    682 MB of weights pass through L2 between two launches of the same layer, so its KV rows are cold)."""
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
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peak, kind = (float(json.load(open(p))["bf16_tflops"]), "measured") if os.path.isfile(p) else (1590.0, "fallback")
    return {"kernel": "rope_qk_kernel + window_tc_kernel", "bound": "tensor", "achieved": flops / (ms * 1e-3) / 1e12, "peak": peak,
            "unit": "TFLOP/s", "frac": flops / (ms * 1e-3) / 1e12 / peak, "peak_kind": kind, "ms": ms, "tokens": n, "heads": H,
            "how": "launched alone on random operands larger than L2, median of 5, CUDA events on the launching stream; "
                   "useful FLOPs only (masked parts of the key tiles not counted)"}


def timed_prefill(make_decoder, reps: int = 3):
    """The reference's prefill protocol (experiments/scaling/bench_efficiency.py:166-198, `--warm 1 --nmed 3`): one untimed
    prefill at the full context (the allocator's pools and every kernel attribute are warm afterwards), then the median of
    `reps` timed ones, each on a fresh decoder (fresh KV stores / forests). Returns (last decoder, median ms, all ms)."""
    import torch
    gd = make_decoder()
    gd.prefill()
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        del gd
        gd = make_decoder()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        gd.prefill()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    return gd, sorted(times)[len(times) // 2], times



def run_fsb_section(args, dev, K, Wm):
    """BASELINE config 3 on the same box: FS-B 341M (serve configuration with the second forest), thresholds calibrated
    as the 50th / 90th percentile of the cell ceilings of a 4096-token warm-up, prefill + forest build at args.ctx,
    then K graph-replayed decode steps (int8 KV store; the forests take in new cells at every 128-token block)."""
    from freesolo_b200.serving import FreeSoloLM, GraphedDecoder, calibrate_fsb_tau, serve_kwargs
    ctx = args.ctx
    torch.manual_seed(0)
    model = FreeSoloLM.from_config(args.model, max_seq_len=ctx + 512, **serve_kwargs("fsb", 0.9)).to(torch.bfloat16).to(dev).eval()
    g = torch.Generator().manual_seed(99)
    warm_ids = torch.randint(0, model.vocab_size, (1, 4096), generator=g)
    calibrate_fsb_tau(model, warm_ids, 0.5, "fsb_tau")
    calibrate_fsb_tau(model, warm_ids, 0.9, "fsb_tau_union")
    ids = torch.randint(0, model.vocab_size, (args.batch, ctx), generator=torch.Generator().manual_seed(4321 + ctx))
    gd, prefill_ms, _ = timed_prefill(lambda: GraphedDecoder(model, ids, Lmax=ctx + Wm + K + 40, device=dev, kv="int8"))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(Wm):
        gd.step()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(K):
        gd.step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    fo = gd.cache[0].fsb
    nL = len(gd.cache)
    out = {"workload": f"FS-B {args.model} (two forests, beam 16+16, token-LSE re-rank to 4), prefill + forest build at {ctx}, "
                       f"then {K} decode steps, batch {args.batch}, int8 KV",
           "decode_tok_s": args.batch * K / (ms * 1e-3), "decode_ms_per_step": ms / K,
           "prefill_ktok_s": args.batch * ctx / prefill_ms, "prefill_ms": prefill_ms,
           "vs_published_decode": (args.batch * K / (ms * 1e-3)) / PUBLISHED_FSB_DECODE_TPS_131K if ctx == 131072 else None,
           "vs_published_prefill": (args.batch * ctx / prefill_ms) / PUBLISHED_FSB_PREFILL_KTOKS_131K if ctx == 131072 else None,
           "gpu_launches": K * gd.launches_per_step(), "forest_bytes_per_layer": gd.fsb_bytes() // nL,
           "admitted_cells_layer0": {"main": fo.m_tot[0].tolist(), "second": fo.m_tot[1].tolist()},
           "kv_faults": list(gd.kv_faults())}
    del gd, model
    torch.cuda.empty_cache()
    return out


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
    torch.manual_seed(0)
    model = FreeSoloLM.from_config(args.model, max_seq_len=ctx + 512, **serve_kwargs("sparse")).to(torch.bfloat16).to(dev).eval()
    B = args.batch
    heads = world > 1 and args.shard == "heads"
    if heads:
        # one sequence, 16/g heads per rank, NCCL all-gather of the head outputs per layer (captured in the step graph)
        from freesolo_b200.parallel import shard_model_heads
        shard_model_heads(model, rank, world)
    ids = torch.randint(0, model.vocab_size, (B, ctx), generator=torch.Generator().manual_seed(4321 + ctx + (0 if heads else rank)))
    total = Wm + 2 * K + 32
    # one short untimed prefill first: library handles, kernel attributes and allocator pools are initialised there
    warm = GraphedDecoder(model, ids[:, :min(ctx, 2048)], Lmax=min(ctx, 2048) + 64, device=dev, kv=args.kv)
    warm.prefill()
    del warm
    if os.environ.get("FSATTN_BENCH_TRACE", "0") == "1":
        torch.cuda.synchronize()
        print(f"[bench] rank {rank}: warm-up prefill ok", file=sys.stderr, flush=True)
    gd, prefill_ms, prefill_all = timed_prefill(lambda: GraphedDecoder(model, ids, Lmax=ctx + total, device=dev, kv=args.kv))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    def mark(what):
        if os.environ.get("FSATTN_BENCH_TRACE", "0") == "1":
            torch.cuda.synchronize()
            print(f"[bench] rank {rank}: {what} ok", file=sys.stderr, flush=True)
    mark("prefill")
    for _ in range(Wm):
        gd.step()
    torch.cuda.synchronize()
    assert gd.graph is not None
    mark("warmup")

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
    mark("timed region")
    # ---- end to end: token id from pinned host memory in, sampled token back to the host, every step --------------
    tok_host = torch.zeros(B, 1, dtype=torch.int64).pin_memory()
    tok_host.copy_(gd.tok.cpu())
    out_host = torch.zeros(B, 1, dtype=torch.int64).pin_memory()
    barrier()
    t0 = time.perf_counter()
    for _ in range(K):
        gd.tok.copy_(tok_host, non_blocking=True)
        gd.step()
        out_host.copy_(gd.tok, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        tok_host.copy_(out_host)
    barrier()
    e2e_s = time.perf_counter() - t0
    mark("e2e region")
    t = torch.tensor([ms, e2e_s * 1e3], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = t.tolist()
    faults = gd.kv_faults()
    if world > 1:
        # every rank leaves the group together; what follows on rank 0 needs no communication. A graph that captured
        # NCCL collectives (head sharding) keeps the communicator busy: NCCL's teardown waits for it, so it goes first.
        barrier()
        gd.graph = None
        import gc
        gc.collect()
        torch.cuda.synchronize()
        dist.destroy_process_group()
        mark("process group closed")
    if rank != 0:
        return
    peak, peak_kind = _peaks()
    a0 = gd.attn_core[0]
    P, Wc = a0._pool_cfg()
    int8 = args.kv != "bf16"
    kbytes = attn_bytes_per_layer(B, a0.n_heads, a0.head_dim, a0.window_size, P, Wc, a0.cell_topk, 32, int8)
    k_avg_ms, k_med_ms = time_decode_kernel(gd)
    achieved = kbytes / (k_avg_ms * 1e-3) / 1e9
    nL = len(gd.cache)
    w_bytes = 2 * sum(p.numel() for n_, p in model.named_parameters() if p.dim() > 1)
    step_bytes = w_bytes + nL * kbytes + B * a0.d_model * 2
    seqs = B if heads else world * B
    value = seqs * K / (ms * 1e-3)
    line = {
        "metric": "fsl_decode_tok_s", "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": Wm,
        "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong" if heads else "weak",
        "vs_baseline": value / PUBLISHED_FSL_DECODE_TPS_131K if (args.model == "340m" and B == 1 and world == 1) else None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"FS-L {args.model} decode after a {ctx}-token prefill, batch {B} per GPU, kv store {args.kv}, greedy, "
                               "one CUDA-graph replay per token", "ctx": ctx, "batch_per_gpu": B, "kv": args.kv,
                   "l2": "every step streams all weights (682 MB for 340m) > 126 MB L2, no flush needed",
                   "parallelism": (f"head-sharded x{world}, NCCL all-gather of head outputs per layer" if heads
                                   else f"batch-sharded x{world}, no collective")},
        "clocks": cs.summary(),
        "e2e": {"value": seqs * K / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": 8 * B, "d2h_bytes_per_step": 8 * B},
        "gpu_launches": K * (gd.launches_per_step() if B <= 8 else nL),      # above 8 rows the projections are library GEMMs
        "roofline": {"kernel": "fsl_decode_kernel", "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": NCU_DECODE_KERNEL_DRAM_BYTES if (B == 1 and args.model == "340m") else None,
                     "traffic_source": "ncu dram__bytes_read+write per launch, profiles/fsl_decode_kernel_340m_ncu_full.md "
                                       "(captured at ctx 32768; the FS-L decode read does not depend on the context)",
                     "peak_kind": peak_kind, "bytes_per_launch": kbytes,
                     "avg_launch_us": k_avg_ms * 1e3, "median_launch_us": k_med_ms * 1e3,
                     "how": "launched alone with an L2 flush before every launch, CUDA events on the launching stream"},
        "step_roofline": {"step_bytes": step_bytes, "achieved_gbs": step_bytes / (ms / K * 1e-3) / 1e9,
                          "frac": step_bytes / (ms / K * 1e-3) / 1e9 / peak, "peak_kind": peak_kind},
        "prefill": {"ktok_s": B * ctx / prefill_ms, "ms": prefill_ms, "runs_ms": prefill_all, "note": "median of 3 after one untimed full-context prefill (the reference's --warm 1 --nmed 3), incl. KV store fill and last-token logits; outside the headline's timed region"},
        "kv_bytes_per_layer": gd.kv_bytes() // nL, "kv_faults": list(faults),
        "peak_mem_gib": torch.cuda.max_memory_allocated() / 2 ** 30,
    }
    if world == 1 and args.model == "340m":
        line["window_roofline"] = time_window_kernel(gd.attn_core[0], dev, ctx)
    if world == 1 and not args.no_fsb:
        del gd, model
        torch.cuda.empty_cache()
        line["fsb"] = run_fsb_section(args, dev, K, Wm)
    if world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline_sample()
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ctx", type=int, default=131072)
    ap.add_argument("--cpu-ctx", type=int, default=4096)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--model", default="340m")
    ap.add_argument("--kv", default="bounded", choices=["bounded", "int8", "bf16"])
    ap.add_argument("--shard", default="batch", choices=["batch", "heads"],
                    help="N > 1: 'batch' = one sequence per rank, no collective (weak scaling); 'heads' = one sequence, heads "
                         "split over the ranks with an all-gather per layer (strong scaling)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-fsb", action="store_true", help="skip the FS-B section (BASELINE config 3) of the N=1 line")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
