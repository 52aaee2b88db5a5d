"""Timed CPU baseline (test/measurement infrastructure, never on the product path): the reference's own eager FS-L decode
on the host cores, run from oracle/_ref (see oracle/make_ref.py), with the CPU port (oracle/model.py) as the fallback when
that copy is absent.

Protocol = the reference's eager decode benchmark (experiments/scaling/bench_efficiency.py:233-298, the `else` branch):
FreeSoloLM("340m", vocab 32000, serve_kwargs("sparse")), seed-0 random init, uniform random prompt, KV caches with the
decode tokens reserved, an untimed prefill, `warm` untimed greedy steps, then `steps` timed greedy steps of
`_trunk_cached` + `_lm_head_fp32`. fp32 on CPU (the reference's CPU path has no bf16 autocast), all host threads.
"""
from __future__ import annotations

import os
import time

import torch


def time_fsl_decode(ctx: int, steps: int, warm: int, model: str = "340m") -> dict:
    """Returns {"value": tok/s, "unit", "cores", "kind": "reference" | "port", "sample", "ms_per_step", "prefill_s"}."""
    from .make_ref import import_reference
    nt_before = torch.get_num_threads()
    torch.set_num_threads(os.cpu_count() or 1)
    try:
        if import_reference():
            return _time_reference(ctx, steps, warm, model)
        return _time_port(ctx, steps, warm)
    finally:
        torch.set_num_threads(nt_before)


def _time_reference(ctx, steps, warm, model):
    from bench_efficiency import serve_kwargs                # the reference's own preset
    from kv_cache import _trunk_cached, make_caches
    from longctx_infer import _lm_head_fp32, extend_rope_cache
    from model import MODEL_CONFIGS, FreeSoloLM
    cfg = dict(MODEL_CONFIGS[model])
    cfg["vocab_size"] = 32000
    cfg["max_seq_len"] = ctx + 512
    torch.manual_seed(0)
    m = FreeSoloLM(**cfg, **serve_kwargs("sparse")).eval()
    extend_rope_cache(m, ctx + 512)
    ids = torch.randint(0, 32000, (1, ctx), generator=torch.Generator().manual_seed(4321 + ctx))
    caches = make_caches(m, reserve=steps + warm + 16)

    def step(tok):
        h = _trunk_cached(m, tok, caches)
        return _lm_head_fp32(m, h[:, -1:, :], 4096)[:, 0, :].argmax(-1).unsqueeze(1)

    with torch.no_grad():
        t0 = time.perf_counter()
        nxt = step(ids)
        prefill_s = time.perf_counter() - t0
        for _ in range(warm):
            nxt = step(nxt)
        t0 = time.perf_counter()
        for _ in range(steps):
            nxt = step(nxt)
        dt = time.perf_counter() - t0
    return {"value": steps / dt, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "reference",
            "ms_per_step": dt / steps * 1e3, "prefill_s": prefill_s,
            "sample": f"{steps} greedy decode steps of the reference's own FreeSoloLM ({model}, FS-L, fp32, eager CPU path, "
                      f"batch 1) after its own {ctx}-token prefill; FS-L's decode step reads the window, the 72-cell pool "
                      f"and 4 cells, so its cost does not grow with the context"}


def _time_port(ctx, steps, warm):
    from .model import CpuFSLModel
    m = CpuFSLModel(max_len=ctx + steps + warm + 64)
    m.synthetic_context(1, ctx)
    tok = torch.zeros(1, 1, dtype=torch.long)
    for _ in range(warm):
        tok = m.step(tok)
    t0 = time.perf_counter()
    for _ in range(steps):
        tok = m.step(tok)
    dt = time.perf_counter() - t0
    return {"value": steps / dt, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "ms_per_step": dt / steps * 1e3, "prefill_s": None,
            "sample": f"{steps} decode steps of the CPU port (oracle/model.py, 341M FS-L, fp32, batch 1) at a synthetic "
                      f"{ctx}-token context; oracle/_ref (the reference's own sources) was not present"}
