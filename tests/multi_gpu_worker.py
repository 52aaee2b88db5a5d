"""Worker of tests/test_gpu_multi.py (launched by torch.distributed.run, one process per GPU): a head-sharded model must
decode like the unsharded one. Each rank runs both on its own GPU and compares."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    serve = sys.argv[1] if len(sys.argv) > 1 else "sparse"
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    from freesolo_b200.parallel import shard_model_heads
    from freesolo_b200.serving import FreeSoloLM, GraphedDecoder, calibrate_fsb_tau, serve_kwargs
    P0, T = 700, 200
    ids = torch.randint(0, 32000, (1, P0), generator=torch.Generator().manual_seed(3))

    def build():
        torch.manual_seed(0)
        m = FreeSoloLM.from_config("debug", max_seq_len=2048, **serve_kwargs(serve, 0.9 if serve == "fsb" else 0.0))
        m = m.to(dev).to(torch.bfloat16).eval()
        if serve == "fsb":
            warm = torch.randint(0, 32000, (1, 1024), generator=torch.Generator().manual_seed(5))
            calibrate_fsb_tau(m, warm, 0.5, "fsb_tau")
            calibrate_fsb_tau(m, warm, 0.9, "fsb_tau_union")
        return m

    def run(m):
        gd = GraphedDecoder(m, ids, Lmax=P0 + T + 8, device=dev, kv="int8", eager_steps=2)
        toks = [gd.prefill().clone()]
        logits0 = None
        for i in range(T - 1):
            toks.append(gd.step().clone())
            if i == 0:
                logits0 = gd.logits.float().clone()
        assert gd.graph is not None and gd.kv_faults() == (0, 0, 0)
        assert gd.peer_status() == 0, "a wait for a peer's head outputs ran out"
        run.used_peer = gd.peer is not None
        return torch.cat(toks, dim=1), logits0

    full_toks, full_logits = run(build())
    m2 = shard_model_heads(build(), rank, world)
    sh_toks, sh_logits = run(m2)
    assert run.used_peer, "the head shards' exchange did not run over peer memory"
    # the same step with the library all-gather instead of the peer-memory kernel: identical bits
    os.environ["FSATTN_PEER_GATHER"] = "0"
    nccl_toks, nccl_logits = run(m2)
    del os.environ["FSATTN_PEER_GATHER"]
    assert not run.used_peer
    assert torch.equal(nccl_toks, sh_toks) and torch.equal(nccl_logits, sh_logits), "peer exchange and all-gather disagree"
    d = (sh_logits - full_logits).abs().max().item()
    agree = (sh_toks == full_toks).float().mean().item()
    # every rank must hold the same tokens (the residual stream is replicated)
    all_toks = [torch.empty_like(sh_toks) for _ in range(world)]
    dist.all_gather(all_toks, sh_toks)
    same = all(torch.equal(all_toks[0], t) for t in all_toks)
    print(f"[rank {rank}] {serve}: first-step logits max-abs diff {d:.4f}, token agreement {agree:.3f}, ranks agree {same}", flush=True)
    assert same, "ranks diverged"
    assert torch.equal(sh_toks[:, 0], full_toks[:, 0]) and d < 0.1, (d, sh_toks[:, :4], full_toks[:, :4])
    assert agree > 0.5, agree
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
