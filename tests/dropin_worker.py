"""Child process of tests/test_gpu_dropin.py: builds the REFERENCE's own FreeSoloLM (its experiments/scaling/model.py from
oracle/_ref) with this package answering to ``src.fsattn`` / ``src.utils.trunk_triton`` through the import-path alias, runs a
prefill and greedy decode steps through the reference's blocks with this package's FSKVCache, and prints a JSON line with the
logits' distance from this package's own model holding the same weights."""
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main(variant: str):
    import freesolo_b200.compat as compat
    compat.install()
    ref_scaling = os.path.join(ROOT, "oracle", "_ref", "experiments", "scaling")
    if not os.path.isfile(os.path.join(ref_scaling, "model.py")):
        print(json.dumps({"skip": "no copy of the reference sources (oracle/_ref)"}))
        return
    sys.path.insert(0, ref_scaling)
    os.environ.update(FS_STRICT_CAUSAL="1", FS_PRUNE_KERNEL="1" if variant == "fsl" else "0")
    from model import FreeSoloLM as RefLM                     # the reference's model class, unmodified
    from freesolo_b200.fsattn import FSAttn, make_caches
    from freesolo_b200.serving import FreeSoloLM, extend_rope_cache, lm_head, serve_kwargs, trunk_cached
    kw = serve_kwargs("sparse") if variant == "fsl" else serve_kwargs("fsb", 0.9)
    cfg = dict(vocab_size=1024, d_model=256, n_layers=4, n_heads=4, d_ff=688, max_seq_len=1024)
    dev = torch.device("cuda:0")
    torch.manual_seed(0)
    ref = RefLM(**cfg, **kw).eval()
    assert all(type(b.attn.fsattn) is FSAttn for b in ref.blocks), "the reference model did not pick up this package's FSAttn"
    torch.manual_seed(0)
    ours = FreeSoloLM(**cfg, **kw).eval()
    missing, unexpected = ours.load_state_dict(ref.state_dict(), strict=False)
    assert not unexpected and all("rope" in k or "fsb_tau_union" in k for k in missing), (missing, unexpected)
    ref, ours = ref.to(dev).to(torch.bfloat16), ours.to(dev).to(torch.bfloat16)
    if variant == "fsb":
        g = torch.Generator().manual_seed(5)
        with torch.no_grad():
            for mr, mo in zip(ref.blocks, ours.blocks):
                t1, t2 = torch.rand(4, generator=g) * 0.3 + 0.2, torch.rand(4, generator=g) * 0.3 + 0.6
                for m in (mr, mo):
                    m.attn.fsattn.fsb_tau.copy_(t1)
                    m.attn.fsattn.fsb_tau_union.copy_(t2)
    P0, T = 330, 40
    ids = torch.randint(0, 1024, (2, P0), generator=torch.Generator().manual_seed(9)).to(dev)
    outs = []
    for m in (ref, ours):
        extend_rope_cache(m, P0 + T + 8)
        caches = make_caches(m, reserve=T + 8)
        logits, step_in = [], ids
        with torch.no_grad():
            for t in range(T):
                h = trunk_cached(m, step_in, caches, last_n=1)
                lg = lm_head(m, h[:, -1]).float()
                logits.append(lg)
                # both runs follow the reference model's greedy tokens so that every step stays comparable
                step_in = (lg if m is ref else outs[0][t]).argmax(-1).view(-1, 1)
        outs.append(torch.stack(logits))
    d = (outs[0] - outs[1]).abs()
    print(json.dumps({"variant": variant, "max_abs": d.max().item(), "mean_rel": (d.sum() / outs[0].abs().sum()).item(),
                      "greedy_agree": (outs[0].argmax(-1) == outs[1].argmax(-1)).float().mean().item(),
                      "ref_class": f"{RefLM.__module__}.{RefLM.__name__}", "steps": T}))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "fsl")
