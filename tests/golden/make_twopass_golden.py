"""Generate tests/golden/gtp.npz: the reference's two-pass candidate head (CF_TWOPASS_M with
CF_TWOPASS_SHARED=1, CF_TWOPASS_SEED=0; reference src/chain_flow/vllm_plugin/flow_proposer.py:
1142-1184, used by _beam_chains :1227-1247 and _beam_tree :1297-1315) on the drafters of
tests/golden/{g64,g128}.npz (the same seeded weights, built by make_golden.build_reference).

Run in a container that has the reference checkout (it is not needed anywhere else):

    python tests/golden/make_twopass_golden.py --ref /path/to/chain-flow/src

For each configuration and M it stores the pass-A candidate set (`FlowDrafterProposer._candidates`,
shortlist-local ids in torch.topk order) and the chain and tree drafts, each from the reference's
own methods on an object built with __new__.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from make_golden import CONFIGS, build_reference  # noqa: E402

TWOPASS_M = {"g64": (64, 128), "g128": (64, 256)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("CF_REFERENCE_SRC"), required="CF_REFERENCE_SRC" not in os.environ,
                    help="the reference checkout's src/ directory (or set CF_REFERENCE_SRC)")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    from chain_flow.vllm_plugin.flow_proposer import FlowDrafterProposer
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    out = {}
    for name, c in CONFIGS.items():
        d, cfg, emb_w, lm_w, g = build_reference(args.ref, c)
        V, R, B = c["V"], c["R"], c["B"]
        # the same draws, in the same order, as make_golden.run_config
        sl = torch.randperm(V, generator=g)[:R].sort().values
        ctx = torch.randn(B, 8, c["H"], generator=g).to(torch.float16).float()
        z0 = torch.randn(B, 6, c["H"], generator=g).to(torch.float16).float()
        known0 = torch.randint(0, V, (B,), generator=g)
        with torch.inference_mode():
            pred = d.integrate(ctx, z0)
            d.init_latents = lambda context: z0.clone()
            for M in TWOPASS_M[name]:
                p = FlowDrafterProposer.__new__(FlowDrafterProposer)
                p.__dict__.update(drafter=d, width=4, K=5, dtype=torch.float32, dev=torch.device("cpu"),
                                  order=4, twopass_m=M, twopass_shared=True, twopass_seed=False,
                                  feedback=False, prof=False, _hw=lm_w[sl].contiguous(),
                                  _w2=d.markov.w2.weight[sl].contiguous(), _sl=sl, path_trim=True,
                                  tree_keep=4, tree_topb=4, tree_depth=5)
                cand = FlowDrafterProposer._candidates(p, pred, 1, 6)
                chains = FlowDrafterProposer._beam_chains(p, ctx, known0)
                tree = FlowDrafterProposer._beam_tree(p, ctx, known0)
                out[f"{name}.m{M}.cand"] = cand[:, 0].numpy().astype(np.int64)
                out[f"{name}.m{M}.chains"] = chains.numpy().astype(np.int64)
                out[f"{name}.m{M}.tree"] = tree.numpy().astype(np.int64)
                print(f"{name} M={M}: chains={chains.tolist()}")
        out[f"{name}.pred"] = pred.numpy().astype(np.float32)
    path = HERE / "gtp.npz"
    np.savez_compressed(path, **out)
    print(f"-> {path} ({path.stat().st_size / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()
