"""Generate the golden fixtures under tests/golden/ by running the REFERENCE implementation.

Run in a container that has the reference checkout (it is not needed anywhere else):

    python tests/golden/make_golden.py --ref /path/to/chain-flow/src

For each fixture config it builds the reference ``TreeFlowDrafter`` (chain_flow/drafters/
tree_flow.py) with seeded random weights (rounded to fp16-representable values so the fp16
CUDA path sees the very same numbers), a stub target LM (embedding + lm_head tensors, the
way flow_proposer.py:596-614 wraps the real ones), and drives the reference's own:

* ``TreeFlowDrafter.integrate(ctx, z0)``                       -> ``pred``
* ``FlowDrafterProposer._beam_chains`` (object from ``__new__``) -> ``chains``
* ``FlowDrafterProposer._beam_tree``                            -> ``tree``
* ``TreeFlowDrafter._residual_from_lastp`` on a probe lastp      -> ``probe_res``
* ``kernels/tree_scan.tree_gated_delta_scan``                   -> ``gdn_o``, ``gdn_states``

``init_latents`` draws noise without a generator (tree_flow.py:154-155), so z0 is made here
and injected. The zero-initialised PathHead output layer and markov ``w2``
(tree_flow.py:95-96, markov_flow.py:69) are re-seeded non-zero so they are exercised.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent

CONFIGS = {
    # name: (H, heads, FM, L, T, V, R, markov_rank, B, path_ffn)
    "g64": dict(H=64, heads=8, FM=2, L=2, T=4, V=1000, R=256, rank=16, B=2, seed=11),
    "g128": dict(H=128, heads=8, FM=6, L=1, T=2, V=2000, R=512, rank=32, B=1, seed=12),
}


def make_tree_parents(n_nodes: int, max_depth: int, max_branch: int, seed: int):
    """BFS-ordered random tree: parent[i] < i, depth <= max_depth, children per node <= max_branch.
    Node 0..r-1 are roots (parent -1). Mirrors chain_flow_b200.gdn.make_tree (kept standalone so
    this script needs only the reference)."""
    g = torch.Generator().manual_seed(seed)
    parent, depth, nchild = [], [], []
    while len(parent) < n_nodes:
        i = len(parent)
        if i == 0:
            parent.append(-1); depth.append(0); nchild.append(0)
            continue
        cands = [j for j in range(i) if depth[j] < max_depth - 1 and nchild[j] < max_branch]
        # prefer the shallowest frontier so the tree is BFS-ordered (parents of later nodes are
        # never shallower than parents of earlier ones)
        dmin = min(depth[j] for j in cands)
        cands = [j for j in cands if depth[j] == dmin]
        p = cands[int(torch.randint(len(cands), (1,), generator=g))]
        parent.append(p); depth.append(depth[p] + 1); nchild[p] += 1; nchild.append(0)
    return torch.tensor(parent), torch.tensor(depth)


def build_reference(ref_src: str, c: dict):
    sys.path.insert(0, ref_src)
    from chain_flow.drafters.tree_flow import TreeFlowDrafter, TreeFlowConfig

    H, V = c["H"], c["V"]
    g = torch.Generator().manual_seed(c["seed"])
    f16 = lambda t: t.to(torch.float16).to(torch.float32)
    emb_w = f16(torch.randn(V, H, generator=g) * 0.5)
    lm_w = f16(torch.randn(V, H, generator=g) * 0.02 * 8)

    class SM:
        def __init__(s):
            s.config = SimpleNamespace(hidden_size=H, vocab_size=V)
        def get_input_embeddings(s):
            return lambda i: F.embedding(i, emb_w)

    class Stub:
        def __init__(s): s.model = SM()

    cfg = TreeFlowConfig(context_size=8, draft_length=6, chunk_size=3, expert_dim=H,
                         num_heads=c["heads"], ffn_multiplier=c["FM"], num_drafter_layers=c["L"],
                         num_flow_steps=c["T"], init_mode="noise", path_order=4,
                         path_ffn_multiplier=2, markov_rank=c["rank"])
    d = TreeFlowDrafter(Stub(), cfg).eval()
    sd = {}
    for k, v in d.state_dict().items():
        if k.endswith("norm.weight") or k.endswith("ffn.0.weight"):
            t = 1.0 + 0.1 * torch.randn(v.shape, generator=g)        # LN gamma
        elif k.endswith("norm.bias") or k.endswith("ffn.0.bias"):
            t = 0.1 * torch.randn(v.shape, generator=g)              # LN beta
        elif k.endswith("time_mlp.0.weight") or k.endswith("time_mlp.0.bias"):
            t = torch.randn(v.shape, generator=g)
        elif k == "markov.w1.weight":
            t = torch.randn(v.shape, generator=g) * 0.5
        elif k.endswith("bias"):
            t = 0.02 * torch.randn(v.shape, generator=g)
        else:
            fan_in = v.shape[-1]
            t = torch.randn(v.shape, generator=g) / fan_in ** 0.5
        sd[k] = f16(t)
    d.load_state_dict(sd)
    return d, cfg, emb_w, lm_w, g


def run_config(ref_src: str, name: str, c: dict) -> dict:
    if ref_src not in sys.path:
        sys.path.insert(0, ref_src)
    from chain_flow.vllm_plugin.flow_proposer import FlowDrafterProposer
    from chain_flow.kernels.tree_scan import tree_gated_delta_scan

    d, cfg, emb_w, lm_w, g = build_reference(ref_src, c)
    H, V, R, B = c["H"], c["V"], c["R"], c["B"]
    sl = torch.randperm(V, generator=g)[:R].sort().values
    ctx = torch.randn(B, 8, H, generator=g).to(torch.float16).float()
    z0 = torch.randn(B, 6, H, generator=g).to(torch.float16).float()
    known0 = torch.randint(0, V, (B,), generator=g)

    with torch.inference_mode():
        pred = d.integrate(ctx, z0)
        d.init_latents = lambda context: z0.clone()
        p = FlowDrafterProposer.__new__(FlowDrafterProposer)
        p.__dict__.update(drafter=d, width=4, K=5, dtype=torch.float32, dev=torch.device("cpu"),
                          order=4, twopass_m=0, twopass_shared=False, twopass_seed=False,
                          feedback=False, prof=False, _hw=lm_w[sl].contiguous(),
                          _w2=d.markov.w2.weight[sl].contiguous(), _sl=sl, path_trim=True,
                          tree_keep=4, tree_topb=4, tree_depth=5)
        chains = FlowDrafterProposer._beam_chains(p, ctx, known0)
        tree = FlowDrafterProposer._beam_tree(p, ctx, known0)
        probe_lastp = torch.tensor([[int(known0[0]), -1, -1, -1],
                                    [3, 7, -1, -1],
                                    [5, 9, 11, 13],
                                    [1, 2, 3, 4]], dtype=torch.long)
        probe_res = d._residual_from_lastp(probe_lastp, None)
        probe_res2 = d._residual_from_lastp(probe_lastp, 2)

    # tree GDN (BASELINE config 4 semantics at small head dims)
    N, Hh, Dk, Dv = 16, 2, 32, 32
    parent, depth = make_tree_parents(N, 5, 4, c["seed"])
    q = torch.randn(N, Hh, Dk, generator=g).to(torch.float16).float()
    k = torch.randn(N, Hh, Dk, generator=g).to(torch.float16).float()
    v = torch.randn(N, Hh, Dv, generator=g).to(torch.float16).float()
    alpha = torch.sigmoid(torch.randn(N, Hh, generator=g))
    beta = torch.sigmoid(torch.randn(N, Hh, generator=g))
    gg = alpha.log()
    init = torch.randn(Hh, Dk, Dv, generator=g) * 0.1
    gdn_o, gdn_states = tree_gated_delta_scan(q, k, v, gg, beta, parent, depth, init)

    out = {f"w.{k}": v.numpy().astype(np.float16) for k, v in d.state_dict().items()}
    out.update({
        "cfg": np.array([H, c["heads"], c["FM"], c["L"], c["T"], V, R, c["rank"], B], np.int64),
        "emb": emb_w.numpy().astype(np.float16), "lm_w": lm_w.numpy().astype(np.float16),
        "sl": sl.numpy().astype(np.int64), "ctx": ctx.numpy().astype(np.float16),
        "z0": z0.numpy().astype(np.float16), "known0": known0.numpy().astype(np.int64),
        "pred": pred.numpy().astype(np.float32), "chains": chains.numpy().astype(np.int64),
        "tree": tree.numpy().astype(np.int64),
        "probe_lastp": probe_lastp.numpy(), "probe_res": probe_res.numpy(),
        "probe_res2": probe_res2.numpy(),
        "gdn_q": q.numpy().astype(np.float16), "gdn_k": k.numpy().astype(np.float16),
        "gdn_v": v.numpy().astype(np.float16), "gdn_g": gg.numpy(), "gdn_beta": beta.numpy(),
        "gdn_parent": parent.numpy(), "gdn_depth": depth.numpy(), "gdn_init": init.numpy(),
        "gdn_o": gdn_o.numpy(), "gdn_states": gdn_states.numpy(),
    })
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("CF_REFERENCE_SRC"), required="CF_REFERENCE_SRC" not in os.environ,
                    help="the reference checkout's src/ directory (or set CF_REFERENCE_SRC)")
    args = ap.parse_args()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name, c in CONFIGS.items():
        out = run_config(args.ref, name, c)
        path = HERE / f"{name}.npz"
        np.savez_compressed(path, **out)
        print(f"{name}: chains={out['chains'].tolist()} -> {path} "
              f"({path.stat().st_size / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()
