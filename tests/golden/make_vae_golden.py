"""Generate tests/golden/gvae.npz by running the REFERENCE's VAE drafter (TreeVAEFlowDrafter,
src/chain_flow/drafters/tree_vae_flow.py:91-175, with its TransformerHiddenVAE,
src/chain_flow/vae/transformer_hidden.py:9-67) on seeded weights and inputs: the shipped
production layout (the flow in the VAE's latent space, the path head and markov head in the
target's hidden space) at small widths.

Run in a container that has the reference checkout (it is not needed anywhere else):

    python tests/golden/make_vae_golden.py --ref /path/to/chain-flow/src

It drives the reference's own ``vae.encode_sequence`` (mu), ``integrate`` in latent space,
``vae.decode_sequence``, ``predict_hidden`` and ``FlowDrafterProposer._beam_chains`` /
``_beam_tree`` (object from ``__new__``). z0 is injected (init_latents draws noise without a
generator); LayerNorm gammas and betas, the PathHead output layer and markov w2 are re-seeded
so that every term is exercised.
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
C = dict(H=128, latent=64, inter=128, vae_layers=2, vae_heads=4, heads=4, FM=2, L=2, T=2, V=1000, R=256,
         rank=32, B=2, DL=8, chunk=4, order=8, seed=31)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("CF_REFERENCE_SRC"), required="CF_REFERENCE_SRC" not in os.environ,
                    help="the reference checkout's src/ directory (or set CF_REFERENCE_SRC)")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    from chain_flow.drafters.tree_vae_flow import TreeVAEFlowConfig, TreeVAEFlowDrafter
    from chain_flow.vllm_plugin.flow_proposer import FlowDrafterProposer
    c = C
    H, V, R, B = c["H"], c["V"], c["R"], c["B"]
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

    cfg = TreeVAEFlowConfig(context_size=8, draft_length=c["DL"], chunk_size=c["chunk"], expert_dim=c["latent"],
                            num_heads=c["heads"], ffn_multiplier=c["FM"], num_drafter_layers=c["L"],
                            num_flow_steps=c["T"], init_mode="noise", path_order=c["order"], path_ffn_multiplier=2,
                            markov_rank=c["rank"], latent_size=c["latent"], vae_intermediate_size=c["inter"],
                            vae_num_layers=c["vae_layers"], vae_num_heads=c["vae_heads"], vae_max_sequence_length=16)
    d = TreeVAEFlowDrafter(Stub(), cfg).eval()
    sd = {}
    for k, v in d.state_dict().items():
        if k.endswith("norm.weight") or k.endswith("ffn.0.weight") or k.endswith("norm1.weight") \
                or k.endswith("norm2.weight"):
            t = 1.0 + 0.1 * torch.randn(v.shape, generator=g)        # LN gamma
        elif k.endswith("norm.bias") or k.endswith("ffn.0.bias") or k.endswith("norm1.bias") \
                or k.endswith("norm2.bias"):
            t = 0.1 * torch.randn(v.shape, generator=g)              # LN beta
        elif k.endswith("time_mlp.0.weight") or k.endswith("time_mlp.0.bias"):
            t = torch.randn(v.shape, generator=g)
        elif k == "markov.w1.weight":
            t = torch.randn(v.shape, generator=g) * 0.5
        elif k.endswith("_pos.weight"):
            t = torch.randn(v.shape, generator=g) * 0.1
        elif k.endswith("bias"):
            t = 0.02 * torch.randn(v.shape, generator=g)
        else:
            t = torch.randn(v.shape, generator=g) / v.shape[-1] ** 0.5
        sd[k] = f16(t)
    d.load_state_dict(sd)
    sl = torch.randperm(V, generator=g)[:R].sort().values
    ctx = torch.randn(B, 8, H, generator=g).to(torch.float16).float()
    z0 = torch.randn(B, c["DL"], c["latent"], generator=g).to(torch.float16).float()
    known0 = torch.randint(0, V, (B,), generator=g)
    with torch.inference_mode():
        mu = d._encode(ctx)
        zf = d.integrate(mu, z0)
        dec = d._decode(zf)
        d.init_latents = lambda context: z0.clone()
        pred = d.predict_hidden(ctx)
        p = FlowDrafterProposer.__new__(FlowDrafterProposer)
        p.__dict__.update(drafter=d, width=4, K=5, dtype=torch.float32, dev=torch.device("cpu"),
                          order=c["order"], twopass_m=0, twopass_shared=False, twopass_seed=False,
                          feedback=False, prof=False, _hw=lm_w[sl].contiguous(),
                          _w2=d.markov.w2.weight[sl].contiguous(), _sl=sl, path_trim=True,
                          tree_keep=4, tree_topb=4, tree_depth=5)
        chains = FlowDrafterProposer._beam_chains(p, ctx, known0)
        tree = FlowDrafterProposer._beam_tree(p, ctx, known0)
    out = {f"w.{k}": v.numpy().astype(np.float16) for k, v in d.state_dict().items()}
    out.update({
        "cfg": np.array([H, c["latent"], c["inter"], c["vae_layers"], c["vae_heads"], c["heads"], c["FM"], c["L"],
                         c["T"], V, R, c["rank"], B, c["DL"], c["chunk"], c["order"]], np.int64),
        "emb": emb_w.numpy().astype(np.float16), "lm_w": lm_w.numpy().astype(np.float16),
        "sl": sl.numpy().astype(np.int64), "ctx": ctx.numpy().astype(np.float16),
        "z0": z0.numpy().astype(np.float16), "known0": known0.numpy().astype(np.int64),
        "mu": mu.numpy().astype(np.float32), "zflow": zf.numpy().astype(np.float32),
        "dec": dec.numpy().astype(np.float32), "pred": pred.numpy().astype(np.float32),
        "chains": chains.numpy().astype(np.int64), "tree": tree.numpy().astype(np.int64),
    })
    path = HERE / "gvae.npz"
    np.savez_compressed(path, **out)
    print(f"gvae: chains={chains.tolist()} -> {path} ({path.stat().st_size / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()
