"""The production drafter's VAE bridge (reference TransformerHiddenVAE + TreeVAEFlowDrafter):
the oracle against the reference's own outputs (tests/golden/make_vae_golden.py), and the GPU
path (VAE plans around the engine's latent flow and hidden-space beam) against them."""
import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN

HIDDEN_RTOL = 2e-2


def load_gvae():
    z = np.load(GOLDEN / "gvae.npz")
    out, W = {}, {}
    for k in z.files:
        a = z[k]
        t = torch.from_numpy(a.astype(np.float32) if a.dtype == np.float16 else a)
        (W if k.startswith("w.") else out)[k[2:] if k.startswith("w.") else k] = t
    (H, lat, inter, vl, vh, heads, FM, L, T, V, R, rank, B, DL, chunk, order) = (int(x) for x in out["cfg"])
    out.update(W=W, H=H, latent=lat, inter=inter, vae_layers=vl, vae_heads=vh, heads=heads, FM=FM, L=L, T=T, V=V,
               R=R, rank=rank, B=B, DL=DL, chunk=chunk, order=order)
    return out


def flow_cfg(g):
    return oracle.FlowConfig(hidden=g["latent"], draft_length=g["DL"], chunk_size=g["chunk"], num_heads=g["heads"],
                             ffn_multiplier=g["FM"], num_layers=g["L"], num_flow_steps=g["T"], path_order=g["order"],
                             markov_rank=g["rank"])


def _rel(a, b):
    return float((a.float().cpu() - b.float().cpu()).abs().max() / b.float().abs().max().clamp_min(1e-12))


def test_vae_oracle_matches_reference():
    g = load_gvae()
    W = g["W"]
    mu = oracle.vae_encode(W, g["ctx"], g["vae_layers"], g["vae_heads"])
    assert _rel(mu, g["mu"]) < 1e-4
    zf = oracle.integrate(W, flow_cfg(g), g["mu"], g["z0"])
    assert _rel(zf, g["zflow"]) < 1e-4
    dec = oracle.vae_decode(W, g["zflow"], g["vae_layers"], g["vae_heads"])
    assert _rel(dec, g["dec"]) < 1e-4
    pred = oracle.predict_hidden_vae(W, flow_cfg(g), g["vae_layers"], g["vae_heads"], g["ctx"], g["z0"])
    assert _rel(pred, g["pred"]) < 1e-4
    sl = g["sl"]
    ch = oracle.beam_chains(W, flow_cfg(g), g["emb"], g["lm_w"][sl], W["markov.w2.weight"][sl], sl, g["pred"],
                            g["known0"], 4, 5)
    assert torch.equal(ch, g["chains"])
    tr = oracle.beam_tree(W, flow_cfg(g), g["emb"], g["lm_w"][sl], W["markov.w2.weight"][sl], sl, g["pred"],
                          g["known0"], 4, 4, 5)
    assert torch.equal(tr, g["tree"])
