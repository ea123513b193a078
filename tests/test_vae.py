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


# ---------------------------------------------------------------------------------------- GPU
def _vae_cfg(g):
    from chain_flow_b200.vae import VaeConfig
    return VaeConfig(hidden=g["H"], latent=g["latent"], intermediate=g["inter"], layers=g["vae_layers"],
                     heads=g["vae_heads"], max_len=16)


def _draft_cfg(g, hidden):
    from chain_flow_b200.weights import DraftConfig
    return DraftConfig(hidden=hidden, context_size=8, draft_length=g["DL"], chunk_size=g["chunk"],
                       num_heads=g["heads"], ffn_multiplier=g["FM"], num_drafter_layers=g["L"],
                       num_flow_steps=g["T"], path_order=g["order"], markov_rank=g["rank"])


@pytest.fixture(scope="module")
def gvae_weights():
    from chain_flow_b200.vae import VaeWeights
    from chain_flow_b200.weights import DrafterWeights, WideWeights
    g = load_gvae()
    W = g["W"]
    vw = VaeWeights(W, _vae_cfg(g), device="cuda", layout="wide")
    ve = VaeWeights(W, _vae_cfg(g), device="cuda", layout="engine")
    fl = DrafterWeights(W, _draft_cfg(g, g["latent"]), None, None, None, device="cuda", parts="flow")
    hd = DrafterWeights(W, _draft_cfg(g, g["H"]), g["emb"], g["lm_w"], g["sl"], device="cuda", parts="head")
    wfl = WideWeights(W, _draft_cfg(g, g["latent"]), None, None, None, device="cuda", parts="flow")
    whd = WideWeights(W, _draft_cfg(g, g["H"]), g["emb"], g["lm_w"], g["sl"], device="cuda", parts="head")
    return g, vw, fl, hd, wfl, whd, ve


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["wide", "engine"])
def test_gpu_vae_encode_decode_match_reference(gvae_weights, layout):
    from chain_flow_b200.vae import VaeEnginePlan, VaePlan
    g, vw, fl, hd, wfl, whd, ve = gvae_weights
    side = VaePlan if layout == "wide" else VaeEnginePlan
    vw = vw if layout == "wide" else ve
    B = g["B"]
    ctx = g["ctx"].half().cuda().contiguous()
    mu = torch.zeros(B, 8, g["latent"], dtype=torch.float16, device="cuda")
    enc = side(vw, False, B, 8, ctx, mu)
    enc.run()
    zf = g["zflow"].float().cuda().contiguous()
    dec = torch.zeros(B, g["DL"], g["H"], dtype=torch.float32, device="cuda")
    dp = side(vw, True, B, g["DL"], zf, dec)
    dp.run()
    torch.cuda.synchronize()
    assert enc.device_error() == 0 and dp.device_error() == 0
    assert _rel(mu, g["mu"]) < HIDDEN_RTOL, _rel(mu, g["mu"])
    assert _rel(dec, g["dec"]) < HIDDEN_RTOL, _rel(dec, g["dec"])


@pytest.mark.gpu
@pytest.mark.parametrize("wide", [False, True])
def test_gpu_vae_draft_matches_reference(gvae_weights, wide):
    """encode -> latent flow -> decode -> beam on the reference's own weights and z0: hidden
    states within tolerance, chain ids equal to the reference's, tree equal or tie-explained."""
    from chain_flow_b200 import _lib
    from chain_flow_b200.vae import VaeDraft
    g, vw, fl, hd, wfl, whd, ve = gvae_weights
    f, h = (wfl, whd) if wide else (fl, hd)
    vw = vw if wide else ve
    sl = g["sl"]
    W = g["W"]
    for mode in (_lib.MODE_CHAIN, _lib.MODE_TREE):
        d = VaeDraft(vw, f, h, mode, g["B"], wide=wide, width=4, depth=5, tree_keep=4, tree_topb=4)
        d.ctx.copy_(g["ctx"].half())
        d.z0.copy_(g["z0"].half())
        d.known0.copy_(g["known0"])
        d.run()
        torch.cuda.synchronize()
        d.check()
        assert _rel(d.mu, g["mu"]) < HIDDEN_RTOL
        assert _rel(d.latent, g["zflow"]) < HIDDEN_RTOL, _rel(d.latent, g["zflow"])
        assert _rel(d.pred, g["pred"]) < HIDDEN_RTOL, _rel(d.pred, g["pred"])
        toks = d.tokens.cpu()
        if mode == _lib.MODE_CHAIN:
            assert torch.equal(toks, g["chains"]), (toks, g["chains"])
            # the beam is exact on the engine's own hidden states too
            want = oracle.beam_chains(W, flow_cfg(g), g["emb"], g["lm_w"][sl], W["markov.w2.weight"][sl], sl,
                                      d.pred.cpu(), g["known0"], 4, 5)
            assert torch.equal(toks, want)
        elif not torch.equal(toks, g["tree"]):
            from beam_check import check_tree
            check_tree(toks, W, flow_cfg(g), g["emb"], g["lm_w"][sl], W["markov.w2.weight"][sl], sl, d.pred.cpu(),
                       g["known0"], 4, 4, 5)


def _model_args(g, init_mode):
    return dict(context_size=8, draft_length=g["DL"], chunk_size=g["chunk"], expert_dim=g["latent"],
                num_heads=g["heads"], ffn_multiplier=g["FM"], num_drafter_layers=g["L"], num_flow_steps=g["T"],
                path_order=g["order"], path_ffn_multiplier=2, markov_rank=g["rank"], init_mode=init_mode,
                latent_size=g["latent"], vae_intermediate_size=g["inter"], vae_num_layers=g["vae_layers"],
                vae_num_heads=g["vae_heads"], vae_max_sequence_length=16)


def _delta_z0(ctx, k):
    """reference TreeFlowDrafter.init_latents, init_mode='delta' (on the encoded context)"""
    last = ctx[:, -1:, :]
    delta = ctx[:, -1:, :] - ctx[:, -2:-1, :]
    steps = torch.arange(1, k + 1, dtype=ctx.dtype).view(1, k, 1)
    return last + steps * delta


@pytest.mark.gpu
@pytest.mark.parametrize("B", [2, 11])
def test_gpu_proposer_runs_vae_drafters(B):
    """FlowDrafterProposer on a TreeVAEFlowDrafter checkpoint: 'delta' latents from the encoded
    context, engine plans up to 8 requests and the wide plans above."""
    from chain_flow_b200.proposer import FlowDrafterProposer
    g = load_gvae()
    W = g["W"]
    p = FlowDrafterProposer.from_components(W, _model_args(g, "delta"), g["emb"], g["lm_w"], g["sl"], width=4, K=5,
                                            device="cuda")
    assert p.vae is not None
    rep = (B + g["B"] - 1) // g["B"]
    ctx = g["ctx"].repeat(rep, 1, 1)[:B]
    known0 = g["known0"].repeat(rep)[:B]
    got = p.predict_hidden(ctx.half().cuda())
    mu = oracle.vae_encode(W, ctx.half().float(), g["vae_layers"], g["vae_heads"])
    z0 = _delta_z0(mu.half().float(), g["DL"]).half().float()
    zf = oracle.integrate(W, flow_cfg(g), mu.half().float(), z0)
    want = oracle.vae_decode(W, zf, g["vae_layers"], g["vae_heads"])
    assert _rel(got, want) < HIDDEN_RTOL, _rel(got, want)
    ch = p._beam_chains(ctx.half().cuda(), known0.cuda()).cpu()
    key = (1, B) if B <= 8 else ("wide", 1, B)
    pred = p._plans[key].pred.cpu()
    sl = g["sl"]
    want = oracle.beam_chains(W, flow_cfg(g), g["emb"], g["lm_w"][sl], W["markov.w2.weight"][sl], sl, pred,
                              known0, 4, 5)
    assert torch.equal(ch, want)
    assert p.device_error() == 0
