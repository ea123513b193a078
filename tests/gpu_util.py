"""Helpers shared by the GPU parity tests: build the engine's weights from a golden fixture or
from seeded random reference-layout state dicts (test infrastructure)."""
from __future__ import annotations

import torch

from chain_flow_b200.engine import Plan
from chain_flow_b200.weights import DraftConfig, DrafterWeights


def golden_weights(g) -> DrafterWeights:
    cfg = DraftConfig(hidden=g["H"], num_heads=g["heads"], ffn_multiplier=g["FM"],
                      num_drafter_layers=g["L"], num_flow_steps=g["T"], markov_rank=g["rank"])
    return DrafterWeights(g["W"], cfg, g["emb"], g["lm_w"], g["sl"], device="cuda")


def random_state_dict(cfg: DraftConfig, vocab: int, seed: int = 0) -> dict:
    """Seeded weights with the reference checkpoint's names and shapes; N(0, 0.02) for matrices,
    LN gamma ~ 1 + N(0, 0.1), beta ~ N(0, 0.1); the zero-initialised PathHead output layer and
    markov w2 of the reference (tree_flow.py:95-96, markov_flow.py:69) are seeded non-zero."""
    g = torch.Generator().manual_seed(seed)
    D, FM, L = cfg.hidden, cfg.ffn_multiplier, cfg.num_drafter_layers
    r = lambda *s, std=0.02: (torch.randn(*s, generator=g) * std).to(torch.float16).float()
    sd = {}
    for e in range(cfg.n_experts):
        p = "expert." if e == 0 else f"extra_experts.{e - 1}."
        sd[p + "position_embedding.weight"] = r(cfg.draft_length, D, std=0.5)
        sd[p + "time_mlp.0.weight"] = r(D, 1, std=1.0)
        sd[p + "time_mlp.0.bias"] = r(D, std=1.0)
        sd[p + "time_mlp.2.weight"] = r(D, D)
        sd[p + "time_mlp.2.bias"] = r(D)
        for l in range(L):
            b = f"{p}blocks.{l}."
            for n in ("self_norm", "cross_norm", "context_norm", "ffn.0"):
                sd[f"{b}{n}.weight"] = 1.0 + r(D, std=0.1)
                sd[f"{b}{n}.bias"] = r(D, std=0.1)
            for a in ("self_attn", "cross_attn"):
                sd[f"{b}{a}.in_proj_weight"] = r(3 * D, D)
                sd[f"{b}{a}.in_proj_bias"] = r(3 * D)
                sd[f"{b}{a}.out_proj.weight"] = r(D, D)
                sd[f"{b}{a}.out_proj.bias"] = r(D)
            sd[f"{b}ffn.1.weight"] = r(FM * D, D)
            sd[f"{b}ffn.1.bias"] = r(FM * D)
            sd[f"{b}ffn.4.weight"] = r(D, FM * D)
            sd[f"{b}ffn.4.bias"] = r(D)
        sd[p + "out_norm.weight"] = 1.0 + r(D, std=0.1)
        sd[p + "out_norm.bias"] = r(D, std=0.1)
        sd[p + "out_proj.weight"] = r(D, D)
        sd[p + "out_proj.bias"] = r(D)
    sd["markov.w1.weight"] = r(vocab, cfg.markov_rank, std=0.5)
    sd["markov.w2.weight"] = r(vocab, cfg.markov_rank, std=0.02)
    for j in range(cfg.path_order):
        sd[f"path_head.offset_proj.{j}.weight"] = r(D, D)
        sd[f"path_head.offset_proj.{j}.bias"] = r(D)
    sd["path_head.norm.weight"] = 1.0 + r(D, std=0.1)
    sd["path_head.norm.bias"] = r(D, std=0.1)
    P2 = cfg.path_ffn_multiplier * D
    sd["path_head.mlp.0.weight"] = r(P2, D)
    sd["path_head.mlp.0.bias"] = r(P2)
    sd["path_head.mlp.3.weight"] = r(D, P2)
    sd["path_head.mlp.3.bias"] = r(D)
    return sd


def run_plan(w: DrafterWeights, mode: int, B: int, ctx=None, z0=None, known0=None, pred=None, **kw) -> Plan:
    p = Plan(w, mode, B, **kw)
    if ctx is not None:
        p.ctx.copy_(ctx.to(torch.float16))
    if z0 is not None:
        p.z0.copy_(z0.to(torch.float16))
    if known0 is not None:
        p.known0.copy_(known0)
    if pred is not None:
        p.pred.copy_(pred.float())
    p.run()
    torch.cuda.synchronize()
    p.check()
    return p
