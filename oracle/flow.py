"""Oracle: flow integrator, path residual and markov bias (fp32, CPU, test infrastructure).

Functional restatement of the reference drafter's arithmetic over a flat weight dict that
uses the reference checkpoint's parameter names (``expert.blocks.0.self_attn.in_proj_weight``
and so on, i.e. the ``TreeFlowDrafter`` state_dict without the ``drafter.`` prefix).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass
class FlowConfig:
    """The ``TreeFlowConfig`` fields the drafting path reads
    (reference ``src/chain_flow/drafters/tree_flow.py:39-72``)."""
    hidden: int
    context_size: int = 8
    draft_length: int = 6
    chunk_size: int = 3
    num_heads: int = 8
    ffn_multiplier: int = 6
    num_layers: int = 4
    num_flow_steps: int = 8
    path_order: int = 4
    path_ffn_multiplier: int = 2
    markov_rank: int = 256

    @property
    def num_experts(self) -> int:
        return self.draft_length // self.chunk_size

    def expert_prefix(self, e: int) -> str:
        # reference tree_flow.py:131-132: expert 0 is `expert`, the rest `extra_experts.{e-1}`
        return "expert." if e == 0 else f"extra_experts.{e - 1}."


def layer_norm(x, w, b, eps: float = 1e-5):
    """nn.LayerNorm semantics (biased variance, eps inside the sqrt)."""
    mu = x.mean(-1, keepdim=True)
    var = ((x - mu) ** 2).mean(-1, keepdim=True)
    return (x - mu) / torch.sqrt(var + eps) * w + b


def mha(q_in, kv_in, W, prefix: str, num_heads: int, mask=None):
    """nn.MultiheadAttention(batch_first=True) forward with packed in-projection.

    q_in [B, Sq, D], kv_in [B, Sk, D]. Scores are scaled by head_dim**-0.5 and the optional
    additive mask [Sq, Sk] is applied before the softmax (reference chunked_flow.py:185-197
    calls it with q=k=v for self-attention and k=v=context for cross-attention).
    """
    w_in, b_in = W[prefix + "in_proj_weight"], W[prefix + "in_proj_bias"]
    D = q_in.shape[-1]
    hd = D // num_heads
    q = q_in @ w_in[:D].T + b_in[:D]
    k = kv_in @ w_in[D:2 * D].T + b_in[D:2 * D]
    v = kv_in @ w_in[2 * D:].T + b_in[2 * D:]
    B, Sq, _ = q.shape
    Sk = k.shape[1]
    q = q.view(B, Sq, num_heads, hd).transpose(1, 2)
    k = k.view(B, Sk, num_heads, hd).transpose(1, 2)
    v = v.view(B, Sk, num_heads, hd).transpose(1, 2)
    s = (q @ k.transpose(-1, -2)) / math.sqrt(hd)
    if mask is not None:
        s = s + mask
    p = torch.softmax(s, dim=-1)
    o = (p @ v).transpose(1, 2).reshape(B, Sq, D)
    return o @ W[prefix + "out_proj.weight"].T + W[prefix + "out_proj.bias"]


def flow_block(x, ctx, W, prefix: str, num_heads: int, mask):
    """One HiddenKVFlowBlock (reference chunked_flow.py:168-202): pre-LN causal self-attention,
    pre-LN cross-attention to the LayerNorm'd context, pre-LN FFN with exact (erf) GELU,
    each added to the residual stream."""
    a = layer_norm(x, W[prefix + "self_norm.weight"], W[prefix + "self_norm.bias"])
    x = x + mha(a, a, W, prefix + "self_attn.", num_heads, mask)
    c = layer_norm(x, W[prefix + "cross_norm.weight"], W[prefix + "cross_norm.bias"])
    kv = layer_norm(ctx, W[prefix + "context_norm.weight"], W[prefix + "context_norm.bias"])
    x = x + mha(c, kv, W, prefix + "cross_attn.", num_heads, None)
    f = layer_norm(x, W[prefix + "ffn.0.weight"], W[prefix + "ffn.0.bias"])
    u = F.gelu(f @ W[prefix + "ffn.1.weight"].T + W[prefix + "ffn.1.bias"])
    return x + u @ W[prefix + "ffn.4.weight"].T + W[prefix + "ffn.4.bias"]


def time_embedding(W, prefix: str, tau: float):
    """time_mlp = Linear(1,D) -> SiLU -> Linear(D,D) at scalar tau (reference
    chunked_flow.py:230-234, 313-321). Every row of a draft shares tau, so this is a [D] vector."""
    t = W[prefix + "time_mlp.0.weight"][:, 0] * tau + W[prefix + "time_mlp.0.bias"]
    t = F.silu(t)
    return W[prefix + "time_mlp.2.weight"] @ t + W[prefix + "time_mlp.2.bias"]


def expert_velocity(W, cfg: FlowConfig, e: int, ctx, z, tau: float):
    """Velocity of chunk expert ``e`` (reference HiddenKVFlowExpert.pre_blocks/forward/post_blocks,
    chunked_flow.py:333-414, with the chunk slicing of tree_flow.py:163-174).

    The expert sees the previous chunks' rows of the CURRENT iterate z (positions 0..start-1)
    followed by its own chunk (positions start..start+chunk-1); only its own rows get the time
    embedding; a causal mask spans all its rows; only its own rows are projected out.
    """
    p = cfg.expert_prefix(e)
    start, chunk = e * cfg.chunk_size, cfg.chunk_size
    x = z[:, :start + chunk, :].clone()
    S = x.shape[1]
    x = x + W[p + "position_embedding.weight"][:S]
    x[:, start:] = x[:, start:] + time_embedding(W, p, tau)
    mask = torch.triu(torch.full((S, S), float("-inf"), device=z.device, dtype=z.dtype), diagonal=1)
    for i in range(cfg.num_layers):
        x = flow_block(x, ctx, W, f"{p}blocks.{i}.", cfg.num_heads, mask)
    cur = layer_norm(x[:, start:], W[p + "out_norm.weight"], W[p + "out_norm.bias"])
    return cur @ W[p + "out_proj.weight"].T + W[p + "out_proj.bias"]


def integrate(W, cfg: FlowConfig, ctx, z0):
    """Explicit Euler over tau = s/T, s = 0..T-1 (reference tree_flow.py:229-235). Every chunk
    expert reads the same iterate z (reference tree_flow.py:163-174), so the experts of one step
    are independent. Computes in the dtype of the expert weights (fp32 for the CPU checks)."""
    wd = W[cfg.expert_prefix(0) + "out_proj.weight"].dtype
    z = z0.to(wd)
    ctx = ctx.to(wd)
    T = cfg.num_flow_steps
    dt = 1.0 / T
    for s in range(T):
        tau = s * dt
        v = torch.cat([expert_velocity(W, cfg, e, ctx, z, tau) for e in range(cfg.num_experts)],
                      dim=1)
        z = z + dt * v
    return z


def path_residual(W, emb, lastp, order: int, nlive: int | None = None):
    """PathHead residual from the last-``order`` path tokens (reference
    tree_flow.py:434-450 / vllm_plugin/fused.py:27-37).

    lastp [N, order] int64 global token ids, -1 = no such ancestor. Offsets >= nlive are
    skipped (they are provably masked, reference flow_proposer.py:1030-1037).
    h = sum_j mask_j * (W_j emb(lastp_j) + b_j);  res = W_m2 gelu(W_m1 LN(h) + b_m1) + b_m2.
    """
    o = order if nlive is None else min(nlive, order)
    wd = W["path_head.offset_proj.0.weight"].dtype
    lp = lastp[:, :o]
    mask = (lp >= 0).to(wd)
    e = emb[lp.clamp_min(0)].to(wd)                           # [N, o, D]
    h = None
    for j in range(o):
        t = (e[:, j] @ W[f"path_head.offset_proj.{j}.weight"].T
             + W[f"path_head.offset_proj.{j}.bias"]) * mask[:, j:j + 1]
        h = t if h is None else h + t
    n = layer_norm(h, W["path_head.norm.weight"], W["path_head.norm.bias"])
    m = F.gelu(n @ W["path_head.mlp.0.weight"].T + W["path_head.mlp.0.bias"])
    return m @ W["path_head.mlp.3.weight"].T + W["path_head.mlp.3.bias"]


def markov_bias(W, w2_sl, prev):
    """MarkovHead bias on the shortlist rows: w1[prev] @ w2[sl]^T (reference
    markov_flow.py:72-74, flow_proposer.py:1024-1025)."""
    return W["markov.w1.weight"][prev].to(w2_sl.dtype) @ w2_sl.T
