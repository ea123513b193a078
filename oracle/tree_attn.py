"""Oracle: the tree-attention fix-up of a full-attention layer (fp32, CPU, test infrastructure).

Restates the reference fork's eager suffix + merge, ``_tree_suffix_eager``
(``src/chain_flow/patches/vllm-0.25.1-chain-flow-tree.patch:529-575``): every tree node attends to
its ancestors (the dense score matrix masked by ``not_anc``), and the result, rounded to the
output dtype, is merged with the paged-prefix result by vLLM's ``merge_attn_states`` (its CUDA
op: a +inf lse counts as -inf; out = prefix * ps / (ps + ss) + suffix * ss / (ps + ss)). The
merged rows land at the nodes' query rows ``idx``.
"""
from __future__ import annotations

import torch


def tree_attn_merge(query, key, value, output, prefix_out, prefix_lse, idx, not_anc, scale):
    """Returns a copy of ``output`` (fp32) with the merged tree rows written; the suffix is rounded to
    ``output.dtype`` before the merge like the eager path's ``.to(output.dtype)``."""
    S, N = idx.shape
    H, D = query.shape[1], query.shape[2]
    rep = H // key.shape[1]
    flat = idx.reshape(-1).long()
    qp = query.float()[flat].view(S, N, H, D)
    kp = key.float()[flat].view(S, N, -1, D).repeat_interleave(rep, dim=2)
    vp = value.float()[flat].view(S, N, -1, D).repeat_interleave(rep, dim=2)
    scores = torch.einsum("snhd,smhd->shnm", qp, kp) * scale
    scores = scores.masked_fill(not_anc.bool().unsqueeze(1), float("-inf"))
    smax = scores.amax(dim=-1, keepdim=True)
    e = torch.exp(scores - smax)
    den = e.sum(dim=-1, keepdim=True)
    s_lse = (smax + torch.log(den)).squeeze(-1)                      # [S, H, N]
    suffix = torch.einsum("shnm,smhd->snhd", e / den, vp)             # [S, N, H, D]
    suffix = suffix.reshape(S * N, H, D).to(output.dtype).float()
    s_lse = s_lse.permute(0, 2, 1).reshape(S * N, H)                  # [S*N, H]
    p_lse = prefix_lse.float().transpose(0, 1)                        # [S*N, H]
    inf = float("inf")
    p_lse = torch.where(p_lse == inf, torch.full_like(p_lse, -inf), p_lse)
    s_lse = torch.where(s_lse == inf, torch.full_like(s_lse, -inf), s_lse)
    mx = torch.maximum(p_lse, s_lse)
    ps, ss = torch.exp(p_lse - mx), torch.exp(s_lse - mx)
    tot = ps + ss
    merged = prefix_out.float() * (ps / tot).unsqueeze(-1) + suffix * (ss / tot).unsqueeze(-1)
    out = output.float().clone()
    out[flat] = merged
    return out


def attention_over(q, keys, values, scale):
    """Plain softmax attention of one query row over explicit key / value rows (fp64): the identity
    the prefix / suffix split must reproduce (test infrastructure)."""
    s = (keys.double() @ q.double()) * scale
    p = torch.softmax(s, dim=0)
    return p @ values.double(), torch.logsumexp(s, dim=0)
