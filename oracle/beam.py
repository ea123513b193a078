"""Oracle: shortlist head + beam search (chain and tree), fp32 CPU, test infrastructure.

Restates ``FlowDrafterProposer._beam_chains`` (reference
``src/chain_flow/vllm_plugin/flow_proposer.py:1188-1269``) and ``_beam_tree`` (``:1273-1332``)
with ``CF_FEEDBACK=0`` and ``CF_PATH_TRIM=1``: the one-pass head (``CF_TWOPASS_M=0``), or the
two-pass candidate head with one candidate set shared by every depth (``CF_TWOPASS_M=M``,
``CF_TWOPASS_SHARED=1``, ``CF_TWOPASS_SEED=0``; ``_candidates`` / ``_gather_cand`` /
``_rescore``, ``flow_proposer.py:1142-1184``).
"""
from __future__ import annotations

import torch

from .flow import FlowConfig, path_residual, markov_bias


def head_logprobs(W, emb, hw, w2_sl, h, lastp, order, nlive):
    """log_softmax over the shortlist of (h + path residual) @ hw^T + markov bias
    (reference flow_proposer.py:1021-1025, 1247-1249). Returns (logits, logprobs) [N, R]."""
    res = path_residual(W, emb, lastp, order, nlive)
    # the reference's dtypes: head and bias in the weights' dtype, log_softmax in fp32
    logits = ((h.to(res.dtype) + res).to(hw.dtype) @ hw.T + markov_bias(W, w2_sl, lastp[:, 0]).to(hw.dtype)).float()
    return logits, torch.log_softmax(logits, dim=-1)


def twopass_candidates(hw, pred, lo: int, hi: int, M: int):
    """Pass A of the two-pass head, shared mode (flow_proposer.py:1142-1165): one GEMM of the
    marginal hiddens pred[:, lo:hi] against the whole shortlist head, log_softmax per depth (fp32),
    the best log-prob of each row over the depths, and its top M -> [B, M] shortlist-local ids
    (sorted by score, as torch.topk returns them)."""
    B, n = pred.shape[0], hi - lo
    hm = pred[:, lo:hi].reshape(B * n, -1)
    logits = (hm.to(hw.dtype) @ hw.T).float()
    lp = torch.log_softmax(logits.view(B, n, -1), dim=-1).amax(dim=1)
    return lp.topk(M, dim=-1).indices


def twopass_logprobs(W, emb, hw, w2_sl, cd, h, lastp, order, nlive, B: int):
    """Pass B (flow_proposer.py:1167-1184): the rows of this depth rescored against the
    gathered candidate rows only; log_softmax over the M candidates. h, lastp [B*F, ...] ->
    [B, F, M]."""
    res = path_residual(W, emb, lastp, order, nlive)
    x = (h.to(res.dtype) + res).view(B, -1, res.shape[-1])
    wc, w2c = hw[cd], w2_sl[cd]                                        # [B, M, D], [B, M, rank]
    mb = W["markov.w1.weight"][lastp[:, 0]].view(B, x.shape[1], -1)
    logits = torch.bmm(x.to(wc.dtype), wc.transpose(1, 2)) + torch.bmm(mb.to(w2c.dtype), w2c.transpose(1, 2))
    return torch.log_softmax(logits.float(), dim=-1)


def beam_chains(W, cfg: FlowConfig, emb, hw, w2_sl, sl, pred, known0, width: int, K: int,
                twopass_m: int = 0, cand=None, return_beams: bool = False):
    """Chain beam over the integrated hiddens ``pred`` [B, draft_length, D].

    Depth 0 is seeded with the committed token (one live beam, cum = [0, -inf, ...]); depths
    1..K each rescore every beam with the path residual + markov bias, keep the top ``width``
    extensions of the width x width candidates, then the best path is walked back.
    Returns [B, K] int64 global token ids.
    """
    B, dev = pred.shape[0], pred.device
    Wd, order = width, cfg.path_order
    lastp = torch.full((B, Wd, order), -1, dtype=torch.long, device=dev)
    lastp[:, :, 0] = known0.view(B, 1)
    cum = torch.full((B, Wd), float("-inf"), device=dev)
    cum[:, 0] = 0.0
    steps = min(K + 1, pred.shape[1])
    toks, bps = [], []
    cd = cand if cand is not None else (
        twopass_candidates(hw, pred, 1, steps, twopass_m) if twopass_m and steps > 1 else None)
    for step in range(1, steps):
        h = pred[:, step].float().unsqueeze(1).expand(B, Wd, -1).reshape(B * Wd, -1)
        if cd is not None:
            lp = twopass_logprobs(W, emb, hw, w2_sl, cd, h, lastp.reshape(B * Wd, order), order, step, B)
            cv, ii = lp.topk(Wd, dim=-1)                                # [B, W, W]
            cv = cv.reshape(B * Wd, Wd)
            ci = cd.gather(1, ii.reshape(B, Wd * Wd))
        else:
            _, lp = head_logprobs(W, emb, hw, w2_sl, h, lastp.reshape(B * Wd, order), order, step)
            cv, ci = lp.topk(Wd, dim=-1)                                # [B*W, W]
            ci = ci.reshape(B, Wd * Wd)
        cand = (cum.reshape(B * Wd, 1) + cv).reshape(B, Wd * Wd)
        cum, flat = cand.topk(Wd, dim=-1)
        src = flat // Wd
        newtok = sl[ci.gather(1, flat)]
        lastp = lastp.gather(1, src.unsqueeze(-1).expand(B, Wd, order))
        lastp = torch.cat([newtok.unsqueeze(-1), lastp[:, :, :-1]], dim=-1)
        toks.append(newtok)
        bps.append(src)
    idx = cum.argmax(dim=-1)
    seq = [None] * len(toks)
    for step in range(len(toks) - 1, -1, -1):
        seq[step] = toks[step].gather(1, idx.unsqueeze(1)).squeeze(1)
        idx = bps[step].gather(1, idx.unsqueeze(1)).squeeze(1)
    best = torch.stack(seq, dim=1)
    if not return_beams:
        return best
    # every final beam's path and cumulative log-prob (for checks of near-tied final beams)
    beams = []
    for w0 in range(Wd):
        idx = torch.full((B,), w0, dtype=torch.long, device=dev)
        sq = [None] * len(toks)
        for step in range(len(toks) - 1, -1, -1):
            sq[step] = toks[step].gather(1, idx.unsqueeze(1)).squeeze(1)
            idx = bps[step].gather(1, idx.unsqueeze(1)).squeeze(1)
        beams.append(torch.stack(sq, dim=1))
    return best, torch.stack(beams, dim=1), cum


def beam_tree(W, cfg: FlowConfig, emb, hw, w2_sl, sl, pred, known0, keep: int, topb: int,
              depth: int, twopass_m: int = 0, cand=None):
    """Tree draft: every surviving extension becomes a BFS-ordered node. Returns [B, 2N]
    = N global token ids followed by N parent node indices (-1 for depth-1 nodes)."""
    B, dev = pred.shape[0], pred.device
    order = cfg.path_order
    fr = 1
    lastp = torch.full((B, fr, order), -1, dtype=torch.long, device=dev)
    lastp[:, :, 0] = known0.view(B, 1)
    cum = torch.zeros(B, fr, device=dev)
    prev_ids = torch.full((B, fr), -1, dtype=torch.long, device=dev)
    toks, pars = [], []
    base = 0
    nstep = min(depth, pred.shape[1] - 1)
    cd = cand if cand is not None else (
        twopass_candidates(hw, pred, 1, nstep + 1, twopass_m) if twopass_m and nstep > 0 else None)
    for step in range(1, nstep + 1):
        h = pred[:, step].float().unsqueeze(1).expand(B, fr, -1).reshape(B * fr, -1)
        if cd is not None:
            lp = twopass_logprobs(W, emb, hw, w2_sl, cd, h, lastp.reshape(B * fr, order), order, step, B)
            cv, ii = lp.topk(topb, dim=-1)                              # [B, fr, TB]
            cv = cv.reshape(B * fr, topb)
            ci = cd.gather(1, ii.reshape(B, fr * topb))
        else:
            _, lp = head_logprobs(W, emb, hw, w2_sl, h, lastp.reshape(B * fr, order), order, step)
            cv, ci = lp.topk(topb, dim=-1)                              # [B*fr, TB]
            ci = ci.reshape(B, fr * topb)
        cand = (cum.reshape(B * fr, 1) + cv).reshape(B, fr * topb)
        k = min(keep, fr * topb)
        cum, flat = cand.topk(k, dim=-1)
        src = flat // topb
        newtok = sl[ci.gather(1, flat)]
        toks.append(newtok)
        pars.append(prev_ids.gather(1, src))
        lastp = lastp.gather(1, src.unsqueeze(-1).expand(B, k, order))
        lastp = torch.cat([newtok.unsqueeze(-1), lastp[:, :, :-1]], dim=-1)
        prev_ids = base + torch.arange(k, device=dev).expand(B, k)
        base += k
        fr = k
    return torch.cat(toks + pars, dim=1)
