"""Tie-aware check of an engine tree draft against the oracle (test infrastructure).

Token ids must match the reference exactly where the competing candidates are not tied. The
engine feeds the head fp16 inputs, so two candidates whose cumulative log-probabilities differ
by less than that rounding may come out in either order. This walks the tree level by level
along the ENGINE's choices and checks each level with the oracle's scores. The selected
(parent, token) pairs must be distinct. They must be in non-increasing score order. Each must
score within `eps` of the oracle's k-th best candidate. Following the reference beam
(flow_proposer.py:1273-1332), each parent row offers its top-`topb` tokens.
"""
from __future__ import annotations

import torch

import oracle


def check_tree(tokens, W, cfg, emb, hw, w2, sl, pred, known0, keep, topb, depth, eps=5e-3, tp_cand=None):
    """tokens [B, 2N] from the engine; raises AssertionError with the first violation. tp_cand [B, M]:
    the two-pass head's candidate rows (log-probs normalised over them), else the one-pass head."""
    B = pred.shape[0]
    order = cfg.path_order
    N = tokens.shape[1] // 2
    for b in range(B):
        lastp = torch.full((1, order), -1, dtype=torch.long)
        lastp[0, 0] = int(known0[b])
        cum = torch.zeros(1)
        fr, base, prev_base = 1, 0, 0
        for step in range(1, min(depth, pred.shape[1] - 1) + 1):
            k = min(keep, fr * topb)
            h = pred[b, step].float().unsqueeze(0).expand(fr, -1)
            if tp_cand is None:
                _, lp = oracle.head_logprobs(W, emb, hw, w2, h, lastp, order, step)
            else:   # scores of the candidates, scattered back to shortlist rows (-inf elsewhere)
                lpc = oracle.twopass_logprobs(W, emb, hw, w2, tp_cand[b:b + 1], h, lastp, order, step, 1)[0]
                lp = torch.full((fr, sl.numel()), float("-inf"))
                lp[:, tp_cand[b]] = lpc
            cv, ci = lp.topk(topb, dim=-1)                                  # [fr, topb]
            cand = (cum.view(fr, 1) + cv).reshape(-1)
            kth = cand.topk(k).values[-1]
            toks = tokens[b, base:base + k]
            pars = tokens[b, N + base:N + base + k]
            seen, scores, new_lastp = set(), [], []
            for i in range(k):
                par = int(pars[i])
                src = 0 if step == 1 else par - prev_base
                assert (par == -1) == (step == 1) and 0 <= src < fr, (b, step, i, par)
                loc = int(torch.searchsorted(sl, toks[i]))
                assert loc < sl.numel() and int(sl[loc]) == int(toks[i]), (b, step, i, "not a shortlist id")
                assert (src, loc) not in seen, (b, step, i, "duplicate candidate")
                seen.add((src, loc))
                assert bool((ci[src] == loc).any()), (b, step, i, "token outside its parent's top-topb")
                s = float(cum[src] + lp[src, loc])
                assert s >= float(kth) - eps, (b, step, i, s, float(kth))
                if scores:
                    assert s <= scores[-1] + eps, (b, step, i, "not in score order")
                scores.append(s)
                new_lastp.append(torch.cat([toks[i:i + 1], lastp[src, :-1]]))
            lastp = torch.stack(new_lastp)
            cum = torch.tensor(scores)
            prev_base, base, fr = base, base + k, k
        assert base == N, (b, base, N)


def chain_logprob(W, cfg, emb, hw, w2, sl, pred_b, known0_b, toks):
    """The oracle's cumulative log-prob of one chain (tokens at depths 1..K) of one request: the
    sum over depths of log_softmax((h + path residual) @ hw^T + markov bias) at the chain's token,
    with the path built from the chain itself (reference flow_proposer.py:1234-1259)."""
    order = cfg.path_order
    lastp = torch.full((1, order), -1, dtype=torch.long)
    lastp[0, 0] = int(known0_b)
    total = 0.0
    for d, t in enumerate(toks.tolist(), start=1):
        _, lp = oracle.head_logprobs(W, emb, hw, w2, pred_b[d].float().unsqueeze(0), lastp, order, d)
        loc = int(torch.searchsorted(sl, torch.tensor(t)))
        assert loc < sl.numel() and int(sl[loc]) == t, (d, t, "not a shortlist id")
        total += float(lp[0, loc])
        lastp = torch.cat([torch.tensor([[t]]), lastp[:, :-1]], dim=1)
    return total


def check_chain(tokens, W, cfg, emb, hw, w2, sl, pred, known0, width, K, eps=5e-3):
    """tokens [B, K] from the engine against the oracle's chain beam over the same hiddens `pred`.
    A request must match exactly, or else (a near-tie the engine's fp16 head inputs can flip) its
    chain must score, under the oracle, within `eps` of the oracle's best final beam. Returns the
    number of requests that matched exactly."""
    want, _, cum = oracle.beam_chains(W, cfg, emb, hw, w2, sl, pred, known0, width, K, return_beams=True)
    exact = 0
    for b in range(tokens.shape[0]):
        if torch.equal(tokens[b], want[b]):
            exact += 1
            continue
        s = chain_logprob(W, cfg, emb, hw, w2, sl, pred[b], known0[b], tokens[b])
        best = float(cum[b].max())
        assert s >= best - eps, (b, tokens[b].tolist(), want[b].tolist(), s, best)
    return exact
