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
