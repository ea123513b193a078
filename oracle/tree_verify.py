"""Oracle: greedy verification of a draft tree (CPU, test infrastructure).

Restates the reference fork's ``tree_rejection_sample`` and ``tree_greedy_descent_kernel``
(``src/chain_flow/patches/vllm-0.25.1-chain-flow-tree.patch:640-723``): the argmax of every logits
row (torch.argmax: the first maximum), then per request a walk from the root row that repeatedly
moves to the first child (node order) whose draft token equals the current row's argmax; the
output is the accepted tokens followed by the bonus token (the argmax of the row where the walk
stops). A request without draft nodes emits its one row's argmax.
"""
from __future__ import annotations

import torch


def tree_verify_greedy(logits, cu_num_draft, cu_num_sampled, draft_tokens, parents, max_spec_len: int):
    """-> (output_tokens [B, max_spec_len + 1], accepted_path [B, max_spec_len], accepted_len [B]),
    int32, -1 padded."""
    row_argmax = logits.float().argmax(dim=-1).tolist()
    cu_d, cu_s = [int(x) for x in cu_num_draft], [int(x) for x in cu_num_sampled]
    dtok, par = [int(x) for x in draft_tokens], [int(x) for x in parents]
    B = len(cu_d)
    out = torch.full((B, max_spec_len + 1), -1, dtype=torch.int32)
    path = torch.full((B, max_spec_len), -1, dtype=torch.int32)
    alen = torch.zeros(B, dtype=torch.int32)
    for r in range(B):
        d0 = cu_d[r - 1] if r else 0
        n = cu_d[r] - d0
        s0 = cu_s[r] - (n + 1)
        cur, pos = -1, 0
        while True:
            tok = row_argmax[s0 + cur + 1]
            out[r, pos] = tok
            nxt = next((i for i in range(n) if par[d0 + i] == cur and dtok[d0 + i] == tok), -1)
            if nxt < 0:
                break
            path[r, pos] = nxt
            cur, pos = nxt, pos + 1
        alen[r] = pos
    return out, path, alen
