"""Oracle: the per-request context ring (fp16 hidden states), CPU, test infrastructure.

Restates ``FlowDrafterProposer._ring_write`` and ``_ring_gather`` (reference
``src/chain_flow/vllm_plugin/flow_proposer.py:916-961``; the ring of ``_init_ring``, ``:881-889``):
slot r of ``ring [slots, C + 1, H]`` holds the last C hidden states of one request, ``rpos[r]``
is its next write position and ``nval[r]`` (<= C) how many rows are valid; row C is a trash row
that masked-off writes go to.
"""
from __future__ import annotations

import torch


def ring_write(ring, rpos, nval, sh, rows, starts, cnt, wmask, path, kmax):
    """Append each request's accepted hidden states (in place). Row j of request b is
    ``sh[start_b + off_j]`` (clamped into sh), off_j = j on a chain step, or 0 for the committed
    token then ``1 + path[rows_b, j - 1]`` for the accepted tree nodes (flow_proposer.py:929-935).
    Rows j >= cnt_b, and every row of a request with wmask_b False, go to the trash row; rpos
    advances by cnt_b (mod C) and nval saturates at C (flow_proposer.py:936-945)."""
    C = ring.shape[1] - 1
    for b in range(rows.numel()):
        r = int(rows[b])
        head = int(rpos[r])
        for j in range(kmax):
            if path is None:
                off = j
            else:
                off = 0 if j == 0 else 1 + int(path[r, j - 1])
            valid = j < int(cnt[b]) and bool(wmask[b])
            src = min(max(int(starts[b]) + off, 0), sh.shape[0] - 1) if valid else 0
            dst = (head + j) % C if valid else C
            ring[r, dst] = sh[src].to(ring.dtype)
        add = int(cnt[b]) if bool(wmask[b]) else 0
        rpos[r] = (head + add) % C
        nval[r] = min(int(nval[r]) + add, C)


def ring_gather(ring, rpos, nval, rows):
    """[B, C, H]: each slot's history oldest first; with m < C valid rows the window is
    front-padded by repeating the oldest row (flow_proposer.py:947-961)."""
    C = ring.shape[1] - 1
    out = torch.empty(rows.numel(), C, ring.shape[2], dtype=ring.dtype)
    for b in range(rows.numel()):
        r = int(rows[b])
        m, head = int(nval[r]), int(rpos[r])
        for j in range(C):
            t = min(max(j - (C - m), 0), max(m - 1, 0))
            out[b, j] = ring[r, (head - m + t) % C]
    return out
