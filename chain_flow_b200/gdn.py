"""Tree-aware Gated-DeltaNet verification on the sm_100a kernel (cfb_tree_gdn).

``tree_gated_delta_scan`` keeps the reference's signature and semantics
(src/chain_flow/kernels/tree_scan.py:43-78) for a single tree, and ``tree_gdn_batched`` runs B
independent trees in one launch. ``make_tree`` builds the seeded BFS parent arrays the
benchmarks use (parent < child, bounded depth and branching).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib


def make_tree(n_nodes: int, max_depth: int, max_branch: int, seed: int):
    """(parent [N] int64, depth [N] int64) of a random BFS-ordered tree: node 0 is the root,
    every parent index is smaller than its child's, depth < max_depth, children <= max_branch."""
    g = torch.Generator().manual_seed(seed)
    parent, depth, nchild = [], [], []
    while len(parent) < n_nodes:
        i = len(parent)
        if i == 0:
            parent.append(-1); depth.append(0); nchild.append(0)
            continue
        cands = [j for j in range(i) if depth[j] < max_depth - 1 and nchild[j] < max_branch]
        if not cands:
            raise ValueError("tree shape cannot hold that many nodes")
        dmin = min(depth[j] for j in cands)
        cands = [j for j in cands if depth[j] == dmin]
        p = cands[int(torch.randint(len(cands), (1,), generator=g))]
        parent.append(p); depth.append(depth[p] + 1); nchild[p] += 1; nchild.append(0)
    return torch.tensor(parent), torch.tensor(depth)


def tree_gdn_batched(q, k, v, g, beta, parent, init, *, use_qk_l2norm: bool = True,
                     states: torch.Tensor | None = None):
    """q,k [B,N,H,128] fp16; v [B,N,H,Dv] fp16; g,beta [B,N,H] fp32; parent [B,N] (parent < child,
    -1 = reads init); init [B,H,128,Dv] fp32 -> (o [B,N,H,Dv] fp32, states [B,N,H,128,Dv] fp32)."""
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (g, "g"), (beta, "beta"), (init, "init")):
        _lib.require_cuda(t, n)
    B, N, H, Dk = q.shape
    Dv = v.shape[-1]
    q = q.to(torch.float16).contiguous(); k = k.to(torch.float16).contiguous()
    v = v.to(torch.float16).contiguous()
    g = g.to(torch.float32).contiguous(); beta = beta.to(torch.float32).contiguous()
    par = parent.to(device=q.device, dtype=torch.int32).contiguous()
    init = init.to(torch.float32).contiguous()
    o = torch.empty(B, N, H, Dv, device=q.device, dtype=torch.float32)
    if states is None:
        states = torch.empty(B, N, H, Dk, Dv, device=q.device, dtype=torch.float32)
    lib = _lib.load()
    _lib.check(lib.cfb_tree_gdn(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(),
                                par.data_ptr(), init.data_ptr(), o.data_ptr(), states.data_ptr(),
                                B, N, H, Dk, Dv, int(use_qk_l2norm), C.c_void_p(_lib.stream_ptr())),
               "cfb_tree_gdn")
    return o, states


def tree_gated_delta_scan(query, key, value, g, beta, parent, depth, initial_state, *,
                          use_qk_l2norm: bool = True):
    """Reference-signature single tree: query,key [N,H,Dk]; value [N,H,Dv]; g,beta [N,H];
    parent [N] (-1 = root); depth [N] (accepted for signature parity: nodes must be in BFS order,
    parent < child, which the kernel relies on instead); initial_state [H,Dk,Dv]."""
    par = parent.view(1, -1)
    if par.numel() and bool((par >= torch.arange(par.shape[1], device=par.device)).any()):
        raise ValueError("tree nodes must be ordered so that parent < child")
    o, st = tree_gdn_batched(query[None], key[None], value[None], g[None], beta[None], par,
                             initial_state[None], use_qk_l2norm=use_qk_l2norm)
    return o[0], st[0]
