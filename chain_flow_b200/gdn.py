"""Tree-aware Gated-DeltaNet verification on the sm_100a kernel (cfb_tree_gdn).

``tree_gated_delta_scan`` keeps the reference's signature and semantics
(src/chain_flow/kernels/tree_scan.py:43-78) for a single tree, and ``tree_gdn_batched`` runs B
independent trees in one launch. ``make_tree`` builds the seeded BFS parent arrays the
benchmarks use (parent < child, bounded depth and branching). ``gdn_verify`` is the in-engine
variant of the reference's vLLM patch (gate from the model's raw parameters, slot-addressed
states, a path-parallel walk of each row's ancestor chain; cfb_tree_gdn_verify).
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
    parent < child, which the kernel relies on instead); initial_state [H,Dk,Dv]. No host sync: a
    node whose parent is neither -1 nor an earlier node gets NaN output and state (so do its
    descendants), and the bad index is never dereferenced."""
    par = parent.view(1, -1)
    o, st = tree_gdn_batched(query[None], key[None], value[None], g[None], beta[None], par,
                             initial_state[None], use_qk_l2norm=use_qk_l2norm)
    return o[0], st[0]


_DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def ancestor_chains(parent: torch.Tensor, max_depth: int):
    """(chain [N, max_depth + 1] int32, depth [N] int32) from a parent array (parent < child,
    -1 = root) on the parent's device: chain[t, kk] is the ancestor kk levels above node t
    (chain[t, 0] = t; entries past depth[t] repeat the top ancestor), the layout the in-engine
    verify walks from chain[t, depth[t]] (the root) down to t. Pointer jumping with device ops
    only: no host sync, so it can be captured in a CUDA graph."""
    p = parent.to(torch.int64).view(-1)
    N = p.numel()
    cur = torch.arange(N, device=p.device)
    cols, depth = [cur], torch.zeros(N, dtype=torch.int64, device=p.device)
    for _ in range(max_depth):
        up = p[cur] if N else cur
        has = up >= 0
        depth = depth + has.to(torch.int64)
        cur = torch.where(has, up, cur)
        cols.append(cur)
    return torch.stack(cols, dim=1).to(torch.int32), depth.to(torch.int32)


def gdn_verify(A_log, dt_bias, a, b, q, k, v, o, state, chain, depth, out_slot, init_slot, rows=None, *,
               scale: float, write_out: bool = True, write_state: bool = True) -> None:
    """The in-engine tree GDN verify (reference vLLM patch ``gdn_verify``,
    src/chain_flow/patches/vllm-0.25.1-chain-flow-tree.patch:4606) on cfb_tree_gdn_verify: for
    each query row (``rows``, default all), walk its ancestor chain from ``state[init_slot]``,
    write o and ``state[out_slot]`` in place. q, k [T, H, 128] and v, o [T, HV, V] fp16 or
    bf16; a, b [T, HV] and A_log, dt_bias [HV] fp32 / fp16 / bf16; state fp32
    [slots, HV, V, 128]; chain, depth, slots, rows int32, all on one CUDA device."""
    lib = _lib.load()
    for t_, n in ((q, "q"), (k, "k"), (v, "v"), (state, "state"), (chain, "chain")):
        _lib.require_cuda(t_, n)
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise _lib.CfbError("gdn_verify: q, k, v must share one dtype, fp16 or bf16")
    if state.dtype != torch.float32 or state.stride(-1) != 1 or not state[0].is_contiguous():
        raise _lib.CfbError("gdn_verify: state must be fp32 [slots, HV, V, K] with contiguous slots")
    for t_ in (q, k, v, a, b, A_log, dt_bias):
        if not t_.is_contiguous():
            raise _lib.CfbError("gdn_verify: q, k, v, a, b, A_log, dt_bias must be contiguous")
    ints = [t_.to(torch.int32).contiguous() for t_ in (chain, depth, out_slot, init_slot)]
    rows_i = rows.to(torch.int32).contiguous() if rows is not None else None
    T_rows = rows_i.numel() if rows_i is not None else q.shape[0]
    H, K = q.shape[1], q.shape[2]
    HV, V = v.shape[1], v.shape[2]
    _lib.check(lib.cfb_tree_gdn_verify(
        A_log.data_ptr(), _DTYPE_CODE[A_log.dtype], dt_bias.data_ptr(), _DTYPE_CODE[dt_bias.dtype],
        a.data_ptr(), _DTYPE_CODE[a.dtype], b.data_ptr(), _DTYPE_CODE[b.dtype],
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr() if o is not None else None,
        _DTYPE_CODE[q.dtype], state.data_ptr(), state.stride(0), ints[0].data_ptr(), ints[0].stride(0),
        ints[1].data_ptr(), ints[2].data_ptr(), ints[3].data_ptr(),
        rows_i.data_ptr() if rows_i is not None else None, float(scale), T_rows, H, HV, K, V,
        int(write_out), int(write_state), _lib.stream_ptr()), "cfb_tree_gdn_verify")


def gdn_factor(A_log, dt_bias, a, b, q, k, v, o, state, chain, depth, init_slot, row_start, row_count, *,
               scale: float, n_max: int) -> None:
    """The shared-root factorisation of the in-engine verify (reference fork ``gdn_factor``,
    src/chain_flow/patches/vllm-0.25.1-chain-flow-tree.patch:4664-5094) on cfb_tree_gdn_factor:
    the outputs ``o`` of ``gdn_verify`` for requests whose rows [row_start[s], + row_count[s]) all
    start from the state slot ``init_slot[row_start[s]]``, reading that state once per (request,
    head) and writing no state. ``chain`` rows hold global row ids. Same dtypes as ``gdn_verify``;
    n_max >= every row_count (<= 64)."""
    lib = _lib.load()
    for t_, n in ((q, "q"), (k, "k"), (v, "v"), (o, "o"), (state, "state"), (chain, "chain")):
        _lib.require_cuda(t_, n)
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype or o.dtype != q.dtype:
        raise _lib.CfbError("gdn_factor: q, k, v, o must share one dtype, fp16 or bf16")
    if state.dtype != torch.float32 or state.stride(-1) != 1 or not state[0].is_contiguous():
        raise _lib.CfbError("gdn_factor: state must be fp32 [slots, HV, V, K] with contiguous slots")
    for t_ in (q, k, v, o, a, b, A_log, dt_bias):
        if not t_.is_contiguous():
            raise _lib.CfbError("gdn_factor: q, k, v, o, a, b, A_log, dt_bias must be contiguous")
    ch, dp, isl, rs, rc = (t_.to(torch.int32).contiguous() for t_ in (chain, depth, init_slot, row_start, row_count))
    H, K = q.shape[1], q.shape[2]
    HV, V = v.shape[1], v.shape[2]
    _lib.check(lib.cfb_tree_gdn_factor(
        A_log.data_ptr(), _DTYPE_CODE[A_log.dtype], dt_bias.data_ptr(), _DTYPE_CODE[dt_bias.dtype],
        a.data_ptr(), _DTYPE_CODE[a.dtype], b.data_ptr(), _DTYPE_CODE[b.dtype], q.data_ptr(), k.data_ptr(),
        v.data_ptr(), o.data_ptr(), _DTYPE_CODE[q.dtype], state.data_ptr(), state.stride(0), ch.data_ptr(),
        ch.stride(0), dp.data_ptr(), isl.data_ptr(), rs.data_ptr(), rc.data_ptr(), rs.numel(), int(n_max),
        float(scale), H, HV, K, V, _lib.stream_ptr()), "cfb_tree_gdn_factor")
