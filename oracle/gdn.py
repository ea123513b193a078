"""Oracle: tree-aware Gated-DeltaNet recurrence (fp32, CPU, test infrastructure).

Restates ``tree_gated_delta_scan`` and ``sequential_path_output`` from the reference
``src/chain_flow/kernels/tree_scan.py:25-96``. Per node n with parent p (p = -1 for a root,
which reads the shared prefix state):

    S_n = S_p * exp(g_n)
    S_n = S_n + k_n (x) (beta_n * (v_n - S_n^T k_n))
    o_n = S_n^T q_n

with q, k L2-normalised as x / (||x|| + 1e-6) and q scaled by Dk**-0.5. States are
[H, Dk, Dv] fp32.
"""
from __future__ import annotations

import torch


def _l2n(x, eps=1e-6):
    return x / (x.norm(dim=-1, keepdim=True) + eps)


def _step(S, q, k, v, g, beta):
    S = S * g.exp()[..., None, None]
    kv = (S * k[..., None]).sum(-2)                     # S^T k  [.., Dv]
    S = S + k[..., None] * ((v - kv) * beta[..., None])[..., None, :]
    o = (S * q[..., None]).sum(-2)
    return S, o


def tree_gdn_scan(q, k, v, g, beta, parent, depth, init, use_qk_l2norm=True):
    """q,k [N,H,Dk]; v [N,H,Dv]; g,beta [N,H]; parent,depth [N]; init [H,Dk,Dv]
    -> (o [N,H,Dv], states [N,H,Dk,Dv]). Depth-synchronous, like the reference."""
    q, k, v, g, beta = (t.float() for t in (q, k, v, g, beta))
    if use_qk_l2norm:
        q, k = _l2n(q), _l2n(k)
    N, H, Dk = q.shape
    Dv = v.shape[-1]
    q = q * Dk ** -0.5
    states = torch.zeros(N, H, Dk, Dv)
    out = torch.zeros(N, H, Dv)
    init = init.float()
    maxd = int(depth.max()) if N else -1
    for d in range(maxd + 1):
        idx = (depth == d).nonzero(as_tuple=True)[0]
        if idx.numel() == 0:
            continue
        Sp = init.unsqueeze(0).expand(idx.numel(), -1, -1, -1) if d == 0 else states[parent[idx]]
        Sn, o = _step(Sp, q[idx], k[idx], v[idx], g[idx], beta[idx])
        states[idx] = Sn
        out[idx] = o
    return out, states


def path_gdn_output(q, k, v, g, beta, path, init, use_qk_l2norm=True):
    """Sequential recurrence along one root..node path; returns the last node's o [H, Dv]."""
    q, k, v, g, beta = (t.float() for t in (q, k, v, g, beta))
    if use_qk_l2norm:
        q, k = _l2n(q), _l2n(k)
    q = q * q.shape[-1] ** -0.5
    S = init.float().clone().unsqueeze(0)
    o = None
    for n in path:
        S, o = _step(S, q[n:n + 1], k[n:n + 1], v[n:n + 1], g[n:n + 1], beta[n:n + 1])
    return o[0]


def tree_gdn_verify(A_log, dt_bias, a, b, q, k, v, state, chain, depth, out_slot, init_slot, scale,
                    rows=None, write_out=True, write_state=True, threshold=20.0):
    """The in-engine tree GDN verify of the reference's vLLM patch (``gdn_verify_kernel``,
    src/chain_flow/patches/vllm-0.25.1-chain-flow-tree.patch:4401-4562, and the Triton
    ``_tree_gdn_kernel`` it replaces, :3285-3385). Path-parallel: every query row t re-walks its
    ancestor chain from its initial state slot:

        S = state[init_slot[t], hv]                        (V x K, fp32)
        for kk = depth[t] .. 0:  n = chain[t, kk]
            kn = k[n, h] * rsqrt(||k[n, h]||^2 + 1e-6)
            S  = S * exp(-exp(A_log[hv]) * softplus(a[n, hv] + dt_bias[hv]))   (softplus = x
                                                                      above `threshold`)
            S  = S + beta_n * (v[n, hv] - S kn) (x) kn,   beta_n = sigmoid(b[n, hv])
        o[t, hv]  = S (q[t, h] * rsqrt(||q[t, h]||^2 + 1e-6) * scale)
        state[out_slot[t], hv] = S

    with h = hv // (HV // H). q, k [T, H, K]; v, o [T, HV, V]; a, b [T, HV]; A_log, dt_bias
    [HV]; state [slots, HV, V, K]; chain [T, >= MAXD + 1]; depth, slots [T]; rows: the query
    rows to run (default all). Returns (o [T, HV, V] fp32, new state); states are read from the
    input `state` only."""
    q, k, v, a, b = (t.float() for t in (q, k, v, a, b))
    A_log, dt_bias = A_log.float(), dt_bias.float()
    T, H, K = q.shape
    HV, V = v.shape[1], v.shape[2]
    rep = HV // H
    st = state.float().clone()
    o = torch.zeros(T, HV, V)
    negA = -A_log.exp()
    rr = range(T) if rows is None else [int(r) for r in rows]
    for t in rr:
        for hv in range(HV):
            h = hv // rep
            S = state[int(init_slot[t]), hv].float().clone()            # [V, K]
            for kk in range(int(depth[t]), -1, -1):
                n = int(chain[t, kk])
                kn = k[n, h] * torch.rsqrt((k[n, h] * k[n, h]).sum() + 1e-6)
                x = a[n, hv] + dt_bias[hv]
                sp = torch.log1p(torch.exp(x)) if x <= threshold else x
                S = S * torch.exp(negA[hv] * sp)
                part = S @ kn                                              # [V]
                beta = torch.sigmoid(b[n, hv])
                S = S + ((v[n, hv] - part) * beta)[:, None] * kn[None, :]
            if write_out:
                qn = q[t, h] * torch.rsqrt((q[t, h] * q[t, h]).sum() + 1e-6) * scale
                o[t, hv] = S @ qn
            if write_state:
                st[int(out_slot[t]), hv] = S
    return o, st


def tree_gdn_factor(A_log, dt_bias, a, b, q, k, v, state, chain, depth, init_slot, row_start, row_count, scale,
                    threshold=20.0):
    """The shared-root factorisation of the verify (reference fork ``gdn_factor``,
    src/chain_flow/patches/vllm-0.25.1-chain-flow-tree.patch:4664-5094): every row of request s
    starts from H = state[init_slot[row_start[s]], hv]; a node's state is
    h_t = D_t H + sum_{m on its path} w_{m,t} u_m kn_m^T (every update is rank 1), so with
    S_t = h_parent kn_t = D_p (H kn_t) + sum_{m on the parent's path} w_{m,p} (kn_m . kn_t) u_m,
    u_t = beta_t (v_t - g_t S_t), D_t = g_t D_p, w_{m,t} = g_t w_{m,p}, w_{t,t} = 1, and
    o_t = D_t (H qn_t) + sum_{m on t's path} w_{m,t} (kn_m . qn_t) u_m. Returns o [T, HV, V] fp32
    (rows outside the requests stay zero). Equal to tree_gdn_verify's o up to rounding."""
    q, k, v, a, b = (t.float() for t in (q, k, v, a, b))
    A_log, dt_bias = A_log.float(), dt_bias.float()
    T, H, K = q.shape
    HV, V = v.shape[1], v.shape[2]
    rep = HV // H
    o = torch.zeros(T, HV, V)
    kn = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    qn = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6) * scale
    x = a + dt_bias[None, :]
    sp = torch.where(x <= threshold, torch.log1p(torch.exp(x)), x)
    g = torch.exp(-A_log.exp()[None, :] * sp)                          # [T, HV]
    beta = torch.sigmoid(b)
    for s in range(len(row_start)):
        base, n = int(row_start[s]), int(row_count[s])
        rows = range(base, base + n)
        order = sorted(rows, key=lambda t: int(depth[t]))              # parents before children
        for hv in range(HV):
            h = hv // rep
            Hs = state[int(init_slot[base]), hv].float()                # [V, K]
            u, D, w = {}, {}, {}
            for t in order:
                d = int(depth[t])
                path = [int(chain[t, j]) for j in range(d + 1)]         # t, parent, ..., top
                if d > 0:
                    p = path[1]
                    S = D[p] * (Hs @ kn[t, h])
                    for j, m in enumerate(path[1:]):                    # w_{m,p} = w[p][j]
                        S = S + w[p][j] * (kn[m, h] @ kn[t, h]) * u[m]
                    D[t] = D[p] * g[t, hv]
                    w[t] = [1.0] + [w[p][j] * g[t, hv] for j in range(d)]
                else:
                    S = Hs @ kn[t, h]
                    D[t] = g[t, hv]
                    w[t] = [1.0]
                u[t] = beta[t, hv] * (v[t, hv] - g[t, hv] * S)
            for t in rows:
                d = int(depth[t])
                acc = D[t] * (Hs @ qn[t, h])
                for j in range(d + 1):
                    m = int(chain[t, j])
                    acc = acc + w[t][j] * (kn[m, h] @ qn[t, h]) * u[m]
                o[t, hv] = acc
    return o
