"""The in-engine tree GDN verify (reference vLLM patch gdn_verify_kernel,
vllm-0.25.1-chain-flow-tree.patch:4401-4562).

* CPU: the oracle's path-parallel verify equals the golden-pinned node-serial recurrence
  (oracle.tree_gdn_scan, checked against the reference's tree_scan outputs) on the same tree,
  with g = -exp(A_log) softplus(a + dt_bias) and beta = sigmoid(b); the two differ only in where
  the 1e-6 of the L2 normalisation sits, far below the tolerance.
* GPU: cfb_tree_gdn_verify against the oracle, <= 1e-2 relative on outputs and states (the GDN
  tolerance), fp16 and bf16 q/k/v, grouped value heads, a row subset, write flags.
"""
import pytest
import torch
import torch.nn.functional as F

import oracle

GDN_RTOL = 1e-2


def _case(seed, T=24, H=2, HV=4, V=64, K=128, max_depth=5, slots=None):
    from chain_flow_b200.gdn import ancestor_chains, make_tree
    g = torch.Generator().manual_seed(seed)
    parent, _ = make_tree(T, max_depth, 4, seed)
    chain, depth = ancestor_chains(parent, max_depth)
    slots = slots or T + 1
    return dict(
        A_log=torch.randn(HV, generator=g) * 0.5, dt_bias=torch.randn(HV, generator=g) * 0.5,
        a=torch.randn(T, HV, generator=g), b=torch.randn(T, HV, generator=g),
        q=torch.randn(T, H, K, generator=g).half(), k=torch.randn(T, H, K, generator=g).half(),
        v=torch.randn(T, HV, V, generator=g).half(),
        state=torch.randn(slots, HV, V, K, generator=g) * 0.1,
        chain=chain, depth=depth, parent=parent,
        init_slot=torch.zeros(T, dtype=torch.int32), out_slot=torch.arange(1, T + 1, dtype=torch.int32))


def _rel(a, b):
    return float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-12))


def test_verify_oracle_equals_pinned_node_serial_recurrence():
    c = _case(3, HV=2)                                        # H == HV: no grouping for the comparison
    T, K = c["q"].shape[0], c["q"].shape[2]
    o, st = oracle.tree_gdn_verify(c["A_log"], c["dt_bias"], c["a"], c["b"], c["q"], c["k"], c["v"], c["state"],
                                   c["chain"], c["depth"], c["out_slot"], c["init_slot"], K ** -0.5)
    g = -c["A_log"].exp()[None, :] * F.softplus(c["a"] + c["dt_bias"][None, :])
    beta = torch.sigmoid(c["b"])
    init = c["state"][0].transpose(-1, -2)                    # [H, K, V]
    o2, st2 = oracle.tree_gdn_scan(c["q"], c["k"], c["v"], g, beta, c["parent"], c["depth"].long(), init)
    assert _rel(o, o2) < 1e-4
    assert _rel(st[1:].transpose(-1, -2), st2) < 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,codes", [(torch.float16, torch.float32), (torch.bfloat16, torch.bfloat16)])
def test_verify_kernel_matches_oracle(dtype, codes):
    from chain_flow_b200.gdn import gdn_verify
    c = _case(5)
    T, K = c["q"].shape[0], c["q"].shape[2]
    dev = "cuda"
    q, k, v = (c[n].to(dtype) for n in ("q", "k", "v"))
    A_log, dt_bias, a, b = (c[n].to(codes) for n in ("A_log", "dt_bias", "a", "b"))
    want_o, want_st = oracle.tree_gdn_verify(A_log, dt_bias, a, b, q, k, v, c["state"], c["chain"], c["depth"],
                                             c["out_slot"], c["init_slot"], K ** -0.5)
    st = c["state"].to(dev)
    o = torch.zeros(T, v.shape[1], v.shape[2], dtype=dtype, device=dev)
    gdn_verify(A_log.to(dev), dt_bias.to(dev), a.to(dev), b.to(dev), q.to(dev), k.to(dev), v.to(dev), o, st,
               c["chain"].to(dev), c["depth"].to(dev), c["out_slot"].to(dev), c["init_slot"].to(dev),
               scale=K ** -0.5)
    torch.cuda.synchronize()
    assert _rel(o.cpu(), want_o) < GDN_RTOL
    assert _rel(st.cpu(), want_st) < GDN_RTOL
    # a row subset, outputs only: the states stay as they are
    rows = torch.tensor([3, 7, 11], dtype=torch.int32)
    st2 = c["state"].to(dev)
    o2 = torch.zeros_like(o)
    gdn_verify(A_log.to(dev), dt_bias.to(dev), a.to(dev), b.to(dev), q.to(dev), k.to(dev), v.to(dev), o2, st2,
               c["chain"].to(dev), c["depth"].to(dev), c["out_slot"].to(dev), c["init_slot"].to(dev),
               rows.to(dev), scale=K ** -0.5, write_state=False)
    torch.cuda.synchronize()
    assert torch.equal(st2.cpu(), c["state"])
    assert _rel(o2.cpu()[rows.long()], want_o[rows.long()]) < GDN_RTOL


@pytest.mark.gpu
def test_verify_depth_past_the_chain_row_gives_nan():
    """A row whose depth does not fit its chain row (depth >= chain_stride, or < 0) walks nothing
    from memory: its output and state are NaN, and every other row still matches the oracle."""
    from chain_flow_b200.gdn import gdn_verify
    c = _case(11)
    T, K = c["q"].shape[0], c["q"].shape[2]
    want_o, want_st = oracle.tree_gdn_verify(c["A_log"], c["dt_bias"], c["a"], c["b"], c["q"], c["k"], c["v"],
                                             c["state"], c["chain"], c["depth"], c["out_slot"], c["init_slot"],
                                             K ** -0.5)
    depth = c["depth"].clone()
    bad = [4, 9]
    depth[4] = c["chain"].shape[1]          # one past the row
    depth[9] = -1
    dev = "cuda"
    st = c["state"].to(dev)
    o = torch.zeros(T, c["v"].shape[1], c["v"].shape[2], dtype=torch.float16, device=dev)
    gdn_verify(*(c[n].to(dev) for n in ("A_log", "dt_bias", "a", "b", "q", "k", "v")), o, st,
               c["chain"].to(dev), depth.to(dev), c["out_slot"].to(dev), c["init_slot"].to(dev), scale=K ** -0.5)
    torch.cuda.synchronize()
    o, st = o.float().cpu(), st.cpu()
    good = [t for t in range(T) if t not in bad]
    for t in bad:
        assert torch.isnan(o[t]).all()
        assert torch.isnan(st[int(c["out_slot"][t])]).all()
    assert _rel(o[good], want_o[good]) < GDN_RTOL
    good_slots = c["out_slot"][good].long()
    assert _rel(st[good_slots], want_st[good_slots]) < GDN_RTOL


def _batched_case(seed, S=2, N=20, H=2, HV=4, V=64, K=128, max_depth=5):
    """S requests of N rows each, request s's rows starting from state slot s (the shared root)."""
    from chain_flow_b200.gdn import ancestor_chains, make_tree
    g = torch.Generator().manual_seed(seed)
    chains, depths = [], []
    for s in range(S):
        par, _ = make_tree(N, max_depth, 4, seed + s)
        ch, dp = ancestor_chains(par, max_depth)
        chains.append(ch + s * N); depths.append(dp)
    T = S * N
    return dict(
        A_log=torch.randn(HV, generator=g) * 0.5, dt_bias=torch.randn(HV, generator=g) * 0.5,
        a=torch.randn(T, HV, generator=g), b=torch.randn(T, HV, generator=g),
        q=torch.randn(T, H, K, generator=g).half(), k=torch.randn(T, H, K, generator=g).half(),
        v=torch.randn(T, HV, V, generator=g).half(), state=torch.randn(S, HV, V, K, generator=g) * 0.1,
        chain=torch.cat(chains), depth=torch.cat(depths),
        init_slot=torch.arange(S, dtype=torch.int32).repeat_interleave(N),
        row_start=torch.arange(S, dtype=torch.int32) * N, row_count=torch.full((S,), N, dtype=torch.int32))


def test_ancestor_chains_walk_to_the_root():
    from chain_flow_b200.gdn import ancestor_chains, make_tree
    par, dep = make_tree(30, 6, 3, seed=9)
    chain, depth = ancestor_chains(par, 5)
    assert torch.equal(depth.long(), dep)
    for t in range(30):
        n = t
        for kk in range(int(depth[t]) + 1):
            assert int(chain[t, kk]) == n
            n = int(par[n])
        assert n == -1


def test_factor_oracle_equals_the_verify_oracle():
    """The factorised algebra is a different expression of the same outputs: pinned to the
    path-parallel verify oracle (itself pinned to the reference's tree_scan goldens)."""
    c = _batched_case(11)
    K = c["q"].shape[2]
    want, _ = oracle.tree_gdn_verify(c["A_log"], c["dt_bias"], c["a"], c["b"], c["q"], c["k"], c["v"], c["state"],
                                     c["chain"], c["depth"], torch.zeros_like(c["init_slot"]), c["init_slot"],
                                     K ** -0.5, write_state=False)
    got = oracle.tree_gdn_factor(c["A_log"], c["dt_bias"], c["a"], c["b"], c["q"], c["k"], c["v"], c["state"],
                                 c["chain"], c["depth"], c["init_slot"], c["row_start"], c["row_count"], K ** -0.5)
    assert _rel(got, want) < 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_factor_kernel_matches_the_verify_oracle(dtype):
    from chain_flow_b200.gdn import gdn_factor
    c = _batched_case(13, S=3, N=41, H=4, HV=8, V=128)
    K = c["q"].shape[2]
    dev = "cuda"
    q, k, v = (c[n].to(dtype) for n in ("q", "k", "v"))
    want, _ = oracle.tree_gdn_verify(c["A_log"], c["dt_bias"], c["a"], c["b"], q, k, v, c["state"], c["chain"],
                                     c["depth"], torch.zeros_like(c["init_slot"]), c["init_slot"], K ** -0.5,
                                     write_state=False)
    o = torch.zeros(q.shape[0], v.shape[1], v.shape[2], dtype=dtype, device=dev)
    gdn_factor(c["A_log"].to(dev), c["dt_bias"].to(dev), c["a"].to(dev), c["b"].to(dev), q.to(dev), k.to(dev),
               v.to(dev), o, c["state"].to(dev), c["chain"].to(dev), c["depth"].to(dev), c["init_slot"].to(dev),
               c["row_start"].to(dev), c["row_count"].to(dev), scale=K ** -0.5, n_max=41)
    torch.cuda.synchronize()
    assert _rel(o.cpu(), want) < GDN_RTOL, _rel(o.cpu(), want)
    # chains computed on the device (no host sync) give the same walk
    from chain_flow_b200.gdn import ancestor_chains, make_tree
    par, _ = make_tree(41, 5, 4, 13)
    ch_d, dp_d = ancestor_chains(par.cuda(), 5)
    ch_h, dp_h = ancestor_chains(par, 5)
    assert torch.equal(ch_d.cpu(), ch_h) and torch.equal(dp_d.cpu(), dp_h)
