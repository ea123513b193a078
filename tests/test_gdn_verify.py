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
