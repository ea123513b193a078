"""Pin the CPU oracle against golden vectors produced by the reference implementation itself
(tests/golden/make_golden.py ran the reference's TreeFlowDrafter, FlowDrafterProposer beam and
tree_scan in the build container)."""
import torch

import oracle
from conftest import golden_flow_config


def test_oracle_integrate_matches_reference(golden):
    g = golden
    cfg = golden_flow_config(g)
    pred = oracle.integrate(g["W"], cfg, g["ctx"], g["z0"])
    ref = g["pred"]
    err = (pred - ref).abs().max() / ref.abs().max()
    assert err < 1e-5, err


def test_oracle_path_residual_matches_reference(golden):
    g = golden
    res = oracle.path_residual(g["W"], g["emb"], g["probe_lastp"], 4, None)
    assert torch.allclose(res, g["probe_res"], atol=1e-5, rtol=1e-5)
    res2 = oracle.path_residual(g["W"], g["emb"], g["probe_lastp"], 4, 2)
    assert torch.allclose(res2, g["probe_res2"], atol=1e-5, rtol=1e-5)


def test_oracle_beam_chains_matches_reference(golden):
    g = golden
    cfg = golden_flow_config(g)
    sl = g["sl"]
    hw = g["lm_w"][sl]
    w2 = g["W"]["markov.w2.weight"][sl]
    ch = oracle.beam_chains(g["W"], cfg, g["emb"], hw, w2, sl, g["pred"], g["known0"], 4, 5)
    assert torch.equal(ch, g["chains"])


def test_oracle_beam_tree_matches_reference(golden):
    g = golden
    cfg = golden_flow_config(g)
    sl = g["sl"]
    hw = g["lm_w"][sl]
    w2 = g["W"]["markov.w2.weight"][sl]
    tr = oracle.beam_tree(g["W"], cfg, g["emb"], hw, w2, sl, g["pred"], g["known0"], 4, 4, 5)
    assert torch.equal(tr, g["tree"])


def test_oracle_tree_gdn_matches_reference(golden):
    g = golden
    o, st = oracle.tree_gdn_scan(g["gdn_q"], g["gdn_k"], g["gdn_v"], g["gdn_g"], g["gdn_beta"],
                                 g["gdn_parent"], g["gdn_depth"], g["gdn_init"])
    assert torch.allclose(o, g["gdn_o"], atol=1e-5, rtol=1e-5)
    assert torch.allclose(st, g["gdn_states"], atol=1e-5, rtol=1e-5)


def test_tree_gdn_depth_scan_equals_per_path_recurrence(golden):
    """The depth-batched scan equals the sequential recurrence along each root..node path
    (the reference's own validation, kernels/tree_scan.py:83-96)."""
    g = golden
    o, _ = oracle.tree_gdn_scan(g["gdn_q"], g["gdn_k"], g["gdn_v"], g["gdn_g"], g["gdn_beta"],
                                g["gdn_parent"], g["gdn_depth"], g["gdn_init"])
    parent = g["gdn_parent"].tolist()
    for n in range(len(parent)):
        path, m = [], n
        while m != -1:
            path.append(m)
            m = parent[m]
        path.reverse()
        on = oracle.path_gdn_output(g["gdn_q"], g["gdn_k"], g["gdn_v"], g["gdn_g"],
                                    g["gdn_beta"], path, g["gdn_init"])
        assert torch.allclose(on, o[n], atol=1e-5, rtol=1e-4)
