"""The two-pass candidate head (reference CF_TWOPASS_M, shared candidate set,
flow_proposer.py:1142-1184): the oracle against the reference's own outputs
(tests/golden/make_twopass_golden.py), and the engine against the oracle."""
import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN, golden_flow_config, load_golden

CASES = [("g64", 64), ("g64", 128), ("g128", 64), ("g128", 256)]


def _gtp():
    z = np.load(GOLDEN / "gtp.npz")
    return {k: torch.from_numpy(z[k]) for k in z.files}


@pytest.mark.parametrize("name,M", CASES)
def test_twopass_oracle_matches_reference(name, M):
    g, t = load_golden(name), _gtp()
    W, sl = g["W"], g["sl"]
    assert torch.equal(t[f"{name}.pred"], g["pred"])          # the same drafter and inputs
    hw, w2 = g["lm_w"][sl], W["markov.w2.weight"][sl]
    cand = oracle.twopass_candidates(hw, g["pred"], 1, 6, M)
    assert torch.equal(cand, t[f"{name}.m{M}.cand"])
    cfg = golden_flow_config(g)
    ch = oracle.beam_chains(W, cfg, g["emb"], hw, w2, sl, g["pred"], g["known0"], 4, 5, twopass_m=M)
    assert torch.equal(ch, t[f"{name}.m{M}.chains"])
    tr = oracle.beam_tree(W, cfg, g["emb"], hw, w2, sl, g["pred"], g["known0"], 4, 4, 5, twopass_m=M)
    assert torch.equal(tr, t[f"{name}.m{M}.tree"])


def _scores(hw, pred, lo, hi):
    """pass A's per-row best log-prob over the depths (the selection key), fp16 hiddens"""
    B, n = pred.shape[0], hi - lo
    lg = (pred[:, lo:hi].reshape(B * n, -1).half().float() @ hw.T).view(B, n, -1)
    return torch.log_softmax(lg, dim=-1).amax(dim=1)


def _check_set(cand, want, sc, M):
    """Equal candidate sets, or differences only between rows whose keys tie at the threshold
    within the fp32 rounding of the GPU's GEMM."""
    for b in range(cand.shape[0]):
        got, ref = set(cand[b].tolist()), set(want[b].tolist())
        if got == ref:
            continue
        thr = sc[b].topk(M).values[-1]
        for r in got ^ ref:
            assert abs(float(sc[b, r] - thr)) < 1e-4, (b, r, float(sc[b, r]), float(thr))


def _check_chain(tokens, W, cfg, g, hw, w2, sl, pred, cand, tol=5e-3):
    """Chain drafts equal to the oracle's on the same candidate set, or, where they differ, the
    engine's path is one of the oracle's final beams whose cumulative log-prob ties the best
    within tol (the engine's fp16 head inputs against the oracle's fp32)."""
    best, beams, cum = oracle.beam_chains(W, cfg, g["emb"], hw, w2, sl, pred, g["known0"], 4, 5, cand=cand,
                                          return_beams=True)
    for b in range(tokens.shape[0]):
        if torch.equal(tokens[b], best[b]):
            continue
        hit = [w for w in range(beams.shape[1]) if torch.equal(beams[b, w], tokens[b])]
        assert hit, (b, tokens[b], best[b])
        assert float(cum[b].max() - cum[b, hit[0]]) < tol, (b, cum[b].tolist(), hit)


@pytest.mark.gpu
@pytest.mark.parametrize("name,M", CASES)
def test_gpu_twopass_engine(name, M):
    """The engine's two-pass head: candidate sets equal to the reference's, chain and tree drafts
    equal to the reference's (on the reference's own hiddens and end to end from the flow)."""
    from chain_flow_b200 import _lib
    from gpu_util import golden_weights, run_plan
    g, t = load_golden(name), _gtp()
    W, sl, B = g["W"], g["sl"], g["B"]
    hw, w2 = g["lm_w"][sl], W["markov.w2.weight"][sl]
    cfg = golden_flow_config(g)
    w = golden_weights(g)
    sc = _scores(hw, g["pred"], 1, 6)
    p = run_plan(w, _lib.MODE_BEAM_CHAIN, B, known0=g["known0"], pred=g["pred"], width=4, depth=5, twopass_m=M)
    cand = p.candidates().long().cpu()
    assert bool((cand[:, 1:] > cand[:, :-1]).all())               # ascending shortlist rows
    _check_set(cand, t[f"{name}.m{M}.cand"], sc, M)
    _check_chain(p.tokens.cpu(), W, cfg, g, hw, w2, sl, g["pred"], cand)
    p = run_plan(w, _lib.MODE_BEAM_TREE, B, known0=g["known0"], pred=g["pred"], depth=5, tree_keep=4,
                 tree_topb=4, twopass_m=M)
    cand = p.candidates().long().cpu()
    want = oracle.beam_tree(W, cfg, g["emb"], hw, w2, sl, g["pred"], g["known0"], 4, 4, 5, cand=cand)
    if not torch.equal(p.tokens.cpu(), want):
        # only where candidates tie within the engine's fp16 head inputs
        from beam_check import check_tree
        check_tree(p.tokens.cpu(), W, cfg, g["emb"], hw, w2, sl, g["pred"], g["known0"], 4, 4, 5, tp_cand=cand)
    # end to end: flow, then the two-pass beam
    p = run_plan(w, _lib.MODE_CHAIN, B, ctx=g["ctx"], z0=g["z0"], known0=g["known0"], width=4, depth=5, twopass_m=M)
    pred = p.pred.cpu()
    _check_chain(p.tokens.cpu(), W, cfg, g, hw, w2, sl, pred, p.candidates().long().cpu())
    assert p.device_error() == 0


@pytest.mark.parametrize("name", ["g64", "g128"])
def test_twopass_over_the_whole_shortlist_is_the_one_pass_head(name):
    """With every shortlist row a candidate, pass B is the full head: the two-pass oracle's
    chains and trees equal the one-pass oracle's."""
    g = load_golden(name)
    W, sl = g["W"], g["sl"]
    hw, w2 = g["lm_w"][sl], W["markov.w2.weight"][sl]
    R = hw.shape[0]
    cfg = golden_flow_config(g)
    one = oracle.beam_chains(W, cfg, g["emb"], hw, w2, sl, g["pred"], g["known0"], 4, 5)
    two = oracle.beam_chains(W, cfg, g["emb"], hw, w2, sl, g["pred"], g["known0"], 4, 5, twopass_m=R)
    assert torch.equal(one, two)
    one_t = oracle.beam_tree(W, cfg, g["emb"], hw, w2, sl, g["pred"], g["known0"], 4, 4, 5)
    two_t = oracle.beam_tree(W, cfg, g["emb"], hw, w2, sl, g["pred"], g["known0"], 4, 4, 5, twopass_m=R)
    assert torch.equal(one_t, two_t)


@pytest.mark.gpu
def test_gpu_twopass_engine_eight_requests():
    """The two-pass head in a plan of 8 requests (the wide-row engine build, whose head epilogue
    runs on the epilogue and worker warps together): g64's two requests repeated four times must
    give each copy the reference's candidate set and a chain the oracle accepts."""
    from chain_flow_b200 import _lib
    from gpu_util import golden_weights, run_plan
    g, t = load_golden("g64"), _gtp()
    M, rep = 64, 4
    W, sl, B0 = g["W"], g["sl"], g["B"]
    hw, w2 = g["lm_w"][sl], W["markov.w2.weight"][sl]
    cfg = golden_flow_config(g)
    w = golden_weights(g)
    g8 = dict(g)
    g8["pred"] = g["pred"].repeat(rep, 1, 1)
    g8["known0"] = g["known0"].repeat(rep)
    B = B0 * rep
    p = run_plan(w, _lib.MODE_BEAM_CHAIN, B, known0=g8["known0"], pred=g8["pred"], width=4, depth=5, twopass_m=M)
    cand = p.candidates().long().cpu()
    assert bool((cand[:, 1:] > cand[:, :-1]).all())
    _check_set(cand, t[f"g64.m{M}.cand"].repeat(rep, 1), _scores(hw, g8["pred"], 1, 6), M)
    _check_chain(p.tokens.cpu(), W, cfg, g8, hw, w2, sl, g8["pred"], cand)
    assert p.device_error() == 0
