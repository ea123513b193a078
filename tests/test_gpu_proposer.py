"""GPU tests of the reference-facing surface (FlowDrafterProposer) and of plan properties the
parity tests do not cover: the 'delta' initial latents (reference tree_flow.py:150-161), a plan
replayed from a CUDA graph, and a plan cut for a smaller grid (different tile split, same
results within the hidden-state tolerance)."""
import pytest
import torch

import oracle
from conftest import golden_flow_config, load_golden

pytestmark = pytest.mark.gpu

HIDDEN_RTOL = 2e-2


def _rel(a, b):
    return float((a.float().cpu() - b.float().cpu()).abs().max() / b.float().abs().max().clamp_min(1e-12))


def _model_args(g, init_mode):
    return dict(context_size=8, draft_length=6, chunk_size=3, num_heads=g["heads"], ffn_multiplier=g["FM"],
                num_drafter_layers=g["L"], num_flow_steps=g["T"], path_order=4, path_ffn_multiplier=2,
                markov_rank=g["rank"], init_mode=init_mode, noise_scale=1.0)


def _delta_z0(ctx, k=6):
    """reference TreeFlowDrafter.init_latents, init_mode='delta'"""
    last = ctx[:, -1:, :]
    delta = ctx[:, -1:, :] - ctx[:, -2:-1, :]
    steps = torch.arange(1, k + 1, dtype=ctx.dtype).view(1, k, 1)
    return last + steps * delta


@pytest.fixture(scope="module", params=["g64", "g128"])
def prop(request):
    from chain_flow_b200.proposer import FlowDrafterProposer
    g = load_golden(request.param)
    p = FlowDrafterProposer.from_components(g["W"], _model_args(g, "delta"), g["emb"], g["lm_w"], g["sl"],
                                            width=4, K=5, tree_keep=4, tree_topb=4, tree_depth=5,
                                            device="cuda")
    return g, p


def test_proposer_delta_latents_match_oracle(prop):
    g, p = prop
    ctx = g["ctx"].half().float()
    want = oracle.integrate(g["W"], golden_flow_config(g), ctx, _delta_z0(ctx).half().float())
    got = p.predict_hidden(g["ctx"].cuda().half())
    assert _rel(got, want) < HIDDEN_RTOL, _rel(got, want)


def test_proposer_beam_chains_and_tree(prop):
    g, p = prop
    sl = g["sl"]
    cfg = golden_flow_config(g)
    ctx = g["ctx"].cuda().half()
    known0 = g["known0"].cuda()
    ch = p._beam_chains(ctx, known0).cpu()
    pred = p._plans[(1, g["B"])].pred.cpu()
    want = oracle.beam_chains(g["W"], cfg, g["emb"], g["lm_w"][sl], g["W"]["markov.w2.weight"][sl], sl,
                              pred, g["known0"], 4, 5)
    assert torch.equal(ch, want), (ch, want)
    tr = p._beam_tree(ctx, known0).cpu()
    pred = p._plans[(2, g["B"])].pred.cpu()
    want = oracle.beam_tree(g["W"], cfg, g["emb"], g["lm_w"][sl], g["W"]["markov.w2.weight"][sl], sl,
                            pred, g["known0"], 4, 4, 5)
    if not torch.equal(tr, want):
        # only where candidates tie within the engine's fp16 head inputs
        from beam_check import check_tree
        check_tree(tr, g["W"], cfg, g["emb"], g["lm_w"][sl], g["W"]["markov.w2.weight"][sl], sl, pred,
                   g["known0"], 4, 4, 5)
    assert p.device_error() == 0


def test_propose_returns_lists(prop):
    g, p = prop
    out = p.propose([[1, int(t)] for t in g["known0"]], context_hidden=g["ctx"].cuda().half())
    assert isinstance(out, list) and len(out) == g["B"] and all(len(r) == 5 for r in out)


def test_plan_replays_from_a_cuda_graph():
    from chain_flow_b200 import _lib
    from gpu_util import golden_weights, run_plan
    g = load_golden("g64")
    w = golden_weights(g)
    p = run_plan(w, _lib.MODE_CHAIN, g["B"], ctx=g["ctx"], z0=g["z0"], known0=g["known0"], width=4, depth=5)
    eager_tokens, eager_pred = p.tokens.clone(), p.pred.clone()
    p.tokens.zero_(); p.pred.zero_()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        p.run()
    for _ in range(2):
        p.tokens.zero_()
        graph.replay()
        torch.cuda.synchronize()
        p.check()
        assert torch.equal(p.tokens, eager_tokens)
        assert torch.equal(p.pred, eager_pred)
    del graph


@pytest.mark.parametrize("grid", [7, 40])
def test_smaller_grid_gives_the_same_draft(grid):
    """A plan cut for fewer CTAs splits tiles differently (more stream-K fixups): the hiddens stay
    within tolerance of the reference and the tokens equal the oracle beam over them."""
    from chain_flow_b200 import _lib
    from gpu_util import golden_weights, run_plan
    g = load_golden("g128")
    w = golden_weights(g)
    p = run_plan(w, _lib.MODE_CHAIN, g["B"], ctx=g["ctx"], z0=g["z0"], known0=g["known0"], width=4, depth=5,
                 grid=grid)
    assert p.grid == grid
    assert _rel(p.pred, g["pred"]) < HIDDEN_RTOL
    sl = g["sl"]
    want = oracle.beam_chains(g["W"], golden_flow_config(g), g["emb"], g["lm_w"][sl], g["W"]["markov.w2.weight"][sl],
                              sl, p.pred.cpu(), g["known0"], 4, 5)
    assert torch.equal(p.tokens.cpu(), want)


def test_batch8_flow_and_chain_match_oracle():
    """B = 8 requests: 64 context rows in the cross K/V projection (the split-n-tile MMA path)
    and 48-row expert jobs; seeded random weights with the reference's names and shapes."""
    from chain_flow_b200 import _lib
    from chain_flow_b200.weights import DraftConfig, DrafterWeights
    from gpu_util import random_state_dict, run_plan
    D, V, R, B = 256, 2000, 512, 8
    cfg = DraftConfig(hidden=D, num_heads=8, ffn_multiplier=2, num_drafter_layers=2, num_flow_steps=2,
                      markov_rank=32)
    sd = random_state_dict(cfg, V, seed=5)
    g = torch.Generator().manual_seed(6)
    emb = (torch.randn(V, D, generator=g) * 0.5).half().float()
    lm = (torch.randn(V, D, generator=g) * 0.02).half().float()
    sl = torch.randperm(V, generator=g)[:R].sort().values
    w = DrafterWeights(sd, cfg, emb, lm, sl, device="cuda")
    ctx = torch.randn(B, 8, D, generator=g).half()
    z0 = torch.randn(B, 6, D, generator=g).half()
    known0 = torch.randint(0, V, (B,), generator=g)
    p = run_plan(w, _lib.MODE_CHAIN, B, ctx=ctx, z0=z0, known0=known0, width=4, depth=5)
    ocfg = oracle.FlowConfig(hidden=D, num_heads=8, ffn_multiplier=2, num_layers=2, num_flow_steps=2,
                             markov_rank=32)
    want = oracle.integrate(sd, ocfg, ctx.float(), z0.float())
    assert _rel(p.pred, want) < HIDDEN_RTOL, _rel(p.pred, want)
    ch = oracle.beam_chains(sd, ocfg, emb, lm[sl], sd["markov.w2.weight"][sl], sl, p.pred.cpu(), known0, 4, 5)
    assert torch.equal(p.tokens.cpu(), ch), (p.tokens.cpu(), ch)
    # the tree draft of the same batch (the wide-row build's head epilogue in tree mode)
    t = run_plan(w, _lib.MODE_TREE, B, ctx=ctx, z0=z0, known0=known0, depth=5, tree_keep=4, tree_topb=4)
    tr = oracle.beam_tree(sd, ocfg, emb, lm[sl], sd["markov.w2.weight"][sl], sl, t.pred.cpu(), known0, 4, 4, 5)
    if not torch.equal(t.tokens.cpu(), tr):
        from beam_check import check_tree
        check_tree(t.tokens.cpu(), sd, ocfg, emb, lm[sl], sd["markov.w2.weight"][sl], sl, t.pred.cpu(), known0,
                   4, 4, 5)


def test_batches_above_one_engine_plan_run_on_the_wide_plan():
    """B = 11 > MAX_PLAN_BATCH: the proposer drafts the whole batch with one wide plan (tcgen05
    GEMMs). The hiddens stay within tolerance of the oracle, and the chain and tree drafts are the
    oracle beam over the wide plan's own hiddens."""
    from chain_flow_b200 import _lib
    from chain_flow_b200.proposer import MAX_PLAN_BATCH, FlowDrafterProposer
    from chain_flow_b200.weights import DraftConfig
    from gpu_util import random_state_dict
    D, V, R, B = 256, 2000, 512, MAX_PLAN_BATCH + 3
    margs = dict(context_size=8, draft_length=6, chunk_size=3, num_heads=8, ffn_multiplier=2,
                 num_drafter_layers=2, num_flow_steps=2, path_order=4, path_ffn_multiplier=2, markov_rank=32,
                 init_mode="delta", noise_scale=1.0)
    cfg = DraftConfig.from_model_args(margs, D)
    sd = random_state_dict(cfg, V, seed=7)
    g = torch.Generator().manual_seed(8)
    emb = (torch.randn(V, D, generator=g) * 0.5).half().float()
    lm = (torch.randn(V, D, generator=g) * 0.02).half().float()
    sl = torch.randperm(V, generator=g)[:R].sort().values
    p = FlowDrafterProposer.from_components(sd, margs, emb, lm, sl, width=4, K=5, tree_keep=4, tree_topb=4,
                                            tree_depth=5, device="cuda")
    ctx = torch.randn(B, 8, D, generator=g).half().cuda()
    known0 = torch.randint(0, V, (B,), generator=g).cuda()
    pred = p.predict_hidden(ctx).clone()
    assert pred.shape[0] == B and ("wide", _lib.MODE_FLOW, B) in p._plans
    ocfg = oracle.FlowConfig(hidden=D, num_heads=8, ffn_multiplier=2, num_layers=2, num_flow_steps=2,
                             markov_rank=32)
    c = ctx.float().cpu()
    want = oracle.integrate(sd, ocfg, c, _delta_z0(c).half().float())
    assert _rel(pred, want) < HIDDEN_RTOL, _rel(pred, want)
    hw, w2 = lm[sl], sd["markov.w2.weight"][sl]
    ch = p._beam_chains(ctx, known0).cpu()
    cp = p._plans[("wide", _lib.MODE_CHAIN, B)].pred.cpu()
    assert torch.equal(ch, oracle.beam_chains(sd, ocfg, emb, hw, w2, sl, cp, known0.cpu(), 4, 5))
    tr = p._beam_tree(ctx, known0).cpu()
    tp = p._plans[("wide", _lib.MODE_TREE, B)].pred.cpu()
    want_tr = oracle.beam_tree(sd, ocfg, emb, hw, w2, sl, tp, known0.cpu(), 4, 4, 5)
    if not torch.equal(tr, want_tr):
        from beam_check import check_tree
        check_tree(tr, sd, ocfg, emb, hw, w2, sl, tp, known0.cpu(), 4, 4, 5)
    assert p.device_error() == 0


def test_phase_table_marks_one_head_phase_per_depth():
    """CFB_BUF_PHASES: a chain plan of depth K has K shortlist-head GEMM phases (post-op: lists
    published), each followed by the beam phase of its depth."""
    from chain_flow_b200 import _lib
    from gpu_util import golden_weights, run_plan
    g = load_golden("g64")
    p = run_plan(golden_weights(g), _lib.MODE_CHAIN, g["B"], ctx=g["ctx"], z0=g["z0"], known0=g["known0"],
                 width=4, depth=5)
    t = p.phase_table()
    heads = [i for i in range(t.shape[0]) if int(t[i, 0]) == _lib.PK_GEMM and int(t[i, 6]) == _lib.PO_PUBLISH]
    assert len(heads) == 5
    assert all(int(t[i + 1, 0]) == _lib.PK_BEAM for i in heads)
