"""The bounded device waits, made to expire on purpose.

cfb_run.wait_budget_ns = 1 gives the waits that order a draft (the engine's grid barrier between
phases; the wide GEMMs' ring waits) a budget of 1 ns, so each gives up at its first poll that
finds it unfinished. The run must then end by itself with the plan's device error word set, leave
the context usable, and keep a failed plan failed (its next run touches no output) until it is
rebuilt; the rebuilt plan, in the same workspace, must reproduce an unforced run bit for bit.
Nothing here waits on a flag that is never set: the expiry comes from the budget alone, and the
waits that let a CTA wind down (copies in flight, issued MMAs) keep the 1 s default.

The reference's grid barrier has no such bound (src/chain_flow/csrc/fused_block.cu:91-106): a
schedule that cannot complete hangs the GPU there.
"""
import pytest
import torch

from conftest import load_golden

pytestmark = pytest.mark.gpu

DEV_TIMEOUT_GRID = 1


def _load(p, g, pred=None):
    p.ctx.copy_(g["ctx"].to(torch.float16))
    p.z0.copy_(g["z0"].to(torch.float16))
    p.known0.copy_(g["known0"])


def test_engine_grid_barrier_budget_expires_and_a_rebuilt_plan_runs_clean():
    from chain_flow_b200 import _lib
    from chain_flow_b200.engine import Plan
    from gpu_util import golden_weights
    g = load_golden("g64")
    w = golden_weights(g)
    ref = Plan(w, _lib.MODE_CHAIN, g["B"], width=4, depth=5)
    _load(ref, g)
    ref.run()
    torch.cuda.synchronize()
    ref.check()

    p = Plan(w, _lib.MODE_CHAIN, g["B"], width=4, depth=5, wait_ns=1)
    _load(p, g)
    p.run()
    torch.cuda.synchronize()
    assert p.device_error() == DEV_TIMEOUT_GRID
    with pytest.raises(_lib.CfbError):
        p.check()
    # a failed plan stays failed: its next run returns at once and leaves the outputs untouched
    p.tokens.fill_(-7)
    p.pred.fill_(3.0)
    p.run()
    torch.cuda.synchronize()
    assert bool((p.tokens == -7).all()) and bool((p.pred == 3.0).all())
    assert p.device_error() == DEV_TIMEOUT_GRID
    # the context is still usable, and the rebuilt plan reproduces the unforced run exactly
    p.rebuild(wait_ns=0)
    p.run()
    torch.cuda.synchronize()
    p.check()
    assert torch.equal(p.tokens, ref.tokens)
    assert torch.equal(p.pred, ref.pred)


def test_wide_gemm_ring_budget_expires_and_a_rebuilt_plan_runs_clean():
    """A wide (tcgen05) plan: its GEMMs' producer and MMA issuer give up their ring waits; the
    row kernels after a failed GEMM (LayerNorm, attention, path gather, beam) still run, and the
    gather and beam steps do nothing once the error word is set."""
    from chain_flow_b200 import _lib
    from chain_flow_b200.engine import WidePlan
    from chain_flow_b200.weights import DraftConfig, WideWeights
    g = load_golden("g128")
    cfg = DraftConfig(hidden=g["H"], num_heads=g["heads"], ffn_multiplier=g["FM"],
                      num_drafter_layers=g["L"], num_flow_steps=g["T"], markov_rank=g["rank"])
    w = WideWeights(g["W"], cfg, g["emb"], g["lm_w"], g["sl"], device="cuda")
    ref = WidePlan(w, _lib.MODE_CHAIN, g["B"], width=4, depth=5)
    _load(ref, g)
    ref.run()
    torch.cuda.synchronize()
    ref.check()

    p = WidePlan(w, _lib.MODE_CHAIN, g["B"], width=4, depth=5, wait_ns=1)
    _load(p, g)
    p.tokens.fill_(-7)
    p.run()
    torch.cuda.synchronize()
    assert p.device_error() != 0
    with pytest.raises(_lib.CfbError):
        p.check()
    assert bool((p.tokens == -7).all())           # no beam step ran after the failure
    p.rebuild(wait_ns=0)
    p.run()
    torch.cuda.synchronize()
    p.check()
    assert torch.equal(p.tokens, ref.tokens)
    assert torch.equal(p.pred, ref.pred)
