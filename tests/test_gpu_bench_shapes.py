"""GPU parity at the configurations bench.py measures, against the fp32 CPU oracle.

The drafters are the benchmark's own (chain_flow_b200.synthetic: seeded random-init weights with
the reference architecture, N(0, 1) hidden states), built through the reference-facing proposer
exactly as bench.py builds them:

* cfg 2, the 4B shape (D = 2560, FFN x6, 4 blocks, 8 Euler steps, R = 62,642 of 248,320): B = 1
  and B = 8 on the persistent engine, B = 32 on the wide (tcgen05) plan;
* cfg 3, the 27B shape (D = 5120): B = 1;
* the shipped 4B production drafter (VAE 2560 -> 640, 8 blocks, 2 steps, draft length 8): B = 1;
* the 27B production shape (VAE 5120 -> 1024, the same flow layout at 1024 wide): B = 1.

Checks, with the tolerances of BASELINE's north_star:

* integrated hidden states: max |engine - oracle| / max |oracle| <= 2e-2 over the whole draft. This
  norm-relative error is what "max relative error" is taken to mean. The element-wise relative
  error over entries with |oracle| > 1e-3 is measured too, but no fp16 implementation holds it to
  2e-2: an entry near zero is the difference of O(1) Euler increments, each carrying the fp16
  rounding of the GEMM inputs (2^-11 relative). So the element-wise figures (the max element-wise
  absolute error, and the share of entries beyond 2e-2 relative) are bounded by those of the
  reference algorithm's own eager fp16 GPU path on the same inputs (the oracle run in fp16 on the
  GPU, the reference's dtypes), with a factor of 2 of margin;
* the depth-1 shortlist head: each request's top-4 ids over all 62,642 rows, from the engine's own
  head input, bit-exact against log_softmax of the same input in fp32 (ties within 1e-4 allowed);
* chain tokens: bit-exact against the oracle's beam over the engine's own hidden states, or, where
  the fp16 head inputs flip a near-tie, a chain the oracle scores within 5e-3 of its best beam.

The oracle runs on the host cores (fp32 torch, all threads). It is test infrastructure only.
"""
import os

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

HIDDEN_RTOL = 2e-2
ELEM_MARGIN = 2.0


def hidden_errors(got, want):
    """(norm-relative max error, max element-wise absolute error, element-wise max relative error
    over |want| > 1e-3, share of those entries whose relative error exceeds HIDDEN_RTOL)."""
    got, want = got.float().cpu(), want.float().cpu()
    err = (got - want).abs()
    norm_rel = float(err.max() / want.abs().max())
    big = want.abs() > 1e-3
    rel = err[big] / want.abs()[big]
    return norm_rel, float(err.max()), float(rel.max()), float((rel > HIDDEN_RTOL).float().mean())


def check_hidden(got, want, ref16, what):
    """ref16: the reference algorithm's eager fp16 GPU result on the same inputs."""
    norm_rel, abs_err, elem_rel, share = hidden_errors(got, want)
    r_norm, r_abs, r_elem, r_share = hidden_errors(ref16, want)
    print(f"{what}: engine norm-relative {norm_rel:.3e}, max abs {abs_err:.3e}, element-wise max rel "
          f"{elem_rel:.3e}, share beyond {HIDDEN_RTOL} {share:.2e} | reference eager fp16: norm-relative "
          f"{r_norm:.3e}, max abs {r_abs:.3e}, element-wise max rel {r_elem:.3e}, share {r_share:.2e}")
    assert norm_rel <= HIDDEN_RTOL, (what, norm_rel)
    assert abs_err <= ELEM_MARGIN * r_abs, (what, abs_err, r_abs)
    assert share <= ELEM_MARGIN * r_share + 1e-4, (what, share, r_share)


class Bench:
    """A benchmark drafter on the GPU (through FlowDrafterProposer) and its fp32 host copy."""

    def __init__(self, name):
        from chain_flow_b200.proposer import FlowDrafterProposer
        from chain_flow_b200.synthetic import WORKLOADS, make_state
        torch.set_num_threads(os.cpu_count() or 1)
        self.wl = wl = WORKLOADS[name]
        sd, emb, lm, sl = make_state(wl, seed=0, device="cuda")
        self.prop = FlowDrafterProposer.from_components(sd, wl.model_args(), emb, lm, sl, width=wl.width,
                                                        K=wl.draft_tokens, device="cuda", seed=1000)
        self.W = {k: v.float().cpu() for k, v in sd.items()}
        self.sd16 = sd                          # the reference's eager fp16 path runs on these
        self.emb = emb.float().cpu()
        self.sl = sl
        self.hw = lm[sl.cuda()].float().cpu()
        self.w2 = self.W["markov.w2.weight"][sl]
        del lm
        torch.cuda.empty_cache()
        self.cfg = oracle.FlowConfig(hidden=wl.flow_width, draft_length=wl.draft_length, chunk_size=wl.chunk,
                                     ffn_multiplier=wl.ffn, num_layers=wl.layers, num_flow_steps=wl.steps,
                                     path_order=wl.path_order, markov_rank=wl.markov_rank)

    def inputs(self, B, seed=1):
        from chain_flow_b200.synthetic import make_inputs
        return make_inputs(self.wl, B, seed=seed, device="cuda")

    def oracle_pred(self, ctx, z0, fp16_gpu=False):
        """The oracle's integrated hidden states: fp32 on the host, or (fp16_gpu) the reference's own
        eager fp16 path on the GPU."""
        W = self.sd16 if fp16_gpu else self.W
        if fp16_gpu:
            c, z = ctx.half().cuda(), z0.half().cuda()
        else:
            c, z = ctx.float().cpu(), z0.float().cpu()
        with torch.inference_mode():
            if self.wl.latent:
                return oracle.predict_hidden_vae(W, self.cfg, self.wl.vae_layers, self.wl.vae_heads, c, z)
            return oracle.integrate(W, self.cfg, c, z)

    def draft(self, B, seed=1):
        """One chain draft of B requests through the proposer: (plan, tokens, ctx, known0)."""
        from chain_flow_b200 import _lib
        from chain_flow_b200.proposer import MAX_PLAN_BATCH
        ctx, known0 = self.inputs(B, seed)
        tokens = self.prop._beam_chains(ctx, known0).cpu()
        key = (_lib.MODE_CHAIN, B) if B <= MAX_PLAN_BATCH else ("wide", _lib.MODE_CHAIN, B)
        plan = self.prop._plans[key]
        torch.cuda.synchronize()
        plan.check()
        return plan, tokens, ctx, known0

    def check_draft(self, B, what, seed=1):
        from beam_check import check_chain
        plan, tokens, ctx, known0 = self.draft(B, seed)
        want = self.oracle_pred(ctx, plan.z0)
        check_hidden(plan.pred, want, self.oracle_pred(ctx, plan.z0, fp16_gpu=True), f"{what} hidden states")
        exact = check_chain(tokens, self.W, self.cfg_head(), self.emb, self.hw, self.w2, self.sl,
                            plan.pred.cpu(), known0.cpu(), self.wl.width, self.wl.draft_tokens)
        print(f"{what}: {exact}/{B} chains bit-exact, the rest tie-explained")
        return plan

    def cfg_head(self):
        """The oracle config of the beam (the path head lives at the hidden width)."""
        return oracle.FlowConfig(hidden=self.wl.hidden, draft_length=self.wl.draft_length, chunk_size=self.wl.chunk,
                                 ffn_multiplier=self.wl.ffn, num_layers=self.wl.layers,
                                 num_flow_steps=self.wl.steps, path_order=self.wl.path_order,
                                 markov_rank=self.wl.markov_rank)

    def check_head_depth1(self, plan, what):
        """Depth-1 top-W ids of every request from the engine's own head input row."""
        from chain_flow_b200 import _lib
        from chain_flow_b200.engine import Plan, untile
        wl, w = self.wl, self.prop.weights
        B = plan.batch
        p = Plan(w, _lib.MODE_BEAM_CHAIN, B, width=wl.width, depth=1)
        p.pred.copy_(plan.pred)
        p.known0.copy_(plan.known0)
        p.run()
        torch.cuda.synchronize()
        p.check()
        rows = B * wl.width
        kh = wl.hidden + wl.markov_rank
        kp = (kh + 127) // 128 * 128
        xin = untile(p.buffer(_lib.BUF_HEAD_IN, torch.float16, (rows * kp,)), rows, kh).float().cpu()
        lastp = p.buffer(_lib.BUF_LASTP, torch.int64, (rows, wl.path_order)).cpu()
        full = torch.cat([self.hw, self.w2], dim=1)
        for b in range(B):
            lp = torch.log_softmax(xin[b * wl.width] @ full.T, dim=-1)
            v, i = lp.topk(wl.width)
            got = lastp[b * wl.width:(b + 1) * wl.width, 0]
            if torch.equal(got, self.sl[i]):
                continue
            # only a tie within the fp32 summation order may reorder the list
            loc = torch.searchsorted(self.sl, got)
            assert bool((self.sl[loc] == got).all()), (what, b, got)
            assert float((lp[loc] - v).abs().max()) < 1e-4, (what, b, got.tolist(), self.sl[i].tolist())
        print(f"{what}: depth-1 top-{wl.width} ids over {self.sl.numel()} rows match")


@pytest.fixture(scope="module")
def cfg2():
    return Bench("4b")


def test_cfg2_4b_b1_draft(cfg2):
    plan = cfg2.check_draft(1, "cfg2 4B b=1")
    cfg2.check_head_depth1(plan, "cfg2 4B b=1")


def test_cfg2_4b_b8_draft(cfg2):
    plan = cfg2.check_draft(8, "cfg2 4B b=8", seed=2)
    cfg2.check_head_depth1(plan, "cfg2 4B b=8")


def test_cfg5_4b_b32_wide_draft(cfg2):
    cfg2.check_draft(32, "cfg5 4B b=32 (wide plan)", seed=3)


def test_4b_production_vae_b1_draft():
    Bench("4b-prod").check_draft(1, "4B production (VAE) b=1")


def test_27b_production_vae_b1_draft():
    Bench("27b-prod").check_draft(1, "27B production (VAE, flow at 1024) b=1")


def test_cfg3_27b_b1_draft():
    Bench("27b").check_draft(1, "cfg3 27B b=1")
