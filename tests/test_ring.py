"""The context ring (reference FlowDrafterProposer._ring_write / _ring_gather,
flow_proposer.py:916-961): the CPU oracle against the reference's own outputs (golden vectors
from tests/golden/make_ring_golden.py), and the CUDA kernels against the same vectors, bit-exact
(the ring only moves fp16 rows)."""
import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN


def _steps():
    z = np.load(GOLDEN / "ring.npz")
    R, C, H, K, S = (int(x) for x in z["dims"])
    steps = []
    for s in range(S):
        path = z[f"s{s}_path"]
        steps.append(dict(rows=torch.from_numpy(z[f"s{s}_rows"]), sh=torch.from_numpy(z[f"s{s}_sh"]),
                          starts=torch.from_numpy(z[f"s{s}_starts"]), cnt=torch.from_numpy(z[f"s{s}_cnt"]),
                          wmask=torch.from_numpy(z[f"s{s}_wmask"]),
                          path=torch.from_numpy(path) if path.size else None,
                          ring=torch.from_numpy(z[f"s{s}_ring"]), rpos=torch.from_numpy(z[f"s{s}_rpos"]),
                          nval=torch.from_numpy(z[f"s{s}_nval"]), grows=torch.from_numpy(z[f"s{s}_grows"]),
                          ctx=torch.from_numpy(z[f"s{s}_ctx"])))
    return R, C, H, K, steps


def test_ring_oracle_matches_reference():
    R, C, H, K, steps = _steps()
    ring = torch.zeros(R, C + 1, H, dtype=torch.float16)
    rpos = torch.zeros(R, dtype=torch.long)
    nval = torch.zeros(R, dtype=torch.long)
    for st in steps:
        oracle.ring_write(ring, rpos, nval, st["sh"], st["rows"], st["starts"], st["cnt"], st["wmask"],
                          st["path"], K)
        assert torch.equal(ring[:, :C], st["ring"])
        assert torch.equal(rpos, st["rpos"]) and torch.equal(nval, st["nval"])
        assert torch.equal(oracle.ring_gather(ring, rpos, nval, st["grows"]), st["ctx"])


@pytest.mark.gpu
def test_ring_kernels_match_reference():
    from chain_flow_b200.ring import ContextRing
    R, C, H, K, steps = _steps()
    ring = ContextRing(R, C, H, device="cuda")
    for st in steps:
        ring.write(st["sh"].cuda(), st["rows"].cuda(), st["starts"].cuda(), st["cnt"].cuda(), st["wmask"].cuda(),
                   None if st["path"] is None else st["path"].cuda(), K)
        torch.cuda.synchronize()
        assert torch.equal(ring.ring[:, :C].cpu(), st["ring"])
        assert torch.equal(ring.rpos.cpu(), st["rpos"]) and torch.equal(ring.nval.cpu(), st["nval"])
        assert torch.equal(ring.gather(st["grows"].cuda()).cpu(), st["ctx"])


@pytest.mark.gpu
def test_proposer_drafts_from_the_ring():
    """The proposer's ring methods (reference names and arguments) feed its draft: a window
    gathered from the ring drafts the same tokens as the same window passed directly."""
    from chain_flow_b200.proposer import FlowDrafterProposer
    from conftest import load_golden
    g = load_golden("g64")
    margs = dict(context_size=8, draft_length=6, chunk_size=3, num_heads=g["heads"], ffn_multiplier=g["FM"],
                 num_drafter_layers=g["L"], num_flow_steps=g["T"], path_order=4, path_ffn_multiplier=2,
                 markov_rank=g["rank"], init_mode="delta", noise_scale=1.0)
    p = FlowDrafterProposer.from_components(g["W"], margs, g["emb"], g["lm_w"], g["sl"], width=4, K=5,
                                            device="cuda", max_reqs=4)
    p._init_ring(g["H"])
    B = g["B"]
    ctx = g["ctx"].half().cuda()                               # [B, 8, H]
    rows = torch.arange(B, device="cuda") + 1                  # slots 1.. of 4
    # two chain steps of 5 then 3 new rows per request fill the 8-row window (the second write
    # wraps the slot's write position back to 0)
    for lo, n in ((0, 5), (5, 3)):
        sh = ctx[:, lo:lo + n].reshape(B * n, -1).contiguous()
        starts = torch.arange(B, device="cuda") * n
        p._ring_write(sh, rows, starts, torch.full((B,), n, device="cuda"), torch.ones(B, dtype=torch.bool,
                      device="cuda"), None, 6)
    got = p._ring_gather(rows)
    assert torch.equal(got, ctx)
    k0 = g["known0"].cuda()
    assert torch.equal(p._draft_from_ring(rows, k0), p._beam_chains(ctx, k0))
