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
