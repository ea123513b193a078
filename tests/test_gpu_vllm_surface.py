"""GPU tests of FlowDrafterProposer as vLLM drives it (reference
src/chain_flow/vllm_plugin/flow_proposer.py:329-2569): built from a vllm_config and a drafter
directory, lazily from the target model the runner hook stashed, then fed step by step through
propose() with the hidden states a runner hands over.

The expected drafts are the proposer's own _beam_chains / _beam_tree over context windows kept
here on the host from the same hidden states (the reference's window rule: the last context_size
committed rows, front-padded by repeating the oldest), so the test checks the ring bookkeeping
(prefill seeding, per-step appends at the spec-decode row offsets, slot migration) and the output
shapes; the drafts' numerics are the parity tests' business.
"""
import json
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from conftest import load_golden

pytestmark = pytest.mark.gpu

ENV = ("CF_DRAFTER_DIR", "VLLM_SPEC_TREE", "CF_TREE_KEEP", "CF_TREE_TOPB", "CF_TREE_DEPTH", "CF_TREE_BRANCH",
       "CF_ASYNC_SPEC", "CF_SHORTLIST", "CF_WIDTH", "CF_DRAFT_BUCKETS", "CF_TWOPASS_M", "CF_CUDAGRAPH")


@pytest.fixture(autouse=True)
def clean_env(monkeypatch):
    for k in ENV:
        monkeypatch.delenv(k, raising=False)


@pytest.fixture(scope="module")
def g64_dir(tmp_path_factory):
    """The g64 golden drafter written out as a reference drafter directory (fp16 weights, the
    reference config file, its shortlist)."""
    from safetensors.torch import save_file
    from chain_flow_b200 import shortlist as sl
    g = load_golden("g64")
    d = tmp_path_factory.mktemp("g64_drafter")
    save_file({"drafter." + k: v.half().contiguous() for k, v in g["W"].items()}, str(d / "model.safetensors"))
    args = dict(context_size=8, draft_length=6, chunk_size=3, num_heads=g["heads"], ffn_multiplier=g["FM"],
                num_drafter_layers=g["L"], num_flow_steps=g["T"], path_order=4, path_ffn_multiplier=2,
                markov_rank=g["rank"], init_mode="delta")
    (d / "chained_flow_tree_config.json").write_text(json.dumps({"model_args": args}))
    sl.save(str(d / "shortlist.pt"), g["sl"], vocab_size=g["V"])
    return g, d


def runner_for(g, req_ids, qsl=None):
    model = SimpleNamespace(model=SimpleNamespace(embed_tokens=SimpleNamespace(weight=g["emb"].half().cuda())),
                            lm_head=SimpleNamespace(weight=g["lm_w"].half().cuda()))
    return SimpleNamespace(model=model, input_batch=SimpleNamespace(req_ids=list(req_ids)),
                           query_start_loc=SimpleNamespace(np=np.asarray(qsl if qsl is not None else [0])))


def vllm_config(num_spec, max_num_seqs=8, async_scheduling=False):
    return SimpleNamespace(speculative_config=SimpleNamespace(num_speculative_tokens=num_spec),
                           scheduler_config=SimpleNamespace(max_num_seqs=max_num_seqs,
                                                            async_scheduling=async_scheduling))


def window(hist, C=8):
    rows = hist[-C:]
    return torch.stack([rows[0]] * (C - len(rows)) + rows)


def run_steps(p, g, stash, tree=False):
    """Prefill (2 requests of 5 and 11 prompt tokens), a decode step with 3 and 1 accepted tokens,
    then a step after the input batch swapped the two requests' rows (slot migration). Yields
    (out, expected context windows, committed tokens) right after each propose()."""
    H, dev = g["H"], "cuda"
    gen = torch.Generator(device=dev).manual_seed(5)
    hs = torch.randn(16, H, device=dev, generator=gen).half()
    hist = {"a": list(hs[0:5]), "b": list(hs[5:16])}
    stash.update(runner=runner_for(g, ["a", "b"], qsl=[0, 5, 16]), hidden_states=hs,
                 sample_hidden_states=hs[[4, 15]], spec_meta=None)
    toks = [[11], [22]]
    out = p.propose(toks, None, None)
    k0 = torch.tensor([11, 22], device=dev)
    ctx = torch.stack([window(hist["a"]), window(hist["b"])])
    yield out, ctx, k0
    # decode: every request carried num_draft rows + 1; a accepted 3 tokens, b one
    nd = 5
    sh = torch.randn(2 * (nd + 1), H, device=dev, generator=gen).half()
    stash.update(hidden_states=None, sample_hidden_states=sh, spec_meta=SimpleNamespace(num_draft_tokens=[nd, nd]))
    hist["a"] += list(sh[0:3])
    hist["b"] += list(sh[6:7])
    toks = [[31, 32, 33], [44]]
    out = p.propose(toks, None, None)
    yield out, torch.stack([window(hist["a"]), window(hist["b"])]), torch.tensor([33, 44], device=dev)
    # the input batch swapped the requests' rows: each slot's history moves with its request
    sh = torch.randn(2 * (nd + 1), H, device=dev, generator=gen).half()
    stash.update(runner=runner_for(g, ["b", "a"]), sample_hidden_states=sh)
    hist["b"] += list(sh[0:2])
    hist["a"] += list(sh[6:7])
    toks = [[51, 52], [61]]
    out = p.propose(toks, None, None)
    yield out, torch.stack([window(hist["b"]), window(hist["a"])]), torch.tensor([52, 61], device=dev)


def test_chain_proposer_from_vllm_config(g64_dir, monkeypatch):
    from chain_flow_b200 import proposer as P
    g, d = g64_dir
    monkeypatch.setenv("CF_DRAFTER_DIR", str(d))
    monkeypatch.setattr(P, "_STASH", {})
    p = P.FlowDrafterProposer(vllm_config(num_spec=5))
    assert not p.built
    for out, ctx, k0 in run_steps(p, g, P._STASH):
        assert p.built and isinstance(out, list) and all(len(r) == 5 for r in out)
        want = p._beam_chains(ctx, k0).tolist()
        assert out == want, (out, want)
    assert p.device_error() == 0


def test_async_output_is_a_gpu_tensor_by_input_batch_row(g64_dir, monkeypatch):
    from chain_flow_b200 import proposer as P
    g, d = g64_dir
    monkeypatch.setenv("CF_DRAFTER_DIR", str(d))
    monkeypatch.setenv("CF_ASYNC_SPEC", "1")
    monkeypatch.setattr(P, "_STASH", {})
    p = P.FlowDrafterProposer(vllm_config(num_spec=5, async_scheduling=True))
    hs = torch.randn(9, g["H"], device="cuda").half()
    P._STASH.update(runner=runner_for(g, ["a", "x", "b"], qsl=[0, 4, 5, 9]), hidden_states=hs,
                    sample_hidden_states=hs[[3, 4, 8]], spec_meta=None)
    out = p.propose([[7], [], [9]], None, None)            # the middle request drafts nothing
    assert torch.is_tensor(out) and out.is_cuda and out.dtype == torch.int32 and tuple(out.shape) == (3, 5)
    ctx = torch.stack([window(list(hs[0:4])), window(list(hs[5:9]))])
    want = p._beam_chains(ctx, torch.tensor([7, 9], device="cuda"))
    assert torch.equal(out[0].long(), want[0]) and torch.equal(out[2].long(), want[1])
    assert int(out[1].abs().sum()) == 0


def test_tree_proposer_stages_its_shape_for_the_verifier(g64_dir, monkeypatch):
    from chain_flow_b200 import proposer as P
    g, d = g64_dir
    monkeypatch.setenv("CF_DRAFTER_DIR", str(d))
    monkeypatch.setenv("VLLM_SPEC_TREE", "1")
    monkeypatch.setenv("CF_TREE_KEEP", "4")
    monkeypatch.setenv("CF_TREE_TOPB", "4")
    monkeypatch.setenv("CF_TREE_DEPTH", "5")
    monkeypatch.setattr(P, "_STASH", {})
    p = P.FlowDrafterProposer(vllm_config(num_spec=21))
    N = 20
    for out, ctx, k0 in run_steps(p, g, P._STASH, tree=True):
        want = p._beam_tree(ctx, k0)
        assert out == want[:, :N].tolist()
        reg = p.tree_registration()
        rids = list(P._STASH["runner"].input_batch.req_ids)
        assert sorted(reg) == sorted(rids)
        for j, rid in enumerate(rids):
            toks, parents, depths = reg[rid]
            assert toks == want[j, :N].tolist() and parents == want[j, N:].tolist()
            assert depths == [dd for dd in range(5) for _ in range(4)]
        assert p.tree_registration() == {}                   # joined once
