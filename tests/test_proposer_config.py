"""CPU tests of the vLLM-facing constructor of FlowDrafterProposer (reference
src/chain_flow/vllm_plugin/flow_proposer.py:329-560): what it reads from a vllm_config and the
environment, what it refuses, and the checkpoint / shortlist resolution of the lazy build. Nothing
here touches a GPU: the build itself (packing, the ring) happens on the first propose()."""
import json
from types import SimpleNamespace

import pytest
import torch

from chain_flow_b200.proposer import FlowDrafterProposer
from chain_flow_b200.weights import DraftConfig

ENV = ("CF_DRAFTER_DIR", "VLLM_SPEC_TREE", "CF_TREE_KEEP", "CF_TREE_TOPB", "CF_TREE_DEPTH", "CF_TREE_BRANCH",
       "CF_ASYNC_SPEC", "CF_SHORTLIST", "CF_WIDTH", "CF_DRAFT_BUCKETS", "CF_TWOPASS_M", "CF_CUDAGRAPH")


@pytest.fixture(autouse=True)
def clean_env(monkeypatch):
    for k in ENV:
        monkeypatch.delenv(k, raising=False)


def vllm_config(num_spec=5, max_num_seqs=16, async_scheduling=False):
    return SimpleNamespace(speculative_config=SimpleNamespace(num_speculative_tokens=num_spec),
                           scheduler_config=SimpleNamespace(max_num_seqs=max_num_seqs,
                                                            async_scheduling=async_scheduling))


@pytest.fixture
def ckpt(tmp_path):
    """A tiny drafter checkpoint directory with the reference's file layout."""
    from safetensors.torch import save_file
    from gpu_util import random_state_dict
    cfg = DraftConfig(hidden=64, num_heads=4, ffn_multiplier=2, num_drafter_layers=1, num_flow_steps=2,
                      markov_rank=16)
    sd = random_state_dict(cfg, 500, seed=3)
    save_file({"drafter." + k: v.half().contiguous() for k, v in sd.items()}, str(tmp_path / "model.safetensors"))
    args = dict(context_size=8, draft_length=6, chunk_size=3, num_heads=4, ffn_multiplier=2, num_drafter_layers=1,
                num_flow_steps=2, path_order=4, path_ffn_multiplier=2, markov_rank=16, init_mode="delta")
    (tmp_path / "chained_flow_tree_config.json").write_text(json.dumps({"model_args": args}))
    return tmp_path


def test_drafter_dir_is_required():
    with pytest.raises(ValueError, match="CF_DRAFTER_DIR"):
        FlowDrafterProposer(vllm_config())


def test_chain_configuration(ckpt, monkeypatch):
    monkeypatch.setenv("CF_DRAFTER_DIR", str(ckpt))
    p = FlowDrafterProposer(vllm_config(num_spec=5, max_num_seqs=12))
    assert (p.K, p.draft_width, p.max_reqs, p.branching) == (5, 5, 12, False)
    assert not p.built                                   # lazily built on the first propose()
    assert p._buckets == [1, 2, 4, 8, 12]
    assert p._wmax() == 6
    assert p.async_spec is False


def test_tree_depth_is_clamped_to_what_the_checkpoint_emits(ckpt, monkeypatch):
    monkeypatch.setenv("CF_DRAFTER_DIR", str(ckpt))
    monkeypatch.setenv("VLLM_SPEC_TREE", "1")
    monkeypatch.setenv("CF_TREE_KEEP", "4")
    monkeypatch.setenv("CF_TREE_TOPB", "8")
    monkeypatch.setenv("CF_TREE_DEPTH", "9")             # draft_length 6 -> at most 5 levels
    p = FlowDrafterProposer(vllm_config(num_spec=4 * 5 + 1))
    assert (p.tree_depth, p.N, p.draft_width, p.K) == (5, 20, 20, 20)
    assert p._wmax() == 6                                # tree_depth + 1 ring rows per commit


def test_tree_speculative_tokens_must_be_n_plus_one(ckpt, monkeypatch):
    monkeypatch.setenv("CF_DRAFTER_DIR", str(ckpt))
    monkeypatch.setenv("VLLM_SPEC_TREE", "1")
    monkeypatch.setenv("CF_TREE_DEPTH", "4")
    with pytest.raises(ValueError, match="num_speculative_tokens=17"):
        FlowDrafterProposer(vllm_config(num_spec=16))


def test_keep_above_topb_is_refused(ckpt, monkeypatch):
    monkeypatch.setenv("CF_DRAFTER_DIR", str(ckpt))
    monkeypatch.setenv("VLLM_SPEC_TREE", "1")
    monkeypatch.setenv("CF_TREE_KEEP", "8")
    monkeypatch.setenv("CF_TREE_TOPB", "4")
    with pytest.raises(ValueError, match="CF_TREE_KEEP=8 > CF_TREE_TOPB=4"):
        FlowDrafterProposer(vllm_config(num_spec=33))


@pytest.mark.parametrize("engine_async, want", [(False, False), (True, True)])
def test_async_output_follows_the_engine(ckpt, monkeypatch, engine_async, want):
    monkeypatch.setenv("CF_DRAFTER_DIR", str(ckpt))
    monkeypatch.setenv("CF_ASYNC_SPEC", "1")
    assert FlowDrafterProposer(vllm_config(async_scheduling=engine_async)).async_spec is want


def test_checkpoint_and_shortlist_resolution(ckpt, monkeypatch, tmp_path_factory):
    from chain_flow_b200 import shortlist as sl
    ids = torch.arange(0, 500, 3)
    sl.save(str(ckpt / "shortlist.pt"), ids, vocab_size=500)
    sub, args, got = FlowDrafterProposer._read_checkpoint(str(ckpt), 500)
    assert torch.equal(got, ids) and args["draft_length"] == 6 and "expert.out_proj.weight" in sub
    # a list built for another vocabulary is refused, not clamped
    with pytest.raises(ValueError, match="vocab_size=500"):
        FlowDrafterProposer._read_checkpoint(str(ckpt), 501)
    # CF_SHORTLIST set and empty: the full head on request
    monkeypatch.setenv("CF_SHORTLIST", "")
    assert FlowDrafterProposer._read_checkpoint(str(ckpt), 500)[2] is None
    monkeypatch.delenv("CF_SHORTLIST")
    # a checkpoint that declares its shortlist refuses a different one
    conf = json.loads((ckpt / "chained_flow_tree_config.json").read_text())
    conf["shortlist"] = {"rows": 10}
    (ckpt / "chained_flow_tree_config.json").write_text(json.dumps(conf))
    with pytest.raises(RuntimeError, match="does not match"):
        FlowDrafterProposer._read_checkpoint(str(ckpt), 500)
