"""Shortlist file format and vocabulary guard (CPU). The behaviours pinned here are the
reference's (src/chain_flow/shortlist.py:54-108, tests/test_shortlist.py): the guard refuses a list
built for another vocabulary, including a larger one, and never clamps; a legacy bare tensor is
usable but is refused when it holds ids past the head; the content identity does not depend on
the order or dtype the ids were saved in."""
import pytest
import torch

from chain_flow_b200 import shortlist


def test_format_round_trip(tmp_path):
    ids = shortlist.synthetic(248320, 62642, seed=7)
    p = tmp_path / "sl.pt"
    shortlist.save(str(p), ids, 248320, tokenizer="qwen3.5", note="test")
    raw = torch.load(p, map_location="cpu")
    assert raw["format"] == 1 and raw["ids"].dtype == torch.int32 and raw["vocab_size"] == 248320
    got, meta = shortlist.load(str(p))
    assert torch.equal(got, ids) and got.dtype == torch.int64
    assert meta["vocab_size"] == 248320 and meta["tokenizer"] == "qwen3.5" and "ids" not in meta
    assert torch.equal(got, torch.unique(got))             # sorted + unique


def test_guard_accepts_the_vocabulary_it_was_built_for(tmp_path):
    p = tmp_path / "sl.pt"
    shortlist.save(str(p), shortlist.synthetic(248320, 1000, seed=1), 248320)
    ids, meta = shortlist.load(str(p))
    assert shortlist.check(ids, meta, 248320) is None


@pytest.mark.parametrize("v", [151936, 248319, 248321, 32000])
def test_guard_refuses_a_different_vocabulary(tmp_path, v):
    p = tmp_path / "sl.pt"
    shortlist.save(str(p), shortlist.synthetic(248320, 1000, seed=1), 248320)
    ids, meta = shortlist.load(str(p))
    why = shortlist.check(ids, meta, v)
    assert why and str(v) in why and "248320" in why


def test_guard_falls_back_to_a_max_id_check_for_a_legacy_bare_tensor(tmp_path):
    p = tmp_path / "legacy.pt"
    torch.save(torch.tensor([0, 5, 999], dtype=torch.int64), p)
    ids, meta = shortlist.load(str(p))
    assert meta == {}
    assert shortlist.check(ids, meta, 1000) is None
    why = shortlist.check(ids, meta, 500)
    assert why and "999" in why and "no vocab_size metadata" in why


def test_content_identity_ignores_order_and_dtype():
    a = torch.tensor([5, 1, 9, 3], dtype=torch.int64)
    b = torch.tensor([1, 3, 5, 9], dtype=torch.int32)
    assert shortlist.ids_content_sha(a) == shortlist.ids_content_sha(b)
    assert shortlist.ids_content_sha(a) != shortlist.ids_content_sha(torch.tensor([1, 3, 5, 8]))


def test_synthetic_is_seeded_sorted_unique_and_in_range():
    a = shortlist.synthetic(1000, 100, seed=3)
    assert torch.equal(a, shortlist.synthetic(1000, 100, seed=3))
    assert torch.equal(a, torch.unique(a)) and a.numel() == 100
    assert int(a.min()) >= 0 and int(a.max()) < 1000
