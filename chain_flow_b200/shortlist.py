"""Shortlist head files: format, load, vocabulary guard, content identity.

Same on-disk format and guard semantics as the reference (src/chain_flow/shortlist.py:54-108):

* ``torch.save({"format": 1, "ids": int32[R] sorted unique, "vocab_size": int, "tokenizer": str,
  "note": str})``, or a legacy bare tensor of ids;
* ``check(ids, meta, V)`` refuses a list built for a different vocabulary (or, for legacy files
  without metadata, one holding ids past the head) and says why; it never clamps ids into range;
* ``ids_content_sha`` hashes the SORTED int32 ids, so the same list saved two ways has one identity.
"""
from __future__ import annotations

import hashlib

import torch


def ids_content_sha(ids) -> str:
    t = ids if isinstance(ids, torch.Tensor) else torch.as_tensor(ids)
    return hashlib.sha256(t.to(torch.int32).flatten().sort().values.cpu().numpy().tobytes()).hexdigest()


def load(path: str):
    """(ids int64 CPU tensor, meta dict) from a shortlist file of either format."""
    obj = torch.load(path, map_location="cpu", weights_only=False)
    if isinstance(obj, dict):
        ids = obj["ids"]
        meta = {k: v for k, v in obj.items() if k != "ids"}
    else:
        ids, meta = obj, {}
    return torch.as_tensor(ids).flatten().long(), meta


def check(ids: torch.Tensor, meta: dict, vocab_size: int) -> str | None:
    """None if the list may be used against a `vocab_size`-row head, else the reason it may not."""
    built = meta.get("vocab_size")
    if built is not None:
        if int(built) != int(vocab_size):
            return (f"built for vocab_size={int(built)} but this model's lm_head has {int(vocab_size)} "
                    f"rows -- the ids would name different tokens")
        return None
    mx = int(ids.max()) if ids.numel() else -1
    if mx >= int(vocab_size):
        return (f"contains token id {mx}, past this model's {int(vocab_size)}-row lm_head, and carries "
                f"no vocab_size metadata")
    return None


def save(path: str, ids, vocab_size: int, tokenizer: str = "", note: str = "") -> None:
    ids = torch.as_tensor(ids).flatten().to(torch.int64).unique().to(torch.int32)
    torch.save({"format": 1, "ids": ids, "vocab_size": int(vocab_size), "tokenizer": tokenizer,
                "note": note}, path)


def synthetic(vocab_size: int, rows: int, seed: int) -> torch.Tensor:
    """A seeded sorted set of `rows` unique ids in [0, vocab_size) (benchmarks and tests)."""
    g = torch.Generator().manual_seed(seed)
    return torch.randperm(vocab_size, generator=g)[:rows].sort().values
