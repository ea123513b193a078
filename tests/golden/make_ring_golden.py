"""Generate tests/golden/ring.npz by running the REFERENCE's context ring
(FlowDrafterProposer._init_ring / _ring_write / _ring_gather, reference
src/chain_flow/vllm_plugin/flow_proposer.py:881-961) on seeded inputs.

Run in a container that has the reference checkout (it is not needed anywhere else):

    python tests/golden/make_ring_golden.py --ref /path/to/chain-flow/src

The object is built with ``__new__`` and only the attributes the ring methods read. A sequence
of steps covers: fresh slots (fewer than ctx_size rows: front padding by the oldest row), ring
wrap-around, requests masked off (wmask False), chain steps (rows taken contiguously from
``start``) and tree steps (accepted path rows scattered through ``path``), and source rows past
the end of the harvested hidden states (clamped).
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
R, C, H, KMAX, STEPS = 6, 8, 16, 6, 7


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("CF_REFERENCE_SRC"), required="CF_REFERENCE_SRC" not in os.environ,
                    help="the reference checkout's src/ directory (or set CF_REFERENCE_SRC)")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    from chain_flow.vllm_plugin.flow_proposer import FlowDrafterProposer
    p = FlowDrafterProposer.__new__(FlowDrafterProposer)
    p.__dict__.update(max_reqs=R, ctx_size=C, dev=torch.device("cpu"), dtype=torch.float16)
    FlowDrafterProposer._init_ring(p, H)
    g = torch.Generator().manual_seed(21)
    out = {"dims": np.array([R, C, H, KMAX, STEPS], np.int64)}
    with torch.inference_mode():
        for s in range(STEPS):
            B = int(torch.randint(2, R + 1, (1,), generator=g))
            rows = torch.randperm(R, generator=g)[:B]
            nsh = int(torch.randint(B, B * KMAX + 1, (1,), generator=g))
            sh = (torch.randn(nsh, H, generator=g) * 2).to(torch.float16)
            starts = torch.randint(0, nsh, (B,), generator=g)
            cnt = torch.randint(1, KMAX + 1, (B,), generator=g)
            wmask = torch.rand(B, generator=g) > 0.2
            tree = s % 2 == 1
            path = torch.randint(0, 12, (R, KMAX + 2), generator=g) if tree else None
            FlowDrafterProposer._ring_write(p, sh, rows, starts, cnt, wmask, path, KMAX)
            grows = torch.randperm(R, generator=g)[:int(torch.randint(1, R + 1, (1,), generator=g))]
            ctx = FlowDrafterProposer._ring_gather(p, grows)
            out.update({f"s{s}_rows": rows.numpy(), f"s{s}_sh": sh.numpy(), f"s{s}_starts": starts.numpy(),
                        f"s{s}_cnt": cnt.numpy(), f"s{s}_wmask": wmask.numpy(),
                        f"s{s}_path": (path.numpy() if tree else np.zeros((0, 0), np.int64)),
                        # copies: the ring tensors are updated in place by the next step
                        f"s{s}_ring": p._ring[:, :C].clone().numpy(), f"s{s}_rpos": p._rpos.clone().numpy(),
                        f"s{s}_nval": p._nval.clone().numpy(), f"s{s}_grows": grows.numpy(),
                        f"s{s}_ctx": ctx.clone().numpy()})
    path = HERE / "ring.npz"
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({path.stat().st_size / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()
