"""Where a draft's time goes, phase by phase, from the engine's own %globaltimer stamps.

    python -m chain_flow_b200.phase_report [--workload 4b-prod] [--batch 1] [--rows 0]

Builds profiled copies (``CFB_RUN_PROFILE``) of the plans a synthetic proposer uses for one
chain draft, runs each a few times on ``cuda:0``, and prints, per plan, its total time and a
table of phase classes (kind, units, tiles). For each class it gives the number of phases, their
summed and mean wall time, and the mean grid-barrier tail: from the last stamp of a phase's work
(any CTA's work-done or epilogue-done stamp) to the last CTA passing the barrier. ``--rows N``
also prints the first N phases one by one. A phase's wall time runs from the previous phase's
last barrier pass to its own.

Profiled plans are separate instantiations of the engine; their stamps cost a little time, so
use this for where time goes and ``bench.py`` for how much.
"""
from __future__ import annotations

import argparse

import torch

from . import _lib


def summarize(t: torch.Tensor, tab: torch.Tensor) -> dict:
    """Aggregate one profiled run. `t`: [phases, grid, 20] int64 stamps (CFB_BUF_PROF), `tab`:
    [phases, 15] int32 phase table (CFB_BUF_PHASES). Returns {"total_us", "phases": per-phase
    rows, "classes": {(kind, units, tiles): {"n", "wall_us", "tail_us"}}}."""
    t = t.double()
    start = t[0, :, 0].min()
    ends = t[:, :, 2].max(dim=1).values
    # the epilogue-done stamp (slot 6) is written by GEMM phases only (kind 1); other phases leave
    # whatever the slot held, so only their work-done stamp (slot 1) counts
    gemm = (tab[:, 0] == 1).unsqueeze(1)
    done = torch.where(gemm, torch.maximum(t[:, :, 1], t[:, :, 6]), t[:, :, 1]).max(dim=1).values
    rows, classes = [], {}
    for i in range(t.shape[0]):
        prev = ends[i - 1] if i else start
        wall = float(ends[i] - prev) / 1e3
        tail = float(ends[i] - done[i]) / 1e3
        key = (int(tab[i, 0]), int(tab[i, 3]), int(tab[i, 4]))
        c = classes.setdefault(key, {"n": 0, "wall_us": 0.0, "tail_us": 0.0})
        c["n"] += 1
        c["wall_us"] += wall
        c["tail_us"] += tail
        rows.append({"kind": key[0], "units": key[1], "tiles": key[2], "whole": int(tab[i, 5]),
                     "wall_us": wall, "tail_us": tail})
    return {"total_us": float(ends[-1] - start) / 1e3, "phases": rows, "classes": classes}


def _profiled_copies(prop, B: int):
    """Profiled plans with the same inputs as the proposer's cached chain-draft plan."""
    from .engine import Plan
    src = next(iter(prop._plans.values()))
    init = _lib.INIT_MODES[prop.init_mode]
    if prop.vae is not None:
        fp = Plan(prop.flow_weights, _lib.MODE_FLOW, B, profile=True, init_mode=init)
        fp.ctx.copy_(src.flow.ctx)
        fp.z0.copy_(src.flow.z0)
        hp = Plan(prop.weights, _lib.MODE_BEAM_CHAIN, B, width=prop.width, depth=prop.K, profile=True,
                  twopass_m=prop.twopass_m)
        hp.pred.copy_(src.head.pred)
        hp.known0.copy_(src.head.known0)
        return [("flow", fp), ("beam", hp)]
    p = Plan(prop.weights, _lib.MODE_CHAIN, B, width=prop.width, depth=prop.K, profile=True,
             init_mode=init, twopass_m=prop.twopass_m)
    p.ctx.copy_(src.ctx)
    p.z0.copy_(src.z0)
    p.known0.copy_(src.known0)
    return [("draft", p)]


def main(argv=None) -> None:
    from .proposer import FlowDrafterProposer
    from .synthetic import WORKLOADS, make_state, make_inputs
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--workload", default="4b-prod", choices=sorted(WORKLOADS))
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--rows", type=int, default=0, help="also print the first N phases")
    args = ap.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("phase_report needs a GPU")
    wl, B = WORKLOADS[args.workload], args.batch
    if not 1 <= B <= 8:
        raise SystemExit("the persistent engine's plans (and so this report) serve 1 to 8 requests")
    dev = torch.device("cuda", 0)
    sd, emb, lm, sl = make_state(wl, device=dev)
    prop = FlowDrafterProposer.from_components(sd, wl.model_args(), emb, lm, sl, width=wl.width, K=wl.draft_tokens,
                                               device=dev)
    ctx, known0 = make_inputs(wl, B, device=dev)
    prop._beam_chains(ctx, known0)
    torch.cuda.synchronize()
    for name, p in _profiled_copies(prop, B):
        for _ in range(3):
            p.run()
        torch.cuda.synchronize()
        p.check()
        s = summarize(p.phase_times(), p.phase_table())
        print(f"== {name}: {len(s['phases'])} phases, {s['total_us']:.1f} us, grid {p.grid}")
        for i, r in enumerate(s["phases"][:args.rows]):
            print(f"  {i:4d} kind {r['kind']} units {r['units']:6d} tiles {r['tiles']:5d} whole {r['whole']} "
                  f"wall {r['wall_us']:7.1f} us  barrier tail {r['tail_us']:5.1f} us")
        print(f"  {'kind':>4} {'units':>6} {'tiles':>5} {'n':>4} {'total us':>9} {'mean us':>8} {'tail us':>8}")
        for (k, u, tl), c in sorted(s["classes"].items(), key=lambda kv: -kv[1]["wall_us"]):
            print(f"  {k:4d} {u:6d} {tl:5d} {c['n']:4d} {c['wall_us']:9.1f} {c['wall_us'] / c['n']:8.2f} "
                  f"{c['tail_us'] / c['n']:8.2f}")


if __name__ == "__main__":
    main()
