"""The multi-GPU contract, on CPU with world_size-2 gloo process groups (no GPU needed).

* Request partitioning (bench.py's weak scaling): every rank drafts its own requests; the only
  collective is the max over ranks of the timed region.
* Row-sharded head: rank r holds rows shard_rows(R, ranks, r) of the shortlist head. Per beam
  row it publishes (max, sumexp, top-k values, top-k shortlist ids). The ranks' lists, gathered
  in rank order and merged as the engine's beam phase merges them, must give exactly the
  unsharded log-softmax and top-k (ties: lower id first). The oracle computes the logits.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from chain_flow_b200.weights import shard_rows


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_rows_cover_the_head_once():
    for R in (1, 7, 256, 62642):
        for ranks in (1, 2, 3, 4, 8):
            if ranks > R:
                continue
            got = [shard_rows(R, ranks, r) for r in range(ranks)]
            assert got[0][0] == 0
            for (a0, an), (b0, _) in zip(got, got[1:]):
                assert a0 + an == b0 and an > 0
            assert got[-1][0] + got[-1][1] == R
    with pytest.raises(ValueError):
        shard_rows(10, 2, 2)


def _merge(lists, K):
    """lists: [(m, s, vals[K], ids[K])] in rank order -> (lse, vals, ids), the engine's merge."""
    m, s = -float("inf"), 0.0
    for mb, sb, _, _ in lists:
        M = max(m, mb)
        s = 0.0 if M == -float("inf") else s * torch.exp(torch.tensor(m - M)).item() + sb * torch.exp(torch.tensor(mb - M)).item()
        m = M
    cand = [(v, i) for _, _, vs, ids in lists for v, i in zip(vs, ids)]
    cand.sort(key=lambda t: (-t[0], t[1]))
    top = cand[:K]
    return m + torch.log(torch.tensor(s)).item(), [v for v, _ in top], [i for _, i in top]


def _sharded_head_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(3)
        R, D, rank_m, K, rows = 300, 32, 16, 4, 3
        hw = torch.randn(R, D, generator=g)
        w2 = torch.randn(R, rank_m, generator=g) * 0.1
        W = {"markov.w1.weight": torch.randn(50, rank_m, generator=g)}
        h = torch.randn(rows, D, generator=g)
        prev = torch.tensor([3, 7, 11])
        logits = h @ hw.T + oracle.markov_bias(W, w2, prev)           # full head, [rows, R]
        r0, n = shard_rows(R, world, rank)
        part = logits[:, r0:r0 + n]
        mine = []
        for r in range(rows):
            mx = part[r].max().item()
            se = torch.exp(part[r] - mx).sum().item()
            v, i = part[r].topk(K)
            mine.append([mx, se] + v.tolist() + (i + r0).float().tolist())
        t = torch.tensor(mine, dtype=torch.float64)
        allt = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(allt, t)
        if rank == 0:
            lp = torch.log_softmax(logits.double(), dim=-1)
            ok = True
            for r in range(rows):
                lists = [(a[r, 0].item(), a[r, 1].item(), a[r, 2:2 + K].tolist(), [int(x) for x in a[r, 2 + K:].tolist()])
                         for a in allt]
                lse, vals, ids = _merge(lists, K)
                v, i = lp[r].topk(K)
                ok &= ids == i.tolist()
                ok &= all(abs((val - lse) - w) < 1e-5 for val, w in zip(vals, v.tolist()))   # fp32 sums
            out.put(bool(ok))
    finally:
        dist.destroy_process_group()


def _requests_worker(rank, world, port, out):
    """bench.py's reduction: each rank times its own requests; rank 0 reports the max."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        t = torch.tensor([1.5 + rank], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            out.put(t.item())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_sharded_head_merge_equals_unsharded_head(world):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    mp.start_processes(_sharded_head_worker, args=(world, _free_port(), q), nprocs=world, start_method="spawn")
    assert q.get() is True


def test_request_partitioning_reports_the_slowest_rank():
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    mp.start_processes(_requests_worker, args=(2, _free_port(), q), nprocs=2, start_method="spawn")
    assert q.get() == 2.5
