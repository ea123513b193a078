"""Row-sharded shortlist head across 2 GPUs (NCCL): every rank drafts the same requests over its
half of the head rows, and the ranks' merged top-k lists are all-gathered once per beam depth.
Both ranks must produce the same hiddens and tokens, and the tokens must equal the oracle beam
over those hiddens (the reference's own tokens where no near-tie flips). Needs 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import oracle
from conftest import golden_flow_config, load_golden

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, name, out):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from chain_flow_b200 import _lib
        from chain_flow_b200.engine import Plan
        from chain_flow_b200.weights import DraftConfig, DrafterWeights
        g = load_golden(name)
        cfg = DraftConfig(hidden=g["H"], num_heads=g["heads"], ffn_multiplier=g["FM"],
                          num_drafter_layers=g["L"], num_flow_steps=g["T"], markov_rank=g["rank"])
        w = DrafterWeights(g["W"], cfg, g["emb"], g["lm_w"], g["sl"], device=dev, head_shard=(rank, world))
        res = {}
        for mode, kw in ((_lib.MODE_CHAIN, dict(width=4, depth=5)),
                         (_lib.MODE_TREE, dict(depth=5, tree_keep=4, tree_topb=4))):
            p = Plan(w, mode, g["B"], **kw)
            assert p.segments == 6, p.segments
            p.ctx.copy_(g["ctx"].half()); p.z0.copy_(g["z0"].half()); p.known0.copy_(g["known0"])
            for _ in range(2):                       # twice: the plan is reusable
                p.run(group=dist.group.WORLD)
            torch.cuda.synchronize(dev)
            p.check()
            res[mode] = (p.pred.cpu().numpy(), p.tokens.cpu().numpy())     # by value through the queue
        gathered = [None] * world
        dist.all_gather_object(gathered, res)
        if rank == 0:
            out.put(gathered)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name", ["g64", "g128"])
def test_row_sharded_head_on_two_gpus(name):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from chain_flow_b200 import _lib
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    mp.start_processes(_worker, args=(2, _free_port(), name, q), nprocs=2, start_method="spawn")
    ranks = q.get()
    g = load_golden(name)
    cfg = golden_flow_config(g)
    sl = g["sl"]
    hw, w2 = g["lm_w"][sl], g["W"]["markov.w2.weight"][sl]
    for mode in (_lib.MODE_CHAIN, _lib.MODE_TREE):
        (pred0, tok0), (pred1, tok1) = [tuple(torch.from_numpy(a) for a in ranks[i][mode]) for i in (0, 1)]
        assert torch.equal(pred0, pred1) and torch.equal(tok0, tok1)
        rel = float((pred0 - g["pred"]).abs().max() / g["pred"].abs().max())
        assert rel < 2e-2, rel
        if mode == _lib.MODE_CHAIN:
            want = oracle.beam_chains(g["W"], cfg, g["emb"], hw, w2, sl, pred0, g["known0"], 4, 5)
            assert torch.equal(tok0, want), (tok0, want)
        else:
            want = oracle.beam_tree(g["W"], cfg, g["emb"], hw, w2, sl, pred0, g["known0"], 4, 4, 5)
            if not torch.equal(tok0, want):
                from beam_check import check_tree
                check_tree(tok0, g["W"], cfg, g["emb"], hw, w2, sl, pred0, g["known0"], 4, 4, 5)
