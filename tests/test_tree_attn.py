"""The tree-attention fix-up of a full-attention layer (reference fork suffix_merge,
src/chain_flow/patches/vllm-0.25.1-chain-flow-tree.patch:5235-5540; eager form :529-575).

CPU: the oracle's prefix/suffix split is pinned by an identity: merging the prefix attention
(with its log-sum-exp) and the ancestor-masked suffix attention must equal plain softmax attention
of each node over the union of the prefix keys and its ancestors' keys. The reference's eager path
needs the patched vLLM and a GPU, so that identity (not a reference run) is what pins the oracle.
GPU: cfb_tree_attn_merge against the oracle at the reference's shipping shapes (4B: H=16, HKV=4,
D=256, a 40-node tree; 27B: H=24) and a batch of requests, within 4 ulps of the I/O dtype."""
import pytest
import torch

import oracle
from chain_flow_b200.gdn import make_tree
from chain_flow_b200.tree import ancestor_mask


def _tree_batch(S, N, depth=5, branch=4, seed=0):
    return torch.stack([make_tree(N, depth, branch, seed=seed + s)[0] for s in range(S)])


def test_ancestor_mask_marks_each_node_and_its_ancestors():
    par = _tree_batch(3, 17, seed=4)
    mask = ancestor_mask(par)
    for s in range(3):
        for m in range(17):
            anc, a = {m}, int(par[s, m])
            while a >= 0:
                anc.add(a)
                a = int(par[s, a])
            want = torch.tensor([0 if n in anc else 1 for n in range(17)], dtype=torch.uint8)
            assert torch.equal(mask[s, m], want), (s, m)


def test_oracle_merge_equals_attention_over_prefix_and_ancestors():
    S, N, H, HKV, D, P = 2, 12, 4, 2, 64, 7
    g = torch.Generator().manual_seed(1)
    T = S * N + 5                                   # tree rows scattered among other rows
    rows = torch.randperm(T, generator=g)[:S * N].view(S, N)
    q = torch.randn(T, H, D, generator=g)
    k = torch.randn(T, HKV, D, generator=g)
    v = torch.randn(T, HKV, D, generator=g)
    pk = torch.randn(S, P, HKV, D, generator=g)     # each request's prefix keys / values
    pv = torch.randn(S, P, HKV, D, generator=g)
    par = _tree_batch(S, N, seed=2)
    mask = ancestor_mask(par)
    scale = D ** -0.5
    rep = H // HKV
    po = torch.zeros(S * N, H, D)
    plse = torch.zeros(H, S * N)
    for s in range(S):
        for m in range(N):
            for h in range(H):
                o, l = oracle.attention_over(q[rows[s, m], h], pk[s, :, h // rep], pv[s, :, h // rep], scale)
                po[s * N + m, h] = o.float()
                plse[h, s * N + m] = float(l)
    out = oracle.tree_attn_merge(q, k, v, torch.zeros(T, H, D), po, plse, rows, mask, scale)
    for s in range(S):
        for m in range(N):
            anc = [n for n in range(N) if mask[s, m, n] == 0]
            for h in range(H):
                keys = torch.cat([pk[s, :, h // rep], k[rows[s, anc], h // rep]])
                vals = torch.cat([pv[s, :, h // rep], v[rows[s, anc], h // rep]])
                want, _ = oracle.attention_over(q[rows[s, m], h], keys, vals, scale)
                assert torch.allclose(out[rows[s, m], h].double(), want, atol=2e-5), (s, m, h)


def _gpu_case(S, N, H, HKV, D, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    T = S * N + 3
    rows = torch.randperm(T, generator=g, device="cuda")[:S * N].view(S, N)
    qkv = torch.randn(T, (H + 2 * HKV) * D, generator=g, device="cuda").to(dtype)   # strided views
    q = qkv[:, :H * D].view(T, H, D)
    k = qkv[:, H * D:(H + HKV) * D].view(T, HKV, D)
    v = qkv[:, (H + HKV) * D:].view(T, HKV, D)
    po = torch.randn(S * N, H, D, generator=g, device="cuda").to(dtype)
    plse = torch.randn(H, S * N, generator=g, device="cuda") * 2
    plse[0, 0] = float("inf")                        # merge op: +inf counts as -inf
    par = _tree_batch(S, N, seed=seed).cuda()
    return q, k, v, po, plse, rows, ancestor_mask(par)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("S, N, H, HKV, D", [(1, 40, 16, 4, 256), (1, 40, 24, 4, 256), (3, 41, 16, 4, 128),
                                              (2, 100, 8, 8, 64)])
def test_tree_attn_merge_matches_oracle(S, N, H, HKV, D, dtype):
    from chain_flow_b200.tree import tree_attn_merge
    q, k, v, po, plse, rows, mask = _gpu_case(S, N, H, HKV, D, dtype, seed=N + H)
    T = q.shape[0]
    out = torch.full((T, H, D), 7.0, device="cuda", dtype=dtype)
    tree_attn_merge(q, k, v, out, po, plse, rows, mask, D ** -0.5)
    torch.cuda.synchronize()
    want = oracle.tree_attn_merge(q.cpu(), k.cpu(), v.cpu(), out.new_full((T, H, D), 7.0).cpu(), po.cpu(),
                                  plse.cpu(), rows.cpu(), mask.cpu(), D ** -0.5)
    want = want.to(dtype).float()
    got = out.float().cpu()
    eps = 2.0 ** -10 if dtype == torch.float16 else 2.0 ** -7
    err = (got - want).abs() / want.abs().clamp_min(1.0)
    assert float(err.max()) <= 4 * eps, float(err.max())
    tree_rows = set(rows.flatten().tolist())
    others = [r for r in range(T) if r not in tree_rows]
    assert bool((got[others] == 7.0).all())          # only the tree rows are written
