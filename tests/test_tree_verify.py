"""Greedy verification of a draft tree (reference fork tree_rejection_sample /
tree_greedy_descent_kernel, src/chain_flow/patches/vllm-0.25.1-chain-flow-tree.patch:640-723).

CPU: the oracle is pinned by what the descent must reduce to: on a chain-shaped tree it is vLLM's
stock greedy acceptance (accept while the draft token is the row's argmax, then the bonus token);
a request without drafts emits its row's argmax; among siblings with the same token the first
wins. GPU: cfb_tree_verify_greedy equals the oracle exactly (integers), for fp32 / bf16 logits at
the 4B vocabulary (248,320), with planted accepted paths, ties and a NaN, over repeated launches
(the workspace counters reset themselves)."""
import pytest
import torch

import oracle
from chain_flow_b200.gdn import make_tree


def _flat(trees):
    """[(parents, draft tokens)] per request -> cu_num_draft, cu_num_sampled, tokens, parents."""
    cu_d, cu_s, toks, pars = [], [], [], []
    d = s = 0
    for par, tok in trees:
        d += len(par)
        s += len(par) + 1
        cu_d.append(d); cu_s.append(s)
        toks += list(tok); pars += list(par)
    return torch.tensor(cu_d), torch.tensor(cu_s), torch.tensor(toks, dtype=torch.int64), torch.tensor(pars)


def test_chain_tree_is_stock_greedy_acceptance():
    g = torch.Generator().manual_seed(0)
    n, V = 6, 50
    logits = torch.randn(n + 1, V, generator=g)
    am = logits.argmax(-1)
    draft = [int(am[0]), int(am[1]), int(am[2]), (int(am[3]) + 1) % V, int(am[4]), int(am[5])]
    cu_d, cu_s, toks, pars = _flat([(list(range(-1, n - 1)), draft)])
    out, path, alen = oracle.tree_verify_greedy(logits, cu_d, cu_s, toks, pars, n)
    # stock: accept drafts 0..2, reject 3, emit argmax of row 3 as the bonus
    assert alen.tolist() == [3]
    assert out[0].tolist() == draft[:3] + [int(am[3])] + [-1] * (n - 3)
    assert path[0].tolist() == [0, 1, 2] + [-1] * (n - 3)


def test_request_without_drafts_emits_its_bonus_and_first_sibling_wins():
    logits = torch.zeros(1 + 4, 10)
    logits[0, 3] = 1.0          # request 0 has no drafts: one row
    logits[1, 7] = 1.0          # request 1's root row: argmax 7
    logits[3, 5] = 1.0          # node 1 (the first sibling carrying 7): argmax 5
    cu_d, cu_s, toks, pars = _flat([([], []), ([-1, -1, -1], [2, 7, 7])])
    out, path, alen = oracle.tree_verify_greedy(logits, cu_d, cu_s, toks, pars, 3)
    assert out.tolist() == [[3, -1, -1, -1], [7, 5, -1, -1]]
    assert alen.tolist() == [0, 1] and path[1].tolist() == [1, -1, -1]


def _planted(B, N, V, dtype, seed):
    """B requests of N-node trees whose draft tokens follow the target's argmax along a random path
    for a random number of steps; ties, and one NaN, planted in the logits."""
    g = torch.Generator().manual_seed(seed)
    trees = []
    for r in range(B):
        par, _ = make_tree(N, 5, 4, seed=seed + r)
        trees.append((par.tolist(), torch.randint(0, V, (N,), generator=g).tolist()))
    cu_d, cu_s, toks, pars = _flat(trees)
    rows = int(cu_s[-1])
    logits = torch.randn(rows, V, generator=g)
    logits[0, 17] = logits[0, 1000] = 40.0                       # a tie: the first index wins
    logits[1, 5] = float("nan")                                  # NaN counts as the maximum
    am = logits.argmax(-1)
    d0 = 0
    for r, (par, tok) in enumerate(trees):
        s0 = int(cu_s[r]) - (len(par) + 1)
        cur = -1
        for _ in range(int(torch.randint(0, 5, (1,), generator=g))):
            kids = [i for i in range(len(par)) if par[i] == cur]
            if not kids:
                break
            i = kids[int(torch.randint(0, len(kids), (1,), generator=g))]
            toks[d0 + i] = int(am[s0 + cur + 1])
            cur = i
        d0 += len(par)
    return logits.to(dtype), cu_d, cu_s, toks, pars


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_tree_verify_greedy_matches_oracle(dtype):
    from chain_flow_b200.tree import TreeVerifier
    B, N, V = 5, 40, 248320
    ver = TreeVerifier(max_rows=B * (N + 1), max_batch=B, max_spec_len=N)
    for seed in (1, 2):                     # two launches in a row: the counters reset themselves
        logits, cu_d, cu_s, toks, pars = _planted(B, N, V, dtype, seed)
        want = oracle.tree_verify_greedy(logits, cu_d, cu_s, toks, pars, N)
        got = ver(logits.cuda(), cu_d.cuda(), cu_s.cuda(), toks.cuda(), pars.cuda())
        torch.cuda.synchronize()
        for a, b in zip(got, want):
            assert torch.equal(a.cpu(), b), (a.cpu(), b)
        assert int(ver.err.item()) == 0
    assert int(ver.accepted_len.max()) >= 2           # the planted paths were walked


@pytest.mark.gpu
def test_tree_verify_greedy_mixed_batch_and_bad_offsets():
    from chain_flow_b200.tree import TreeVerifier
    logits = torch.zeros(1 + 4, 10)
    logits[0, 3] = 1.0
    logits[1, 7] = 1.0
    logits[3, 5] = 1.0
    cu_d, cu_s, toks, pars = _flat([([], []), ([-1, -1, -1], [2, 7, 7])])
    ver = TreeVerifier(max_rows=5, max_batch=2, max_spec_len=3)
    out, path, alen = ver(logits.cuda(), cu_d.cuda(), cu_s.cuda(), toks.cuda(), pars.cuda())
    torch.cuda.synchronize()
    assert out.cpu().tolist() == [[3, -1, -1, -1], [7, 5, -1, -1]] and alen.cpu().tolist() == [0, 1]
    # offsets past the logits rows: that request emits nothing and the error word is set
    bad_s = torch.tensor([1, 9])
    out, path, alen = ver(logits.cuda(), cu_d.cuda(), bad_s.cuda(), toks.cuda(), pars.cuda())
    torch.cuda.synchronize()
    assert out.cpu().tolist()[1] == [-1, -1, -1, -1] and int(ver.err.item()) != 0
