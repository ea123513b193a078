"""Edge cases and size-independent properties of the tree Gated-DeltaNet oracle (CPU): an empty
tree, the identity step (no decay, no write), sibling independence under a reordering of the
nodes, and a chain tree against the per-path recurrence."""
import torch

from oracle.gdn import path_gdn_output, tree_gdn_scan

H, DK, DV = 2, 8, 4


def _inputs(N, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(N, H, DK, generator=g)
    k = torch.randn(N, H, DK, generator=g)
    v = torch.randn(N, H, DV, generator=g)
    gl = -torch.rand(N, H, generator=g)               # log decay, <= 0
    beta = torch.rand(N, H, generator=g)
    init = torch.randn(H, DK, DV, generator=g)
    return q, k, v, gl, beta, init


def test_empty_tree():
    q, k, v, gl, beta, init = _inputs(0)
    parent = torch.zeros(0, dtype=torch.long)
    out, states = tree_gdn_scan(q, k, v, gl, beta, parent, parent.clone(), init)
    assert out.shape == (0, H, DV) and states.shape == (0, H, DK, DV)


def test_no_decay_no_write_keeps_the_prefix_state():
    N = 5
    q, k, v, _, _, init = _inputs(N, seed=1)
    parent = torch.tensor([-1, 0, 0, 1, 2])
    depth = torch.tensor([0, 1, 1, 2, 2])
    zero = torch.zeros(N, H)
    out, states = tree_gdn_scan(q, k, v, zero, zero, parent, depth, init)
    for n in range(N):
        assert torch.allclose(states[n], init)
    qn = q / (q.norm(dim=-1, keepdim=True) + 1e-6) * DK ** -0.5
    ref = torch.einsum("nhk,hkv->nhv", qn, init)
    assert torch.allclose(out, ref, atol=1e-6)


def test_siblings_do_not_depend_on_node_order():
    # root 0 with children 1, 2; 1 has child 3; 2 has child 4
    parent = torch.tensor([-1, 0, 0, 1, 2])
    depth = torch.tensor([0, 1, 1, 2, 2])
    q, k, v, gl, beta, init = _inputs(5, seed=2)
    out, states = tree_gdn_scan(q, k, v, gl, beta, parent, depth, init)
    # the same tree with its nodes listed as 0, 2, 1, 4, 3
    perm = torch.tensor([0, 2, 1, 4, 3])
    inv = torch.argsort(perm)
    parent_p = torch.tensor([-1 if int(parent[i]) < 0 else int(inv[parent[i]]) for i in perm])
    out_p, states_p = tree_gdn_scan(q[perm], k[perm], v[perm], gl[perm], beta[perm], parent_p, depth[perm], init)
    assert torch.equal(out_p, out[perm]) and torch.equal(states_p, states[perm])


def test_chain_tree_equals_the_path_recurrence():
    N = 6
    q, k, v, gl, beta, init = _inputs(N, seed=3)
    parent = torch.arange(N) - 1
    depth = torch.arange(N)
    out, _ = tree_gdn_scan(q, k, v, gl, beta, parent, depth, init)
    for n in range(N):
        path = torch.arange(n + 1)
        o = path_gdn_output(q, k, v, gl, beta, path, init)
        assert torch.allclose(out[n], o, rtol=1e-5, atol=1e-6)
