"""cfb_tree_gdn_noalloc (no device allocation, node states in the library's fixed device array)
against cfb_tree_gdn (caller-owned states), both called through the C ABI, on two calls in a row
with different trees and inputs. Tolerance: the GDN tolerance of the parity tests (1e-2 relative).

Collected last on purpose: it must pass in a fresh process and after every other test.
"""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu

GDN_RTOL = 1e-2


def _inputs(B, N, H, D, seed):
    from chain_flow_b200.gdn import make_tree
    g = torch.Generator(device="cuda").manual_seed(seed)
    dev = "cuda"
    q = torch.randn(B, N, H, D, device=dev, generator=g).half()
    k = torch.randn(B, N, H, D, device=dev, generator=g).half()
    v = torch.randn(B, N, H, D, device=dev, generator=g).half()
    gl = torch.log(torch.sigmoid(torch.randn(B, N, H, device=dev, generator=g)))
    beta = torch.sigmoid(torch.randn(B, N, H, device=dev, generator=g))
    par = torch.stack([make_tree(N, 5, 4, seed + b)[0] for b in range(B)]).to(dev, torch.int32)
    init = torch.randn(B, H, D, D, device=dev, generator=g) * 0.1
    return q, k, v, gl, beta, par, init


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _call_existing(lib, stream, q, k, v, gl, beta, par, init):
    B, N, H, D = q.shape
    o = torch.full((B, N, H, D), float("nan"), device="cuda")
    states = torch.empty(B, N, H, D, D, device="cuda")
    st = lib.cfb_tree_gdn(_ptr(q), _ptr(k), _ptr(v), _ptr(gl), _ptr(beta), _ptr(par), _ptr(init), _ptr(o),
                          _ptr(states), B, N, H, D, D, 1, stream)
    assert st == 0, st
    return o


def _call_noalloc(lib, stream, q, k, v, gl, beta, par, init):
    B, N, H, D = q.shape
    o = torch.full((B, N, H, D), float("nan"), device="cuda")
    st = lib.cfb_tree_gdn_noalloc(_ptr(q), _ptr(k), _ptr(v), _ptr(gl), _ptr(beta), _ptr(par), _ptr(init),
                                  _ptr(o), B, N, H, D, D, 1, stream)
    assert st == 0, st
    return o


def _rel(a, b):
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-12))


def test_noalloc_matches_existing_entry_point_on_two_calls_in_a_row():
    from chain_flow_b200 import _lib
    lib = _lib.load()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    # first call fills the whole array (4 trees x 16 nodes x 16 heads x 128 x 128 fp32 = 64 MiB);
    # the second, smaller call runs over the first call's leftover node states
    for B, seed in ((4, 101), (2, 202)):
        args = _inputs(B, 16, 16, 128, seed)
        want = _call_existing(lib, stream, *args)
        got = _call_noalloc(lib, stream, *args)
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert _rel(got, want) <= GDN_RTOL, _rel(got, want)


def test_noalloc_rejects_sizes_beyond_its_array():
    from chain_flow_b200 import _lib
    lib = _lib.load()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    q, k, v, gl, beta, par, init = _inputs(1, 16, 16, 128, 7)
    o = torch.empty(5, 16, 16, 128, device="cuda")
    # 5 x 16 x 16 x 128 x 128 fp32 is one tree more than the 64 MiB array holds; rejected before launch
    st = lib.cfb_tree_gdn_noalloc(_ptr(q), _ptr(k), _ptr(v), _ptr(gl), _ptr(beta), _ptr(par), _ptr(init),
                                  _ptr(o), 5, 16, 16, 128, 128, 1, stream)
    assert st == 3                                   # CFB_ERR_WORKSPACE


def test_noalloc_malformed_parent_is_nan_not_leftover_state():
    """A call after a larger one leaves node states of the first call in the shared array. A node
    whose parent index points past its own position (p == n) must not read them: its output, and
    its descendants' outputs, are NaN; every other node equals the existing entry point's."""
    from chain_flow_b200 import _lib
    lib = _lib.load()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    _call_noalloc(lib, stream, *_inputs(4, 16, 16, 128, 303))        # fills the array
    q, k, v, gl, beta, par, init = _inputs(1, 16, 16, 128, 404)
    bad = 9
    par[0, bad] = bad                                                 # parent == self
    got = _call_noalloc(lib, stream, q, k, v, gl, beta, par, init)
    want = _call_existing(lib, stream, q, k, v, gl, beta, par, init)
    torch.cuda.synchronize()
    p = par[0].tolist()
    tainted = set()
    for n in range(16):
        if n == bad or p[n] in tainted:
            tainted.add(n)
    for n in range(16):
        if n in tainted:
            assert torch.isnan(got[0, n]).all() and torch.isnan(want[0, n]).all(), n
        else:
            assert torch.isfinite(got[0, n]).all(), n
            assert _rel(got[0, n], want[0, n]) <= GDN_RTOL, (n, _rel(got[0, n], want[0, n]))
