"""CPU tests of the C ABI: the library loads, exports every symbol include/cfb.h declares, and the
native plan lowering (which never dereferences device pointers) sizes workspaces and rejects
unsupported shapes without a GPU."""
import ctypes as C
import re
from pathlib import Path

import pytest

from chain_flow_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "cfb.h").read_text()
    return sorted(set(re.findall(r"\b(cfb_[a-z_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert sorted(_lib.EXPORTED) == declared_symbols()


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.cfb_abi_version() == _lib.ABI_VERSION == 5


def test_packed_bytes():
    lib = _lib.load()
    assert lib.cfb_packed_bytes(64, 16) == 64 * 64 * 2           # k padded to 64
    assert lib.cfb_packed_bytes(65, 32) == 128 * 64 * 2          # rows padded to 64
    assert lib.cfb_packed_bytes(62642, 2816) == 62656 * 2816 * 2
    assert lib.cfb_packed_bytes(64, 15) == 0                     # k must be a multiple of 16


FAKE = 0x10000                       # host-side lowering only does pointer arithmetic


def fake_linear(nout, k, ln=False):
    return _lib.Linear(FAKE, FAKE, FAKE if ln else None, nout, k)


def fake_drafter(D=2560, L=4, T=8, FM=6, R=62642, rank=256, order=4):
    blocks = []
    experts = (_lib.Expert * 2)()
    for e in range(2):
        bl = (_lib.Block * L)()
        for l in range(L):
            bl[l] = _lib.Block(fake_linear(3 * D, D, True), fake_linear(D, D), fake_linear(D, D, True),
                               fake_linear(2 * D, D, True), fake_linear(D, D), fake_linear(FM * D, D, True),
                               fake_linear(D, FM * D))
        blocks.append(bl)
        experts[e] = _lib.Expert(FAKE, FAKE, fake_linear(D, D, True), C.cast(bl, C.POINTER(_lib.Block)))
    d = _lib.Drafter()
    d.hidden, d.heads, d.layers, d.steps, d.draft_len, d.chunk, d.ctx_rows, d.n_experts = D, 8, L, T, 6, 3, 8, 2
    d.experts = C.cast(experts, C.POINTER(_lib.Expert))
    d.path_order, d.markov_rank, d.vocab, d.shortlist_rows = order, rank, 248320, R
    d.embed = FAKE
    d.path_offsets = fake_linear(D, order * D)
    d.path_offset_bias = FAKE
    d.path_up = fake_linear(2 * D, D, True)
    d.path_down = fake_linear(D, 2 * D)
    d.markov_w1 = FAKE
    d.head = fake_linear(R, D + rank)
    d.shortlist = FAKE
    return d, (experts, blocks)


def fake_run(mode, B, grid=148, ranks=1):
    r = _lib.Run()
    r.mode, r.batch, r.width, r.depth, r.tree_keep, r.tree_topb, r.grid = mode, B, 4, 5, 4, 8, grid
    r.ctx = r.z0 = r.known0 = r.pred = r.tokens = FAKE
    r.ranks, r.rank = ranks, 0
    if ranks > 1:
        r.xloc = r.xall = FAKE
    return r


@pytest.mark.parametrize("mode", [_lib.MODE_FLOW, _lib.MODE_CHAIN, _lib.MODE_TREE,
                                  _lib.MODE_BEAM_CHAIN, _lib.MODE_BEAM_TREE])
def test_plan_workspace_sizes(mode):
    lib = _lib.load()
    d, keep = fake_drafter()
    for B in (1, 8):
        n = C.c_size_t(0)
        st = lib.cfb_plan_workspace(C.byref(d), C.byref(fake_run(mode, B)), C.byref(n))
        assert st == 0, _lib.STATUS_NAMES[st]
        assert 0 < n.value < 512 << 20


def test_plan_rejects_unsupported_shapes():
    lib = _lib.load()
    n = C.c_size_t(0)
    d, keep = fake_drafter(D=2560)
    assert lib.cfb_plan_workspace(C.byref(d), C.byref(fake_run(_lib.MODE_CHAIN, 11)), C.byref(n)) == 2  # 66 rows
    r = fake_run(_lib.MODE_CHAIN, 1); r.width = 9
    assert lib.cfb_plan_workspace(C.byref(d), C.byref(r), C.byref(n)) == 2                           # top-k > 8
    r = fake_run(_lib.MODE_CHAIN, 1); r.depth = 6
    assert lib.cfb_plan_workspace(C.byref(d), C.byref(r), C.byref(n)) == 2                           # > draft_len-1
    d2, keep2 = fake_drafter(D=2560 + 32)
    assert lib.cfb_plan_workspace(C.byref(d2), C.byref(fake_run(_lib.MODE_FLOW, 1)), C.byref(n)) == 2
    r = fake_run(_lib.MODE_CHAIN, 1); r.pred = None
    assert lib.cfb_plan_workspace(C.byref(d), C.byref(r), C.byref(n)) == 1


def test_untile_inverts_the_tiled_activation_layout():
    """The tiled fp16 activation layout documented in cfb.h, and engine.untile's inverse."""
    import torch
    from chain_flow_b200.engine import untile
    for R, K in ((6, 2560), (4, 160), (3, 64), (8, 256)):
        kp = (K + 127) // 128 * 128
        x = torch.randn(R, K)
        buf = torch.full((R * kp,), float("nan"))
        for r in range(R):
            for k in range(K):
                idx = ((k >> 6) * R + r) * 64 + ((((k & 63) >> 3) ^ (r & 7)) << 3) + (k & 7)
                buf[idx] = x[r, k]
        assert torch.equal(untile(buf, R, K), x)


@pytest.mark.parametrize("ranks", [2, 4, 8])
def test_sharded_head_plans(ranks):
    """A row-sharded 27B-shaped head: each rank packs rows [row0, row0 + n) of the shortlist;
    the plan needs the exchange buffers, and refuses a shard on a single GPU."""
    lib = _lib.load()
    R = 62642
    n = C.c_size_t(0)
    for rank in range(ranks):
        row0, rows = rank * R // ranks, (rank + 1) * R // ranks - rank * R // ranks
        d, keep = fake_drafter(D=5120, R=R)
        d.head = fake_linear(rows, 5120 + 256)
        d.head_row0 = row0
        r = fake_run(_lib.MODE_CHAIN, 1, ranks=ranks)
        r.rank = rank
        assert lib.cfb_plan_workspace(C.byref(d), C.byref(r), C.byref(n)) == 0
        r.xall = None
        assert lib.cfb_plan_workspace(C.byref(d), C.byref(r), C.byref(n)) == 1      # no exchange buffer
        assert lib.cfb_plan_workspace(C.byref(d), C.byref(fake_run(_lib.MODE_CHAIN, 1)), C.byref(n)) == 1
