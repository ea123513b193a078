"""One persistent-kernel plan per (drafter weights, run shape): caller-owned, graph-stable buffers.

The reference keeps one scratch set per (expert, batch) and never resizes it because CUDA graphs
bake addresses (reference src/chain_flow/cuda_block.py:243-263, 382-388); a ``Plan`` is the
same contract for the whole draft: inputs, outputs and workspace are allocated here once, bound
into the phase table by ``cfb_plan_build``, and every ``run()`` is a single cooperative launch
with no allocation and no host synchronisation (capturable in a CUDA graph).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from .weights import DrafterWeights


def tree_levels(keep: int, topb: int, depth: int) -> list[int]:
    """Nodes added per tree level: depth 1 expands one node (reference flow_proposer.py:1315)."""
    fr, out = 1, []
    for _ in range(depth):
        k = min(keep, fr * topb)
        out.append(k)
        fr = k
    return out


def untile(buf: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """Row-major [rows, cols] view of a tiled fp16 activation buffer (layout in cfb.h)."""
    kp = (cols + 63) // 64 * 64
    t = buf.reshape(-1)[: rows * kp].view(kp // 64, rows, 8, 8)        # [slice, r, chunk, 8]
    r = torch.arange(rows, device=buf.device).view(1, rows, 1)
    c = torch.arange(8, device=buf.device).view(1, 1, 8)
    src = (c ^ (r & 7)).expand(kp // 64, rows, 8)                       # chunk holding logical c
    t = torch.gather(t, 2, src.unsqueeze(-1).expand(-1, -1, -1, 8))
    return t.permute(1, 0, 2, 3).reshape(rows, kp)[:, :cols]


class Plan:
    """With weights packed for a row-sharded head (DrafterWeights(head_shard=(rank, ranks))), every
    rank builds the same plan; ``run(group=...)`` then runs it segment by segment and all-gathers
    the ranks' merged top-k lists between segments (one small NCCL all_gather per beam depth)."""

    def __init__(self, w: DrafterWeights, mode: int, batch: int, *, width: int = 4, depth: int = 5,
                 tree_keep: int = 4, tree_topb: int = 8, grid: int = 0, profile: bool = False,
                 init_mode: int = 0, twopass_m: int = 0, wait_ns: int = 0):
        self.w, self.mode, self.batch = w, mode, batch
        cfg, dev = w.cfg, w.dev
        D = cfg.hidden
        self.lib = w.lib
        self.ctx = torch.zeros(batch, cfg.context_size, D, dtype=torch.float16, device=dev)
        self.z0 = torch.zeros(batch, cfg.draft_length, D, dtype=torch.float16, device=dev)
        self.known0 = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.pred = torch.zeros(batch, cfg.draft_length, D, dtype=torch.float32, device=dev)
        self.tree = mode in (_lib.MODE_TREE, _lib.MODE_BEAM_TREE)
        if self.tree:
            depth = min(depth, cfg.draft_length - 1)
            self.levels = tree_levels(tree_keep, tree_topb, depth)
            self.N = sum(self.levels)
            self.tokens = torch.zeros(batch, 2 * self.N, dtype=torch.int64, device=dev)
        else:
            self.N = depth
            self.tokens = torch.zeros(batch, depth, dtype=torch.int64, device=dev)
        r = _lib.Run()
        r.mode, r.batch, r.width, r.depth = mode, batch, width, depth
        r.init_mode = init_mode
        r.tree_keep, r.tree_topb, r.grid = tree_keep, tree_topb, grid
        r.flags = _lib.RUN_PROFILE if profile else 0
        r.twopass_m = twopass_m if mode != _lib.MODE_FLOW else 0
        r.wait_budget_ns = wait_ns
        self.twopass_m = r.twopass_m
        r.ctx, r.z0, r.known0 = self.ctx.data_ptr(), self.z0.data_ptr(), self.known0.data_ptr()
        r.pred, r.tokens = self.pred.data_ptr(), self.tokens.data_ptr()
        self.ranks = w.head_ranks
        if self.ranks > 1:
            self.xloc = torch.zeros(_lib.XROWS * _lib.XFLOATS, dtype=torch.float32, device=dev)
            self.xall = torch.zeros(self.ranks * _lib.XROWS * _lib.XFLOATS, dtype=torch.float32, device=dev)
            r.ranks, r.rank = self.ranks, w.head_rank
            r.xloc, r.xall = self.xloc.data_ptr(), self.xall.data_ptr()
        self.run_desc = r
        nbytes = C.c_size_t(0)
        _lib.check(self.lib.cfb_plan_workspace(C.byref(w.desc), C.byref(r), C.byref(nbytes)),
                   "cfb_plan_workspace")
        self.ws = torch.empty(int(nbytes.value) + 256, dtype=torch.uint8, device=dev)
        self.ws_ptr = (self.ws.data_ptr() + 255) // 256 * 256
        self.ws_bytes = int(nbytes.value)
        _lib.check(self.lib.cfb_plan_build(C.byref(w.desc), C.byref(r), C.c_void_p(self.ws_ptr),
                                           C.c_size_t(self.ws_bytes)), "cfb_plan_build")
        g, t, s, p = C.c_int(), C.c_int(), C.c_int(), C.c_int()
        _lib.check(self.lib.cfb_plan_info(C.c_void_p(self.ws_ptr), C.byref(g), C.byref(t), C.byref(s),
                                          C.byref(p)), "cfb_plan_info")
        self.grid, self.threads, self.smem, self.phases = g.value, t.value, s.value, p.value
        n = C.c_int()
        _lib.check(self.lib.cfb_plan_segments(C.c_void_p(self.ws_ptr), C.byref(n)), "cfb_plan_segments")
        self.segments = n.value

    def rebuild(self, wait_ns: int = 0) -> None:
        """Rebuild the plan in its own workspace (cfb_plan_build), with the given wait budget
        (0 = the default): clears the sticky device error word after a failed run."""
        torch.cuda.synchronize(self.ws.device)
        self.run_desc.wait_budget_ns = wait_ns
        _lib.check(self.lib.cfb_plan_build(C.byref(self.w.desc), C.byref(self.run_desc), C.c_void_p(self.ws_ptr),
                                           C.c_size_t(self.ws_bytes)), "cfb_plan_build")

    def run(self, stream=None, group=None) -> None:
        """One persistent launch on `stream` (default: torch's current stream); a sharded-head plan
        runs its segments with an all_gather over `group` (torch.distributed) between them."""
        sp = C.c_void_p(_lib.stream_ptr(stream))
        if self.segments == 1:
            _lib.check(self.lib.cfb_plan_run(C.c_void_p(self.ws_ptr), sp), "cfb_plan_run")
            return
        import torch.distributed as dist
        for seg in range(self.segments):
            _lib.check(self.lib.cfb_plan_run_segment(C.c_void_p(self.ws_ptr), seg, sp), "cfb_plan_run_segment")
            if seg + 1 < self.segments:
                if stream is not None and stream != torch.cuda.current_stream():
                    raise _lib.CfbError("a sharded-head plan runs on torch's current stream")
                dist.all_gather_into_tensor(self.xall, self.xloc, group=group)

    def buffer(self, which: int, dtype, shape) -> torch.Tensor:
        """A copy of one intermediate buffer of this plan (CFB_BUF_*), for stage-by-stage checks."""
        ptr, nbytes = C.c_void_p(), C.c_size_t()
        _lib.check(self.lib.cfb_plan_buffer(C.c_void_p(self.ws_ptr), which, C.byref(ptr), C.byref(nbytes)),
                   "cfb_plan_buffer")
        off = ptr.value - self.ws.data_ptr()
        n = 1
        for s_ in shape:
            n *= s_
        elt = torch.empty(0, dtype=dtype).element_size()
        if off < 0 or off + n * elt > self.ws.numel() or n * elt > nbytes.value:
            raise _lib.CfbError("buffer view out of range")
        return self.ws[off:off + n * elt].view(dtype).view(*shape).clone()

    def phase_times(self) -> torch.Tensor:
        """[phases, grid, 20] int64 ns of the last profiled run (see CFB_BUF_PROF in cfb.h).
        Needs a plan built with profile=True."""
        return self.buffer(_lib.BUF_PROF, torch.int64, (self.phases, self.grid, 20))

    def candidates(self) -> torch.Tensor:
        """[B, twopass_m] int32 copy of the two-pass head's candidate shortlist rows of the last
        run (CFB_BUF_TP_CAND), ascending per request."""
        return self.buffer(_lib.BUF_TP_CAND, torch.int32, (self.batch, self.twopass_m))

    def phase_table(self) -> torch.Tensor:
        """[phases, 15] int32 copy of the plan's phase table (CFB_BUF_PHASES in cfb.h): [:, 0] kind,
        [:, 6] post-op."""
        return self.buffer(_lib.BUF_PHASES, torch.int32, (self.phases, 15))

    def device_error(self) -> int:
        """Synchronous read of the plan's sticky device error word (0 = every run so far completed)."""
        v = C.c_int(0)
        self.lib.cfb_plan_error(C.c_void_p(self.ws_ptr), C.byref(v))
        return v.value

    def check(self) -> None:
        err = self.device_error()
        if err:
            raise _lib.CfbError(f"device-side failure (code {err}: {_lib.DEV_ERRORS.get(err, '?')}); "
                                f"outputs are invalid")


class WidePlan:
    """The wide (batched) plan over WideWeights: same inputs and outputs as ``Plan`` (ctx, z0,
    known0 -> pred, tokens), run as a fixed list of tcgen05 GEMM and row-kernel launches on one
    stream (capturable in a CUDA graph). For batches above what one persistent launch holds."""

    def __init__(self, w, mode: int, batch: int, *, width: int = 4, depth: int = 5, tree_keep: int = 4,
                 tree_topb: int = 8, init_mode: int = 0, wait_ns: int = 0):
        self.w, self.mode, self.batch = w, mode, batch
        cfg, dev = w.cfg, w.dev
        D = cfg.hidden
        self.lib = w.lib
        self.ctx = torch.zeros(batch, cfg.context_size, D, dtype=torch.float16, device=dev)
        self.z0 = torch.zeros(batch, cfg.draft_length, D, dtype=torch.float16, device=dev)
        self.known0 = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.pred = torch.zeros(batch, cfg.draft_length, D, dtype=torch.float32, device=dev)
        self.tree = mode in (_lib.MODE_TREE, _lib.MODE_BEAM_TREE)
        if self.tree:
            depth = min(depth, cfg.draft_length - 1)
            self.levels = tree_levels(tree_keep, tree_topb, depth)
            self.N = sum(self.levels)
            self.tokens = torch.zeros(batch, 2 * self.N, dtype=torch.int64, device=dev)
        else:
            self.N = depth
            self.tokens = torch.zeros(batch, depth, dtype=torch.int64, device=dev)
        r = _lib.Run()
        r.mode, r.batch, r.width, r.depth = mode, batch, width, depth
        r.init_mode = init_mode
        r.tree_keep, r.tree_topb = tree_keep, tree_topb
        r.wait_budget_ns = wait_ns
        r.ctx, r.z0, r.known0 = self.ctx.data_ptr(), self.z0.data_ptr(), self.known0.data_ptr()
        r.pred, r.tokens = self.pred.data_ptr(), self.tokens.data_ptr()
        self.run_desc = r
        nbytes = C.c_size_t(0)
        _lib.check(self.lib.cfb_wide_workspace(C.byref(w.desc), C.byref(r), C.byref(nbytes)), "cfb_wide_workspace")
        self.ws = torch.empty(int(nbytes.value) + 256, dtype=torch.uint8, device=dev)
        self.ws_ptr = (self.ws.data_ptr() + 255) // 256 * 256
        self.ws_bytes = int(nbytes.value)
        self._h = None
        self._create()

    def _create(self) -> None:
        h = C.c_void_p()
        _lib.check(self.lib.cfb_wide_create(C.byref(self.w.desc), C.byref(self.run_desc), C.c_void_p(self.ws_ptr),
                                            C.c_size_t(self.ws_bytes), C.byref(h)), "cfb_wide_create")
        self._h = h
        n = C.c_int()
        _lib.check(self.lib.cfb_wide_info(h, C.byref(n)), "cfb_wide_info")
        self.launches = n.value
        self.segments = 1

    def rebuild(self, wait_ns: int = 0) -> None:
        """Re-create the plan in its own workspace with the given wait budget (0 = the default):
        clears the sticky device error word after a failed run."""
        torch.cuda.synchronize(self.ws.device)
        if self._h is not None and self._h.value:
            self.lib.cfb_wide_destroy(self._h)
            self._h = None
        self.run_desc.wait_budget_ns = wait_ns
        self._create()

    def run(self, stream=None, group=None) -> None:
        if group is not None and self.w is not None and getattr(self.w, "head_ranks", 1) > 1:
            raise _lib.CfbError("the wide plan has no row-sharded head")
        _lib.check(self.lib.cfb_wide_run(self._h, C.c_void_p(_lib.stream_ptr(stream))), "cfb_wide_run")

    def device_error(self) -> int:
        v = C.c_int(0)
        _lib.check(self.lib.cfb_wide_error(self._h, C.byref(v)), "cfb_wide_error")
        return v.value

    def check(self) -> None:
        err = self.device_error()
        if err:
            raise _lib.CfbError(f"device-side failure (code {err}: {_lib.DEV_ERRORS.get(err, '?')}); "
                                f"outputs are invalid")

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            self.lib.cfb_wide_destroy(h)
            self._h = None
