"""The per-request context ring on the GPU (reference FlowDrafterProposer._init_ring /
_ring_write / _ring_gather, src/chain_flow/vllm_plugin/flow_proposer.py:881-961), over the
cfb_ring_write / cfb_ring_gather kernels. Every index stays on the GPU: no host sync, and the
buffers never move (CUDA-graph capturable)."""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib


class ContextRing:
    def __init__(self, slots: int, ctx_size: int, hidden: int, device=None, dtype=torch.float16):
        if dtype != torch.float16:
            raise _lib.CfbError("the context ring holds fp16 hidden states")
        self.lib = _lib.load()
        self.slots, self.C, self.H = slots, ctx_size, hidden
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.ring = torch.zeros(slots, ctx_size + 1, hidden, dtype=dtype, device=dev)
        self.rpos = torch.zeros(slots, dtype=torch.long, device=dev)     # next write position
        self.nval = torch.zeros(slots, dtype=torch.long, device=dev)     # valid rows, <= C

    def write(self, sh, rows, starts, cnt, wmask, path, kmax: int, stream=None) -> None:
        """Append each request's accepted hidden states (reference _ring_write, :916-945)."""
        for t, n in ((sh, "sh"), (rows, "rows"), (starts, "starts"), (cnt, "cnt"), (wmask, "wmask")):
            _lib.require_cuda(t, n)
        sh = sh.to(torch.float16).contiguous()
        rows, starts, cnt = (t.to(torch.long).contiguous() for t in (rows, starts, cnt))
        wmask = wmask.to(torch.bool).contiguous()
        if path is not None:
            path = path.to(torch.long).contiguous()
        _lib.check(self.lib.cfb_ring_write(
            self.ring.data_ptr(), self.rpos.data_ptr(), self.nval.data_ptr(), self.slots, self.C, self.H,
            sh.data_ptr(), sh.shape[0], rows.data_ptr(), starts.data_ptr(), cnt.data_ptr(), wmask.data_ptr(),
            path.data_ptr() if path is not None else None, path.shape[1] if path is not None else 0,
            rows.numel(), kmax, C.c_void_p(_lib.stream_ptr(stream))), "cfb_ring_write")

    def gather(self, rows, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """[B, C, H] fp16 context windows, oldest first, front-padded (reference _ring_gather, :947-961)."""
        _lib.require_cuda(rows, "rows")
        rows = rows.to(torch.long).contiguous()
        if out is None:
            out = torch.empty(rows.numel(), self.C, self.H, dtype=torch.float16, device=self.ring.device)
        _lib.check(self.lib.cfb_ring_gather(
            self.ring.data_ptr(), self.rpos.data_ptr(), self.nval.data_ptr(), self.slots, self.C, self.H,
            rows.data_ptr(), rows.numel(), out.data_ptr(), C.c_void_p(_lib.stream_ptr(stream))), "cfb_ring_gather")
        return out
