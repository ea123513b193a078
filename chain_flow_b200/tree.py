"""Tree verification around the draft: the target model's side of a tree step, on the sm_100a
kernels of libcfb.so (cfb_tree.cu).

* ``tree_attn_merge``: the tree-attention fix-up of one full-attention layer (the reference fork's
  ``suffix_merge``, src/chain_flow/patches/vllm-0.25.1-chain-flow-tree.patch:5516-5537; eager form
  ``_tree_suffix_eager`` :529-575 + vLLM's ``merge_attn_states``).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib

_DT = {torch.float16: 1, torch.bfloat16: 2}


def tree_attn_merge(query, key, value, output, prefix_out, prefix_lse, idx, not_anc, scale: float,
                    stream=None) -> torch.Tensor:
    """Each tree node attends to its ancestors (``not_anc[s, m, n] == 0``) and the result is merged by
    log-sum-exp with the paged-prefix attention (``prefix_out [S*N, H, D]``, ``prefix_lse [H, S*N]``);
    the merged rows are written into ``output`` at the nodes' query rows ``idx [S, N]``.
    query/output ``[T, H, D]``, key/value ``[T, HKV, D]``, fp16 or bf16. Returns ``output``."""
    lib = _lib.load()
    for t, n in ((query, "query"), (key, "key"), (value, "value"), (output, "output"), (prefix_out, "prefix_out"),
                 (prefix_lse, "prefix_lse"), (idx, "idx"), (not_anc, "not_anc")):
        _lib.require_cuda(t, n)
    dt = _DT.get(query.dtype)
    if dt is None or any(t.dtype != query.dtype for t in (key, value, output, prefix_out)):
        raise _lib.CfbError("tree_attn_merge: query/key/value/output/prefix_out must share fp16 or bf16")
    for t, n in ((query, "query"), (key, "key"), (value, "value"), (output, "output"), (prefix_out, "prefix_out")):
        if t.stride(2) != 1:
            raise _lib.CfbError(f"tree_attn_merge: {n} needs a contiguous head dim")
    S, N = idx.shape
    H, D = query.shape[1], query.shape[2]
    idx = idx.to(torch.int64).contiguous()
    not_anc = not_anc.to(torch.uint8).contiguous()
    prefix_lse = prefix_lse.to(torch.float32).contiguous()
    _lib.check(lib.cfb_tree_attn_merge(
        query.data_ptr(), query.stride(0), query.stride(1), key.data_ptr(), key.stride(0), key.stride(1),
        value.data_ptr(), value.stride(0), value.stride(1), output.data_ptr(), output.stride(0), output.stride(1),
        prefix_out.data_ptr(), prefix_out.stride(0), prefix_out.stride(1), prefix_lse.data_ptr(), idx.data_ptr(),
        not_anc.data_ptr(), float(scale), S, N, H, key.shape[1], D, dt, C.c_void_p(_lib.stream_ptr(stream))),
        "cfb_tree_attn_merge")
    return output


def ancestor_mask(parents: torch.Tensor) -> torch.Tensor:
    """[S, N] parents (-1 = the committed token, parent < child) -> [S, N, N] uint8 not-ancestor mask
    (0 where column n is node m itself or one of its ancestors), on the parents' device."""
    S, N = parents.shape
    anc = torch.eye(N, dtype=torch.bool, device=parents.device).unsqueeze(0).repeat(S, 1, 1)
    p = parents.long()
    for m in range(N):                       # BFS order: a parent's row is complete before its child's
        pm = p[:, m]
        has = pm >= 0
        rows = anc[torch.arange(S, device=parents.device), pm.clamp(min=0)]
        anc[:, m] |= rows & has.unsqueeze(1)
    return (~anc).to(torch.uint8)


class TreeVerifier:
    """Greedy tree verification (the reference fork's tree_rejection_sample,
    vllm-0.25.1-chain-flow-tree.patch:640-723) on cfb_tree_verify_greedy: one launch computes the
    argmax of every logits row and walks each request's draft tree. The workspace and outputs are
    allocated once for up to ``max_rows`` logits rows and ``max_batch`` requests and reused, so a
    call allocates nothing (CUDA-graph capturable)."""

    def __init__(self, max_rows: int, max_batch: int, max_spec_len: int, device=None):
        self.lib = _lib.load()
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.max_rows, self.max_batch, self.max_spec = max_rows, max_batch, max_spec_len
        nbytes = int(self.lib.cfb_tree_verify_workspace(max_rows, max_batch))
        self.ws = torch.zeros(nbytes + 256, dtype=torch.uint8, device=dev)
        self.ws_ptr = (self.ws.data_ptr() + 255) // 256 * 256
        self.ws_bytes = nbytes
        self.out_tokens = torch.empty(max_batch, max_spec_len + 1, dtype=torch.int32, device=dev)
        self.accepted_path = torch.empty(max_batch, max_spec_len, dtype=torch.int32, device=dev)
        self.accepted_len = torch.empty(max_batch, dtype=torch.int32, device=dev)
        self.row_argmax = torch.empty(max_rows, dtype=torch.int32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)

    def __call__(self, logits, cu_num_draft, cu_num_sampled, draft_tokens, parents, stream=None):
        """(output_tokens [B, max_spec + 1], accepted_path [B, max_spec], accepted_len [B]) int32
        views of this verifier's buffers, for B = len(cu_num_draft) requests."""
        for t, n in ((logits, "logits"), (cu_num_draft, "cu_num_draft"), (cu_num_sampled, "cu_num_sampled"),
                     (draft_tokens, "draft_tokens"), (parents, "parents")):
            _lib.require_cuda(t, n)
        dt = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}.get(logits.dtype)
        if dt is None or logits.stride(1) != 1:
            raise _lib.CfbError("logits: fp32 / fp16 / bf16 rows with a contiguous vocabulary dim")
        rows, V = logits.shape
        B = cu_num_draft.numel()
        if rows > self.max_rows or B > self.max_batch:
            raise _lib.CfbError(f"{rows} rows / {B} requests exceed this verifier ({self.max_rows} / {self.max_batch})")
        i32 = lambda t: t.to(torch.int32).contiguous()
        cu_d, cu_s, dtok, par = i32(cu_num_draft), i32(cu_num_sampled), i32(draft_tokens), i32(parents)
        _lib.check(self.lib.cfb_tree_verify_greedy(
            logits.data_ptr(), logits.stride(0), rows, V, dt, cu_d.data_ptr(), cu_s.data_ptr(), dtok.data_ptr(),
            par.data_ptr(), B, self.max_spec, self.out_tokens.data_ptr(), self.accepted_path.data_ptr(),
            self.accepted_len.data_ptr(), self.row_argmax.data_ptr(), C.c_void_p(self.ws_ptr), self.ws_bytes,
            self.err.data_ptr(), C.c_void_p(_lib.stream_ptr(stream))), "cfb_tree_verify_greedy")
        return self.out_tokens[:B], self.accepted_path[:B], self.accepted_len[:B]
