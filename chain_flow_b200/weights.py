"""Drafter weights in the engine's device layout.

``DrafterWeights`` takes a ``TreeFlowDrafter`` state dict (the reference checkpoint's parameter
names, i.e. the ``drafter.``-prefixed keys of ``model.safetensors`` with the prefix removed,
reference src/chain_flow/vllm_plugin/flow_proposer.py:638-648) plus the target model's input
embedding and ``lm_head`` and the shortlist ids, and prepares everything once on the GPU with
the C-ABI packing kernels:

* every Linear -> packed fp16 stream layout, with the LayerNorm in front of it folded in
  (gamma into the columns, beta into the bias, column sums for the mean correction);
* ``time_mlp`` evaluated at every Euler step's tau (it is the same for every row);
* the shortlist head ``[lm_head[sl] | markov.w2[sl]]`` packed as ONE [R, D + rank] matrix, so the
  head GEMV and the markov bias are a single stream (reference flow_proposer.py:739-740, 1021-1025);
* the PathHead offset projections packed side by side as one [D, order*D] matrix
  (the batched form of reference vllm_plugin/fused.py:14-39).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib


@dataclass
class DraftConfig:
    """The ``TreeFlowConfig`` fields the drafting path needs (reference tree_flow.py:39-72)."""
    hidden: int
    context_size: int = 8
    draft_length: int = 6
    chunk_size: int = 3
    num_heads: int = 8
    ffn_multiplier: int = 6
    num_drafter_layers: int = 4
    num_flow_steps: int = 8
    path_order: int = 4
    path_ffn_multiplier: int = 2
    markov_rank: int = 256

    @property
    def n_experts(self) -> int:
        return self.draft_length // self.chunk_size

    @staticmethod
    def from_model_args(args: dict, hidden: int) -> "DraftConfig":
        keys = {f for f in DraftConfig.__dataclass_fields__ if f != "hidden"}
        return DraftConfig(hidden=hidden, **{k: v for k, v in args.items() if k in keys})


def expert_prefix(e: int) -> str:
    return "expert." if e == 0 else f"extra_experts.{e - 1}."


def shard_rows(rows: int, ranks: int, rank: int) -> tuple[int, int]:
    """(first row, row count) of rank `rank`'s contiguous share of a `rows`-row head."""
    if ranks < 1 or not 0 <= rank < ranks:
        raise ValueError(f"rank {rank} of {ranks}")
    r0, r1 = rank * rows // ranks, (rank + 1) * rows // ranks
    return r0, r1 - r0


class EnginePacker:
    """Packs fp16 weights into the persistent engine's stream layout (cfb_pack_linear) on `dev`,
    folding the LayerNorm that feeds a Linear into it (gamma into the columns, beta into the bias,
    column sums for the mean correction: cfb_fold_bias). Every device buffer is appended to
    `keep`."""

    def __init__(self, lib, dev, keep: list, stream=None):
        self.lib, self.dev, self.keep = lib, dev, keep
        self.stream = stream if stream is not None else torch.cuda.current_stream(dev)

    def pack_buffer(self, nout: int, k: int) -> torch.Tensor:
        nbytes = self.lib.cfb_packed_bytes(nout, k)
        buf = torch.zeros(nbytes, dtype=torch.uint8, device=self.dev)
        self.keep.append(buf)
        return buf

    def pack_into(self, w16: torch.Tensor, buf: torch.Tensor, nout: int, k: int, ktotal: int, kofs: int,
                  rows: torch.Tensor | None = None, gamma: torch.Tensor | None = None):
        _lib.check(self.lib.cfb_pack_linear(
            w16.data_ptr(), w16.stride(0), rows.data_ptr() if rows is not None else None, nout, k,
            gamma.data_ptr() if gamma is not None else None, buf.data_ptr(), ktotal, kofs,
            self.stream.cuda_stream), "cfb_pack_linear")

    def linear(self, w16: torch.Tensor, bias32: torch.Tensor | None, ln=None) -> "_lib.Linear":
        """Pack one nn.Linear (optionally with the LayerNorm (gamma, beta) that feeds it)."""
        w16 = w16.to(device=self.dev, dtype=torch.float16).contiguous()
        if bias32 is not None:
            bias32 = bias32.to(device=self.dev, dtype=torch.float32).contiguous()
        if ln is not None:
            ln = tuple(t.to(device=self.dev, dtype=torch.float32).contiguous() for t in ln)
        nout, k = w16.shape
        buf = self.pack_buffer(nout, k)
        gamma = ln[0] if ln is not None else None
        self.pack_into(w16, buf, nout, k, k, 0, gamma=gamma)
        colsum = None
        if ln is not None:
            b_out = torch.empty(nout, device=self.dev, dtype=torch.float32)
            colsum = torch.empty(nout, device=self.dev, dtype=torch.float32)
            _lib.check(self.lib.cfb_fold_bias(
                w16.data_ptr(), w16.stride(0), nout, k, ln[0].data_ptr(), ln[1].data_ptr(),
                bias32.data_ptr() if bias32 is not None else None, b_out.data_ptr(), colsum.data_ptr(),
                self.stream.cuda_stream), "cfb_fold_bias")
            bias32 = b_out
            self.keep.append(colsum)
        if bias32 is not None:
            self.keep.append(bias32)
        return _lib.Linear(buf.data_ptr(), bias32.data_ptr() if bias32 is not None else None,
                           colsum.data_ptr() if colsum is not None else None, nout, k)


class DrafterWeights:
    """The drafter's weights packed for the engine. With head_shard=(rank, ranks) only that rank's
    contiguous share of the shortlist head is packed (row-sharded head across GPUs); everything
    else is replicated. ``parts`` selects what is packed: "all", "flow" (the experts only: a
    FLOW-mode plan, e.g. the production drafter's flow in its VAE latent space, where cfg.hidden is
    the latent width) or "head" (path head, markov and shortlist head only: a BEAM-mode plan at the
    target's hidden width)."""

    def __init__(self, sd: dict, cfg: DraftConfig, embed: torch.Tensor | None, lm_head: torch.Tensor | None,
                 shortlist: torch.Tensor | None, device=None, head_shard: tuple[int, int] | None = None,
                 parts: str = "all"):
        self.lib = _lib.load()
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if dev.type != "cuda":
            raise _lib.CfbError("DrafterWeights needs a CUDA device: the engine has no CPU path")
        if parts not in ("all", "flow", "head"):
            raise ValueError(f"parts={parts!r}")
        self.dev, self.cfg, self.parts = dev, cfg, parts
        D = cfg.hidden
        if D % 64 or cfg.draft_length % cfg.chunk_size:
            raise _lib.CfbError(f"unsupported drafter shape: hidden={D} must be a multiple of 64")
        self._keep = []            # every device tensor the packed structs point at
        self.stream = torch.cuda.current_stream(dev)
        self._pk = EnginePacker(self.lib, dev, self._keep, self.stream)
        f16 = lambda t: t.to(device=dev, dtype=torch.float16).contiguous()
        f32 = lambda t: t.to(device=dev, dtype=torch.float32).contiguous()
        want = {"all": None, "flow": ("expert.", "extra_experts."), "head": ("path_head.", "markov.")}[parts]
        self.sd16 = {k: f16(v) for k, v in sd.items() if want is None or k.startswith(want)}
        self.sd32 = {}

        def p32(name):
            if name not in self.sd32:
                self.sd32[name] = f32(sd[name])
            return self.sd32[name]

        self.experts = (_lib.Expert * cfg.n_experts)()
        self._blocks = []
        if parts != "head":
            for e in range(cfg.n_experts):
                p = expert_prefix(e)
                blocks = (_lib.Block * cfg.num_drafter_layers)()
                for l in range(cfg.num_drafter_layers):
                    b = f"{p}blocks.{l}."
                    w_in = self.sd16[b + "self_attn.in_proj_weight"]
                    b_in = p32(b + "self_attn.in_proj_bias")
                    cw = self.sd16[b + "cross_attn.in_proj_weight"]
                    cb = p32(b + "cross_attn.in_proj_bias")
                    blocks[l].qkv = self.linear(w_in, b_in, ln=(p32(b + "self_norm.weight"), p32(b + "self_norm.bias")))
                    blocks[l].self_out = self.linear(self.sd16[b + "self_attn.out_proj.weight"], p32(b + "self_attn.out_proj.bias"))
                    blocks[l].cross_q = self.linear(cw[:D], cb[:D], ln=(p32(b + "cross_norm.weight"), p32(b + "cross_norm.bias")))
                    blocks[l].cross_kv = self.linear(cw[D:], cb[D:], ln=(p32(b + "context_norm.weight"), p32(b + "context_norm.bias")))
                    blocks[l].cross_out = self.linear(self.sd16[b + "cross_attn.out_proj.weight"], p32(b + "cross_attn.out_proj.bias"))
                    blocks[l].ffn_up = self.linear(self.sd16[b + "ffn.1.weight"], p32(b + "ffn.1.bias"), ln=(p32(b + "ffn.0.weight"), p32(b + "ffn.0.bias")))
                    blocks[l].ffn_down = self.linear(self.sd16[b + "ffn.4.weight"], p32(b + "ffn.4.bias"))
                self._blocks.append(blocks)
                ex = self.experts[e]
                pos = p32(p + "position_embedding.weight")
                temb = torch.empty(cfg.num_flow_steps, D, device=dev, dtype=torch.float32)
                _lib.check(self.lib.cfb_time_embed(
                    p32(p + "time_mlp.0.weight")[:, 0].contiguous().data_ptr(), p32(p + "time_mlp.0.bias").data_ptr(),
                    self.sd16[p + "time_mlp.2.weight"].data_ptr(), p32(p + "time_mlp.2.bias").data_ptr(),
                    D, cfg.num_flow_steps, temb.data_ptr(), self.stream.cuda_stream), "cfb_time_embed")
                self._keep += [pos, temb]
                ex.pos_emb, ex.temb = pos.data_ptr(), temb.data_ptr()
                ex.out_proj = self.linear(self.sd16[p + "out_proj.weight"], p32(p + "out_proj.bias"),
                                          ln=(p32(p + "out_norm.weight"), p32(p + "out_norm.bias")))
                ex.blocks = C.cast(blocks, C.POINTER(_lib.Block))

        # ---- path head, markov bias, shortlist head
        self.embed, self.vocab, self.shortlist, self.R = None, 0, None, 0
        self.head_rank, self.head_ranks, self.head_row0 = 0, 1, 0
        if parts != "flow":
            self.embed = f16(embed)
            self.vocab = self.embed.shape[0]
            sl = shortlist.to(device=dev, dtype=torch.int64).contiguous()
            self.shortlist = sl
            R = sl.numel()
            rank = cfg.markov_rank

            order = cfg.path_order
            po = self.pack_buffer(D, order * D)
            for j in range(order):
                self._pack_into(self.sd16[f"path_head.offset_proj.{j}.weight"], po, D, D, order * D, j * D)
            self.path_offsets = _lib.Linear(po.data_ptr(), None, None, D, order * D)
            self.path_offset_bias = torch.stack([p32(f"path_head.offset_proj.{j}.bias") for j in range(order)]).contiguous()
            self._keep.append(self.path_offset_bias)
            self.path_up = self.linear(self.sd16["path_head.mlp.0.weight"], p32("path_head.mlp.0.bias"),
                                       ln=(p32("path_head.norm.weight"), p32("path_head.norm.bias")))
            self.path_down = self.linear(self.sd16["path_head.mlp.3.weight"], p32("path_head.mlp.3.bias"))
            self.markov_w1 = self.sd16["markov.w1.weight"]
            self.head_rank, self.head_ranks = head_shard if head_shard is not None else (0, 1)
            self.head_row0, hrows = shard_rows(R, self.head_ranks, self.head_rank)
            rows_sl = sl[self.head_row0:self.head_row0 + hrows].contiguous()
            hb = self.pack_buffer(hrows, D + rank)
            lm16 = lm_head if lm_head.device == dev and lm_head.dtype == torch.float16 else None
            if lm16 is None:
                # only the rows this rank packs travel to the device
                lm16 = lm_head[rows_sl.to(lm_head.device)].to(device=dev, dtype=torch.float16).contiguous()
                self._pack_into(lm16, hb, hrows, D, D + rank, 0)
            else:
                self._pack_into(lm16, hb, hrows, D, D + rank, 0, rows=rows_sl)
            self._pack_into(self.sd16["markov.w2.weight"], hb, hrows, rank, D + rank, D, rows=rows_sl)
            del lm16
            self.head = _lib.Linear(hb.data_ptr(), None, None, hrows, D + rank)
            self.R = R

        d = _lib.Drafter()
        d.hidden, d.heads, d.layers, d.steps = D, cfg.num_heads, cfg.num_drafter_layers, cfg.num_flow_steps
        d.draft_len, d.chunk, d.ctx_rows, d.n_experts = cfg.draft_length, cfg.chunk_size, cfg.context_size, cfg.n_experts
        if parts != "head":
            d.experts = C.cast(self.experts, C.POINTER(_lib.Expert))
        d.path_order, d.markov_rank = cfg.path_order, cfg.markov_rank
        if parts != "flow":
            d.vocab, d.shortlist_rows = self.vocab, self.R
            d.embed = self.embed.data_ptr()
            d.path_offsets = self.path_offsets
            d.path_offset_bias = self.path_offset_bias.data_ptr()
            d.path_up, d.path_down = self.path_up, self.path_down
            d.markov_w1 = self.markov_w1.data_ptr()
            d.head = self.head
            d.shortlist = self.shortlist.data_ptr()
            d.head_row0 = self.head_row0
        self.desc = d
        # the raw fp16 state dict is no longer needed except the tables the engine reads
        keep = {"markov.w1.weight"}
        self.sd16 = {k: v for k, v in self.sd16.items() if k in keep}
        self.sd32 = {}
        torch.cuda.synchronize(dev)

    # ------------------------------------------------------------------------------------------
    def pack_buffer(self, nout: int, k: int) -> torch.Tensor:
        return self._pk.pack_buffer(nout, k)

    def _pack_into(self, w16, buf, nout, k, ktotal, kofs, rows=None, gamma=None):
        self._pk.pack_into(w16, buf, nout, k, ktotal, kofs, rows=rows, gamma=gamma)

    def linear(self, w16: torch.Tensor, bias32: torch.Tensor | None, ln=None) -> "_lib.Linear":
        """Pack one nn.Linear (optionally with the LayerNorm (gamma, beta) that feeds it)."""
        return self._pk.linear(w16, bias32, ln)

    @property
    def packed_bytes(self) -> int:
        """Bytes of packed weight buffers (what the engine streams)."""
        return sum(t.numel() for t in self._keep if t.dtype == torch.uint8)

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self._keep) + (self.embed.numel() * 2 if self.embed is not None else 0)


class WidePacker:
    """Packs fp16 weights into the wide GEMM's tiled layout (cfb_wide_pack) on `dev`, folding the
    LayerNorm that feeds a Linear into it: w = fp16(W16 * gamma), bias = b + W16 beta (the
    persistent engine's folding rule). Every device buffer is appended to `keep`."""

    def __init__(self, lib, dev, keep: list):
        self.lib, self.dev, self.keep = lib, dev, keep
        self.stream = torch.cuda.current_stream(dev)

    def pack(self, w16: torch.Tensor) -> torch.Tensor:
        """row-major fp16 [nout, k] -> the wide GEMM's tiled layout"""
        nout, k = w16.shape
        buf = torch.empty(self.lib.cfb_wide_packed_bytes(nout, k), dtype=torch.uint8, device=self.dev)
        _lib.check(self.lib.cfb_wide_pack(w16.data_ptr(), w16.stride(0), nout, k, buf.data_ptr(),
                                          self.stream.cuda_stream), "cfb_wide_pack")
        self.keep.append(buf)
        return buf

    def linear(self, w, b, ln=None) -> "_lib.Linear":
        w16 = w.to(device=self.dev, dtype=torch.float16).contiguous()
        bias = (b.to(device=self.dev, dtype=torch.float32) if b is not None
                else torch.zeros(w16.shape[0], device=self.dev))
        if ln is not None:
            g = ln[0].to(device=self.dev, dtype=torch.float32)
            beta = ln[1].to(device=self.dev, dtype=torch.float32)
            bias = bias + w16.float() @ beta
            w16 = (w16.float() * g).to(torch.float16).contiguous()
        bias = bias.contiguous()
        self.keep.append(bias)
        buf = self.pack(w16)         # w16 may be freed after this: the allocator orders reuse on the stream
        return _lib.Linear(buf.data_ptr(), bias.data_ptr(), None, w16.shape[0], w16.shape[1])


class WideWeights:
    """The drafter's weights for the wide (batched, tcgen05) plan: every Linear as an fp16 [nout, k]
    matrix in the wide GEMM's tiled layout (cfb_wide_pack), with the LayerNorm that feeds it folded in (w = fp16(W16 * gamma),
    bias = b + W16 beta, the same folding as the persistent engine's packing), the time MLP
    evaluated at every Euler step, the path offsets side by side as [D, order * D], and the
    shortlist head [lm_head[sl] | markov.w2[sl]] as one [R, D + rank] matrix. ``parts`` as for
    DrafterWeights ("all", "flow" or "head")."""

    def __init__(self, sd: dict, cfg: DraftConfig, embed: torch.Tensor | None, lm_head: torch.Tensor | None,
                 shortlist: torch.Tensor | None, device=None, parts: str = "all"):
        self.lib = _lib.load()
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if dev.type != "cuda":
            raise _lib.CfbError("WideWeights needs a CUDA device: the wide path has no CPU path")
        if parts not in ("all", "flow", "head"):
            raise ValueError(f"parts={parts!r}")
        self.dev, self.cfg, self.parts = dev, cfg, parts
        D = cfg.hidden
        if D % 64 or cfg.draft_length % cfg.chunk_size:
            raise _lib.CfbError(f"unsupported drafter shape: hidden={D} must be a multiple of 64")
        self._keep = []
        stream = torch.cuda.current_stream(dev)
        f32 = lambda t: t.to(device=dev, dtype=torch.float32).contiguous()
        f16 = lambda t: t.to(device=dev, dtype=torch.float16).contiguous()

        packer = WidePacker(self.lib, dev, self._keep)
        pack, linear = packer.pack, packer.linear

        self.experts = (_lib.Expert * cfg.n_experts)()
        self._blocks = []
        if parts != "head":
            for e in range(cfg.n_experts):
                p = expert_prefix(e)
                blocks = (_lib.Block * cfg.num_drafter_layers)()
                for l in range(cfg.num_drafter_layers):
                    b = f"{p}blocks.{l}."
                    cw, cb = sd[b + "cross_attn.in_proj_weight"], sd[b + "cross_attn.in_proj_bias"]
                    blocks[l].qkv = linear(sd[b + "self_attn.in_proj_weight"], sd[b + "self_attn.in_proj_bias"],
                                           ln=(sd[b + "self_norm.weight"], sd[b + "self_norm.bias"]))
                    blocks[l].self_out = linear(sd[b + "self_attn.out_proj.weight"], sd[b + "self_attn.out_proj.bias"])
                    blocks[l].cross_q = linear(cw[:D], cb[:D], ln=(sd[b + "cross_norm.weight"], sd[b + "cross_norm.bias"]))
                    blocks[l].cross_kv = linear(cw[D:], cb[D:], ln=(sd[b + "context_norm.weight"], sd[b + "context_norm.bias"]))
                    blocks[l].cross_out = linear(sd[b + "cross_attn.out_proj.weight"], sd[b + "cross_attn.out_proj.bias"])
                    blocks[l].ffn_up = linear(sd[b + "ffn.1.weight"], sd[b + "ffn.1.bias"],
                                              ln=(sd[b + "ffn.0.weight"], sd[b + "ffn.0.bias"]))
                    blocks[l].ffn_down = linear(sd[b + "ffn.4.weight"], sd[b + "ffn.4.bias"])
                self._blocks.append(blocks)
                ex = self.experts[e]
                pos = f32(sd[p + "position_embedding.weight"])
                temb = torch.empty(cfg.num_flow_steps, D, device=dev, dtype=torch.float32)
                w1t, b1t = f32(sd[p + "time_mlp.0.weight"][:, 0]), f32(sd[p + "time_mlp.0.bias"])
                w2t, b2t = f16(sd[p + "time_mlp.2.weight"]), f32(sd[p + "time_mlp.2.bias"])
                _lib.check(self.lib.cfb_time_embed(w1t.data_ptr(), b1t.data_ptr(), w2t.data_ptr(), b2t.data_ptr(),
                                                   D, cfg.num_flow_steps, temb.data_ptr(), stream.cuda_stream),
                           "cfb_time_embed")
                self._keep += [pos, temb, w1t, b1t, w2t, b2t]
                ex.pos_emb, ex.temb = pos.data_ptr(), temb.data_ptr()
                ex.out_proj = linear(sd[p + "out_proj.weight"], sd[p + "out_proj.bias"],
                                     ln=(sd[p + "out_norm.weight"], sd[p + "out_norm.bias"]))
                ex.blocks = C.cast(blocks, C.POINTER(_lib.Block))
        self.embed, self.vocab, self.shortlist, self.R = None, 0, None, 0
        pb = None
        if parts != "flow":
            self.embed = f16(embed)
            self.vocab = self.embed.shape[0]
            sl = shortlist.to(device=dev, dtype=torch.int64).contiguous()
            self.shortlist = sl
            R, rank = sl.numel(), cfg.markov_rank
            order = cfg.path_order
            po = pack(torch.cat([f16(sd[f"path_head.offset_proj.{j}.weight"]) for j in range(order)], dim=1).contiguous())
            pb = torch.stack([f32(sd[f"path_head.offset_proj.{j}.bias"]) for j in range(order)]).contiguous()
            self._keep.append(pb)
            self.path_offsets = _lib.Linear(po.data_ptr(), None, None, D, order * D)
            self.path_up = linear(sd["path_head.mlp.0.weight"], sd["path_head.mlp.0.bias"],
                                  ln=(sd["path_head.norm.weight"], sd["path_head.norm.bias"]))
            self.path_down = linear(sd["path_head.mlp.3.weight"], sd["path_head.mlp.3.bias"])
            self.markov_w1 = f16(sd["markov.w1.weight"])
            rows = sl.to(lm_head.device)
            kh = (D + rank + 63) // 64 * 64          # zero columns pad the head's K to a multiple of 64
            head = torch.zeros(R, kh, dtype=torch.float16, device=dev)
            head[:, :D] = lm_head[rows].to(device=dev, dtype=torch.float16)
            head[:, D:D + rank] = f16(sd["markov.w2.weight"])[sl]
            hp = pack(head)
            self._keep.append(self.markov_w1)
            self.head = _lib.Linear(hp.data_ptr(), None, None, R, kh)
            del head
            self.R = R
        d = _lib.Drafter()
        d.hidden, d.heads, d.layers, d.steps = D, cfg.num_heads, cfg.num_drafter_layers, cfg.num_flow_steps
        d.draft_len, d.chunk, d.ctx_rows, d.n_experts = cfg.draft_length, cfg.chunk_size, cfg.context_size, cfg.n_experts
        if parts != "head":
            d.experts = C.cast(self.experts, C.POINTER(_lib.Expert))
        d.path_order, d.markov_rank = cfg.path_order, cfg.markov_rank
        if parts != "flow":
            d.vocab, d.shortlist_rows = self.vocab, self.R
            d.embed = self.embed.data_ptr()
            d.path_offsets = self.path_offsets
            d.path_offset_bias = pb.data_ptr()
            d.path_up, d.path_down = self.path_up, self.path_down
            d.markov_w1 = self.markov_w1.data_ptr()
            d.head = self.head
            d.shortlist = self.shortlist.data_ptr()
        d.head_row0 = 0
        self.desc = d
        torch.cuda.synchronize(dev)

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self._keep) + (self.embed.numel() * 2 if self.embed is not None else 0)
