"""Seeded synthetic drafters and inputs with the shapes of the benchmark configurations.

There are no checkpoints or datasets on the benchmark machines, so the benchmark drafters are
random-initialised with the reference architecture (``TreeFlowDrafter`` state-dict names and
shapes): matrices ~N(0, 0.02), LayerNorm gamma ~1 + N(0, 0.1) and beta ~N(0, 0.1), the
zero-initialised PathHead output layer and markov ``w2`` (reference tree_flow.py:95-96,
markov_flow.py:69) seeded non-zero so they carry weight, target embedding / lm_head ~N(0, 0.02)
(lm_head) and N(0, 0.5) (embedding), a seeded shortlist of unique ids.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .weights import DraftConfig


@dataclass
class Workload:
    name: str
    hidden: int
    layers: int
    steps: int
    ffn: int = 6
    vocab: int = 248320
    shortlist_rows: int = 62642
    markov_rank: int = 256
    width: int = 4
    draft_tokens: int = 5

    def config(self) -> DraftConfig:
        return DraftConfig(hidden=self.hidden, context_size=8, draft_length=6, chunk_size=3, num_heads=8,
                           ffn_multiplier=self.ffn, num_drafter_layers=self.layers, num_flow_steps=self.steps,
                           path_order=4, path_ffn_multiplier=2, markov_rank=self.markov_rank)

    def model_args(self) -> dict:
        c = self.config()
        return dict(context_size=c.context_size, draft_length=c.draft_length, chunk_size=c.chunk_size,
                    num_heads=c.num_heads, ffn_multiplier=c.ffn_multiplier,
                    num_drafter_layers=c.num_drafter_layers, num_flow_steps=c.num_flow_steps,
                    path_order=c.path_order, path_ffn_multiplier=c.path_ffn_multiplier,
                    markov_rank=c.markov_rank, init_mode="noise", noise_scale=1.0)

    def weight_bytes_per_draft(self, head_fraction: float = 1.0) -> int:
        """Packed fp16 weight bytes one draft streams (the algorithmic bytes of the engine):
        cross K/V once; per Euler step every block of both chunk experts plus their out_proj;
        per beam depth the live PathHead offsets, the PathHead MLP and the [lm_head | markov w2]
        shortlist head (reference flow_proposer.py:1115-1117 counts the head the same way).
        head_fraction: the share of the shortlist head one GPU holds when it is row-sharded."""
        D, L, T, FM = self.hidden, self.layers, self.steps, self.ffn
        E = 2
        crosskv = E * L * 2 * D * D
        per_step = E * L * (3 + 1 + 1 + 1 + FM + FM) * D * D + E * D * D
        head = 0
        for d in range(1, self.draft_tokens + 1):
            head += min(d, 4) * D * D + 2 * (2 * D * D) + head_fraction * self.shortlist_rows * (D + self.markov_rank)
        return int(2 * (crosskv + T * per_step + head))

    def flops_per_draft(self, batch: int) -> int:
        """Multiply-add FLOPs (2 per MAC) of the Linear layers of one draft of `batch` requests:
        every Euler step runs each block of chunk expert e over batch x 3(e+1) rows and out_proj
        over batch x 3 rows; cross K/V runs once over batch x 8 context rows; each beam depth runs
        the path head and the shortlist head over batch x width beam rows. Attention and the
        row kernels are not counted (under 1%)."""
        D, L, T, FM = self.hidden, self.layers, self.steps, self.ffn
        flow = 0
        for e in range(2):
            rows = batch * 3 * (e + 1)
            flow += rows * L * (6 + 2 * FM) * D * D + batch * 3 * D * D
        cross = batch * 8 * 2 * L * 2 * D * D
        head = 0
        bw = batch * self.width
        for d in range(1, self.draft_tokens + 1):
            head += bw * (min(d, 4) * D * D + 4 * D * D + self.shortlist_rows * (D + self.markov_rank))
        return int(2 * (T * flow + cross + head))


WORKLOADS = {
    # BASELINE config 1 (CPU plumbing) at flow width = hidden (no VAE)
    "cpu": Workload("cfg1-cpu-plumbing", hidden=256, layers=2, steps=4, ffn=2, vocab=32000,
                    shortlist_rows=4096, markov_rank=256),
    # Qwen3.5-4B-shaped drafter
    "4b": Workload("cfg2-4B-shaped", hidden=2560, layers=4, steps=8),
    # Qwen3.5-27B-shaped drafter
    "27b": Workload("cfg3-27B-shaped", hidden=5120, layers=4, steps=8),
    # profiler-sized 4B-width case: one block, one Euler step, a 65,536-row vocabulary (about
    # 1.3 GB on the device, still far larger than L2), for full hardware-counter captures
    "4b-ncu": Workload("4B-width-ncu-case", hidden=2560, layers=1, steps=1, vocab=65536),
}


def make_state(w: Workload, seed: int = 0, device="cuda"):
    """(state_dict, embed, lm_head, shortlist_ids) for workload `w`, all fp16 on `device`
    (shortlist int64 on CPU)."""
    cfg = w.config()
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    D, FM, L, V, rank = w.hidden, w.ffn, w.layers, w.vocab, w.markov_rank

    def r(*shape, std=0.02, mean=0.0):
        return (torch.randn(*shape, generator=g, device=dev) * std + mean).to(torch.float16)

    sd = {}
    for e in range(cfg.n_experts):
        p = "expert." if e == 0 else f"extra_experts.{e - 1}."
        sd[p + "position_embedding.weight"] = r(cfg.draft_length, D, std=0.5)
        sd[p + "time_mlp.0.weight"] = r(D, 1, std=1.0)
        sd[p + "time_mlp.0.bias"] = r(D, std=1.0)
        sd[p + "time_mlp.2.weight"] = r(D, D)
        sd[p + "time_mlp.2.bias"] = r(D)
        for l in range(L):
            b = f"{p}blocks.{l}."
            for n in ("self_norm", "cross_norm", "context_norm", "ffn.0"):
                sd[f"{b}{n}.weight"] = r(D, std=0.1, mean=1.0)
                sd[f"{b}{n}.bias"] = r(D, std=0.1)
            for a in ("self_attn", "cross_attn"):
                sd[f"{b}{a}.in_proj_weight"] = r(3 * D, D)
                sd[f"{b}{a}.in_proj_bias"] = r(3 * D)
                sd[f"{b}{a}.out_proj.weight"] = r(D, D)
                sd[f"{b}{a}.out_proj.bias"] = r(D)
            sd[f"{b}ffn.1.weight"] = r(FM * D, D)
            sd[f"{b}ffn.1.bias"] = r(FM * D)
            sd[f"{b}ffn.4.weight"] = r(D, FM * D)
            sd[f"{b}ffn.4.bias"] = r(D)
        sd[p + "out_norm.weight"] = r(D, std=0.1, mean=1.0)
        sd[p + "out_norm.bias"] = r(D, std=0.1)
        sd[p + "out_proj.weight"] = r(D, D)
        sd[p + "out_proj.bias"] = r(D)
    sd["markov.w1.weight"] = r(V, rank, std=0.5)
    sd["markov.w2.weight"] = r(V, rank)
    for j in range(cfg.path_order):
        sd[f"path_head.offset_proj.{j}.weight"] = r(D, D)
        sd[f"path_head.offset_proj.{j}.bias"] = r(D)
    sd["path_head.norm.weight"] = r(D, std=0.1, mean=1.0)
    sd["path_head.norm.bias"] = r(D, std=0.1)
    P2 = cfg.path_ffn_multiplier * D
    sd["path_head.mlp.0.weight"] = r(P2, D)
    sd["path_head.mlp.0.bias"] = r(P2)
    sd["path_head.mlp.3.weight"] = r(D, P2)
    sd["path_head.mlp.3.bias"] = r(D)
    embed = r(V, D, std=0.5)
    lm_head = r(V, D)
    sl = torch.randperm(V, generator=torch.Generator().manual_seed(seed + 7))[: w.shortlist_rows].sort().values
    return sd, embed, lm_head, sl


def make_inputs(w: Workload, batch: int, seed: int = 1, device="cuda"):
    """(ctx [B, 8, H] fp16, known0 [B] int64): one final hidden state ~N(0, 1) per request,
    front-padded to the 8-row window by repetition (what the reference's context ring does for a
    fresh request, flow_proposer.py:947-961), and a committed token per request."""
    g = torch.Generator(device=device).manual_seed(seed)
    h = torch.randn(batch, 1, w.hidden, generator=g, device=device)
    ctx = h.expand(batch, 8, w.hidden).to(torch.float16).contiguous()
    known0 = torch.randint(0, w.vocab, (batch,), generator=g, device=device)
    return ctx, known0
