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
    draft_length: int = 6
    chunk: int = 3
    path_order: int = 4
    # latent > 0: a production TreeVAEFlowDrafter (reference drafters/tree_vae_flow.py:91-175), the
    # flow at this latent width between a TransformerHiddenVAE encode and decode
    latent: int = 0
    vae_inter: int = 1920
    vae_layers: int = 2
    vae_heads: int = 8

    @property
    def flow_width(self) -> int:
        return self.latent or self.hidden

    @property
    def n_experts(self) -> int:
        return self.draft_length // self.chunk

    def config(self, hidden: int | None = None) -> DraftConfig:
        return DraftConfig(hidden=hidden or self.hidden, context_size=8, draft_length=self.draft_length,
                           chunk_size=self.chunk, num_heads=8, ffn_multiplier=self.ffn,
                           num_drafter_layers=self.layers, num_flow_steps=self.steps, path_order=self.path_order,
                           path_ffn_multiplier=2, markov_rank=self.markov_rank)

    def model_args(self) -> dict:
        c = self.config()
        a = dict(context_size=c.context_size, draft_length=c.draft_length, chunk_size=c.chunk_size,
                 num_heads=c.num_heads, ffn_multiplier=c.ffn_multiplier,
                 num_drafter_layers=c.num_drafter_layers, num_flow_steps=c.num_flow_steps,
                 path_order=c.path_order, path_ffn_multiplier=c.path_ffn_multiplier,
                 markov_rank=c.markov_rank, init_mode="noise", noise_scale=1.0)
        if self.latent:
            a.update(expert_dim=self.latent, latent_size=self.latent, vae_intermediate_size=self.vae_inter,
                     vae_num_layers=self.vae_layers, vae_num_heads=self.vae_heads, vae_max_sequence_length=16)
        return a

    def vae_macs_per_row(self) -> tuple[int, int]:
        """(encoder, decoder) multiply-adds per sequence row of the VAE's Linear layers: in-projection,
        per layer in_proj 3I^2 + out_proj I^2 + FFN 2 * 4I^2, then mu / decoder_out."""
        if not self.latent:
            return 0, 0
        H, I, Z, nl = self.hidden, self.vae_inter, self.latent, self.vae_layers
        body = nl * 12 * I * I
        return H * I + body + I * Z, Z * I + body + I * H

    def weight_bytes_per_draft(self, head_fraction: float = 1.0, twopass_m: int = 0, batch: int = 1) -> int:
        """Packed fp16 weight bytes one draft streams (the algorithmic bytes of the engine):
        cross K/V once; per Euler step every block of every chunk expert plus its out_proj;
        per beam depth the live PathHead offsets, the PathHead MLP and the [lm_head | markov w2]
        shortlist head (reference flow_proposer.py:1115-1117 counts the head the same way); for a
        production drafter the VAE encoder and decoder once each.
        head_fraction: the share of the shortlist head one GPU holds when it is row-sharded.
        twopass_m > 0: the two-pass head instead streams the whole head once (pass A), reads and
        writes each request's twopass_m candidate rows once, and reads them at every depth."""
        Df, Dh, L, T, FM, E = self.flow_width, self.hidden, self.layers, self.steps, self.ffn, self.n_experts
        crosskv = E * L * 2 * Df * Df
        per_step = E * L * (3 + 1 + 1 + 1 + FM + FM) * Df * Df + E * Df * Df
        head = 0
        row = Dh + self.markov_rank
        for d in range(1, self.draft_tokens + 1):
            head += min(d, self.path_order) * Dh * Dh + 2 * (2 * Dh * Dh)
            head += (batch * twopass_m * row) if twopass_m else head_fraction * self.shortlist_rows * row
        if twopass_m:
            head += self.shortlist_rows * row + 2 * batch * twopass_m * row
        enc, dec = self.vae_macs_per_row()
        return int(2 * (crosskv + T * per_step + head + enc + dec))

    def flow_weight_bytes(self) -> int:
        """Packed fp16 weight bytes of the flow alone (cross K/V once, then every block of every
        chunk expert plus its out_proj per Euler step): what one MODE_FLOW launch streams."""
        Df, L, T, FM, E = self.flow_width, self.layers, self.steps, self.ffn, self.n_experts
        return int(2 * (E * L * 2 * Df * Df + T * (E * L * (6 + 2 * FM) * Df * Df + E * Df * Df)))

    def flops_per_draft(self, batch: int) -> int:
        """Multiply-add FLOPs (2 per MAC) of the Linear layers of one draft of `batch` requests:
        every Euler step runs each block of chunk expert e over batch x chunk (e+1) rows and
        out_proj over batch x chunk rows; cross K/V runs once over batch x 8 context rows; each
        beam depth runs the path head and the shortlist head over batch x width beam rows; the VAE
        encodes batch x 8 context rows and decodes batch x draft_length rows. Attention and the
        row kernels are not counted (under 1%)."""
        Df, Dh, L, T, FM, E, CH = self.flow_width, self.hidden, self.layers, self.steps, self.ffn, self.n_experts, self.chunk
        flow = 0
        for e in range(E):
            rows = batch * CH * (e + 1)
            flow += rows * L * (6 + 2 * FM) * Df * Df + batch * CH * Df * Df
        cross = batch * 8 * E * L * 2 * Df * Df
        head = 0
        bw = batch * self.width
        for d in range(1, self.draft_tokens + 1):
            head += bw * (min(d, self.path_order) * Dh * Dh + 4 * Dh * Dh + self.shortlist_rows * (Dh + self.markov_rank))
        enc, dec = self.vae_macs_per_row()
        vae = batch * 8 * enc + batch * self.draft_length * dec
        return int(2 * (T * flow + cross + head + vae))


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
    # the shipped 4B production drafter (the reference's published draft timings are for this
    # shape): VAE 2560 -> 640 (intermediate 1920, 2 layers, 8 heads), 8 blocks, 2 Euler steps,
    # draft_length 8 in chunks of 4, path order 8
    "4b-prod": Workload("4B-production-vae", hidden=2560, layers=8, steps=2, draft_length=8, chunk=4,
                        path_order=8, latent=640),
    # the 27B production shape: the same drafter layout with the flow in a 1024-wide latent space
    # (the reference's fused-kernel D = 1024 instantiation, shared by its 9B and 27B drafters). The
    # VAE intermediate width keeps the 4B drafter's 3 x latent ratio; the published D = 1024
    # integrate() figure covers the flow alone, which does not depend on it.
    "27b-prod": Workload("27B-production-vae", hidden=5120, layers=8, steps=2, draft_length=8, chunk=4,
                         path_order=8, latent=1024, vae_inter=3072),
}


def make_state(w: Workload, seed: int = 0, device="cuda"):
    """(state_dict, embed, lm_head, shortlist_ids) for workload `w`, all fp16 on `device`
    (shortlist int64 on CPU)."""
    cfg = w.config()
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    D, FM, L, V, rank = w.flow_width, w.ffn, w.layers, w.vocab, w.markov_rank

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
    D = w.hidden                     # the path head, markov head and shortlist head: hidden width
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
    if w.latent:
        I, Z = w.vae_inter, w.latent
        for side, din, dout, inp, out in (("encoder", D, Z, "encoder_in", "mu"),
                                          ("decoder", Z, D, "decoder_in", "decoder_out")):
            sd[f"vae.{inp}.weight"] = r(I, din, std=din ** -0.5)
            sd[f"vae.{inp}.bias"] = r(I)
            sd[f"vae.{side}_pos.weight"] = r(16, I, std=0.1)
            for i in range(w.vae_layers):
                q = f"vae.{side}.layers.{i}."
                for n in ("norm1", "norm2"):
                    sd[f"{q}{n}.weight"] = r(I, std=0.1, mean=1.0)
                    sd[f"{q}{n}.bias"] = r(I, std=0.1)
                sd[q + "self_attn.in_proj_weight"] = r(3 * I, I)
                sd[q + "self_attn.in_proj_bias"] = r(3 * I)
                sd[q + "self_attn.out_proj.weight"] = r(I, I)
                sd[q + "self_attn.out_proj.bias"] = r(I)
                sd[q + "linear1.weight"] = r(4 * I, I)
                sd[q + "linear1.bias"] = r(4 * I)
                sd[q + "linear2.weight"] = r(I, 4 * I)
                sd[q + "linear2.bias"] = r(I)
            sd[f"vae.{side}_norm.weight"] = r(I, std=0.1, mean=1.0)
            sd[f"vae.{side}_norm.bias"] = r(I, std=0.1)
            sd[f"vae.{out}.weight"] = r(dout, I, std=I ** -0.5)
            sd[f"vae.{out}.bias"] = r(dout)
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
