"""The production drafter: the flow in a VAE latent space, the beam in the target's hidden space.

The shipped chain-flow drafters are ``TreeVAEFlowDrafter``s (reference
src/chain_flow/drafters/tree_vae_flow.py:91-175): ``predict_hidden(ctx)`` encodes the context
window with a frozen ``TransformerHiddenVAE`` (src/chain_flow/vae/transformer_hidden.py:51-58,
mu only), integrates the flow at the latent width, and decodes the integrated latents back to
hidden states (:60-67); the path head, markov head and shortlist head then run at the hidden
width exactly as for ``TreeFlowDrafter``.

Here one draft is four stages on one stream, each bound to the next one's input buffer:

  encode  ctx fp16 [B, C, H]       -> mu fp16 [B, C, latent] = the flow's ctx
  flow    MODE_FLOW at the latent width -> z fp32 [B, DL, latent]
  decode  z                        -> pred fp32 [B, DL, H]   = the beam's pred
  beam    MODE_BEAM_CHAIN / _TREE at the hidden width -> tokens

Up to 8 requests every stage is one persistent-engine launch (VaeEnginePlan, Plan); above that
the VAE sides are wide launch lists (VaePlan) and the flow and beam wide plans.

No stage allocates or synchronises; the whole draft can be captured in a CUDA graph.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib
from .engine import Plan, WidePlan
from .weights import EnginePacker, WidePacker


@dataclass
class VaeConfig:
    """``HiddenVAEConfig`` as ``TreeVAEFlowDrafter`` fills it (tree_vae_flow.py:50-56)."""
    hidden: int
    latent: int = 640
    intermediate: int = 1920
    layers: int = 2
    heads: int = 8
    max_len: int = 16

    @property
    def eff_heads(self) -> int:
        """TransformerHiddenVAE falls back to one head when the width does not divide
        (transformer_hidden.py:13)."""
        return self.heads if self.intermediate % self.heads == 0 else 1

    @staticmethod
    def from_model_args(args: dict, hidden: int) -> "VaeConfig":
        return VaeConfig(hidden=hidden, latent=int(args.get("latent_size", 640)),
                         intermediate=int(args.get("vae_intermediate_size", 1920)),
                         layers=int(args.get("vae_num_layers", 2)), heads=int(args.get("vae_num_heads", 8)),
                         max_len=int(args.get("vae_max_sequence_length", 16)))


def is_vae_drafter(state_dict: dict, model_args: dict) -> bool:
    return "latent_size" in model_args or any(k.startswith("vae.") for k in state_dict)


class VaeWeights:
    """Both sides of the VAE, every pre-LN folded into the Linear after it: norm1 into
    self_attn.in_proj, norm2 into linear1, the encoder's final LayerNorm into ``mu``, the
    decoder's into ``decoder_out``. ``logvar`` is not needed (the drafter uses mu).
    layout "engine": the persistent engine's stream layout (cfb_pack_linear, with LayerNorm
    column sums); "wide": the wide GEMM's tiled layout (cfb_wide_pack)."""

    def __init__(self, sd: dict, cfg: VaeConfig, device=None, layout: str = "engine"):
        self.lib = _lib.load()
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if dev.type != "cuda":
            raise _lib.CfbError("VaeWeights needs a CUDA device: the VAE has no CPU path")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        if layout not in ("engine", "wide"):
            raise ValueError(f"layout={layout!r}")
        self.dev, self.cfg, self.layout = dev, cfg, layout
        self._keep = []
        pk = WidePacker(self.lib, dev, self._keep) if layout == "wide" else EnginePacker(self.lib, dev, self._keep)
        f32 = lambda t: t.to(device=dev, dtype=torch.float32).contiguous()
        self._layers = {}

        def side(name: str, inp: str, out: str, in_dim: int, out_dim: int) -> _lib.VaeSide:
            p = f"vae.{name}."
            layers = (_lib.VaeLayer * max(cfg.layers, 1))()
            for i in range(cfg.layers):
                q = f"{p}layers.{i}."
                layers[i].qkv = pk.linear(sd[q + "self_attn.in_proj_weight"], sd[q + "self_attn.in_proj_bias"],
                                          ln=(sd[q + "norm1.weight"], sd[q + "norm1.bias"]))
                layers[i].attn_out = pk.linear(sd[q + "self_attn.out_proj.weight"], sd[q + "self_attn.out_proj.bias"])
                layers[i].ffn_up = pk.linear(sd[q + "linear1.weight"], sd[q + "linear1.bias"],
                                             ln=(sd[q + "norm2.weight"], sd[q + "norm2.bias"]))
                layers[i].ffn_down = pk.linear(sd[q + "linear2.weight"], sd[q + "linear2.bias"])
            self._layers[name] = layers
            pos = f32(sd[f"vae.{name}_pos.weight"])
            self._keep.append(pos)
            v = _lib.VaeSide()
            v.in_dim, v.width, v.out_dim = in_dim, cfg.intermediate, out_dim
            v.layers, v.heads, v.max_len = cfg.layers, cfg.eff_heads, pos.shape[0]
            v.in_proj = pk.linear(sd[f"vae.{inp}.weight"], sd[f"vae.{inp}.bias"])
            v.pos = pos.data_ptr()
            v.layer = C.cast(layers, C.POINTER(_lib.VaeLayer))
            v.out_proj = pk.linear(sd[f"vae.{out}.weight"], sd[f"vae.{out}.bias"],
                                   ln=(sd[f"vae.{name}_norm.weight"], sd[f"vae.{name}_norm.bias"]))
            return v

        self.encoder = side("encoder", "encoder_in", "mu", cfg.hidden, cfg.latent)
        self.decoder = side("decoder", "decoder_in", "decoder_out", cfg.latent, cfg.hidden)
        torch.cuda.synchronize(dev)

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self._keep)


class VaePlan:
    """One VAE side over `batch` requests of `rows` positions, bound to caller-owned tensors:
    encode reads fp16 [batch, rows, hidden] and writes fp16 [batch, rows, latent]; decode reads
    fp32 [batch, rows, latent] and writes fp32 [batch, rows, hidden]."""

    def __init__(self, vw: VaeWeights, decode: bool, batch: int, rows: int, inp: torch.Tensor, out: torch.Tensor):
        self.vw, self.lib = vw, vw.lib
        side = vw.decoder if decode else vw.encoder
        want_in = (torch.float32 if decode else torch.float16, (batch, rows, side.in_dim))
        want_out = (torch.float32 if decode else torch.float16, (batch, rows, side.out_dim))
        for t, (dt, shape), what in ((inp, want_in, "input"), (out, want_out, "output")):
            if t.dtype != dt or tuple(t.shape) != shape or not t.is_contiguous() or t.device != vw.dev:
                raise _lib.CfbError(f"VAE {what}: want a contiguous {dt} {shape} tensor on {vw.dev}")
        self.side, self.inp, self.out = side, inp, out
        nbytes = C.c_size_t(0)
        _lib.check(self.lib.cfb_vae_workspace(C.byref(side), batch, rows, int(decode), C.byref(nbytes)),
                   "cfb_vae_workspace")
        self.ws = torch.empty(int(nbytes.value) + 256, dtype=torch.uint8, device=vw.dev)
        self.ws_ptr = (self.ws.data_ptr() + 255) // 256 * 256
        h = C.c_void_p()
        _lib.check(self.lib.cfb_vae_create(C.byref(side), batch, rows, int(decode), inp.data_ptr(), out.data_ptr(),
                                           C.c_void_p(self.ws_ptr), C.c_size_t(int(nbytes.value)), C.byref(h)),
                   "cfb_vae_create")
        self._h = h
        n = C.c_int()
        _lib.check(self.lib.cfb_wide_info(h, C.byref(n)), "cfb_wide_info")
        self.launches = n.value

    def run(self, stream=None) -> None:
        _lib.check(self.lib.cfb_wide_run(self._h, C.c_void_p(_lib.stream_ptr(stream))), "cfb_wide_run")

    def device_error(self) -> int:
        v = C.c_int(0)
        _lib.check(self.lib.cfb_wide_error(self._h, C.byref(v)), "cfb_wide_error")
        return v.value

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            self.lib.cfb_wide_destroy(h)
            self._h = None


class VaeEnginePlan:
    """One VAE side as a persistent-engine plan (batch * rows <= 64), same I/O as VaePlan; runs
    and reports like a drafting ``Plan`` (cfb_plan_run / cfb_plan_error)."""

    def __init__(self, vw: VaeWeights, decode: bool, batch: int, rows: int, inp: torch.Tensor, out: torch.Tensor):
        if vw.layout != "engine":
            raise _lib.CfbError("VaeEnginePlan needs VaeWeights(layout='engine')")
        self.vw, self.lib = vw, vw.lib
        side = vw.decoder if decode else vw.encoder
        want_in = (torch.float32 if decode else torch.float16, (batch, rows, side.in_dim))
        want_out = (torch.float32 if decode else torch.float16, (batch, rows, side.out_dim))
        for t, (dt, shape), what in ((inp, want_in, "input"), (out, want_out, "output")):
            if t.dtype != dt or tuple(t.shape) != shape or not t.is_contiguous() or t.device != vw.dev:
                raise _lib.CfbError(f"VAE {what}: want a contiguous {dt} {shape} tensor on {vw.dev}")
        self.side, self.inp, self.out = side, inp, out
        nbytes = C.c_size_t(0)
        _lib.check(self.lib.cfb_vae_plan_workspace(C.byref(side), batch, rows, int(decode), C.byref(nbytes)),
                   "cfb_vae_plan_workspace")
        self.ws = torch.empty(int(nbytes.value) + 256, dtype=torch.uint8, device=vw.dev)
        self.ws_ptr = (self.ws.data_ptr() + 255) // 256 * 256
        _lib.check(self.lib.cfb_vae_plan_build(C.byref(side), batch, rows, int(decode), inp.data_ptr(), out.data_ptr(),
                                               C.c_void_p(self.ws_ptr), C.c_size_t(int(nbytes.value))),
                   "cfb_vae_plan_build")
        self.launches = 1

    def run(self, stream=None) -> None:
        _lib.check(self.lib.cfb_plan_run(C.c_void_p(self.ws_ptr), C.c_void_p(_lib.stream_ptr(stream))), "cfb_plan_run")

    def device_error(self) -> int:
        v = C.c_int(0)
        self.lib.cfb_plan_error(C.c_void_p(self.ws_ptr), C.byref(v))
        return v.value


_BEAM_MODE = {_lib.MODE_CHAIN: _lib.MODE_BEAM_CHAIN, _lib.MODE_TREE: _lib.MODE_BEAM_TREE}


class VaeDraft:
    """A whole production draft (encode -> latent flow -> decode -> beam) with the same buffers
    as ``Plan``: write ``ctx`` (fp16 [B, C, hidden]), ``z0`` (fp16 [B, DL, latent], init_mode
    'noise') and ``known0``; ``run()``; read ``pred`` (fp32 [B, DL, hidden]) and ``tokens``.
    ``wide`` selects the wide (tcgen05, batched) plans for the flow and the beam instead of the
    persistent engine; the VAE sides follow the layout of ``vw`` (engine plans or wide lists)."""

    def __init__(self, vw: VaeWeights, flow_w, head_w, mode: int, batch: int, *, wide: bool = False,
                 width: int = 4, depth: int = 5, tree_keep: int = 4, tree_topb: int = 8, init_mode: int = 0,
                 twopass_m: int = 0):
        self.mode, self.batch = mode, batch
        vc = vw.cfg
        kind = WidePlan if wide else Plan
        self.flow = kind(flow_w, _lib.MODE_FLOW, batch, init_mode=init_mode)
        fc = flow_w.cfg
        dev = vw.dev
        C_, DL = fc.context_size, fc.draft_length
        if fc.hidden != vc.latent:
            raise _lib.CfbError(f"flow width {fc.hidden} != VAE latent {vc.latent}")
        if max(C_, DL) > vc.max_len:
            raise _lib.CfbError(f"VAE max_sequence_length {vc.max_len} < {max(C_, DL)} rows")
        self.head = None
        if mode != _lib.MODE_FLOW:
            if head_w is None or head_w.cfg.hidden != vc.hidden:
                raise _lib.CfbError("a beam draft needs head weights at the VAE's hidden width")
            extra = {"twopass_m": twopass_m} if twopass_m else {}
            self.head = kind(head_w, _BEAM_MODE[mode], batch, width=width, depth=depth, tree_keep=tree_keep,
                             tree_topb=tree_topb, **extra)
        self.ctx = torch.zeros(batch, C_, vc.hidden, dtype=torch.float16, device=dev)
        self.z0 = self.flow.z0
        if self.head is not None:
            self.known0, self.pred, self.tokens = self.head.known0, self.head.pred, self.head.tokens
            self.N = self.head.N
        else:
            self.known0 = torch.zeros(batch, dtype=torch.int64, device=dev)
            self.pred = torch.zeros(batch, DL, vc.hidden, dtype=torch.float32, device=dev)
            self.tokens = None
        side = VaeEnginePlan if vw.layout == "engine" else VaePlan
        self.encode = side(vw, False, batch, C_, self.ctx, self.flow.ctx)
        self.decode = side(vw, True, batch, DL, self.flow.pred, self.pred)
        self.segments = 1 + (self.head.segments if self.head is not None else 0)
        self.launches = self.encode.launches + getattr(self.flow, "launches", 1) + self.decode.launches + \
            (getattr(self.head, "launches", 1) if self.head is not None else 0)

    @property
    def latent(self) -> torch.Tensor:
        """fp32 [B, DL, latent]: the integrated latents of the last run."""
        return self.flow.pred

    @property
    def mu(self) -> torch.Tensor:
        """fp16 [B, C, latent]: the encoded context of the last run."""
        return self.flow.ctx

    def run(self, stream=None, group=None) -> None:
        self.encode.run(stream)
        self.flow.run(stream)
        self.decode.run(stream)
        if self.head is not None:
            self.head.run(stream, group=group)

    def device_error(self) -> int:
        errs = [self.encode.device_error(), self.flow.device_error(), self.decode.device_error()]
        if self.head is not None:
            errs.append(self.head.device_error())
        return max(errs)

    def check(self) -> None:
        err = self.device_error()
        if err:
            raise _lib.CfbError(f"device-side wait timed out (code {err}); outputs are invalid")
