"""FlowDrafterProposer: the reference's drafting surface on the sm_100a engine.

Mirrors ``chain_flow.vllm_plugin.flow_proposer.FlowDrafterProposer`` (reference
src/chain_flow/vllm_plugin/flow_proposer.py:328-2569) where the drafting path is concerned:

* ``_beam_chains(ctx[B,C,H], known0[B]) -> [B, K]`` int64 token ids (reference :1188-1269);
* ``_beam_tree(ctx, known0) -> [B, 2N]``: N BFS-ordered tokens, then their parents (:1273-1332);
* ``predict_hidden(ctx) -> [B, draft_length, H]`` (drafters/tree_flow.py:243);
* the drafter checkpoint layout (``model.safetensors`` keys ``drafter.*`` +
  ``chained_flow_tree_config.json``) and the shortlist file format and guard
  (``CF_SHORTLIST`` -> ``<ckpt>/shortlist.pt``), with the declared-identity check (:1006-1016, :739-765);
* the ``CF_*`` knobs of the path: ``CF_WIDTH``, ``CF_FLOW_STEPS``, ``CF_TREE_KEEP``, ``CF_TREE_TOPB``,
  ``CF_TREE_DEPTH``, ``CF_TWOPASS_M`` (0: the one-pass head; M > 0: the two-pass candidate head
  with one candidate set for every depth, ``CF_TWOPASS_SHARED=1``, ``CF_TWOPASS_SEED=0``), ``CF_PATH_TRIM``
  (always on: it is exact).

Every draft is ONE persistent kernel launch (flow + beam); there is no CPU fallback. The engine
plans (and their graph-stable I/O buffers) are cached per (mode, batch). A production drafter
(``TreeVAEFlowDrafter``: ``latent_size`` in the model args, ``vae.*`` weights) drafts as VAE
encode -> latent flow -> VAE decode -> hidden-width beam (chain_flow_b200.vae).
"""
from __future__ import annotations

import json
import os

import torch

from . import _lib, shortlist as _sl
from .engine import Plan, WidePlan
from .ring import ContextRing
from .vae import VaeConfig, VaeDraft, VaeWeights, is_vae_drafter
from .weights import DraftConfig, DrafterWeights, WideWeights


# requests one persistent-engine plan drafts at once: its jobs hold at most 64 activation rows
# (B x context rows, B x draft_length, B x beam width). Larger batches run on the wide plan
# (tcgen05 GEMMs over all requests at once), or, with a row-sharded head, as several engine plans.
MAX_PLAN_BATCH = 8


def _env_int(name: str, default: int) -> int:
    v = os.environ.get(name)
    return int(v) if v not in (None, "") else default


class FlowDrafterProposer:
    """Drafting engine with the reference proposer's interface.

    Build it with ``from_components`` (state dict + target embedding / lm_head tensors) or
    ``from_checkpoint`` (a drafter directory); ``FlowDrafterProposer(vllm_config)`` reads the
    speculative config and builds lazily from the loaded target model on first ``propose``.
    """

    def __init__(self, vllm_config=None, **kw):
        self.vllm_config = vllm_config
        self.width = _env_int("CF_WIDTH", 4)
        self.tree_keep = _env_int("CF_TREE_KEEP", 4)
        self.tree_topb = _env_int("CF_TREE_TOPB", 8)
        self.tree_depth = _env_int("CF_TREE_DEPTH", 4)
        self.tree = os.environ.get("VLLM_SPEC_TREE", "0") == "1"
        # the two-pass candidate head (reference flow_proposer.py:1142-1184): only its shared,
        # unseeded form (the reference's defaults CF_TWOPASS_SHARED=1, CF_TWOPASS_SEED=0)
        self.twopass_m = _env_int("CF_TWOPASS_M", 0)
        if self.twopass_m < 0:
            raise ValueError(f"CF_TWOPASS_M={self.twopass_m} must be >= 0")
        if self.twopass_m and os.environ.get("CF_TWOPASS_SHARED", "1") in ("0", "false", "no"):
            raise _lib.CfbError("CF_TWOPASS_SHARED=0 (a candidate set per depth) is not implemented; "
                                "the shared candidate set (CF_TWOPASS_SHARED=1) is")
        if self.twopass_m and os.environ.get("CF_TWOPASS_SEED", "0") == "1":
            raise _lib.CfbError("CF_TWOPASS_SEED=1 is not implemented (the reference measured it worse)")
        self.K = 5
        self.max_reqs = 256                 # context-ring slots (the scheduler's max_num_seqs)
        self._ring = None
        if vllm_config is not None:
            spec = vllm_config.speculative_config
            self.K = int(spec.num_speculative_tokens) - (1 if self.tree else 0)
            sched = getattr(vllm_config, "scheduler_config", None)
            if sched is not None and getattr(sched, "max_num_seqs", None):
                self.max_reqs = int(sched.max_num_seqs)
        self.weights: DrafterWeights | None = None
        self.vae: VaeWeights | None = None          # production (TreeVAEFlowDrafter) drafters only
        self.flow_weights: DrafterWeights | None = None
        self._plans: dict = {}
        self._gen = None
        self.init_mode = "delta"
        self.noise_scale = 1.0
        self.group = None
        for k, v in kw.items():
            setattr(self, k, v)

    # ------------------------------------------------------------------ construction
    @classmethod
    def from_components(cls, state_dict: dict, model_args: dict, embed: torch.Tensor, lm_head: torch.Tensor,
                        shortlist_ids: torch.Tensor | None = None, *, width: int | None = None, K: int = 5,
                        tree_keep: int | None = None, tree_topb: int | None = None,
                        tree_depth: int | None = None, device=None, seed: int = 0,
                        head_shard: tuple[int, int] | None = None, group=None,
                        max_reqs: int | None = None) -> "FlowDrafterProposer":
        """head_shard=(rank, ranks): this process packs only its share of the shortlist head rows
        and every draft all-gathers the ranks' merged top-k lists over `group` (torch.distributed,
        NCCL); all ranks must draft the same requests with the same inputs."""
        self = cls()
        hidden = int(embed.shape[1])
        args = dict(model_args)
        if os.environ.get("CF_FLOW_STEPS"):
            steps = int(os.environ["CF_FLOW_STEPS"])
            if steps < 1:
                raise ValueError(f"CF_FLOW_STEPS must be >= 1, got {steps}")
            args["num_flow_steps"] = steps
        cfg = DraftConfig.from_model_args(args, hidden)
        if shortlist_ids is None:
            shortlist_ids = torch.arange(embed.shape[0])        # full head
        self.vae = None
        self.flow_weights = None
        self.flow_cfg = cfg
        if is_vae_drafter(state_dict, args):
            # TreeVAEFlowDrafter (reference drafters/tree_vae_flow.py:91-175): the flow runs at the
            # VAE's latent width (expert_dim is forced to latent_size), the beam at the hidden width
            vcfg = VaeConfig.from_model_args(args, hidden)
            self.flow_cfg = DraftConfig.from_model_args(args, vcfg.latent)
            self.vae = VaeWeights(state_dict, vcfg, device=device, layout="engine")
            self._vae_cfg = vcfg
            self._wide_vae = None
            self.flow_weights = DrafterWeights(state_dict, self.flow_cfg, None, None, None, device=device,
                                               parts="flow")
        self.weights = DrafterWeights(state_dict, cfg, embed, lm_head, shortlist_ids, device=device,
                                      head_shard=head_shard, parts="head" if self.vae is not None else "all")
        # the wide plan's row-major weights are built on first use by a batch above MAX_PLAN_BATCH
        self._wide_src = None if head_shard is not None else (state_dict, embed, lm_head, shortlist_ids)
        self._wide_weights = None
        self._wide_flow_weights = None
        self.group = group
        self.cfg = cfg
        self.dev = self.weights.dev
        self.init_mode = args.get("init_mode", "delta")
        self.noise_scale = float(args.get("noise_scale", 1.0))
        if self.init_mode not in _lib.INIT_MODES:
            raise ValueError(f"init_mode {self.init_mode!r} is not one of {sorted(_lib.INIT_MODES)}")
        if width is not None: self.width = width
        if max_reqs is not None: self.max_reqs = max_reqs
        if tree_keep is not None: self.tree_keep = tree_keep
        if tree_topb is not None: self.tree_topb = tree_topb
        if tree_depth is not None: self.tree_depth = tree_depth
        self.K = K
        if self.K > cfg.draft_length - 1:
            raise ValueError(f"K={self.K} but this drafter can only emit {cfg.draft_length - 1} chain tokens "
                             f"(draft_length={cfg.draft_length}; depth 0 reconstructs the committed token)")
        if self.tree_keep > self.tree_topb:
            raise ValueError(f"CF_TREE_KEEP={self.tree_keep} > CF_TREE_TOPB={self.tree_topb}: depth 1 "
                             f"expands a single node and can hold at most {self.tree_topb} children")
        self._gen = torch.Generator(device=self.dev).manual_seed(seed)
        return self

    @classmethod
    def from_checkpoint(cls, drafter_dir: str, embed: torch.Tensor, lm_head: torch.Tensor, **kw):
        """Load ``<dir>/model.safetensors`` (``drafter.*`` keys) and ``chained_flow_tree_config.json``
        and resolve the shortlist (``CF_SHORTLIST``, else ``<dir>/shortlist.pt``, else the full head),
        refusing a list built for another vocabulary or not matching the checkpoint's declaration."""
        from safetensors.torch import load_file
        with open(os.path.join(drafter_dir, "chained_flow_tree_config.json")) as f:
            conf = json.load(f)
        sd = load_file(os.path.join(drafter_dir, "model.safetensors"))
        sub = {k[len("drafter."):]: v for k, v in sd.items() if k.startswith("drafter.")}
        if not sub:
            raise KeyError(f"{drafter_dir}/model.safetensors holds no 'drafter.' keys")
        V = int(embed.shape[0])
        ids = None
        cands = []
        if os.environ.get("CF_SHORTLIST"):
            if not os.path.exists(os.environ["CF_SHORTLIST"]):
                raise FileNotFoundError(f"CF_SHORTLIST={os.environ['CF_SHORTLIST']} does not exist")
            cands.append(os.environ["CF_SHORTLIST"])
        elif "CF_SHORTLIST" not in os.environ and os.path.exists(os.path.join(drafter_dir, "shortlist.pt")):
            cands.append(os.path.join(drafter_dir, "shortlist.pt"))
        for path in cands:
            got, meta = _sl.load(path)
            bad = _sl.check(got, meta, V)
            if bad:
                raise ValueError(f"shortlist {path} refused: {bad}")
            got = got[(got >= 0) & (got < V)].unique()
            decl = conf.get("shortlist") or {}
            if decl:
                sha = _sl.ids_content_sha(got)
                if (decl.get("rows") and int(decl["rows"]) != got.numel()) or \
                        (decl.get("ids_sha256") and decl["ids_sha256"] != sha):
                    raise RuntimeError(f"shortlist {path} does not match what this drafter declares "
                                       f"({decl}); got {got.numel()} rows, ids-sha256 {sha}")
            ids = got
            break
        return cls.from_components(sub, conf["model_args"], embed, lm_head, ids, **kw)

    # ------------------------------------------------------------------ engine plans
    def _plan(self, mode: int, B: int) -> Plan:
        key = (mode, B)
        p = self._plans.get(key)
        if p is None:
            init = _lib.INIT_MODES[self.init_mode]
            depth = self.tree_depth if mode == _lib.MODE_TREE else self.K
            tp = self.twopass_m if mode != _lib.MODE_FLOW else 0
            if self.vae is not None:
                p = VaeDraft(self.vae, self.flow_weights, self.weights, mode, B, width=self.width, depth=depth,
                             tree_keep=self.tree_keep, tree_topb=self.tree_topb, init_mode=init, twopass_m=tp)
            else:
                p = Plan(self.weights, mode, B, width=self.width, depth=depth,
                         tree_keep=self.tree_keep, tree_topb=self.tree_topb, init_mode=init, twopass_m=tp)
            self._plans[key] = p
        return p

    def _wide_plan(self, mode: int, B: int) -> WidePlan:
        key = ("wide", mode, B)
        p = self._plans.get(key)
        if p is None:
            if self._wide_weights is None:
                sd, embed, lm_head, ids = self._wide_src
                if ids is None:
                    ids = torch.arange(embed.shape[0])
                vae = self.vae is not None
                self._wide_weights = WideWeights(sd, self.cfg, embed, lm_head, ids, device=self.dev,
                                                 parts="head" if vae else "all")
                if vae:
                    self._wide_flow_weights = WideWeights(sd, self.flow_cfg, None, None, None, device=self.dev,
                                                          parts="flow")
            init = _lib.INIT_MODES[self.init_mode]
            depth = self.tree_depth if mode == _lib.MODE_TREE else self.K
            if self.vae is not None:
                if self._wide_vae is None:
                    self._wide_vae = VaeWeights(self._wide_src[0], self._vae_cfg, device=self.dev, layout="wide")
                p = VaeDraft(self._wide_vae, self._wide_flow_weights, self._wide_weights, mode, B, wide=True,
                             width=self.width, depth=depth, tree_keep=self.tree_keep, tree_topb=self.tree_topb,
                             init_mode=init)
            else:
                p = WidePlan(self._wide_weights, mode, B, width=self.width, depth=depth,
                             tree_keep=self.tree_keep, tree_topb=self.tree_topb, init_mode=init)
            self._plans[key] = p
        return p

    def _load_inputs(self, p: Plan, ctx: torch.Tensor, known0: torch.Tensor | None):
        _lib.require_cuda(ctx, "ctx")
        p.ctx.copy_(ctx.to(torch.float16), non_blocking=True)
        if known0 is not None:
            p.known0.copy_(known0.view(-1).to(torch.int64), non_blocking=True)
        if self.init_mode == "noise":
            # the reference draws torch.randn at every draft (tree_flow.py:154-155); the
            # generator here is seeded per proposer so drafts are reproducible
            p.z0.normal_(generator=self._gen).mul_(self.noise_scale)

    # ------------------------------------------------------------------ drafting interface
    def _run(self, mode: int, ctx: torch.Tensor, known0: torch.Tensor | None, out: str) -> torch.Tensor:
        """Up to MAX_PLAN_BATCH requests: one persistent-engine launch. More: one wide plan over
        the whole batch (a row-sharded head, or the two-pass head, instead runs engine plans of
        MAX_PLAN_BATCH requests)."""
        B = ctx.shape[0]
        wide_ok = self._wide_src is not None and not (self.twopass_m and mode != _lib.MODE_FLOW)
        if B <= MAX_PLAN_BATCH or wide_ok:
            p = self._plan(mode, B) if B <= MAX_PLAN_BATCH else self._wide_plan(mode, B)
            self._load_inputs(p, ctx, known0)
            p.run(group=self.group)
            return getattr(p, out)
        parts = []
        for b0 in range(0, B, MAX_PLAN_BATCH):
            b1 = min(B, b0 + MAX_PLAN_BATCH)
            p = self._plan(mode, b1 - b0)
            self._load_inputs(p, ctx[b0:b1], None if known0 is None else known0[b0:b1])
            p.run(group=self.group)
            parts.append(getattr(p, out).clone())
        return torch.cat(parts, dim=0)

    @torch.inference_mode()
    def predict_hidden(self, ctx: torch.Tensor) -> torch.Tensor:
        return self._run(_lib.MODE_FLOW, ctx, None, "pred")

    @torch.inference_mode()
    def _beam_chains(self, ctx: torch.Tensor, known0: torch.Tensor) -> torch.Tensor:
        """[B, K] int64 chain drafts; ``known0`` is the token vLLM just committed."""
        return self._run(_lib.MODE_CHAIN, ctx, known0.view(-1), "tokens")

    @torch.inference_mode()
    def _beam_tree(self, ctx: torch.Tensor, known0: torch.Tensor) -> torch.Tensor:
        """[B, 2N] int64: N BFS-ordered draft tokens followed by their N parent indices (-1 = root)."""
        return self._run(_lib.MODE_TREE, ctx, known0.view(-1), "tokens")

    # ------------------------------------------------------------------ context ring
    def _init_ring(self, H: int):
        """One ring slot of ctx_size hidden states per request slot (reference
        flow_proposer.py:881-889), on the GPU kernels of chain_flow_b200.ring."""
        self._ring = ContextRing(self.max_reqs, self.cfg.context_size, H, device=self.dev)

    def _ring_write(self, sh, rows_g, starts_g, cnt_g, wmask_g, path_g, Kmax: int):
        """Append each request's newly accepted hidden states to its slot (reference
        flow_proposer.py:916-945): row j is sh[start + j] on a chain step, or the committed
        token's row then the accepted path's rows (start + 1 + path[j - 1]) on a tree step."""
        self._ring.write(sh, rows_g, starts_g, cnt_g, wmask_g, path_g, Kmax)

    def _ring_gather(self, rows_g) -> torch.Tensor:
        """[B, ctx_size, H] fp16 windows, oldest first, front-padded by repeating the oldest row
        (reference flow_proposer.py:947-961)."""
        return self._ring.gather(rows_g)

    @torch.inference_mode()
    def _draft_from_ring(self, rows_g, k0_g) -> torch.Tensor:
        """The whole draft from the ring: gather the windows, then the chain or tree beam."""
        ctx = self._ring_gather(rows_g)
        return self._beam_tree(ctx, k0_g) if self.tree else self._beam_chains(ctx, k0_g)

    def device_error(self) -> int:
        """Synchronous: non-zero if a bounded device-side wait expired in any cached plan's last run."""
        return max((p.device_error() for p in self._plans.values()), default=0)

    # ------------------------------------------------------------------ vLLM entry point
    def propose(self, sampled_token_ids, num_tokens_no_spec=None, token_ids_cpu=None, slot_mappings=None,
                **kw):
        """vLLM ``custom_class`` entry (reference flow_proposer.py:1699). The context window of each
        request (its last ``context_size`` final hidden states, front-padded with the oldest one) is
        taken from ``kw['context_hidden']`` [B, C, H] when the caller supplies it; the vLLM
        runner-hook plumbing that assembles it inside a live engine is not part of this package."""
        ctx = kw.get("context_hidden")
        if ctx is None:
            raise NotImplementedError(
                "propose() needs context_hidden=[B, C, H]: the vLLM hidden-state hook and context ring "
                "of the reference proposer are not implemented by this engine")
        known0 = torch.as_tensor([int(t[-1]) for t in sampled_token_ids], device=ctx.device)
        out = self._beam_tree(ctx, known0) if self.tree else self._beam_chains(ctx, known0)
        return out.tolist()
