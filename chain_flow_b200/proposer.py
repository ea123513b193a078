"""FlowDrafterProposer: the reference's drafting surface on the sm_100a engine.

Mirrors ``chain_flow.vllm_plugin.flow_proposer.FlowDrafterProposer`` (reference
src/chain_flow/vllm_plugin/flow_proposer.py:328-2569) where the drafting path is concerned:

* ``FlowDrafterProposer(vllm_config)`` (:329-560): reads ``speculative_config``,
  ``scheduler_config.max_num_seqs`` and the ``CF_*`` / ``VLLM_SPEC_TREE`` knobs, requires
  ``CF_DRAFTER_DIR`` (a local drafter directory, or a hub repo id that is snapshot-downloaded),
  clamps ``CF_TREE_DEPTH`` to what the checkpoint can emit and refuses inconsistent tree shapes;
  it installs the runner hook that stashes the target's hidden states, and builds lazily on the
  first ``propose`` from the loaded target model's embedding and ``lm_head`` (``_build``, :579-867);
* ``propose(sampled_token_ids, num_tokens_no_spec, token_ids_cpu, slot_mappings=None)`` (:1699):
  appends each request's accepted hidden states to its ring slot (slot migration, recycling and
  prefill seeding as :1989-2109), drafts from the ring, and returns ``list[list[int]]``, or under
  ``CF_ASYNC_SPEC`` a GPU int32 ``[num_reqs, draft_width]`` tensor (:2327-2357); a tree draft also
  stages its shape for the verifier (``tree_registration``, :2360-2406);

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
import sys

import numpy as np
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


# What the runner hook hands the proposer each step (reference flow_proposer.py:34-59): the runner,
# the sampled rows' hidden states, the whole step's hidden states (prefill seeding) and the spec
# decode metadata. A host that drives the proposer without vLLM fills the same keys.
_STASH: dict = {}


def _install_hidden_state_hook() -> bool:
    """vLLM's custom_class hook passes only token ids; the hidden states are in scope one frame up,
    in ``GPUModelRunner.propose_draft_token_ids`` (reference flow_proposer.py:40-59). Patched only
    when vLLM is already loaded in this process (a proposer built by a running engine); returns
    whether the hook is in place."""
    if "vllm" not in sys.modules:
        return False
    try:
        from vllm.v1.worker.gpu_model_runner import GPUModelRunner
    except Exception:                     # noqa: BLE001 - another vLLM layout: the caller stashes
        return False
    if getattr(GPUModelRunner, "_cfb_hooked", False):
        return True
    orig = getattr(GPUModelRunner, "propose_draft_token_ids", None)
    if orig is None:
        return False

    def patched(self, scheduler_output, sampled_token_ids, sampling_metadata, hidden_states,
                sample_hidden_states, *args, **kwargs):
        _STASH["runner"] = self
        _STASH["sample_hidden_states"] = sample_hidden_states
        _STASH["hidden_states"] = hidden_states
        _STASH["spec_meta"] = args[1] if len(args) > 1 else None
        _STASH["sampling_metadata"] = sampling_metadata
        return orig(self, scheduler_output, sampled_token_ids, sampling_metadata, hidden_states,
                    sample_hidden_states, *args, **kwargs)

    GPUModelRunner.propose_draft_token_ids = patched
    GPUModelRunner._cfb_hooked = True
    return True


def _truthy(v, default: bool) -> bool:
    if v in (None, ""):
        return default
    return str(v).lower() not in ("0", "false", "no", "off")


class FlowDrafterProposer:
    """Drafting engine with the reference proposer's interface.

    ``FlowDrafterProposer(vllm_config)`` is what vLLM's custom_class loader calls: it reads the
    speculative / scheduler config and the ``CF_*`` knobs, and builds lazily, on the first
    ``propose``, from the target model the runner hook stashed (its embedding and ``lm_head``) and
    the checkpoint in ``CF_DRAFTER_DIR``. Outside vLLM, build it with ``from_components`` (state
    dict + target embedding / lm_head tensors) or ``from_checkpoint`` (a drafter directory).
    """

    def __init__(self, vllm_config=None, **kw):
        self.vllm_config = vllm_config
        self.width = _env_int("CF_WIDTH", 4)
        self.tree_keep = _env_int("CF_TREE_KEEP", 4)
        self.tree_topb = _env_int("CF_TREE_TOPB", 8)
        self.tree_depth = _env_int("CF_TREE_DEPTH", 4)
        self.tree = os.environ.get("VLLM_SPEC_TREE", "0") == "1"
        self.branching = self.tree and os.environ.get("CF_TREE_BRANCH", "1") == "1"
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
        self.ckd = None
        self.async_spec = False
        self.use_cg = False
        self.draft_width = None
        self.N = None
        self._buckets: list[int] = []
        self.ring_trim = True
        if vllm_config is not None:
            self._configure(vllm_config)
        self.weights: DrafterWeights | None = None
        self.vae: VaeWeights | None = None          # production (TreeVAEFlowDrafter) drafters only
        self.flow_weights: DrafterWeights | None = None
        self._plans: dict = {}
        self._gen = None
        self.init_mode = "delta"
        self.noise_scale = 1.0
        self.group = None
        self._slot_req: list = []
        self._req_slot: dict = {}
        self._pin: dict = {}
        self._cg: dict = {}
        self._dtok = None
        self._ptree = None
        self._areg = None
        for k, v in kw.items():
            setattr(self, k, v)

    def _configure(self, vllm_config) -> None:
        """The constructor's reading of the engine config and the environment (reference
        flow_proposer.py:329-560); nothing is loaded until the first ``propose``."""
        self.hooked = _install_hidden_state_hook()
        spec = vllm_config.speculative_config
        # CF_TREE_DEPTH cannot exceed what the checkpoint emits (draft_length - 1 levels)
        self.tree_depth = self._clamp_depth(self.tree_depth)
        if self.branching and self.tree_keep > self.tree_topb:
            raise ValueError(
                f"CF_TREE_KEEP={self.tree_keep} > CF_TREE_TOPB={self.tree_topb}: depth 1 expands a single "
                f"node, so it can hold at most {self.tree_topb} children while N=keep*depth assumes "
                f"{self.tree_keep}. Raise CF_TREE_TOPB to >= CF_TREE_KEEP.")
        self.N = self.tree_keep * self.tree_depth
        if self.branching and int(spec.num_speculative_tokens) != self.N + 1:
            # one spare state column of the verifier: configure N + 1, emit N (reference :356-364)
            raise ValueError(f"set num_speculative_tokens={self.N + 1} for CF_TREE_KEEP={self.tree_keep} x "
                             f"CF_TREE_DEPTH={self.tree_depth} (got {int(spec.num_speculative_tokens)})")
        self.K = int(spec.num_speculative_tokens) - (1 if self.tree else 0)
        self.draft_width = self.N if self.branching else self.K
        self.ckd = os.environ.get("CF_DRAFTER_DIR")
        if not self.ckd:
            raise ValueError("set CF_DRAFTER_DIR to the drafter checkpoint dir or a HF repo id")
        if not os.path.isdir(self.ckd):
            try:
                from huggingface_hub import snapshot_download
            except ImportError as e:
                raise FileNotFoundError(f"CF_DRAFTER_DIR={self.ckd} is not a directory, and huggingface_hub "
                                        f"is not installed to fetch it as a repo id") from e
            self.ckd = snapshot_download(self.ckd, allow_patterns=["model.safetensors",
                                                                   "chained_flow_tree_config.json", "shortlist.pt"])
        sched = getattr(vllm_config, "scheduler_config", None)
        if sched is not None and getattr(sched, "max_num_seqs", None):
            self.max_reqs = int(sched.max_num_seqs)
        # GPU-token output only when the engine itself schedules asynchronously (reference
        # defaults.finalize_async): a GPU draft handed to a synchronous engine would be ignored
        self.async_spec = os.environ.get("CF_ASYNC_SPEC", "0") == "1" and \
            bool(getattr(sched, "async_scheduling", False))
        # the whole draft (ring gather + plan launch) replayed from a CUDA graph per batch bucket
        self.use_cg = _truthy(os.environ.get("CF_CUDAGRAPH"), True)
        self.ring_trim = _truthy(os.environ.get("CF_RING_TRIM"), True)
        self._buckets = self._bucket_ladder()

    def _clamp_depth(self, depth: int) -> int:
        """CF_TREE_DEPTH clamped to draft_length - 1 from the checkpoint config when it is local
        (reference flow_proposer.py:990-1004); ``_build`` re-checks once the drafter is loaded."""
        try:
            cfg_path = os.path.join(os.environ.get("CF_DRAFTER_DIR", ""), "chained_flow_tree_config.json")
            if os.path.isfile(cfg_path):
                with open(cfg_path) as f:
                    dl = int(json.load(f)["model_args"]["draft_length"])
                if depth > dl - 1:
                    return dl - 1
        except (OSError, KeyError, ValueError, TypeError):
            pass
        return depth

    def _bucket_ladder(self) -> list[int]:
        """Batch buckets of the draft's CUDA graphs: CF_DRAFT_BUCKETS, else powers of two up to
        max_num_seqs plus max_num_seqs itself (reference flow_proposer.py:1511-1540)."""
        env = os.environ.get("CF_DRAFT_BUCKETS")
        if env:
            return sorted({int(x) for x in env.split(",") if x.strip()})
        out, b = [], 1
        while b < self.max_reqs:
            out.append(b)
            b *= 2
        out.append(self.max_reqs)
        return out

    def _wmax(self) -> int:
        """Ring rows one step's commit can fill: tree_depth + 1 for a branching tree, else K + 1
        (reference flow_proposer.py:1091-1112; the extra rows would only ever go to the trash row)."""
        if getattr(self, "ring_trim", True) and self.branching:
            return self.tree_depth + 1
        return self.K + 1

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
        self._setup(state_dict, model_args, embed, lm_head, shortlist_ids, width=width, K=K, tree_keep=tree_keep,
                    tree_topb=tree_topb, tree_depth=tree_depth, device=device, seed=seed, head_shard=head_shard,
                    group=group, max_reqs=max_reqs)
        return self

    def _setup(self, state_dict, model_args, embed, lm_head, shortlist_ids, *, width=None, K=5, tree_keep=None,
               tree_topb=None, tree_depth=None, device=None, seed=0, head_shard=None, group=None,
               max_reqs=None, check_chain_k=True):
        """Pack the drafter for the engine (the body of from_components and of the lazy _build)."""
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
        if check_chain_k and self.K > cfg.draft_length - 1:
            raise ValueError(f"K={self.K} but this drafter can only emit {cfg.draft_length - 1} chain tokens "
                             f"(draft_length={cfg.draft_length}; depth 0 reconstructs the committed token)")
        if self.tree_keep > self.tree_topb:
            raise ValueError(f"CF_TREE_KEEP={self.tree_keep} > CF_TREE_TOPB={self.tree_topb}: depth 1 "
                             f"expands a single node and can hold at most {self.tree_topb} children")
        self._gen = torch.Generator(device=self.dev).manual_seed(seed)

    @staticmethod
    def _read_checkpoint(drafter_dir: str, vocab: int):
        """(drafter state dict, model_args, shortlist ids or None) from a drafter directory: the
        ``drafter.*`` keys of ``model.safetensors``, ``chained_flow_tree_config.json`` and the
        shortlist resolved as ``CF_SHORTLIST`` (set and empty: the full head), else
        ``<dir>/shortlist.pt``, refusing a list built for another vocabulary or not matching the
        checkpoint's declaration (reference flow_proposer.py:375-388, 616-648, 739-765, 1006-1016)."""
        from safetensors.torch import load_file
        with open(os.path.join(drafter_dir, "chained_flow_tree_config.json")) as f:
            conf = json.load(f)
        sd = load_file(os.path.join(drafter_dir, "model.safetensors"))
        sub = {k[len("drafter."):]: v for k, v in sd.items() if k.startswith("drafter.")}
        if not sub:
            raise KeyError(f"{drafter_dir}/model.safetensors holds no 'drafter.' keys")
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
            bad = _sl.check(got, meta, vocab)
            if bad:
                raise ValueError(f"shortlist {path} refused: {bad}")
            got = got[(got >= 0) & (got < vocab)].unique()
            decl = conf.get("shortlist") or {}
            if decl:
                sha = _sl.ids_content_sha(got)
                if (decl.get("rows") and int(decl["rows"]) != got.numel()) or \
                        (decl.get("ids_sha256") and decl["ids_sha256"] != sha):
                    raise RuntimeError(f"shortlist {path} does not match what this drafter declares "
                                       f"({decl}); got {got.numel()} rows, ids-sha256 {sha}")
            ids = got
            break
        return sub, conf["model_args"], ids

    @classmethod
    def from_checkpoint(cls, drafter_dir: str, embed: torch.Tensor, lm_head: torch.Tensor, **kw):
        """Load ``<dir>/model.safetensors`` (``drafter.*`` keys) and ``chained_flow_tree_config.json``
        and resolve the shortlist (``CF_SHORTLIST``, else ``<dir>/shortlist.pt``, else the full head),
        refusing a list built for another vocabulary or not matching the checkpoint's declaration."""
        sub, args, ids = cls._read_checkpoint(drafter_dir, int(embed.shape[0]))
        return cls.from_components(sub, args, embed, lm_head, ids, **kw)

    # ------------------------------------------------------------------ lazy build (vLLM)
    @property
    def built(self) -> bool:
        return self.weights is not None

    def _build(self) -> None:
        """Build from the target model the runner hook stashed (reference flow_proposer.py:579-867):
        its input embedding and lm_head, read off the LOADED model, and the checkpoint in
        CF_DRAFTER_DIR; then the context ring of max_num_seqs slots."""
        runner = _STASH.get("runner")
        if runner is None:
            raise RuntimeError("FlowDrafterProposer: no target model stashed; the runner hook "
                               "(_install_hidden_state_hook) or the host must set _STASH['runner']")
        model = runner.model
        inner = model.language_model.model if hasattr(model, "language_model") else model.model
        embed_w = inner.embed_tokens.weight
        lm = model.language_model.lm_head if hasattr(model, "language_model") else model.lm_head
        lm_w = lm.weight
        sub, args, ids = self._read_checkpoint(self.ckd, int(embed_w.shape[0]))
        dl = int(args.get("draft_length", 6))
        if self.branching:
            emit = min(self.tree_depth, dl - 1)
            if emit != self.tree_depth:
                raise ValueError(f"CF_TREE_DEPTH={self.tree_depth} but the drafter can only emit {emit} levels "
                                 f"(draft_length={dl}); set CF_TREE_DEPTH<={emit} and "
                                 f"num_speculative_tokens={self.tree_keep * emit + 1}")
        elif self.K > dl - 1:
            raise ValueError(f"num_speculative_tokens={self.K} but this drafter can only emit {dl - 1} chain "
                             f"tokens (draft_length={dl}); set num_speculative_tokens<={dl - 1}")
        keep = dict(tree=self.tree, branching=self.branching, N=self.N, draft_width=self.draft_width,
                    ckd=self.ckd, async_spec=self.async_spec, use_cg=self.use_cg, _buckets=self._buckets,
                    ring_trim=self.ring_trim, hooked=getattr(self, "hooked", False))
        self._setup(sub, args, embed_w, lm_w, ids, width=self.width, K=self.K, tree_keep=self.tree_keep,
                    tree_topb=self.tree_topb, tree_depth=self.tree_depth, device=embed_w.device,
                    max_reqs=self.max_reqs, check_chain_k=False)
        for k, v in keep.items():
            setattr(self, k, v)
        self._init_ring(int(embed_w.shape[1]))

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
        self._slot_req = [None] * self.max_reqs      # slot -> request id occupying it
        self._req_slot = {}                          # request id -> slot (detects migration)

    def _h2d(self, key: str, arr, pad_to: int = 0) -> torch.Tensor:
        """int64 numpy -> the GPU through a persistent pinned buffer: an asynchronous copy, no host
        sync (reference flow_proposer.py:891-914). Rows past len(arr) up to pad_to are 0."""
        n = int(arr.shape[0])
        m = max(n, pad_to)
        ent = self._pin.get(key)
        if ent is None or ent[0].shape[0] < m:
            cap = max(m, self.max_reqs * (self.K + 2))
            ent = (torch.empty(cap, dtype=torch.long, pin_memory=True),
                   torch.empty(cap, dtype=torch.long, device=self.dev))
            self._pin[key] = ent
        cpu, gpu = ent
        cpu[:n].copy_(torch.from_numpy(np.ascontiguousarray(arr, dtype=np.int64)))
        if m > n:
            cpu[n:m].fill_(0)
        gpu[:m].copy_(cpu[:m], non_blocking=True)
        return gpu[:m] if pad_to else gpu[:n]

    def _seed_prompt_ctx(self, i: int):
        """A fresh request's window from the prefill's hidden states: the last ctx_size rows of
        request i's span [query_start_loc[i], query_start_loc[i+1]) of the step's hidden states
        (reference flow_proposer.py:1668-1697); None when that is not available (a decode step)."""
        hs, runner = _STASH.get("hidden_states"), _STASH.get("runner")
        if hs is None or runner is None:
            return None
        qsl = getattr(runner, "query_start_loc", None)
        q = None
        for attr in ("np", "cpu"):
            v = getattr(qsl, attr, None)
            if v is not None:
                q = v.tolist() if hasattr(v, "tolist") else list(v)
                break
        if q is None or i + 1 >= len(q):
            return None
        start, end = int(q[i]), int(q[i + 1])
        if end <= start or end > hs.shape[0]:
            return None
        return start, end

    @torch.inference_mode()
    def _ctx_gpu(self, rows, req_ids, sh, sampled_token_ids):
        """Append this step's accepted hidden states to each drafting request's ring slot and return
        (rows_g [bucket] slots, k0_g [bucket] committed tokens, B). Every index is computed from
        host-resident metadata, so nothing is read back from the GPU (reference :1989-2109):

        * row j of request i is sample_hidden_states[start_i + j], start_i = sum over earlier
          requests of (num_draft_tokens + 1) (one row per request without drafts);
        * a slot whose occupant changed is a MIGRATION (the request moved to a lower input-batch
          index: its history moves with it) or a RECYCLE (a new request: reset, then seeded from
          its prefill hidden states when they are in this step, in which case this step's row is
          not appended again)."""
        C = self.cfg.context_size
        smd = _STASH.get("spec_meta")
        nreq = len(sampled_token_ids)
        nd = getattr(smd, "num_draft_tokens", None) if smd is not None else None
        if nd is not None:
            nd = np.asarray(nd, dtype=np.int64)
            if nd.shape[0] < nreq:
                nd = np.concatenate([nd, np.zeros(nreq - nd.shape[0], dtype=np.int64)])
            starts_all = np.cumsum(nd + 1) - (nd + 1)
        else:
            starts_all = np.arange(nreq, dtype=np.int64)
        rows_np = np.asarray(rows, dtype=np.int64)
        cnt_np = np.asarray([len(sampled_token_ids[i]) for i in rows], dtype=np.int64)
        k0_np = np.asarray([sampled_token_ids[i][-1] for i in rows], dtype=np.int64)
        fresh, migrate = [], []
        prev = list(self._slot_req)                  # occupants before this step (slots may swap)
        for i in rows:
            rid = req_ids[i] if i < len(req_ids) else str(i)
            if prev[i] == rid:
                continue
            old = self._req_slot.get(rid)
            if old is not None and old != i and prev[old] == rid:
                migrate.append((i, old))
            else:
                fresh.append(i)
            self._slot_req[i] = rid
            self._req_slot[rid] = i
        live = set(req_ids)
        for k in [k for k in self._req_slot if k not in live]:
            self._req_slot.pop(k, None)
        ring = self._ring
        if migrate:
            snap, sp, sn = ring.ring.clone(), ring.rpos.clone(), ring.nval.clone()   # slots may swap
            ng = self._h2d("mig_new", np.asarray([m[0] for m in migrate]))
            og = self._h2d("mig_old", np.asarray([m[1] for m in migrate]))
            ring.ring.index_copy_(0, ng, snap.index_select(0, og))
            ring.rpos.index_copy_(0, ng, sp.index_select(0, og))
            ring.nval.index_copy_(0, ng, sn.index_select(0, og))
        wmask_np = np.ones(rows_np.shape[0], dtype=np.int64)
        if fresh:
            fg = self._h2d("reset", np.asarray(fresh))
            ring.rpos.index_fill_(0, fg, 0)
            ring.nval.index_fill_(0, fg, 0)
            seeds = [(i, self._seed_prompt_ctx(i)) for i in fresh]
            seeds = [(i, span) for i, span in seeds if span is not None]
            if seeds:
                hs = _STASH["hidden_states"]
                for j, i in enumerate(rows):
                    if any(i == si for si, _ in seeds):
                        wmask_np[j] = 0
                sl_np = np.asarray([i for i, _ in seeds])
                lo = np.asarray([max(a, b - C) for _, (a, b) in seeds])
                ln = np.asarray([min(b - a, C) for _, (a, b) in seeds])
                ring.write(hs, self._h2d("seed_rows", sl_np), self._h2d("seed_lo", lo), self._h2d("seed_n", ln),
                           torch.ones(len(seeds), dtype=torch.bool, device=self.dev), None, C)
        B = rows_np.shape[0]
        bucket = next((b for b in getattr(self, "_buckets", [B]) if b >= B), B)
        rows_g = self._h2d("rows", rows_np, pad_to=bucket)
        k0_g = self._h2d("k0", k0_np, pad_to=bucket)
        starts_g = self._h2d("starts", starts_all[rows_np])
        cnt_g = self._h2d("cnt", cnt_np)
        wmask_g = self._h2d("wmask", wmask_np).bool()
        ring.write(sh, rows_g[:B], starts_g, cnt_g, wmask_g, self._accepted_path_gpu(), self._wmax())
        return rows_g, k0_g, B

    def _accepted_path_gpu(self):
        """The tree verifier's accepted node path [num_reqs, N] on the GPU, when the verifier
        publishes one (the fork's tree_state); None in chain mode, where draft j is node j."""
        if not self.branching:
            return None
        path = _STASH.get("accepted_path")
        if path is not None:
            return path
        try:
            from vllm.v1.spec_decode import tree_state
        except Exception:                           # noqa: BLE001 - the fork-only module is absent
            return None
        ts = tree_state.get_current()
        return None if ts is None else ts.accepted_path

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
        return self._beam_tree(ctx, k0_g) if self.branching else self._beam_chains(ctx, k0_g)

    @torch.inference_mode()
    def _ring_cg(self, rows_g, k0_g, B: int) -> torch.Tensor:
        """The draft of the padded batch bucket rows_g, replayed from a CUDA graph captured on the
        first use of the bucket (reference flow_proposer.py:1580-1590): the ring gather, the input
        copies and the plan launches; no host work. Drafts whose initial latents are drawn per
        draft (init_mode 'noise') run eagerly."""
        bucket = rows_g.shape[0]
        if not self.use_cg or self.init_mode == "noise" or bucket not in self._buckets:
            return self._draft_from_ring(rows_g, k0_g)[:B]
        if bucket not in self._cg:
            side = torch.cuda.Stream(self.dev)
            side.wait_stream(torch.cuda.current_stream(self.dev))
            with torch.cuda.stream(side):
                self._draft_from_ring(rows_g, k0_g)         # builds the plans (allocations) first
            torch.cuda.current_stream(self.dev).wait_stream(side)
            torch.cuda.synchronize(self.dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                out = self._draft_from_ring(rows_g, k0_g)
            self._cg[bucket] = (g, out)
        g, out = self._cg[bucket]
        g.replay()
        return out[:B]

    def device_error(self) -> int:
        """Synchronous: non-zero if a bounded device-side wait expired in any cached plan's last run."""
        return max((p.device_error() for p in self._plans.values()), default=0)

    # ------------------------------------------------------------------ vLLM entry point
    def propose(self, sampled_token_ids, num_tokens_no_spec=None, token_ids_cpu=None, slot_mappings=None,
                **kw):
        """vLLM ``custom_class`` entry (reference flow_proposer.py:1699-1988, the GPU-ring path).

        sampled_token_ids[i]: the tokens request i (input-batch row i) committed this step (empty:
        nothing to draft). The hidden states come from the runner hook (``_STASH``): row j of
        request i's run is ``sample_hidden_states[start_i + j]``. Builds on the first call.
        Returns one list per request (K chain tokens, or the N tree tokens; ``[]`` where nothing
        was drafted), or, with ``CF_ASYNC_SPEC`` under an async engine, a GPU int32
        ``[num_reqs, draft_width]`` tensor indexed by input-batch row.

        ``context_hidden=[B, C, H]`` (keyword) drafts every request from the given windows instead
        of the ring (a host that keeps its own context)."""
        ctx = kw.get("context_hidden")
        if ctx is not None:
            known0 = torch.as_tensor([int(t[-1]) for t in sampled_token_ids], device=ctx.device)
            out = self._beam_tree(ctx, known0) if self.branching else self._beam_chains(ctx, known0)
            if self.branching:
                self._stage_registration(out, list(range(len(sampled_token_ids))),
                                         [str(i) for i in range(len(sampled_token_ids))])
                out = out[:, :out.shape[1] // 2]
            return out.tolist()
        if not self.built:
            self._build()
        out: list[list[int]] = [[] for _ in sampled_token_ids]
        sh = _STASH.get("sample_hidden_states")
        if sh is None:
            return self._no_draft(out, len(sampled_token_ids))
        runner = _STASH.get("runner")
        req_ids = list(getattr(getattr(runner, "input_batch", None), "req_ids", None) or
                       [str(i) for i in range(len(sampled_token_ids))])
        rows = [i for i, t in enumerate(sampled_token_ids) if t]
        if not rows:
            return self._no_draft(out, len(sampled_token_ids))
        rows_g, k0_g, B = self._ctx_gpu(rows, req_ids, sh, sampled_token_ids)
        ch = self._ring_cg(rows_g, k0_g, B)
        if self.branching:
            self._stage_registration(ch, rows, req_ids)
        if self.async_spec:
            return self._async_draft_tensor(ch, rows, len(sampled_token_ids))
        W = self.draft_width if self.draft_width is not None else ch.shape[1]
        chains = ch[:, :W].tolist()              # the one host sync of the step
        for j, i in enumerate(rows):
            out[i] = chains[j]
        return out

    def _no_draft(self, out, nreq: int):
        """No draft this step: the empty lists, or under CF_ASYNC_SPEC a full-width tensor of zeros
        (a narrower one would leave the previous step's tokens in the persistent buffer; reference
        flow_proposer.py:1473-1509)."""
        if not self.async_spec:
            return out
        v = self._dtok_buffer()[:nreq]
        v.zero_()
        self._areg = None
        return v

    def _dtok_buffer(self) -> torch.Tensor:
        if self._dtok is None:
            self._dtok = torch.zeros((self.max_reqs, self.draft_width), dtype=torch.int32, device=self.dev)
        return self._dtok

    @torch.inference_mode()
    def _async_draft_tensor(self, ch, rows, nreq: int) -> torch.Tensor:
        """The draft as a GPU int32 [num_reqs, draft_width] tensor indexed by input-batch row, in a
        persistent buffer (the draft's own output is overwritten by the next draft), with zeros in
        the rows that did not draft (reference flow_proposer.py:2327-2357). No host sync."""
        N = self.draft_width
        if int(ch.shape[1]) < N:
            raise RuntimeError(f"draft is {tuple(ch.shape)} but {N} columns were declared to vLLM")
        v = self._dtok_buffer()[:nreq]
        if len(rows) == nreq:
            v.copy_(ch[:nreq, :N])
        else:
            v.zero_()
            v.index_copy_(0, self._h2d("dtokrows", np.asarray(rows)), ch[:len(rows), :N].to(v.dtype))
        return v

    @torch.inference_mode()
    def _stage_registration(self, ch, rows, req_ids, stream=None) -> None:
        """The tree hand-off to the verifier (reference flow_proposer.py:2360-2406): the draft's
        (tokens | parents) rows start a non-blocking copy into pinned host memory with an event, and
        the parents are copied into a persistent GPU tensor [max_reqs, N] (the draft's own output
        is overwritten by the next draft). ``tree_registration()`` joins the host copy; the fork's
        ``tree_state`` receives both when that module is present. Nothing to do for a chain: node
        j's parent is j - 1."""
        if not self.branching:
            return
        Bq, Wd = int(ch.shape[0]), int(ch.shape[1])
        N = Wd // 2
        if getattr(self, "_areg_pin", None) is None or self._areg_pin.shape != (self.max_reqs, Wd):
            self._areg_pin = torch.empty((self.max_reqs, Wd), dtype=ch.dtype, pin_memory=True)
            self._areg_ev = torch.cuda.Event()
        self._areg_pin[:Bq].copy_(ch, non_blocking=True)
        self._areg_ev.record(stream or torch.cuda.current_stream(ch.device))
        self._areg = (Bq, list(rows), list(req_ids), N)
        if self._ptree is None or self._ptree.shape != (self.max_reqs, N):
            self._ptree = torch.empty((self.max_reqs, N), dtype=ch.dtype, device=ch.device)
        self._ptree[:Bq].copy_(ch[:, N:])
        try:
            from vllm.v1.spec_decode import tree_state
        except Exception:                           # noqa: BLE001 - the fork-only module is absent
            return
        if list(rows) == list(range(len(req_ids))):
            tree_state.publish_gpu_tree(parents=self._ptree[:Bq], req_ids=req_ids, n=N, discard=lambda: None)
        else:
            tree_state.drop_gpu_tree()

    def tree_parents_gpu(self) -> torch.Tensor | None:
        """[B, N] parents (-1 = the committed token) of the last tree draft, on the GPU."""
        return None if self._areg is None else self._ptree[:self._areg[0]]

    def tree_registration(self) -> dict:
        """Join the staged host copy of the last tree draft and return {request id: (tokens, parents,
        depths)}, the registration the tree verifier needs (reference _async_register,
        flow_proposer.py:2420-2460). Node depths follow from the level-major BFS shape."""
        a = self._areg
        if a is None:
            return {}
        self._areg = None
        Bq, rows, req_ids, N = a
        self._areg_ev.synchronize()
        depths = [d for d in range(self.tree_depth) for _ in range(self.tree_keep)][:N]
        table = self._areg_pin[:Bq].tolist()
        reg = {}
        for j, i in enumerate(rows):
            rid = req_ids[i] if i < len(req_ids) else str(i)
            reg[rid] = (table[j][:N], table[j][N:], depths)
        try:
            from vllm.v1.spec_decode import tree_state
            for rid, (t, p, d) in reg.items():
                tree_state.register(rid, t, p, d)
            tree_state.drop(req_ids)
        except Exception:                           # noqa: BLE001 - the fork-only module is absent
            pass
        return reg
