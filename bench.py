#!/usr/bin/env python
"""Benchmark of the chain-flow drafting hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--workload 4b|27b|cpu]
    python bench.py --impl reference ...       # the reference algorithm on the host CPU cores
    torchrun --nproc-per-node N bench.py --gpus N ...

A step is one 5-token chain draft (flow integrator + shortlist head + top-4 beam) of B
independent requests per GPU: one persistent kernel launch up to 8 requests, above that the wide
plan (tcgen05 GEMMs over the whole batch plus row kernels). Requests are partitioned across
GPUs with no collective on the data path (weak scaling). The timed region holds inputs already
resident in HBM; the drafter's weights (2.6 GB at the 4B shape) exceed the 126 MB L2, so every
step streams them from HBM. `e2e` repeats the measurement through the proposer API with host
buffers: per step the H2D of the context window and committed token from pinned memory and
the D2H of the drafted tokens.

Prints ONE JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "drafted tokens/s (5-token chain drafts, b per GPU; ms per draft in ms_per_step)"
UNIT = "tok/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=1, help="requests per GPU")
    ap.add_argument("--workload", default="4b", choices=["4b", "27b", "cpu", "4b-ncu", "4b-prod", "27b-prod", "gdn", "gdn-verify", "ring",
                                                         "tree-attn", "tree-verify", "4b-head"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ref-device", default="cpu", choices=["cpu", "cuda"],
                    help="--impl reference: the reference algorithm on the host cores (default, fp32) or in "
                         "eager PyTorch fp16 on the GPU (the reference's eager GPU draft)")
    ap.add_argument("--twopass", type=int, default=0, metavar="M",
                    help="the two-pass candidate head with M candidates (the reference's CF_TWOPASS_M; "
                         "its default is 8192); 0 = the one-pass head BASELINE specifies")
    ap.add_argument("--head-shard", default="auto", choices=["auto", "on", "off"],
                    help="row-shard the shortlist head across the GPUs (auto: the 27B shape on >1 GPU)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-drafts", type=int, default=0, help="CPU baseline sample size (0 = auto)")
    return ap.parse_args()


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d.get("hbm_gbs", 6650.0)), "measured"
    return 6650.0, "fallback"


def measured_tensor_peak():
    """Dense fp16/bf16 tensor peak in TFLOP/s: the sustained cuBLAS figure (the wide plan is timed
    over a multi-millisecond step under the power cap)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        if "bf16_tflops_sustained" in d:
            return float(d["bf16_tflops_sustained"]), "measured (sustained)"
    return 1400.0, "fallback (sustained)"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms while active."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[1])); mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() in ("active", "1"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------------------
def oracle_flow_config(oracle, wl):
    """The flow's configuration (at the latent width for a production VAE drafter)."""
    return oracle.FlowConfig(hidden=wl.flow_width, draft_length=wl.draft_length, chunk_size=wl.chunk,
                             ffn_multiplier=wl.ffn, num_layers=wl.layers, num_flow_steps=wl.steps,
                             path_order=wl.path_order, markov_rank=wl.markov_rank)


def oracle_draft(oracle, wl, cfg, W, emb, hw, w2, sl, ctx, z0, known0):
    """One draft of the reference algorithm (oracle/ restatement): predict_hidden (with the VAE
    encode / decode around the flow for a production drafter), then the one-pass chain beam."""
    if wl.latent:
        pred = oracle.predict_hidden_vae(W, cfg, wl.vae_layers, wl.vae_heads, ctx, z0)
    else:
        pred = oracle.integrate(W, cfg, ctx, z0)
    return oracle.beam_chains(W, cfg, emb, hw, w2, sl, pred, known0, wl.width, wl.draft_tokens)


def cpu_reference_draft_rate(wl, n_drafts: int, seed: int = 0, budget_s: float = 30.0, warmup: int = 1):
    """The reference algorithm on the host cores (oracle/ restatement, fp32, all threads):
    returns (tok/s, seconds per draft, threads, sample description, timed drafts). Runs `warmup`
    untimed drafts (at least 1), then stops after `n_drafts` timed drafts or once `budget_s`
    seconds of drafting have been timed (at least 2 drafts)."""
    import oracle
    from chain_flow_b200.synthetic import make_state, make_inputs
    torch.set_num_threads(os.cpu_count() or 1)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    sd, emb, lm, sl = make_state(wl, seed=seed, device=dev)
    W = {k: v.float().cpu() for k, v in sd.items()}
    emb = emb.float().cpu()
    hw = lm[sl.to(lm.device)].float().cpu()
    w2 = W["markov.w2.weight"][sl]
    del lm, sd
    ctx, known0 = make_inputs(wl, 1, device=dev)
    ctx, known0 = ctx.float().cpu(), known0.cpu()
    cfg = oracle_flow_config(oracle, wl)
    g = torch.Generator().manual_seed(seed)
    times = []
    nw = max(1, warmup)
    with torch.inference_mode():
        for i in range(n_drafts + nw):
            z0 = torch.randn(1, wl.draft_length, wl.flow_width, generator=g)
            t0 = time.perf_counter()
            oracle_draft(oracle, wl, cfg, W, emb, hw, w2, sl, ctx, z0, known0)
            if i >= nw:                    # the warm-up drafts warm caches and threads
                times.append(time.perf_counter() - t0)
                if len(times) >= 2 and sum(times) > budget_s:
                    break
    spd = sum(times) / len(times)
    return wl.draft_tokens / spd, spd, torch.get_num_threads(), \
        f"{len(times)} drafts of the {wl.name} chain at b=1, fp32 torch on CPU (after {nw} warm-up draft{'s' if nw > 1 else ''})", \
        len(times)


def eager_gpu_reference_rate(wl, n_drafts: int, warmup: int, seed: int = 0):
    """The reference algorithm (oracle/ restatement of its eager PyTorch drafter and one-pass beam)
    in eager fp16 on cuda:0: (tok/s, seconds per draft, sample description)."""
    import oracle
    from chain_flow_b200.synthetic import make_state, make_inputs
    dev = torch.device("cuda", 0)
    sd, emb, lm, sl = make_state(wl, seed=seed, device=dev)
    sl = sl.to(dev)
    hw = lm[sl].contiguous()
    w2 = sd["markov.w2.weight"][sl].contiguous()
    del lm
    ctx, known0 = make_inputs(wl, 1, device=dev)
    cfg = oracle_flow_config(oracle, wl)
    g = torch.Generator(device=dev).manual_seed(seed)

    def draft():
        z0 = torch.randn(1, wl.draft_length, wl.flow_width, generator=g, device=dev, dtype=torch.float16)
        return oracle_draft(oracle, wl, cfg, sd, emb, hw, w2, sl, ctx, z0, known0)

    with torch.inference_mode():
        for _ in range(max(1, warmup)):
            draft()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n_drafts):
            draft()
        e1.record()
        torch.cuda.synchronize(dev)
    spd = e0.elapsed_time(e1) / 1e3 / n_drafts
    return wl.draft_tokens / spd, spd, (f"{n_drafts} drafts of the {wl.name} chain at b=1: the reference algorithm "
                                       f"in eager PyTorch fp16 on the GPU (no CUDA graph, no compile)")


def run_reference(args, wl):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    n = max(1, args.steps)
    if args.ref_device == "cuda":
        rate, spd, sample = eager_gpu_reference_rate(wl, n, args.warmup)
        line = {
            "metric": METRIC, "value": rate, "unit": UNIT, "impl": "reference", "n_gpus": 1, "steps": n,
            "warmup": args.warmup, "ms_per_step": spd * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded random weights and inputs)",
            "config": {"workload": wl.name, "batch_per_gpu": 1, "draft_tokens": wl.draft_tokens,
                       "hidden": wl.hidden, "blocks": wl.layers, "euler_steps": wl.steps,
                       "shortlist_rows": wl.shortlist_rows, "beam_width": wl.width, "device": "cuda"},
            "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "reference_sample": sample,
        }
        print(json.dumps(line), flush=True)
        return
    rate, spd, threads, sample, timed = cpu_reference_draft_rate(wl, n, warmup=args.warmup)
    line = {
        "metric": METRIC, "value": rate, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
        "steps": timed, "warmup": max(1, args.warmup), "ms_per_step": spd * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random weights and inputs)",
        "config": {"workload": wl.name, "batch_per_gpu": 1, "draft_tokens": wl.draft_tokens,
                   "hidden": wl.hidden, "blocks": wl.layers, "euler_steps": wl.steps,
                   "shortlist_rows": wl.shortlist_rows, "beam_width": wl.width},
        "cpu_baseline": {"value": rate, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------
def run_ours(args, wl):
    import torch.distributed as dist
    from chain_flow_b200 import _lib
    from chain_flow_b200.proposer import FlowDrafterProposer
    from chain_flow_b200.synthetic import make_state, make_inputs

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (the engine has no CPU path)")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    B = args.batch
    shard = world > 1 and (args.head_shard == "on" or (args.head_shard == "auto" and wl.hidden >= 5120))
    if args.twopass:
        if shard:
            raise SystemExit("--twopass runs on unsharded heads only")
        os.environ["CF_TWOPASS_M"] = str(args.twopass)
    sd, emb, lm, sl = make_state(wl, seed=0, device=dev)
    # sharded head: every rank drafts the same requests (same inputs and noise), each over its
    # share of the head rows; otherwise each rank drafts its own requests
    prop = FlowDrafterProposer.from_components(sd, wl.model_args(), emb, lm, sl, width=wl.width,
                                               K=wl.draft_tokens, device=dev,
                                               seed=1000 + (0 if shard else rank),
                                               head_shard=(rank, world) if shard else None,
                                               group=dist.group.WORLD if shard else None)
    del sd, lm
    torch.cuda.empty_cache()
    ctx, known0 = make_inputs(wl, B, seed=1 + (0 if shard else rank), device=dev)
    stream = torch.cuda.current_stream(dev)

    # ---- device-resident throughput: K drafts, inputs in HBM. The clock sampler starts first:
    # nvidia-smi's start-up must not fall inside the timed region.
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(1.0)
    for _ in range(args.warmup):
        prop._beam_chains(ctx, known0)
    torch.cuda.synchronize(dev)
    barrier(); torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        out = prop._beam_chains(ctx, known0)
    e1.record(stream)
    torch.cuda.synchronize(dev); barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    clk = clocks.stop()
    if prop.device_error():
        raise SystemExit(f"device-side wait timed out (code {prop.device_error()})")

    # ---- the plan alone (roofline): back-to-back runs of the bound plan. Up to MAX_PLAN_BATCH
    # requests that is one persistent-engine launch; above it, the wide plan's launch list
    # (tcgen05 GEMMs and row kernels); a sharded head runs engine plans of MAX_PLAN_BATCH.
    from chain_flow_b200.proposer import MAX_PLAN_BATCH
    wide = B > MAX_PLAN_BATCH and not shard and not args.twopass
    plan = prop._wide_plan(_lib.MODE_CHAIN, B) if wide else prop._plan(_lib.MODE_CHAIN, min(B, MAX_PLAN_BATCH))
    plans_per_step = 1 if wide else (B + MAX_PLAN_BATCH - 1) // MAX_PLAN_BATCH
    torch.cuda.synchronize(dev)
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0.record(stream)
    for _ in range(args.steps):
        plan.run(group=prop.group)
    k1.record(stream)
    torch.cuda.synchronize(dev)
    kernel_ms = max_over_ranks(k0.elapsed_time(k1) / args.steps)

    # ---- a production draft's latent flow alone: the work of the reference's fused-kernel
    # integrate() (all Euler steps of both chunk experts over the 8-block stack at the latent
    # width, one persistent-engine launch here), back-to-back launches on resident inputs
    flow = None
    flow_plan = getattr(plan, "flow", None)
    if wl.latent and flow_plan is not None:
        for _ in range(3):
            flow_plan.run()
        torch.cuda.synchronize(dev)
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            flow_plan.run()
        f1.record(stream)
        torch.cuda.synchronize(dev)
        flow_plan.check()
        fbytes = wl.flow_weight_bytes()
        f_ms = max_over_ranks(f0.elapsed_time(f1) / args.steps)
        flow = {"ms": f_ms, "latent": wl.latent, "blocks": wl.layers, "euler_steps": wl.steps,
                "bytes_per_launch": fbytes, "achieved_gbs": fbytes / (f_ms / 1e3) / 1e9,
                # the reference kernel's published integrate() at B = 1 (RTX PRO 6000, compiled and
                # graph-replayed; reference docs/BENCHMARKING.md:141-146)
                "reference_integrate_ms": {640: 0.803, 1024: 1.364}.get(wl.latent)}

    # ---- end to end through the proposer API with host buffers
    h_ctx = ctx.cpu().pin_memory()
    h_k0 = known0.cpu().pin_memory()
    h_out = torch.empty((B, wl.draft_tokens), dtype=torch.int64).pin_memory()
    d_ctx = torch.empty_like(ctx); d_k0 = torch.empty_like(known0)
    for _ in range(2):
        d_ctx.copy_(h_ctx, non_blocking=True); d_k0.copy_(h_k0, non_blocking=True)
        h_out.copy_(prop._beam_chains(d_ctx, d_k0), non_blocking=True)
        torch.cuda.synchronize(dev)
    barrier(); torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(args.steps):
        d_ctx.copy_(h_ctx, non_blocking=True)
        d_k0.copy_(h_k0, non_blocking=True)
        h_out.copy_(prop._beam_chains(d_ctx, d_k0), non_blocking=True)
        stream.synchronize()                     # the host reads the drafted tokens every step
    e1.record(stream)
    torch.cuda.synchronize(dev); barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    h2d = h_ctx.numel() * h_ctx.element_size() + h_k0.numel() * h_k0.element_size()
    d2h = h_out.numel() * h_out.element_size()

    # ---- the shortlist head alone (engine plans): a profiled run of the same plan. Each beam
    # depth's head phase is the GEMM phase whose post-op publishes the head lists (the plan's
    # phase table); its wall is from the previous phase's last grid-barrier pass to its own.
    head = None
    peak_hbm = measured_peaks()[0]
    if not wide and not shard and rank == 0 and not args.twopass:
        from chain_flow_b200.engine import Plan
        if prop.vae is not None:        # the beam plan of a production draft, on that draft's hidden states
            pp = Plan(prop.weights, _lib.MODE_BEAM_CHAIN, min(B, MAX_PLAN_BATCH), width=wl.width,
                      depth=wl.draft_tokens, profile=True)
            pp.pred.copy_(plan.pred); pp.known0.copy_(plan.known0)
        else:
            pp = Plan(prop.weights, _lib.MODE_CHAIN, min(B, MAX_PLAN_BATCH), width=wl.width, depth=wl.draft_tokens,
                      profile=True, init_mode=_lib.INIT_MODES[prop.init_mode])
            pp.ctx.copy_(plan.ctx); pp.z0.copy_(plan.z0); pp.known0.copy_(plan.known0)
        for _ in range(2):
            pp.run()
        torch.cuda.synchronize(dev)
        pp.check()
        t = pp.phase_times().double()                       # [phases, grid, 20] ns
        kinds = pp.phase_table()
        ends = t[:, :, 2].max(dim=1).values
        walls, streams = [], []
        for i in range(1, t.shape[0]):
            if int(kinds[i, 0]) == _lib.PK_GEMM and int(kinds[i, 6]) == _lib.PO_PUBLISH:
                walls.append(float(ends[i] - ends[i - 1]) / 1e3)
                has = t[i, :, 10] > 0
                streams.append(float(t[i, has, 11].max() - ends[i - 1]) / 1e3)
        hbytes = wl.shortlist_rows * (wl.hidden + wl.markov_rank) * 2
        # plans of more than 2 requests run an engine build without the profiling stamps
        if walls and min(walls) > 0 and min(streams) > 0:
            w_us = statistics.median(walls)
            s_us = statistics.median(streams)
            head = {"depths": len(walls), "bytes_per_depth": hbytes, "us_per_depth": w_us,
                    "achieved_gbs": hbytes / (w_us * 1e3), "frac": hbytes / (w_us * 1e3) / peak_hbm,
                    "stream_us": s_us, "stream_gbs": hbytes / (s_us * 1e3),
                    "how": "median over beam depths of the head phase's wall (previous phase's last barrier "
                           "pass to its own), from a CFB_RUN_PROFILE run of the same plan; stream = to the "
                           "last weight unit ready"}
        del pp

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:   # the host baseline: N=1 only
        n = args.cpu_drafts or (3 if wl.hidden >= 2560 else 20)
        if wl.hidden <= 2560:
            rate, spd, threads, sample, _ = cpu_reference_draft_rate(wl, n)
            cpu = {"value": rate, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample}

    if rank == 0:
        peak, peak_kind = measured_peaks()
        algo = wl.weight_bytes_per_draft(head_fraction=1.0 / world if shard else 1.0, twopass_m=args.twopass,
                                         batch=min(B, MAX_PLAN_BATCH))   # per GPU, per plan
        achieved = algo / (kernel_ms / 1e3) / 1e9
        flops = wl.flops_per_draft(B if wide else min(B, MAX_PLAN_BATCH))
        tpeak, tpeak_kind = measured_tensor_peak()
        tensor_bound = wide and flops / (tpeak * 1e12) > algo / (peak * 1e9)
        traffic, traffic_note = None, None
        tf = ROOT / "profiles" / "engine_dram_traffic.json"
        if tf.exists():
            tj = json.loads(tf.read_text())
            t = tj.get(wl.name)
            if not (t and int(t.get("batch", -1)) == B):
                t = tj.get(f"{wl.name}-b{B}")
            if t and int(t.get("batch", -1)) == B:
                traffic = t.get("bytes_per_launch")
                traffic_note = "measured" if t.get("measured") else f"scaled from {t.get('scaled_from')}"
        tokens = (1 if shard else world) * B * wl.draft_tokens
        line = {
            "metric": METRIC, "value": tokens / (ms / 1e3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if shard else "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded random-init reference-architecture drafter, N(0,1) hidden states)",
            "config": {"workload": wl.name, "batch_per_gpu": B, "draft_tokens": wl.draft_tokens,
                       "hidden": wl.hidden, "blocks": wl.layers, "euler_steps": wl.steps,
                       "ffn_multiplier": wl.ffn, "shortlist_rows": wl.shortlist_rows,
                       "beam_width": wl.width, "plans_per_step": plans_per_step,
                       "head": (f"two-pass, {args.twopass} shared candidates (CF_TWOPASS_M)" if args.twopass
                                else "one-pass fused top-k (CF_TWOPASS_M=0)"),
                       **({"vae": {"latent": wl.latent, "intermediate": wl.vae_inter, "layers": wl.vae_layers,
                                   "heads": wl.vae_heads},
                           "draft_length": wl.draft_length, "chunk": wl.chunk, "path_order": wl.path_order}
                          if wl.latent else {}),
                       "path": (("VAE encode -> latent flow -> VAE decode -> beam: "
                                 + ("wide launch lists and wide plans" if wide else "four persistent-engine launches"))
                                if wl.latent else
                                "wide plan: tcgen05 GEMMs + row kernels, one launch list per step" if wide
                                else "persistent engine: one cooperative launch per plan"),
                       "parallelism": (f"shortlist head rows sharded over {world} GPUs, flow replicated, "
                                       f"one NCCL all_gather of merged top-k lists per depth") if shard
                       else f"requests split over {world} GPU(s)",
                       "l2": f"inputs larger than L2: {algo / 1e9:.2f} GB of fp16 weights stream from HBM "
                             f"every step"},
            "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
            "gpu_launches": args.steps * plans_per_step * getattr(plan, "launches", plan.segments),
            "roofline": ({"bound": "tensor", "achieved": flops / (kernel_ms / 1e3) / 1e12, "peak": tpeak,
                          "unit": "TFLOP/s", "frac": flops / (kernel_ms / 1e3) / 1e12 / tpeak, "traffic": None,
                          "peak_source": tpeak_kind, "kernel": "wide plan (all launches; tcgen05 GEMMs dominate)",
                          "kernel_ms": kernel_ms, "algorithmic_flops_per_step": flops,
                          "hbm_gbs": achieved} if tensor_bound else
                         {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                          "frac": achieved / peak, "traffic": traffic if not wide else None,
                          "traffic_source": traffic_note if not wide else None,
                          "peak_source": peak_kind,
                          "kernel": ("whole production draft (VAE launches + flow + beam)" if wl.latent else
                                     "wide plan (all launches; tcgen05 GEMMs dominate)" if wide else "engine_kernel"),
                          "kernel_ms": kernel_ms, "algorithmic_bytes_per_launch": algo,
                          "tflops": flops / (kernel_ms / 1e3) / 1e12}),
            "clocks": clk,
            "shortlist_head": head,
            **({"flow_integrate": flow} if flow else {}),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------------------------------------
def run_gdn(args):
    """tree-aware Gated-DeltaNet verification of one layer, 16 heads,
    Dk = Dv = 128, fp32 state, a 16-node tree of depth 5 and branching <= 4 per request, at
    B = 1, 8 and 64 (one JSON line per B). A step is one cfb_tree_gdn launch over B requests.
    Algorithmic bytes per request: the prefix state read and the 16 node states written (fp32),
    q/k/v (fp16), g/beta (fp32), o (fp32)."""
    from chain_flow_b200.gdn import make_tree, tree_gdn_batched
    import oracle
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    dev = torch.device("cuda", 0)
    N, H, Dk, Dv = 16, 16, 128, 128
    peak, peak_kind = measured_peaks()
    per_req = H * Dk * Dv * 4 * (1 + N) + N * H * ((2 * Dk + Dv) * 2 + 8 + Dv * 4)
    for B in (1, 8, 64):
        g = torch.Generator(device=dev).manual_seed(B)
        q = torch.nn.functional.normalize(torch.randn(B, N, H, Dk, device=dev, generator=g), dim=-1).half()
        k = torch.nn.functional.normalize(torch.randn(B, N, H, Dk, device=dev, generator=g), dim=-1).half()
        v = torch.randn(B, N, H, Dv, device=dev, generator=g).half()
        gl = torch.log(torch.sigmoid(torch.randn(B, N, H, device=dev, generator=g)))
        beta = torch.sigmoid(torch.randn(B, N, H, device=dev, generator=g))
        par = torch.stack([make_tree(N, 5, 4, seed=b)[0] for b in range(B)]).to(dev)
        init = torch.randn(B, H, Dk, Dv, device=dev, generator=g) * 0.1
        states = torch.empty(B, N, H, Dk, Dv, device=dev)
        for _ in range(max(3, args.warmup)):
            tree_gdn_batched(q, k, v, gl, beta, par, init, states=states)
        torch.cuda.synchronize(dev)
        # device time from graph replays: one request's launch is shorter than a Python call
        ms, timed = _graph_time_ms(lambda: tree_gdn_batched(q, k, v, gl, beta, par, init, states=states), args.steps)
        achieved = B * per_req / (ms / 1e3) / 1e9
        # CPU baseline: the reference recurrence (oracle) on the host cores, one request
        torch.set_num_threads(os.cpu_count() or 1)
        qc, kc, vc = q[0].cpu(), k[0].cpu(), v[0].cpu()
        gc, bc, ic = gl[0].cpu(), beta[0].cpu(), init[0].cpu()
        pc = par[0].cpu()
        dep = make_tree(N, 5, 4, seed=0)[1]
        oracle.tree_gdn_scan(qc, kc, vc, gc, bc, pc, dep, ic)
        t0 = time.perf_counter()
        reps = 3
        for _ in range(reps):
            oracle.tree_gdn_scan(qc, kc, vc, gc, bc, pc, dep, ic)
        cpu_s = (time.perf_counter() - t0) / reps
        line = {"metric": "tree GDN verification: requests/s (16-node trees, 16 heads, Dk=Dv=128)",
                "value": B / (ms / 1e3), "unit": "req/s", "n_gpus": 1, "steps": timed,
                "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded q,k,v,alpha,beta,trees)",
                "config": {"workload": "cfg4-tree-gdn", "batch": B, "nodes": N, "heads": H, "dk": Dk, "dv": Dv,
                           "timing": f"CUDA graph replays, {timed} launches"},
                "gpu_launches": timed,
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "traffic": None, "peak_source": peak_kind,
                             "kernel": "tree_gdn_kernel", "algorithmic_bytes_per_launch": B * per_req},
                "cpu_baseline": {"value": 1.0 / cpu_s, "unit": "req/s", "cores": torch.get_num_threads(),
                                 "kind": "port", "sample": f"{reps} single-request scans, oracle fp32 on CPU"}}
        print(json.dumps(line), flush=True)


def run_gdn_verify(args):
    """The in-engine tree GDN verify of the reference's vLLM patch at its own shapes: one GDN
    layer of the 4B target (16 key heads, 32 value heads, K = V = 128, fp32 state of 2 MiB per
    slot), a 41-node draft tree per request (the reference's 40 + root) walked path-parallel from
    the request's prefix slot, bf16 q/k/v. One JSON line per B in (1, 8). Algorithmic bytes per
    request: its prefix state read once and 41 node states written (fp32), plus q/k/v/a/b/o."""
    from chain_flow_b200.gdn import ancestor_chains, gdn_verify, make_tree
    import oracle
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    dev = torch.device("cuda", 0)
    N, H, HV, K, V, MAXD = 41, 16, 32, 128, 128, 6
    peak, peak_kind = measured_peaks()
    slot = HV * V * K * 4
    per_req = slot * (1 + N) + N * (H * K * 2 * 2 + HV * V * 2 * 2 + HV * 8)
    for B in (1, 8):
        g = torch.Generator(device=dev).manual_seed(B)
        T = B * N
        q = torch.randn(T, H, K, device=dev, generator=g).bfloat16()
        k = torch.randn(T, H, K, device=dev, generator=g).bfloat16()
        v = torch.randn(T, HV, V, device=dev, generator=g).bfloat16()
        a = torch.randn(T, HV, device=dev, generator=g)
        b = torch.randn(T, HV, device=dev, generator=g)
        A_log = torch.randn(HV, device=dev, generator=g) * 0.5
        dt_bias = torch.randn(HV, device=dev, generator=g) * 0.5
        chains, depths = [], []
        for r in range(B):
            par, _ = make_tree(N, MAXD, 4, seed=r)
            ch, dp = ancestor_chains(par, MAXD)
            chains.append(ch + r * N); depths.append(dp)
        chain = torch.cat(chains).to(dev); depth = torch.cat(depths).to(dev)
        init_slot = (torch.arange(T, device=dev) // N).to(torch.int32)            # request r's prefix: slot r
        out_slot = (B + torch.arange(T, device=dev)).to(torch.int32)
        state = torch.randn(B + T, HV, V, K, device=dev, generator=g) * 0.1
        o = torch.empty(T, HV, V, device=dev, dtype=torch.bfloat16)
        run = lambda: gdn_verify(A_log, dt_bias, a, b, q, k, v, o, state, chain, depth, out_slot, init_slot,
                                 scale=K ** -0.5)
        for _ in range(max(3, args.warmup)):
            run()
        torch.cuda.synchronize(dev)
        # device time from graph replays: one request's launch is about as long as a Python call
        ms, timed = _graph_time_ms(run, args.steps)
        achieved = B * per_req / (ms / 1e3) / 1e9
        # CPU baseline: the oracle's restatement of the reference kernel, one request, all threads
        torch.set_num_threads(os.cpu_count() or 1)
        sl = slice(0, N)
        args_c = [t.cpu() for t in (A_log, dt_bias, a[sl], b[sl], q[sl], k[sl], v[sl])]
        st_c = state[:1].cpu()
        t0 = time.perf_counter()
        oracle.tree_gdn_verify(*args_c, st_c, chain[sl].cpu(), depth[sl].cpu(), torch.zeros(N, dtype=torch.int32),
                               torch.zeros(N, dtype=torch.int32), K ** -0.5, write_state=False)
        cpu_s = time.perf_counter() - t0
        line = {"metric": "in-engine tree GDN verify: requests/s (41-row trees, 32 value heads, K=V=128)",
                "value": B / (ms / 1e3), "unit": "req/s", "n_gpus": 1, "steps": timed,
                "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32 state, bf16 q/k/v",
                "data": "synthetic (seeded q,k,v,a,b,A_log,dt_bias,trees)",
                "config": {"workload": "gdn-verify (reference in-engine shape)", "batch": B, "rows_per_request": N,
                           "heads": H, "value_heads": HV, "dk": K, "dv": V,
                           "timing": f"CUDA graph replays, {timed} launches"},
                "gpu_launches": timed,
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "traffic": None, "peak_source": peak_kind,
                             "kernel": "tree_gdn_verify_kernel", "algorithmic_bytes_per_launch": B * per_req},
                "cpu_baseline": {"value": 1.0 / cpu_s, "unit": "req/s", "cores": torch.get_num_threads(),
                                 "kind": "port", "sample": "1 request (41 rows), oracle fp32 on CPU"}}
        print(json.dumps(line), flush=True)
        # the same outputs by the shared-root factorisation (reference fork gdn_factor): the root
        # state is read once per (request, head) and no state is written
        from chain_flow_b200.gdn import gdn_factor
        row_start = (torch.arange(B, device=dev) * N).to(torch.int32)
        row_count = torch.full((B,), N, dtype=torch.int32, device=dev)
        fac = lambda: gdn_factor(A_log, dt_bias, a, b, q, k, v, o, state, chain, depth, init_slot, row_start,
                                 row_count, scale=K ** -0.5, n_max=N)
        for _ in range(max(3, args.warmup)):
            fac()
        torch.cuda.synchronize(dev)
        fms, ftimed = _graph_time_ms(fac, args.steps)
        fbytes = B * (slot + N * (H * K * 2 * 2 + HV * V * 2 * 2 + HV * 8))
        t0 = time.perf_counter()
        oracle.tree_gdn_factor(*args_c, st_c, chain[sl].cpu(), depth[sl].cpu(), torch.zeros(N, dtype=torch.int32),
                               torch.zeros(1, dtype=torch.int32), torch.full((1,), N, dtype=torch.int32), K ** -0.5)
        fcpu = time.perf_counter() - t0
        line = {"metric": "tree GDN verify outputs, shared-root factorisation: requests/s (41-row trees, 32 value heads)",
                "value": B / (fms / 1e3), "unit": "req/s", "n_gpus": 1, "steps": ftimed,
                "warmup": max(3, args.warmup), "ms_per_step": fms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32 state, bf16 q/k/v",
                "data": "synthetic (seeded q,k,v,a,b,A_log,dt_bias,trees)",
                "config": {"workload": "gdn-factor (reference in-engine shape)", "batch": B, "rows_per_request": N,
                           "heads": H, "value_heads": HV, "dk": K, "dv": V,
                           "note": "outputs only; the accepted leaf's state is materialised afterwards by the verify",
                           "timing": f"CUDA graph replays, {ftimed} launches"},
                "gpu_launches": ftimed,
                "roofline": {"bound": "latency (hbm figure for context)", "achieved": fbytes / (fms / 1e3) / 1e9,
                             "peak": peak, "unit": "GB/s", "frac": fbytes / (fms / 1e3) / 1e9 / peak, "traffic": None,
                             "peak_source": peak_kind, "kernel": "tree_gdn_factor_kernel",
                             "algorithmic_bytes_per_launch": fbytes},
                "cpu_baseline": {"value": 1.0 / fcpu, "unit": "req/s", "cores": torch.get_num_threads(),
                                 "kind": "port", "sample": "1 request (41 rows), factor oracle fp32 on CPU"}}
        print(json.dumps(line), flush=True)


def run_ring(args):
    """The context ring (reference _ring_write / _ring_gather, flow_proposer.py:916-961) at the 4B
    hidden size: 256 request slots of C=8 rows, each step appends K+1 = 6 accepted rows per request
    (a chain step) and gathers every request's window, at B = 1, 8, 64 and 256 requests. A step is
    one cfb_ring_write and one cfb_ring_gather launch. Algorithmic bytes per request: the appended
    rows read and written, the window read and written (fp16)."""
    from chain_flow_b200.ring import ContextRing
    import oracle
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    dev = torch.device("cuda", 0)
    slots, C, H, K1 = 256, 8, 2560, 6
    peak, peak_kind = measured_peaks()
    per_req = 2 * K1 * H * 2 + 2 * C * H * 2
    for B in (1, 8, 64, 256):
        g = torch.Generator(device=dev).manual_seed(B)
        ring = ContextRing(slots, C, H, device=dev)
        rows = torch.randperm(slots, generator=g, device=dev)[:B]
        sh = torch.randn(B * K1, H, generator=g, device=dev).half()
        starts = torch.arange(B, device=dev) * K1
        cnt = torch.full((B,), K1, dtype=torch.long, device=dev)
        wmask = torch.ones(B, dtype=torch.bool, device=dev)
        out = torch.empty(B, C, H, dtype=torch.float16, device=dev)
        for _ in range(max(3, args.warmup)):
            ring.write(sh, rows, starts, cnt, wmask, None, K1)
            ring.gather(rows, out=out)
        torch.cuda.synchronize(dev)
        # the two launches take a few microseconds; issued one by one from Python the host is the
        # bottleneck, so the timed steps replay a CUDA graph of `per_graph` steps (no allocation
        # or host sync happens inside either call)
        per_graph = 20
        side = torch.cuda.Stream(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph, stream=side):
                for _ in range(per_graph):
                    ring.write(sh, rows, starts, cnt, wmask, None, K1, stream=side)
                    ring.gather(rows, out=out, stream=side)
        torch.cuda.synchronize(dev)
        graph.replay()
        torch.cuda.synchronize(dev)
        reps_g = max(1, args.steps // per_graph)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps_g):
            graph.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / (reps_g * per_graph)
        achieved = B * per_req / (ms / 1e3) / 1e9
        # CPU baseline: the reference's ring semantics (oracle) on the host cores
        torch.set_num_threads(os.cpu_count() or 1)
        rc, rp, nv = ring.ring.cpu(), ring.rpos.cpu(), ring.nval.cpu()
        args_c = (sh.cpu(), rows.cpu(), starts.cpu(), cnt.cpu(), wmask.cpu(), None, K1)
        t0 = time.perf_counter()
        reps = 3
        for _ in range(reps):
            oracle.ring_write(rc, rp, nv, *args_c)
            oracle.ring_gather(rc, rp, nv, rows.cpu())
        cpu_s = (time.perf_counter() - t0) / reps
        line = {"metric": "context ring: requests/s (append 6 rows + gather the 8-row window, H=2560)",
                "value": B / (ms / 1e3), "unit": "req/s", "n_gpus": 1, "steps": reps_g * per_graph,
                "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded hidden states and slots)",
                "config": {"workload": "a1-context-ring", "batch": B, "slots": slots, "rows": C, "hidden": H,
                           "appended": K1, "timing": f"CUDA graph of {per_graph} steps, replayed {reps_g} times"},
                "gpu_launches": 2 * per_graph * reps_g,
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "traffic": None, "peak_source": peak_kind,
                             "kernel": "ring_write_kernel + ring_gather_kernel",
                             "algorithmic_bytes_per_launch": B * per_req},
                "cpu_baseline": {"value": B / cpu_s, "unit": "req/s", "cores": torch.get_num_threads(),
                                 "kind": "port", "sample": f"{reps} steps of {B} requests, oracle on CPU"}}
        print(json.dumps(line), flush=True)


def _graph_time_ms(fn, steps: int, per_graph: int = 20) -> tuple[float, int]:
    """Mean device time of one fn() call, from a CUDA graph of per_graph calls replayed until
    `steps` calls have been timed (CUDA events around the replays): the kernels are a few
    microseconds long, so launched one by one from Python the host would be the bound."""
    dev = torch.device("cuda", 0)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(per_graph):
            fn()
    graph.replay()
    torch.cuda.synchronize(dev)
    reps = max(1, steps // per_graph)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    del graph
    return e0.elapsed_time(e1) / (reps * per_graph), reps * per_graph


def run_tree_attn(args):
    """The tree-attention fix-up of one full-attention layer of the target (the reference fork's
    suffix_merge, vllm-0.25.1-chain-flow-tree.patch:5235-5540): every node of a 40-node draft tree
    attends to its ancestors and is merged with the paged-prefix result. The reference measures
    5.33 us per layer at 4B (H=16, HKV=4, D=256) and 5.74 us at 27B (H=24) on its RTX PRO 6000,
    under CUDA-graph replay (patch:2819-2824). A step is one cfb_tree_attn_merge launch; one JSON
    line per shape. Algorithmic bytes per launch: the q, k, v, prefix and output rows, the prefix
    log-sum-exps, the node table and the ancestor mask."""
    from chain_flow_b200.gdn import make_tree
    from chain_flow_b200.tree import ancestor_mask, tree_attn_merge
    import oracle
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    dev = torch.device("cuda", 0)
    peak, peak_kind = measured_peaks()
    N, D = 40, 256
    for S, H, HKV, shape in ((1, 16, 4, "4B"), (1, 24, 4, "27B"), (8, 16, 4, "4B")):
        g = torch.Generator(device=dev).manual_seed(S * H)
        T = S * N
        dt = torch.bfloat16
        q = torch.randn(T, H, D, device=dev, generator=g).to(dt)
        k = torch.randn(T, HKV, D, device=dev, generator=g).to(dt)
        v = torch.randn(T, HKV, D, device=dev, generator=g).to(dt)
        po = torch.randn(T, H, D, device=dev, generator=g).to(dt)
        plse = torch.randn(H, T, device=dev, generator=g)
        idx = torch.arange(T, device=dev).view(S, N)
        par = torch.stack([make_tree(N, 5, 4, seed=s)[0] for s in range(S)]).to(dev)
        mask = ancestor_mask(par)
        out = torch.empty(T, H, D, device=dev, dtype=dt)
        scale = D ** -0.5
        ms, n = _graph_time_ms(lambda: tree_attn_merge(q, k, v, out, po, plse, idx, mask, scale), max(args.steps, 20))
        nbytes = T * H * D * 2 * 3 + T * HKV * D * 2 * 2 + H * T * 4 + T * 8 + S * N * N
        torch.set_num_threads(os.cpu_count() or 1)
        args_c = [t.cpu() for t in (q, k, v, out, po, plse, idx, mask)]
        t0 = time.perf_counter()
        oracle.tree_attn_merge(*args_c, scale)
        cpu_s = time.perf_counter() - t0
        line = {"metric": "tree-attention suffix + LSE merge: us per full-attention layer (40-node tree)",
                "value": ms * 1e3, "unit": "us", "n_gpus": 1, "steps": n, "warmup": 3, "ms_per_step": ms,
                "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (fp32 math)",
                "data": "synthetic (seeded q,k,v,prefix rows, BFS trees of depth 5)",
                "config": {"workload": f"tree-attn ({shape} target layer)", "requests": S, "nodes": N, "heads": H,
                           "kv_heads": HKV, "head_dim": D,
                           "timing": "CUDA graph of 20 launches (the reference's figure is under graph replay)",
                           "reference_us_per_layer": 5.33 if H == 16 else 5.74},
                "gpu_launches": n,
                "roofline": {"bound": "latency (hbm figure for context)", "achieved": nbytes / (ms / 1e3) / 1e9,
                             "peak": peak, "unit": "GB/s", "frac": nbytes / (ms / 1e3) / 1e9 / peak, "traffic": None,
                             "peak_source": peak_kind, "kernel": "tree_attn_merge_kernel",
                             "algorithmic_bytes_per_launch": nbytes},
                "cpu_baseline": {"value": cpu_s * 1e6, "unit": "us", "cores": torch.get_num_threads(),
                                 "kind": "port", "sample": "1 layer, oracle fp32 on CPU"}}
        print(json.dumps(line), flush=True)


def run_tree_verify(args):
    """Greedy verification of a draft tree (the reference fork's tree_rejection_sample,
    vllm-0.25.1-chain-flow-tree.patch:640-723): the argmax of every logits row (41 rows per request:
    the committed token and 40 tree nodes, over the 248,320-token vocabulary) and the walk down the
    tree, in one launch. A step is one cfb_tree_verify_greedy launch; one JSON line per batch.
    Algorithmic bytes: the logits rows."""
    from chain_flow_b200.gdn import make_tree
    from chain_flow_b200.tree import TreeVerifier
    import oracle
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    dev = torch.device("cuda", 0)
    peak, peak_kind = measured_peaks()
    N, V = 40, 248320
    for B, dt in ((1, torch.bfloat16), (8, torch.bfloat16), (8, torch.float32)):
        g = torch.Generator(device=dev).manual_seed(B)
        rows = B * (N + 1)
        logits = torch.randn(rows, V, device=dev, generator=g).to(dt)
        pars = torch.cat([make_tree(N, 5, 4, seed=b)[0] for b in range(B)]).to(dev)
        toks = torch.randint(0, V, (B * N,), device=dev, generator=g)
        cu_d = torch.arange(1, B + 1, device=dev) * N
        cu_s = torch.arange(1, B + 1, device=dev) * (N + 1)
        ver = TreeVerifier(rows, B, N, device=dev)
        ms, n = _graph_time_ms(lambda: ver(logits, cu_d, cu_s, toks, pars), max(args.steps, 20))
        nbytes = rows * V * logits.element_size()
        torch.set_num_threads(os.cpu_count() or 1)
        lc = logits.cpu()
        t0 = time.perf_counter()
        oracle.tree_verify_greedy(lc, cu_d.cpu(), cu_s.cpu(), toks.cpu(), pars.cpu(), N)
        cpu_s = time.perf_counter() - t0
        line = {"metric": "greedy tree verification: us per verify (argmax of 41 logits rows per request + descent)",
                "value": ms * 1e3, "unit": "us", "n_gpus": 1, "steps": n, "warmup": 3, "ms_per_step": ms,
                "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16 logits" if dt == torch.bfloat16 else "f32 logits",
                "data": "synthetic (seeded logits, BFS trees of depth 5)",
                "config": {"workload": "tree-verify", "requests": B, "nodes": N, "vocab": V,
                           "timing": "CUDA graph of 20 launches; logits larger than L2 at 8 requests"},
                "gpu_launches": n,
                "roofline": {"bound": "hbm", "achieved": nbytes / (ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                             "frac": nbytes / (ms / 1e3) / 1e9 / peak, "traffic": None, "peak_source": peak_kind,
                             "kernel": "tree_verify_greedy_kernel", "algorithmic_bytes_per_launch": nbytes},
                "cpu_baseline": {"value": cpu_s * 1e6, "unit": "us", "cores": torch.get_num_threads(),
                                 "kind": "port", "sample": f"1 verify of {B} requests, oracle on CPU"}}
        print(json.dumps(line), flush=True)


def run_head(args):
    """The beam half of a cfg 2 (4B) draft alone: a CFB_MODE_BEAM_CHAIN engine plan over given
    integrated hidden states, b=1 and 8, i.e. per depth the path residual, the shortlist head (62,642
    rows of [lm_head | markov w2], 352.8 MB) with its fused log-sum-exp / top-k, and the beam step.
    Here the head is the dominant traffic, so the plan's HBM fraction is the head's (north_star: >=
    0.70 of HBM on the shortlist head). Timed with CUDA events over back-to-back launches; the
    2 GB of head and path weights a draft streams exceed L2."""
    from chain_flow_b200 import _lib
    from chain_flow_b200.engine import Plan
    from chain_flow_b200.proposer import FlowDrafterProposer
    from chain_flow_b200.synthetic import WORKLOADS, make_state
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    dev = torch.device("cuda", 0)
    wl = WORKLOADS["4b"]
    peak, peak_kind = measured_peaks()
    sd, emb, lm, sl = make_state(wl, seed=0, device=dev)
    prop = FlowDrafterProposer.from_components(sd, wl.model_args(), emb, lm, sl, width=wl.width, K=wl.draft_tokens,
                                               device=dev, seed=1000)
    del sd, lm
    torch.cuda.empty_cache()
    row = wl.hidden + wl.markov_rank
    for B in (1, 8):
        p = Plan(prop.weights, _lib.MODE_BEAM_CHAIN, B, width=wl.width, depth=wl.draft_tokens)
        g = torch.Generator(device=dev).manual_seed(B)
        p.pred.copy_(torch.randn(p.pred.shape, device=dev, generator=g))
        p.known0.copy_(torch.randint(0, wl.vocab, (B,), device=dev, generator=g))
        for _ in range(max(3, args.warmup)):
            p.run()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            p.run()
        e1.record()
        torch.cuda.synchronize(dev)
        p.check()
        ms = e0.elapsed_time(e1) / args.steps
        head = wl.draft_tokens * wl.shortlist_rows * row * 2
        path = sum(2 * (min(d, wl.path_order) * wl.hidden ** 2 + 4 * wl.hidden ** 2)
                   for d in range(1, wl.draft_tokens + 1))
        nbytes = head + path
        line = {"metric": "beam half of a 4B draft (path residual + shortlist head + beam, 5 depths): ms per draft",
                "value": ms, "unit": "ms", "n_gpus": 1, "steps": args.steps, "warmup": max(3, args.warmup),
                "ms_per_step": ms, "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
                "data": "synthetic (seeded random-init head, N(0,1) hidden states)",
                "config": {"workload": "cfg2-4B beam plan (CFB_MODE_BEAM_CHAIN)", "batch": B, "depths": wl.draft_tokens,
                           "shortlist_rows": wl.shortlist_rows, "head_bytes_per_depth": wl.shortlist_rows * row * 2,
                           "l2": "inputs larger than L2: 1.76 GB of head weights stream from HBM every step"},
                "gpu_launches": args.steps,
                "roofline": {"bound": "hbm", "achieved": nbytes / (ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                             "frac": nbytes / (ms / 1e3) / 1e9 / peak, "traffic": None, "peak_source": peak_kind,
                             "kernel": "engine_kernel (beam plan)", "algorithmic_bytes_per_launch": nbytes,
                             "head_share_of_bytes": head / nbytes}}
        print(json.dumps(line), flush=True)
        del p


def main():
    args = parse()
    if args.workload == "4b-head":
        run_head(args)
        return
    if args.workload == "tree-attn":
        run_tree_attn(args)
        return
    if args.workload == "tree-verify":
        run_tree_verify(args)
        return
    if args.workload == "ring":
        run_ring(args)
        return
    if args.workload == "gdn":
        run_gdn(args)
        return
    if args.workload == "gdn-verify":
        run_gdn_verify(args)
        return
    from chain_flow_b200.synthetic import WORKLOADS
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, wl)
    else:
        run_ours(args, wl)


if __name__ == "__main__":
    main()
