#!/usr/bin/env python
"""Routed tokens/s of one SPALMER micro-expert MoE layer forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config m100] [--impl ours|reference]

One step = one full layer forward (router GEMM, exact top-k, dispatch, grouped
expert SwiGLU, shared SwiGLU + combine, statistics, auxiliary loss) over the
configuration's tokens.  Multi-GPU runs are data parallel (every rank owns its
own tokens and a replica of the weights; no collective in the forward), so
``value`` is weak-scaled: total tokens of all ranks / slowest rank's time.

``value`` is timed on the device with CUDA events around K back-to-back steps,
inputs resident in HBM and larger than L2 (two hidden-state batches
alternated, plus the weights).  ``e2e`` is the
same metric through the public module API with host buffers: pinned H2D of the
step's hidden states, the forward, and D2H of the update and auxiliary loss,
all inside the timed region.  ``--impl reference`` times the CPU restatement
of the reference path (``oracle/``, numpy + the standard-library top-k) on the
host cores, on a bounded token sample per step.
"""

from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    # 100M-preset shape, a seeded 25% of the experts in MXFP8, the rest BF16 (the headline workload).
    "m100": dict(cfg=dict(d_model=768, num_experts=200, expert_inter_dim=128, shared_inter_dim=768,
                          active_experts=8), batch=64, seq=1024, cpu_sample=1024, ref_sample=16384, mxfp8_fraction=0.25),
    # The same shape with a seeded 25% of the experts in NVFP4 (E2M1, UE4M3 per 1x16, per-tensor
    # scales; the reference's ("nvfp4", "nvfp4") pair), the rest BF16.
    "m100_nvfp4": dict(cfg=dict(d_model=768, num_experts=200, expert_inter_dim=128, shared_inter_dim=768,
                                active_experts=8, expert_execution="loop"), batch=64, seq=1024, cpu_sample=1024, ref_sample=8192,
                       mxfp8_fraction=0.25, lowp_format="nvfp4"),
    # The same shape with every expert in BF16.
    "m100_bf16": dict(cfg=dict(d_model=768, num_experts=200, expert_inter_dim=128, shared_inter_dim=768,
                               active_experts=8), batch=64, seq=1024, cpu_sample=1024, ref_sample=16384),
    # Skewed expert parallel (Zipf(1.1) router bias), 131072 tokens in total,
    # experts sharded E/N per GPU with NCCL all-to-all (strong scaling).  S = 2*d (reference default).
    "ep_skew": dict(cfg=dict(d_model=1024, num_experts=200, expert_inter_dim=256, shared_inter_dim=2048,
                             active_experts=8, router_bias=True), batch=128, seq=1024, cpu_sample=256, ref_sample=8192,
                    zipf=True, expert_parallel=True),
    # The same with the rows moved by NCCL all-to-all-v instead of stores into the peers' buffers.
    "ep_skew_nccl": dict(cfg=dict(d_model=1024, num_experts=200, expert_inter_dim=256, shared_inter_dim=2048,
                                  active_experts=8, router_bias=True), batch=128, seq=1024, cpu_sample=256, ref_sample=8192,
                         zipf=True, expert_parallel=True, exchange="nccl"),
    # The same with token rows sent once per destination GPU and pair rows summed
    # at the expert's GPU before they return.
    "ep_skew_dedup": dict(cfg=dict(d_model=1024, num_experts=200, expert_inter_dim=256, shared_inter_dim=2048,
                                   active_experts=8, router_bias=True), batch=128, seq=1024, cpu_sample=256, ref_sample=8192,
                          zipf=True, expert_parallel=True, dedup=True),
    # Decode-shaped steps through a 16-layer stack (independent seeded weights per
    # layer, 10% of each layer's experts in MXFP8); the forward of the stack is one CUDA graph.
    "decode": dict(cfg=dict(d_model=768, num_experts=200, expert_inter_dim=128, shared_inter_dim=768,
                            active_experts=8), batch=1, seq=64, cpu_sample=64, mxfp8_fraction=0.10,
                   decode_layers=16, decode_tokens=(1, 8, 64)),
    # Training step (forward + backward) of the 100M-shape layer, BF16 experts
    # (the MXFP8 lane has no backward); loss = sum(update * dU) + aux.
    "m100_train": dict(cfg=dict(d_model=768, num_experts=200, expert_inter_dim=128, shared_inter_dim=768,
                                active_experts=8), batch=64, seq=1024, cpu_sample=256, ref_sample=4096, train=True),
    # Paged expert offload (the reference's inference offload, experts/offload.py): the expert
    # bank stays in pinned host memory behind a device cache of half the experts; every step
    # stages the experts it selects through the cache page by page.
    "m100_paged": dict(cfg=dict(d_model=768, num_experts=200, expert_inter_dim=128, shared_inter_dim=768,
                                active_experts=8), batch=64, seq=1024, cpu_sample=256, ref_sample=16384,
                      paged=dict(cache_size=100)),
    # Decode-shaped paged steps: 64 new tokens per step through one layer, a 64-expert cache.
    "decode_paged": dict(cfg=dict(d_model=768, num_experts=200, expert_inter_dim=128, shared_inter_dim=768,
                                  active_experts=8), batch=1, seq=64, cpu_sample=64, paged=dict(cache_size=64)),
    # 10M-preset shape.
    "m10": dict(cfg=dict(d_model=256, num_experts=200, expert_inter_dim=64, shared_inter_dim=256,
                         active_experts=8), batch=32, seq=512, cpu_sample=4096, ref_sample=16384),
    # CPU-runnable smoke layer.
    "smoke": dict(cfg=dict(d_model=128, num_experts=200, expert_inter_dim=32, shared_inter_dim=128,
                           active_experts=4), batch=2, seq=256, cpu_sample=512),
}
METRIC = "routed tokens/sec per MoE layer"
E2E_REPS = 5  # repetitions of the timed steps for the end-to-end figure (median reported)
# DRAM bytes (read + write) of the roofline stage's launches in one forward,
# from an ncu capture of the same workload (dram__bytes_read.sum +
# dram__bytes_write.sum over the stage's launches): hidden-state quantiser +
# both expert GEMM1 lanes for m100.
STAGE_TRAFFIC_BYTES = {"m100": 624.8e6}
CPU_ALL_BF16_NOTE = ("; all experts BF16: the reference has no CPU MXFP8 path and rejects BF16 experts "
                     "mixed with MXFP8 (experts/config.py:140-161)")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data["hbm_gbs"], "bf16_tflops": data["bf16_tflops"],
                "bf16_tflops_sustained": data.get("bf16_tflops_sustained"), "source": "measured"}
    return dict(FALLBACK_PEAKS)


def mxfp8_experts(num_experts: int, fraction: float):
    """Seeded MXFP8 expert set: the first ceil(fraction * E) of randperm(E, seed 2)."""

    import math

    perm = torch.randperm(num_experts, generator=torch.Generator().manual_seed(2))
    lane = torch.zeros(num_experts, dtype=torch.bool)
    lane[perm[: math.ceil(fraction * num_experts)]] = True
    return lane


def build_mixer(spec: dict, device=None, seed: int = 0):
    """The bench layer: seed-0 random init; MXFP8 configs run their seeded expert set in MXFP8.

    The reference expresses a mixed layer as MXFP8 expert weights whose promoted
    experts run BF16 (experts/bank.py:462-475, experts/config.py:140-161), so
    every expert outside the MXFP8 set is marked promoted.
    """

    from spalmer_b200 import B200MicroExpertChannelMixer, MicroExpertsConfig

    fraction = spec.get("mxfp8_fraction", 0.0)
    zipf = spec.get("zipf", False)
    cfg = dict(spec["cfg"])
    if fraction > 0:
        fmt = spec.get("lowp_format", "mxfp8")
        cfg.update(expert_weight_format=fmt, expert_activation_format=fmt, expert_promotion_format="bfloat16")
    config = MicroExpertsConfig(**cfg)
    torch.manual_seed(seed)
    mixer = B200MicroExpertChannelMixer(config).to(torch.bfloat16).eval()
    lane = None
    if fraction > 0:
        lane = mxfp8_experts(config.num_experts, fraction)
        with torch.no_grad():
            mixer.potentiation_controller.promoted_mask.copy_(~lane)
    if zipf:
        # b_e = alpha * ln(rank_e) over randperm(E, seed 3); alpha fitted for Zipf(1.1) popularity
        alpha = json.loads((ROOT / "tests" / "golden" / "zipf_ep_skew.json").read_text())["alpha"]
        perm = torch.randperm(config.num_experts, generator=torch.Generator().manual_seed(3))
        rank = torch.empty(config.num_experts)
        rank[perm] = torch.arange(1, config.num_experts + 1, dtype=torch.float32)
        with torch.no_grad():
            mixer.router.proj.bias.copy_(alpha * torch.log(rank))
    if device is not None:
        mixer = mixer.to(device)
    return mixer, lane


def layer_flops(cfg: dict, tokens: int) -> dict:
    d, E, I, k = cfg["d_model"], cfg["num_experts"], cfg["expert_inter_dim"], cfg["active_experts"]
    S = cfg["shared_inter_dim"]
    P = tokens * k
    return {
        "router_gemm": 2.0 * tokens * d * E,
        "expert_gemm1_swiglu": 2.0 * P * d * 2 * I,
        "expert_gemm2_scatter": 2.0 * P * I * d,
        "shared_gemm1_swiglu": 2.0 * tokens * d * 2 * S,
        "shared_gemm2_combine": 2.0 * tokens * S * d,
    }


def workload_config(name: str, world: int) -> dict:
    spec = CONFIGS[name]
    cfg = spec["cfg"]
    ep = spec.get("expert_parallel", False)
    extra = {}
    if ep:
        extra = {"total_tokens": spec["batch"] * spec["seq"], "experts_per_gpu": cfg["num_experts"] // world,
                 "row_dedup": bool(spec.get("dedup", False)),
                 "router_bias": "Zipf(1.1) popularity: b_e = alpha*ln(rank_e), alpha from tests/golden/zipf_ep_skew.json",
                 "exchange": ("NCCL all_to_all_single (counts, rows out, rows back); one host read of the counts"
                              if spec.get("exchange") == "nccl" or spec.get("dedup") else
                              "counts all-gathered (one host read); rows stored straight into the peers' IPC "
                              "buffers by spx_rows_to_peers, a one-element NCCL all-reduce after each move")}
    return {
        "workload": f"{name}: SPALMER micro-expert layer forward" + (" (expert parallel)" if ep and world > 1 else ""),
        **extra,
        "tokens_per_gpu": spec["batch"] * spec["seq"] // (world if ep else 1),
        "batch": spec["batch"], "seq_len": spec["seq"],
        "d_model": cfg["d_model"], "num_experts": cfg["num_experts"],
        "expert_inter_dim": cfg["expert_inter_dim"], "top_k": cfg["active_experts"],
        "shared_inter_dim": cfg["shared_inter_dim"],
        "expert_precision": (
            (f"NVFP4 (E2M1, UE4M3 per 1x16 along K, per-tensor FP32 scales) for a seeded "
             f"{spec['mxfp8_fraction']:.0%} of the experts (randperm seed 2), BF16 for the rest")
            if spec.get("lowp_format") == "nvfp4" else
            (f"MXFP8 (E4M3, E8M0 per 1x32 along K) for a seeded {spec['mxfp8_fraction']:.0%} "
             "of the experts (randperm seed 2), BF16 for the rest")
            if spec.get("mxfp8_fraction") else "BF16 for all experts"),
        "weights": "random init, torch.manual_seed(0), N(0,0.02)",
        "l2": (f"inputs larger than L2: two {spec['batch'] * spec['seq'] * cfg['d_model'] * 2 / 1e6 / (world if ep else 1):.1f} MB "
               "hidden-state batches alternated, plus the weights; steps timed back to back"),
        "parallelism": f"ep{world}" if ep and world > 1 else f"dp{world}",
    }


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(device_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(",") for r in out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" in r[5 + i] and "Not" not in r[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


REF_SITE = ROOT / "baseline" / "_ref"


def reference_package():
    """The reference package as installed by ``oracle/install_ref.py`` (unmodified
    mESmaC/spalmer sources under baseline/_ref), or None when it is absent."""

    if not (REF_SITE / "spalmer" / "experts" / "mixer.py").is_file():
        return None
    if str(REF_SITE) not in sys.path:
        sys.path.insert(0, str(REF_SITE))
    import spalmer.experts as ref_experts

    return ref_experts


def reference_mixer(spec: dict, seed: int = 0):
    """The reference's own MicroExpertChannelMixer (experts/mixer.py:54-241) for the
    workload, built under torch.manual_seed(seed) and cast to BF16 on the CPU.
    Every expert is BF16: the reference has no CPU MXFP8/NVFP4 path and rejects
    BF16 experts mixed with a low-precision promotion (experts/config.py:140-161)."""

    E = reference_package()
    config = E.MicroExpertsConfig(**spec["cfg"])
    torch.manual_seed(seed)
    mixer = E.MicroExpertChannelMixer(config).to(torch.bfloat16).eval()
    if spec.get("zipf"):
        alpha = json.loads((ROOT / "tests" / "golden" / "zipf_ep_skew.json").read_text())["alpha"]
        perm = torch.randperm(config.num_experts, generator=torch.Generator().manual_seed(3))
        rank = torch.empty(config.num_experts)
        rank[perm] = torch.arange(1, config.num_experts + 1, dtype=torch.float32)
        with torch.no_grad():
            mixer.router.proj.bias.copy_(alpha * torch.log(rank))
    return mixer


def reference_step(spec: dict, mixer, x: torch.Tensor, du: torch.Tensor | None):
    """One step of the reference on the CPU: its forward under torch.no_grad(),
    or for training configs forward + backward through its own autograd graph."""

    if du is None:
        with torch.no_grad():
            mixer(x)
        return
    mixer.zero_grad(set_to_none=True)
    xg = x.detach().requires_grad_(True)
    out = mixer(xg)
    torch.autograd.backward([out.update, out.auxiliary_loss], [du, torch.ones((), dtype=out.auxiliary_loss.dtype)])


def reference_inputs(spec: dict, d_model: int, sample: int):
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(1, sample, d_model, generator=gen).to(torch.bfloat16)
    du = (0.05 * torch.randn(1, sample, d_model, generator=gen)).to(torch.bfloat16) if spec.get("train") else None
    return x, du


def reference_note(spec: dict, name: str, sample: int, runs: str) -> str:
    what = "forward + backward (autograd)" if spec.get("train") else "forward under torch.no_grad()"
    return (f"{sample} tokens of the {name} workload through the reference's own "
            f"MicroExpertChannelMixer {what} (baseline/_ref, torch CPU BF16, "
            f"expert_execution={spec['cfg'].get('expert_execution', 'grouped')!r}), {runs}"
            + CPU_ALL_BF16_NOTE * bool(spec.get("mxfp8_fraction")))


def run_reference_arm(args) -> None:
    """The reference's own CPU implementation of the layer, timed on the host
    cores with every thread torch may use: one step = one forward (training
    configs: forward + backward) over a bounded token sample of the workload;
    value = sample tokens / median step time.  Without the reference install,
    the CPU restatement in oracle/ stands in (kind "port")."""

    world, rank, _ = init_dist()
    if rank != 0:
        return
    spec = CONFIGS[args.config]
    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()
    ref_error = None
    try:
        ref = reference_package()
    except Exception as exc:  # noqa: BLE001 - reported in the line
        ref, ref_error = None, f"{type(exc).__name__}: {exc}"
    if ref is not None:
        sample = spec.get("ref_sample", spec["cpu_sample"])
        mixer = reference_mixer(spec)
        x, du = reference_inputs(spec, mixer.config.d_model, sample)
        try:
            for _ in range(args.warmup):
                reference_step(spec, mixer, x, du)
        except RuntimeError as exc:  # e.g. a host without a verified CPU BF16 lane
            ref, ref_error = None, f"{type(exc).__name__}: {exc}"
    if ref is not None:
        times = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            reference_step(spec, mixer, x, du)
            times.append(time.perf_counter() - t0)
        kind = "reference"
        note = reference_note(spec, args.config, sample, f"median of {len(times)} steps after {args.warmup} warm-up")
    else:
        import numpy as np  # noqa: F401

        from oracle import mixer_ref as R
        from tests.helpers import bf16_bits, oracle_params

        mixer, _ = build_mixer(spec)
        config = mixer.config
        params = oracle_params(mixer)
        sample = spec["cpu_sample"]
        xt = torch.randn(sample, config.d_model, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
        x_bits = bf16_bits(xt)
        k = config.active_experts
        for _ in range(args.warmup):
            R.mixer_forward(params, x_bits, k)
        times = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            R.mixer_forward(params, x_bits, k)
            times.append(time.perf_counter() - t0)
        kind = "port"
        note = (f"{sample} tokens of the {args.config} workload through the CPU restatement (oracle/, numpy), "
                f"median of {len(times)} steps; reference install unavailable ({ref_error or 'baseline/_ref absent'})"
                + CPU_ALL_BF16_NOTE * bool(spec.get("mxfp8_fraction")))
    med_s = statistics.median(times)
    value = sample / med_s
    line = {
        "impl": "reference", "metric": METRIC + (" (training step: forward + backward)" if spec.get("train") else ""),
        "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": med_s * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {**workload_config(args.config, world),
                   **({"workload": f"{args.config}: SPALMER micro-expert layer forward + backward"}
                      if spec.get("train") else {})},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": kind, "sample": note},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline(args, mixer, x_cpu) -> dict:
    """The reference's own CPU forward (or, without the reference install, the
    oracle restatement) on a bounded sample of this workload: median of at
    least 3 runs after one warm-up, about 15 s of CPU work at most."""

    spec = CONFIGS[args.config]
    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()
    try:
        ref = reference_package()
    except Exception:  # noqa: BLE001
        ref = None
    if ref is not None:
        sample = spec.get("ref_sample", spec["cpu_sample"])
        rmixer = reference_mixer(spec)
        x, du = reference_inputs(spec, rmixer.config.d_model, sample)
        try:
            reference_step(spec, rmixer, x, du)
        except RuntimeError:
            ref = None
    if ref is not None:
        times = []
        t_end = time.perf_counter() + 15.0
        while len(times) < 3 or (time.perf_counter() < t_end and len(times) < 10):
            t0 = time.perf_counter()
            reference_step(spec, rmixer, x, du)
            times.append(time.perf_counter() - t0)
        med = statistics.median(times)
        return {"value": sample / med, "unit": "tokens/s", "cores": cores, "kind": "reference",
                "sample": reference_note(spec, args.config, sample, f"median of {len(times)} runs")}
    from oracle import mixer_ref as R
    from tests.helpers import bf16_bits, oracle_params

    sample = spec["cpu_sample"]
    params = oracle_params(mixer)
    x_bits = bf16_bits(x_cpu.reshape(-1, x_cpu.shape[-1])[:sample])
    k = mixer.config.active_experts
    R.mixer_forward(params, x_bits, k)
    times = []
    t_end = time.perf_counter() + 15.0
    while len(times) < 3 or (time.perf_counter() < t_end and len(times) < 10):
        t0 = time.perf_counter()
        R.mixer_forward(params, x_bits, k)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": sample / med, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{sample} tokens of the {args.config} workload, median of {len(times)} runs "
                      f"(CPU restatement, numpy/OpenBLAS on all host threads; reference install absent)"
                      + CPU_ALL_BF16_NOTE * bool(spec.get("mxfp8_fraction"))}


def run_ours(args) -> None:
    world, rank, local = init_dist()
    import torch.distributed as dist

    from spalmer_b200 import _lib

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    spec = CONFIGS[args.config]
    batch, seq = spec["batch"], spec["seq"]
    tokens = batch * seq
    mixer, lane = build_mixer(spec, device)
    config = mixer.config
    x_cpu = torch.randn(batch, seq, config.d_model, generator=torch.Generator().manual_seed(1 + rank))
    x_cpu = x_cpu.to(torch.bfloat16)
    x_host = x_cpu.pin_memory()
    # Two distinct input batches, alternated step to step: 2 x 100.7 MB of hidden
    # states plus 121.6 MB of weights exceed the 126 MB L2 (and every step also
    # streams ~1 GB of intermediates), so no step starts from a warm L2.
    x_bufs = [x_host.to(device), x_host.roll(1, dims=0).to(device)]
    K, W = args.steps, args.warmup

    def barrier():
        if world > 1:
            dist.barrier()

    with torch.inference_mode():
        # Warm-up runs the timed loop's exact pattern (the previous step's outputs
        # stay alive while the next step allocates), so the caching allocator
        # holds both output sets before timing starts.
        out = None
        for i in range(W):
            out = mixer(x_bufs[i % 2])
        torch.cuda.synchronize()
        stage_sets = [[torch.cuda.Event(enable_timing=True) for _ in range(_lib.STAGE_EVENTS)] for _ in range(K)]
        for st in stage_sets:
            for ev in st:
                ev.record()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        sampler = ClockSampler(local)
        time.sleep(0.3)
        t0.record()
        for i in range(K):
            mixer.record_stage_events(stage_sets[i])
            out = mixer(x_bufs[i % 2])
        t1.record()
        torch.cuda.synchronize()
        barrier()
        clocks = sampler.stop()
        mixer.record_stage_events(None)
        status = mixer.device_status()
        total_ms = t0.elapsed_time(t1)
        stages = {}
        for j, name in enumerate(_lib.STAGE_NAMES):
            stages[name] = sum(st[j].elapsed_time(st[j + 1]) for st in stage_sets) / K

        # e2e through the module API with host buffers.  Every step copies its
        # own hidden states in from pinned host memory and its update + aux
        # loss back out; the copies run on their own streams (double-buffered)
        # so step i's H2D/D2H overlap the neighbouring steps' compute.
        main = torch.cuda.current_stream(device)
        s_in = torch.cuda.Stream(device)
        s_out = torch.cuda.Stream(device)
        x_dev = [torch.empty_like(x_bufs[0]) for _ in range(2)]
        out_host = [torch.empty(batch, seq, config.d_model, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        aux_host = [torch.empty((), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        freed = [torch.cuda.Event() for _ in range(2)]  # x_dev[b] consumed by its forward
        for ev in freed:
            ev.record(main)

        def e2e_steps(n):
            for i in range(n):
                b = i % 2
                with torch.cuda.stream(s_in):
                    s_in.wait_event(freed[b])
                    x_dev[b].copy_(x_host, non_blocking=True)
                    loaded = torch.cuda.Event()
                    loaded.record(s_in)
                main.wait_event(loaded)
                o = mixer(x_dev[b])
                freed[b].record(main)
                with torch.cuda.stream(s_out):
                    s_out.wait_stream(main)
                    o.update.record_stream(s_out)
                    o.auxiliary_loss.record_stream(s_out)
                    out_host[b].copy_(o.update, non_blocking=True)
                    aux_host[b].copy_(o.auxiliary_loss, non_blocking=True)

        # E2E_REPS repetitions of the K timed steps, each bracketed like the
        # device-timed region; the line reports the median repetition (a host
        # stall in one repetition, e.g. another job on the box's cores, moves
        # the median little) and lists every repetition.
        e2e_steps(W)
        e2e_reps = []
        for _ in range(E2E_REPS):
            torch.cuda.synchronize()
            barrier()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(main)
            s_in.wait_stream(main)
            e2e_steps(K)
            main.wait_stream(s_out)
            e1.record(main)
            torch.cuda.synchronize()
            barrier()
            e2e_reps.append(e0.elapsed_time(e1))

        # The host link alone: the same pinned copies per step (hidden states in,
        # update and aux loss out) on the same two copy streams, no forward.
        # e2e cannot beat this; with N ranks the copies of all ranks share the
        # host's PCIe / memory bandwidth.
        def copy_steps(n):
            for i in range(n):
                b = i % 2
                with torch.cuda.stream(s_in):
                    x_dev[b].copy_(x_host, non_blocking=True)
                with torch.cuda.stream(s_out):
                    out_host[b].copy_(x_bufs[b].view(batch, seq, config.d_model), non_blocking=True)
                    aux_host[b].copy_(out.auxiliary_loss, non_blocking=True)

        copy_steps(W)
        copy_reps = []
        for _ in range(E2E_REPS):
            torch.cuda.synchronize()
            barrier()
            c0 = torch.cuda.Event(enable_timing=True)
            c1 = torch.cuda.Event(enable_timing=True)
            c0.record(main)
            s_in.wait_stream(main)
            s_out.wait_stream(main)
            copy_steps(K)
            main.wait_stream(s_in)
            main.wait_stream(s_out)
            c1.record(main)
            torch.cuda.synchronize()
            barrier()
            copy_reps.append(c0.elapsed_time(c1))

    # max over ranks (every repetition separately), then the median repetition
    t = torch.tensor([total_ms] + e2e_reps + copy_reps, dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    t = t.tolist()
    total_ms = t[0]
    e2e_reps, copy_reps = t[1:1 + E2E_REPS], t[1 + E2E_REPS:]
    e2e_ms, copy_ms = statistics.median(e2e_reps), statistics.median(copy_reps)
    ms_per_step = total_ms / K
    value = world * tokens / (ms_per_step / 1e3)
    e2e_value = world * tokens / (e2e_ms / K / 1e3)

    if rank == 0:
        pk = peaks()
        flops = layer_flops(spec["cfg"], tokens)
        dom = "expert_gemm1_swiglu"
        dom_ms = stages[dom]
        achieved = flops[dom] / (dom_ms / 1e3) / 1e12
        # MXFP8 pairs run at twice the BF16 tensor rate: the roofline peak of the
        # stage is the FLOP-weighted blend of the two lanes' peaks.
        mx_share = 0.0
        if lane is not None:
            util = out.metrics["expert_utilization"].float().cpu()
            mx_share = float(util[lane].sum())
        nvfp4 = spec.get("lowp_format") == "nvfp4"
        lowp_speed = 4.0 if nvfp4 else 2.0  # dense FP4 / FP8 tensor rate over BF16
        peak = pk["bf16_tflops"] / ((1.0 - mx_share) + mx_share / lowp_speed)
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1) hidden states, seeded random-init weights)",
            "config": workload_config(args.config, world),
            "e2e": {"value": e2e_value, "unit": "tokens/s",
                    "h2d_bytes_per_step": tokens * config.d_model * 2,
                    "d2h_bytes_per_step": tokens * config.d_model * 2 + 2,
                    "ms_per_step": e2e_ms / K,
                    "reps_ms_per_step": [r / K for r in e2e_reps],
                    "what": f"median of {E2E_REPS} repetitions of the {K} steps; max over ranks per repetition",
                    "host_link_bound": {
                        "value": world * tokens / (copy_ms / K / 1e3), "unit": "tokens/s",
                        "ms_per_step": copy_ms / K,
                        "gbs_all_ranks": world * (2 * tokens * config.d_model * 2 + 2) / (copy_ms / K / 1e3) / 1e9,
                        "what": "the same pinned H2D + D2H copies per step on the same streams, no forward; "
                                "max over ranks"}},
            "gpu_launches": K * ((17 if nvfp4 else 14) if lane is not None else 11),
            "roofline": {"bound": "tensor",
                         "kernel": ("gemm_kernel<kEpiSwiglu> (expert GEMM1; BF16 lane gathered rows, "
                                    + ("NVFP4 lane E2M1 rows)" if nvfp4 else "MXFP8 lane)")),
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": STAGE_TRAFFIC_BYTES.get(args.config),
                         "traffic_unit": "bytes per forward (ncu dram read+write of the stage's launches)",
                         "mxfp8_pair_share": mx_share,
                         "peak_source": f"{pk['source']} bf16 burst; " + ("NVFP4 share at 4x" if nvfp4
                                                                             else "MXFP8 share at 2x")},
            "layer_tensor_tflops": sum(flops.values()) / (ms_per_step / 1e3) / 1e12,
            "stages_ms": stages,
            "device_status": status,
        }
        if clocks is not None:
            line["clocks"] = clocks
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args, mixer, x_cpu)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_ep(args) -> None:
    """Strong-scaled expert-parallel forward: the configuration's tokens split
    over the ranks, experts sharded E/N per GPU, rows exchanged over NCCL."""

    world, rank, local = init_dist()
    import torch.distributed as dist

    from spalmer_b200.ep import ExpertParallelMixer

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    spec = CONFIGS[args.config]
    total = spec["batch"] * spec["seq"]
    batch = spec["batch"] // world
    seq = spec["seq"]
    tokens = batch * seq
    mixer, _ = build_mixer(spec, device)
    config = mixer.config
    layer = (ExpertParallelMixer(mixer, dedup=spec.get("dedup", False), exchange=spec.get("exchange"))
             if world > 1 else None)
    x_cpu = torch.randn(spec["batch"], seq, config.d_model, generator=torch.Generator().manual_seed(1))
    x_cpu = x_cpu.to(torch.bfloat16)[rank * batch:(rank + 1) * batch].contiguous()
    x_host = x_cpu.pin_memory()
    x_bufs = [x_host.to(device), x_host.roll(1, dims=0).to(device)]
    K, W = args.steps, args.warmup

    def step(x):
        if layer is not None:
            return layer(x)["update"]
        return mixer(x).update

    def barrier():
        if world > 1:
            dist.barrier()

    with torch.inference_mode():
        for i in range(W):
            out = step(x_bufs[i % 2])
        torch.cuda.synchronize()
        barrier()
        sampler = ClockSampler(local)
        time.sleep(0.3)
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for i in range(K):
            out = step(x_bufs[i % 2])
        t1.record()
        torch.cuda.synchronize()
        barrier()
        clocks = sampler.stop()
        total_ms = t0.elapsed_time(t1)
        loads = None
        exchanged = None
        stage_ms = None
        if layer is not None:
            r = layer(x_bufs[0])
            loads = r.get("recv_pairs", r["recv_rows"])
            exchanged = sum(r["send_rows"])
            # stage split: events at every stage boundary on the compute stream
            # (outside the timed region; the stages stay stream-ordered)
            layer.record_stages(True)
            for i in range(max(K // 2, 3)):
                layer(x_bufs[i % 2])
            stage_ms = layer.stage_times()
            layer.record_stages(False)
            torch.cuda.synchronize()
            barrier()
        # e2e: pinned H2D of this rank's tokens, forward, D2H of the update, per step
        out_host = torch.empty(batch, seq, config.d_model, dtype=torch.bfloat16).pin_memory()
        xd = torch.empty_like(x_bufs[0])
        for _ in range(W):
            xd.copy_(x_host, non_blocking=True)
            out_host.copy_(step(xd), non_blocking=True)
        torch.cuda.synchronize()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(K):
            xd.copy_(x_host, non_blocking=True)
            out_host.copy_(step(xd), non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        barrier()
        e2e_ms = e0.elapsed_time(e1)
    t = torch.tensor([total_ms, e2e_ms], dtype=torch.float64, device=device)
    recv = torch.tensor([float(sum(loads)) if loads else float(tokens * config.active_experts)],
                        dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        all_recv = [torch.zeros_like(recv) for _ in range(world)]
        dist.all_gather(all_recv, recv)
        recv_loads = [float(v) for v in all_recv]
    else:
        recv_loads = [float(recv)]
    total_ms, e2e_ms = float(t[0]), float(t[1])
    ms_per_step = total_ms / K
    if rank == 0:
        pk = peaks()
        flops = sum(layer_flops(spec["cfg"], total).values()) / world
        line = {
            "metric": METRIC, "value": total / (ms_per_step / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) hidden states, seeded random-init weights, Zipf router bias)",
            "config": workload_config(args.config, world),
            "e2e": {"value": total / (e2e_ms / K / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": tokens * config.d_model * 2, "d2h_bytes_per_step": tokens * config.d_model * 2},
            "gpu_launches": K * (13 if world > 1 else 11),
            "roofline": {"bound": "tensor", "kernel": "whole layer per GPU (expert-parallel stages)",
                         "achieved": flops / (ms_per_step / 1e3) / 1e12, "peak": pk["bf16_tflops_sustained"] or pk["bf16_tflops"],
                         "unit": "TFLOP/s", "traffic": None, "peak_source": f"{pk['source']} bf16 sustained"},
            "expert_rows_per_gpu": recv_loads,
            "rows_sent_per_gpu_rank0": exchanged,
            "max_over_mean_expert_load": max(recv_loads) / (sum(recv_loads) / len(recv_loads)),
            "stages_ms_rank0": stage_ms,
        }
        line["roofline"]["frac"] = line["roofline"]["achieved"] / line["roofline"]["peak"]
        if clocks is not None:
            line["clocks"] = clocks
        print(json.dumps(line), flush=True)
    if layer is not None:
        layer.close()
    if world > 1:
        dist.destroy_process_group()


def run_decode(args) -> None:
    """Decode-shaped steps: T tokens (T = 1, 8, 64) through a 16-layer stack
    of MoE layers with residual adds, captured once as a CUDA graph per T and
    replayed.  value = routed tokens/s per layer at the largest T; the other
    token counts are reported beside it.  Data parallel replicas for N > 1."""

    world, rank, local = init_dist()
    import torch.distributed as dist

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    spec = CONFIGS[args.config]
    L = spec["decode_layers"]
    layers = [build_mixer(spec, device, seed=l)[0] for l in range(L)]
    config = layers[0].config
    K, W = max(args.steps, 10), args.warmup
    per_t = {}
    clocks = None
    e2e = {}
    token_counts = [args.tokens] if args.tokens else list(spec["decode_tokens"])
    with torch.inference_mode():
        for T in token_counts:
            x_host = torch.randn(1, T, config.d_model, generator=torch.Generator().manual_seed(1 + rank))
            x_host = x_host.to(torch.bfloat16).pin_memory()
            x_static = x_host.to(device)

            def stack(x):
                for m in layers:
                    x = x + m(x).update
                return x

            for _ in range(W):  # eager warm-up: packs weights, sizes workspaces, caches launch attributes
                out = stack(x_static)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                out_static = stack(x_static)
            for _ in range(W):
                graph.replay()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            sampler = ClockSampler(local) if T == token_counts[-1] else None
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record()
            for _ in range(K):
                graph.replay()
            t1.record()
            torch.cuda.synchronize()
            if sampler is not None:
                clocks = sampler.stop()
            ms = t0.elapsed_time(t1) / K
            # e2e: pinned H2D of the step's tokens, the graph, D2H of the output
            out_host = torch.empty(1, T, config.d_model, dtype=torch.bfloat16).pin_memory()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(K):
                x_static.copy_(x_host, non_blocking=True)
                graph.replay()
                out_host.copy_(out_static, non_blocking=True)
            e1.record()
            torch.cuda.synchronize()
            t = torch.tensor([ms, e0.elapsed_time(e1) / K], dtype=torch.float64, device=device)
            if world > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            per_t[T] = (float(t[0]), float(t[1]))
            del graph
    T = token_counts[-1]
    ms, e2e_ms = per_t[T]
    if rank == 0:
        pk = peaks()
        # weight bytes a step must read per layer: distinct experts (expected 200(1-(1-k/E)^T)) x their
        # BF16/MXFP8 bytes, plus shared and router weights
        E, d, I, k, S = config.num_experts, config.d_model, config.resolved_inter_dim, config.active_experts, 768
        frac = spec["mxfp8_fraction"]
        per_expert = (1 - frac) * 3 * d * I * 2 + frac * (3 * d * I + 3 * d * I // 32)
        distinct = E * (1 - (1 - k / E) ** T)
        bytes_layer = distinct * per_expert + 3 * d * S * 2 + E * d * 2
        line = {
            "metric": METRIC, "value": world * T * L / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) tokens, seeded random-init layers)",
            "config": {"workload": f"decode: {T} tokens x {L}-layer MoE stack per step (CUDA graph)",
                       "layers": L, "tokens_per_step": T, "d_model": d, "num_experts": E, "expert_inter_dim": I,
                       "top_k": k, "shared_inter_dim": S,
                       "expert_precision": f"MXFP8 for a seeded {frac:.0%} of each layer's experts, BF16 rest",
                       "l2": "each layer's weights (~122 MB) are read once per step; 16 layers exceed L2",
                       "parallelism": f"dp{world} replicas"},
            "per_token_count": {str(tt): {"ms_per_step": v[0], "tokens_per_s_per_layer": world * tt * L / (v[0] / 1e3),
                                          "e2e_ms_per_step": v[1]} for tt, v in per_t.items()},
            "e2e": {"value": world * T * L / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": T * d * 2, "d2h_bytes_per_step": T * d * 2},
            "gpu_launches": K * L * 15,
            "roofline": {"bound": "hbm", "kernel": "whole stack (weight bytes of the routed experts)",
                         "achieved": bytes_layer * L / (ms / 1e3) / 1e9, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "traffic": None, "peak_source": pk["source"]},
        }
        line["roofline"]["frac"] = line["roofline"]["achieved"] / line["roofline"]["peak"]
        if clocks is not None:
            line["clocks"] = clocks
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_train(args) -> None:
    """One training step of the layer per timed step: forward (native kernels),
    then backward (spx_layer_backward for the routed experts -- their weight
    gradients included -- and the router scores; library GEMMs for the
    router's weight and input gradients and the shared SwiGLU).  value =
    tokens / step time; data-parallel replicas for N > 1 (no gradient
    all-reduce: the layer's own work only)."""

    world, rank, local = init_dist()
    import torch.distributed as dist

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    spec = CONFIGS[args.config]
    batch, seq = spec["batch"], spec["seq"]
    tokens = batch * seq
    mixer, _ = build_mixer(spec, device)
    mixer.train()
    config = mixer.config
    d = config.d_model
    gen = torch.Generator().manual_seed(1 + rank)
    x_host = torch.randn(batch, seq, d, generator=gen).to(torch.bfloat16).pin_memory()
    du_host = (0.05 * torch.randn(batch, seq, d, generator=gen)).to(torch.bfloat16).pin_memory()
    x_bufs = [x_host.to(device), x_host.roll(1, dims=0).to(device)]
    du = du_host.to(device)
    one = torch.ones((), dtype=torch.bfloat16, device=device)

    def step(x):
        mixer.zero_grad(set_to_none=True)
        xg = x.detach().requires_grad_(True)
        out = mixer(xg)
        torch.autograd.backward([out.update, out.auxiliary_loss], [du, one])
        return xg.grad

    for i in range(args.warmup):
        step(x_bufs[i % 2])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    K = args.steps
    sampler = ClockSampler(local)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(K):
        step(x_bufs[i % 2])
    t1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = t0.elapsed_time(t1) / K
    # forward alone, same inputs, for the split
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    with torch.no_grad():
        f0.record()
        for i in range(K):
            mixer(x_bufs[i % 2])
        f1.record()
    torch.cuda.synchronize()
    fwd_ms = f0.elapsed_time(f1) / K
    # e2e: pinned H2D of the step's tokens and upstream gradient, the step, D2H of the input gradient
    gx_host = torch.empty(batch, seq, d, dtype=torch.bfloat16).pin_memory()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(K):
        x_bufs[0].copy_(x_host, non_blocking=True)
        du.copy_(du_host, non_blocking=True)
        gx = step(x_bufs[0])
        gx_host.copy_(gx, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([ms, fwd_ms, e0.elapsed_time(e1) / K], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, fwd_ms, e2e_ms = (float(v) for v in t)
    if rank == 0:
        pk = peaks()
        fl = layer_flops(spec["cfg"], tokens)
        step_flops = 3.0 * sum(fl.values())  # forward + backward (input and weight gradients)
        line = {
            "metric": METRIC + " (training step: forward + backward)", "value": world * tokens / (ms / 1e3),
            "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) hidden states and upstream gradients, seeded random-init weights)",
            "config": {**workload_config(args.config, world),
                       "workload": "m100_train: SPALMER micro-expert layer forward + backward"},
            "forward_ms": fwd_ms, "backward_ms": ms - fwd_ms,
            "e2e": {"value": world * tokens / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": 2 * tokens * d * 2, "d2h_bytes_per_step": tokens * d * 2},
            "gpu_launches": K * (14 + 11),
            "roofline": {"bound": "tensor", "kernel": "whole step (3x the forward's GEMM FLOPs)",
                         "achieved": step_flops / (ms / 1e3) / 1e12, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                         "traffic": None, "peak_source": pk["source"]},
            "clocks": clocks,
        }
        line["roofline"]["frac"] = line["roofline"]["achieved"] / line["roofline"]["peak"]
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = (cpu_baseline(args, mixer, None) if reference_package() is not None
                                    else cpu_train_baseline(spec, mixer))
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def cpu_train_baseline(spec: dict, mixer) -> dict:
    """The reference's training step restated in PyTorch autograd on the host
    cores (oracle/mixer_autograd.py), on a bounded token sample."""

    from oracle import mixer_autograd as MA

    torch.set_num_threads(os.cpu_count() or 1)
    sample = spec["cpu_sample"]
    d = spec["cfg"]["d_model"]
    sd = {n: p.detach().cpu() for n, p in mixer.named_parameters()}
    params = {n: sd[n] for n in MA.PARAM_NAMES if n in sd}
    gen = torch.Generator().manual_seed(7)
    x = torch.randn(sample, d, generator=gen).to(torch.bfloat16)
    du = (0.05 * torch.randn(sample, d, generator=gen)).to(torch.bfloat16)
    times = []
    for _ in range(3):
        t0 = time.perf_counter()
        MA.gradients(params, x, spec["cfg"]["active_experts"], du, 1.0)
        times.append(time.perf_counter() - t0)
    sec = sorted(times)[1]
    return {"value": sample / sec, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{sample} tokens, forward + backward through PyTorch CPU autograd, median of 3"}


def run_paged(args) -> None:
    """The layer with its expert bank offloaded to pinned host memory behind a
    device cache (spalmer_b200.offload); each step pages the selected experts.
    Replicas only for N > 1 (no collective)."""

    world, rank, local = init_dist()
    import torch.distributed as dist

    from spalmer_b200.offload import enable_expert_offload

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    spec = CONFIGS[args.config]
    batch, seq = spec["batch"], spec["seq"]
    tokens = batch * seq
    mixer, _ = build_mixer(spec, device)
    capacity = spec["paged"]["cache_size"]
    enable_expert_offload(mixer, device, cache_size=capacity)
    config = mixer.config
    bank = mixer.experts
    cache = bank._offload
    # Four distinct seeded batches, cycled, so consecutive steps select different experts.
    gen = torch.Generator().manual_seed(1 + rank)
    x_cpu = [torch.randn(batch, seq, config.d_model, generator=gen).to(torch.bfloat16) for _ in range(4)]
    x_host = [x.pin_memory() for x in x_cpu]
    x_dev = [x.to(device) for x in x_host]
    K, W = args.steps, args.warmup

    def barrier():
        if world > 1:
            dist.barrier()

    with torch.inference_mode():
        for i in range(W):
            mixer(x_dev[i % 4])
        torch.cuda.synchronize()
        barrier()
        c0, b0, ch = bank.expert_offload_counters, cache.physical_bytes_copied, 0
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        sampler = ClockSampler(local)
        time.sleep(0.3)
        t0.record()
        for i in range(K):
            mixer(x_dev[i % 4])
            ch += cache.last_chunks
        t1.record()
        torch.cuda.synchronize()
        clocks = sampler.stop()
        barrier()
        c1, b1 = bank.expert_offload_counters, cache.physical_bytes_copied
        total_ms = t0.elapsed_time(t1)
        status = mixer.device_status()
        # e2e: hidden states in from pinned host memory, update and aux loss out, every step
        out_host = torch.empty(batch, seq, config.d_model, dtype=torch.bfloat16).pin_memory()
        aux_host = torch.empty((), dtype=torch.bfloat16).pin_memory()
        x_in = torch.empty_like(x_dev[0])
        for i in range(W):
            x_in.copy_(x_host[i % 4], non_blocking=True)
            o = mixer(x_in)
            out_host.copy_(o.update, non_blocking=True)
            aux_host.copy_(o.auxiliary_loss, non_blocking=True)
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(K):
            x_in.copy_(x_host[i % 4], non_blocking=True)
            o = mixer(x_in)
            out_host.copy_(o.update, non_blocking=True)
            aux_host.copy_(o.auxiliary_loss, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        barrier()
        e2e_ms = e0.elapsed_time(e1)
    t = torch.tensor([total_ms, e2e_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, e2e_ms = float(t[0]), float(t[1])
    ms_per_step = total_ms / K
    if rank == 0:
        rows = (c1[1] - c0[1]) / K
        phys = (b1 - b0) / K
        line = {
            "metric": METRIC, "value": world * tokens / (ms_per_step / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (four seeded N(0,1) hidden-state batches cycled, seeded random-init weights)",
            "config": {**workload_config(args.config, world),
                       "expert_offload": f"paged: expert bank in pinned host memory, device cache of {capacity} "
                                         f"of {config.num_experts} experts, LRU spare slots",
                       "l2": "expert weights re-staged from the host every step; hidden states cycled over 4 batches",
                       "parallelism": f"replicas{world}" if world > 1 else "dp1"},
            "e2e": {"value": world * tokens / (e2e_ms / K / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": tokens * config.d_model * 2 + int(phys),
                    "d2h_bytes_per_step": tokens * config.d_model * 2 + 2 + 4 * config.num_experts},
            "gpu_launches": int(K * 9 + 3 * ch),
            "roofline": None,
            "paging": {"cache_size": capacity, "transferred_experts_per_step": rows,
                       "stage_operations_per_step": (c1[0] - c0[0]) / K,
                       "h2d_packed_bytes_per_step": phys,
                       "h2d_gbs_over_step": phys / (ms_per_step / 1e3) / 1e9,
                       "chunks_per_step": ch / K},
            "device_status": status,
        }
        if clocks is not None:
            line["clocks"] = clocks
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="m100", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tokens", type=int, default=None,
                    help="decode configs: run this one token count per step instead of the configuration's list")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    # No cyclic-garbage collection pauses inside the host-driven timed loops
    # (the process is short-lived; reference counting still frees tensors).
    gc.collect()
    gc.disable()
    if args.impl == "reference":
        run_reference_arm(args)
    elif CONFIGS[args.config].get("expert_parallel"):
        run_ep(args)
    elif CONFIGS[args.config].get("decode_layers"):
        run_decode(args)
    elif CONFIGS[args.config].get("train"):
        run_train(args)
    elif CONFIGS[args.config].get("paged"):
        run_paged(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
