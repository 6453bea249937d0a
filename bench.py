#!/usr/bin/env python
"""Training-step benchmark of the tinygs hot path on B200.

Workload (N = 1): BASELINE config 2 -- 3M Gaussians, SH degree 3, fp16
rasterizer with fp32 parameters/gradients/Adam, 1920x1080, cameras from a
seeded 60-view orbit of radius 4, seeded U[0,1] targets (synthetic stand-ins:
no dataset is named and the reference's scenes are absent).  One step =
forward render -> 0.8 L1 + 0.2 (1-SSIM) (x grad_scaler 10) -> backward ->
Adam (max_grad_1 0.3), i.e. Orchestrator::train_step with
record_trajectory off and the data loader replaced by resident targets.

N > 1 (torchrun, one process per GPU, NCCL): every rank renders its own orbit
view of the same replicated model each step, the gradient arena (236 B per
Gaussian) is summed with one NCCL all-reduce and every rank applies the same
Adam step with gradient scale 1/(grad_scaler*N) -- the reference's
accumulate_grad_steps=N semantics (orchestrator.cu:343-403).  Weak scaling:
`value` counts view-steps of all ranks per second.

Reported: `value` (device-resident inputs, CUDA events, max over ranks),
`e2e` (target uploaded from pinned host memory and the loss scalar read back
every step, through the public API), per-stage times, the roofline of the
fused Adam kernel (the HBM-bound kernel whose time is measured live), clocks
sampled during the timed region, and a CPU baseline (the oracle restatement,
timed on a bounded sample on the host cores).

`--impl reference` times the reference's own training step on the same
workload and GPU -- its CUDA kernels built unchanged from its sources into
oracle/_ref (rasterizer forward/backward, L1, fused SSIM, SimpleAdam) -- and
prints it in the same format (the CPU restatement where that library is not
built).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "train iters/s (fwd+bwd+SSIM+Adam) @3M Gaussians 1080p; render Mpix/s"
GRAD_SCALER = 10.0
ADAM_BYTES_PER_GAUSSIAN = 7 * 59 * 4  # read theta, g, m, v; write theta, m, v
# measured DRAM bytes per Gaussian of the fused backward + Adam (ncu, 1M)
TRAFFIC_BWD_ADAM_PER_GAUSSIAN = 1476.7


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="cfg2")
    ap.add_argument("--n", type=int, default=0, help="override the Gaussian count (profiling small cases)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=25.0, help="seconds of CPU work for the baseline sample")
    ap.add_argument("--dp", choices=["auto", "owner", "inbox", "multicast", "peer", "nccl"], default="auto",
                    help="several GPUs: each rank preprocesses and back-propagates its own slice of the Gaussians "
                         "for every rank's view, with the records and screen-space gradients exchanged through "
                         "the ranks' arenas over NVLink, and Adam on its slice (owner); gradients stored into "
                         "their owners' inboxes by the backward, then "
                         "accumulation + Adam + parameter broadcast in one kernel (inbox); accumulation + Adam in "
                         "one kernel through NVLink SHARP (multicast) or over peer memory (peer); or an NCCL "
                         "all-reduce followed by Adam on every rank (nccl, the baseline); auto = owner")
    args = ap.parse_args()
    args.steps_given = args.steps is not None
    if args.steps is None:
        args.steps = 20
    return args


# ----------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(f"/tmp/tgs_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.gpu)], stdout=self.fh,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        # nvidia-smi takes a moment to start: wait (at most 10 s) for its
        # first sample, so that the sampling covers the timed regions
        t0 = time.time()
        while time.time() - t0 < 10.0 and self.proc.poll() is None:
            self.fh.flush()
            if self.path.stat().st_size > 0:
                break
            time.sleep(0.02)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        self.path.unlink(missing_ok=True)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "power_w_max": max(power), "samples": len(sm)}


# ------------------------------------------------------------ CPU oracle

def scene_config(name: str, n: int = 0):
    import dataclasses

    from tinygs_b200 import scenes

    cfg = scenes.CONFIGS[name]
    return dataclasses.replace(cfg, n=n) if n else cfg


def cpu_oracle_step_time(cfg_name: str, budget_s: float, fp32_math: bool = True, n: int = 0) -> dict:
    """Time one oracle training step of the workload on the host cores.
    Per-Gaussian and per-pixel stages run in full; the two blend stages run on
    every k-th tile (k chosen from a probe so the sample fits the budget) and
    their time is scaled by k."""
    import numpy as np

    from oracle import pyoracle as O
    from tinygs_b200 import scenes

    cfg = scene_config(cfg_name, n)
    params = scenes.gaussian_params(cfg.n, cfg.sh_degree, cfg.means, cfg.seed)
    cam = scenes.cameras(cfg)[0]
    W, H = cfg.width, cfg.height
    target = scenes.target_image(W, H, cfg.seed + 100).reshape(-1)
    fp16 = False if fp32_math else cfg.dtype == "float16"
    lib = O.load()
    t = {}
    t0 = time.perf_counter()
    prims = O.preprocess(params, cfg.sh_degree, cam, fp16)
    t["preprocess"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    bins = O.binning(prims, cam, fp16)
    t["binning"] = time.perf_counter() - t0
    # probe the blend cost on 1/256 of the tiles, then pick the stride
    lib.orc_set_tile_stride(256)
    t0 = time.perf_counter()
    O.blend_forward(prims, bins, cam, fp16)
    probe = max(time.perf_counter() - t0, 1e-4)
    remaining = max(budget_s - sum(t.values()), 2.0)
    est_full_fwd = probe * 256
    stride = int(min(256, max(1, (3.0 * est_full_fwd) / remaining)))
    lib.orc_set_tile_stride(stride)
    t0 = time.perf_counter()
    fwd = O.blend_forward(prims, bins, cam, fp16)
    t["blend_forward"] = (time.perf_counter() - t0) * stride
    lib.orc_set_tile_stride(1)
    dt = np.float16 if fp16 else np.float32
    img = fwd["image"]
    loss_map = np.zeros(img.shape, dt)
    grad_img = np.zeros(img.shape, dt)
    t0 = time.perf_counter()
    O.l1(img, target.astype(dt), loss_map, grad_img, W, H, 0.8 * GRAD_SCALER)
    O.ssim(img, target.astype(dt), loss_map, grad_img, W, H, 0.2 * GRAD_SCALER)
    t["loss"] = time.perf_counter() - t0
    lib.orc_set_tile_stride(stride)
    t0 = time.perf_counter()
    screen = O.blend_backward(prims, bins, fwd, grad_img, cam, fp16)
    t["blend_backward"] = (time.perf_counter() - t0) * stride
    lib.orc_set_tile_stride(1)
    t0 = time.perf_counter()
    grads = O.preprocess_backward(params, cfg.sh_degree, cam, prims["n_touched"], screen)
    t["preprocess_backward"] = time.perf_counter() - t0
    from types import SimpleNamespace
    acfg = SimpleNamespace(beta1=0.9, beta2=0.999, epsilon=1e-8, max_grad_1=0.3, means_lr=1.6e-4, shs_lr=2.5e-3,
                           opacities_lr=5e-2, scales_lr=5e-3, rotations_lr=1e-3, opacities_l1=0.0, scales_l1=0.0,
                           scene_scale=1.0, global_lr=1.0, decay_reduction_mean=True)
    m = {k: np.zeros_like(v) for k, v in params.items()}
    v = {k: np.zeros_like(x) for k, x in params.items()}
    t0 = time.perf_counter()
    O.adam_step(params, grads, m, v, acfg, 1, 1.0 / GRAD_SCALER)
    t["adam"] = time.perf_counter() - t0
    total = sum(t.values())
    return {"seconds_per_step": total, "stages_s": {k: round(x, 4) for k, x in t.items()}, "tile_stride": stride,
            "threads": O.threads(), "fp16_emulated": fp16, "n_instances": bins["n_instances"]}


def densify_sample(n: int, seed: int = 3):
    """Seeded cfg3-sized state for one densification refine: parameters and
    moments of `n` Gaussians and their accumulated view-space gradient
    statistics, about a third of them above the growth threshold."""
    import numpy as np

    from tinygs_b200 import scenes

    c = scenes.CONFIGS["cfg3"]
    params = scenes.gaussian_params(n, c.sh_degree, c.means, seed)
    rng = np.random.default_rng(seed + 1)
    # a tenth of the Gaussians transparent enough to be pruned
    params["opacities"][rng.random(n) < 0.1] = -7.0
    thr = 2e-4 * GRAD_SCALER
    counter = rng.integers(1, 20, n).astype(np.float32)
    dens = np.zeros((n, 4), np.float32)
    dens[:, 0] = counter
    dens[:, 1] = counter * thr * rng.choice([0.3, 3.0], size=n, p=[0.67, 0.33]).astype(np.float32)
    dens[:, 2] = dens[:, 1]
    dens[:, 3] = rng.uniform(1.0, 60.0, n).astype(np.float32)
    return params, dens


def densify_bench(n: int, capacity: int, cpu: bool) -> dict:
    """One DefaultStrategy refine (grow + prune + compaction of parameters,
    gradients and both moments) at strategy step 600, timed with CUDA events
    around tgs_densify_step; the oracle's refine on the same state beside it."""
    import ctypes
    import time

    import numpy as np
    import torch

    from tinygs_b200 import _abi
    from tinygs_b200 import runtime as rt

    params, dens = densify_sample(n)
    lib = _abi.load_library()
    cfgp = rt.DensifyParams(reset_every=3000)
    sets = [rt.GaussianSet.from_numpy(params, 3, capacity=capacity) for _ in range(1)]
    P = sets[0]
    G, M, V = P.zeros_like(), P.zeros_like(), P.zeros_like()
    d = torch.zeros((capacity, 4), dtype=torch.float32, device="cuda")
    d[:n] = torch.from_numpy(dens).cuda()
    h = ctypes.c_void_p()
    _abi.check(lib.tgs_densify_create(capacity, ctypes.byref(h)), "tgs_densify_create")
    rng = _abi.TgsPcg32()
    lib.tgs_pcg32_seed(ctypes.byref(rng), 42, 1)
    c = cfgp.abi(1.0, GRAD_SCALER, 1280, 720)
    nn = ctypes.c_int64(n)
    p, g, m, v = P.abi(), G.abi(), M.abi(), V.abi()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    _abi.check(lib.tgs_densify_step(h, ctypes.byref(p), ctypes.byref(g), ctypes.byref(m), ctypes.byref(v),
                                    d.data_ptr(), ctypes.byref(c), 600, ctypes.byref(rng), ctypes.byref(nn), None),
               "tgs_densify_step")
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    lib.tgs_densify_destroy(h)
    n_out = nn.value
    grown = int(((dens[:, 1] / np.maximum(dens[:, 0], 1.0)) > 2e-4 * GRAD_SCALER).sum())
    # bytes a refine has to move: statistics and scales read for the grow
    # test, grown rows written (parameters; zeros for gradients and moments),
    # the prune test's reads, and the kept rows of the four sets gathered and
    # copied back
    alg = n * (16 + 12) + grown * 236 * 5 + (n + grown) * (4 + 12 + 16 + 16)
    if n_out < n + grown:  # the compaction runs only when something is pruned
        alg += n_out * 4 * 236 * 3
    out = {"refine_ms": ms, "gaussians_in": n, "grown": grown, "gaussians_out": n_out,
           "algorithmic_bytes": alg, "achieved_gbs": alg / (ms * 1e-3) / 1e9,
           "note": "one refine at strategy step 600 (grow, split/clone, prune, stable compaction of params, "
                   "grads and both moments), cfg3 start size, seeded statistics; host syncs included"}
    if cpu:
        from oracle import pyoracle as O

        cap = capacity
        Pa, Ga = O.alloc_set(cap, params), O.alloc_set(cap)
        Ma, Va = O.alloc_set(cap), O.alloc_set(cap)
        da = np.zeros((cap, 4), np.float32)
        da[:n] = dens
        oc = O.densify_config(reset_every=3000)
        t0 = time.perf_counter()
        on = O.densify_step(n, Pa, Ga, Ma, Va, da, oc, 600, O.pcg32(42, 1))
        cpu_s = time.perf_counter() - t0
        out["cpu_refine_ms"] = cpu_s * 1e3
        out["cpu_gaussians_out"] = on
    return out


def workload(cfg, n_views: int, world: int) -> dict:
    """The `config` object of both arms' lines."""
    return {"workload": f"{cfg.name}: {cfg.n} Gaussians SH{cfg.sh_degree}, {cfg.dtype} rasterizer, "
                        f"{cfg.width}x{cfg.height}, {n_views}-view orbit r={cfg.cam_distance}",
            "gaussians": cfg.n, "width": cfg.width, "height": cfg.height, "sh_degree": cfg.sh_degree,
            "views_per_gpu_step": 1, "parallelism": f"dp{world}",
            "l2": "inputs larger than L2 (parameters+gradients+moments 2.8 GB per step)"}


def run_reference(args):
    """--impl reference: the reference's own training step on the GPU.

    oracle/_ref/libtgs_ref.so holds the reference's CUDA kernels built
    unchanged from its sources (fastgs_ours_fp16 / fastgs_ours rasterizers,
    L1Loss, FusedSSIMLoss, SimpleAdam).  One step is what
    Orchestrator::train_step (orchestrator.cu:335-439) runs for this
    workload: zero the gradient container, the loss map and the gradient
    image; rasterizer forward; L1 (weight 0.8) and fused SSIM (0.2) scaled
    by grad_scaler 10; rasterizer backward; SimpleAdam::step(1/10) with
    max_grad_1 0.3 -- with the reference's own host synchronisations inside
    its forward and backward.  The reference has no multi-GPU code: under
    torchrun rank 0 alone runs it on its GPU and the other ranks exit.
    Where the library is absent (or no GPU is present), the CPU restatement
    (the oracle) is timed instead."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    from oracle import refpy

    if not refpy.available() or not torch.cuda.is_available():
        return run_reference_cpu(args)
    import numpy as np

    from tinygs_b200 import runtime as rt
    from tinygs_b200 import scenes

    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    cfg = scene_config(args.config, args.n)
    W, H = cfg.width, cfg.height
    fp16 = cfg.dtype == "float16"
    dt = torch.float16 if fp16 else torch.float32
    params = scenes.gaussian_params(cfg.n, cfg.sh_degree, cfg.means, cfg.seed)
    adam = refpy.RefAdam(cfg.n, cfg.sh_degree, {"max_grad_1": 0.3})
    for name in refpy.RefAdam.SEGMENTS:
        adam.param(name).copy_(torch.from_numpy(np.ascontiguousarray(params[name], np.float32).reshape(-1)))
    del params

    class Arrays:  # the containers as the harness's pointer struct source
        def __init__(self, s):
            self.full = {k: _Ptr(getattr(s, k)) for k in refpy.RefAdam.SEGMENTS}
            self.n, self.sh_degree = cfg.n, cfg.sh_degree

    class _Ptr:
        def __init__(self, p):
            self.p = p

        def data_ptr(self):
            return self.p

    g, gr = Arrays(adam.params), Arrays(adam.grads)
    grad_views = [adam.grad(k) for k in refpy.RefAdam.SEGMENTS]
    cams = scenes.cameras(cfg)
    n_targets = 4
    targets = [torch.from_numpy(scenes.target_image(W, H, cfg.seed + 100 + k).reshape(-1)).to(dt).cuda()
               for k in range(n_targets)]
    numel = rt.image_numel(W, H)
    image = torch.zeros(numel, dtype=dt, device="cuda")
    grad_image = torch.zeros_like(image)
    loss_map = torch.zeros_like(image)
    ref = refpy.RefRasterizer()
    stream = torch.cuda.current_stream()
    counts = [0, 0, 0]

    def step(k, ev=None):
        cam = cams[k % len(cams)]
        for v in grad_views:
            v.zero_()
        loss_map.zero_()
        grad_image.zero_()
        if ev is not None:
            ev[0].record(stream)
        counts[:] = ref.forward(g, cam, image, fp16)
        if ev is not None:
            ev[1].record(stream)
        tgt = targets[k % n_targets]
        refpy.l1(fp16, W, H, image, tgt, loss_map, grad_image, 0.8 * GRAD_SCALER)
        ref.ssim(fp16, W, H, image, tgt, loss_map, grad_image, 0.2 * GRAD_SCALER)
        if ev is not None:
            ev[2].record(stream)
        ref.backward(g, cam, image, grad_image, gr, fp16)
        if ev is not None:
            ev[3].record(stream)
        adam.step(1.0 / GRAD_SCALER)
        if ev is not None:
            ev[4].record(stream)

    sampler = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")))
    sampler.start()
    for k in range(args.warmup):
        step(k)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for k in range(args.steps):
        step(args.warmup + k)
    e1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms_step = e0.elapsed_time(e1) / args.steps
    rows = []
    for k in range(max(3, min(args.steps, 5))):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        step(args.warmup + args.steps + k, ev)
        torch.cuda.synchronize()
        rows.append({"forward": ev[0].elapsed_time(ev[1]), "loss": ev[1].elapsed_time(ev[2]),
                     "backward": ev[2].elapsed_time(ev[3]), "adam": ev[3].elapsed_time(ev[4])})
    stages = {nm: round(statistics.median(r[nm] for r in rows), 4) for nm in ("forward", "loss", "backward", "adam")}
    if not torch.isfinite(adam.param("means")).all():
        stages["non_finite_parameters"] = True
    value = 1e3 / ms_step
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "iters/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "f16 raster / f32 params+grads+Adam" if fp16 else "f32", "data": "synthetic",
            "config": workload(cfg, len(cams), 1),
            "cpu_baseline": {"value": value, "unit": "iters/s", "cores": 1, "kind": "reference",
                             "sample": (f"{args.steps} full training steps of the reference's own CUDA kernels "
                                        f"(oracle/_ref, built unchanged from its sources) on one B200, driven by "
                                        f"one host thread")},
            "e2e": {"value": value, "unit": "iters/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "stages_ms": stages,
            "counts": {"visible": counts[0], "instances": counts[1], "buckets": counts[2]},
            "clocks": clocks}
    print(json.dumps(line), flush=True)
    ref.close()
    adam.close()


def run_reference_cpu(args):
    """The CPU restatement of the reference's algorithm (the oracle), timed
    on the host cores: the reference arm where oracle/_ref is not built."""
    from tinygs_b200 import scenes

    cfg = scene_config(args.config, args.n)
    steps_run, times = 0, []
    budget = 150.0
    start = time.perf_counter()
    for k in range(max(1, args.steps)):
        r = cpu_oracle_step_time(args.config, args.cpu_budget, n=args.n)
        times.append(r["seconds_per_step"])
        steps_run += 1
        if time.perf_counter() - start > budget:
            break
    sec = statistics.median(times)
    value = 1.0 / sec
    cores = r["threads"]
    sample = (f"one oracle training step of {args.config} per step ({cfg.n} Gaussians, {cfg.width}x{cfg.height}, "
              f"fp32 arithmetic); blend stages on every {r['tile_stride']}th tile, time scaled by the stride; "
              f"{steps_run} of {args.steps} steps run (budget)")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "iters/s", "n_gpus": 0,
            "steps": steps_run, "warmup": 0, "ms_per_step": sec * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload(cfg, len(scenes.cameras(cfg)), 1),
            "cpu_baseline": {"value": value, "unit": "iters/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "iters/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "stages_s": r["stages_s"]}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------- ours

def kernels_per_step(width: int, height: int, world: int, owner: bool = False) -> int:
    """Launches of this library's kernels in one training step (what
    launch_preprocess / launch_binning / launch_blend_* / the loss and the
    backward enqueue).  owner: the owner split's preprocess covers every
    view in one launch and its per-Gaussian backward + Adam is one launch."""
    grid_w, grid_h = (width + 15) // 16, (height + 15) // 16
    n_super = ((grid_w + 7) // 8) * ((grid_h + 3) // 4)
    entry_passes = max(1, ((max(1, n_super - 1)).bit_length() + 7) // 8)
    forward = (1  # preprocess
               + 2  # candidate compaction: block-sum scan, compaction
               + 4 * 3  # depth sort: 4 passes of histogram, scan, scatter
               + 3  # per-block entry counts, their scan, entry creation
               + 3 * entry_passes  # entry sort by super-tile
               + (1 if entry_passes > 1 else 0) + 1  # super-tile ranges (multi-pass sort only), chunk table
               + 4  # tile tests, chunk prefix, tile offsets, emission
               + 1)  # blend forward
    # loss forward + backward; blend backward; per-Gaussian backward fused
    # with Adam (one GPU) or routed backward + accumulation/Adam kernel
    if owner:
        return forward + 2 + 1 + 1
    return forward + 2 + 1 + (1 if world == 1 else 2)


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from tinygs_b200 import runtime as rt
    from tinygs_b200 import scenes
    from tinygs_b200 import dp as dpm
    from tinygs_b200.dp import DataParallel

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dp = DataParallel.from_env()
    cfg = scene_config(args.config, args.n)
    W, H = cfg.width, cfg.height
    fp16 = cfg.dtype == "float16"
    dt = torch.float16 if fp16 else torch.float32
    params = scenes.gaussian_params(cfg.n, cfg.sh_degree, cfg.means, cfg.seed)
    peer = world > 1 and args.dp != "nccl"
    dp_impl = args.dp if world > 1 else "none"
    opt = None
    owner = None
    if peer and args.dp in ("auto", "owner"):
        # every rank keeps the whole parameter arena but reads and updates only
        # its own slice; the split object is made once the rasterizer exists
        g = rt.GaussianSet.from_numpy(params, cfg.sh_degree)
        grads = None
        opt = "owner"
        dp_impl = "owner"
    if peer and opt is None and args.dp == "inbox":
        # parameters the other ranks map (CUDA IPC) and a gradient inbox per
        # rank: the backward stores each Gaussian's gradients into the inbox
        # of the rank that owns its slice (no local gradient arena)
        g = dpm.shared_gaussian_set(cfg.n, cfg.sh_degree)
        g.copy_from_numpy(params)
        grads = None
        opt = dpm.InboxAdam(dp, g, rt.AdamParams(max_grad_1=0.3))
        dp_impl = "inbox"
    if peer and opt is None and args.dp == "multicast":
        # arenas bound to a multicast object (NVLink SHARP)
        g = dpm.symmetric_gaussian_set(dp, cfg.n, cfg.sh_degree)
        g.copy_from_numpy(params)
        grads = dpm.symmetric_gaussian_set(dp, cfg.n, cfg.sh_degree)
        opt = dpm.MulticastAdam(dp, g, grads, rt.AdamParams(max_grad_1=0.3))
        dp_impl = "multicast"
    if peer and opt is None:
        # parameters and gradient arenas the other ranks map (CUDA IPC)
        g = dpm.shared_gaussian_set(cfg.n, cfg.sh_degree)
        g.copy_from_numpy(params)
        grads = dpm.shared_gaussian_set(cfg.n, cfg.sh_degree)
        opt = dpm.PeerAdam(dp, g, grads, rt.AdamParams(max_grad_1=0.3))
        dp_impl = "peer"
    if not peer:
        g = rt.GaussianSet.from_numpy(params, cfg.sh_degree)
        grads = g.zeros_like()
        opt = rt.SimpleAdam(g, grads, rt.AdamParams(max_grad_1=0.3))
    del params
    cams = scenes.cameras(cfg)
    n_targets = 4
    # targets are 8-bit images in the tiled layout, as the reference's
    # dataset holds them (png_folder.cpp); the device copies are converted by
    # the data path's kernel (tgs_image_from_u8), as the loader does
    dt_code = rt._abi.TGS_FLOAT16 if fp16 else rt._abi.TGS_FLOAT32
    host_targets = [torch.from_numpy(np.rint(scenes.target_image(W, H, cfg.seed + 100 + k).reshape(-1) * 255.0)
                                     .astype(np.uint8)).pin_memory() for k in range(n_targets)]
    numel = rt.image_numel(W, H)
    lib = rt.load_library()

    def to_target(raw, out, st):
        rt.check(lib.tgs_image_from_u8(raw.data_ptr(), rt._abi.TGS_IMAGE_TILED_CHW, 3, W, H, out.data_ptr(), dt_code,
                                       st.cuda_stream), "tgs_image_from_u8")

    dev_targets = []
    for t in host_targets:
        dev_targets.append(torch.empty(numel, dtype=dt, device="cuda"))
        to_target(t.cuda(), dev_targets[-1], torch.cuda.current_stream())
    # end-to-end runs upload each step's 8-bit target from pinned host memory
    # on a copy stream, one step ahead, and convert it there into two
    # alternating device buffers
    copy_stream = torch.cuda.Stream()
    up_raw = [torch.empty_like(host_targets[0], device="cuda") for _ in range(2)]
    up_bufs = [torch.empty_like(dev_targets[0]) for _ in range(2)]
    up_done = [torch.cuda.Event() for _ in range(2)]
    buf_free = [torch.cuda.Event() for _ in range(2)]
    image = torch.zeros(numel, dtype=dt, device="cuda")
    grad_image = torch.zeros_like(image)
    loss_map = torch.zeros_like(image)
    loss_sum = torch.zeros(1, device="cuda")
    loss_host = torch.zeros(2, dtype=torch.float32).pin_memory()
    loss = rt.FusedLoss(W, H)
    loss.set_accumulate(False)  # writes the whole loss map and gradient image: no per-step zeroing
    stream = torch.cuda.current_stream()

    def make_raster(cap_inst):
        r = rt.FastGSB200Rasterizer(cfg.n, W, H, cap_inst)
        r.set_gaussians(g)
        return r

    # size the instance capacity from the views this rank will render
    rast = make_raster(24 * cfg.n)
    ctx = rt.RasterizeContext(stream=stream, grad_scaler=GRAD_SCALER, fwd_output_image=image,
                              grad_output_image=grad_image, gaussians_grad=grads, accumulate=False)
    max_inst = 0
    for v in range(0, len(cams), max(1, len(cams) // 8)):
        ctx.fwd_input = cams[v]
        rast.forward(ctx)
        c = rast.counts()
        max_inst = max(max_inst, c.n_instances)
        if c.overflow:
            raise SystemExit("instance capacity too small for the sizing pass")
    rast.close()
    rast = make_raster(int(max_inst * 1.5) + 1024)
    if dp_impl == "owner":
        owner = dpm.OwnerSplit(dp, rast, g, rt.AdamParams(max_grad_1=0.3),
                               rt._abi.TGS_FLOAT16 if fp16 else rt._abi.TGS_FLOAT32)
        opt = owner

    def views_of(step):
        # the views of all ranks at `step`, in rank order
        return [cams[(step * world + r) % len(cams)] for r in range(world)]

    def view_of(step):
        return cams[dp.view_index(step, len(cams))]

    # one GPU: backward and Adam in one pass (tgs_raster_backward_adam); with
    # several GPUs the gradients must be all-reduced between the two
    fused = world == 1

    def upload(k):
        # the buffer was last read by the loss of step k - 2
        b = k % 2
        copy_stream.wait_event(buf_free[b])
        with torch.cuda.stream(copy_stream):
            up_raw[b].copy_(host_targets[k % n_targets], non_blocking=True)
            to_target(up_raw[b], up_bufs[b], copy_stream)
            up_done[b].record(copy_stream)

    def step(k, e2e=False, ev=None, last=None):
        ctx.fwd_input = view_of(k)
        if e2e and k + 1 < last:
            upload(k + 1)  # overlaps this step's forward
        if owner is not None:
            # preprocess of this rank's slice for all views (ev[7]..ev[8]),
            # barrier, binning + blend of this rank's view
            if ev is not None:
                ev[7].record(stream)
            owner.forward(views_of(k), image, stream=stream, events=None if ev is None else ev[8:10])
        else:
            rast.forward(ctx)
        if ev is not None:
            ev[0].record(stream)
        if e2e:
            stream.wait_event(up_done[k % 2])
            tgt = up_bufs[k % 2]
        else:
            tgt = dev_targets[k % n_targets]
        loss.evaluate(image, tgt, loss_map, grad_image, W, H, grad_scaler=GRAD_SCALER, loss_sum=loss_sum,
                      stream=stream)
        if e2e:
            buf_free[k % 2].record(stream)
        if ev is not None:
            ev[1].record(stream)
        if fused:
            opt.fused_backward_step(rast, ctx, 1.0 / GRAD_SCALER)
        elif owner is not None:
            # blend backward (ev[1]..ev[5]), barrier (..ev[6]), per-Gaussian
            # backward of the slice over all views + Adam (..ev[2])
            owner.backward_adam(views_of(k), image, grad_image, dp.gradient_scale(GRAD_SCALER), stream=stream,
                                events=None if ev is None else ev[5:7])
            if ev is not None:
                ev[2].record(stream)
        elif dp_impl == "inbox":
            rast.backward_routed(ctx, *opt.route())
            if ev is not None:
                ev[2].record(stream)
            # barrier, kernel (between ev[5] and ev[6]), barrier
            opt.step(dp.gradient_scale(GRAD_SCALER), stream=stream, events=None if ev is None else ev[5:7])
            if ev is not None:
                ev[3].record(stream)
                ev[4].record(stream)
        elif peer:
            rast.backward(ctx)
            if ev is not None:
                ev[2].record(stream)
            # barrier, kernel (between ev[5] and ev[6]), barrier
            opt.step(dp.gradient_scale(GRAD_SCALER), stream=stream, events=None if ev is None else ev[5:7])
            if ev is not None:
                ev[3].record(stream)
                ev[4].record(stream)
        else:
            rast.backward(ctx)
            if ev is not None:
                ev[2].record(stream)
            dp.reduce_gradients(grads.storage)
            if ev is not None:
                ev[3].record(stream)
            opt.step(dp.gradient_scale(GRAD_SCALER), stream=stream)
            if ev is not None:
                ev[4].record(stream)
        if e2e:
            loss_host[k % 2].copy_(loss_sum[0], non_blocking=True)

    def timed(n_steps, e2e, offset):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        if e2e:
            copy_stream.wait_stream(stream)  # the first upload starts inside the timed region
            upload(offset)
        for k in range(n_steps):
            step(offset + k, e2e, last=offset + n_steps)
        e1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        return dp.max_over_ranks(e0.elapsed_time(e1), "cuda")

    # clocks are sampled (every 200 ms, as the profiling recipe does: a
    # tighter loop of driver queries competes with the e2e region's own API
    # calls) from the start of the warm-up to the end of both timed regions
    sampler = ClockSampler(local)
    sampler.start()
    for k in range(args.warmup):
        step(k)
    torch.cuda.synchronize()
    counts = rast.counts()
    if counts.overflow:
        raise SystemExit("capacity overflow during warm-up")
    ms_dev = timed(args.steps, False, args.warmup)
    ms_e2e = timed(args.steps, True, args.warmup + args.steps)
    clocks = sampler.stop()
    torch.cuda.synchronize()
    if not np.isfinite(float(loss_host[0])):
        raise SystemExit("non-finite loss")

    # per-stage times on a separate pass (not part of the headline): the
    # handle records CUDA events between its stages on the stream, the bench
    # brackets the loss (and, with several GPUs, the all-reduce and Adam)
    n_stage = max(3, min(args.steps, 10))
    rast.set_stage_timing(True)
    rows = []
    for k in range(n_stage):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(10)]
        step(args.warmup + 2 * args.steps + k, False, evs)
        torch.cuda.synchronize()
        t = rast.stage_times()
        row = {"preprocess": t[0], "binning": t[1], "blend_forward": t[2], "loss": evs[0].elapsed_time(evs[1]),
               "blend_backward": t[3]}
        if fused:
            row["gaussian_backward_adam"] = t[4]
        elif owner is not None:
            row["preprocess"] = evs[7].elapsed_time(evs[8])
            row["forward_barrier"] = evs[8].elapsed_time(evs[9])
            row["blend_backward"] = evs[1].elapsed_time(evs[5])
            row["backward_barrier"] = evs[5].elapsed_time(evs[6])
            row["gaussian_backward_adam"] = evs[6].elapsed_time(evs[2])
        elif peer:
            row["gaussian_backward"] = t[4]
            row["peer_reduce_adam"] = evs[2].elapsed_time(evs[3])
            row["peer_kernel"] = evs[5].elapsed_time(evs[6])
        else:
            row["gaussian_backward"] = t[4]
            row["allreduce"] = evs[2].elapsed_time(evs[3])
            row["adam"] = evs[3].elapsed_time(evs[4])
        rows.append(row)
    rast.set_stage_timing(False)
    stages = {nm: statistics.median(r[nm] for r in rows) for nm in rows[0]}

    # forward-only render throughput (render Mpix/s)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    r0.record(stream)
    for k in range(args.steps):
        ctx.fwd_input = view_of(k)
        rast.forward(ctx)
    r1.record(stream)
    torch.cuda.synchronize()
    render_ms = r0.elapsed_time(r1) / args.steps

    counts = rast.counts()
    # Gaussians that touch a tile (the backward reads their screen gradients)
    touched_v = int((rast.debug_array(0, torch.int32, cfg.n) > 0).sum())
    # evaluated (pixel, Gaussian) pairs of the last view: forward = the
    # per-pixel contributor counts (Gaussians walked up to the last one that
    # contributed); backward = 32 x 256 per bucket (every bucket sweeps its
    # tile's 256 pixels past its 32 Gaussians)
    plane = rt.image_numel(W, H) // 3
    ncon = rast.debug_array(4, torch.int16 if fp16 else torch.int32, plane)
    fwd_pairs = int((ncon.to(torch.int64) & (0xFFFF if fp16 else 0xFFFFFFFF)).sum())
    bwd_pairs = int(counts.n_buckets) * 32 * 256
    ms_step = ms_dev / args.steps
    value = world * 1e3 / ms_step
    e2e_ms = ms_e2e / args.steps
    if owner is not None:
        # k_views_backward_adam over this rank's slice: parameters read and
        # written, both moments read and written (6 x 236 B), and per view
        # the touched-tile count and the 48-byte screen gradients (peer
        # memory for the other ranks' views)
        nl = owner.last - owner.first
        kernel = ("k_views_backward_adam (the rank's slice back-propagated through every rank's view, summed "
                  "on chip, Adam in the same pass)")
        kernel_bytes = nl * (6 * 236 + world * (4 + 48))
        kernel_ms = stages["gaussian_backward_adam"]
    elif fused:
        # k_preprocess_backward<true>: parameters, both moments read and
        # written, the touched-tile counts, and the 48-byte screen-space
        # gradients of the visible Gaussians
        kernel = "k_preprocess_backward<true> (per-Gaussian backward fused with Adam)"
        kernel_bytes = cfg.n * (6 * 236 + 4) + touched_v * 48
        kernel_ms = stages["gaussian_backward_adam"]
        # DRAM read + write per Gaussian of this kernel from one ncu capture
        # at 1M Gaussians (profiles/k_preprocess_backward_adam_cfg2_1M.md:
        # 823.5 + 653.2 MB); traffic grows with the Gaussians processed
        kernel_traffic = TRAFFIC_BWD_ADAM_PER_GAUSSIAN * cfg.n
    elif dp_impl == "inbox":
        # k_preprocess_backward<false, true>: as below, but (N-1)/N of the
        # gradient stores cross NVLink into the owners' inboxes
        kernel = "k_preprocess_backward<false,true> (per-Gaussian backward, gradients routed to the owners' inboxes)"
        kernel_bytes = cfg.n * (2 * 236 + 4) + touched_v * 48
        kernel_ms = stages["gaussian_backward"]
    elif peer:
        # k_preprocess_backward<false>: parameters read, gradients written,
        # the touched-tile counts and screen-space gradients read
        kernel = "k_preprocess_backward<false> (per-Gaussian backward, gradients to the shared arena)"
        kernel_bytes = cfg.n * (2 * 236 + 4) + touched_v * 48
        kernel_ms = stages["gaussian_backward"]
    else:
        kernel = "k_adam (fused Adam over the 59-float arena)"
        kernel_bytes = ADAM_BYTES_PER_GAUSSIAN * cfg.n
        kernel_ms = stages["adam"]
    if not fused:
        kernel_traffic = None  # no capture of the multi-GPU kernels
    kernel_gbs = kernel_bytes / (kernel_ms * 1e-3) / 1e9
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        hbm_peak, peak_src = float(peaks["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        hbm_peak, peak_src = 6650.0, "fallback"

    dens_row = None
    if rank == 0 and world == 1 and args.config == "cfg2" and args.n == 0:
        dens_row = densify_bench(1_000_000, 3_000_000, cpu=not args.no_cpu_baseline)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r = cpu_oracle_step_time(args.config, args.cpu_budget, n=args.n)
        cpu = {"value": 1.0 / r["seconds_per_step"], "unit": "iters/s", "cores": r["threads"], "kind": "port",
               "sample": (f"one oracle step of {args.config} ({cfg.n} Gaussians, {W}x{H}, fp32 arithmetic); "
                          f"blend stages on every {r['tile_stride']}th tile, scaled by the stride"),
               "stages_s": r["stages_s"]}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "iters/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 raster / f32 params+grads+Adam" if fp16 else "f32",
            "data": "synthetic",
            "config": workload(cfg, len(cams), world),
            "e2e": {"value": world * 1e3 / e2e_ms, "unit": "iters/s",
                    "h2d_bytes_per_step": int(host_targets[0].numel() * host_targets[0].element_size()),
                    "d2h_bytes_per_step": 4,
                    "target": "8-bit tiled image uploaded and converted on the device (tgs_image_from_u8) "
                              "every step",
                    "gpu_launches": (kernels_per_step(W, H, world, owner is not None) + 1) * args.steps},
            "render_mpix_s": W * H / (render_ms * 1e-3) / 1e6,
            "blend_pairs": {"forward_pairs": fwd_pairs, "backward_pairs": bwd_pairs,
                            "forward_gpairs_per_s": fwd_pairs / (stages["blend_forward"] * 1e-3) / 1e9,
                            "backward_gpairs_per_s": bwd_pairs / (stages["blend_backward"] * 1e-3) / 1e9,
                            "unit": "evaluated (pixel, Gaussian) pairs of one view; forward = sum of the per-pixel "
                                    "contributor counts, backward = buckets x 32 x 256"},
            "stages_ms": {k: round(v, 4) for k, v in stages.items()},
            "roofline": {"bound": "hbm", "kernel": kernel, "achieved": kernel_gbs, "peak": hbm_peak,
                         "unit": "GB/s", "frac": kernel_gbs / hbm_peak, "peak_source": peak_src, "traffic": kernel_traffic,
                         "algorithmic_bytes_per_launch": kernel_bytes, "avg_launch_ms": kernel_ms},
            "counts": {"visible": counts.n_visible, "instances": counts.n_instances, "buckets": counts.n_buckets},
            "gpu_launches": kernels_per_step(W, H, world, owner is not None) * args.steps,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        if dens_row is not None:
            line["densify"] = dens_row
        if world > 1:
            line["config"]["dp_impl"] = dp_impl
        if owner is not None:
            line["owner_split"] = {
                "slice": [owner.first, owner.last],
                "preprocess_ms": stages["preprocess"], "forward_barrier_ms": stages["forward_barrier"],
                "backward_barrier_ms": stages["backward_barrier"],
                "gaussian_backward_adam_ms": stages["gaussian_backward_adam"],
                "note": "records (preprocess) stored into the view ranks' arenas and screen-space gradients "
                        "read back over NVLink; no gradient all-reduce"}
            # NVLink bytes per GPU per step, estimated from this rank's view
            # (its candidate and touched fractions stand for every view's):
            # out during the preprocess, per other view, the touched-count
            # and bounds words of every slice Gaussian (12 B) plus the depth
            # key, mean2d and primitive record of each candidate (28 B fp16,
            # 40 B fp32); in during the backward, per other view, the touched
            # counts (4 B) plus the 48-byte screen gradients of each touched
            # Gaussian.  Peak: the recipe's measured peer copy (770 GB/s per
            # direction per GPU).
            nl = owner.last - owner.first
            others = world - 1
            rec_bytes = others * nl * (12 + (28 if fp16 else 40) * counts.n_visible / cfg.n)
            grad_bytes = others * nl * (4 + 48 * touched_v / cfg.n)
            pre_ms, bwd_ms = stages["preprocess"], stages["gaussian_backward_adam"]
            line["owner_split"]["nvlink"] = {
                "records_out_bytes": rec_bytes, "records_out_gbs": rec_bytes / (pre_ms * 1e-3) / 1e9,
                "screen_grads_in_bytes": grad_bytes, "screen_grads_in_gbs": grad_bytes / (bwd_ms * 1e-3) / 1e9,
                "peak_gbs_each_way": 770.0,
                "link_floor_ms": max(rec_bytes, grad_bytes) / 770e9 * 1e3,
                "peak_source": "peer copy per direction measured on this pool (profiling recipe), not re-measured here",
                "estimate": "per-view candidate/touched fractions taken from this rank's view"}
        elif peer:
            # NVLink bytes into each GPU (and the same out of it) per step.
            # peer: its slice's gradients loaded from the other ranks plus the
            # other ranks' new parameters stored into it, 2 * 236 B * n/N *
            # (N-1) (the bytes of a ring all-reduce).  multicast: 236 B * n
            # through the switch (reduced gradients of its slice in, the other
            # slices' parameters in).  inbox: the kernel moves only the
            # parameters, 236 B * n/N * (N-1); the gradients crossed during the
            # backward.  "ms" is the kernel alone; with_barriers_ms adds the two
            # one-element all-reduces that order it and absorb the ranks' skew
            slice_bytes = 236 * cfg.n / world
            link_bytes = {"multicast": 236 * cfg.n, "inbox": slice_bytes * (world - 1)}.get(
                dp_impl, 2 * slice_bytes * (world - 1))
            ms = stages["peer_kernel"]
            kname = {"multicast": "k_dp_adam_mc (gradient sum by NVLink SHARP reducing loads + Adam + multicast "
                                  "parameter stores)",
                     "inbox": "k_dp_adam over the local inbox (gradient sum of the N slots + Adam + parameter "
                              "broadcast to the peers)"}.get(
                dp_impl, "k_dp_adam (gradient sum over peer memory + Adam + parameter broadcast)")
            line["peer_reduce_adam"] = {
                "kernel": kname, "ms": ms, "with_barriers_ms": stages["peer_reduce_adam"],
                "nvlink_bytes_each_way_per_gpu": link_bytes,
                "achieved_gbs_each_way": link_bytes / (ms * 1e-3) / 1e9,
                "peak_gbs_each_way": 770.0, "frac": link_bytes / (ms * 1e-3) / 1e9 / 770.0,
                "peak_source": "measured peer copy on this pool (profiling recipe)"}
            if dp_impl == "inbox":
                line["peer_reduce_adam"]["routed_gradient_bytes_each_way_per_gpu"] = slice_bytes * (world - 1)
        print(json.dumps(line), flush=True)
    if peer:
        opt.close()  # peer mappings closed on every rank before any owner frees its memory
        dist.barrier()
    rast.close()
    loss.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_cfg3(args):
    """BASELINE config 3, the densification-heavy run: 1M Gaussians (SH3,
    fp32, 1280x720, 60-view orbit) trained for `steps` iterations (3000 by
    default) with DefaultStrategy refining every 100 steps from step 100
    (clone/split where the mean 2D gradient norm exceeds 2e-4, prune below
    opacity 0.005, growth while below 3M -- the reference's soft cap,
    default.cu:53), no opacity reset inside the run.  The whole run is timed
    (refines and their two host synchronisations included); the line reports
    iterations per second over it, the Gaussian count after each refine and
    the refine times.  One GPU."""
    import numpy as np
    import torch

    from tinygs_b200 import runtime as rt
    from tinygs_b200 import scenes

    torch.cuda.set_device(0)
    cfg = scene_config("cfg3", args.n)
    W, H = cfg.width, cfg.height
    iters = args.steps if args.steps_given else 3000
    cap_soft = 3 * cfg.n
    capacity = int(cap_soft * 1.5)
    params = scenes.gaussian_params(cfg.n, cfg.sh_degree, cfg.means, cfg.seed)
    g = rt.GaussianSet.from_numpy(params, cfg.sh_degree, capacity=capacity)
    del params
    opt = rt.SimpleAdam(g, g.zeros_like(), rt.AdamParams(max_grad_1=0.3))
    dens = rt.Densifier(g, None, opt, rt.DensifyParams(refine_every=100, start_refine=100, end_refine=iters,
                                                       reset_every=0, duplicate_grad_threshold=2e-4,
                                                       pruning_opacity_threshold=0.005,
                                                       max_num_gaussians=cap_soft))
    cams = scenes.cameras(cfg)
    targets = [torch.from_numpy(scenes.target_image(W, H, cfg.seed + 100 + k).reshape(-1)).cuda() for k in range(4)]
    image = torch.zeros(rt.image_numel(W, H), dtype=torch.float32, device="cuda")
    grad_image, loss_map = torch.zeros_like(image), torch.zeros_like(image)
    loss = rt.FusedLoss(W, H)
    loss.set_accumulate(False)
    rast = rt.FastGSB200Rasterizer(capacity, W, H, 24 * capacity)
    rast.set_gaussians(g)
    stream = torch.cuda.current_stream()
    ctx = rt.RasterizeContext(stream=stream, grad_scaler=GRAD_SCALER, fwd_output_image=image,
                              grad_output_image=grad_image, gaussians_grad=None, accumulate=False)
    refine_ms, counts = [], []

    def step(k, timed_refines=False):
        ctx.fwd_input = cams[k % len(cams)]
        ctx.densification_info = dens.densification_info
        rast.forward(ctx)
        loss.evaluate(image, targets[k % 4], loss_map, grad_image, W, H, grad_scaler=GRAD_SCALER, stream=stream)
        opt.fused_backward_step(rast, ctx, 1.0 / GRAD_SCALER)
        refine = dens.step_count % 100 == 0 and 100 <= dens.step_count <= iters
        if refine and timed_refines:
            r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            r0.record(stream)
        n_before = g.n
        dens.step(ctx)
        if refine and timed_refines:
            r1.record(stream)
            r1.synchronize()
            refine_ms.append(r0.elapsed_time(r1))
            counts.append((dens.step_count - 1, n_before, g.n))

    sampler = ClockSampler(0)
    sampler.start()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for k in range(iters):
        step(k, timed_refines=True)
    e1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    c = rast.counts()
    if c.overflow:
        raise SystemExit("capacity overflow during the cfg3 run")
    ms = e0.elapsed_time(e1)
    # the statistic the refines test, over the steps after the last refine
    # (accumulated, not yet consumed): how many Gaussians pass the threshold
    info = dens.densification_info[: g.n].float()
    seen = info[:, 0] > 0
    mean_grad = info[seen, 1] / info[seen, 0]
    q = torch.quantile(mean_grad[: 1 << 24], torch.tensor([0.5, 0.99, 0.999], device=mean_grad.device))
    grad_stats = {"seen": int(seen.sum()), "above_threshold": int((mean_grad > 2e-4).sum()),
                  "median": float(q[0]), "p99": float(q[1]), "p999": float(q[2]), "max": float(mean_grad.max())}
    line = {"metric": "train iters/s over the densification-heavy run (cfg3)", "value": iters * 1e3 / ms,
            "unit": "iters/s", "n_gpus": 1, "steps": iters, "warmup": 0, "ms_per_step": ms / iters,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"cfg3: {cfg.n} Gaussians at start, SH{cfg.sh_degree}, fp32, {W}x{H}, "
                                   f"{len(cams)}-view orbit; refine every 100 from 100 (grad 2e-4, prune opacity "
                                   f"0.005), soft cap {cap_soft}", "gaussians_start": cfg.n,
                       "gaussians_final": g.n, "capacity": capacity, "parallelism": "dp1"},
            "refines": [{"step": s_, "n_in": a, "n_out": b, "ms": round(t, 3)}
                        for (s_, a, b), t in zip(counts, refine_ms)],
            "mean_grad2d_after_last_refine": grad_stats,
            "clocks": clocks}
    print(json.dumps(line), flush=True)
    rast.close()
    loss.close()
    dens.close()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.config == "cfg3" and args.gpus == 1:
        run_cfg3(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
