"""Benchmark of the training step (BASELINE.json metric) on synthetic C1.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  python bench.py --config C3 [--iterations 7000]     (training-run report)
  python bench.py --config C4 [--gpus N] [--steps K]  (batched views, 8 per step)

Workload (N=1): BASELINE.json config 1 -- 1,000,000 seeded synthetic
Gaussians rendered at 1297x840 from 16 cameras on a radius-4 sphere, the
target of each camera a render of an independent seed-1 scene (mip-NeRF 360
garden at 4x downscale is not available; see msplat_b200/synthetic.py).
A step is one full training iteration of one view: projection + SH,
binning, sort, forward raster, L1 + SSIM loss, backward, Adam on all six
groups and the densification statistics.  `value` is training views/s over
the whole job with every input resident in HBM; the per-step footprint
(~2 GB of parameters, moments and buffers) exceeds the 126 MB L2.
`e2e` is the same loop through the public API with the step's target image
copied from pinned host memory (msplat_stage_input: a copy stream, so the
upload overlaps the previous step) and the loss read back every step;
wall clock over K steps, median of three runs after W untimed ones.

Under torchrun (N > 1) every rank trains its own view of the same scene
each step and the ranks combine their gradients before Adam
(msplat_b200.multigpu): by default one kernel per rank sums its shard of the
gradients over NVLink peer memory, applies Adam and writes the shard into
every replica (--dp-mode nccl: an NCCL all-reduce, then Adam on every
replica); per-GPU work is fixed, so scaling is weak.

--config C4 is BASELINE.json's batched-view configuration: 6,000,000
Gaussians, a batch of 8 views at 1920x1080 per step, each of N in
{1, 2, 4, 8} GPUs training 8/N of them (gradients accumulated per rank),
one exchange and one Adam update per step; the batch is fixed, so scaling
is strong.  It reports views/s and the exchange's time and NVLink bytes.

--impl reference times the reference's CPU implementation of the path (the
oracle port, or oracle/_ref when the reference was compiled) on the host
cores, rank 0 only, on the same workload.
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "train steps/s + render FPS @1M Gaussians 1297×840; 1/2/4/8-GPU views/s"
UNIT = "views/s"
CONFIG = "C1"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--dp-mode", choices=("peer", "nccl"), default="peer",
                    help="N > 1: optimiser over NVLink peer memory, or NCCL all-reduce")
    ap.add_argument("--no-cpu-baseline", action="store_true",
                    help="skip the timed CPU oracle sample (profiling runs)")
    ap.add_argument("--config", choices=("C1", "C3", "C4"), default="C1",
                    help="C1 (default): the headline step benchmark; C3: BASELINE.json config 3, "
                         "a 7000-iteration training run with densification, reporting steps/s "
                         "and held-out PSNR/SSIM (one GPU); C4: BASELINE.json config 4, "
                         "6M Gaussians, 8 views of 1920x1080 per step over N GPUs")
    ap.add_argument("--iterations", type=int, default=7000, help="C3: training iterations")
    return ap.parse_args()


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


# Per-step figures from one ncu capture of the first C1 training step
# (profiles/kernels_c1_train_step.md): DRAM bytes of the optimiser stage
# (rest_adam_kernel + project_backward_adam_kernel) and warp instructions of
# the issue-bound kernels.  Instruction counts vary a little with the view;
# the capture's view stands for all.
C1_OPT_STAGE_TRAFFIC = 510080000 + 344294912 + 235875840 + 117640448
C1_WARP_INSTR = {"rast_fwd": ("raster_forward_kernel<0>", 364023216),
                 "rast_bwd": ("raster_backward_kernel<0,2>", 564315330),
                 "loss_fwd_bwd": ("ssim_loss_fused_kernel", 105998350)}
SM_COUNT, ISSUE_PER_SM_CLK = 148, 4


def issue_rooflines(stage_ms: dict, sm_mhz: float) -> list:
    """Achieved warp-instruction issue rate of the issue-bound kernels
    against the SMs' issue slots (148 SMs x 4 schedulers x 1/clock at the SM
    clock sampled during the timed region)."""
    peak = SM_COUNT * ISSUE_PER_SM_CLK * sm_mhz * 1e6 / 1e9   # G warp-instr/s
    out = []
    for stage, (kernel, instr) in C1_WARP_INSTR.items():
        ms = stage_ms.get(stage, 0.0)
        if ms <= 0:
            continue
        ach = instr / (ms / 1000.0) / 1e9
        out.append({"bound": "issue", "kernel": kernel, "achieved": round(ach, 1),
                    "peak": round(peak, 1), "unit": "G warp-instr/s", "frac": round(ach / peak, 4),
                    "launch_ms": round(ms, 4), "warp_instructions": instr})
    return out


# ---------------------------------------------------------------------------

def scene(config: str, seed: int = 0):
    """synthetic.scene(config, seed=seed), kept as .npz files in the directory
    MSPLAT_BENCH_SCENE_CACHE names (when set) so that several runs in one
    session draw each large scene once; a file is written whole under a
    temporary name and then renamed, so concurrent ranks never read a
    partial one."""
    from msplat_b200 import synthetic
    cache = os.environ.get("MSPLAT_BENCH_SCENE_CACHE")
    if not cache:
        return synthetic.scene(config, seed=seed)
    path = os.path.join(cache, f"{config}_seed{seed}.npz")
    _, cams = synthetic.scene(config, n=1, seed=seed)
    if os.path.exists(path):
        with np.load(path) as z:
            return synthetic.Gaussians(*[z[f"g{i}"] for i in range(6)]), cams
    g, cams = synthetic.scene(config, seed=seed)
    os.makedirs(cache, exist_ok=True)
    tmp = f"{path}.{os.getpid()}.tmp.npz"
    np.savez(tmp, **{f"g{i}": a for i, a in enumerate(g.groups())})
    os.replace(tmp, path)
    return g, cams


def build_workload(config: str = CONFIG):
    import torch
    from msplat_b200 import camera, engine
    g, cams = scene(config)
    setups = [camera.prepare_camera(c, step=10**9, sh_degree=3, sh_degree_interval=1000,
                                    rest_bases=15) for c in cams]
    # targets: renders of an independent seed-1 scene, one per camera
    tgt, _ = scene(config, seed=1)
    tmodel = engine.GaussianModel(tgt.groups())
    gts = []
    h, w = setups[0].height, setups[0].width
    for cs in setups:
        ptr = engine.render(tmodel, cs)
        buf = torch.empty((h, w, 3), dtype=torch.float32, device="cuda")
        from msplat_b200 import _lib
        _lib.check(_lib.load().msplat_copy(buf.data_ptr(), ptr, buf.numel() * 4, 2, 0), "copy")
        gts.append(buf)
    torch.cuda.synchronize()
    del tmodel
    model = engine.GaussianModel(g.groups())
    return g, setups, gts, model


def algorithmic_bytes_proj_bwd(n_total: int, n_vis: int, rest_floats: int) -> float:
    """Algorithmic HBM bytes of the fused projection-backward + Adam + stats
    kernel for one step: every Gaussian reads its radius and runs Adam on
    11 floats of means/scales/quats/opacity (read p, m, v; write p, m, v);
    a visible one also reads its 9 raster gradients and its conic/opacity
    record, runs Adam on 3 dc and `rest_floats` SH-rest floats, and updates
    3 statistics (read + write)."""
    per_all = 4 + 11 * 24
    per_vis = 9 * 4 + 16 + 3 * 24 + rest_floats * 24 + 3 * 8
    return float(n_total * per_all + n_vis * per_vis)


def algorithmic_bytes_proj_bwd_grads(n_total: int, n_vis: int, rest_floats: int) -> float:
    """The same kernel in its data-parallel form (N > 1): every Gaussian
    reads its radius and writes its (15 + rest_floats)-float gradient row
    and visibility flag; a visible one also reads its 9 raster gradients,
    its conic/opacity record and its 10 geometry floats, and updates 3
    statistics."""
    per_all = 4 + (15 + rest_floats) * 4
    per_vis = 9 * 4 + 16 + 10 * 4 + 3 * 8
    return float(n_total * per_all + n_vis * per_vis)


def run_ours(args, rank: int, world: int):
    import torch
    from msplat_b200 import _lib, engine
    lib = _lib.load()
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    engine.bind_stream()
    g, setups, gts, model = build_workload()
    dist = None
    if world > 1:
        from msplat_b200 import multigpu
        dist = multigpu.DataParallel(model, rank, world, mode=args.dp_mode)
    ncam = len(setups)

    def view_of(step):
        return (step * world + rank) % ncam

    def one_step(step):
        cs = setups[view_of(step)]
        if dist is None:
            engine.train_step(model, cs, gts[view_of(step)])
        else:
            dist.train_step(cs, gts[view_of(step)])

    for s in range(args.warmup):
        one_step(s)
    torch.cuda.synchronize()
    # The model state the timed steps start from: the end-to-end runs below
    # restart from it, so both phases time the same K steps on the same views.
    def model_state():
        return ([t.clone() for t in model._bufs + model._m + model._v + model._stats],
                model.step_count)

    def restore(state):
        tensors, step_count = state
        for dst, src in zip(model._bufs + model._m + model._v + model._stats, tensors):
            dst.copy_(src)
        model.step_count = step_count

    start_state = model_state()
    if dist is not None:
        dist.barrier()
    # --- timed: device-resident training ---------------------------------
    lib.msplat_kernel_launches(1)
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for s in range(args.steps):
        one_step(args.warmup + s)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    launches = int(lib.msplat_kernel_launches(1))
    ms = e0.elapsed_time(e1)

    # --- per-stage breakdown: the same steps from the same state, with the
    # engine's stage events (kept out of the timed run above) ---------------
    restore(start_state)
    if dist is not None:
        dist.barrier()
    nstage = 6
    buf = (C_double * (nstage * 4096))()
    lib.msplat_enable_gpu_timing(1)
    lib.msplat_drain_gpu_times(None, 0)
    lib.msplat_drain_stage_times(buf, nstage, 4096, None, None)
    torch.cuda.synchronize()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for s in range(args.steps):
        one_step(args.warmup + s)
    e3.record(stream)
    torch.cuda.synchronize()
    lib.msplat_enable_gpu_timing(0)
    staged_ms_per_step = e2.elapsed_time(e3) / args.steps
    nsamp = C_int()
    names = (C_char_p * nstage)()
    ns = lib.msplat_drain_stage_times(buf, nstage, 4096, C_byref(nsamp), names)
    stage_ms = {}
    for si in range(ns):
        vals = [buf[si * 4096 + j] for j in range(nsamp.value)]
        stage_ms[names[si].decode()] = float(np.mean(vals)) if vals else 0.0
    ms_max = ms
    if dist is not None:
        ms_max = dist.max_over_ranks(ms)
    views = args.steps * world
    value = views / (ms_max / 1000.0)

    # --- render FPS (forward only) ------------------------------------------
    torch.cuda.synchronize()
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for s in range(3):
        engine.render(model, setups[s % ncam])
    r0.record(stream)
    for s in range(args.steps):
        engine.render(model, setups[s % ncam])
    r1.record(stream)
    torch.cuda.synchronize()
    render_ms = r0.elapsed_time(r1) / args.steps
    n_isect = int(lib.msplat_num_intersections())
    radii = engine.debug_buffer("radii", model.n, np.int32)
    n_vis = int((radii > 0).sum())

    # --- end to end through the public API with host buffers ----------------
    h, w = setups[0].height, setups[0].width
    host_gts = [t.cpu().pin_memory() for t in gts[:4]]
    gt_bytes = host_gts[0].numel() * 4
    staged = C_void_p()

    def e2e_steps(first, count):
        for s in range(first, first + count):
            # msplat_stage_input: the upload of this step's target overlaps
            # the previous step's kernels (copy stream, two staging buffers)
            hg = host_gts[s % len(host_gts)]
            _lib.check(lib.msplat_stage_input(C_void_p(hg.data_ptr()), gt_bytes,
                                              C_byref(staged)), "msplat_stage_input")
            dev_gt = engine.DevicePtr(staged.value)
            if dist is None:
                engine.train_step(model, setups[view_of(s)], dev_gt)
            else:
                dist.train_step(setups[view_of(s)], dev_gt)
            lib.msplat_last_loss(0)          # the step's loss, read without a wait
        lib.msplat_last_loss(1)              # and the last one, waited for

    # untimed warm-up of the same path (staging buffers, pinned pages), then
    # three timed runs of the device-resident phase's K steps, each from its
    # starting state; the median is reported, all three listed
    e2e_steps(0, args.warmup)
    torch.cuda.synchronize()
    runs = []
    for r in range(3):
        restore(start_state)
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        e2e_steps(args.warmup, args.steps)
        torch.cuda.synchronize()
        e2e_s = time.perf_counter() - t0
        if dist is not None:
            e2e_s = dist.max_over_ranks(e2e_s * 1000.0) / 1000.0
        runs.append(views / e2e_s)
    e2e_value = statistics.median(runs)

    # --- roofline of the dominant HBM-bound kernel ---------------------------
    pk = peaks()
    dom = "proj_bwd_adam"
    if world == 1:
        algo = algorithmic_bytes_proj_bwd(model.n, n_vis, 45)
    else:
        algo = algorithmic_bytes_proj_bwd_grads(model.n, n_vis, 45)
    dom_ms = stage_ms.get(dom, 0.0)
    achieved = algo / (dom_ms / 1000.0) / 1e9 if dom_ms > 0 else 0.0
    kname = ("rest_adam_kernel + project_backward_adam_kernel<false> (projection VJP + Adam)"
             if world == 1 else "project_backward_adam_kernel<true> (gradient output)")
    roofline = {"bound": "hbm", "kernel": kname, "achieved": round(achieved, 1),
                "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                "peak_source": pk["source"], "algorithmic_bytes": algo, "launch_ms": round(dom_ms, 4),
                "traffic": C1_OPT_STAGE_TRAFFIC if world == 1 else None,
                "traffic_source": "ncu dram__bytes_read+write of the stage's kernels, first C1 step"
                if world == 1 else None}

    result = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded C1 scene; targets are renders of a seed-1 scene)",
        "config": {"workload": "C1: 1,000,000 Gaussians, SH degree 3, 1297x840, 16 cameras, "
                               "one view per GPU per step",
                   "gaussians": model.n, "width": w, "height": h, "cameras": ncam,
                   "l2": "inputs larger than L2 (per-step footprint ~2 GB)",
                   "parallelism": (f"dp{world}: replicated Gaussians; " + (
                       "each rank sums its 1/N gradient shard over NVLink peer memory, "
                       "applies Adam and writes the shard into every replica"
                       if args.dp_mode == "peer" else "NCCL all-reduce of the gradient, "
                       "then Adam on every replica")) if world > 1 else "single GPU"},
        "train_steps_per_s": round(args.steps / (ms_max / 1000.0), 2),
        "render_fps": round(1000.0 / render_ms, 1),
        "stage_ms": {k: round(v, 4) for k, v in stage_ms.items()},
        "stage_run_ms_per_step": round(staged_ms_per_step, 4),
        "intersections": n_isect, "visible_gaussians": n_vis,
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT,
                "h2d_bytes_per_step": int(h * w * 3 * 4 + 512),
                "d2h_bytes_per_step": 12, "runs": [round(x, 2) for x in runs],
                "timing": "wall clock around the device-resident phase's K steps (same "
                          "starting model state and views, restored before each run), median "
                          "of 3 runs after W untimed steps"},
        "roofline": roofline,
        "issue_roofline": issue_rooflines(stage_ms, float(clk.get("sm_mhz") or 1965.0)),
        "gpu_launches": launches,
        "clocks": clk,
        "loss": float(lib.msplat_last_loss(1)),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(g, setups, gts)
    if dist is not None:
        if dist.mode == "peer":
            errs = dist.peer_errors()
            if errs:
                raise RuntimeError(f"peer-memory optimiser reported error bits {errs}: "
                                   "a cross-GPU wait timed out, the run is invalid")
        dist.shutdown()
    return result


def _oracle_kind():
    ref = os.path.join(ROOT, "oracle", "_ref", "libmsplat_ref.so")
    return ("reference", ref) if os.path.exists(ref) else ("port", None)


def cpu_baseline(g, setups, gts, steps: int = 1, warmup: int = 0) -> dict:
    """One C1 training step of the CPU implementation on all host threads."""
    from oracle import oracle
    kind, _ = _oracle_kind()
    kind = "port"  # the reference shim is timed by --impl reference
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    cs = setups[0]
    gt = gts[0].cpu().numpy() if hasattr(gts[0], "cpu") else gts[0]
    params = [x.copy() for x in g.groups()]
    m = [np.zeros_like(x) for x in params]
    v = [np.zeros_like(x) for x in params]
    st = [np.zeros(g.n, np.float32) for _ in range(3)]
    run = oracle.Run(cs, g.n, adam_steps=[1e-3] * 6, adam_bc2=[0.0316] * 6)
    for _ in range(warmup):
        run.train_step(params, m, v, gt, *st)
    t0 = time.perf_counter()
    for _ in range(steps):
        run.train_step(params, m, v, gt, *st)
    dt = time.perf_counter() - t0
    return {"value": round(steps / dt, 4), "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"{steps} full C1 training step(s) of one 1297x840 view, 1M Gaussians "
                      f"(CPU oracle, OpenMP over {threads} threads)"}


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return None
    from msplat_b200 import camera, synthetic
    from oracle import oracle
    g, cams = synthetic.scene(CONFIG)
    setups = [camera.prepare_camera(c, step=10**9, sh_degree=3, sh_degree_interval=1000,
                                    rest_bases=15) for c in cams]
    gts = [synthetic.target_image(setups[0].width, setups[0].height, 1 + i) for i in range(2)]
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    params = [x.copy() for x in g.groups()]
    m = [np.zeros_like(x) for x in params]
    v = [np.zeros_like(x) for x in params]
    st = [np.zeros(g.n, np.float32) for _ in range(3)]
    # the reference's own kernels (oracle/_ref, built from its Metal source)
    # when present -- about 15x slower than the C port, so fewer steps --
    # else the C port
    kind, _ = _oracle_kind()
    impl = "reference" if kind == "reference" else "oracle"
    steps = max(1, min(args.steps, 3 if impl == "reference" else 8))
    warm = max(0, min(args.warmup, 1))
    times = []
    for s in range(warm + steps):
        cs = setups[s % len(setups)]
        run = oracle.Run(cs, g.n, adam_steps=[1e-3] * 6, adam_bc2=[0.0316] * 6)
        t0 = time.perf_counter()
        run.train_step(params, m, v, gts[s % 2], *st, impl=impl)
        if s >= warm:
            times.append(time.perf_counter() - t0)
    value = len(times) / sum(times)
    return {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT,
            "n_gpus": world, "steps": len(times), "warmup": warm,
            "ms_per_step": round(1000 * sum(times) / len(times), 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "C1: 1,000,000 Gaussians, SH degree 3, 1297x840, one view "
                                   "per step (CPU)"},
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads,
                             "kind": "port" if kind == "port" else "reference",
                             "sample": f"{len(times)} full C1 training steps (capped at "
                                       f"{3 if impl == 'reference' else 8} of --steps "
                                       f"{args.steps}); " + (
                                           "the reference's Metal kernels compiled for the CPU "
                                           "(MSL shim: SIMD lanes as fibers, OpenMP over "
                                           "threadgroups)" if impl == "reference" else
                                           "the C restatement of the reference's kernels")},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def run_c3(args) -> dict:
    """a full synthetic training run at 1024x768.
    Ground truth: a seed-7 scene of 500,000 Gaussians drawn as in config 1,
    rendered to 72 cameras on the radius-4 sphere (every 9th held out: 64
    train, 8 test).  Student: 100,000 Gaussians, means U[-2,2]^3, the rest
    as in config 0.  The reference's schedule (Model::afterTrain defaults):
    densification every 100 steps from 500 until half the run, gradient
    threshold 2e-4, opacity reset every 3000 steps, SH degree +1 every 1000
    steps, means learning rate decayed over the run; one view per step in a
    reshuffled order.  Timed on the device (CUDA events around the whole
    run, densification included); held-out PSNR / SSIM by
    msplat_eval_metrics on the 8 test views."""
    import math as _m

    import torch
    from msplat_b200 import _lib, camera, engine, synthetic
    lib = _lib.load()
    engine.bind_stream()
    w, h, iters = 1024, 768, args.iterations
    cams = synthetic.fibonacci_cameras(72, 4.0, w, h)
    test_idx = list(range(0, 72, 9))
    train_idx = [i for i in range(72) if i not in test_idx]
    final = [camera.prepare_camera(c, step=10**9, sh_degree=3, sh_degree_interval=1000,
                                   rest_bases=15) for c in cams]
    truth = synthetic.gaussians(500_000, 7, mean_range=2.0, log_scale_mu=_m.log(0.01),
                                log_scale_sigma=0.4)
    tmodel = engine.GaussianModel(truth.groups())
    gts = []
    for cs in final:
        ptr = engine.render(tmodel, cs)
        buf = torch.empty((h, w, 3), dtype=torch.float32, device="cuda")
        _lib.check(lib.msplat_copy(buf.data_ptr(), ptr, buf.numel() * 4, 2, 0), "copy")
        gts.append(buf)
    torch.cuda.synchronize()
    del tmodel
    student = synthetic.gaussians(100_000, 8, mean_range=2.0, log_scale_mu=_m.log(0.02),
                                  log_scale_sigma=0.3)
    model = engine.GaussianModel(student.groups())
    sched = engine.Schedule(max_steps=iters, num_cameras=len(train_idx))
    rng = np.random.default_rng(42)
    order = []
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    lib.msplat_kernel_launches(1)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e0.record(stream)
    for step in range(1, iters + 1):
        if not order:
            order = list(rng.permutation(train_idx))
        ci = int(order.pop())
        cs = camera.prepare_camera(cams[ci], step=step, sh_degree=3, sh_degree_interval=1000,
                                   rest_bases=15)
        engine.train_step(model, cs, gts[ci])
        model.schedule_means_lr(step, iters)
        sched.after_train(model, step, w, h)
    e1.record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    clk = clocks.stop()
    launches = int(lib.msplat_kernel_launches(1))
    ms = e0.elapsed_time(e1)
    psnr, ssim, l1 = [], [], []
    for ci in test_idx:
        cs = camera.prepare_camera(cams[ci], step=iters, sh_degree=3, sh_degree_interval=1000,
                                   rest_bases=15)
        ptr = engine.render(model, cs)
        out = [C_float() for _ in range(3)]
        _lib.check(lib.msplat_eval_metrics(C_void_p(ptr), C_void_p(gts[ci].data_ptr()), h, w, 11,
                                           1.5, *[C_byref(o) for o in out]), "eval")
        psnr.append(out[0].value)
        ssim.append(out[1].value)
        l1.append(out[2].value)
    steps_per_s = iters / (ms / 1000.0)
    return {
        "metric": "C3 training run: steps/s + held-out PSNR/SSIM", "value": round(steps_per_s, 2),
        "unit": "steps/s", "n_gpus": 1, "steps": iters, "warmup": 0,
        "ms_per_step": round(ms / iters, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seed-7 ground-truth scene rendered to 72 cameras; seed-8 student)",
        "config": {"workload": "C3: 100,000 -> densified Gaussians, 7000 iterations at 1024x768, "
                               "64 train / 8 held-out cameras",
                   "iterations": iters, "width": w, "height": h},
        "heldout_psnr": round(float(np.mean(psnr)), 3), "heldout_ssim": round(float(np.mean(ssim)), 4),
        "heldout_l1": round(float(np.mean(l1)), 5), "final_gaussians": model.n,
        "wall_s": round(wall, 2), "gpu_launches": launches, "clocks": clk,
    }


def exchange_bytes(n: int, world: int, compact: bool, mode: str) -> int:
    """Bytes one rank moves over NVLink per step in the optimiser exchange.
    peer: it reads its 1/world shard of every other rank's gradient buffer
    (60 floats per Gaussian, or 15 in the compact layout) and writes its
    updated shard of the 59 parameter floats into every other replica.
    nccl: a ring all-reduce of the 60-float buffer sends 2 (world-1)/world of
    it per rank."""
    if world <= 1:
        return 0
    share = (world - 1) / world
    if mode == "nccl":
        return int(2 * share * n * 60 * 4)
    return int(share * n * ((15 if compact else 60) + 59) * 4)


# Peer copy bandwidth per direction between two B200s of one node over
# NVLink 5 / NVSwitch, as measured on this pool (nominal: 900 GB/s).
NVLINK_PEER_GBS = 770.0


def exchange_roofline(n: int, world: int, compact: bool, mode: str, ms: float):
    """The exchange's NVLink bound: the larger of the bytes one rank receives
    and sends per step (links are full duplex), at the measured per-direction
    peer bandwidth, against the measured exchange time.  peer: receives its
    shard of every other rank's gradient rows, sends its updated parameter
    shard to every other replica; nccl ring all-reduce: 2 (world-1)/world of
    the 60-float buffer each way."""
    if world <= 1 or not ms:
        return None
    share = (world - 1) / world
    if mode == "nccl":
        rx = tx = 2 * share * n * 60 * 4
    else:
        rx = share * n * (15 if compact else 60) * 4
        tx = share * n * 59 * 4
    bound_ms = max(rx, tx) / (NVLINK_PEER_GBS * 1e9) * 1e3
    return {"bound": "nvlink", "peak_gbs_per_direction": NVLINK_PEER_GBS,
            "peak_source": "measured peer copy on this pool", "bytes_in": int(rx),
            "bytes_out": int(tx), "bound_ms": round(bound_ms, 3),
            "frac": round(bound_ms / ms, 4)}


def run_c4(args, rank: int, world: int) -> dict:
    """BASELINE.json config 4, multi-GPU batched views: 6,000,000 Gaussians
    drawn as in config 1 (seed 0), 8 cameras on the radius-4 sphere at
    1920x1080, targets rendered from an independent seed-1 scene of the same
    size.  A step trains the batch of all 8 views: rank r of N takes views
    r, r + N, ... (8/N of them), accumulating their gradients of the batch's
    mean loss; then one exchange over NVLink and one Adam update
    (multigpu.DataParallel.train_views; on one GPU multigpu.train_batch).
    Timed on the device, max over ranks; the exchange is timed in a second
    pass over the same number of steps with CUDA events around it."""
    import torch
    from msplat_b200 import _lib, engine, multigpu
    batch = 8
    if world not in (1, 2, 4, 8):
        raise SystemExit("C4 runs its batch of 8 views on 1, 2, 4 or 8 GPUs")
    vpr = batch // world
    lib = _lib.load()
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    engine.bind_stream()
    g, setups, gts, model = build_workload("C4")
    mine = [rank + k * world for k in range(vpr)]
    cams = [setups[v] for v in mine]
    tgts = [gts[v] for v in mine]
    dist = None
    if world == 1:
        grad = torch.empty(multigpu.grad_floats(model.n, model.rest_bases), dtype=torch.float32,
                           device="cuda")

        def one_step():
            multigpu.train_batch(model, cams, tgts, grad)
    else:
        dist = multigpu.DataParallel(model, rank, world, mode=args.dp_mode, views_per_rank=vpr)

        def one_step():
            dist.train_views(cams, tgts)
    steps = args.steps
    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    lib.msplat_kernel_launches(1)
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(steps):
        one_step()
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    launches = int(lib.msplat_kernel_launches(1))
    ms = e0.elapsed_time(e1)
    ms_max = dist.max_over_ranks(ms) if dist is not None else ms
    # second pass: the exchange (peer kernel or all-reduce) plus Adam, timed
    # per step between the rank's last backward and the step's end
    ex_ms = None
    if dist is not None:
        dist.barrier()
        torch.cuda.synchronize()
        evs = []
        for _ in range(steps):
            model.step_count += 1
            multigpu.accumulate_views(dist.ops, model, cams, tgts, dist.grad, dist.compact)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            dist.apply(cams[0])
            b.record(stream)
            evs.append((a, b))
        torch.cuda.synchronize()
        ex_ms = dist.max_over_ranks(float(np.mean([a.elapsed_time(b) for a, b in evs])))
    n_isect = int(lib.msplat_num_intersections())
    xbytes = exchange_bytes(model.n, world, dist.compact if dist else False, args.dp_mode)
    result = {
        "metric": "C4 batched views: views/s (8 views per step, 6M Gaussians, 1920x1080)",
        "value": round(batch * steps / (ms_max / 1000.0), 2), "unit": "views/s",
        "n_gpus": world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": round(ms_max / steps, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded C4 scene; targets are renders of a seed-1 scene)",
        "config": {"workload": "C4: 6,000,000 Gaussians, SH degree 3, 8 views of 1920x1080 per "
                               "step on a radius-4 sphere",
                   "gaussians": model.n, "width": setups[0].width, "height": setups[0].height,
                   "views_per_step": batch, "views_per_gpu": vpr,
                   "l2": "inputs larger than L2 (parameters and moments ~4.2 GB)",
                   "parallelism": "single GPU" if world == 1 else (
                       f"dp{world}: replicated Gaussians, " + (
                           "peer-memory reduce + Adam + parameter write-back"
                           + (" (compact v_rgb exchange)" if dist.compact else "")
                           if args.dp_mode == "peer" else "NCCL all-reduce, Adam on every replica"))},
        "exchange": None if dist is None else {
            "mode": args.dp_mode, "ms_per_step": round(ex_ms, 3),
            "nvlink_bytes_per_rank": xbytes,
            "gbs_per_rank": round(xbytes / (ex_ms / 1000.0) / 1e9, 1) if ex_ms else None,
            "roofline": exchange_roofline(model.n, world, dist.compact, args.dp_mode, ex_ms),
            "timing": "CUDA events around the exchange + Adam of each step (includes waiting "
                      "for the slowest rank's gradients), mean over steps, max over ranks"},
        "intersections_last_view": n_isect,
        "gpu_launches": launches, "clocks": clk,
    }
    if dist is not None:
        if dist.mode == "peer" and dist.peer_errors():
            raise RuntimeError("peer-memory optimiser reported a timed-out wait: run invalid")
        dist.shutdown()
    return result


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.config == "C3":
        if rank == 0:
            print(json.dumps(run_c3(args)), flush=True)
        return
    if args.config == "C4":
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable":
                                  "C4 is a multi-GPU configuration; the reference trains one "
                                  "view on one device"}), flush=True)
            return
        res = run_c4(args, rank, world)
        if rank == 0:
            print(json.dumps(res), flush=True)
        return
    if args.impl == "reference":
        res = run_reference(args, rank, world)
    else:
        res = run_ours(args, rank, world)
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)


from ctypes import byref as C_byref, c_char_p as C_char_p, c_double as C_double, c_int as C_int  # noqa: E402
from ctypes import c_float as C_float, c_void_p as C_void_p  # noqa: E402

if __name__ == "__main__":
    main()
