"""Benchmark of the training step (BASELINE.json metric) on synthetic C1.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  python bench.py --config C3 [--iterations 7000]     (training-run report)
  python bench.py --config C4 [--gpus N] [--steps K]  (batched views, 8 per step)
  python bench.py --config C2                         (3M clustered Gaussians, 1920x1080)
  python bench.py --profile-step                      (one C1 step for ncu)
  python bench.py --summarize-ncu CSV... --hash-file F (per-kernel counter summary)

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
The default C1 run appends the same C4 measurement on the same N GPUs as
its `c4` object (--no-c4 skips it).

Rooflines: `roofline` is the HBM-bound optimiser stage; `hbm_rooflines`
adds the projection forward; `issue_roofline` the issue-bound stages
(instruction counts from the committed per-kernel ncu summary
profiles/counters_c1_train_step.txt, used only when its build hash equals
this build's); `raster_work` the engine's count of the reference loop's
pixel.Gaussian work (E) and the rasterizers' FP32 rooflines.

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
    ap.add_argument("--config", choices=("C1", "C2", "C3", "C4"), default="C1",
                    help="C1 (default): the headline step benchmark, followed by a C4 leg "
                         "(--no-c4 skips it); C2: BASELINE.json config 2, the same step on 3M "
                         "clustered Gaussians at 1920x1080; C3: BASELINE.json config 3, "
                         "a 7000-iteration training run with densification, reporting steps/s "
                         "and held-out PSNR/SSIM (one GPU); C4: BASELINE.json config 4, "
                         "6M Gaussians, 8 views of 1920x1080 per step over N GPUs")
    ap.add_argument("--iterations", type=int, default=7000, help="C3: training iterations")
    ap.add_argument("--no-c4", action="store_true",
                    help="C1: skip the C4 batched-view leg reported under 'c4'")
    ap.add_argument("--profile-step", action="store_true",
                    help="for ncu: the C1 workload, W warm-up steps, then one training step "
                         "between cudaProfilerStart and cudaProfilerStop; prints the build hash")
    ap.add_argument("--summarize-ncu", nargs="+", metavar="CSV",
                    help="write the per-kernel counter summary from ncu --csv logs of "
                         "--profile-step runs (no GPU needed)")
    ap.add_argument("--hash-file", help="--summarize-ncu: the JSON line --profile-step printed")
    ap.add_argument("--profile-config", choices=("C1", "C4q"), default="C1",
                    help="--profile-step: C1, or C4q (C4's distributions at a quarter of the "
                         "Gaussians and pixels: C4's ~4,000 intersections per tile, small enough "
                         "for detailed captures)")
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


# ---------------------------------------------------------------------------
# Per-kernel counters of one C1 training step, from ncu.  They live in a
# committed text summary, one row per kernel, tagged with the hash of the
# sources they were captured from; a run whose sources hash differently
# reports them as stale and derives nothing from them.
#
# Capture (one GPU, one kernel per ncu command, one launch each; the step is
# bracketed by cudaProfilerStart/Stop in --profile-step mode):
#   python bench.py --profile-step > ncu_out/profile_step.json &&
#   ncu --profile-from-start off --clock-control none --kernel-name-base function \
#       -k regex:<KERNEL> -c 1 --metrics <COUNTER_METRICS> --csv --print-units base \
#       --log-file ncu_out/ctr_<KERNEL>.csv python bench.py --profile-step
# Summary:
#   python bench.py --summarize-ncu ncu_out/ctr_*.csv \
#       --hash-file ncu_out/profile_step.json
# ---------------------------------------------------------------------------
COUNTERS_FILE = os.path.join(ROOT, "profiles", "counters_c1_train_step.txt")
COUNTER_METRICS = ("dram__bytes_read.sum", "dram__bytes_write.sum", "smsp__inst_executed.sum",
                   "gpu__time_duration.sum")
# kernel (ncu base name) -> stage of the engine's stage timer it runs in
PROFILED_KERNELS = {
    "project_forward_kernel": "proj_sh_fwd",
    "scan_tiles_kernel": "bin_sort",
    "scatter_kernel": "bin_sort",
    "sort_large_tiles_kernel": "bin_sort",
    "sort_tiles_kernel": "bin_sort",
    "raster_forward_kernel": "rast_fwd",
    "ssim_loss_fused_kernel": "loss_fwd_bwd",
    "raster_backward_kernel": "rast_bwd",
    "project_backward_adam_kernel": "proj_bwd_adam",
    "rest_adam_kernel": "proj_bwd_adam",
}
SM_COUNT, ISSUE_PER_SM_CLK, FP32_LANES_PER_SM = 148, 4, 128


def build_hash() -> str:
    """First 12 hex digits of the SHA-256 of the engine's sources (kernels,
    host code, headers and the build recipe), files in name order."""
    import hashlib
    h = hashlib.sha256()
    for d in (os.path.join("msplat_b200", "csrc"), "include"):
        base = os.path.join(ROOT, d)
        for f in sorted(os.listdir(base)):
            if f.endswith((".cu", ".cuh", ".h", ".hpp")):
                h.update(f.encode())
                with open(os.path.join(base, f), "rb") as fh:
                    h.update(fh.read())
    with open(os.path.join(ROOT, "msplat_b200", "build.py"), "rb") as fh:
        h.update(fh.read())
    return h.hexdigest()[:12]


def load_counters(path: str = COUNTERS_FILE) -> dict:
    """{"build": hash, "view": camera index, "kernels": {name: {...}}} from
    the committed summary, or {} when it is absent."""
    if not os.path.exists(path):
        return {}
    out = {"build": None, "view": None, "kernels": {}}
    cols = None
    with open(path) as f:
        for line in f:
            line = line.rstrip("\n")
            if line.startswith("# build "):
                out["build"] = line.split()[2]
            elif line.startswith("# view "):
                out["view"] = int(line.split()[2])
            elif not line or line.startswith("#"):
                continue
            elif cols is None:
                cols = line.split("\t")
            else:
                row = dict(zip(cols, line.split("\t")))
                out["kernels"][row["kernel"]] = {
                    k: (v if k in ("kernel", "launch") else float(v)) for k, v in row.items()}
    return out


def summarize_ncu(csv_paths, hash_file: str, out_path: str = COUNTERS_FILE) -> str:
    """Write the counters summary from ncu --csv logs of --profile-step runs
    (one kernel each).  The build hash and the profiled view come from the
    JSON line --profile-step printed."""
    import csv as _csv
    with open(hash_file) as f:
        info = json.loads([ln for ln in f if ln.strip().startswith("{")][-1])
    rows = {}
    for pth in csv_paths:
        with open(pth) as f:
            lines = [ln for ln in f if ln.startswith('"')]
        for rec in _csv.DictReader(lines):
            name = rec.get("Kernel Name", "")
            head = name.split("(")[0].strip()            # "void ns::kernel<0, 2>"
            if head.startswith("void "):
                head = head[5:]
            base = head.split("<")[0].split("::")[-1].strip()
            if base not in PROFILED_KERNELS:
                continue
            r = rows.setdefault(base, {"kernel": base, "launch": head.split("::")[-1]})
            metric, val = rec.get("Metric Name"), rec.get("Metric Value", "").replace(",", "")
            if metric in COUNTER_METRICS:
                r[metric] = float(val)
    cols = ["kernel", "launch", "dram_read_bytes", "dram_write_bytes", "warp_instructions",
            "duration_ns"]
    keys = dict(zip(cols[2:], COUNTER_METRICS))
    lines = ["# ncu counters of one C1 training step: one launch of each kernel, captured",
             "# alone (--clock-control none; durations are cold-cache and serialised).",
             f"# build {info['build_hash']}",
             f"# view {info['view']}",
             "# command, per kernel K (repository root, one GPU):",
             "#   python bench.py --profile-step > ncu_out/profile_step.json &&",
             "#   ncu --profile-from-start off --clock-control none --kernel-name-base function \\",
             f"#       -k regex:K -c 1 --metrics {','.join(COUNTER_METRICS)} \\",
             "#       --csv --print-units base \\",
             "#       --log-file ncu_out/ctr_K.csv python bench.py --profile-step",
             "# summary: python bench.py --summarize-ncu ncu_out/ctr_*.csv "
             "--hash-file ncu_out/profile_step.json",
             "\t".join(cols)]
    for k in PROFILED_KERNELS:
        if k in rows and all(m in rows[k] for m in COUNTER_METRICS):
            r = rows[k]
            lines.append("\t".join([r["kernel"], r["launch"]] +
                                   [str(int(r[keys[c]])) for c in cols[2:]]))
    with open(out_path, "w") as f:
        f.write("\n".join(lines) + "\n")
    return out_path


def counters_status(ctr: dict) -> dict:
    here = build_hash()
    return {"source": os.path.relpath(COUNTERS_FILE, ROOT) if ctr else None,
            "captured_build": ctr.get("build"), "this_build": here,
            "matches_this_build": bool(ctr) and ctr.get("build") == here,
            "profiled_view": ctr.get("view")}


def issue_rooflines(stage_ms: dict, sm_mhz: float, ctr: dict, scale: dict) -> list:
    """Achieved warp-instruction issue rate of the issue-bound stages against
    the SMs' issue slots (148 SMs x 4 schedulers x 1/clock at the SM clock
    sampled during the timed region).  Instructions: the profiled view's
    ncu counts, scaled to the timed steps' mean work (`scale[stage]`: mean
    over the timed views of the stage's work unit -- E for the rasterizers,
    intersections for binning and sort -- over the profiled view's)."""
    peak = SM_COUNT * ISSUE_PER_SM_CLK * sm_mhz * 1e6 / 1e9   # G warp-instr/s
    out = []
    for stage in ("rast_fwd", "rast_bwd", "loss_fwd_bwd", "bin_sort"):
        kern = [k for k, st in PROFILED_KERNELS.items() if st == stage and k in ctr]
        ms = stage_ms.get(stage, 0.0)
        if not kern or ms <= 0:
            continue
        instr = sum(ctr[k]["warp_instructions"] for k in kern) * scale.get(stage, 1.0)
        ach = instr / (ms / 1000.0) / 1e9
        out.append({"bound": "issue", "stage": stage, "kernels": kern, "achieved": round(ach, 1),
                    "peak": round(peak, 1), "unit": "G warp-instr/s", "frac": round(ach / peak, 4),
                    "launch_ms": round(ms, 4), "warp_instructions": int(instr),
                    "work_scale": round(scale.get(stage, 1.0), 4)})
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


WORKLOADS = {
    "C1": "C1: 1,000,000 Gaussians, SH degree 3, 1297x840, 16 cameras, one view per GPU per step",
    "C2": "C2: 3,000,000 Gaussians (70% in 10 clusters), SH degree 3, 1920x1080, one camera at "
          "distance 3, one view per GPU per step",
}


def run_ours(args, rank: int, world: int, config: str = CONFIG):
    import torch
    from msplat_b200 import _lib, engine
    lib = _lib.load()
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    engine.bind_stream()
    g, setups, gts, model = build_workload(config)
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

    # --- raster work of the timed steps, replayed from the same state: per
    # step the engine's count of the reference loop's pixel.Gaussian work
    # (msplat_count_raster_work) and the intersections --------------------
    restore(start_state)
    if dist is not None:
        dist.barrier()
    work = np.zeros((args.steps, 4), np.float64)
    step_isect = np.zeros(args.steps, np.float64)
    wbuf = (C_ulonglong * 4)()
    for s in range(args.steps):
        one_step(args.warmup + s)
        if lib.msplat_count_raster_work(wbuf) == 0:
            work[s] = [float(x) for x in wbuf]
        step_isect[s] = float(lib.msplat_num_intersections())

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

    # --- per-kernel counters of the profiled step (committed ncu summary) ----
    ctr_all = load_counters()
    ctr_state = counters_status(ctr_all)
    use_ctr = ctr_state["matches_this_build"] and config == "C1" and world == 1
    ctr = ctr_all.get("kernels", {}) if use_ctr else {}
    # work of the profiled step (the first timed step: same state and view as
    # --profile-step after the same warm-up) against the timed steps' mean
    prof = work[0] if args.steps else np.zeros(4)
    mean_w = work.mean(axis=0) if args.steps else np.zeros(4)
    same_view = ctr_all.get("view") == view_of(args.warmup)
    scale = {}
    if use_ctr and same_view and prof[0] > 0:
        scale = {"rast_fwd": mean_w[0] / prof[0], "rast_bwd": mean_w[3] / max(prof[3], 1.0),
                 "bin_sort": float(step_isect.mean() / max(step_isect[0], 1.0)),
                 "loss_fwd_bwd": 1.0}
    elif use_ctr:
        use_ctr, ctr = False, {}
        ctr_state["note"] = "profiled view differs from the first timed view: counters unused"
    sm_mhz = float(clk.get("sm_mhz") or 1965.0)

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
    stage_traffic = None
    if ctr and all(k in ctr for k in ("project_backward_adam_kernel", "rest_adam_kernel")):
        stage_traffic = int(sum(ctr[k]["dram_read_bytes"] + ctr[k]["dram_write_bytes"]
                                for k in ("project_backward_adam_kernel", "rest_adam_kernel")))
    roofline = {"bound": "hbm", "kernel": kname, "achieved": round(achieved, 1),
                "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                "peak_source": pk["source"], "algorithmic_bytes": algo, "launch_ms": round(dom_ms, 4),
                "traffic": stage_traffic,
                "traffic_source": "ncu dram__bytes_read+write of the stage's two kernels, profiled "
                                  "step (profile_counters)" if stage_traffic else None}
    # the projection forward against HBM: every Gaussian reads its mean,
    # scale and rotation (40 B) to be culled or kept; a kept one reads its
    # opacity, dc and SH-rest (196 B) and writes its 56 B record; a culled
    # one writes its zero radius
    pf_ms = stage_ms.get("proj_sh_fwd", 0.0)
    pf_algo = float(model.n * 40 + n_vis * (196 + 56) + (model.n - n_vis) * 4)
    pf_ach = pf_algo / (pf_ms / 1000.0) / 1e9 if pf_ms > 0 else 0.0
    pf_traffic = None
    if ctr and "project_forward_kernel" in ctr:
        k = ctr["project_forward_kernel"]
        pf_traffic = int(k["dram_read_bytes"] + k["dram_write_bytes"])
    hbm_more = [{"bound": "hbm", "kernel": "project_forward_kernel", "achieved": round(pf_ach, 1),
                 "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(pf_ach / pk["hbm_gbs"], 4),
                 "algorithmic_bytes": pf_algo, "launch_ms": round(pf_ms, 4),
                 "traffic": pf_traffic}]

    # --- raster work: E and what the rasterizers spend on it -----------------
    fp32_peak = SM_COUNT * FP32_LANES_PER_SM * sm_mhz * 1e6 / 1e9    # G lane-ops/s
    V, S_, E, Wk = (float(x) for x in mean_w)
    fwd_ops = 9 * V + 4 * S_ + 7 * E
    bwd_ops = 9 * Wk + 56 * E
    raster_work = {
        "definition": "per step, summed over pixels (msplat_count_raster_work): visited = list "
                      "positions the reference's forward loop visits; sigma_passed = pairs with "
                      "0 <= sigma < 5.55; E = pairs blended into the pixel (contributing "
                      "pixel.Gaussian evaluations); bwd_walk = positions the reference's "
                      "backward walks",
        "visited": round(V), "sigma_passed": round(S_), "E": round(E), "bwd_walk": round(Wk),
        "steps_counted": int(args.steps),
        "fp32_roofline": [], "instructions_per_evaluation": None,
    }
    for stage, ops, label in (("rast_fwd", fwd_ops, "9 per visited + 4 per sigma-passed "
                                                     "(exp as 1) + 7 per E"),
                              ("rast_bwd", bwd_ops, "9 per walked position + 56 per E")):
        ms_ = stage_ms.get(stage, 0.0)
        if ms_ > 0 and ops > 0:
            ach = ops / (ms_ / 1000.0) / 1e9
            raster_work["fp32_roofline"].append({
                "stage": stage, "algorithmic_fp32_ops": round(ops), "ops_count": label,
                "achieved": round(ach, 1), "peak": round(fp32_peak, 1),
                "unit": "G FP32 lane-ops/s", "frac": round(ach / fp32_peak, 4)})
    if ctr and prof[2] > 0:
        per = {}
        for kern, unit_idx in (("raster_forward_kernel", 2), ("raster_backward_kernel", 2)):
            if kern in ctr:
                thr = ctr[kern]["warp_instructions"] * 32.0
                per[kern] = {"thread_instr_per_E": round(thr / prof[unit_idx], 2),
                             "thread_instr_per_visited" if kern.startswith("raster_forward")
                             else "thread_instr_per_walked":
                             round(thr / prof[0 if kern.startswith("raster_forward") else 3], 2)}
        raster_work["instructions_per_evaluation"] = per
        raster_work["profiled_step"] = {"visited": int(prof[0]), "sigma_passed": int(prof[1]),
                                        "E": int(prof[2]), "bwd_walk": int(prof[3])}

    result = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": f"synthetic (seeded {config} scene; targets are renders of a seed-1 scene)",
        "config": {"workload": WORKLOADS[config],
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
        "issue_roofline": issue_rooflines(stage_ms, sm_mhz, ctr, scale),
        "hbm_rooflines": hbm_more,
        "raster_work": raster_work,
        "build_hash": ctr_state["this_build"],
        "profile_counters": ctr_state,
        "gpu_launches": launches,
        "clocks": clk,
        "loss": float(lib.msplat_last_loss(1)),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v0 = view_of(args.warmup)
        cap = int(max(16 * model.n, 2 * (step_isect.max() if args.steps else 0)))
        result["cpu_baseline"] = cpu_baseline(g, [setups[v0]], [gts[v0]], config=config,
                                              isect_capacity=cap)
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


def cpu_baseline(g, setups, gts, steps: int = 1, config: str = CONFIG,
                 isect_capacity: int | None = None) -> dict:
    """One training step of the CPU port (the oracle's C restatement) on all
    host threads, on the GPU arm's first timed view: same scene, target and
    Adam scalars (first step of a fresh model)."""
    from msplat_b200 import engine
    from oracle import oracle
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    cs = setups[0]
    gt = gts[0].cpu().numpy() if hasattr(gts[0], "cpu") else gts[0]
    params = [x.copy() for x in g.groups()]
    m = [np.zeros_like(x) for x in params]
    v = [np.zeros_like(x) for x in params]
    st = [np.zeros(g.n, np.float32) for _ in range(3)]
    dt = 0.0
    for k in range(steps):
        sz, bc2 = engine.adam_scalars(k + 1, engine.LR_INIT)
        run = oracle.Run(cs, g.n, adam_steps=sz, adam_bc2=bc2, isect_capacity=isect_capacity)
        t0 = time.perf_counter()
        run.train_step(params, m, v, gt, *st)
        dt += time.perf_counter() - t0
    h, w = cs.height, cs.width
    return {"value": round(steps / dt, 4), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{steps} full {config} training step(s) of one {w}x{h} view, {g.n:,} "
                      f"Gaussians, the GPU arm's target (CPU oracle, OpenMP over {threads} "
                      "threads)"}


def run_reference(args, rank: int, world: int):
    """The reference's own CPU implementation of the step on this host's
    cores, on the GPU arm's workload: the C1 scene, its 16 cameras in the
    same order (step s trains camera s mod 16), targets rendered from the
    seed-1 scene (by the oracle, bit-exact with the engine's renders the GPU
    arm trains on), Adam scalars of a model at step s + 1, W untimed and K
    timed full steps in sequence on one evolving model.  The kernels are the
    reference's Metal source compiled for the CPU (oracle/_ref, MSL shim)
    when that build is present, else the C port."""
    if rank != 0:
        return None
    from msplat_b200 import camera, engine
    from oracle import oracle
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    kind, _ = _oracle_kind()
    impl = "reference" if kind == "reference" else "oracle"
    g, cams = scene(CONFIG)
    setups = [camera.prepare_camera(c, step=10**9, sh_degree=3, sh_degree_interval=1000,
                                    rest_bases=15) for c in cams]
    ncam = len(setups)
    h, w = setups[0].height, setups[0].width
    tg, _ = scene(CONFIG, seed=1)
    gts = {}
    for vi in sorted({s % ncam for s in range(args.warmup + args.steps)}):
        r = oracle.Run(setups[vi], tg.n)
        r.render(tg.groups())
        gts[vi] = r.out_img.reshape(h, w, 3).copy()
    del tg
    params = [x.copy() for x in g.groups()]
    m = [np.zeros_like(x) for x in params]
    v = [np.zeros_like(x) for x in params]
    st = [np.zeros(g.n, np.float32) for _ in range(3)]
    times = []
    for s in range(args.warmup + args.steps):
        vi = s % ncam
        sz, bc2 = engine.adam_scalars(s + 1, engine.LR_INIT)
        run = oracle.Run(setups[vi], g.n, adam_steps=sz, adam_bc2=bc2)
        t0 = time.perf_counter()
        rc = run.train_step(params, m, v, gts[vi], *st, impl=impl)
        dt = time.perf_counter() - t0
        if rc != 0:
            raise RuntimeError("reference step reported a per-tile overflow")
        if s >= args.warmup:
            times.append(dt)
    value = len(times) / sum(times)
    what = ("the reference's Metal kernels compiled for the CPU (MSL shim: SIMD lanes as "
            "fibers, OpenMP over threadgroups)" if impl == "reference" else
            "the C restatement of the reference's kernels")
    return {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT,
            "n_gpus": world, "steps": len(times), "warmup": args.warmup,
            "ms_per_step": round(1000 * sum(times) / len(times), 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded C1 scene; targets are renders of a seed-1 scene)",
            "config": {"workload": WORKLOADS[CONFIG], "gaussians": g.n, "width": w, "height": h,
                       "cameras": ncam, "parallelism": f"CPU, {threads} threads (rank 0 only)"},
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads,
                             "kind": kind,
                             "sample": f"{len(times)} full C1 training steps after "
                                       f"{args.warmup} untimed ones, views in the GPU arm's "
                                       f"order; {what}"},
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
    peer bandwidth, against the measured exchange time.  peer: a rank
    receives its shard of every other rank's gradient rows and every other
    rank's updated parameter shard (59 floats per Gaussian) into its
    replica, and sends as much (its gradient rows to the shards' owners, its
    own shard to every other replica); nccl ring all-reduce: 2 (world-1)/world
    of the 60-float buffer each way."""
    if world <= 1 or not ms:
        return None
    share = (world - 1) / world
    if mode == "nccl":
        rx = tx = 2 * share * n * 60 * 4
    else:
        rx = tx = share * n * ((15 if compact else 60) + 59) * 4
    bound_ms = max(rx, tx) / (NVLINK_PEER_GBS * 1e9) * 1e3
    return {"bound": "nvlink", "peak_gbs_per_direction": NVLINK_PEER_GBS,
            "peak_source": "measured peer copy on this pool", "bytes_in": int(rx),
            "bytes_out": int(tx), "bound_ms": round(bound_ms, 3),
            "frac": round(bound_ms / ms, 4)}


def view_cost(model, cs) -> int:
    """A view's work estimate: its intersections (one render)."""
    from msplat_b200 import _lib, engine
    engine.render(model, cs)
    return int(_lib.load().msplat_num_intersections())


def balanced_views(costs, world: int) -> list:
    """The batch's views split into `world` groups of len(costs) / world,
    balancing the summed cost: longest first, each to the least-loaded group
    with room (ties to the lower index).  Every rank computes the same
    split from the same costs; which rank trains which view does not change
    the step (the exchange sums every view's gradients)."""
    per = len(costs) // world
    groups = [[] for _ in range(world)]
    loads = [0] * world
    for v in sorted(range(len(costs)), key=lambda v: (-costs[v], v)):
        r = min((q for q in range(world) if len(groups[q]) < per), key=lambda q: (loads[q], q))
        groups[r].append(v)
        loads[r] += costs[v]
    return [sorted(gr) for gr in groups]


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
    assign = balanced_views([view_cost(model, cs) for cs in setups], world)
    mine = assign[rank]
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
    ex_ms = ex_alone_ms = None
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
        # third pass: the exchange alone, every rank starting it together
        # (device idle and a barrier before each), so the time holds no wait
        # for a slower rank's views
        evs = []
        for _ in range(steps):
            model.step_count += 1
            multigpu.accumulate_views(dist.ops, model, cams, tgts, dist.grad, dist.compact)
            torch.cuda.synchronize()
            dist.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            dist.apply(cams[0])
            b.record(stream)
            evs.append((a, b))
            torch.cuda.synchronize()
        ex_alone_ms = dist.max_over_ranks(float(np.mean([a.elapsed_time(b) for a, b in evs])))
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
                   "view_assignment": "views split over the ranks by intersection count "
                                      "(longest first to the least-loaded rank)",
                   "l2": "inputs larger than L2 (parameters and moments ~4.2 GB)",
                   "parallelism": "single GPU" if world == 1 else (
                       f"dp{world}: replicated Gaussians, " + (
                           "peer-memory reduce + Adam + parameter write-back"
                           + (" (compact v_rgb exchange)" if dist.compact else "")
                           if args.dp_mode == "peer" else "NCCL all-reduce, Adam on every replica"))},
        "exchange": None if dist is None else {
            "mode": args.dp_mode, "ms_per_step": round(ex_ms, 3),
            "ms_aligned": round(ex_alone_ms, 3),
            "roofline_aligned": exchange_roofline(model.n, world, dist.compact, args.dp_mode,
                                                  ex_alone_ms),
            "nvlink_bytes_per_rank": xbytes,
            "gbs_per_rank": round(xbytes / (ex_ms / 1000.0) / 1e9, 1) if ex_ms else None,
            "roofline": exchange_roofline(model.n, world, dist.compact, args.dp_mode, ex_ms),
            "timing": "CUDA events around the exchange + Adam of each step (includes waiting "
                      "for the slowest rank's gradients), mean over steps, max over ranks; "
                      "ms_aligned: the same with the device idle and a barrier before each "
                      "exchange (no wait for a slower rank)"},
        "intersections_last_view": n_isect,
        "gpu_launches": launches, "clocks": clk,
    }
    if dist is not None:
        if dist.mode == "peer" and dist.peer_errors():
            raise RuntimeError("peer-memory optimiser reported a timed-out wait: run invalid")
        dist.shutdown()
    return result


def profile_step(args) -> dict:
    """One training step (C1, or --profile-config) after W warm-up steps, alone between
    cudaProfilerStart and cudaProfilerStop (ncu --profile-from-start off)."""
    import torch
    from msplat_b200 import engine
    torch.cuda.set_device(0)
    engine.bind_stream()
    g, setups, gts, model = build_workload(args.profile_config)
    ncam = len(setups)
    for s in range(args.warmup):
        engine.train_step(model, setups[s % ncam], gts[s % ncam])
    torch.cuda.synchronize()
    view = args.warmup % ncam
    torch.cuda.profiler.start()
    engine.train_step(model, setups[view], gts[view])
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    return {"build_hash": build_hash(), "view": view, "warmup": args.warmup,
            "config": args.profile_config}


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.summarize_ncu:
        print(summarize_ncu(args.summarize_ncu, args.hash_file))
        return
    if args.profile_step:
        print(json.dumps(profile_step(args)), flush=True)
        return
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
        if args.config != "C1":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable":
                                  f"the reference arm times the headline C1 workload only "
                                  f"({args.config} requested)"}), flush=True)
            return
        res = run_reference(args, rank, world)
    else:
        # one process group for the whole run: the headline leg and the C4
        # leg share it (a group destroyed and created again between them
        # could meet ranks still drawing the C4 scene with the old group's
        # NCCL bootstrap address)
        group = shared_group(rank, world)
        res = run_ours(args, rank, world, args.config)
        if args.config == "C1" and not args.no_c4:
            res["c4"] = c4_leg(args, rank, world)
        if group:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)


def shared_group(rank: int, world: int) -> bool:
    """The default NCCL process group for world > 1 (127.0.0.1 rendezvous
    from torchrun's environment), created once here so that every leg's
    DataParallel uses it instead of creating and destroying its own; a
    10-minute timeout bounds the wait for a rank still drawing a scene."""
    if world <= 1:
        return False
    import datetime

    import torch
    import torch.distributed as dist
    if dist.is_initialized():
        return False
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    dist.init_process_group(backend="nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=600),
                            device_id=torch.device("cuda", torch.cuda.current_device()))
    return True


def c4_leg(args, rank: int, world: int) -> dict:
    """BASELINE.json config 4 beside the headline line: the batched-view step
    (8 views of 1920x1080 per step, 6M Gaussians) on the same N GPUs, with
    the same K and W; its scenes are drawn once per host and kept in a cache
    directory (MSPLAT_BENCH_SCENE_CACHE, else one under the system temporary
    directory) so that the runs at several N reuse them."""
    import gc

    import torch
    from msplat_b200 import _lib
    gc.collect()
    torch.cuda.empty_cache()
    _lib.load().cleanup_msplat_cuda()
    if not os.environ.get("MSPLAT_BENCH_SCENE_CACHE"):
        import tempfile
        os.environ["MSPLAT_BENCH_SCENE_CACHE"] = os.path.join(tempfile.gettempdir(),
                                                              "msplat_bench_scenes")
    if world not in (1, 2, 4, 8):
        return {"skipped": f"C4 splits its batch of 8 views over 1, 2, 4 or 8 GPUs, not {world}"}
    r = run_c4(args, rank, world)
    keep = ("value", "unit", "ms_per_step", "steps", "warmup", "scaling", "exchange",
            "gpu_launches", "clocks")
    out = {k: r[k] for k in keep if k in r}
    out["metric"] = r["metric"]
    out["workload"] = r["config"]["workload"]
    out["views_per_gpu"] = r["config"]["views_per_gpu"]
    out["parallelism"] = r["config"]["parallelism"]
    return out


from ctypes import byref as C_byref, c_char_p as C_char_p, c_double as C_double, c_int as C_int  # noqa: E402
from ctypes import c_float as C_float, c_ulonglong as C_ulonglong, c_void_p as C_void_p  # noqa: E402

if __name__ == "__main__":
    main()
