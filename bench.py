"""Benchmark: DINOv3 ViT-S+/16 forward, 224x224, batch 64 per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one process per GPU)

Our arm. A step is one forward of 64 images per GPU (one CUDA graph replay). Every rank loads its
own model replica (data-parallel replicas, no collective on the forward; NCCL only for the
barrier and the max-over-ranks of the timings).
  value   images/s over all ranks with the inputs already resident in HBM: K steps timed with CUDA
          events on the model's stream, the L2 flushed (a 160 MiB memset, more than the 126 MB
          L2) between timed steps,
          value = N * 64 * K / max over ranks of the summed step time.
  e2e     the same through the public API with host buffers, host<->device copies of every step
          inside the timed region: the serving calls dv3_submit / dv3_wait with two steps in
          flight (pinned host input and output per step; the library overlaps one step's upload
          and another's download with the forward in between), host clock between device
          synchronisations, max over ranks. `e2e_sync` beside it: one blocking dv3_forward per
          step (upload, forward and download in series), CUDA events on the model's stream.
  roofline the dominant kernel (gate/up GEMM + SwiGLU, 46.5 % of the FLOPs): its algorithmic FLOPs
          per launch / its average launch time, measured inside whole forwards after the timed
          region (dv3_profile_forward: CUDA events on the model's stream around graphs of the
          first j launches of the plan, `--profile-iters` replays each with the L2 flushed
          before each; launch j takes T(j) - T(j-1), so the launch times add up to a forward and
          keep the production graph's overlap of each kernel's set-up with the previous
          kernel's tail), against the measured burst bf16/f16 dense peak (MEASURED_PEAKS.json
          bf16_tflops; `frac_of_sustained` beside it). `per_kernel` lists every kernel of the
          plan the same way: FLOPs and algorithmic bytes per launch, the measured time, the
          floor max(FLOPs / tensor peak, bytes / HBM bandwidth) and floor / time. `traffic` comes
          from the committed ncu summary in profiles/ when it lists the kernel.
  cpu_baseline the float64 CPU oracle (C restatement of the reference's own float64 forward,
          tests/support/reference.rs) on this host, OpenMP over images, rank 0 at N = 1 only.
Reference arm (--impl reference): the same CPU oracle with all host threads, rank 0 only; a
step is one forward of as many images as host threads (a bounded sample of the batch-64 step).
--serve: BASELINE config 4, seeded call sizes uniform over 1..64 images from pinned host memory,
synchronous dv3_forward calls and dv3_submit / dv3_wait two calls deep, aggregate images/s and
per-call p50 / p99 latency (host clock).
--forward-only [--batch B]: run the plan's forwards without timing (for ncu launch lists).
--copies: the end-to-end step's host<->device transfers alone (no forward), per rank, to show how
much copy bandwidth the host gives N GPUs at once.
--ops: BASELINE config 3, every kernel entry point (include/dinov3_kernels.h) alone at batch 64
(12,864 token rows), inputs N(0,1) and weights N(0,1)/sqrt(K), with cold L2: each timed graph
cycles over enough copies of the operands to exceed twice the L2, so no launch finds its inputs
cached (a warm figure, one set of operands repeated, is given beside it).
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (os.path.join(ROOT, "dinov3-loom_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

BATCH = 64
METRIC = "images/sec (224², ViT-S+/16) at batch 64 on 1/2/4/8 B200; p50 batch-1 latency"
UNIT = "images/s"
GFLOP_PER_IMAGE = 12.2415
R64, P64 = 201 * BATCH, 196 * BATCH  # token rows and patch rows at batch 64
FLUSH_BYTES = 160 << 20  # written between timed steps: more than the B200's 126 MB L2


def kernel_work(name: str, b: int = BATCH, last: bool = False):
    """(FLOPs, algorithmic bytes) of one launch of kernel `name` over b images: FLOPs 2*M*K*N per
    GEMM and 4*T^2*d per attention slice; bytes = every input and weight read once, every output
    written once, the residual read and written (the minimum HBM traffic)."""
    r, p, d = 201 * b, 196 * b, 384
    f16, f32 = 2, 4
    if name == "patchify":
        return 0.0, b * 3 * 224 * 224 * f32 + p * 768 * f16 + b * 5 * d * f16
    if name == "gemm_patch_embed":
        return 2.0 * p * 768 * d, (p * 768 + d * 768 + p * d) * f16 + d * f32
    if name in ("layernorm_f16", "layernorm_f32out"):
        return 0.0, r * d * f16 + r * d * (f32 if name == "layernorm_f32out" else f16) + 2 * d * f32
    if name == "layernorm_rowstat":  # folded LayerNorm: (rstd, -mean rstd) and aux row per row
        return 0.0, r * d * f16 + r * (2 * f32 + 16 * f16)
    if name in ("gemm_qkv_rope", "gemm_qkv_rope_folded"):
        fold = r * 2 * f32 + (r + 1152) * 16 * f16 if name.endswith("folded") else 0
        return 2.0 * r * d * 1152, ((r * d + 1152 * d + r * 1152) * f16 + (1152 + 2 * 196 * 64) * f32
                                    + fold)
    if name == "attention":
        return 4.0 * 201 * 201 * 64 * 6 * b, (r * 1152 + r * d) * f16
    if name in ("gemm_o_resid", "gemm_o_resid_layernorm", "gemm_o_resid_rowstat"):
        ln = name.endswith("layernorm")
        stats = r * (2 * f32 + 16 * f16) if name.endswith("rowstat") else 0
        return 2.0 * r * d * d, ((r * d + d * d + 2 * r * d + (r * d if ln else 0)) * f16
                                 + 4 * d * f32 + stats)
    if name in ("gemm_gateup_swiglu", "gemm_gateup_swiglu_folded"):
        fold = r * 2 * f32 + (r + 3072) * 16 * f16 if name.endswith("folded") else 0
        return 2.0 * r * d * 3072, (r * d + 3072 * d + r * 1536) * f16 + 3072 * f32 + fold
    if name in ("gemm_down_resid", "gemm_down_resid_layernorm", "gemm_down_resid_rowstat"):
        ln = name.endswith("layernorm")
        out = (r * d * (f32 if last else f16)) if ln else 0
        stats = r * (2 * f32 + 16 * f16) if name.endswith("rowstat") else 0
        return 2.0 * r * 1536 * d, (r * 1536 + d * 1536 + 2 * r * d) * f16 + out + 4 * d * f32 + stats
    return 0.0, 0.0


def roofline_entry(name, ms, flops, nbytes, peaks):
    """Floor = max(FLOPs / burst tensor peak, bytes / HBM copy bandwidth); frac = floor / time."""
    t_tensor = flops / (peaks["bf16_tflops"] * 1e12) * 1e3 if flops else 0.0
    t_hbm = nbytes / (peaks["hbm_gbs"] * 1e9) * 1e3
    floor = max(t_tensor, t_hbm)
    return {"kernel": name, "us": ms * 1e3, "gflop": flops / 1e9, "mbytes": nbytes / 1e6,
            "bound": "tensor" if t_tensor >= t_hbm else "hbm",
            "tflops": flops / ms / 1e9 if flops else 0.0, "gbs": nbytes / ms / 1e6,
            "floor_us": floor * 1e3, "frac": floor / ms}


FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
WORKLOAD = "DINOv3 ViT-S+/16 forward, 224x224, batch 64 per GPU (config 2), fp16 weights/activations, fp32 accumulate"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--profile-iters", type=int, default=20)
    ap.add_argument("--cpu-budget-s", type=float, default=20.0)
    ap.add_argument("--forward-only", action="store_true",
                    help="profiling driver: load, stage one batch, replay warmup+steps forwards, exit")
    ap.add_argument("--batch", type=int, default=BATCH, help="images per forward (--forward-only)")
    ap.add_argument("--serve", action="store_true",
                    help="serving measurement (BASELINE config 4): calls of seeded random size "
                         "1..64 from pinned host memory, synchronous and two-deep pipelined")
    ap.add_argument("--serve-images", type=int, default=8192,
                    help="images over all GPUs in the serving measurement")
    ap.add_argument("--copies", action="store_true",
                    help="the end-to-end step's host<->device copies alone (38.5 MB up, 19.8 MB "
                         "down per GPU per step, pinned buffers, both directions at once): the "
                         "bandwidth the host side gives every rank")
    ap.add_argument("--ops", action="store_true",
                    help="per-op microbenchmark (BASELINE config 3): every kernel entry point "
                         "alone at batch 64, cold and warm L2")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {k: float(p[k]) for k in FALLBACK_PEAKS}, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


def committed_traffic(kernel: str):
    """dram read+write bytes per launch of `kernel` at batch 64 from the committed ncu summary
    (lines `traffic_bytes_per_launch <kernel> <bytes>` in profiles/*.md), else None."""
    pdir = os.path.join(ROOT, "profiles")
    if not os.path.isdir(pdir):
        return None
    for name in sorted(os.listdir(pdir)):
        if not name.endswith(".md"):
            continue
        for line in open(os.path.join(pdir, name)):
            m = re.match(r"\s*traffic_bytes_per_launch\s+(\S+)\s+([0-9.eE+]+)", line)
            if m and m.group(1) == kernel:
                return float(m.group(2))
    return None


class Clocks:
    """nvidia-smi samples of one GPU during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.device), "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def host_threads() -> int:
    """Every core this process may run on (torchrun sets OMP_NUM_THREADS=1 for its workers, so
    the OpenMP default is not used)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_oracle_throughput(images, budget_s: float, threads: int | None = None):
    """images/s of the float64 C oracle on this host; returns (value, cores, sample, step_times)."""
    import numpy as np

    import ref_c
    from dinov3_b200 import synth

    threads = threads or host_threads()
    model = ref_c.Model(synth.weights(0, "baseline"))
    n = max(1, threads)
    sample = np.ascontiguousarray(images[:n] if len(images) >= n else np.resize(images, (n,) + images.shape[1:]))
    t0 = time.perf_counter()
    model.forward(sample, threads=threads)
    dt = time.perf_counter() - t0
    return n / dt, threads, n, dt, model, sample


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import numpy as np

    import ref_c
    from dinov3_b200 import synth

    threads = host_threads()
    images = synth.images(1000, threads)
    model = ref_c.Model(synth.weights(0, "baseline"))
    # One step = one float64 forward of `threads` images (one per thread), OpenMP over images.
    t0 = time.perf_counter()
    model.forward(images, threads=threads)
    est = time.perf_counter() - t0
    steps = max(1, min(args.steps, int(args.cpu_budget_s * 6 // max(est, 1e-3))))
    # the same warm-up count as our arm, within the CPU time budget (the estimate above was a
    # first warm-up forward already)
    warm = max(0, min(args.warmup - 1, int(args.cpu_budget_s * 2 // max(est, 1e-3))))
    for _ in range(warm):
        model.forward(images, threads=threads)
    t0 = time.perf_counter()
    for _ in range(steps):
        model.forward(images, threads=threads)
    dt = time.perf_counter() - t0
    value = threads * steps / dt
    cpu = {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
           "sample": f"{steps} steps x {threads} seeded 224x224 images (batch-64 workload sample), "
                     f"float64 C oracle of tests/support/reference.rs, OpenMP over images "
                     f"({steps} of the requested {args.steps} steps fit the CPU time budget)"}
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": steps, "warmup": warm + 1, "ms_per_step": 1000 * dt / steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "batch_per_gpu": threads, "images_per_step": threads,
                       "sample_of": f"the batch-{BATCH} step: one float64 forward of {threads} "
                                    f"images (one per host thread) per step",
                       "parallelism": f"replicas{args.gpus}"},
            "cpu_baseline": cpu,
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "host": cpu_model()}
    print(json.dumps(line), flush=True)


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip() + f" x{os.cpu_count()}"
    except Exception:
        pass
    return f"unknown x{os.cpu_count()}"


def kernel_table(prof, peaks):
    """Per kernel of the plan: launches, average time, algorithmic work per launch and its roofline
    (roofline_entry); the time shares; the gate/up GEMM's entry."""
    total_ms = sum(ms for _, ms in prof)
    agg = {}
    n_down = sum(1 for n, _ in prof if n.startswith("gemm_down"))
    seen_down = 0
    for name, ms in prof:
        last = False
        if name.startswith("gemm_down"):
            seen_down += 1
            last = seen_down == n_down
        flops, nbytes = kernel_work(name, BATCH, last)
        a = agg.setdefault(name, [0, 0.0, 0.0, 0.0])
        a[0] += 1
        a[1] += ms
        a[2] += flops
        a[3] += nbytes
    table, share = [], {}
    for name, (n, ms, flops, nbytes) in agg.items():
        e = roofline_entry(name, ms / n, flops / n, nbytes / n, peaks)
        e["launches"] = n
        e["traffic"] = committed_traffic(name)
        table.append(e)
        share[name] = round(ms / total_ms, 4)
    gate = next(e for e in table if e["kernel"].startswith("gemm_gateup_swiglu"))
    return table, share, gate


def run_ours(args):
    import numpy as np
    import torch

    import dinov3_b200 as dv
    from dinov3_b200 import synth
    from dinov3_b200.replicas import Replicas

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    # one replica per GPU; NCCL only for the barriers around timed regions and the max over ranks
    reps = Replicas("nccl", timeout_s=120)
    barrier, max_over_ranks = reps.barrier, reps.max

    wdir = tempfile.mkdtemp(prefix=f"dv3_bench_{rank}_")
    wpath = synth.write_weights(os.path.join(wdir, "w.safetensors"), seed=0, flavor="baseline")
    model = dv.DINOv3.load(wpath, dv.Options(local, BATCH))
    images = synth.images(1000, BATCH, first=reps.first_image(BATCH))  # this rank's slice
    stream = torch.cuda.ExternalStream(model.stream, device=torch.device("cuda", local))
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    n_img = BATCH * 3 * 224 * 224

    class _Dev:
        def __init__(self, ptr, n):
            self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3}

    staged = torch.as_tensor(_Dev(model.input_buffer, n_img), device="cuda")
    staged.copy_(torch.from_numpy(images).reshape(-1))
    torch.cuda.synchronize()

    if args.serve:
        run_serving(args, model, images, reps)
        return

    if args.forward_only:
        b = max(1, min(args.batch, BATCH))
        for _ in range(args.warmup + args.steps):
            model.run(b)
        model.synchronize()
        print(json.dumps({"forward_only": True, "batch": b, "forwards": args.warmup + args.steps,
                          "launches_per_forward": model.launches_per_forward(b)}), flush=True)
        model.close()
        return

    # ---- device-resident throughput ----
    launches = model.launches_per_forward(BATCH)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            model.run(BATCH)
        model.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        barrier()
        clocks = Clocks(local)
        with clocks:
            wall0 = time.perf_counter()
            for s, e in ev:
                flush.zero_()  # evict L2 between timed steps (outside the events)
                s.record(stream)
                model.run(BATCH)
                e.record(stream)
            model.synchronize()
            wall = time.perf_counter() - wall0
        barrier()
    total_ms = sum(s.elapsed_time(e) for s, e in ev)
    total_ms = max_over_ranks(total_ms)
    value = reps.throughput(BATCH * args.steps, total_ms / 1000.0)

    # ---- end to end through the public API (pinned host buffers) ----
    pin_in = torch.from_numpy(images).pin_memory()
    pin_out = torch.empty((BATCH, 201, 384), dtype=torch.float32).pin_memory()
    e2e_steps = max(3, min(args.steps, 200))
    for _ in range(max(3, args.warmup // 4)):
        model.forward(pin_in, out=pin_out)
    ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(e2e_steps)]
    barrier()
    for s, e in ev2:
        with torch.cuda.stream(stream):
            flush.zero_()
        s.record(stream)
        model.forward(pin_in, out=pin_out)
        e.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_sync_ms = max_over_ranks(sum(s.elapsed_time(e) for s, e in ev2))
    e2e_sync = reps.throughput(BATCH * e2e_steps, e2e_sync_ms / 1000.0)
    assert np.isfinite(pin_out.numpy()).all()

    # ---- end to end, pipelined through the serving API (dv3_submit / dv3_wait) ----
    # Two submissions in flight, each with its own pinned input and output: the upload of step
    # i overlaps the forward of step i-1 and the download of step i-2 (three streams inside the
    # library). Every step's host->device copy and device->host read are inside the timed
    # region; the L2 is flushed on the compute stream before each step's forward (the flush
    # time is included). Timed by the host clock between two device synchronisations, max over
    # ranks.
    pins_in = [pin_in, torch.from_numpy(images).pin_memory()]
    pins_out = [pin_out, torch.empty((BATCH, 201, 384), dtype=torch.float32).pin_memory()]

    def run_pipelined(steps: int) -> None:
        tickets = []
        for i in range(steps):
            if len(tickets) == 2:
                model.wait(tickets.pop(0))
            with torch.cuda.stream(stream):
                flush.zero_()
            tickets.append(model.submit(pins_in[i % 2], pins_out[i % 2]))
        for t in tickets:
            model.wait(t)

    run_pipelined(4)
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    run_pipelined(e2e_steps)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1000.0)
    barrier()
    e2e_value = reps.throughput(BATCH * e2e_steps, e2e_ms / 1000.0)
    assert all(np.isfinite(o.numpy()).all() for o in pins_out)

    # ---- batch-1 latency (p50), device-resident and end to end ----
    lat_dev, lat_e2e = [], []
    one_in = torch.from_numpy(images[:1]).pin_memory()
    one_out = torch.empty((1, 201, 384), dtype=torch.float32).pin_memory()
    for i in range(60):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        model.run(1)
        e.record(stream)
        model.synchronize()
        t0 = time.perf_counter()
        model.forward(one_in, out=one_out)
        t1 = time.perf_counter()
        if i >= 10:
            lat_dev.append(s.elapsed_time(e))
            lat_e2e.append((t1 - t0) * 1000)

    # ---- per-kernel times inside whole forwards (L2 flushed before each) and rooflines ----
    prof = model.profile_forward(BATCH, args.profile_iters, FLUSH_BYTES)
    peaks, peak_src = load_peaks()
    per_kernel, kernel_share, gate = kernel_table(prof, peaks)
    gate_ms = gate["us"] / 1e3
    achieved = gate["tflops"]

    steps_launches = launches * args.steps
    model.synchronize()
    model.close()

    cpu = None
    cpu_single = None
    if rank == 0 and world == 1:
        value_cpu, cores, n, dt, model_cpu, sample = cpu_oracle_throughput(images, args.cpu_budget_s)
        cpu = {"value": value_cpu, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"{n} seeded 224x224 images of the batch-64 workload, float64 C oracle of "
                         f"tests/support/reference.rs, OpenMP over images, {dt:.1f} s"}
        # The reference's own CPU path is single-threaded (matrixmultiply without its threading
        # feature): the same oracle on one image with one thread.
        t0 = time.perf_counter()
        model_cpu.forward(np.ascontiguousarray(sample[:1]), threads=1)
        dt1 = time.perf_counter() - t0
        cpu_single = {"value": 1.0 / dt1, "unit": UNIT, "cores": 1, "kind": "port",
                      "sample": f"1 seeded 224x224 image, float64 C oracle, 1 thread, {dt1:.2f} s"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "global_batch": BATCH * world, "batch_per_gpu": BATCH,
                       "seq_len": 201, "parallelism": f"replicas{world}",
                       "weights": "seeded random-init (baseline flavour: trunc-normal 0.02, biases 0, LN 1/0, LayerScale 0.1)",
                       "l2": "flushed between timed steps (160 MiB memset; L2 is 126 MB)"},
            "e2e": {"value": e2e_value, "unit": UNIT,
                    "h2d_bytes_per_step": BATCH * 3 * 224 * 224 * 4,
                    "d2h_bytes_per_step": BATCH * 201 * 384 * 4 + 8,
                    "api": "dv3_submit/dv3_wait, two steps in flight (copies overlap the "
                           "neighbouring steps' forwards), host clock, L2 flushed per step",
                    "steps": e2e_steps},
            "e2e_sync": {"value": e2e_sync, "unit": UNIT,
                         "api": "dv3_forward, one blocking call per step (upload, forward, "
                                "download in series), CUDA events on the model's stream"},
            "gpu_launches": steps_launches,
            "roofline": {"kernel": gate["kernel"], "bound": "tensor", "achieved": achieved,
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": achieved / peaks["bf16_tflops"],
                         "frac_of_sustained": achieved / peaks["bf16_tflops_sustained"],
                         "peak_source": f"{peak_src} bf16_tflops (burst; of measured)",
                         "traffic": committed_traffic(gate["kernel"]),
                         "algorithmic_flops": gate["gflop"] * 1e9,
                         "algorithmic_bytes": gate["mbytes"] * 1e6, "avg_launch_ms": gate_ms,
                         "timing": f"dv3_profile_forward: CUDA events on the model's stream "
                                   f"around graphs of the plan's first j launches, "
                                   f"{args.profile_iters} replays each, L2 flushed before each; "
                                   "launch j = T(j) - T(j-1)",
                         "profiled_forward_ms": sum(e["us"] * e["launches"]
                                                    for e in per_kernel) / 1e3,
                         "per_kernel": per_kernel},
            "cpu_baseline": cpu,
            "cpu_baseline_single": cpu_single,
            "p50_batch1_latency_ms": {"device": statistics.median(lat_dev), "e2e": statistics.median(lat_e2e)},
            "tflops_whole_forward": value / world * GFLOP_PER_IMAGE / 1000.0,
            "kernel_time_share": kernel_share,
            "clocks": clocks.summary(),
            "wall_s_timed_region": wall,
        }
        print(json.dumps(line), flush=True)
    reps.close()


def run_serving(args, model, images, reps):
    """each rank serves its share of `--serve-images` images in calls of seeded
    uniform random size 1..64, from pinned host memory into pinned host memory, timed on the
    host clock per call. Two passes: synchronous dv3_forward per call, then dv3_submit with two
    calls in flight (a call is submitted, the call two before it is waited). Rank 0 prints one
    JSON line: aggregate images/s over all ranks (images / max wall time) and per-call p50/p99."""
    import numpy as np
    import torch

    rank, world = reps.rank, reps.world
    barrier, max_over_ranks = reps.barrier, reps.max
    rng = np.random.default_rng(4 + rank)
    share = reps.share(args.serve_images)
    sizes = []
    while sum(sizes) < share:
        sizes.append(int(min(rng.integers(1, BATCH + 1), share - sum(sizes))))
    pin_in = torch.from_numpy(images).pin_memory()
    outs = [torch.empty((BATCH, 201, 384), dtype=torch.float32).pin_memory() for _ in range(3)]
    # warm the CUDA graphs of every batch size used, for both serving slots
    for k in sorted(set(sizes)):
        model.forward(pin_in[:k], out=outs[0][:k])
        for slot in range(2):
            model.wait(model.submit(pin_in[:k], outs[slot][:k]))

    def percentile(v, q):
        return float(np.percentile(np.asarray(v), q))

    results = {}
    for mode in ("sync", "pipelined"):
        lat = []
        barrier()
        t_start = time.perf_counter()
        if mode == "sync":
            for k in sizes:
                t0 = time.perf_counter()
                model.forward(pin_in[:k], out=outs[0][:k])
                lat.append((time.perf_counter() - t0) * 1000)
        else:
            pending = []  # (ticket, submit time)
            for i, k in enumerate(sizes):
                if len(pending) == 2:
                    tk, ts = pending.pop(0)
                    model.wait(tk)
                    lat.append((time.perf_counter() - ts) * 1000)
                ts = time.perf_counter()
                pending.append((model.submit(pin_in[:k], outs[i % 3][:k]), ts))
            for tk, ts in pending:
                model.wait(tk)
                lat.append((time.perf_counter() - ts) * 1000)
        wall = time.perf_counter() - t_start
        wall_max = max_over_ranks(wall)
        results[mode] = {"images_per_s": args.serve_images / wall_max,
                         "p50_ms": percentile(lat, 50), "p99_ms": percentile(lat, 99),
                         "calls_per_gpu": len(sizes), "wall_s": wall_max}
    if rank == 0:
        print(json.dumps({
            "metric": "serving: aggregate images/s and per-call latency, calls of 1..64 images (config 4)",
            "value": results["pipelined"]["images_per_s"], "unit": UNIT, "n_gpus": world,
            "higher_is_better": True, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "BASELINE config 4: seeded uniform call sizes 1..64, pinned host "
                                   "buffers in and out, every call's full output read back",
                       "images": args.serve_images, "parallelism": f"replicas{world}"},
            "sync": results["sync"], "pipelined": results["pipelined"]}), flush=True)
    model.close()
    reps.close()


def run_ops(args):
    """each kernel entry point of include/dinov3_kernels.h alone at batch 64
    (12,864 token rows, 12,544 patch rows), activations N(0,1), weights N(0,1)/sqrt(K). Each op's
    launches are captured K times into a CUDA graph that cycles over S copies of its operands,
    S x (operand bytes) > 2 x L2 (cold: every launch reads operands the L2 no longer holds), and
    over one copy (warm); one replay after a warm-up replay is timed with CUDA events on the
    launching stream, time per launch = interval / K. Rank 0 only; prints one JSON line."""
    import numpy as np
    import torch

    from dinov3_b200 import _lib

    rank, world, local = dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    lib = _lib.load()
    peaks, peak_src = load_peaks()
    l2 = 126 << 20
    gen = torch.Generator(device=dev)
    gen.manual_seed(3)
    r, p, d = R64, P64, 384
    st = torch.zeros(2, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def randn(shape, scale=1.0, dtype=torch.float16):
        return (torch.randn(shape, generator=gen, device=dev) * scale).to(dtype)

    def empty(shape, dtype=torch.float16):
        return torch.empty(shape, dtype=dtype, device=dev)

    def vec(n, lo=-0.1, hi=0.1):
        return torch.rand(n, generator=gen, device=dev) * (hi - lo) + lo

    ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
    w = {"patch": randn((d, 768), 768 ** -0.5), "qkv": randn((1152, d), d ** -0.5),
         "o": randn((d, d), d ** -0.5), "gateup": randn((3072, d), d ** -0.5),
         "down": randn((d, 1536), 1536 ** -0.5)}
    v = {"bias": vec(3072), "lam": vec(d, 0.05, 0.2), "gamma": vec(d, 0.5, 1.5), "beta": vec(d),
         "cos": vec(196 * 64, -1, 1), "sin": vec(196 * 64, -1, 1), "prefix": vec(5 * d, -1, 1)}

    def check(rc):
        if rc != 0:
            raise RuntimeError(_lib.last_error())

    def time_op(name, make, launch, flops, nbytes, set_bytes):
        sets = [make() for _ in range(max(2, -(-2 * l2 // set_bytes) + 1))]
        with torch.cuda.stream(stream):
            for ops in sets:  # validates the arguments and configures the kernel outside capture
                check(launch(ops, stream.cuda_stream))
        stream.synchronize()
        out = {}
        for mode, use in (("cold", sets), ("warm", sets[:1])):
            k = len(use) * max(2, -(-24 // len(use)))
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                cs = torch.cuda.current_stream().cuda_stream
                for i in range(k):
                    check(launch(use[i % len(use)], cs))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                g.replay()
                e0.record(stream)
                g.replay()
                e1.record(stream)
            e1.synchronize()
            out[mode] = e0.elapsed_time(e1) / k
            del g
        if st.cpu().tolist() != [0, 0]:
            raise RuntimeError(f"{name}: device status {st.cpu().tolist()}")
        del sets
        torch.cuda.empty_cache()
        e = roofline_entry(name, out["cold"], flops, nbytes, peaks)
        e["warm_us"] = out["warm"] * 1e3
        e["operand_sets"] = -(-2 * l2 // set_bytes) + 1
        return e

    f16b, f32b = 2, 4
    results = []
    results.append(time_op(
        "patchify", lambda: (randn((BATCH, 3, 224, 224), dtype=torch.float32), empty((p, 768)),
                             empty((r, d))),
        lambda o, s: lib.dv3k_patchify(ptr(o[0]), BATCH, ptr(v["prefix"]), ptr(o[1]), ptr(o[2]),
                                       ptr(st), s),
        *kernel_work("patchify"), BATCH * 150528 * f32b + p * 768 * f16b + r * d * f16b))
    results.append(time_op(
        "gemm_patch_embed", lambda: (randn((p, 768)), empty((r, d))),
        lambda o, s: lib.dv3k_patch_embed(ptr(o[0]), p, ptr(w["patch"]), ptr(v["bias"]), ptr(o[1]),
                                          ptr(st), s),
        *kernel_work("gemm_patch_embed"), (p * 768 + r * d) * f16b))
    results.append(time_op(
        "layernorm_f16", lambda: (randn((r, d)), empty((r, d))),
        lambda o, s: lib.dv3k_layernorm_f16(ptr(o[0]), r, ptr(v["gamma"]), ptr(v["beta"]),
                                            ptr(o[1]), s),
        *kernel_work("layernorm_f16"), 2 * r * d * f16b))
    results.append(time_op(
        "layernorm_f32out", lambda: (randn((r, d)), empty((r, d), torch.float32)),
        lambda o, s: lib.dv3k_layernorm_f32out(ptr(o[0]), r, ptr(v["gamma"]), ptr(v["beta"]),
                                               ptr(o[1]), s),
        *kernel_work("layernorm_f32out"), r * d * (f16b + f32b)))
    results.append(time_op(
        "gemm_qkv_rope", lambda: (randn((r, d)), empty((r, 1152))),
        lambda o, s: lib.dv3k_qkv_rope(ptr(o[0]), r, ptr(w["qkv"]), ptr(v["bias"]), ptr(v["cos"]),
                                       ptr(v["sin"]), ptr(o[1]), ptr(st), s),
        *kernel_work("gemm_qkv_rope"), r * (d + 1152) * f16b))
    results.append(time_op(
        "attention", lambda: (randn((r, 1152)), empty((r, d))),
        lambda o, s: lib.dv3k_attention(ptr(o[0]), r, ptr(o[1]), ptr(st), s),
        *kernel_work("attention"), r * (1152 + d) * f16b))
    for k, wname in ((384, "o"), (1536, "down")):
        base = "gemm_o_resid" if k == 384 else "gemm_down_resid"
        results.append(time_op(
            base, lambda k=k: (randn((r, k)), randn((r, d))),
            lambda o, s, k=k, wname=wname: lib.dv3k_matmul_resid(
                ptr(o[0]), r, k, ptr(w[wname]), ptr(v["bias"]), ptr(v["lam"]), ptr(o[1]), ptr(st), s),
            *kernel_work(base), r * (k + d) * f16b))
        results.append(time_op(
            base + "_layernorm", lambda k=k: (randn((r, k)), randn((r, d)), empty((r, d))),
            lambda o, s, k=k, wname=wname: lib.dv3k_matmul_resid_layernorm(
                ptr(o[0]), r, k, ptr(w[wname]), ptr(v["bias"]), ptr(v["lam"]), ptr(o[1]),
                ptr(v["gamma"]), ptr(v["beta"]), ptr(o[2]), None, ptr(st), s),
            *kernel_work(base + "_layernorm"), r * (k + 2 * d) * f16b))
    results.append(time_op(
        "gemm_gateup_swiglu", lambda: (randn((r, d)), empty((r, 1536))),
        lambda o, s: lib.dv3k_matmul_swiglu(ptr(o[0]), r, ptr(w["gateup"]), ptr(v["bias"]),
                                            ptr(o[1]), ptr(st), s),
        *kernel_work("gemm_gateup_swiglu"), r * (d + 1536) * f16b))
    # the folded-LayerNorm forms the plan uses at this batch size: the residual GEMMs leave the
    # row statistics (rstd, -mean rstd) and an f16 aux row; QKV and gate/up read x and add the
    # rank-2 correction in one more K=16 step from the weight aux rows
    waux = {"qkv": randn((1152, 16), 0.1), "gateup": randn((3072, 16), 0.1)}
    stats = lambda: (torch.stack([vec(r, 0.5, 1.5), vec(r)], 1).contiguous(),  # noqa: E731
                     randn((r, 16), 0.1))
    results.append(time_op(
        "layernorm_rowstat",
        lambda: (randn((r, d)), empty((r, 2), torch.float32), empty((r, 16))),
        lambda o, s: lib.dv3k_layernorm_rowstat(ptr(o[0]), r, ptr(o[1]), ptr(o[2]), s),
        *kernel_work("layernorm_rowstat"), r * d * f16b + r * (2 * f32b + 16 * f16b)))
    results.append(time_op(
        "gemm_qkv_rope_folded", lambda: (randn((r, d)), *stats(), empty((r, 1152))),
        lambda o, s: lib.dv3k_qkv_rope_folded(ptr(o[0]), r, ptr(w["qkv"]), ptr(waux["qkv"]),
                                              ptr(o[1]), ptr(o[2]), ptr(v["cos"]), ptr(v["sin"]),
                                              ptr(o[3]), ptr(st), s),
        *kernel_work("gemm_qkv_rope_folded"), r * (d + 1152 + 16) * f16b + r * 2 * f32b))
    for k, wname in ((384, "o"), (1536, "down")):
        name = ("gemm_o_resid" if k == 384 else "gemm_down_resid") + "_rowstat"
        results.append(time_op(
            name, lambda k=k: (randn((r, k)), randn((r, d)), empty((r, 2), torch.float32),
                               empty((r, 16))),
            lambda o, s, k=k, wname=wname: lib.dv3k_matmul_resid_rowstat(
                ptr(o[0]), r, k, ptr(w[wname]), ptr(v["bias"]), ptr(v["lam"]), ptr(o[1]),
                ptr(o[2]), ptr(o[3]), ptr(st), s),
            *kernel_work(name), r * (k + d + 16) * f16b + r * 2 * f32b))
    results.append(time_op(
        "gemm_gateup_swiglu_folded", lambda: (randn((r, d)), *stats(), empty((r, 1536))),
        lambda o, s: lib.dv3k_matmul_swiglu_folded(ptr(o[0]), r, ptr(w["gateup"]),
                                                   ptr(waux["gateup"]), ptr(o[1]), ptr(o[2]),
                                                   ptr(o[3]), ptr(st), s),
        *kernel_work("gemm_gateup_swiglu_folded"), r * (d + 1536 + 16) * f16b + r * 2 * f32b))

    def splitk_pair(o, s, splits=2):
        rc = lib.dv3k_matmul_splitk(ptr(o[0]), r, ptr(w["down"]), splits, ptr(o[2]), ptr(st), s)
        return rc or lib.dv3k_splitk_reduce(ptr(o[2]), r, splits, ptr(v["bias"]), ptr(v["lam"]),
                                            ptr(o[1]), s)

    e = time_op("gemm_down_splitk2+splitk_reduce",
                lambda: (randn((r, 1536)), randn((r, d)), empty((2, r, d), torch.float32)),
                splitk_pair, *kernel_work("gemm_down_resid"), r * (1536 + d) * f16b + 2 * r * d * f32b)
    e["note"] = "two launches (split-K GEMM over 2 K slices into f32 slabs, then the reduce)"
    results.append(e)
    line = {"metric": "per-op device time at batch 64 (BASELINE config 3), cold L2",
            "unit": "us", "n_gpus": 1, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "each kernel entry point alone, 12864 token rows (12544 patch "
                                   "rows), activations N(0,1), weights N(0,1)/sqrt(K)",
                       "l2": "cold: operand copies cycled, more than twice the L2 in total"},
            "peaks": {"tflops": peaks["bf16_tflops"], "hbm_gbs": peaks["hbm_gbs"],
                      "source": f"{peak_src} (burst)"},
            "ops": results}
    print(json.dumps(line), flush=True)


def run_copies(args):
    """The transfers of one end-to-end step without the forward: every rank copies a batch-64
    input (pinned, 38.5 MB) to the GPU and a batch-64 output (19.8 MB) back to pinned memory,
    on two streams so both directions run at once, `--steps` times; host clock between device
    synchronisations, max over ranks. Rank 0 prints the aggregate and per-rank GB/s."""
    import torch

    from dinov3_b200.replicas import Replicas

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    reps = Replicas("nccl", timeout_s=120)
    up_h = torch.empty(BATCH * 3 * 224 * 224, dtype=torch.float32).pin_memory()
    down_h = torch.empty(BATCH * 201 * 384, dtype=torch.float32).pin_memory()
    up_d = torch.empty_like(up_h, device="cuda")
    down_d = torch.zeros_like(down_h, device="cuda")
    s_up, s_down = torch.cuda.Stream(), torch.cuda.Stream()

    def step():
        with torch.cuda.stream(s_up):
            up_d.copy_(up_h, non_blocking=True)
        with torch.cuda.stream(s_down):
            down_h.copy_(down_d, non_blocking=True)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    reps.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    torch.cuda.synchronize()
    dt = reps.max(time.perf_counter() - t0)
    reps.barrier()
    per_step = up_h.numel() * 4 + down_h.numel() * 4
    if rank == 0:
        print(json.dumps({
            "metric": "host<->device copy bandwidth of the end-to-end step's transfers",
            "value": world * per_step * args.steps / dt / 1e9, "unit": "GB/s", "n_gpus": world,
            "per_gpu_gbs": per_step * args.steps / dt / 1e9, "steps": args.steps,
            "bytes_per_step_per_gpu": per_step,
            "equivalent_images_per_s": world * BATCH * args.steps / dt,
            "config": {"workload": "batch-64 input up and output down per step, pinned host "
                                   "buffers, both directions concurrently, no forward",
                       "parallelism": f"replicas{world}"}}), flush=True)
    reps.close()


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.ops:
        run_ops(args)
    elif args.copies:
        run_copies(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
