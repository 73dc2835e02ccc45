#!/usr/bin/env python3
"""Throughput of the SCUNet forward pass on B200, in megapixels per second.

Workload (configuration 4 of the benchmark set): seeded 1920x1080 RGB uint8 frames (smooth field
plus luma-dependent and 2x2-correlated noise), replicate-padded to 1920x1088 on the
device, colour SCUNet with seeded weights. A step is one pass over `--frames`
frames per GPU (batch sharding, no collective: weak scaling); frames go through
the library in micro-batches of `--micro` frames per `scb_forward_dev` call.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One JSON line on rank 0. `value` is device-timed (CUDA events on the launch
stream, max over ranks) with inputs resident in HBM; `e2e` is the same metric
through the host-pointer C-ABI call `scb_forward_host`, one call per step over the
step's frames (pinned host uint8 in, float32 out, copies inside the timed region;
the library overlaps them with the compute of the neighbouring micro-batches). `roofline` is the dominant op class
from a live per-launch event profile (`scb_set_profiling` / `scb_profile_bytes`),
against HBM or the tensor pipe by its arithmetic intensity, with the DRAM traffic
ncu measured for it (`profiles/traffic.json`, written by `--ncu-traffic-kernels`). `cpu_baseline` times
the CPU oracle port (`oracle/scunet_torch.py`, the reference's algorithm restated in
torch float32, all host threads) on a bounded 512x512 crop.

`--workload band` measures configuration 5 instead: one seeded 8192x8192
RGB uint8 image split into 64-row-aligned row bands, one band per rank
(`scb_band_init` + `scb_forward_band`; halo rows cross NVLink with NCCL send/recv
inside the forward). A step is one forward of the whole image; the total work is
fixed as N grows (strong scaling).

`--impl reference` times the reference's CPU implementation of the path. The
reference's own CPU code is Rust and cannot be built here (no cargo, unvendored
crates), so the arm runs the oracle port (torch float32) on all host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import datetime
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

H, W, C = 1080, 1920, 3
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def args_():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=["frames", "band"], default="frames",
                    help="frames: config 4 batch sharding (default); band: config 5 row bands")
    ap.add_argument("--size", type=int, default=8192, help="band workload: image side")
    ap.add_argument("--frames", type=int, default=16, help="frames per GPU per step")
    ap.add_argument("--micro", type=int, default=4, help="frames per library call")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--trans32-lanes", type=int, choices=[0, 1], default=None,
                    help="full-resolution transformer kernel: 1 independent pair lanes, 0 warp-specialised")
    ap.add_argument("--residual32", action="store_true",
                    help="keep the in-stage residual stream in fp32 (SCB_OPT_RESIDUAL32, the reference's precision)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ncu-traffic-kernels", metavar="RAW_CSV:KERNEL:SKIP", nargs="+",
                    help="write profiles/traffic.json from per-kernel ncu captures of a 1-frame forward and exit")
    ap.add_argument("--traffic-out", default=str(ROOT / "profiles" / "traffic.json"),
                    help="where --ncu-traffic-kernels writes its JSON")
    ap.add_argument("--ncu-launches", metavar="CSV", help="print a per-kernel launch table of an ncu capture and exit")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


class Clocks:
    """nvidia-smi sampled every 200 ms during the timed region."""
    Q = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid):
        self.uuid = uuid
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.flush()
        rows = [r.split(", ") for r in Path(self.f.name).read_text().splitlines() if r.strip()]
        rows = [r for r in rows if len(r) >= 9 and (self.uuid is None or self.uuid in r[0])]
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows)}


CPU_SAMPLE = 512  # side of the square crop of a config-4 frame the CPU legs time


def cpu_oracle_mps(img_u8, size, reps=1):
    """The CPU oracle port (`oracle/scunet_torch.py`: the reference forward restated
    in torch float32, strict FP32, every host thread) on a size x size crop; returns
    (MP/s, seconds per forward, threads)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import torch
    import scunet_torch
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    scb = importlib.import_module("scunet-rs_b200")
    wt = scb.Weights.seeded(3, 0).tensors
    x = img_u8[None, :, :size, :size].astype(np.float32) / 255.0
    t0 = time.perf_counter()
    for _ in range(reps):
        scunet_torch.forward(x, wt, device="cpu")
    dt = (time.perf_counter() - t0) / reps
    return size * size / 1e6 / dt, dt, threads


def reference_arm(a, rank, world):
    """Rank 0 times the CPU implementation of the path; other ranks exit. The
    reference's own CPU path is Rust and cannot be built here, so this is the oracle
    port (the same arithmetic, torch float32 on every host thread)."""
    if rank != 0:
        return
    scb = importlib.import_module("scunet-rs_b200")
    img = scb.synth.frames(4000, 1, H, W)[0]
    size = CPU_SAMPLE
    times = []
    cores = 1
    for i in range(a.warmup + a.steps):
        mps, dt, cores = cpu_oracle_mps(img, size)
        if i >= a.warmup:
            times.append(dt)
    tot = sum(times)
    value = a.steps * size * size / 1e6 / tot
    sample = (f"one {size}x{size} crop of a config-4 frame per step: the oracle port of the reference forward "
              f"(oracle/scunet_torch.py, torch float32 on the CPU, {cores} threads)")
    print(json.dumps({
        "impl": "reference", "metric": "megapixels/sec (device-timed, max over ranks)", "value": value,
        "unit": "MP/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1e3 * tot / a.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config4: 1920x1080 RGB uint8 frames -> 1920x1088 padded, colour SCUNet "
                               "(bounded CPU sample)", "sample": sample},
        "cpu_baseline": {"value": value, "unit": "MP/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "MP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def arith_label(be):
    """The arithmetic the context's options give, for the bench line."""
    scb = importlib.import_module("scunet-rs_b200")
    r32 = be.options.get(scb.backend.SCB_OPT_RESIDUAL32, 0)
    stream = "fp32 in-stage residual stream" if r32 else "fp16 in-stage residual stream"
    return f"fp16 tensor-core operands, {stream}, fp32 accumulate and U-Net skips"



def class_totals(prof):
    """{class: [flops, bytes, ms, launches]} over one profiled forward."""
    cls = {}
    for name, fl, nb, t in prof:
        c = cls.setdefault(name, [0.0, 0.0, 0.0, 0])
        c[0] += fl
        c[1] += nb
        c[2] += t
        c[3] += 1
    return cls


def kernel_totals(prof, kernels):
    """{kernel: {flops, bytes, ms, launches, classes}} over one profiled forward."""
    out = {}
    for (cls, fl, nb, t), k in zip(prof, kernels):
        if k.startswith("("):  # halo exchanges and memsets are not kernels of this library
            continue
        e = out.setdefault(k, {"flops": 0.0, "bytes": 0.0, "ms": 0.0, "launches": 0, "classes": set()})
        e["flops"] += fl
        e["bytes"] += nb
        e["ms"] += t
        e["launches"] += 1
        e["classes"].add(cls)
    return out


def roofline_from_profile(prof, kernels):
    """The dominant kernel (most device time) of one profiled forward against its
    roofline: HBM when its arithmetic intensity is below the ridge point of the
    measured peaks, the tensor pipe otherwise. `achieved` = the kernel's algorithmic
    bytes (or FLOPs) per launch / its average launch time (CUDA events on the launch
    stream). `traffic` = DRAM bytes per launch: the DRAM / algorithmic byte ratio ncu
    measured on a few launches of the same kernel (profiles/traffic.json, per-kernel
    captures of a one-frame forward) times this workload's algorithmic bytes per
    launch."""
    cls = class_totals(prof)
    tot_ms = sum(v[2] for v in cls.values())
    ks = kernel_totals(prof, kernels)
    dom = max(ks, key=lambda k: ks[k]["ms"])
    d = ks[dom]
    fl, nb, ms, n = d["flops"], d["bytes"], d["ms"], d["launches"]
    pk, pk_kind = peaks()
    tflops = float(pk.get("bf16_tflops_sustained", pk.get("bf16_tflops")))
    hbm = float(pk["hbm_gbs"])
    ridge = tflops * 1e12 / (hbm * 1e9)
    memory_bound = fl / max(nb, 1.0) < ridge
    t_launch = ms / n / 1e3
    if memory_bound:
        achieved, peak, unit, bound = nb / n / t_launch / 1e9, hbm, "GB/s", "hbm"
        src = f"{pk_kind} HBM copy bandwidth"
    else:
        achieved, peak, unit, bound = fl / n / t_launch / 1e12, tflops, "TFLOP/s", "tensor"
        src = f"{pk_kind} bf16/fp16 dense sustained"
    traffic, ratio = None, None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists():
        c = json.loads(tf.read_text()).get("kernels", {}).get(dom)
        if c:
            ratio = c["dram_bytes"] / c["algorithmic_bytes"]
            traffic = ratio * nb / n
    return {
        "kernel": dom, "classes": sorted(d["classes"]),
        "bound": bound, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
        "peak_source": src, "traffic": traffic, "traffic_over_algorithmic": ratio,
        "algorithmic_bytes_per_launch": nb / n, "flops_per_launch": fl / n, "launches": n,
        "share_of_forward": ms / tot_ms,
        "kernels_ms_share": {k: round(v["ms"] / tot_ms, 4) for k, v in sorted(ks.items(), key=lambda kv: -kv[1]["ms"])},
        "classes_ms_share": {k: round(v[2] / tot_ms, 4) for k, v in sorted(cls.items(), key=lambda kv: -kv[1][2])},
        "whole_forward_tflops": sum(v[0] for v in cls.values()) / (tot_ms / 1e3) / 1e12,
    }


def read_ncu_csv(path):
    """ncu --csv --log-file output -> [(kernel name, {metric: value})] in launch order."""
    import csv
    rows = list(csv.reader(l for l in Path(path).read_text().splitlines() if l.startswith('"')))
    h = rows[0]
    iid, iname, im, iv = h.index("ID"), h.index("Kernel Name"), h.index("Metric Name"), h.index("Metric Value")
    launches = {}
    for r in rows[1:]:
        d = launches.setdefault(int(r[iid]), [r[iname], {}])
        d[1][r[im]] = float(r[iv].replace(",", ""))
    return [launches[k] for k in sorted(launches)]


def ncu_launch_summary(path):
    """Markdown table: per kernel, launches, total device time and share."""
    ls = read_ncu_csv(path)
    per = {}
    for name, m in ls:
        k = name.split("(")[0]
        t = m.get("gpu__time_duration.sum", 0.0)
        e = per.setdefault(k, [0, 0.0])
        e[0] += 1
        e[1] += t
    tot = sum(v[1] for v in per.values())
    out = ["| kernel | launches | total (ms) | share |", "|---|---|---|---|"]
    for k, (n, t) in sorted(per.items(), key=lambda kv: -kv[1][1]):
        out.append(f"| `{k}` | {n} | {t / 1e6:.3f} | {100 * t / tot:.1f} % |")
    out.append(f"| all | {len(ls)} | {tot / 1e6:.3f} | |")
    return "\n".join(out)


NCU_UNITS = {"byte": 1.0, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "nsecond": 1.0, "ns": 1.0, "usecond": 1e3,
             "us": 1e3, "msecond": 1e6, "ms": 1e6}


def read_ncu_raw(path):
    """`ncu -i <rep> --page raw --csv` output -> [(kernel name, {metric: value})], with
    byte metrics in bytes and durations in nanoseconds."""
    import csv
    rows = list(csv.reader(l for l in Path(path).read_text().splitlines() if l.startswith('"')))
    if len(rows) < 3:
        raise SystemExit(f"{path}: no captured launches")
    h, units = rows[0], rows[1]
    out = []
    for r in rows[2:]:
        m = {}
        for k, u, v in zip(h, units, r):
            try:
                m[k] = float(v.replace(",", "")) * NCU_UNITS.get(u, 1.0)
            except ValueError:
                m[k] = v
        out.append((m.get("Kernel Name", "?"), m))
    return out


def ncu_traffic_kernels(specs, out_path):
    """Per-kernel DRAM traffic from small ncu captures of a one-frame forward.

    Each spec is RAW_CSV:KERNEL:SKIP - an `ncu -i ... --page raw --csv` export of a
    capture of launches SKIP+1 .. SKIP+N of KERNEL (as scb_profile_kernels names it).
    The captured launches are matched to the same occurrences of that kernel in a
    profiled forward of the same configuration (their algorithmic bytes); writes
    profiles/traffic.json and prints the table."""
    import torch
    scb = importlib.import_module("scunet-rs_b200")
    be = scb.B200(scb.Weights.seeded(3, 0), device=0)
    fr = torch.from_numpy(scb.synth.frames(4000, 1, H, W)).cuda()
    y = torch.empty((1, C, H, W), dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    be.set_profiling(True)
    be.forward_dev(fr.data_ptr(), scb.SCB_U8, 1, C, H, W, y.data_ptr(), scb.SCB_F32, s.cuda_stream)
    torch.cuda.synchronize()
    prof, kern = be.profile(), be.profile_kernels()
    be.close()
    out = {}
    for spec in specs:
        path, kname, skip = spec.rsplit(":", 2)
        rows = read_ncu_raw(path)
        occ = [i for i, k in enumerate(kern) if k == kname][int(skip):int(skip) + len(rows)]
        if len(occ) != len(rows):
            raise SystemExit(f"{path}: {len(rows)} captured launches, {len(occ)} matching ops of {kname}")
        e = out.setdefault(kname, {"captured_launches": 0, "dram_bytes": 0.0, "algorithmic_bytes": 0.0,
                                   "ncu_us": 0.0, "classes": set(), "source": []})
        for (name, m), i in zip(rows, occ):
            e["captured_launches"] += 1
            e["dram_bytes"] += m["dram__bytes_read.sum"] + m["dram__bytes_write.sum"]
            e["algorithmic_bytes"] += prof[i][2]
            e["ncu_us"] += m["gpu__time_duration.sum"] / 1e3
            e["classes"].add(prof[i][0])
        e["source"].append(Path(path).name)
    for e in out.values():
        e["classes"] = sorted(e["classes"])
    res = {"workload": "one 1920x1080 frame per call (padded 1920x1088), seeded config-4 frame and weights; "
                       "DRAM bytes from per-kernel ncu captures of 1-3 launches each",
           "kernels": out}
    Path(out_path).write_text(json.dumps(res, indent=1) + "\n")
    lines = ["| kernel | classes | captured launches | DRAM MB per launch | algorithmic MB per launch | DRAM / algorithmic |",
             "|---|---|---|---|---|---|"]
    for k, e in sorted(out.items(), key=lambda kv: -kv[1]["dram_bytes"] / kv[1]["captured_launches"]):
        n = e["captured_launches"]
        lines.append(f"| `{k}` | {', '.join(e['classes'])} | {n} | {e['dram_bytes'] / n / 1e6:.1f} | "
                     f"{e['algorithmic_bytes'] / n / 1e6:.1f} | {e['dram_bytes'] / e['algorithmic_bytes']:.2f} |")
    print("\n".join(lines))


class Job:
    """Process-group plumbing shared by both workloads."""

    def __init__(self, a):
        import torch
        import torch.distributed as dist
        self.torch, self.dist = torch, dist
        self.rank, self.world, self.local = dist_env()
        torch.cuda.set_device(self.local)
        if self.world > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local))
        self.uuid = None
        try:
            self.uuid = str(torch.cuda.get_device_properties(self.local).uuid)
        except Exception:
            pass

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def gather(self, v):
        """[v of rank 0, v of rank 1, ...] on every rank."""
        if self.world == 1:
            return [v]
        t = self.torch.zeros(self.world, dtype=self.torch.float64, device="cuda")
        t[self.rank] = v
        self.dist.all_reduce(t)
        return [float(u) for u in t.cpu()]

    def max_over_ranks(self, v):
        if self.world == 1:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def timed(self, step, steps, stream):
        """ms per step: CUDA events on `stream`, barrier + synchronize on both sides,
        max over ranks; clocks sampled during the region."""
        torch = self.torch
        self.barrier()
        clk = Clocks(self.uuid)
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        t0.record(stream)
        for _ in range(steps):
            step()
        t1.record(stream)
        torch.cuda.synchronize()
        clocks = clk.stop()
        mine = t0.elapsed_time(t1) / steps
        self.per_rank = self.gather(mine)
        ms = max(self.per_rank)
        self.barrier()
        return ms, clocks

    def close(self):
        if self.world > 1:
            self.dist.destroy_process_group()


def frames_workload(a, job, scb):
    torch = job.torch
    rank, world, local = job.rank, job.world, job.local
    F, micro = a.frames, a.micro
    assert F % micro == 0, "--frames must be a multiple of --micro"
    wt = scb.Weights.seeded(3, 0)
    be = scb.B200(wt, device=local)
    if a.residual32:
        be.set_option(scb.backend.SCB_OPT_RESIDUAL32, 1)
    if a.trans32_lanes is not None:
        be.set_option(scb.backend.SCB_OPT_TRANS32_LANES, a.trans32_lanes)
    frames = scb.synth.frames(4000 + rank, F, H, W, distinct=min(F, 4))
    x_dev = torch.from_numpy(frames).cuda()
    y_dev = torch.empty((F, C, H, W), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    # An explicit stream: the library's kernels and the timing events must share it
    # (the legacy default stream's handle is 0, which the C ABI reads as "use the
    # context's own stream").
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    assert sp != 0

    def step():
        for i in range(0, F, micro):
            be.forward_dev(x_dev[i].data_ptr(), scb.SCB_U8, micro, C, H, W, y_dev[i].data_ptr(), scb.SCB_F32, sp)

    for _ in range(max(a.warmup, 3)):
        step()
    torch.cuda.synchronize()
    launches_per_call = be.last_launch_count()
    ms, clocks = job.timed(step, a.steps, stream)
    per_rank = [round(v, 3) for v in job.per_rank]
    mp_step = F * H * W * world / 1e6
    value = mp_step / (ms / 1e3)

    # ---- live per-launch profile of one call (untimed above) -> roofline ----
    be.set_profiling(True)
    be.forward_dev(x_dev[0].data_ptr(), scb.SCB_U8, micro, C, H, W, y_dev[0].data_ptr(), scb.SCB_F32, sp)
    torch.cuda.synchronize()
    roofline = roofline_from_profile(be.profile(), be.profile_kernels())
    be.set_profiling(False)

    # ---- end to end through the host-pointer C ABI ----
    e2e = None
    if not a.no_e2e:
        hx = torch.from_numpy(frames).pin_memory()
        hy = torch.empty((F, C, H, W), dtype=torch.float32).pin_memory()

        be.set_option(scb.backend.SCB_OPT_HOST_CHUNK, micro)

        def e2e_step():
            rc = be.lib.scb_forward_host(be.ctx, hx.data_ptr(), scb.SCB_U8, F, C, H, W, hy.data_ptr(), scb.SCB_F32)
            if rc:
                raise RuntimeError(be.lib.scb_last_error(be.ctx).decode())

        e2e_step()
        job.barrier()
        t = time.perf_counter()
        for _ in range(a.steps):
            e2e_step()
        dt = (time.perf_counter() - t) / a.steps
        dt = job.max_over_ranks(dt)
        e2e = {"value": mp_step / dt, "unit": "MP/s", "h2d_bytes_per_step": int(hx.numel()) * world,
               "d2h_bytes_per_step": int(hy.numel() * 4) * world,
               "api": f"scb_forward_host, one call of {F} frames per step (pinned host buffers; {micro}-frame "
                      f"compute chunks, copies of the neighbouring chunks overlapped)",
               "timing": "host wall clock around the synchronous calls, max over ranks"}

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        mps, dt, cores = cpu_oracle_mps(frames[0], CPU_SAMPLE, reps=2)
        cpu = {"value": mps, "unit": "MP/s", "cores": cores, "kind": "port",
               "sample": f"two forwards of a {CPU_SAMPLE}x{CPU_SAMPLE} crop of frame 0 ({dt:.1f} s each): the "
                         f"oracle port of the reference forward, torch float32 on {cores} CPU threads"}

    if rank == 0:
        print(json.dumps({
            "metric": "megapixels/sec (device-timed, max over ranks)", "value": value, "unit": "MP/s",
            "n_gpus": world, "steps": a.steps, "warmup": max(a.warmup, 3), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic (seeded config-4 frames; seeded weights)",
            "config": {"workload": "config4: 1920x1080 RGB uint8 frames -> 1920x1088 padded, colour SCUNet",
                       "frames_per_gpu": F, "global_batch": F * world, "micro_batch": micro,
                       "parallelism": f"dp{world} (batch sharding, no collective)",
                       "l2": "inputs larger than L2 (each step streams %.1f GB of activations)" % (
                           scb.need_bytes(micro, 3, 1088, 1920) / 1e9),
                       "arith": arith_label(be)},
            "clocks": clocks, "per_rank_ms": per_rank, "slowest_rank": int(np.argmax(per_rank)),
            "e2e": e2e, "gpu_launches": launches_per_call * (F // micro) * a.steps,
            "roofline": roofline, "cpu_baseline": cpu,
        }), flush=True)
    be.close()


def band_workload(a, job, scb):
    """Config 5: one image, one row band per rank, halo exchange inside the forward."""
    torch, dist = job.torch, job.dist
    rank, world, local = job.rank, job.world, job.local
    S = a.size
    wt = scb.Weights.seeded(3, 0)
    be = scb.B200(wt, device=local)
    # Rank 0 makes the image on its GPU and broadcasts it over NCCL; every rank
    # passes the whole image to scb_forward_band and computes its own band.
    x_dev = torch.empty((1, C, S, S), dtype=torch.uint8, device="cuda")
    if rank == 0:
        x_dev.copy_(scb.synth.noisy_image_device(1005, C, S, S, 25.0 / 255.0, device="cuda"))
    uid = [scb.band_unique_id() if rank == 0 else None]
    if world > 1:
        dist.broadcast(x_dev, 0)
        dist.broadcast_object_list(uid, 0)
    be.band_init(uid[0], rank, world)
    y_dev = torch.empty((1, C, S, S), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    assert sp != 0
    hp = (S + 63) // 64 * 64
    r0, rows = scb.shard.band_rows(hp, rank, world)
    rows = max(0, min(rows, S - r0))

    def step():
        be.forward_band(x_dev.data_ptr(), scb.SCB_U8, C, S, S, y_dev.data_ptr(), scb.SCB_F32, sp)

    for _ in range(max(a.warmup, 3)):
        step()
    torch.cuda.synchronize()
    launches_per_call = be.last_launch_count()
    ms, clocks = job.timed(step, a.steps, stream)
    per_rank = [round(v, 3) for v in job.per_rank]
    mp_step = S * S / 1e6
    value = mp_step / (ms / 1e3)

    # Profile one banded forward (every rank runs it: the halo exchange pairs them).
    be.set_profiling(True)
    step()
    torch.cuda.synchronize()
    roofline = roofline_from_profile(be.profile(), be.profile_kernels())
    be.set_profiling(False)
    job.barrier()

    e2e = None
    if not a.no_e2e:
        # Host image in (only the input rows this rank's band reads, one copy per
        # colour plane), this rank's output rows out, copies on the compute stream.
        hx = torch.empty((1, C, S, S), dtype=torch.uint8).pin_memory()
        hx.copy_(x_dev.cpu())
        hy = torch.empty((1, C, rows, S), dtype=torch.float32).pin_memory()
        lo, hi = scb.shard.band_input_rows(S, hp, rank, world)
        h2d_bytes = int(sum(job.gather(float(C * (hi - lo) * S))))

        def e2e_step():
            with torch.cuda.stream(stream):
                for ch in range(C):
                    x_dev[0, ch, lo:hi].copy_(hx[0, ch, lo:hi], non_blocking=True)
                step()
                for ch in range(C):
                    hy[0, ch].copy_(y_dev[0, ch, r0:r0 + rows], non_blocking=True)
            stream.synchronize()

        e2e_step()
        job.barrier()
        t = time.perf_counter()
        for _ in range(a.steps):
            e2e_step()
        dt = job.max_over_ranks((time.perf_counter() - t) / a.steps)
        e2e = {"value": mp_step / dt, "unit": "MP/s", "h2d_bytes_per_step": h2d_bytes,
               "d2h_bytes_per_step": S * S * C * 4,
               "api": "scb_forward_band (each rank's input rows, its band and one row each side, copied "
                      "from pinned host memory; its band rows back)"}

    if rank == 0:
        print(json.dumps({
            "metric": "megapixels/sec (device-timed, max over ranks)", "value": value, "unit": "MP/s",
            "n_gpus": world, "steps": a.steps, "warmup": max(a.warmup, 3), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic (seeded config-5 image generated on the GPU; seeded weights)",
            "config": {"workload": f"config5: one {S}x{S} RGB uint8 image in 64-row-aligned row bands",
                       "bands": world, "rows_per_band_rank0": rows,
                       "parallelism": f"row bands over {world} GPU(s), halo rows by NCCL send/recv",
                       "l2": "inputs larger than L2 (one forward streams %.0f GB of activations)" % (
                           scb.need_bytes(1, 3, hp, hp) / 1e9),
                       "arith": arith_label(be)},
            "clocks": clocks, "per_rank_ms": per_rank, "slowest_rank": int(np.argmax(per_rank)),
            "e2e": e2e, "gpu_launches": launches_per_call * a.steps,
            "roofline": roofline, "cpu_baseline": None,
        }), flush=True)
    be.close()


def main():
    a = args_()
    if a.ncu_launches:
        print(ncu_launch_summary(a.ncu_launches))
        return
    if a.ncu_traffic_kernels:
        ncu_traffic_kernels(a.ncu_traffic_kernels, a.traffic_out)
        return
    rank, world, local = dist_env()
    if a.impl == "reference":
        reference_arm(a, rank, world)
        return
    scb = importlib.import_module("scunet-rs_b200")
    job = Job(a)
    try:
        (band_workload if a.workload == "band" else frames_workload)(a, job, scb)
    finally:
        job.close()


if __name__ == "__main__":
    main()
