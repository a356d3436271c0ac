"""Benchmark of the B200 fused causal softmax (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one step): the batched multi-head configuration, B=8 x H=32 causal
softmaxes of 4096 x 4096 FP16 scores (256 matrices, 8 GiB in, 8 GiB out),
values half(N(0,1)*3) from seed 3, scale 1/sqrt(128), heads sharded evenly
over the N ranks (one process per GPU, launched by torchrun for N > 1). There
is no collective on the data path: ranks meet only at the timing barriers.

value  = algorithmic bytes of all ranks per step (triangle read 2*T + full
         write 2*M*N per matrix) / step time, in GB/s; step time is the max
         over ranks of CUDA-event time over K back-to-back launches
         (inputs are 8/N GiB > L2, so no flush is needed between steps).
e2e    = the same metric through the host-buffer API (cs_session_softmax_host):
         pinned host input -> device -> kernel -> pinned host output per step.
roofline, cpu_baseline, clocks: see DESIGN.md (measurement section).

--impl reference times the reference's CPU path (the C restatement of
reference/src/lib.rs:85-108 in oracle/, there being no Rust toolchain to build
the reference itself) on the host cores of rank 0, on a bounded sample of the
same workload per step.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "gb200-sm100a-tma-fused-causal-attention-softmax_b200")
sys.path.insert(0, PKG_DIR)

WORKLOAD = {
    "workload": "batched multi-head causal softmax, B=8 H=32 L=4096: 256 matrices of "
                "4096x4096 FP16 scores, heads sharded over ranks",
    "matrices": 256, "rows": 4096, "cols": 4096, "pitch": 4096,
    "values": "half(N(0,1)*3)", "seed": 3, "scale": "1/sqrt(128)",
    "l2": "inputs larger than L2 (8/N GiB per rank), no flush",
}
METRIC = "achieved HBM GB/s (% of tri-read+write roofline) and matrices/s, 1/2/4/8 B200"
CONFIG_ID, SEED, MATRICES, L = 4, 3, 256, 4096


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def scale_f32() -> float:
    import numpy as np

    return float(np.float32(1.0 / math.sqrt(128.0)))


def measured_peak() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def ncu_traffic_per_matrix() -> float | None:
    """DRAM bytes per 4096^2 matrix from the committed ncu summary, if present."""
    p = os.path.join(ROOT, "profiles", "tma_rowres_c4.md")
    try:
        for line in open(p):
            if line.strip().startswith("dram_bytes_per_matrix"):
                return float(line.split("=")[1].split()[0])
    except Exception:
        pass
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while the timed region runs."""

    def __init__(self, device: int, period_s: float = 0.002):
        self.device, self.period = device, period_s
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        self.ok = False

    def __enter__(self):
        try:
            import pynvml as nv

            nv.nvmlInit()
            uuid_env = os.environ.get("CUDA_VISIBLE_DEVICES", "")
            idx = self.device
            if uuid_env and "," not in uuid_env and uuid_env.isdigit():
                idx = int(uuid_env)
            elif uuid_env and "," in uuid_env:
                parts = uuid_env.split(",")
                if all(p.isdigit() for p in parts):
                    idx = int(parts[self.device])
            self.h = nv.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
            self.nv = nv
            self.ok = True
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception as e:  # NVML missing: clocks are reported as unavailable
            log(f"clock sampling unavailable: {e}")
        return self

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((mhz, reasons))
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self) -> dict | None:
        if not self.ok or not self.samples:
            return None
        names = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
                 0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
                 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
                 0x100: "display_clock_setting"}
        seen = set()
        for _, r in self.samples:
            for bit, n in names.items():
                if r & bit and n != "gpu_idle":
                    seen.add(n)
        return {"sm_mhz": statistics.median(m for m, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": sorted(seen),
                "samples": len(self.samples)}


def cpu_baseline_single(n_seconds: float = 12.0) -> dict:
    """The reference CPU path (oracle restatement, single thread like
    host/examples/cpu_bench.rs:67) on whole matrices of the workload."""
    import numpy as np

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle_ctypes as O
    import causal_softmax as cs

    x = cs.generate(CONFIG_ID, SEED, batch=1, rows=L, cols=L)[0].ravel()
    s = scale_f32()
    O.softmax_strided(x, 1, 0, 256, L, L, 0, s, threads=1)  # warm-up (untimed)
    done, t0 = 0, time.perf_counter()
    while True:
        O.softmax_strided(x, 1, 0, L, L, L, 0, s, threads=1)
        done += 1
        if time.perf_counter() - t0 >= n_seconds:
            break
    dt = time.perf_counter() - t0
    alg = cs.roofline_bytes(L, L) * done
    return {"value": round(alg / dt / 1e9, 4), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"{done} whole 4096x4096 matrices of the workload (seed 3), single thread, "
                      f"{dt:.1f} s; matrices/s = {done / dt:.4f}"}


def run_reference(args) -> None:
    """Reference arm: the CPU path on all host threads of rank 0."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle_ctypes as O
    import causal_softmax as cs

    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    # Each step is a bounded sample of the workload: `per_step` whole matrices
    # (at least one per 8 threads) processed row-parallel over all threads.
    per_step = max(1, min(MATRICES, threads // 8))
    x = cs.generate(CONFIG_ID, SEED, batch=per_step, rows=L, cols=L).ravel()
    s = scale_f32()
    for _ in range(args.warmup):
        O.softmax_strided(x, per_step, L * L, L, L, L, 0, s, threads=threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        O.softmax_strided(x, per_step, L * L, L, L, L, 0, s, threads=threads)
        times.append(time.perf_counter() - t0)
    step = statistics.mean(times)
    alg = cs.roofline_bytes(L, L) * per_step
    value = alg / step / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "io_dtype": "f16", "data": "synthetic",
        "config": dict(WORKLOAD, sample_matrices_per_step=per_step),
        "matrices_per_s": round(per_step / step, 4),
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads,
                         "kind": "port",
                         "sample": f"{per_step} whole matrices per step, rows split over "
                                   f"{threads} threads (C restatement of reference/src/lib.rs:85-108)"},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--kernel", default="auto")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--tuning", default="",
                    help="vec,stages,l2_hint,zero_fill_tma for the row-resident kernel")
    ap.add_argument("--matrices", type=int, default=MATRICES,
                    help="heads in the batch (256 = the benchmark workload; smaller only for "
                         "profiling captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        log("warmup raised to 3 (timing rule)")
        args.warmup = 3

    if args.impl == "reference":
        run_reference(args)
        return 0

    import numpy as np
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        log(f"--gpus {args.gpus} but WORLD_SIZE {world}: using WORLD_SIZE")
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    import build

    build.build_library()
    import causal_softmax as cs

    n_total = args.matrices
    if n_total % world:
        raise SystemExit(f"{n_total} heads must split evenly over the ranks")
    n_local = n_total // world
    first = rank * n_local
    scale = scale_f32()

    # Host input of this rank's heads (pinned), then device copies.
    t0 = time.perf_counter()
    h_in = torch.empty((n_local, L, L), dtype=torch.int16, pin_memory=True)
    cs.generate(CONFIG_ID, SEED, batch=n_local, rows=L, cols=L, first_batch=first,
                out=h_in.numpy().view(np.uint16))
    d_in = h_in.cuda().view(torch.float16)
    d_out = torch.empty_like(d_in)
    log(f"rank {rank}: {n_local} matrices generated and resident in {time.perf_counter() - t0:.1f} s")

    stream = torch.cuda.current_stream()
    plan = cs.Plan.for_tensors(d_in, d_out, cols=L)
    if args.tuning:
        plan.set_tuning(*(int(t) for t in args.tuning.split(",")))
    info = plan.describe(args.kernel)
    log(f"rank {rank}: launch {info}")

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        plan.launch(args.kernel, scale, stream)
    torch.cuda.synchronize()
    rc, st = plan.status()
    if rc != 0:
        raise SystemExit(f"device status {st} after warm-up")

    # Spot check of the timed kernel's output (structure of two matrices).
    host_out = d_out[:2].view(torch.int16).cpu().numpy().view(np.uint16)
    chk = cs.check_output(host_out, batch=min(2, n_local), rows=L, cols=L, pitch=L)
    if chk["mask_violations"] or chk["nonfinite_or_negative"] or chk["rowsum_violations"]:
        raise SystemExit(f"output self-check failed: {chk}")

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            plan.launch(args.kernel, scale, stream)
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms_total = start.elapsed_time(end)
    rc, st = plan.status()
    if rc != 0:
        raise SystemExit(f"device status {st} after the timed region")
    t = torch.tensor([ms_total], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    ms_step = ms_max / args.steps
    alg_local = info["algorithmic_bytes"]
    alg_total = alg_local * world
    value = alg_total / (ms_step / 1e3) / 1e9

    # Roofline of the (single) kernel: per-launch bytes / per-launch time on this rank.
    peak, peak_kind = measured_peak()
    achieved = alg_local / (ms_total / args.steps / 1e3) / 1e9
    tpm = ncu_traffic_per_matrix()
    roofline = {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
                "traffic": round(tpm * n_local) if tpm else None,
                "algorithmic_bytes_per_launch": alg_local,
                "kernel": f"{info['kernel_name']} grid={info['grid']} block={info['block']} "
                          f"smem={info['smem_bytes']} stages={info['stages']} "
                          f"vec={info['vec_per_thread']}"}
    clk = clocks.summary()

    # End to end through the host-buffer API (pinned input -> device -> pinned output).
    e2e = None
    if not args.no_e2e:
        del d_out
        torch.cuda.empty_cache()
        h_out = torch.empty_like(h_in, pin_memory=True)
        hin_np = h_in.numpy().view(np.uint16).reshape(-1)
        hout_np = h_out.numpy().view(np.uint16).reshape(-1)
        with cs.Session(local) as sess:
            sess.softmax_host(hin_np, hout_np, batch=n_local, rows=L, cols=L, scale=scale,
                              kernel=args.kernel)  # warm-up: device buffers allocated here
            times = []
            for _ in range(max(1, args.e2e_steps)):
                barrier()
                t0 = time.perf_counter()
                sess.softmax_host(hin_np, hout_np, batch=n_local, rows=L, cols=L, scale=scale,
                                  kernel=args.kernel)
                times.append(time.perf_counter() - t0)
            e_step = torch.tensor([statistics.mean(times)], dtype=torch.float64, device="cuda")
            if world > 1:
                dist.all_reduce(e_step, op=dist.ReduceOp.MAX)
            e_s = float(e_step.item())
        # The host result equals the device result of the timed kernel (first matrix).
        e2e = {"value": round(alg_total / e_s / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": int(n_local * L * L * 2 * world),
               "d2h_bytes_per_step": int(n_local * L * L * 2 * world),
               "ms_per_step": round(e_s * 1e3, 2),
               "timing": "host wall clock around the blocking call, max over ranks"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_single(args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "io_dtype": "f16", "data": "synthetic",
            "config": dict(WORKLOAD, kernel=info["kernel_name"], matrices=n_total,
                           matrices_per_rank=n_local),
            "matrices_per_s": round(n_total / (ms_step / 1e3), 2),
            "roofline_pct": round(100.0 * value / (peak * world), 2),
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk,
            "gpu_launches": args.steps * world, "gpu_launches_per_rank": args.steps,
        }
        print(json.dumps(line), flush=True)
    plan.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
