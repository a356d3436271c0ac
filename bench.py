"""Benchmark of the B200 fused causal softmax (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c4|c1|c2a|c2b|c3|c5] [--weak]

Default workload (one step): the batched multi-head configuration, B=8 x H=32
causal softmaxes of 4096 x 4096 FP16 scores (256 matrices, 8 GiB in, 8 GiB
out), values half(N(0,1)*3) from seed 3, scale 1/sqrt(128). With N ranks (one
process per GPU, launched by torchrun for N > 1) the 256 heads are sharded
evenly: rank k runs matrices [k*256/N, (k+1)*256/N) of the seeded stream
(strong scaling: the job stays 256 matrices). --weak gives every rank its own
256 heads instead (the job grows to N x 256; labelled "weak"). The
single-matrix workloads (c1 4096^2, c2a 1000x1037 pitch 1040, c2b 4096x32, c3
8192^2 stress, c5 32768^2) shard one matrix over the ranks (strong scaling):
rank k holds row block [t_k, t_k+1) and its mirror [M - t_k+1, M - t_k) of
the M rows, stored one after the other (a folded plan: row_offset plus
cs_plan_set_row_split), so each rank's row pairs are those of the whole
matrix; --contiguous-rows (and matrices with more rows than columns, or too
few rows to fold) use contiguous blocks of equal causal cost. There is no
collective on the data path: ranks meet only at the timing barriers.

value  = algorithmic bytes of all ranks per step (triangle read 2*T + full
         write 2*M*N per matrix) / step time, in GB/s; step time is the max
         over ranks of CUDA-event time over K back-to-back launches. When one
         rank's buffers are smaller than 2 x L2, R copies are rotated so that
         consecutive launches touch more than 2 x L2 of memory.
e2e    = the same metric through the host-buffer API (cs_session_softmax_host):
         pinned host input -> device -> kernel -> pinned host output per step,
         host wall clock around the blocking call, max over ranks. The call
         moves only causal row blocks over PCIe (h2d/d2h bytes below) and
         writes the output's masked tails with host threads.
gather = N > 1 only: every rank's output shard sent to rank 0 over NCCL
         (NVLink), after the timed region; GB/s of the bytes rank 0 receives.
         For row blocks rank 0 assembles the matrix and checks its row sums.
graph  = single-matrix workloads only: the same launches captured k at a time
         in a CUDA graph, device time per launch (labelled; not the value).
launch_stats = min / median / p95 / max of single launches (the reference's
         BenchStats), from a separate pass with an event after each launch.
roofline  = the single kernel's per-launch algorithmic bytes / per-launch time
            against the measured HBM copy bandwidth (MEASURED_PEAKS.json).
cpu_baseline = the reference CPU path (C restatement of
            reference/src/lib.rs:85-108 in oracle/, single thread like
            host/examples/cpu_bench.rs) on rank 0 at N=1, on a bounded sample.

--impl reference times that CPU path on all host threads of rank 0 (there is
no Rust toolchain to build the reference itself): every step runs whole
matrices of the workload, row-parallel, with inputs from the oracle's copy of
the seeded generator. That arm loads only the oracle library, never this
package's CUDA library, and prints the same config as this arm.
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "gb200-sm100a-tma-fused-causal-attention-softmax_b200")
sys.path.insert(0, PKG_DIR)

METRIC = "achieved HBM GB/s (% of tri-read+write roofline) and matrices/s, 1/2/4/8 B200"
L2_BYTES = 126 * 2**20
INV_SQRT128 = 1.0 / math.sqrt(128.0)

WORKLOADS = {
    "c4": dict(config=4, seed=3, matrices=256, rows=4096, cols=4096, pitch=4096, scale=INV_SQRT128,
               shard="heads", values="half(N(0,1)*3)",
               desc="batched multi-head causal softmax, B=8 H=32 L=4096: 256 matrices of "
                    "4096x4096 FP16 scores, heads sharded evenly over the ranks"),
    "c1": dict(config=1, seed=0, matrices=1, rows=4096, cols=4096, pitch=4096, scale=INV_SQRT128,
               shard="rows", values="half(N(0,1)*4)",
               desc="single 4096x4096 causal softmax, row blocks sharded over ranks"),
    "c2a": dict(config=2, seed=1, matrices=1, rows=1000, cols=1037, pitch=1040, scale=0.0883883,
                shard="rows", values="half(U(-8,8))",
                desc="odd shape 1000x1037, pitch 1040, row blocks sharded over ranks"),
    "c2b": dict(config=2, seed=1, matrices=1, rows=4096, cols=32, pitch=32, scale=0.0883883,
                shard="rows", values="half(U(-8,8))",
                desc="narrow 4096x32 (warp path), row blocks sharded over ranks"),
    "c3": dict(config=3, seed=2, matrices=1, rows=8192, cols=8192, pitch=8192, scale=1.0,
               shard="rows", values="half(N(0,1)*8), 1% +-60000, planted row-max ties",
               desc="stress 8192x8192 causal softmax, row blocks sharded over ranks"),
    "c5": dict(config=5, seed=4, matrices=1, rows=32768, cols=32768, pitch=32768,
               scale=INV_SQRT128, shard="rows", values="half(N(0,1)*2 + 0.001*c)",
               desc="long context 32768x32768 causal softmax, folded row-block shards over "
                    "ranks"),
}


def log(*a):
    # One write per line, so that lines of concurrent ranks do not interleave.
    sys.stderr.write(" ".join(str(x) for x in a) + "\n")
    sys.stderr.flush()


def f32(x: float) -> float:
    return float(np.float32(x))


def measured_peak() -> tuple[float, str]:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def ncu_traffic_per_matrix(kernel: str, workload: str) -> float | None:
    """DRAM bytes per matrix of the kernel on the workload, from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", f"{kernel}_{workload}.md")
    try:
        for line in open(p):
            if line.strip().startswith("dram_bytes_per_matrix"):
                return float(line.split("=")[1].split()[0])
    except Exception:
        pass
    return None


def row_blocks(rows: int, cols: int, parts: int) -> list[tuple[int, int]]:
    """Split rows into `parts` contiguous blocks of equal cost, cost(r) =
    2*min(r+1, cols) (causal read) + 2*cols (full write). Needs rows >= parts
    (every rank gets at least one row)."""
    if rows < parts:
        raise ValueError(f"{rows} rows cannot be split over {parts} ranks: every rank needs a row")
    cost = [2 * min(r + 1, cols) + 2 * cols for r in range(rows)]
    total = sum(cost)
    bounds, acc, k = [0], 0, 1
    for r, c in enumerate(cost):
        acc += c
        if k < parts and acc >= total * k / parts and r + 1 <= rows - (parts - k):
            bounds.append(r + 1)
            k += 1
    while len(bounds) < parts:  # keep one row for each remaining rank
        bounds.append(max(bounds[-1] + 1, rows - (parts - len(bounds))))
    bounds.append(rows)
    return [(bounds[i], bounds[i + 1]) for i in range(parts)]


def can_fold(rows: int, cols: int, parts: int) -> bool:
    """Folded shards need rows <= cols and at least one row per rank in every
    block and its mirror (rows // 2 >= parts)."""
    return rows <= cols and rows // 2 >= parts


def rank_segments(rows: int, cols: int, parts: int, rank: int, fold: bool = True) -> list[tuple[int, int]]:
    """Row segments (first absolute row, row count) of one rank's shard of a
    single matrix, in the order they are stored.

    Folded (rows <= cols, so every row but possibly the last is shorter than
    the row width, and rows // 2 >= parts): rank k < parts-1 holds rows
    [t_k, t_k+1) and their mirror [rows - t_k+1, rows - t_k),
    t_k = k * (rows // 2) // parts, and the last rank the middle block
    [t_parts-1, rows - t_parts-1). Each shard's row pairs then carry rows + 1
    causal elements, as in the whole matrix, and the shards are equal.
    Otherwise (fold off, tall matrices, or too few rows to give every rank a
    block and its mirror): contiguous blocks of equal causal cost."""
    if not fold or not can_fold(rows, cols, parts):
        a, b = row_blocks(rows, cols, parts)[rank]
        return [(a, b - a)]
    t = [k * (rows // 2) // parts for k in range(parts)]
    if rank == parts - 1:
        return [(t[rank], rows - 2 * t[rank])]
    return [(t[rank], t[rank + 1] - t[rank]), (rows - t[rank + 1], t[rank + 1] - t[rank])]


def head_range(matrices: int, parts: int, rank: int) -> tuple[int, int]:
    """First matrix and matrix count of one rank's even share of the heads."""
    if matrices < parts:
        raise ValueError(f"{matrices} heads cannot be split over {parts} ranks")
    a, b = rank * matrices // parts, (rank + 1) * matrices // parts
    return a, b - a


def rank_share(w: dict, world: int, rank: int, weak: bool, contiguous: bool,
               row_block: tuple[int, int] | None = None):
    """(first matrix, matrices, row segments, scaling, job matrices) of one rank.
    `row_block` (profiling captures of one GPU only): rows [a, a + n) of a
    single matrix instead of the rank's shard."""
    if w["shard"] == "heads":
        if weak:
            # Every rank runs its own full batch of independent heads
            # (matrices rank*M .. rank*M + M - 1 of the seeded stream).
            return rank * w["matrices"], w["matrices"], [(0, w["rows"])], "weak", w["matrices"] * world
        first_b, n_local = head_range(w["matrices"], world, rank)
        return first_b, n_local, [(0, w["rows"])], "strong", w["matrices"]
    if row_block is not None:
        return 0, w["matrices"], [row_block], "strong", w["matrices"]
    segs = rank_segments(w["rows"], w["cols"], world, rank, fold=not contiguous)
    return 0, w["matrices"], segs, "strong", w["matrices"]


def rotation(w: dict, n_local: int, rows_local: int) -> tuple[int, int, str]:
    """Buffer sets rotated per launch so that consecutive launches touch more
    than 2 x L2, the bytes of one set (in + out), and the config's l2 note."""
    copy_bytes = 2 * n_local * rows_local * w["pitch"] * 2
    n_rot = 1 if copy_bytes >= 2 * L2_BYTES else math.ceil(2 * L2_BYTES / copy_bytes) + 1
    note = (f"{n_rot} rotated buffer sets of {copy_bytes / 2**20:.2f} MiB (in+out) per rank"
            if n_rot > 1 else f"inputs larger than L2 ({copy_bytes / 2**20:.0f} MiB in+out per rank), no flush")
    return n_rot, copy_bytes, note


def job_config(args, w: dict, world: int) -> tuple[dict, str]:
    """The `config` object of the JSON line and the scaling label. Both arms
    (this library and --impl reference) print exactly this, computed without
    loading either implementation."""
    row_block = getattr(args, "row_block", None)
    first_b, n_local, segs, scaling, job_matrices = rank_share(w, world, 0, args.weak,
                                                               args.contiguous_rows, row_block)
    _, _, l2 = rotation(w, n_local, sum(n for _, n in segs))
    cfg = {"workload": w["desc"], "name": args.workload, "matrices": job_matrices,
           "matrices_per_rank": n_local, "rows": w["rows"], "cols": w["cols"], "pitch": w["pitch"],
           "values": w["values"], "seed": w["seed"], "scale": w["scale"], "kernel": args.kernel,
           "shard": ("heads, every rank its own full batch (weak)" if scaling == "weak" else
                     "heads split evenly over the ranks" if w["shard"] == "heads" else
                     "folded row blocks of one matrix (a block and its mirror per rank)"
                     if not args.contiguous_rows and can_fold(w["rows"], w["cols"], world) else
                     "contiguous row blocks of one matrix, equal causal cost"),
           "l2": l2}
    if row_block is not None:
        cfg["row_block"] = {"first_row": args.row_block[0], "rows": args.row_block[1]}
    return cfg, scaling


class ClockSampler:
    """Samples SM clock and clock-event (throttle) reasons through NVML while
    the timed region runs."""

    REASONS = {0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

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
            idx = self.device
            vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
            parts = [p for p in vis.split(",") if p]
            if parts and all(p.isdigit() for p in parts):
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
                self.samples.append((nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM),
                                     nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)))
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
        seen = {n for _, r in self.samples for bit, n in self.REASONS.items() if r & bit}
        return {"sm_mhz": statistics.median(m for m, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": sorted(seen), "samples": len(self.samples)}


def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle_ctypes

    return oracle_ctypes


def host_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def cpu_sample(w: dict, seconds: float, threads: int) -> dict:
    """Times the reference CPU path on whole matrices of the workload (row
    blocks of at most 4096 rows for the long-context matrix) for ~`seconds`."""
    O = _oracle()
    rows, cols, pitch = w["rows"], w["cols"], w["pitch"]
    blk = min(rows, 4096)
    scale = f32(w["scale"])
    x = O.generate(w["config"], w["seed"], 1, blk, cols, pitch)[0].ravel()
    O.softmax_strided(x, 1, 0, min(blk, 64), cols, pitch, 0, scale, threads=1)  # warm-up
    done_bytes, done_rows, t0 = 0.0, 0, time.perf_counter()
    while True:
        # Successive blocks walk down the matrix (row offsets), so long rows are sampled too.
        off = (done_rows // blk * blk) % rows
        n = min(blk, rows - off)
        O.softmax_strided(x, 1, 0, n, cols, pitch, off, scale, threads=threads)
        done_bytes += O.roofline_bytes(n, cols, off)
        done_rows += n
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": round(done_bytes / dt / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{done_rows} rows ({done_rows / rows:.2f} matrices) of the {w['rows']}x{w['cols']} "
                      f"workload, {threads} thread(s), {dt:.1f} s; "
                      f"matrices/s = {done_bytes / O.roofline_bytes(rows, cols) / dt:.4f}"}


def run_reference(args, w: dict) -> None:
    """Reference arm: the reference's CPU path (the oracle's C restatement of
    reference/src/lib.rs:85-108, kind "port") on all host threads of rank 0.
    Every step softmaxes whole matrices of the workload, row-parallel; the
    inputs come from the oracle's copy of the seeded generator. Nothing of
    this package (its CUDA library included) is loaded."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    O = _oracle()
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    config, scaling = job_config(args, w, world)
    threads = host_threads()
    rows, cols, pitch = w["rows"], w["cols"], w["pitch"]
    scale = f32(w["scale"])
    # A pool of distinct matrices of the workload (the heads stream from seed;
    # single-matrix workloads have one), cycled step after step.
    pool_n = min(4, config["matrices"])
    x = O.generate(w["config"], w["seed"], pool_n, rows, cols, pitch, threads=threads)
    y = np.empty_like(x[0])
    mat_bytes = O.roofline_bytes(rows, cols)
    done = [0]

    def one_matrix():
        O.softmax_strided(x[done[0] % pool_n].ravel(), 1, 0, rows, cols, pitch, 0, scale,
                          threads=threads)
        done[0] += 1

    t0 = time.perf_counter()
    one_matrix()
    t_one = time.perf_counter() - t0
    # Whole matrices per step: enough for ~50 ms of work (one for the large workloads).
    per_step = max(1, min(64, round(0.05 / max(t_one, 1e-6))))
    for _ in range(args.warmup):
        for _ in range(per_step):
            one_matrix()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        for _ in range(per_step):
            one_matrix()
        times.append(time.perf_counter() - t0)
    del y
    step = statistics.mean(times)
    value = per_step * mat_bytes / step / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step * 1e3, 3), "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None,
        "dtype": "f32", "io_dtype": "f16", "data": "synthetic",
        "config": config,
        "matrices_per_s": round(per_step / step, 4),
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{per_step} whole {rows}x{cols} "
                                   f"{'matrix' if per_step == 1 else 'matrices'} per step (a pool of "
                                   f"{pool_n} seeded matrices, cycled), rows split over {threads} "
                                   f"threads; C restatement of reference/src/lib.rs:85-108, f32, "
                                   f"glibc expf, on the host cores of rank 0"},
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
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c4")
    ap.add_argument("--kernel", default="auto")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gather", action="store_true",
                    help="N > 1: skip the separately reported gather of all outputs to rank 0")
    ap.add_argument("--contiguous-rows", action="store_true",
                    help="single matrices: contiguous row blocks instead of folded shards")
    ap.add_argument("--weak", action="store_true",
                    help="batched workload: every rank runs its own full batch (weak scaling)")
    ap.add_argument("--no-graph", action="store_true",
                    help="skip the CUDA-graph timing of the single-matrix workloads")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--tuning", default="",
                    help="vec,stages,l2_hint,zero_fill_tma (0/-1 = automatic)")
    ap.add_argument("--matrices", type=int, default=0,
                    help="override the number of matrices (profiling captures only)")
    ap.add_argument("--row-block", default="",
                    help="FIRST:COUNT rows of a single-matrix workload on one GPU "
                         "(profiling captures only)")
    args = ap.parse_args()
    if args.row_block:
        a, n = (int(v) for v in args.row_block.split(":"))
        w0 = WORKLOADS[args.workload]
        if w0["shard"] != "rows" or args.gpus != 1 or not (0 <= a and 0 < n and a + n <= w0["rows"]):
            raise SystemExit("--row-block: FIRST:COUNT inside a single-matrix workload, on one GPU")
        args.row_block = (a, n)
        args.no_e2e = args.no_cpu_baseline = True  # a kernel capture, not a bench line
    else:
        args.row_block = None
    if args.warmup < 3:
        log("warmup raised to 3 (timing rule)")
        args.warmup = 3
    w = dict(WORKLOADS[args.workload])
    if args.matrices:
        w["matrices"] = args.matrices

    if args.impl == "reference":
        run_reference(args, w)
        return 0

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

    rows_full, cols, pitch = w["rows"], w["cols"], w["pitch"]
    scale = f32(w["scale"])
    # Heads split evenly over the ranks (or, with --weak, a full batch per
    # rank); single matrices as folded row-block shards (a block and its
    # mirror, stored one after the other) or contiguous blocks. No exchange
    # between ranks on this path.
    first_b, n_local, segs, scaling, job_matrices = rank_share(w, world, rank, args.weak,
                                                               args.contiguous_rows, args.row_block)
    config, _ = job_config(args, w, world)
    rows = sum(n for _, n in segs)
    r0 = segs[0][0]

    # This rank's input on the host (pinned) and on the device; rotate copies
    # when one copy (in + out) is smaller than 2 x L2.
    t0 = time.perf_counter()
    h_in = torch.empty((n_local, rows, pitch), dtype=torch.int16, pin_memory=True)
    off = 0
    for a, n in segs:  # one segment per matrix batch, or n_local == 1
        cs.generate(w["config"], w["seed"], batch=n_local, rows=n, cols=cols, pitch=pitch,
                    first_batch=first_b, first_row=a, out=h_in.numpy().view(np.uint16)[:, off:off + n])
        off += n
    n_rot, copy_bytes, _ = rotation(w, n_local, rows)
    d_in = [h_in.cuda().view(torch.float16) for _ in range(n_rot)]
    d_out = [torch.empty_like(d_in[0]) for _ in range(n_rot)]
    seg_text = " + ".join(f"{a}..{a + n}" for a, n in segs)
    log(f"rank {rank}: matrices {first_b}..{first_b + n_local} rows {seg_text} x {cols}, "
        f"{n_rot} buffer set(s), ready in {time.perf_counter() - t0:.1f} s")

    stream = torch.cuda.current_stream()
    plans = [cs.Plan.for_tensors(a, b, cols=cols, row_offset=r0) for a, b in zip(d_in, d_out)]
    if len(segs) > 1:
        for p in plans:
            p.set_row_split(segs[0][1], segs[1][0])
    if args.tuning:
        for p in plans:
            p.set_tuning(*(int(t) for t in args.tuning.split(",")))
    info = plans[0].describe(args.kernel)
    log(f"rank {rank}: launch {info}")

    def barrier():
        if world > 1:
            dist.barrier()

    for i in range(args.warmup):
        plans[i % n_rot].launch(args.kernel, scale, stream)
    torch.cuda.synchronize()
    for p in plans:
        rc, st = p.status()
        if rc != 0:
            raise SystemExit(f"device status {st} after warm-up")

    # Spot check of the timed kernel's output (oracle-free structure check).
    nchk = min(2, n_local)
    host_out = d_out[0][:nchk].view(torch.int16).cpu().numpy().view(np.uint16)
    off = 0
    for a, n in segs:
        chk = cs.check_output(host_out[:, off:off + n], batch=nchk, rows=n, cols=cols, pitch=pitch,
                              row_offset=a)
        off += n
        if chk["mask_violations"] or chk["nonfinite_or_negative"] or chk["rowsum_violations"]:
            raise SystemExit(f"output self-check failed (rows {a}..{a + n}): {chk}")

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        start.record(stream)
        for i in range(args.steps):
            plans[i % n_rot].launch(args.kernel, scale, stream)
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms_total = start.elapsed_time(end)
    log(f"rank {rank}: {ms_total / args.steps * 1e3:.1f} us per step, "
        f"{info['algorithmic_bytes'] / (ms_total / args.steps * 1e6):.0f} GB/s on this rank's share")
    for p in plans:
        rc, st = p.status()
        if rc != 0:
            raise SystemExit(f"device status {st} after the timed region")
    t = torch.tensor([ms_total], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = float(t.item()) / args.steps
    alg_local = info["algorithmic_bytes"]
    alg_total = cs.roofline_bytes(rows_full, cols) * job_matrices
    if args.row_block is not None:
        alg_total = alg_local  # a block of rows only (profiling captures)
    value = alg_total / (ms_step / 1e3) / 1e9

    peak, peak_kind = measured_peak()
    achieved = alg_local / (ms_total / args.steps / 1e3) / 1e9
    tpm = ncu_traffic_per_matrix(info["kernel_name"], args.workload)
    roofline = {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} hbm_gbs (burst copy)",
                "traffic": round(tpm * n_local * rows / rows_full) if tpm else None,
                "algorithmic_bytes_per_launch": alg_local,
                "kernel": f"{info['kernel_name']} grid={info['grid']} block={info['block']} "
                          f"smem={info['smem_bytes']} stages={info['stages']} "
                          f"vec={info['vec_per_thread']}"}
    clk = clocks.summary()

    # Per-launch distribution (the reference's BenchStats: min / median / p95)
    # from a separate pass with an event after every launch; `value` comes
    # from the uninterrupted timed region above.
    launch_stats = None
    try:
        n_s = max(20, min(args.steps, 200))
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(n_s + 1)]
        ev[0].record(stream)
        for i in range(n_s):
            plans[i % n_rot].launch(args.kernel, scale, stream)
            ev[i + 1].record(stream)
        torch.cuda.synchronize()
        st = cs.bench_stats([ev[i].elapsed_time(ev[i + 1]) for i in range(n_s)])
        launch_stats = {k: round(st[k], 5) for k in ("min_ms", "median_ms", "p95_ms", "max_ms", "cv_pct")}
        launch_stats["samples"] = n_s
        launch_stats["timing"] = "separate pass, CUDA event after every launch (not the value)"
    except Exception as e:  # diagnostics only: never costs the line
        log(f"rank {rank}: launch stats unavailable: {e}")
    for p in plans:
        rc, st_word = p.status()
        if rc != 0:
            raise SystemExit(f"device status {st_word} after the per-launch pass")

    # Single-matrix workloads: the same launches captured in one CUDA graph
    # (k launches per replay, device time / k), which removes the host's
    # per-launch cost; reported beside the stream-launched value, not in it.
    graph = None
    if w["matrices"] == 1 and not args.no_graph:
        k = max(1, min(args.steps, 100))
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side, capture_error_mode="thread_local"):
            for i in range(k):
                plans[i % n_rot].launch(args.kernel, scale)
        g.replay()
        torch.cuda.synchronize()
        reps = max(3, 2000 // k)
        ga, gb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        ga.record()
        for _ in range(reps):
            g.replay()
        gb.record()
        torch.cuda.synchronize()
        gt = torch.tensor([ga.elapsed_time(gb) / (reps * k)], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(gt, op=dist.ReduceOp.MAX)
        g_ms = float(gt.item())
        for p in plans:
            rc, st = p.status()
            if rc != 0:
                raise SystemExit(f"device status {st} after the graph replays")
        graph = {"value": round(alg_total / (g_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                 "us_per_launch": round(g_ms * 1e3, 3), "launches_per_graph": k, "replays": reps,
                 "timing": "CUDA graph of k launches replayed R times, device time / (R k), max over ranks"}
        del g
    for p in plans:
        p.close()

    # Optional final gather (N > 1): every rank's output shard to rank 0 over
    # NCCL, outside the timed region and reported on its own. For row blocks
    # rank 0 assembles the whole matrix and checks its row sums.
    gather = None
    if world > 1 and not args.no_gather:
        shard = d_out[0].reshape(-1)  # fp16 (NCCL moves the bits unchanged)
        counts = torch.tensor([shard.numel()], dtype=torch.int64, device="cuda")
        all_counts = [torch.zeros_like(counts) for _ in range(world)]
        dist.all_gather(all_counts, counts)
        sizes = [int(c.item()) for c in all_counts]
        recv = None
        if rank == 0:
            recv = torch.empty(sum(sizes), dtype=torch.float16, device="cuda")
            recv[:sizes[0]].copy_(shard)
        def gather_once():
            if rank == 0:
                ops, off = [], sizes[0]
                for r in range(1, world):
                    ops.append(dist.P2POp(dist.irecv, recv[off:off + sizes[r]], r))
                    off += sizes[r]
            else:
                ops = [dist.P2POp(dist.isend, shard, 0)]
            for req in dist.batch_isend_irecv(ops):
                req.wait()

        gather_once()  # untimed: NCCL sets up its peer connections on first use
        ga, gb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        ga.record()
        gather_once()
        gb.record()
        torch.cuda.synchronize()
        gt = torch.tensor([ga.elapsed_time(gb)], dtype=torch.float64, device="cuda")
        dist.all_reduce(gt, op=dist.ReduceOp.MAX)
        moved = 2 * (sum(sizes) - sizes[0])
        gather = {"value": round(moved / (float(gt.item()) / 1e3) / 1e9, 2), "unit": "GB/s",
                  "bytes": moved, "ms": round(float(gt.item()), 3),
                  "timing": "NCCL send/recv of every rank's output to rank 0, device time, max over ranks"}
        if rank == 0 and w["shard"] == "rows":
            # Place every rank's segments at their rows.
            full = torch.empty((rows_full, pitch), dtype=torch.float16, device="cuda")
            pos = 0
            for r in range(world):
                for a, n in rank_segments(rows_full, cols, world, r, fold=not args.contiguous_rows):
                    full[a:a + n].copy_(recv[pos:pos + n * pitch].view(n, pitch))
                    pos += n * pitch
            sums = full[:, :cols].double().sum(dim=1)
            err = float((sums - 1.0).abs().max())
            gather["max_rowsum_err"] = round(err, 6)
            if err > 2e-3:
                raise SystemExit(f"gathered matrix fails the row-sum check: {err}")
        del recv

    # End to end through the host-buffer API.
    e2e = None
    if not args.no_e2e:
        del d_in, d_out
        torch.cuda.empty_cache()
        if pitch == cols:
            dense_in = h_in
        else:
            dense_in = torch.empty((n_local, rows, cols), dtype=torch.int16, pin_memory=True)
            dense_in.copy_(h_in[:, :, :cols])
        dense_out = torch.empty_like(dense_in, pin_memory=True)
        # One host-path call per segment of the shard (views into the
        # pinned buffers; a folded shard has two).
        calls, off = [], 0
        for a, n in segs:
            si = dense_in.numpy().view(np.uint16)[:, off:off + n]
            so = dense_out.numpy().view(np.uint16)[:, off:off + n]
            if not (si.flags.c_contiguous and so.flags.c_contiguous):
                raise SystemExit("host-path segments must be contiguous (one matrix per folded shard)")
            calls.append((si.reshape(-1), so.reshape(-1), n, a))
            off += n

        def host_step(sess):
            for si, so, n, a in calls:
                sess.softmax_host(si, so, batch=n_local, rows=n, cols=cols, scale=scale,
                                  kernel=args.kernel, row_offset=a)

        with cs.Session(local) as sess:
            host_step(sess)  # warm-up: allocates buffers
            times = []
            for _ in range(max(1, args.e2e_steps)):
                barrier()
                t0 = time.perf_counter()
                host_step(sess)
                times.append(time.perf_counter() - t0)
        e_step = torch.tensor([statistics.mean(times)], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(e_step, op=dist.ReduceOp.MAX)
        e_s = float(e_step.item())
        # Bytes the host path moved (causal row blocks), summed over ranks.
        moved = torch.tensor([float(sum(cs.host_copy_bytes(n_local, n, cols, a) for a, n in segs))],
                             dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(moved)
        moved_b = int(moved.item())
        e2e = {"value": round(alg_total / e_s / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": moved_b, "d2h_bytes_per_step": moved_b,
               "ms_per_step": round(e_s * 1e3, 3),
               "timing": "host wall clock around the blocking call, max over ranks"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_sample(w, args.cpu_seconds, 1)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": "f32", "io_dtype": "f16", "data": "synthetic",
            "config": config,
            "matrices_per_s": round(job_matrices / (ms_step / 1e3), 2),
            "roofline_pct": round(100.0 * value / (peak * world), 2),
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk, "graph": graph,
            "launch_stats": launch_stats,
            "gather": gather,
            "gpu_launches": args.steps * world, "gpu_launches_per_rank": args.steps,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
