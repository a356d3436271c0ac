"""Resource gate over the library's ptxas report, and the BENCH-line parser.

CPU only: the report is written by every build (`-Xptxas -v` into
lib/ptxas.txt); csm's BENCH lines are checked as text.
"""
import json

import pytest

import build
from causal_softmax import benchlog, resources


def test_library_report_passes_the_gate():
    build.build_library()
    with open(resources.REPORT, encoding="utf-8") as fh:
        problems, kernels = resources.check(fh.read())
    assert not problems, problems
    names = {k["name"] for k in kernels.values()}
    # Every launchable kernel family is reported: 8 row-resident variants x 2
    # store modes, the two online shapes, baseline and 6 narrow instantiations.
    assert sum(n.startswith("rowres_kernel<") for n in names) == 16
    assert {"online_kernel<1>", "online_kernel<2>", "baseline_kernel", "probe_kernel", "cluster_kernel"} <= names
    assert sum(n.startswith("narrow_kernel<") for n in names) == 6


REPORT = """ptxas info    : Compiling entry function '_ZN2cs13rowres_kernelILi4ELi384ELi2ELb1EEEvNS_12RowResParamsE' for 'sm_100a'
ptxas info    : Function properties for _ZN2cs13rowres_kernelILi4ELi384ELi2ELb1EEEvNS_12RowResParamsE
    192 bytes stack frame, {st} bytes spill stores, {ld} bytes spill loads
ptxas info    : Used {regs} registers, used 2 barriers
"""


def test_gate_flags_spills_and_lost_residency():
    ok, _ = resources.check(REPORT.format(st=0, ld=0, regs=80))
    assert ok == []
    bad, _ = resources.check(REPORT.format(st=8, ld=8, regs=80))
    assert any("spill bytes" in p for p in bad)
    # 88 registers: 6 warps x 2816 > 16384 per sub-partition, one CTA of 384 only.
    bad, _ = resources.check(REPORT.format(st=0, ld=0, regs=88))
    assert any("launch bounds promise 2" in p for p in bad)
    bad, _ = resources.check(REPORT.format(st=0, ld=0, regs=80).replace("sm_100a", "sm_90a"))
    assert any("wrong-target" in p for p in bad)
    bad, _ = resources.check("ptxas fatal   : something\n")
    assert bad


def test_resident_ctas_matches_measured_occupancy():
    # cudaOccupancyMaxActiveBlocksPerMultiprocessor on B200 (register-limited cases).
    assert resources.resident_ctas(87, 352) == 1
    assert resources.resident_ctas(87, 288) == 2
    assert resources.resident_ctas(72, 224) == 4
    assert resources.resident_ctas(148, 160) == 2
    assert resources.resident_ctas(56, 352) == 3


SUITE = """BENCH hardware=NVIDIA B200 sms=148 clock=CUDA_event_and_host_wall verify=1 warmup=2 repetitions=5
BENCH category=shape clock=cuda_event kernel=tma rows=4096 cols=4096 n=5 min_ms=0.01600 median_ms=0.01620 p95_ms=0.01700 p99_ms=0.01700 max_ms=0.01700 mean_ms=0.01630 stddev_ms=0.00010 cv_pct=0.61 approx_logical_GBps=3107.15 Melem_per_s=517.8 speedup_vs_baseline=2.310
BENCH category=queue clock=cuda_event queued=64 kernel=pipeline rows=1024 cols=1024 n=5 min_ms=0.00619 median_ms=0.00622 p95_ms=0.00626 p99_ms=0.00626 max_ms=0.00626 mean_ms=0.00622 stddev_ms=0.00002 cv_pct=0.36 approx_logical_GBps=506.03 Melem_per_s=168.6
BENCH category=concurrency clock=host_wall streams=8 calls_per_stream=4 kernel=pipeline rows=512 cols=512 n=5 batch_p50_ms=0.15518 batch_p95_ms=0.15693 batch_p99_ms=0.15693 kernels_per_s=206206.83 throughput_speedup=1.638 approx_logical_GBps=162.27
"""


def test_bench_lines_to_json(tmp_path):
    doc = benchlog.summarize(SUITE, "suite.txt")
    assert doc["record_count"] == 3
    assert doc["categories"] == {"shape": 1, "queue": 1, "concurrency": 1}
    shape = doc["records"][0]
    assert shape["rows"] == 4096 and isinstance(shape["n"], int)
    assert shape["median_ms"] == pytest.approx(0.0162) and shape["speedup_vs_baseline"] == pytest.approx(2.31)
    assert doc["records"][1]["queued"] == 64
    assert doc["records"][2]["streams"] == 8 and doc["records"][2]["throughput_speedup"] == pytest.approx(1.638)
    log = tmp_path / "suite.txt"
    log.write_text(SUITE)
    out = tmp_path / "suite.json"
    assert benchlog.main([str(log), "--output", str(out)]) == 0
    assert json.loads(out.read_text())["record_count"] == 3


def test_bench_lines_rejected():
    for bad in ("BENCH category=shape kernel=tma rows=0 cols=4 median_ms=1",
                "BENCH kernel=tma rows=4 cols=4 median_ms=1",
                "BENCH category=shape rows=4 cols=4 median_ms=1",
                "BENCH category=shape kernel=tma rows=4 cols=4 median_ms=nan",
                "BENCH category=shape kernel=tma rows=4 cols=4 median_ms=-1"):
        with pytest.raises(ValueError):
            benchlog.parse_log(bad)
    with pytest.raises(ValueError):
        benchlog.parse_log("no records here")
