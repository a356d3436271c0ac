"""The csm CLI (mirror of gpu/src/driver.rs:386-428 over the C ABI).

CPU: flag parsing and validation messages (host/src/lib.rs:103-182).
GPU: --probe, the --gpu-tests self-check matrix, a --bench line, and the
--bench-suite categories of gpu/src/driver/bench.rs:139-369.
"""
import os
import subprocess

import pytest

import build

CSM = build.CLI_PATH


@pytest.fixture(scope="module", autouse=True)
def built():
    build.build_cli()
    assert os.path.exists(CSM)


def run(*args):
    return subprocess.run([CSM, *args], capture_output=True, text=True, timeout=600)


def test_help_and_errors():
    r = run("--help")
    assert r.returncode == 0 and "--probe" in r.stdout
    for args, msg in [(["--rows", "0"], "rows and cols must be positive"),
                      (["--scale", "NaN"], "scale must be finite"),
                      (["--cols", "33", "--kernel", "warp"], "warp specialization requires cols <= 32"),
                      (["--kernel", "wrong"], "unknown kernel"),
                      (["--x"], "unknown flag: --x"),
                      (["--cols"], "missing value for --cols"),
                      (["--cols", "2147483647"], "padded pitch exceeds device i32 indexing")]:
        r = run(*args)
        assert r.returncode == 2 and msg in r.stderr, (args, r.stderr)


@pytest.mark.gpu
def test_cli_on_gpu():
    r = run("--probe")
    assert r.returncode == 0 and "PASS probe" in r.stdout, r.stderr
    r = run("--gpu-tests")
    assert r.returncode == 0 and "PASS GPU self-checks" in r.stdout, r.stdout + r.stderr
    r = run("--rows", "1000", "--cols", "1037", "--scale", "0.0883883")
    assert r.returncode == 0 and r.stdout.startswith("PASS"), r.stdout + r.stderr
    r = run("--bench", "--rows", "2048", "--cols", "2048", "--iterations", "5", "--warmup", "2")
    assert r.returncode == 0 and r.stdout.count("BENCH kernel=") == 4, r.stdout + r.stderr


@pytest.mark.gpu
def test_bench_suite_categories():
    r = run("--bench-suite", "--rows", "2048", "--cols", "2048", "--iterations", "3", "--warmup", "1")
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr
    lines = r.stdout.splitlines()
    assert lines[0].startswith("BENCH hardware=")
    cats = {}
    for ln in lines[1:]:
        assert ln.startswith("BENCH category="), ln
        cat = ln.split()[1].split("=")[1]
        cats[cat] = cats.get(cat, 0) + 1
    # 12 shapes x supported kernels (all 5 up to 32 columns, else 4); 4 queue
    # depths x kernels; 3 transfer stages; 1 device copy; 6 patterns x 4 scales
    # x kernels; 1/2/4/8 streams.
    assert cats["shape"] == 3 * 5 + 9 * 4 and cats["queue"] == 4 * 4, cats
    assert cats["transfer"] == 3 and cats["device_copy"] == 1, cats
    assert cats["pattern"] == 6 * 4 * 4 and cats["concurrency"] == 4, cats
    assert all("median_ms=" in ln or "batch_p50_ms=" in ln for ln in lines[1:])
